// gqa_mma_kernel.cuh — split-KV paged GQA/MHA/MQA decode on warp-level
// tensor-core tiles (sm_100a), for page sizes that are multiples of 16.
//
// Same math, work decomposition (balanced stream-K cut of all chunks into
// one range per CTA), producer warp, workspace and combine as
// gqa_kernel.cuh; what differs is the consumer arithmetic.  A warp owns one
// KV head and GW <= 16 of its query heads.  Per 16-token chunk:
//
//   S[heads x 16 tok]  = Q[heads x D] . K^T          mma m16n8k16, fp32 acc
//   online softmax over the token axis (rows = heads; 4 lanes per head row)
//   O^T[D x heads]    += V^T[D x 16 tok] . P[16 tok x heads]
//
// so the query heads pad the M=16 rows of the QK tile and form the N=8 (or
// 16) columns of the PV tile; the P fragment comes straight out of the QK
// accumulator registers (the C layout of the QK tile is the B layout of the
// PV tile).  Arithmetic per KV byte stays far below the tensor pipe, so the
// kernel is bound by HBM, not by issue slots as a CUDA-core dot-product
// kernel is at group sizes >= 8 or with FP8 caches.
//
// Shared-memory tiles: the 5-D TMA box {line, 16 tok, D/line, HK, 1} with
// 128-byte swizzle lands each (head, 128-byte dim chunk) as 16 consecutive
// 128-byte lines, one per token, so ldmatrix row addresses (8 tokens, same
// 16-byte column) hit 8 different bank groups.
//  * bf16/fp16 caches: K fragments by ldmatrix, V^T fragments by
//    ldmatrix.trans.
//  * fp8-e4m3 caches: fragments are built from 32-bit shared loads and
//    converted in registers (e4m3 -> fp16 * 2^-8, exact).  The dot product's
//    dimension order and the P.V row order are permuted so that each lane's
//    4 consecutive bytes fill whole fragment registers; the query and the
//    output use the same permutation.
#pragma once

#include "gqa_kernel.cuh"

// FP8 fragments: hardware cvt (exact values) or the bit-move conversion
// (values * 2^-8, folded into the scales).
#ifndef B2D_FP8_HW_CVT
#define B2D_FP8_HW_CVT 1
#endif

namespace b2d {

__device__ __forceinline__ uint32_t fp8_pair(uint32_t w) {
#if B2D_FP8_HW_CVT
  return e4m3x2_to_f16x2_cvt(w);
#else
  return e4m3x2_to_f16x2_scaled(w);
#endif
}
constexpr float kFp8FragScale = B2D_FP8_HW_CVT ? 1.f : 256.f;

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}

// D += A . B, m16n8k16, 16-bit inputs (BF16 selects bf16, else fp16), fp32 acc.
template <bool BF16>
__device__ __forceinline__ void mma16816(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  if constexpr (BF16) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (BF16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}

// 5-D tiled TMA load (no multicast); c0 (innermost) is always 0.
__device__ __forceinline__ void tma_load_5d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int c1, int c2, int c3, int c4, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cta.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4, %5, %6}], [%7], %8;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(0), "r"(c1), "r"(c2), "r"(c3), "r"(c4),
      "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// 3-D tiled TMA load (no multicast).
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cta.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar)),
      "l"(policy)
      : "memory");
}

// Byte address of (line, 16-byte chunk) under the 128-byte TMA swizzle.
__device__ __forceinline__ uint32_t swz(uint32_t base, int line, int chunk) {
  return base + (uint32_t)(line * 128) + (uint32_t)(((chunk ^ (line & 7)) & 7) << 4);
}

// Query element (head row, dim) as fp32 (0 for padding rows).
template <typename QT>
__device__ __forceinline__ float q_at(const QT* qrow, bool valid, int dim) {
  return valid ? static_cast<float>(qrow[dim]) : 0.f;
}

// VL: vLLM cache layout (K [blocks, Hkv, D/8, P, 8], V [blocks, Hkv, D, P]).
// K tiles arrive as [head][D/8][16 tokens][8 elements] (no swizzle: an
// ldmatrix's 8 token rows are 16 bytes apart); V tiles arrive transposed
// ([head][D][16 tokens], 32-byte rows, no swizzle) and feed the P.V product
// through plain (non-transposing) ldmatrix.
template <int D, int KIND, typename QT, int NP, bool VL = false>
__global__ void __launch_bounds__(32 * 9, 1)
    gqa_mma_kernel(const __grid_constant__ CUtensorMap tmap_k,
                   const __grid_constant__ CUtensorMap tmap_v, const GqaParams p) {
  constexpr bool FP8 = (KIND == kKvFp8);
  constexpr bool MMA_BF16 = (KIND == kKvBf16);   // fp16 and fp8 caches use fp16 MMAs
  constexpr int ES = FP8 ? 1 : 2;
  constexpr int LINE = 128 / ES;                 // elements per 128-byte line
  constexpr int DC = D / LINE;                   // lines per token row of one head
  constexpr int KS = D / 16;                     // QK k-steps
  constexpr int MT = D / 16;                     // PV m-tiles (dims)
  constexpr int T = 16;                          // tokens per chunk
  constexpr float kLn2 = 0.69314718055994530942f;

  extern __shared__ __align__(1024) uint8_t smem[];
  const int R = p.B * p.HG;
  const int cta = blockIdx.x;
  // Stage buffers start on a 1024-byte boundary (the 128-byte swizzle
  // pattern repeats every 1024 bytes); the host reserves 1 KB of slack.
  uint8_t* tiles = smem + ((1024u - (smem_u32(smem) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(tiles + (size_t)p.stages * 2 * p.stage_bytes);
  uint64_t* empty = full + p.stages;
  int32_t* row_start = reinterpret_cast<int32_t*>(empty + p.stages);
  int32_t* warp_tmp = row_start + (R + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, p.NW);
    }
    fence_barrier_init();
  }
  if (warp == p.NW && lane == 0) {
    prefetch_tmap(&tmap_k);
    prefetch_tmap(&tmap_v);
  }
  // Everything above touches only shared memory and kernel parameters: with
  // programmatic dependent launch it overlaps the previous kernel's tail.
  griddep_wait();
  griddep_launch();
  build_row_start(p, R, row_start, warp_tmp);
  if (cta == 0) {
    for (int i = threadIdx.x; i <= R; i += blockDim.x) p.row_start_g[i] = row_start[i];
  }
  const int64_t W = row_start[R];
  const int G = W < (int64_t)gridDim.x ? (int)W : (int)gridDim.x;
  if (p.merge_count != nullptr && warp < p.NW) {
    // No combine kernel follows: rows of zero length get out = 0, lse = -inf
    // here, spread over the CTAs; each consumer warp writes its own heads.
    const int hk_w = warp / p.WPH, gw_w = p.group / p.WPH;
    for (int r = cta; r < R; r += gridDim.x) {
      if (row_start[r + 1] != row_start[r]) continue;
      const int b = r / p.HG;
      warp_zero_heads<D, QT>(p, b, r - b * p.HG, p.HK * p.group,
                             hk_w * p.group + (warp - hk_w * p.WPH) * gw_w, gw_w);
    }
  }
  if (W == 0 || cta >= G) return;
  const int x0 = (int)((int64_t)cta * W / G);
  const int x1 = (int)((int64_t)(cta + 1) * W / G);
  const int cap = p.max_pages * p.P;

  if (warp == p.NW) {
    // ---------------- producer warp (one K and one V box per chunk) --------
    // (test flag no_loads: issue nothing, so every consumer wait runs out)
    if (p.no_loads) return;
    const uint64_t policy = policy_evict_first();
    bool ok = true;
    int s = 0;
    uint32_t ph = 0;
    for (int gbase = x0; gbase < x1 && ok; gbase += 32) {
      const int x = gbase + lane;
      int my_page = 0, my_off = 0, my_h0 = 0;
      if (x < x1) {
        const int rr = find_row(row_start, R, x);
        const int b = rr / p.HG, hg = rr - b * p.HG;
        const int tok0 = (x - row_start[rr]) * T;
        const int pidx = tok0 / p.P;
        my_off = tok0 - pidx * p.P;
        my_h0 = hg * p.HK;
        int pg = __ldg(p.block_table + (int64_t)b * p.bt_stride + pidx);
        if (pg < 0 || pg >= p.num_pages) {
          record_status(p.status, kStatusBounds);
          pg = 0;
        }
        my_page = pg;
      }
      const int cnt = (x1 - gbase) < 32 ? (x1 - gbase) : 32;
      for (int k = 0; k < cnt; ++k) {
        const int page = __shfl_sync(0xffffffffu, my_page, k);
        const int off = __shfl_sync(0xffffffffu, my_off, k);
        const int h0 = __shfl_sync(0xffffffffu, my_h0, k);
        if (lane == 0 && ok) {
          if (!mbar_wait(empty + s, ph ^ 1u, p.wait_ns)) {
            record_status(p.status, kStatusTimeout);
            ok = false;
          } else {
            uint8_t* kdst = tiles + (size_t)s * 2 * p.stage_bytes;
            mbar_arrive_expect_tx(full + s, 2u * p.stage_bytes);
            if constexpr (VL) {
              const int ph_idx = page * p.Hkv + h0;   // flattened (block, head)
              tma_load_3d(kdst, &tmap_k, full + s, off * 8, 0, ph_idx, policy);
              tma_load_3d(kdst + p.stage_bytes, &tmap_v, full + s, p.P == 16 ? 0 : off, 0, ph_idx,
                          policy);
            } else {
              tma_load_5d(kdst, &tmap_k, full + s, off, 0, h0, page, policy);
              tma_load_5d(kdst + p.stage_bytes, &tmap_v, full + s, off, 0, h0, page, policy);
            }
          }
        }
        if (++s == p.stages) {
          s = 0;
          ph ^= 1u;
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
      }
    }
    return;
  }

  // ---------------- consumer warps ----------------
  const int hk = warp / p.WPH;            // KV head within the tile
  const int qg = warp - hk * p.WPH;       // which GW-head group of that KV head
  const int GW = p.group / p.WPH;         // query heads of this warp (<= 8 * NP)
  const int HQC = p.HK * p.group;
  const int g = lane >> 2, t = lane & 3;
  const uint32_t tiles_u32 = smem_u32(tiles);

  uint32_t qa[KS][NP == 2 ? 4 : 2];   // Q fragments (rows g, and g + 8 when NP == 2)
  float acc[NP][MT][4];
  float m_r[2], l_r[2];               // softmax state of rows g and g + 8
  float sc = 1.f, vscale = 1.f;
  int cur_row = -1, L = 0;

  auto start_row = [&](int row) {
    const int b = row / p.HG, hg = row - b * p.HG;
    int Lb = __ldg(p.seqlens + b);
    L = Lb < 0 ? 0 : (Lb > cap ? cap : Lb);
    const int kvh = hg * p.HK + hk;
    sc = p.scale_log2;
    vscale = 1.f;
    if constexpr (FP8) {
      sc *= (p.k_scale ? __ldg(p.k_scale + kvh) : 1.f) * kFp8FragScale;
      vscale = (p.v_scale ? __ldg(p.v_scale + kvh) : 1.f) * kFp8FragScale;
    }
    const int qh0 = kvh * p.group + qg * GW;
    const QT* qb = reinterpret_cast<const QT*>(p.q) + (int64_t)b * p.q_sb;
    const QT* q_lo = qb + (int64_t)(qh0 + g) * p.q_sh;
    const QT* q_hi = qb + (int64_t)(qh0 + g + 8) * p.q_sh;
    const bool v_lo = g < GW, v_hi = g + 8 < GW;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      // 16-bit: cols (2t, 2t+1) and (2t+8, 2t+9) of the k-step; fp8: the
      // permuted cols (4t, 4t+1) and (4t+2, 4t+3).
      const int c0 = FP8 ? 16 * ks + 4 * t : 16 * ks + 2 * t;
      const int c1 = FP8 ? c0 + 2 : c0 + 8;
      qa[ks][0] = pack2<MMA_BF16>(q_at(q_lo, v_lo, c0), q_at(q_lo, v_lo, c0 + 1));
      qa[ks][NP == 2 ? 2 : 1] = pack2<MMA_BF16>(q_at(q_lo, v_lo, c1), q_at(q_lo, v_lo, c1 + 1));
      if constexpr (NP == 2) {
        qa[ks][1] = pack2<MMA_BF16>(q_at(q_hi, v_hi, c0), q_at(q_hi, v_hi, c0 + 1));
        qa[ks][3] = pack2<MMA_BF16>(q_at(q_hi, v_hi, c1), q_at(q_hi, v_hi, c1 + 1));
      }
    }
#pragma unroll
    for (int n = 0; n < NP; ++n)
#pragma unroll
      for (int i = 0; i < MT; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[n][i][e] = 0.f;
    m_r[0] = m_r[1] = -INFINITY;
    l_r[0] = l_r[1] = 0.f;
  };

  // dim of O^T row (tile i, row rr in {g, g + 8}) in the output
  auto out_dim = [&](int i, int hi) -> int {
    if constexpr (FP8) return 32 * (i >> 1) + 4 * g + 2 * (i & 1) + hi;
    else return 16 * i + g + 8 * hi;
  };

  auto finish_row = [&](int row) {
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      l_r[r] += __shfl_xor_sync(0xffffffffu, l_r[r], 1);
      l_r[r] += __shfl_xor_sync(0xffffffffu, l_r[r], 2);
    }
    const int b = row / p.HG, hg = row - b * p.HG;
    const int cf = cta_of_chunk(row_start[row], W, G);
    const int cl = cta_of_chunk(row_start[row + 1] - 1, W, G);
    const int kvh = hg * p.HK + hk;
    const int qh_row0 = hk * p.group + qg * GW;  // first query head of the warp, in the row
#pragma unroll
    for (int n = 0; n < NP; ++n) {
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int hw = 8 * n + 2 * t + c;        // head within the warp (PV column)
        const int src = 4 * (2 * t + c);         // lane holding that head's row state
        const float lh = __shfl_sync(0xffffffffu, l_r[n], src);
        const float mh = __shfl_sync(0xffffffffu, m_r[n], src);
        if (hw >= GW) continue;
        const float inv = vscale / lh;
        const int qh_row = qh_row0 + hw;
        if (cf == cl) {
          QT* dst = reinterpret_cast<QT*>(p.out) + (int64_t)b * p.o_sb +
                    (int64_t)(hg * HQC + qh_row) * p.o_sh;
#pragma unroll
          for (int i = 0; i < MT; ++i) {
            dst[out_dim(i, 0)] = QT(acc[n][i][c] * inv);
            dst[out_dim(i, 1)] = QT(acc[n][i][2 + c] * inv);
          }
          if (p.lse != nullptr && g == 0)
            p.lse[(int64_t)b * p.lse_sb + hg * HQC + qh_row] = (mh + fast_log2(lh)) * kLn2;
        } else {
          const int64_t seg = (int64_t)row + cta;
          float* dst = p.part_o + (seg * HQC + qh_row) * D;
#pragma unroll
          for (int i = 0; i < MT; ++i) {
            dst[out_dim(i, 0)] = acc[n][i][c] * inv;
            dst[out_dim(i, 1)] = acc[n][i][2 + c] * inv;
          }
          if (g == 0) p.part_lse[seg * HQC + qh_row] = mh + fast_log2(lh);
        }
      }
    }
    (void)kvh;
    if (cf != cl && p.merge_count != nullptr) {
      // In-kernel merge: every warp that wrote a partial of these heads
      // counts itself in with one acquire-release atomic (the __syncwarp
      // orders the other lanes' partial stores before lane 0's release);
      // the warp that arrives last has acquired every other partial, merges
      // all cl - cf + 1 of them and re-arms the counter for the next call.
      __syncwarp();
      int* cnt = p.merge_count + (int64_t)row * p.NW + warp;
      int old = 0;
      if (lane == 0) old = atomic_add_acq_rel_gpu(cnt, 1);
      old = __shfl_sync(0xffffffffu, old, 0);
      if (old == cl - cf) {
        __syncwarp();   // lane 0's acquire, then the other lanes' loads
        warp_merge_heads<D, QT>(p, b, hg, HQC, qh_row0, GW, (int64_t)row + cf, cl - cf + 1);
        if (lane == 0) *cnt = 0;
      }
    }
  };

  int row = find_row(row_start, R, x0);
  int s = 0;
  uint32_t ph = 0;
  const int line0 = hk * DC * T;   // first line of this warp's KV head in a tile
  for (int x = x0; x < x1; ++x) {
    while (x >= row_start[row + 1]) ++row;
    if (row != cur_row) {
      if (cur_row >= 0) finish_row(cur_row);
      start_row(row);
      cur_row = row;
    }
    if (!mbar_wait(full + s, ph, p.wait_ns)) {
      record_status(p.status, kStatusTimeout);
      return;
    }
    const int tok0 = (x - row_start[row]) * T;
    const int nvalid = min(T, L - tok0);
    const uint32_t kb = tiles_u32 + (uint32_t)s * 2u * p.stage_bytes;
    const uint32_t vb = kb + p.stage_bytes;

    if (VL && nvalid < T) {
      // Same for the transposed V tile: elements (dim, token >= nvalid).
      const uint32_t vbh = vb + (uint32_t)(hk * D * 32);
      for (int idx = lane; idx < D * (T - nvalid); idx += 32) {
        const int dim = idx / (T - nvalid), tk = nvalid + idx % (T - nvalid);
        const uint32_t a = vbh + (uint32_t)(dim * 32 + tk * 2);
        asm volatile("st.shared.u16 [%0], %1;" ::"r"(a), "h"((unsigned short)0) : "memory");
      }
      __syncwarp();
    } else if (nvalid < T) {
      // Token slots past the sequence end (same page) may hold anything, even
      // NaN: zero those V lines of this head so P = 0 multiplies zeros.
      for (int idx = lane; idx < DC * (T - nvalid) * 8; idx += 32) {
        const int chunk = idx & 7, rest = idx >> 3;
        const int dc = rest / (T - nvalid), tk = nvalid + rest % (T - nvalid);
        const uint32_t a = vb + (uint32_t)((line0 + dc * T + tk) * 128 + chunk * 16);
        asm volatile("st.shared.v4.b32 [%0], {%1, %1, %1, %1};" ::"r"(a), "r"(0) : "memory");
      }
      __syncwarp();
    }

    // ---- S = Q . K^T for 16 tokens (two n-tiles of 8) ----
    float sfr[2][4];
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) sfr[j][e] = 0.f;
    if constexpr (!FP8) {
#pragma unroll
      for (int kk = 0; kk < D / 32; ++kk) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int mtx = lane >> 3, rr = lane & 7;
          const int dim = 32 * kk + 8 * mtx;
          uint32_t bfr[4];
          if constexpr (VL) {
            ldsm_x4(kb + (uint32_t)(hk * D * 32 + ((dim / 8) * 16 + 8 * j + rr) * 16), bfr);
          } else {
            const int line = line0 + (dim / LINE) * T + 8 * j + rr;
            ldsm_x4(swz(kb, line, (dim % LINE) / 8), bfr);
          }
          uint32_t a0[4], a1[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            a0[e] = (NP == 2) ? qa[2 * kk][e] : (e == 0 ? qa[2 * kk][0] : (e == 2 ? qa[2 * kk][1] : 0u));
            a1[e] = (NP == 2) ? qa[2 * kk + 1][e]
                              : (e == 0 ? qa[2 * kk + 1][0] : (e == 2 ? qa[2 * kk + 1][1] : 0u));
          }
          mma16816<MMA_BF16>(sfr[j], a0, bfr[0], bfr[1]);
          mma16816<MMA_BF16>(sfr[j], a1, bfr[2], bfr[3]);
        }
      }
    } else {
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        uint32_t a[4];
#pragma unroll
        for (int e = 0; e < 4; ++e)
          a[e] = (NP == 2) ? qa[ks][e] : (e == 0 ? qa[ks][0] : (e == 2 ? qa[ks][1] : 0u));
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int dim = 16 * ks;
          const int line = line0 + (dim / LINE) * T + 8 * j + g;
          const uint32_t w = lds32(swz(kb, line, (dim % LINE) / 16) + 4 * t);
          mma16816<false>(sfr[j], a, fp8_pair(w), fp8_pair(w >> 16));
        }
      }
    }

    // ---- online softmax over tokens (rows g and g + 8) ----
    float rmax[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int tok = 8 * j + 2 * t + (e & 1);
        float v = sfr[j][e] * sc;
        v = (tok < nvalid) ? v : -INFINITY;
        sfr[j][e] = v;
        rmax[e >> 1] = fmaxf(rmax[e >> 1], v);
      }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      rmax[r] = fmaxf(rmax[r], __shfl_xor_sync(0xffffffffu, rmax[r], 1));
      rmax[r] = fmaxf(rmax[r], __shfl_xor_sync(0xffffffffu, rmax[r], 2));
    }
    const bool grow = (rmax[0] > m_r[0]) || (NP == 2 && rmax[1] > m_r[1]);
    if (__any_sync(0xffffffffu, grow)) {
      float alpha[2];
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const float mn = fmaxf(m_r[r], rmax[r]);
        alpha[r] = (mn == -INFINITY) ? 1.f : fast_exp2(m_r[r] - mn);
        m_r[r] = mn;
        l_r[r] *= alpha[r];
      }
#pragma unroll
      for (int n = 0; n < NP; ++n) {
        const float a0 = __shfl_sync(0xffffffffu, alpha[n], 4 * (2 * t));
        const float a1 = __shfl_sync(0xffffffffu, alpha[n], 4 * (2 * t + 1));
#pragma unroll
        for (int i = 0; i < MT; ++i) {
          acc[n][i][0] *= a0;
          acc[n][i][1] *= a1;
          acc[n][i][2] *= a0;
          acc[n][i][3] *= a1;
        }
      }
    }
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float pv = fast_exp2(sfr[j][e] - m_r[e >> 1]);
        sfr[j][e] = pv;
        l_r[e >> 1] += pv;
      }
    // P as the B operand of the PV tile: tokens (2t, 2t+1) from n-tile 0 and
    // (2t+8, 2t+9) from n-tile 1, head column g (n = 0) or g + 8 (n = 1).
    uint32_t pb[NP][2];
#pragma unroll
    for (int n = 0; n < NP; ++n) {
      pb[n][0] = pack2<MMA_BF16>(sfr[0][2 * n], sfr[0][2 * n + 1]);
      pb[n][1] = pack2<MMA_BF16>(sfr[1][2 * n], sfr[1][2 * n + 1]);
    }

    // ---- O^T += V^T . P ----
    if constexpr (VL) {
      // V^T rows are dims: matrices (dims 0-7 | 8-15) x (tokens 0-7 | 8-15)
      // give the A fragment directly.
      const uint32_t vbh = vb + (uint32_t)(hk * D * 32);
#pragma unroll
      for (int i = 0; i < MT; ++i) {
        const int mtx = lane >> 3, rr = lane & 7;
        const int dim = 16 * i + 8 * (mtx & 1) + rr;
        uint32_t afr[4];
        ldsm_x4(vbh + (uint32_t)(dim * 32 + (mtx >> 1) * 16), afr);
#pragma unroll
        for (int n = 0; n < NP; ++n) mma16816<MMA_BF16>(acc[n][i], afr, pb[n][0], pb[n][1]);
      }
    } else if constexpr (!FP8) {
#pragma unroll
      for (int i = 0; i < MT; ++i) {
        const int mtx = lane >> 3, rr = lane & 7;
        const int dim = 16 * i + 8 * (mtx & 1);
        const int line = line0 + (dim / LINE) * T + 8 * (mtx >> 1) + rr;
        uint32_t afr[4];
        ldsm_x4_t(swz(vb, line, (dim % LINE) / 8), afr);
#pragma unroll
        for (int n = 0; n < NP; ++n) mma16816<MMA_BF16>(acc[n][i], afr, pb[n][0], pb[n][1]);
      }
    } else {
#pragma unroll
      for (int qd = 0; qd < D / 32; ++qd) {
        const int byte = (32 * qd) % LINE + 4 * g;
        const int dcl = (32 * qd) / LINE;
        const int lb = line0 + dcl * T;
        const uint32_t w0 = lds32(swz(vb, lb + 2 * t, byte / 16) + (byte & 15));
        const uint32_t w1 = lds32(swz(vb, lb + 2 * t + 1, byte / 16) + (byte & 15));
        const uint32_t w2 = lds32(swz(vb, lb + 2 * t + 8, byte / 16) + (byte & 15));
        const uint32_t w3 = lds32(swz(vb, lb + 2 * t + 9, byte / 16) + (byte & 15));
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          // tile 2qd+u: row g <-> byte 2u, row g+8 <-> byte 2u+1 of the 4-byte group
          const uint32_t s0 = (2 * u) | ((4 + 2 * u) << 4);
          const uint32_t s1 = (2 * u + 1) | ((4 + 2 * u + 1) << 4);
          uint32_t afr[4];
          afr[0] = fp8_pair(__byte_perm(w0, w1, s0));
          afr[1] = fp8_pair(__byte_perm(w0, w1, s1));
          afr[2] = fp8_pair(__byte_perm(w2, w3, s0));
          afr[3] = fp8_pair(__byte_perm(w2, w3, s1));
#pragma unroll
          for (int n = 0; n < NP; ++n) mma16816<false>(acc[n][2 * qd + u], afr, pb[n][0], pb[n][1]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty + s);
    if (++s == p.stages) {
      s = 0;
      ph ^= 1u;
    }
  }
  if (cur_row >= 0) finish_row(cur_row);
}

}  // namespace b2d
