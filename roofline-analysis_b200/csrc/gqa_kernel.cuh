// gqa_kernel.cuh — split-KV paged GQA/MHA/MQA decode for sm_100a.
//
// Math (per query head h with KV head g = h / group):
//   s_t = softmax_scale * <q_h, K[g, t]>,  out_h = sum_t softmax(s)_t V[g, t],
//   lse_h = ln sum_t exp(s_t)
// — the same quantity as torch SDPA with enable_gqa
// (decodebench/torch_sdpa_benchmark.py:100-102) gathered through the block
// table like flash_attn_with_kvcache (decodebench/flashattn_kvcache_kernel.py:
// 161-169).  Splits are merged with the LSE rule of
// cute_attention/cluster_decode/cluster_decode_reduce.py:67-91.
//
// Work decomposition.  A "row" is (sequence b, group of HK KV heads).  Row r
// holds n_r = ceil(L_b / T) chunks of T tokens.  All chunks of all rows form
// one line of W chunks, cut into G equal contiguous ranges, one per CTA (a
// balanced, static stream-K split: every CTA streams the same number of
// bytes whatever the length distribution).  A CTA whose range covers a whole
// row writes the final output; otherwise it writes a normalised partial
// (o, log2-sum-exp) for segment id (row + cta), merged afterwards by the
// combine kernel.
//
// Pipeline.  Warp NW (the producer) streams each chunk's K and V tiles
// [T tokens][HK heads][D] from the paged cache into a ring of shared-memory
// stages with 4-D TMA loads (full/empty mbarrier pairs).  Consumer warp w
// owns KV head w / WPH of the tile and HQW of its query heads; lane
// (r = lane / LPR, c = lane % LPR) reads 8 consecutive elements of token row
// r with one 16-byte (8-byte for fp8) shared load, so each quarter-warp reads
// 128 contiguous bytes (no bank conflicts, no swizzle needed).  The HQW
// partial dot products of a row are reduce-scattered over its LPR lanes, so
// a lane ends up owning one head's full score; the online softmax keeps
// (m, l) per owned head in log2 units; P·V accumulates in fp32 with packed
// f32x2 FMAs.
#pragma once

#include <type_traits>

#include "common.cuh"

// Register cap of the split-KV kernel: 96 lets two 9-warp CTAs share an SM
// (five warps per SM sub-partition at 96 x 32 registers each).
#ifndef B2D_GQA_MAXNREG
#define B2D_GQA_MAXNREG 96
#endif

namespace b2d {

enum KvKind : int { kKvBf16 = 0, kKvFp16 = 1, kKvFp8 = 2 };

struct GqaParams {
  const void* q;
  int64_t q_sb, q_sh;
  void* out;
  int64_t o_sb, o_sh;
  float* lse;
  int64_t lse_sb;
  const int32_t* seqlens;
  const int32_t* block_table;
  int64_t bt_stride;
  const float* k_scale;
  const float* v_scale;
  float* part_o;     // [(R + G) * HQC * D]
  float* part_lse;   // [(R + G) * HQC], log2 units
  int32_t* row_start_g;  // [R + 1], written by CTA 0 for the combine
  int32_t* merge_count;  // [R * NW] arrival counters of the in-kernel merge, or
                         // null when a separate combine kernel merges
  int* status;
  unsigned long long wait_ns;  // bounded-wait limit of every mbarrier wait
  int no_loads;                // test only: the producer issues no loads
  int B, Hq, Hkv, group, HK, HG, P, T, stages, NW, WPH;
  int num_pages, max_pages;
  float scale_log2;        // softmax_scale * log2(e)
  uint32_t stage_bytes;    // bytes of one K (or V) tile
};

// Exclusive block-wide scan of n_r = ceil(min(L_b, cap) / T) over R rows
// into smem row_start[0..R].
__device__ __forceinline__ void build_row_start(const GqaParams& p, int R, int32_t* row_start,
                                                int32_t* warp_tmp) {
  const int tid = threadIdx.x, nth = blockDim.x;
  const int lane = tid & 31, warp = tid >> 5, nwarps = nth >> 5;
  const int cap = p.max_pages * p.P;
  int carry = 0;
  for (int base = 0; base < R; base += nth) {
    const int r = base + tid;
    int n = 0;
    if (r < R) {
      int L = __ldg(p.seqlens + r / p.HG);
      L = L < 0 ? 0 : (L > cap ? cap : L);
      n = (L + p.T - 1) / p.T;
    }
    int x = n;  // inclusive warp scan
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) warp_tmp[warp] = x;
    __syncthreads();
    if (warp == 0) {
      int w = lane < nwarps ? warp_tmp[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += y;
      }
      if (lane < nwarps) warp_tmp[lane] = w;  // inclusive over warps
    }
    __syncthreads();
    const int before = carry + (warp > 0 ? warp_tmp[warp - 1] : 0) + x - n;
    if (r < R) row_start[r] = before;
    const int total = warp_tmp[nwarps - 1];
    __syncthreads();
    carry += total;
  }
  if (tid == 0) row_start[R] = carry;
  __syncthreads();
}

// CTA index whose chunk range contains global chunk x (ranges start at
// floor(c * W / G)).
__device__ __forceinline__ int cta_of_chunk(int64_t x, int64_t W, int G) {
  return static_cast<int>(((x + 1) * G - 1) / W);
}

__device__ __forceinline__ int find_row(const int32_t* row_start, int R, int64_t x) {
  int lo = 0, hi = R - 1;  // last r with row_start[r] <= x
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (row_start[mid] <= x) lo = mid; else hi = mid - 1;
  }
  while (lo + 1 <= R - 1 && row_start[lo + 1] <= x) ++lo;  // skip empty rows
  return lo;
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float fast_log2(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <typename QT>
__device__ __forceinline__ void load_q8(const QT* src, float* dst) {
  const uint4 w = *reinterpret_cast<const uint4*>(src);
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f;
    if constexpr (std::is_same<QT, __nv_bfloat16>::value) f = bf16x2_to_f2(ws[i]);
    else f = f16x2_to_f2(ws[i]);
    dst[2 * i] = f.x;
    dst[2 * i + 1] = f.y;
  }
}

template <typename QT>
__device__ __forceinline__ void store_out8(QT* dst, const float* v) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if constexpr (std::is_same<QT, __nv_bfloat16>::value) {
      __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
      w[i] = *reinterpret_cast<uint32_t*>(&h);
    } else {
      __half2 h = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
      w[i] = *reinterpret_cast<uint32_t*>(&h);
    }
  }
  *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
}

// Load 8 KV elements of one row as fp32 (fp8 values come out times 2^-8).
template <int KIND>
__device__ __forceinline__ void load_kv8(uint32_t addr, float2* v) {
  if constexpr (KIND == kKvFp8) {
    const uint2 w = lds64(addr);
    v[0] = f16x2_to_f2(e4m3x2_to_f16x2_scaled(w.x));
    v[1] = f16x2_to_f2(e4m3x2_to_f16x2_scaled(w.x >> 16));
    v[2] = f16x2_to_f2(e4m3x2_to_f16x2_scaled(w.y));
    v[3] = f16x2_to_f2(e4m3x2_to_f16x2_scaled(w.y >> 16));
  } else {
    const uint4 w = lds128(addr);
    if constexpr (KIND == kKvBf16) {
      v[0] = bf16x2_to_f2(w.x);
      v[1] = bf16x2_to_f2(w.y);
      v[2] = bf16x2_to_f2(w.z);
      v[3] = bf16x2_to_f2(w.w);
    } else {
      v[0] = f16x2_to_f2(w.x);
      v[1] = f16x2_to_f2(w.y);
      v[2] = f16x2_to_f2(w.z);
      v[3] = f16x2_to_f2(w.w);
    }
  }
}

template <int D, int KIND, typename QT, int HQW>
__global__ void __maxnreg__(B2D_GQA_MAXNREG)
    gqa_decode_kernel(const __grid_constant__ CUtensorMap tmap_k,
                      const __grid_constant__ CUtensorMap tmap_v, const GqaParams p) {
  constexpr int ES = (KIND == kKvFp8) ? 1 : 2;  // bytes per KV element
  constexpr int LPR = D / 8;                    // lanes per token row
  constexpr int RPW = 32 / LPR;                 // token rows per warp step
  constexpr int IT = (RPW >= 4 || HQW == 4) ? 2 : 4;  // warp steps per softmax update
  constexpr float kLn2 = 0.69314718055994530942f;

  extern __shared__ __align__(1024) uint8_t smem[];
  const int R = p.B * p.HG;
  const int cta = blockIdx.x;

  // Shared-memory map: [stages][K tile | V tile] | full[stages] | empty[stages]
  //                    | row_start[R + 1] | warp scratch[32]
  uint8_t* tiles = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)p.stages * 2 * p.stage_bytes);
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
  build_row_start(p, R, row_start, warp_tmp);  // ends with __syncthreads
  if (cta == 0) {
    for (int i = threadIdx.x; i <= R; i += blockDim.x) p.row_start_g[i] = row_start[i];
  }

  const int64_t W = row_start[R];
  // With fewer chunks than CTAs only the first W CTAs work (one chunk or
  // more each), so no segment id is ever left unwritten.
  const int G = W < (int64_t)gridDim.x ? (int)W : (int)gridDim.x;
  if (W == 0 || cta >= G) return;
  // Chunk indices fit in 32 bits (the host bounds W); only the range cut
  // itself needs 64-bit products.
  const int x0 = (int)((int64_t)cta * W / G);
  const int x1 = (int)((int64_t)(cta + 1) * W / G);
  const int cap = p.max_pages * p.P;

  if (warp == p.NW) {
    // ---------------- producer warp ----------------
    if (p.no_loads) return;  // test flag: every consumer wait then runs out
    const uint64_t policy = policy_evict_first();
    bool ok = true;
    int s = 0;
    uint32_t ph = 0;
    for (int gbase = x0; gbase < x1 && ok; gbase += 32) {
      // Each lane resolves one chunk's page id (coalesced block-table reads).
      const int x = gbase + lane;
      int my_page = 0, my_off = 0, my_h0 = 0;
      if (x < x1) {
        const int rr = find_row(row_start, R, x);
        const int b = rr / p.HG, hg = rr - b * p.HG;
        const int tok0 = (int)(x - row_start[rr]) * p.T;
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
            tma_load_4d(kdst, &tmap_k, full + s, 0, h0, off, page, policy);
            tma_load_4d(kdst + p.stage_bytes, &tmap_v, full + s, 0, h0, off, page, policy);
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
  // Lane layout: r_in = lane / LPR picks the token row of a warp step,
  // c_in = lane % LPR the 8-element column block.  After the dot products
  // the HQW partial scores of a row are reduce-scattered over its LPR lanes:
  // the top one or two bits of c_in pick the query head a lane keeps (its
  // "own" head), so each lane holds one full score per row instead of HQW.
  const int hk = warp / p.WPH;           // KV head within the tile
  const int qg = warp - hk * p.WPH;      // group of HQW query heads
  const int r_in = lane / LPR;           // token row within a warp step
  const int c_in = lane % LPR;           // 8-element column block
  const int HQC = p.HK * p.group;        // query heads per row
  constexpr int HB = (HQW == 4) ? 2 : (HQW == 2 ? 1 : 0);  // head bits
  constexpr int TOP = LPR >> 1;          // top bit of c_in
  // lane of the same row that keeps head h
  auto head_lane = [&](int h) {
    int hb = 0;
    if constexpr (HB == 2) hb = ((h >> 1) ? TOP : 0) | ((h & 1) ? (TOP >> 1) : 0);
    else if constexpr (HB == 1) hb = h ? TOP : 0;
    constexpr int mask = (HB == 2) ? (TOP | (TOP >> 1)) : (HB == 1 ? TOP : 0);
    return (lane & ~mask) | hb;
  };
  const uint32_t row_bytes = (uint32_t)(p.HK * D * ES);
  const uint32_t tiles_u32 = smem_u32(tiles);
  const uint32_t col_off = (uint32_t)(hk * D * ES + c_in * 8 * ES);

  float2 q[HQW][4];
  float2 acc[HQW][4];
  float m_own = -INFINITY, l_own = 0.f;   // online-softmax state of the own head
  int cur_row = -1;
  int L = 0;
  float vscale = 1.f;

  auto finish_row = [&](int row) {
    // Reduce l and acc over the RPW token rows of the warp.
#pragma unroll
    for (int o = LPR; o < 32; o <<= 1) l_own += __shfl_xor_sync(0xffffffffu, l_own, o);
#pragma unroll
    for (int h = 0; h < HQW; ++h) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
#pragma unroll
        for (int o = LPR; o < 32; o <<= 1) {
          acc[h][e].x += __shfl_xor_sync(0xffffffffu, acc[h][e].x, o);
          acc[h][e].y += __shfl_xor_sync(0xffffffffu, acc[h][e].y, o);
        }
      }
    }
    const float lse2_own = m_own + fast_log2(l_own);
    const float inv_own = 1.f / l_own;
    const int b = row / p.HG, hg = row - b * p.HG;
    const int cf = cta_of_chunk(row_start[row], W, G);
    const int cl = cta_of_chunk(row_start[row + 1] - 1, W, G);
#pragma unroll
    for (int h = 0; h < HQW; ++h) {
      const float inv = __shfl_sync(0xffffffffu, inv_own, head_lane(h)) * vscale;
      const float lse2 = __shfl_sync(0xffffffffu, lse2_own, head_lane(h));
      if (r_in != 0) continue;
      const int qh_row = hk * p.group + qg * HQW + h;  // query head within the row
      float o8[8];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        o8[2 * e] = acc[h][e].x * inv;
        o8[2 * e + 1] = acc[h][e].y * inv;
      }
      if (cf == cl) {
        const int qh = hg * HQC + qh_row;
        QT* dst = reinterpret_cast<QT*>(p.out) + (int64_t)b * p.o_sb + (int64_t)qh * p.o_sh + c_in * 8;
        store_out8<QT>(dst, o8);
        if (p.lse != nullptr && c_in == 0) p.lse[(int64_t)b * p.lse_sb + qh] = lse2 * kLn2;
      } else {
        const int64_t seg = (int64_t)row + cta;
        float* dst = p.part_o + (seg * HQC + qh_row) * D + c_in * 8;
        *reinterpret_cast<float4*>(dst) = make_float4(o8[0], o8[1], o8[2], o8[3]);
        *reinterpret_cast<float4*>(dst + 4) = make_float4(o8[4], o8[5], o8[6], o8[7]);
        if (c_in == 0) p.part_lse[seg * HQC + qh_row] = lse2;
      }
    }
  };

  auto start_row = [&](int row) {
    const int b = row / p.HG, hg = row - b * p.HG;
    int Lb = __ldg(p.seqlens + b);
    L = Lb < 0 ? 0 : (Lb > cap ? cap : Lb);
    const int kvh = hg * p.HK + hk;
    float qs = p.scale_log2;
    vscale = 1.f;
    if constexpr (KIND == kKvFp8) {
      qs *= (p.k_scale ? __ldg(p.k_scale + kvh) : 1.f) * 256.f;
      vscale = (p.v_scale ? __ldg(p.v_scale + kvh) : 1.f) * 256.f;
    }
#pragma unroll
    for (int h = 0; h < HQW; ++h) {
      const int qh = kvh * p.group + qg * HQW + h;
      const QT* src = reinterpret_cast<const QT*>(p.q) + (int64_t)b * p.q_sb + (int64_t)qh * p.q_sh + c_in * 8;
      float qf[8];
      load_q8<QT>(src, qf);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        q[h][e] = make_float2(qf[2 * e] * qs, qf[2 * e + 1] * qs);
        acc[h][e] = make_float2(0.f, 0.f);
      }
    }
    m_own = -INFINITY;
    l_own = 0.f;
  };

  // One softmax step over IT warp steps (IT * RPW tokens) starting at t0.
  // MASKED: some rows may lie past the sequence end (last chunk only).
  auto process = [&](uint32_t kbase, uint32_t vbase, int t0, int nvalid, auto masked_tag) {
    constexpr bool MASKED = decltype(masked_tag)::value;
    float s_own[IT];
#pragma unroll
    for (int it = 0; it < IT; ++it) {
      const int t = t0 + it * RPW + r_in;
      int tc = t;
      if constexpr (MASKED) tc = t < p.T ? t : p.T - 1;
      float2 kv[4];
      load_kv8<KIND>(kbase + (uint32_t)tc * row_bytes, kv);
      float part[HQW];
#pragma unroll
      for (int h = 0; h < HQW; ++h) {
        float2 a = __fmul2_rn(q[h][0], kv[0]);
#pragma unroll
        for (int e = 1; e < 4; ++e) a = __ffma2_rn(q[h][e], kv[e], a);
        part[h] = a.x + a.y;
      }
      // reduce-scatter the HQW partial dots over the LPR lanes of the row
      float mine;
      if constexpr (HB == 2) {
        const bool up = (c_in & TOP) != 0;
        const float s0 = up ? part[0] : part[2], s1 = up ? part[1] : part[3];
        const float r0 = __shfl_xor_sync(0xffffffffu, s0, TOP);
        const float r1 = __shfl_xor_sync(0xffffffffu, s1, TOP);
        const float k0 = (up ? part[2] : part[0]) + r0;
        const float k1 = (up ? part[3] : part[1]) + r1;
        const bool up2 = (c_in & (TOP >> 1)) != 0;
        const float r2 = __shfl_xor_sync(0xffffffffu, up2 ? k0 : k1, TOP >> 1);
        mine = (up2 ? k1 : k0) + r2;
#pragma unroll
        for (int o = TOP >> 2; o >= 1; o >>= 1) mine += __shfl_xor_sync(0xffffffffu, mine, o);
      } else if constexpr (HB == 1) {
        const bool up = (c_in & TOP) != 0;
        const float r0 = __shfl_xor_sync(0xffffffffu, up ? part[0] : part[1], TOP);
        mine = (up ? part[1] : part[0]) + r0;
#pragma unroll
        for (int o = TOP >> 1; o >= 1; o >>= 1) mine += __shfl_xor_sync(0xffffffffu, mine, o);
      } else {
        mine = part[0];
#pragma unroll
        for (int o = TOP; o >= 1; o >>= 1) mine += __shfl_xor_sync(0xffffffffu, mine, o);
      }
      if constexpr (MASKED) mine = (t < nvalid) ? mine : -INFINITY;
      s_own[it] = mine;
    }
    // online softmax of the own head (log2 domain)
    float cm = s_own[0];
#pragma unroll
    for (int it = 1; it < IT; ++it) cm = fmaxf(cm, s_own[it]);
#pragma unroll
    for (int o = LPR; o < 32; o <<= 1) cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, o));
    const bool grow = cm > m_own;
    if (__any_sync(0xffffffffu, grow)) {
      const float m_new = fmaxf(m_own, cm);
      const float alpha_own = fast_exp2(m_own - m_new);
      l_own *= alpha_own;
      m_own = m_new;
#pragma unroll
      for (int h = 0; h < HQW; ++h) {
        const float al = __shfl_sync(0xffffffffu, alpha_own, head_lane(h));
        const float2 a2 = make_float2(al, al);
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[h][e] = __fmul2_rn(acc[h][e], a2);
      }
    }
#pragma unroll
    for (int it = 0; it < IT; ++it) {
      s_own[it] = fast_exp2(s_own[it] - m_own);
      l_own += s_own[it];
    }
#pragma unroll
    for (int it = 0; it < IT; ++it) {
      const int t = t0 + it * RPW + r_in;
      int tc = t;
      if constexpr (MASKED) tc = t < p.T ? t : p.T - 1;
      float2 vv[4];
      load_kv8<KIND>(vbase + (uint32_t)tc * row_bytes, vv);
      if constexpr (MASKED) {
        if (t >= nvalid) {  // the page tail past L may hold anything, even NaN
#pragma unroll
          for (int e = 0; e < 4; ++e) vv[e] = make_float2(0.f, 0.f);
        }
      }
#pragma unroll
      for (int h = 0; h < HQW; ++h) {
        const float ph = __shfl_sync(0xffffffffu, s_own[it], head_lane(h));
        const float2 pp = make_float2(ph, ph);
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[h][e] = __ffma2_rn(pp, vv[e], acc[h][e]);
      }
    }
  };

  int row = find_row(row_start, R, x0);
  int s = 0;
  uint32_t ph = 0;
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
    const int tok0 = (x - row_start[row]) * p.T;
    const int nvalid = min(p.T, L - tok0);
    const uint32_t kbase = tiles_u32 + (uint32_t)s * 2u * p.stage_bytes + col_off;
    const uint32_t vbase = kbase + p.stage_bytes;
    constexpr int STEP = IT * RPW;
    if (nvalid == p.T && (p.T % STEP) == 0) {
      for (int t0 = 0; t0 < p.T; t0 += STEP)
        process(kbase, vbase, t0, nvalid, std::false_type{});
    } else {
      for (int t0 = 0; t0 < nvalid; t0 += STEP)
        process(kbase, vbase, t0, nvalid, std::true_type{});
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

// One warp merges the split partials of query heads [qh_row0, qh_row0 + nh)
// of row (b, hg) over segments seg0 .. seg0 + nseg - 1 (the LSE rule of
// cluster_decode_reduce.py:67-91 in log2 units) and writes out and lse.
// Used by the split-KV kernel's last-arriving warp, at the very end of the
// kernel, so it is pure latency: two heads are merged at once (half a warp
// each, 2 * D / 32 elements per lane) and every segment's lse and partial
// output of a batch of U segments are loaded together, folded in with a
// running maximum.  The partials of other CTAs are read past L1 (__ldcg),
// after the acquire fence of the arrival counter.
template <int D, typename QT>
__device__ __forceinline__ void warp_merge_heads(const GqaParams& p, int b, int hg, int HQC,
                                                 int qh_row0, int nh, int64_t seg0, int nseg) {
  constexpr float kLn2 = 0.69314718055994530942f;
  constexpr int EPL = D / 16;              // elements per lane (half a warp per head)
  constexpr int U = D <= 128 ? 8 : 4;      // segments per load batch
  const int lane = threadIdx.x & 31;
  const int half = lane >> 4, hl = lane & 15;
  for (int hw0 = 0; hw0 < nh; hw0 += 2) {
    const int hw = hw0 + half;
    const bool live = hw < nh;
    const int qh_row = qh_row0 + (live ? hw : hw0);
    float acc[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e) acc[e] = 0.f;
    float wsum = 0.f, mx = -INFINITY;
    for (int j0 = 0; j0 < nseg; j0 += U) {
      float lv[U];
      float2 v[U][EPL / 2];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int j = j0 + u < nseg ? j0 + u : nseg - 1;
        lv[u] = __ldcg(p.part_lse + (seg0 + j) * HQC + qh_row);
        const float2* src = reinterpret_cast<const float2*>(
            p.part_o + ((seg0 + j) * HQC + qh_row) * D + hl * EPL);
#pragma unroll
        for (int e = 0; e < EPL / 2; ++e) v[u][e] = __ldcg(src + e);
      }
      float bm = mx;
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (j0 + u < nseg) bm = fmaxf(bm, lv[u]);
      const float r = (mx == -INFINITY) ? 0.f : fast_exp2(mx - bm);
      wsum *= r;
#pragma unroll
      for (int e = 0; e < EPL; ++e) acc[e] *= r;
      mx = bm;
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const float w = (j0 + u < nseg) ? fast_exp2(lv[u] - mx) : 0.f;
        wsum += w;
#pragma unroll
        for (int e = 0; e < EPL / 2; ++e) {
          acc[2 * e] += w * v[u][e].x;
          acc[2 * e + 1] += w * v[u][e].y;
        }
      }
    }
    if (live) {
      const int qh = hg * HQC + qh_row;
      QT* dst = reinterpret_cast<QT*>(p.out) + (int64_t)b * p.o_sb + (int64_t)qh * p.o_sh + hl * EPL;
      const float inv = 1.f / wsum;
#pragma unroll
      for (int e = 0; e < EPL; ++e) dst[e] = QT(acc[e] * inv);
      if (p.lse != nullptr && hl == 0) p.lse[(int64_t)b * p.lse_sb + qh] = (mx + fast_log2(wsum)) * kLn2;
    }
  }
}

// One warp writes out = 0, lse = -inf for query heads [qh_row0, qh_row0 + nh)
// of a zero-length row (b, hg).
template <int D, typename QT>
__device__ __forceinline__ void warp_zero_heads(const GqaParams& p, int b, int hg, int HQC,
                                                int qh_row0, int nh) {
  constexpr int EPL = D / 32;
  const int lane = threadIdx.x & 31;
  for (int hw = 0; hw < nh; ++hw) {
    const int qh = hg * HQC + qh_row0 + hw;
    QT* dst = reinterpret_cast<QT*>(p.out) + (int64_t)b * p.o_sb + (int64_t)qh * p.o_sh + lane * EPL;
#pragma unroll
    for (int e = 0; e < EPL; ++e) dst[e] = QT(0.f);
    if (p.lse != nullptr && lane == 0) p.lse[(int64_t)b * p.lse_sb + qh] = -INFINITY;
  }
}

// Merge the split partials of every row that more than one CTA touched
// (cluster_decode_reduce.py:67-91 in log2 units), and write out = 0,
// lse = -inf for rows of zero length.  `wpp` warps (1, 2, 4 or 8) merge one
// (row, query head): with few rows (small batches) each row is split over
// many CTAs and one warp per merge would leave most SMs idle.
template <int D, typename QT>
__global__ void __launch_bounds__(256) gqa_combine_kernel(const GqaParams p, int G, int wpp) {
  constexpr float kLn2 = 0.69314718055994530942f;
  constexpr int EPL = D / 32;  // elements per lane
  static_assert(EPL % 2 == 0, "combine loads float2 pairs");
  // U segments per step, all loads issued before any is used (a chain of
  // dependent L2 round trips otherwise).
  constexpr int U = D >= 512 ? 2 : (D >= 256 ? 4 : 8);
  __shared__ float red_acc[8][EPL][32];
  __shared__ float red_w[8];
  const int R = p.B * p.HG;
  const int HQC = p.HK * p.group;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = warp % wpp;
  const int64_t gw = (int64_t)blockIdx.x * (8 / wpp) + warp / wpp;
  const int64_t W = p.row_start_g[R];
  if (W < (int64_t)G) G = (int)W;  // the decode kernel's effective CTA count
  int mode = 0;                    // 0: nothing, 1: zero-length row, 2: merge
  int row = 0, b = 0, qh = 0, qh_row = 0, nseg = 0;
  int64_t seg0 = 0;
  if (gw < (int64_t)R * HQC) {
    row = (int)(gw / HQC);
    qh_row = (int)(gw - (int64_t)row * HQC);
    b = row / p.HG;
    const int hg = row - b * p.HG;
    qh = hg * HQC + qh_row;
    const int rs = p.row_start_g[row], re = p.row_start_g[row + 1];
    if (re == rs) {
      mode = 1;
    } else {
      const int cf = cta_of_chunk(rs, W, G), cl = cta_of_chunk(re - 1, W, G);
      if (cf != cl) {  // else written directly by the decode kernel
        mode = 2;
        nseg = cl - cf + 1;
        seg0 = (int64_t)row + cf;
      }
    }
  }
  QT* dst = reinterpret_cast<QT*>(p.out) + (int64_t)b * p.o_sb + (int64_t)qh * p.o_sh + lane * EPL;
  if (mode == 1 && sub == 0) {
#pragma unroll
    for (int e = 0; e < EPL; ++e) dst[e] = QT(0.f);
    if (p.lse != nullptr && lane == 0) p.lse[(int64_t)b * p.lse_sb + qh] = -INFINITY;
  }
  float acc[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) acc[e] = 0.f;
  float wsum = 0.f, mx = -INFINITY;
  if (mode == 2) {
    for (int j = lane; j < nseg; j += 32) mx = fmaxf(mx, p.part_lse[(seg0 + j) * HQC + qh_row]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    for (int j0 = sub * U; j0 < nseg; j0 += wpp * U) {
      float lv[U];
      float2 v[U][EPL / 2];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int j = j0 + u < nseg ? j0 + u : nseg - 1;
        lv[u] = p.part_lse[(seg0 + j) * HQC + qh_row];
        const float* src = p.part_o + ((seg0 + j) * HQC + qh_row) * D + lane * EPL;
#pragma unroll
        for (int e = 0; e < EPL / 2; ++e) v[u][e] = *reinterpret_cast<const float2*>(src + 2 * e);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const float w = (j0 + u < nseg) ? fast_exp2(lv[u] - mx) : 0.f;
        wsum += w;
#pragma unroll
        for (int e = 0; e < EPL / 2; ++e) {
          acc[2 * e] += w * v[u][e].x;
          acc[2 * e + 1] += w * v[u][e].y;
        }
      }
    }
  }
  if (wpp > 1) {
#pragma unroll
    for (int e = 0; e < EPL; ++e) red_acc[warp][e][lane] = acc[e];
    if (lane == 0) red_w[warp] = wsum;
    __syncthreads();
    if (mode == 2 && sub == 0) {
      for (int w = 1; w < wpp; ++w) {
#pragma unroll
        for (int e = 0; e < EPL; ++e) acc[e] += red_acc[warp + w][e][lane];
        wsum += red_w[warp + w];
      }
    }
  }
  if (mode == 2 && sub == 0) {
    const float inv = 1.f / wsum;
#pragma unroll
    for (int e = 0; e < EPL; ++e) dst[e] = QT(acc[e] * inv);
    if (p.lse != nullptr && lane == 0) p.lse[(int64_t)b * p.lse_sb + qh] = (mx + fast_log2(wsum)) * kLn2;
  }
}

}  // namespace b2d
