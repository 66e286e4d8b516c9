// mla_kernel.cuh — absorbed-MLA paged decode on tcgen05 tensor cores (sm_100a).
//
// Math (decodebench/trtllm_mla_kernel.py:115-132): 128 query heads of width
// 576 (512 latent + 64 rope) attend to one shared latent KV head of width
// 576; V is the first 512 columns of the same cache row.
//   S = q . K^T * scale,  out = softmax(S) . V,  lse = ln sum exp(S)
//
// Work: a CTA pair shares one range of 64-token chunks (the same balanced
// stream-K cut over all sequences as the GQA kernel); CTA 2r+h computes the
// 64 query heads [64h, 64h+64) of range r.  Both CTAs of a pair stream the
// same KV tiles close together in time, so the second read is an L2 hit.
//
// Tensor memory (512 columns x 128 lanes, fp32): an M=64 UMMA writes its 64
// rows to 16 lanes of each 32-lane quadrant, lane half 0 (lanes 0-15,
// 32-47, ...) or lane half 1 (16-31, ...) as the address selects.  The O
// accumulator [64 heads x 512] takes columns 0-255 of both halves (half 0:
// dims 0-255, half 1: dims 256-511); the score tiles S [64 heads x 64 tokens]
// (double-buffered) take columns 256-383 of half 0.  Thread i of softmax
// warp w owns head 16w + (i & 15): lanes < 16 read its S row (one whole row
// per thread: row max and sum need no shuffles) and hold O dims 0-255, lanes
// >= 16 hold O dims 256-511.  Rescaling O rewrites columns 0-255 only, so it
// never touches a score tile the tensor core may be writing.
//
// Shared memory: Q [9 x 64 heads x 64] and each KV stage [9 x 32 tok x 64]
// bf16 arrive by TMA with 128-byte swizzle (K-major canonical UMMA layout:
// 8-row x 128-byte atoms, 1024-byte stride).  The same KV stage is the
// K-major B operand of S = Q.K^T and the MN-major B operand of O += P.V
// (V = its first 8 column blocks), so each latent row is fetched once.
// P goes to shared memory as bf16 in the same swizzled K-major layout.
//
// Warp roles: warps 0-3 softmax + epilogue, warp 4 TMA producer, warp 5
// TMEM allocator + single-thread MMA issuer.  Online softmax uses a lazy
// rescale: the running max moves only when a score exceeds it by 8 (log2
// units), so P <= 256 fits bf16 and O is rescaled (TMEM round trip) rarely.
#pragma once

#include "gqa_kernel.cuh"
#include "gqa_mma_kernel.cuh"

namespace b2d {

struct MlaParams {
  const int32_t* seqlens;
  const int32_t* block_table;
  int64_t bt_stride;
  void* out;                 // bf16 [B, 128, 512]
  int64_t o_sb, o_sh;
  float* lse;
  int64_t lse_sb;
  float* part_o;             // [(B + NR) * 128 * 512]
  float* part_lse;           // [(B + NR) * 128], log2 units
  int32_t* row_start_g;      // [B + 1]
  int* status;
  int B, P, num_pages, max_pages;
  float scale_log2;
};

namespace mla {
constexpr int kHeads = 64;         // query heads per CTA
constexpr int kDqk = 576, kDv = 512;
constexpr int kCB = kDqk / 64;     // 128-byte column blocks per row (9)
constexpr int kT = 64;             // tokens per chunk (one TMA box; page size % 64 == 0)
constexpr int kStages = 2;
constexpr uint32_t kQBytes = kCB * kHeads * 128;     // 73728
constexpr uint32_t kStageBytes = kCB * kT * 128;     // 73728
constexpr int kSplit = 1;          // independent QK accumulators per score tile
constexpr int kSBuf = 2;           // score tiles in TMEM (lane half 0, columns 256 + 64k)
constexpr int kPBuf = 1;           // P tile in shared memory (64 heads x 64 tokens bf16)
constexpr uint32_t kPBytes = kHeads * 128;           // 8192
constexpr int kAhead = 1;          // QK tiles issued ahead of the oldest pending P.V
constexpr float kLazy = 8.f;                         // lazy-rescale threshold, log2 units
#ifndef B2D_MLA_L2_AHEAD
#define B2D_MLA_L2_AHEAD 2
#endif
constexpr int kL2Ahead = B2D_MLA_L2_AHEAD;           // chunks prefetched into L2 past the ring
constexpr int kThreads = 6 * 32;
// shared-memory map (offsets from the 1024-aligned base)
constexpr uint32_t kOffQ = 0;
constexpr uint32_t kOffKV = kOffQ + kQBytes;
constexpr uint32_t kOffP = kOffKV + kStages * kStageBytes;
constexpr uint32_t kOffBar = kOffP + kPBuf * kPBytes;
// kv full/empty, q full/empty, s full, p full, pv done, o full/empty
constexpr uint32_t kNumBars = 2 * kStages + 2 + kSBuf + kPBuf + kPBuf + 2;
constexpr uint32_t kOffTmem = kOffBar + kNumBars * 8;
constexpr uint32_t kOffRows = kOffTmem + 16;
}  // namespace mla

#ifndef B2D_MLA_EVICT_FIRST
#define B2D_MLA_EVICT_FIRST 0
#endif
// Cache policy of the KV loads: the head-pair partner CTA reads each tile
// again shortly after, so by default it stays in L2 normally.
__device__ __forceinline__ uint64_t kv_policy() {
  uint64_t p;
  if (B2D_MLA_EVICT_FIRST)
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  else
    asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// L2 prefetch of one 5-D TMA box (no shared-memory destination).
__device__ __forceinline__ void tma_prefetch_5d(const CUtensorMap* map, int c1, int c2, int c3,
                                                int c4) {
  asm volatile(
      "cp.async.bulk.prefetch.tensor.5d.L2.global.tile [%0, {%1, %2, %3, %4, %5}];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
      : "memory");
}

__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr, uint32_t lbo_bytes,
                                                    uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;          // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;          // 128-byte swizzle
  return d;
}

// Instruction descriptor: bf16 x bf16 -> fp32, A K-major, B K- or MN-major.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int M, int N, bool b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((b_mn_major ? 1u : 0u) << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"((uint32_t)accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 32 consecutive fp32 TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, "
      "%29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, "
      "%29, %30, %31, %32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Named barrier over the 128 softmax threads; returns whether any thread's
// predicate was true.
__device__ __forceinline__ bool softmax_group_any(bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.b32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 1, 128, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ void softmax_group_sync() {
  asm volatile("bar.sync 1, 128;" ::: "memory");
}

// Wait helper that records a timeout; returns false when the kernel must stop.
__device__ __forceinline__ bool mla_wait(uint64_t* bar, uint32_t parity, int* status) {
  if (mbar_wait(bar, parity)) return true;
  record_status(status, kStatusTimeout);
  return false;
}

__global__ void __launch_bounds__(mla::kThreads, 1)
    mla_decode_kernel(const __grid_constant__ CUtensorMap tmap_q,
                      const __grid_constant__ CUtensorMap tmap_kv, const MlaParams p) {
  using namespace mla;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const uint32_t sbase = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* kv_full = bars;
  uint64_t* kv_empty = bars + kStages;
  uint64_t* q_full = bars + 2 * kStages;
  uint64_t* q_empty = q_full + 1;
  uint64_t* s_full = q_full + 2;      // [kSBuf]
  uint64_t* p_full = s_full + kSBuf;  // [kPBuf]
  uint64_t* pv_done = p_full + kPBuf; // [kPBuf]
  uint64_t* o_full = pv_done + kPBuf;
  uint64_t* o_empty = o_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffTmem);
  int32_t* row_start = reinterpret_cast<int32_t*>(smem + kOffRows);
  int32_t* warp_tmp = row_start + (p.B + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int R = p.B;
  const int NR = gridDim.x >> 1;      // ranges
  const int half = blockIdx.x & 1;
  const int range = blockIdx.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(kv_full + s, 1);
      mbar_init(kv_empty + s, 1);
    }
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int j = 0; j < kSBuf; ++j) mbar_init(s_full + j, 1);
    for (int j = 0; j < kPBuf; ++j) {
      mbar_init(p_full + j, 128);
      mbar_init(pv_done + j, 1);
    }
    mbar_init(o_full, 1);
    mbar_init(o_empty, 128);
    fence_barrier_init();
  }
  if (warp == 5) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(
                     smem_u32(tmem_slot))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (warp == 4 && lane == 0) {
    prefetch_tmap(&tmap_q);
    prefetch_tmap(&tmap_kv);
  }
  // Row table (chunks of kT tokens per sequence); reuses the GQA scan.
  {
    GqaParams gp{};
    gp.seqlens = p.seqlens;
    gp.HG = 1;
    gp.T = kT;
    gp.P = p.P;
    gp.max_pages = p.max_pages;
    build_row_start(gp, R, row_start, warp_tmp);  // ends with __syncthreads
  }
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (blockIdx.x == 0) {
    for (int i = threadIdx.x; i <= R; i += blockDim.x) p.row_start_g[i] = row_start[i];
  }
  const int64_t W = row_start[R];
  const int G = W < (int64_t)NR ? (int)W : NR;
  const bool active = W > 0 && range < G;
  const int x0 = active ? (int)((int64_t)range * W / G) : 0;
  const int x1 = active ? (int)((int64_t)(range + 1) * W / G) : 0;
  const int cap = p.max_pages * p.P;

  if (warp == 4) {
    // ---------------- TMA producer ----------------
    if (lane == 0 && active) {
      const uint64_t policy = kv_policy();
      int row = find_row(row_start, R, x0);
      int cur = -1, nq = 0, s = 0;
      uint32_t ph = 0;
      for (int x = x0; x < x1; ++x) {
        while (x >= row_start[row + 1]) ++row;
        if (row != cur) {
          cur = row;
          if (!mla_wait(q_empty, (nq & 1) ^ 1u, p.status)) break;
          mbar_arrive_expect_tx(q_full, kQBytes);
          tma_load_5d(smem + kOffQ, &tmap_q, q_full, kHeads * half, 0, row, 0, 0);
          ++nq;
        }
        const int tok0 = (x - row_start[row]) * kT;
        const int pidx = tok0 / p.P;
        int pg = __ldg(p.block_table + (int64_t)row * p.bt_stride + pidx);
        if (pg < 0 || pg >= p.num_pages) {
          record_status(p.status, kStatusBounds);
          pg = 0;
        }
        // Warm L2 for the chunks after the ones the stage ring can hold, so
        // their loads (and the head-pair partner's) come from L2.
#pragma unroll
        for (int d = kStages; d < kStages + kL2Ahead; ++d) {
          const int xa = x + d;
          if (xa >= x1) break;
          int ra = row;
          while (xa >= row_start[ra + 1]) ++ra;
          const int ta = (xa - row_start[ra]) * kT;
          const int pa = ta / p.P;
          const int pga = __ldg(p.block_table + (int64_t)ra * p.bt_stride + pa);
          if (pga >= 0 && pga < p.num_pages) tma_prefetch_5d(&tmap_kv, ta - pa * p.P, 0, pga, 0);
        }
        if (!mla_wait(kv_empty + s, ph ^ 1u, p.status)) break;
        mbar_arrive_expect_tx(kv_full + s, kStageBytes);
        tma_load_5d(smem + kOffKV + s * kStageBytes, &tmap_kv, kv_full + s, tok0 - pidx * p.P, 0,
                    pg, 0, policy);
        if (++s == kStages) {
          s = 0;
          ph ^= 1u;
        }
      }
    }
  } else if (warp == 5) {
    // ---------------- MMA issuer ----------------
    if (active) {
      const uint32_t idesc_qk = umma_idesc_bf16(64, kT, false);
      const uint32_t idesc_pv = umma_idesc_bf16(64, 256, true);
      const uint32_t t_o = tmem;                          // O: cols 0..255, both lane halves
      const uint32_t t_s = tmem + 256u;                   // S: lane half 0, cols 256..319
      int row = find_row(row_start, R, x0);
      int cur = -1, nq = 0, nrow = 0, s = 0;
      uint32_t ph = 0;
      bool ok = true;
      auto issue_pv = [&](int j, int stage, bool first_of_row) -> bool {
        if (!mla_wait(p_full + j % kPBuf, (uint32_t)((j / kPBuf) & 1), p.status)) return false;
        if (first_of_row && nrow > 1) {
          if (!mla_wait(o_empty, (uint32_t)((nrow - 2) & 1), p.status)) return false;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t pa = sbase + kOffP + (uint32_t)((j % kPBuf) * kPBytes);
          const uint32_t vb = sbase + kOffKV + stage * kStageBytes;
          const uint64_t pd0 = umma_desc_sw128(pa, 16, 1024);
          const uint64_t vd0 = umma_desc_sw128(vb, kT * 128, 1024);
#pragma unroll
          for (int ks = 0; ks < kT / 16; ++ks) {
            const uint64_t ad = pd0 + (uint64_t)((ks * 32) >> 4);
#pragma unroll
            for (int hv = 0; hv < 2; ++hv) {
              const uint64_t bd = vd0 + (uint64_t)((hv * 4 * (kT * 128) + ks * 16 * 128) >> 4);
              umma_bf16(t_o + ((uint32_t)hv << 20), ad, bd, idesc_pv, !(first_of_row && ks == 0));
            }
          }
          umma_commit(kv_empty + stage);
          umma_commit(pv_done + j % kPBuf);
        }
        __syncwarp();
        return true;
      };
      // Chunks whose QK is issued but whose P.V is not (a short FIFO): QK runs
      // kAhead chunks ahead so the tensor pipe has work while the softmax
      // warps turn S(i) into P(i).
      int pend_i[kAhead + 1], pend_s[kAhead + 1];
      bool pend_f[kAhead + 1];
      int np = 0;
      auto pop_pv = [&]() -> bool {
        const bool r = issue_pv(pend_i[0], pend_s[0], pend_f[0]);
        for (int k = 1; k < np; ++k) {
          pend_i[k - 1] = pend_i[k];
          pend_s[k - 1] = pend_s[k];
          pend_f[k - 1] = pend_f[k];
        }
        --np;
        return r;
      };
      auto drain_row = [&]() -> bool {
        while (np > 0)
          if (!pop_pv()) return false;
        if (lane == 0) {
          umma_commit(o_full);
          umma_commit(q_empty);
        }
        __syncwarp();
        return true;
      };
      int i = 0;
      for (int x = x0; x < x1 && ok; ++x, ++i) {
        while (x >= row_start[row + 1]) ++row;
        const bool first = row != cur;
        if (first) {
          if (cur >= 0 && !(ok = drain_row())) break;
          cur = row;
          ++nrow;
          if (!mla_wait(q_full, (uint32_t)(nq & 1), p.status)) { ok = false; break; }
          ++nq;
        }
        if (!mla_wait(kv_full + s, ph, p.status)) { ok = false; break; }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t kb = sbase + kOffKV + s * kStageBytes;
          const uint32_t qb = sbase + kOffQ;
          const uint32_t ts = t_s + (uint32_t)((i % kSBuf) * kSplit * kT);
          // Descriptors differ from the tile bases only in the start-address
          // field (16-byte units), so each k-step adds a constant.
          const uint64_t ad0 = umma_desc_sw128(qb, 16, 1024);
          const uint64_t bd0 = umma_desc_sw128(kb, 16, 1024);
#pragma unroll
          for (int kk = 0; kk < kDqk / 16; ++kk) {
            const int cb = kk >> 2, ko = (kk & 3) * 32;
            const uint64_t ad = ad0 + (uint64_t)((cb * (kHeads * 128) + ko) >> 4);
            const uint64_t bd = bd0 + (uint64_t)((cb * (kT * 128) + ko) >> 4);
            umma_bf16(ts + (uint32_t)((kk % kSplit) * kT), ad, bd, idesc_qk, kk >= kSplit);
          }
          umma_commit(s_full + i % kSBuf);
        }
        __syncwarp();
        pend_i[np] = i;
        pend_s[np] = s;
        pend_f[np] = first;
        ++np;
        while (np > kAhead && ok) ok = pop_pv();
        if (++s == kStages) {
          s = 0;
          ph ^= 1u;
        }
      }
      if (ok && cur >= 0) drain_row();
    }
  } else {
    // ---------------- softmax + epilogue (warps 0-3) ----------------
    if (active) {
      const int hr = 16 * warp + (lane & 15);         // head row within this CTA
      const bool s_lane = lane < 16;                  // holds the S row and O dims 0-255
      const uint32_t t_warp = tmem + ((uint32_t)(32 * warp) << 16);
      constexpr float kLn2 = 0.69314718055994530942f;
      int row = find_row(row_start, R, x0);
      int cur = -1, nrow = 0, L = 0;
      float m = -INFINITY, l = 0.f;
      bool ok = true;
      int i = 0;
      for (int x = x0; x < x1 && ok; ++x, ++i) {
        while (x >= row_start[row + 1]) ++row;
        if (row != cur) {
          cur = row;
          ++nrow;
          const int Lb = __ldg(p.seqlens + row);
          L = Lb < 0 ? 0 : (Lb > cap ? cap : Lb);
          m = -INFINITY;
          l = 0.f;
        }
        const bool first_chunk = (x == row_start[row]) || (x == x0);
        const bool last = (x + 1 == x1) || (x + 1 >= row_start[row + 1]);
        const int tok0 = (x - row_start[row]) * kT;
        const int nvalid = min(kT, L - tok0);
        const int stage = i % kStages;

        if (!mla_wait(s_full + i % kSBuf, (uint32_t)((i / kSBuf) & 1), p.status)) { ok = false; break; }
        tc_fence_after();
        float sv[kT];
#pragma unroll
        for (int c = 0; c < kT; c += 32)
          tmem_ld32(t_warp + 256u + (uint32_t)((i % kSBuf) * kSplit * kT + c), sv + c);
#pragma unroll
        for (int part = 1; part < kSplit; ++part) {
          float sp[kT];
          tmem_ld32(t_warp + 256u + (uint32_t)(((i % kSBuf) * kSplit + part) * kT), sp);
#pragma unroll
          for (int t = 0; t < kT; ++t) sv[t] += sp[t];
        }
        // Lanes >= 16 read unused columns of lane half 1 here; lanes < 16 hold the S row.
        float cm = -INFINITY;
#pragma unroll
        for (int t = 0; t < kT; ++t) {
          sv[t] = (t < nvalid) ? sv[t] * p.scale_log2 : -INFINITY;
          cm = fmaxf(cm, sv[t]);
        }
        const bool need = s_lane && (m == -INFINITY || cm > m + kLazy);
        const bool any_need = softmax_group_any(need);
        float alpha = 1.f;
        if (need) {
          const float mn = (m == -INFINITY) ? cm : fmaxf(m, cm);
          alpha = (m == -INFINITY) ? 0.f : fast_exp2(m - mn);
          m = mn;
          l *= alpha;
        }
        // both O threads of this head use the S-row thread's factor
        const float alpha_o = __shfl_sync(0xffffffffu, alpha, lane & 15);
        if (any_need && !first_chunk) {
          // O must be complete up to the previous chunk before it is rescaled.
          if (!mla_wait(pv_done + (i - 1) % kPBuf, (uint32_t)(((i - 1) / kPBuf) & 1), p.status)) { ok = false; break; }
          tc_fence_after();
          for (int c = 0; c < kDv / 2; c += 32) {
            float ov[32];
            tmem_ld32(t_warp + (uint32_t)c, ov);
#pragma unroll
            for (int e = 0; e < 32; ++e) ov[e] *= alpha_o;
            tmem_st32(t_warp + (uint32_t)c, ov);
          }
          tc_fence_before();
        }
        // P(i - kPBuf) must be consumed before its TMEM buffer is rewritten.
        if (i >= kPBuf) {
          if (!mla_wait(pv_done + i % kPBuf, (uint32_t)(((i - kPBuf) / kPBuf) & 1), p.status)) { ok = false; break; }
        }
        if (s_lane) {
          // P row (bf16) into the swizzled K-major P tile: row hr is 128-byte
          // line hr, its 16-byte chunk c (8 tokens) sits at c ^ (hr & 7).
          uint8_t* pbuf = smem + kOffP + (i % kPBuf) * kPBytes;
          float psum = 0.f;
          uint32_t pk[kT / 2];
#pragma unroll
          for (int t = 0; t < kT; t += 2) {
            const float p0 = fast_exp2(sv[t] - m), p1 = fast_exp2(sv[t + 1] - m);
            psum += p0 + p1;
            pk[t / 2] = pack2<true>(p0, p1);
          }
          l += psum;
#pragma unroll
          for (int c = 0; c < kT / 8; ++c) {
            const uint32_t a = smem_u32(pbuf) + hr * 128 + (((c ^ (hr & 7)) & 7) << 4);
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(pk[4 * c]),
                         "r"(pk[4 * c + 1]), "r"(pk[4 * c + 2]), "r"(pk[4 * c + 3])
                         : "memory");
          }
        }
        if (nvalid < kT) {
          // Slots past the sequence end may hold anything, even NaN: zero those
          // V rows of the stage (first 8 column blocks) before P.V reads them.
          const uint32_t vb = sbase + kOffKV + stage * kStageBytes;
          const int nrows = kT - nvalid;
          for (int idx = threadIdx.x; idx < 8 * nrows * 8; idx += 128) {
            const int chunk = idx & 7, rest = idx >> 3;
            const int cb = rest / nrows, tk = nvalid + rest % nrows;
            const uint32_t a = vb + cb * (kT * 128) + tk * 128 + chunk * 16;
            asm volatile("st.shared.v4.b32 [%0], {%1, %1, %1, %1};" ::"r"(a), "r"(0) : "memory");
          }
        }
        fence_async_smem();
        tc_fence_before();
        mbar_arrive(p_full + i % kPBuf);

        if (last) {
          if (!mla_wait(o_full, (uint32_t)((nrow - 1) & 1), p.status)) { ok = false; break; }
          tc_fence_after();
          const float l_o = __shfl_sync(0xffffffffu, l, lane & 15);
          const float m_o = __shfl_sync(0xffffffffu, m, lane & 15);
          const int cf = cta_of_chunk(row_start[row], W, G);
          const int cl = cta_of_chunk(row_start[row + 1] - 1, W, G);
          const int head = kHeads * half + hr;
          const float inv = 1.f / l_o;
          const int dv0 = s_lane ? 0 : kDv / 2;   // this thread's half of the head dims
          for (int c = 0; c < kDv / 2; c += 32) {
            float ov[32];
            tmem_ld32(t_warp + (uint32_t)c, ov);
            {
              if (cf == cl) {
                __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.out) +
                                     (int64_t)row * p.o_sb + (int64_t)head * p.o_sh + dv0 + c;
#pragma unroll
                for (int e = 0; e < 32; e += 8) {
                  uint4 w;
                  w.x = pack2<true>(ov[e] * inv, ov[e + 1] * inv);
                  w.y = pack2<true>(ov[e + 2] * inv, ov[e + 3] * inv);
                  w.z = pack2<true>(ov[e + 4] * inv, ov[e + 5] * inv);
                  w.w = pack2<true>(ov[e + 6] * inv, ov[e + 7] * inv);
                  *reinterpret_cast<uint4*>(dst + e) = w;
                }
              } else {
                const int64_t seg = (int64_t)row + range;
                float* dst = p.part_o + (seg * 128 + head) * kDv + dv0 + c;
#pragma unroll
                for (int e = 0; e < 32; e += 4)
                  *reinterpret_cast<float4*>(dst + e) =
                      make_float4(ov[e] * inv, ov[e + 1] * inv, ov[e + 2] * inv, ov[e + 3] * inv);
              }
            }
          }
          if (s_lane) {
            const float lse2 = m_o + fast_log2(l_o);
            if (cf == cl) {
              if (p.lse) p.lse[(int64_t)row * p.lse_sb + head] = lse2 * kLn2;
            } else {
              p.part_lse[((int64_t)row + range) * 128 + head] = lse2;
            }
          }
          tc_fence_before();
          mbar_arrive(o_empty);
        }
      }
    }
  }
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
  }
}

}  // namespace b2d
