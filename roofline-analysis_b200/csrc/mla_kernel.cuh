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
// Tensor memory (512 columns x 128 lanes).  An M=64 UMMA uses 16 lanes of
// each 32-lane quadrant: lane half 0 (lanes 0-15, 32-47, ...) or lane half 1
// (16-31, ...).  Half 0 holds the two score tiles S [64 heads x 64 tokens]
// (columns 0-127) and the query Q [64 heads x 576] as packed bf16 pairs
// (columns 128-415): S = Q.K^T reads Q straight from tensor memory (an
// A-from-TMEM MMA, whose A must sit in the accumulator's lane half), so Q is
// not re-read from shared memory for every chunk.  Half 1 holds the output
// accumulator O [64 heads x 512] fp32 (columns 0-511).  All tensor-memory
// traffic of the softmax warps uses the 16-lane 16x256b shape, which touches
// one lane half only: thread t of warp w serves heads 16w + t/4 and
// 16w + t/4 + 8, columns 2 (t % 4) + {0, 1} of every group of 8 (16 scores
// per head per chunk; the 4 threads of a head combine max and sum with two
// shuffles).
//
// Shared memory: three KV stages [9 x 64 tok x 64] bf16 by TMA with 128-byte
// swizzle (K-major canonical UMMA layout: 8-row x 128-byte atoms, 1024-byte
// stride), and P [64 heads x 64 tok] bf16 in the same layout.  The same KV
// stage is the K-major B operand of S = Q.K^T and the MN-major B operand of
// O += P.V (V = its first 8 column blocks), so each latent row is fetched
// once.
//
// Warp roles: warps 0-3 softmax + epilogue (and the Q writes), warp 4 TMA
// producer, warp 5 TMEM allocator + single-thread MMA issuer.  Online softmax
// uses a lazy rescale: the running max moves only when a score exceeds it by
// 8 (log2 units), so P <= 256 fits bf16 and O is rescaled (TMEM round trip)
// rarely.
#pragma once

#include "gqa_kernel.cuh"
#include "gqa_mma_kernel.cuh"

namespace b2d {

struct MlaParams {
  const void* q;             // bf16 [B, 128, 576] (strides in elements)
  int64_t q_sb, q_sh;
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
  unsigned long long wait_ns;  // bounded-wait limit of every mbarrier wait
  int B, P, num_pages, max_pages;
  float scale_log2;
};

namespace mla {
constexpr int kHeads = 64;         // query heads per CTA
constexpr int kDqk = 576, kDv = 512;
constexpr int kCB = kDqk / 64;     // 128-byte column blocks per row (9)
constexpr int kT = 64;             // tokens per chunk (one TMA box; page size % 64 == 0)
constexpr int kStages = 3;
constexpr uint32_t kStageBytes = kCB * kT * 128;     // 73728
constexpr int kSBuf = 2;           // score tiles in TMEM (lane half 0, columns 64k)
constexpr uint32_t kPBytes = kHeads * 128;           // 8192
constexpr uint32_t kColQ = kSBuf * kT;               // Q: lane half 0, columns 128-415
constexpr uint32_t kHalf1 = 16u << 16;               // TMEM lane offset of lane half 1 (O)
constexpr float kLazy = 8.f;                         // lazy-rescale threshold, log2 units
#ifndef B2D_MLA_L2_AHEAD
#define B2D_MLA_L2_AHEAD 2
#endif
constexpr int kL2Ahead = B2D_MLA_L2_AHEAD;           // chunks prefetched into L2 past the ring
constexpr int kThreads = 6 * 32;
// shared-memory map (offsets from the 1024-aligned base)
constexpr uint32_t kOffKV = 0;
constexpr uint32_t kOffP = kOffKV + kStages * kStageBytes;
constexpr uint32_t kOffBar = kOffP + kPBytes;
// kv full/empty, q full, s full, p full, pv done, o full/empty
constexpr uint32_t kNumBars = 2 * kStages + 1 + kSBuf + 2 + 2;
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

// Wait helper that records a timeout; returns false when the kernel must stop.
__device__ __forceinline__ bool mla_wait(uint64_t* bar, uint32_t parity, int* status,
                                         unsigned long long limit_ns) {
  if (mbar_wait(bar, parity, limit_ns)) return true;
  record_status(status, kStatusTimeout);
  return false;
}


// A-from-TMEM MMA: D (TMEM) (+)= A (TMEM, K-major, packed 16-bit pairs) .
// B (shared-memory descriptor).
__device__ __forceinline__ void umma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                             uint32_t idesc, bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}"
      ::"r"(d_tmem), "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"((uint32_t)accumulate), "r"(0u),
      "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}

// 16-lane tensor-memory access, 8 column groups of 8 columns (16x256b.x8):
// register 4j + e of thread t is lane (t / 4) + 8 (e >> 1), column
// 8j + 2 (t % 4) + (e & 1), counted from the address's lane and column.
__device__ __forceinline__ void tmem_ld16x8(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.16x256b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, "
      "%29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_st16x8(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.16x256b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, "
      "%29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 16-lane store of 4 column groups (16x256b.x4), same register mapping.
__device__ __forceinline__ void tmem_st16x4(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.16x256b.x4.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}

__global__ void __launch_bounds__(mla::kThreads, 1)
    mla_decode_kernel(const __grid_constant__ CUtensorMap tmap_kv, const MlaParams p) {
  using namespace mla;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const uint32_t sbase = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* kv_full = bars;
  uint64_t* kv_empty = bars + kStages;
  uint64_t* q_full = bars + 2 * kStages;   // Q of the next sequence written to TMEM
  uint64_t* s_full = q_full + 1;          // [kSBuf]
  uint64_t* p_full = s_full + kSBuf;
  uint64_t* pv_done = p_full + 1;
  uint64_t* o_full = pv_done + 1;
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
    mbar_init(q_full, 128);
    for (int j = 0; j < kSBuf; ++j) mbar_init(s_full + j, 1);
    mbar_init(p_full, 128);
    mbar_init(pv_done, 1);
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
  if (warp == 4 && lane == 0) prefetch_tmap(&tmap_kv);
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
    // ---------------- TMA producer (KV stages only) ----------------
    if (lane == 0 && active) {
      const uint64_t policy = kv_policy();
      int row = find_row(row_start, R, x0);
      int s = 0;
      uint32_t ph = 0;
      for (int x = x0; x < x1; ++x) {
        while (x >= row_start[row + 1]) ++row;
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
        if (!mla_wait(kv_empty + s, ph ^ 1u, p.status, p.wait_ns)) break;
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
      const uint32_t t_o = tmem + kHalf1;                 // O: lane half 1, columns 0..511
      const uint32_t t_q = tmem + kColQ;                  // Q: lane half 0, columns 128..415
      int row = find_row(row_start, R, x0);
      int cur = -1, nq = 0, nrow = 0, s = 0;
      uint32_t ph = 0;
      bool ok = true;
      auto issue_pv = [&](int j, int stage, bool first_of_row) -> bool {
        if (!mla_wait(p_full, (uint32_t)(j & 1), p.status, p.wait_ns)) return false;
        if (first_of_row && nrow > 1) {
          if (!mla_wait(o_empty, (uint32_t)((nrow - 2) & 1), p.status, p.wait_ns)) return false;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint64_t pd0 = umma_desc_sw128(sbase + kOffP, 16, 1024);
          const uint64_t vd0 = umma_desc_sw128(sbase + kOffKV + stage * kStageBytes, kT * 128, 1024);
#pragma unroll
          for (int ks = 0; ks < kT / 16; ++ks) {
            const uint64_t ad = pd0 + (uint64_t)((ks * 32) >> 4);
#pragma unroll
            for (int hv = 0; hv < 2; ++hv) {
              const uint64_t bd = vd0 + (uint64_t)((hv * 4 * (kT * 128) + ks * 16 * 128) >> 4);
              umma_bf16(t_o + (uint32_t)(hv * 256), ad, bd, idesc_pv, !(first_of_row && ks == 0));
            }
          }
          umma_commit(kv_empty + stage);
          umma_commit(pv_done);
        }
        __syncwarp();
        return true;
      };
      // QK of chunk i is issued before P.V of chunk i - 1, so the tensor pipe
      // has work while the softmax warps turn S(i - 1) into P(i - 1).
      int pend_i = -1, pend_s = 0;
      bool pend_f = false;
      auto drain_row = [&]() -> bool {
        if (pend_i >= 0 && !issue_pv(pend_i, pend_s, pend_f)) return false;
        pend_i = -1;
        if (lane == 0) umma_commit(o_full);
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
          if (!mla_wait(q_full, (uint32_t)(nq & 1), p.status, p.wait_ns)) { ok = false; break; }
          ++nq;
        }
        if (!mla_wait(kv_full + s, ph, p.status, p.wait_ns)) { ok = false; break; }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t ts = tmem + (uint32_t)((i % kSBuf) * kT);
          // The K descriptor differs from the tile base only in its start
          // address (16-byte units); Q's k-step is 8 TMEM columns (16 bf16).
          const uint64_t bd0 = umma_desc_sw128(sbase + kOffKV + s * kStageBytes, 16, 1024);
#pragma unroll
          for (int kk = 0; kk < kDqk / 16; ++kk) {
            const int cb = kk >> 2, ko = (kk & 3) * 32;
            const uint64_t bd = bd0 + (uint64_t)((cb * (kT * 128) + ko) >> 4);
            umma_bf16_ts(ts, t_q + (uint32_t)(kk * 8), bd, idesc_qk, kk > 0);
          }
          umma_commit(s_full + i % kSBuf);
        }
        __syncwarp();
        if (pend_i >= 0 && !(ok = issue_pv(pend_i, pend_s, pend_f))) break;
        pend_i = i;
        pend_s = s;
        pend_f = first;
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
      const uint32_t t_warp = tmem + ((uint32_t)(32 * warp) << 16);
      // 16-lane O / Q accesses: this thread's two heads (lanes t/4, t/4 + 8 of
      // the warp's lane half) and columns 2 (t % 4) + {0, 1} of every group of 8.
      const int h_a = 16 * warp + (lane >> 2), h_b = h_a + 8;
      const int cq = 2 * (lane & 3);
      constexpr float kLn2 = 0.69314718055994530942f;
      // Q of a sequence into TMEM (lane half 0, columns 128..415, bf16 pairs
      // with the lower dim in the low half), then release it to the MMA warp.
      auto write_q = [&](int qrow) {
        const __nv_bfloat16* qb = reinterpret_cast<const __nv_bfloat16*>(p.q) +
                                  (int64_t)qrow * p.q_sb;
        const __nv_bfloat16* qa = qb + (int64_t)(kHeads * half + h_a) * p.q_sh;
        const __nv_bfloat16* qc = qb + (int64_t)(kHeads * half + h_b) * p.q_sh;
#pragma unroll 1
        for (int g0 = 0; g0 < kDqk / 16; g0 += 4) {   // 4 groups of 16 dims per store
          uint32_t r[16];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int d = 16 * (g0 + j) + 2 * cq;
            const uint2 va = *reinterpret_cast<const uint2*>(qa + d);
            const uint2 vc = *reinterpret_cast<const uint2*>(qc + d);
            r[4 * j + 0] = va.x;
            r[4 * j + 1] = va.y;
            r[4 * j + 2] = vc.x;
            r[4 * j + 3] = vc.y;
          }
          tmem_st16x4(t_warp + kColQ + (uint32_t)(8 * g0), r);
        }
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        tc_fence_before();
        mbar_arrive(q_full);
      };
      int row = find_row(row_start, R, x0);
      write_q(row);
      int cur = -1, nrow = 0, L = 0;
      // running max (log2 units) and partial sum of this thread's two heads;
      // the 4 threads of a head hold the same max and disjoint partial sums
      float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;
      bool ok = true;
      int i = 0;
      for (int x = x0; x < x1 && ok; ++x, ++i) {
        while (x >= row_start[row + 1]) ++row;
        if (row != cur) {
          cur = row;
          ++nrow;
          const int Lb = __ldg(p.seqlens + row);
          L = Lb < 0 ? 0 : (Lb > cap ? cap : Lb);
          m_a = m_b = -INFINITY;
          l_a = l_b = 0.f;
        }
        const bool first_chunk = (x == row_start[row]) || (x == x0);
        const bool last = (x + 1 == x1) || (x + 1 >= row_start[row + 1]);
        const int tok0 = (x - row_start[row]) * kT;
        const int nvalid = min(kT, L - tok0);
        const int stage = i % kStages;

        if (!mla_wait(s_full + i % kSBuf, (uint32_t)((i / kSBuf) & 1), p.status, p.wait_ns)) { ok = false; break; }
        tc_fence_after();
        // Scores of heads a and b, tokens 8j + cq + {0, 1} (j = 0..7).
        float sa[16], sb[16];
        {
          uint32_t r[32];
          tmem_ld16x8(t_warp + (uint32_t)((i % kSBuf) * kT), r);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const bool valid = 8 * j + cq + e < nvalid;
              sa[2 * j + e] = valid ? __uint_as_float(r[4 * j + e]) * p.scale_log2 : -INFINITY;
              sb[2 * j + e] = valid ? __uint_as_float(r[4 * j + 2 + e]) * p.scale_log2 : -INFINITY;
            }
          }
        }
        float cm_a = -INFINITY, cm_b = -INFINITY;
#pragma unroll
        for (int t = 0; t < 16; ++t) {
          cm_a = fmaxf(cm_a, sa[t]);
          cm_b = fmaxf(cm_b, sb[t]);
        }
#pragma unroll
        for (int o = 1; o <= 2; o <<= 1) {
          cm_a = fmaxf(cm_a, __shfl_xor_sync(0xffffffffu, cm_a, o));
          cm_b = fmaxf(cm_b, __shfl_xor_sync(0xffffffffu, cm_b, o));
        }
        const bool need_a = m_a == -INFINITY || cm_a > m_a + kLazy;
        const bool need_b = m_b == -INFINITY || cm_b > m_b + kLazy;
        const bool any_need = softmax_group_any(need_a || need_b);
        float al_a = 1.f, al_b = 1.f;
        if (need_a) {
          const float mn = (m_a == -INFINITY) ? cm_a : fmaxf(m_a, cm_a);
          al_a = (m_a == -INFINITY) ? 0.f : fast_exp2(m_a - mn);
          m_a = mn;
          l_a *= al_a;
        }
        if (need_b) {
          const float mn = (m_b == -INFINITY) ? cm_b : fmaxf(m_b, cm_b);
          al_b = (m_b == -INFINITY) ? 0.f : fast_exp2(m_b - mn);
          m_b = mn;
          l_b *= al_b;
        }
        // P.V of the previous chunk must be complete before O is rescaled or
        // the P tile is rewritten.
        if (i > 0) {
          if (!mla_wait(pv_done, (uint32_t)((i - 1) & 1), p.status, p.wait_ns)) { ok = false; break; }
          tc_fence_after();
        }
        if (any_need && !first_chunk) {
          for (int c = 0; c < kDv; c += 64) {
            uint32_t r[32];
            tmem_ld16x8(t_warp + kHalf1 + (uint32_t)c, r);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              r[4 * j + 0] = __float_as_uint(__uint_as_float(r[4 * j + 0]) * al_a);
              r[4 * j + 1] = __float_as_uint(__uint_as_float(r[4 * j + 1]) * al_a);
              r[4 * j + 2] = __float_as_uint(__uint_as_float(r[4 * j + 2]) * al_b);
              r[4 * j + 3] = __float_as_uint(__uint_as_float(r[4 * j + 3]) * al_b);
            }
            tmem_st16x8(t_warp + kHalf1 + (uint32_t)c, r);
          }
        }
        {
          // P (bf16) into the swizzled K-major P tile: head row h is 128-byte
          // line h, tokens 8j..8j+7 are its 16-byte chunk j ^ (h & 7); this
          // thread writes tokens 8j + cq, +1 of heads a and b.
          const uint32_t pa = sbase + kOffP + (uint32_t)(h_a * 128 + 2 * cq);
          const uint32_t pb = sbase + kOffP + (uint32_t)(h_b * 128 + 2 * cq);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float a0 = fast_exp2(sa[2 * j] - m_a), a1 = fast_exp2(sa[2 * j + 1] - m_a);
            const float b0 = fast_exp2(sb[2 * j] - m_b), b1 = fast_exp2(sb[2 * j + 1] - m_b);
            l_a += a0 + a1;
            l_b += b0 + b1;
            asm volatile("st.shared.b32 [%0], %1;" ::"r"(pa + (((j ^ (h_a & 7)) & 7) << 4)),
                         "r"(pack2<true>(a0, a1))
                         : "memory");
            asm volatile("st.shared.b32 [%0], %1;" ::"r"(pb + (((j ^ (h_b & 7)) & 7) << 4)),
                         "r"(pack2<true>(b0, b1))
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
        mbar_arrive(p_full);

        if (last) {
          // S of this row's last chunk has been read, so its QK MMAs are done
          // and the Q columns are free: stage the next sequence's Q now.
          if (x + 1 < x1) write_q(row + 1);
          float lt_a = l_a, lt_b = l_b;
#pragma unroll
          for (int o = 1; o <= 2; o <<= 1) {
            lt_a += __shfl_xor_sync(0xffffffffu, lt_a, o);
            lt_b += __shfl_xor_sync(0xffffffffu, lt_b, o);
          }
          if (!mla_wait(o_full, (uint32_t)((nrow - 1) & 1), p.status, p.wait_ns)) { ok = false; break; }
          tc_fence_after();
          const int cf = cta_of_chunk(row_start[row], W, G);
          const int cl = cta_of_chunk(row_start[row + 1] - 1, W, G);
          const float inv_a = 1.f / lt_a, inv_b = 1.f / lt_b;
          const int head_a = kHeads * half + h_a, head_b = kHeads * half + h_b;
          for (int c = 0; c < kDv; c += 64) {
            uint32_t r[32];
            tmem_ld16x8(t_warp + kHalf1 + (uint32_t)c, r);
            if (cf == cl) {
              __nv_bfloat16* da = reinterpret_cast<__nv_bfloat16*>(p.out) +
                                  (int64_t)row * p.o_sb + (int64_t)head_a * p.o_sh + c + cq;
              __nv_bfloat16* db = reinterpret_cast<__nv_bfloat16*>(p.out) +
                                  (int64_t)row * p.o_sb + (int64_t)head_b * p.o_sh + c + cq;
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                *reinterpret_cast<uint32_t*>(da + 8 * j) =
                    pack2<true>(__uint_as_float(r[4 * j]) * inv_a, __uint_as_float(r[4 * j + 1]) * inv_a);
                *reinterpret_cast<uint32_t*>(db + 8 * j) =
                    pack2<true>(__uint_as_float(r[4 * j + 2]) * inv_b, __uint_as_float(r[4 * j + 3]) * inv_b);
              }
            } else {
              const int64_t seg = (int64_t)row + range;
              float* da = p.part_o + (seg * 128 + head_a) * kDv + c + cq;
              float* db = p.part_o + (seg * 128 + head_b) * kDv + c + cq;
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                *reinterpret_cast<float2*>(da + 8 * j) =
                    make_float2(__uint_as_float(r[4 * j]) * inv_a, __uint_as_float(r[4 * j + 1]) * inv_a);
                *reinterpret_cast<float2*>(db + 8 * j) =
                    make_float2(__uint_as_float(r[4 * j + 2]) * inv_b, __uint_as_float(r[4 * j + 3]) * inv_b);
              }
            }
          }
          if ((lane & 3) == 0) {
            const float lse_a = m_a + fast_log2(lt_a), lse_b = m_b + fast_log2(lt_b);
            if (cf == cl) {
              if (p.lse) {
                p.lse[(int64_t)row * p.lse_sb + head_a] = lse_a * kLn2;
                p.lse[(int64_t)row * p.lse_sb + head_b] = lse_b * kLn2;
              }
            } else {
              p.part_lse[((int64_t)row + range) * 128 + head_a] = lse_a;
              p.part_lse[((int64_t)row + range) * 128 + head_b] = lse_b;
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
