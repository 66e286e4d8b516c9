// gqa_host.cu — host side of the GQA decode: argument validation, the split
// plan, TMA descriptor encoding, workspace layout and the two launches.
// Exposed through the C ABI in include/b2d_decode.h.
#include <stdlib.h>

#include "b2d_decode.h"
#include "gqa_kernel.cuh"
#include "gqa_mma_kernel.cuh"
#include "host_common.h"

namespace b2d {

// Rows (sequence x KV-head group) handled by one launch; larger batches are
// cut into slices of whole sequences that reuse the same workspace in order.
constexpr int kMaxRowsPerLaunch = 2048;
// Default shared-memory budget for the K/V stage ring of one CTA.
constexpr size_t kStageRingBytes = 96 * 1024;
// Most resident CTAs per SM (and the wave the workspace is sized for).  8
// lets the small tiles of one-KV-head-per-rank tensor parallelism (2 warps
// per CTA) reach ~6 CTAs per SM: 141 -> 100 us for a config-5 rank at TP 8;
// B2D_GQA_MAX_CTAS_PER_SM overrides it (1..16).
static int max_ctas_per_sm();

// Tuning knobs read once from the environment (for measurement sweeps):
// B2D_GQA_HQW caps the query heads per consumer warp (1, 2 or 4) and
// B2D_GQA_RING_KB sets the stage-ring budget per CTA.
static int env_int(const char* name, int dflt) {
  const char* v = getenv(name);
  return v ? atoi(v) : dflt;
}

static int max_ctas_per_sm() {
  static const int v = [] {
    const int e = env_int("B2D_GQA_MAX_CTAS_PER_SM", 8);
    return e < 1 ? 1 : (e > 16 ? 16 : e);
  }();
  return v;
}

struct GqaPlan;
static int plan_ctas_per_sm(const GqaPlan& pl);

struct GqaPlan {
  bool mma;  // tensor-core consumer (page size % 16 == 0) or CUDA-core consumer
  int np;    // mma: PV column tiles (1: <= 8 query heads per warp, 2: <= 16)
  int group, hqw, wph, hk, hg, nw, T, stages, ctas, rows_per_launch, seqs_per_launch;
  uint32_t stage_bytes;
  size_t smem;
  size_t off_row_start, off_part_lse, off_part_o, ws_bytes;
  int* launch_count;  // when set: count the launches a call makes, launch nothing
};

// Most CTAs of this plan that can be resident on one SM: max_ctas_per_sm(),
// bounded by the SM's shared memory (228 KB, 1 KB reserved per CTA) and
// threads (2048).  The workspace is sized for this many CTAs per SM and the
// launch never uses more, so small tiles get up to 8 CTAs per SM without
// inflating the workspace of the large ones.
static int plan_ctas_per_sm(const GqaPlan& pl) {
  const int threads = 32 * (pl.nw + 1);
  int cap = max_ctas_per_sm();
  const int by_smem = (int)(233472 / (pl.smem + 1024));
  const int by_threads = 2048 / threads;
  if (by_smem < cap) cap = by_smem;
  if (by_threads < cap) cap = by_threads;
  return cap < 1 ? 1 : cap;
}

static int kv_elem_bytes(int kv_dtype) { return kv_dtype == B2D_FP8_E4M3 ? 1 : 2; }

static int largest_divisor_leq(int n, int cap) {
  for (int d = cap < n ? cap : n; d >= 1; --d)
    if (n % d == 0) return d;
  return 1;
}

static int validate(const b2d_gqa_args* a, bool need_pointers) {
  if (a == nullptr) return B2D_ERR_INVALID_ARG;
  if (a->batch < 0 || a->num_q_heads <= 0 || a->num_kv_heads <= 0 || a->page_size <= 0 ||
      a->max_pages_per_seq <= 0)
    return B2D_ERR_INVALID_ARG;
  if (a->num_q_heads % a->num_kv_heads != 0) return B2D_ERR_INVALID_ARG;
  if (a->head_dim != 64 && a->head_dim != 128 && a->head_dim != 192 && a->head_dim != 256)
    return B2D_ERR_UNSUPPORTED;
  if (a->q_dtype != B2D_BF16 && a->q_dtype != B2D_FP16) return B2D_ERR_UNSUPPORTED;
  if (a->kv_dtype != a->q_dtype && a->kv_dtype != B2D_FP8_E4M3) return B2D_ERR_UNSUPPORTED;
  const int group = a->num_q_heads / a->num_kv_heads;
  if (group > 32) return B2D_ERR_UNSUPPORTED;
  if (a->page_size > (1 << 24)) return B2D_ERR_TOO_LARGE;
  // Token positions (max_pages_per_seq * page_size) are 32-bit in the kernels.
  if ((int64_t)a->max_pages_per_seq * a->page_size > (int64_t)INT32_MAX) return B2D_ERR_TOO_LARGE;
  if (a->wait_limit_us < 0) return B2D_ERR_INVALID_ARG;
  if (a->kv_layout != B2D_KV_STRIDED && a->kv_layout != B2D_KV_VLLM) return B2D_ERR_INVALID_ARG;
  if (a->kv_layout == B2D_KV_VLLM) {
    // K [blocks, Hkv, D/8, P, 8] and V [blocks, Hkv, D, P]: the kernel reads
    // (block, head) as one flattened index, so blocks must be dense.
    if (a->kv_dtype == B2D_FP8_E4M3 || a->page_size % 16 != 0) return B2D_ERR_UNSUPPORTED;
    if (need_pointers) {
      const int64_t blk = (int64_t)a->head_dim * a->page_size;
      if (a->k_stride_head != blk || a->v_stride_head != blk ||
          a->k_stride_page != blk * a->num_kv_heads || a->v_stride_page != blk * a->num_kv_heads)
        return B2D_ERR_INVALID_ARG;
      if (a->num_pages * a->num_kv_heads > (int64_t)INT32_MAX) return B2D_ERR_TOO_LARGE;
    }
  }
  if (!need_pointers) return B2D_OK;
  if (a->batch == 0) return B2D_OK;
  if (!a->q || !a->k_cache || !a->v_cache || !a->cache_seqlens || !a->block_table || !a->out)
    return B2D_ERR_INVALID_ARG;
  if (a->num_pages <= 0 || a->num_pages > (int64_t)INT32_MAX) return B2D_ERR_INVALID_ARG;
  const int es = kv_elem_bytes(a->kv_dtype);
  const uintptr_t al = 15;
  if (((uintptr_t)a->k_cache & al) || ((uintptr_t)a->v_cache & al) || ((uintptr_t)a->q & al) ||
      ((uintptr_t)a->out & al))
    return B2D_ERR_ALIGNMENT;
  const int64_t strides[6] = {a->k_stride_page, a->k_stride_tok, a->k_stride_head,
                              a->v_stride_page, a->v_stride_tok, a->v_stride_head};
  for (int i = 0; i < 6; ++i) {
    if (a->kv_layout == B2D_KV_VLLM && (i == 1 || i == 4)) continue;  // token strides implied
    if (strides[i] <= 0 || (strides[i] * es) % 16 != 0) return B2D_ERR_ALIGNMENT;
  }
  if ((a->q_stride_b * 2) % 16 || (a->q_stride_h * 2) % 16 || (a->out_stride_b * 2) % 16 ||
      (a->out_stride_h * 2) % 16)
    return B2D_ERR_ALIGNMENT;
  return B2D_OK;
}

static int make_plan(const b2d_gqa_args* a, GqaPlan* pl) {
  const int group = a->num_q_heads / a->num_kv_heads;
  pl->group = group;
  const int es = kv_elem_bytes(a->kv_dtype);
  static const int use_mma = env_int("B2D_GQA_MMA", 1);
  // KV heads per tile: with 16-bit caches a whole token row of up to 8 heads
  // (one contiguous 2 KB run per token at D = 128) streams best; fp8 tiles
  // are half as wide and do better with more, smaller rows in flight.
  static const int hk_cap_env = env_int("B2D_GQA_HKMAX", 0);
  const int hk_cap = hk_cap_env > 0 ? hk_cap_env : (a->kv_dtype == B2D_FP8_E4M3 ? 4 : 8);
  // fp8 tiles use whole 128-byte lines per head row, so head_dim >= 128.
  pl->mma = use_mma && (a->page_size % 16 == 0) &&
            !(a->kv_dtype == B2D_FP8_E4M3 && a->head_dim < 128);
  // head_dim 192 is built for the tensor-core path with 16-bit caches only
  // (fp8 tiles need whole 128-byte lines per head row: head_dim % 128 == 0).
  if (a->head_dim == 192 && (!pl->mma || a->kv_dtype == B2D_FP8_E4M3)) return B2D_ERR_UNSUPPORTED;
  if (a->kv_layout == B2D_KV_VLLM && !pl->mma) return B2D_ERR_UNSUPPORTED;
  if (pl->mma) {
    // Tensor-core consumer: a warp takes GW <= 16 query heads (<= 8 at
    // head_dim 192 and 256, to bound the accumulator registers) of one KV head; a
    // chunk is 16 tokens of HK KV heads.
    const int gw_cap = a->head_dim >= 192 ? 8 : 16;
    int wph = 1;
    while (group % wph != 0 || group / wph > gw_cap) ++wph;
    pl->wph = wph;
    pl->np = (group / wph) > 8 ? 2 : 1;
    pl->hqw = group / wph;
    if (wph > 8) return B2D_ERR_UNSUPPORTED;
    int cap_hk = 8 / wph < hk_cap ? 8 / wph : hk_cap;
    if (cap_hk < 1) cap_hk = 1;
    pl->hk = largest_divisor_leq(a->num_kv_heads, cap_hk);
    pl->T = 16;
    // Small problems (few sequences, short caches): narrower tiles give more
    // chunks, so every CTA still gets about two.  The chunk count is bounded
    // by the block table's width; the lengths themselves live on the device.
    if (hk_cap_env <= 0) {
      int sms = 148;
      device_sm_count(&sms);
      const int64_t toks = (int64_t)a->max_pages_per_seq * a->page_size;
      const int64_t per_head_row = (int64_t)a->batch * ((toks + 15) / 16);
      while (pl->hk > 1 && per_head_row * (a->num_kv_heads / pl->hk) < 4LL * sms)
        pl->hk = largest_divisor_leq(a->num_kv_heads, pl->hk / 2);
    }
  } else {
    static const int hqw_cap = env_int("B2D_GQA_HQW", 2);
    pl->np = 0;
    pl->hqw = (group % 4 == 0 && hqw_cap >= 4) ? 4 : (group % 2 == 0 && hqw_cap >= 2 ? 2 : 1);
    pl->wph = group / pl->hqw;
    if (pl->wph > 8) return B2D_ERR_UNSUPPORTED;
    pl->hk = largest_divisor_leq(a->num_kv_heads, 8 / pl->wph);
  }
  pl->hg = a->num_kv_heads / pl->hk;
  pl->nw = pl->hk * pl->wph;
  const int row_bytes = pl->hk * a->head_dim * es;
  if (!pl->mma) {
    // Chunk: the largest divisor of the page size that keeps one K tile at
    // <= 16 KB and the TMA box at <= 256 rows.
    int tmax = 16384 / row_bytes;
    if (tmax < 1) tmax = 1;
    if (tmax > 256) tmax = 256;
    pl->T = largest_divisor_leq(a->page_size, tmax);
  }
  pl->stage_bytes = (uint32_t)(pl->T * row_bytes);
  static const size_t ring = (size_t)env_int("B2D_GQA_RING_KB", (int)(kStageRingBytes / 1024)) * 1024;
  int stages = (int)(ring / (2 * (size_t)pl->stage_bytes));
  pl->stages = stages < 2 ? 2 : (stages > 8 ? 8 : stages);
  pl->seqs_per_launch = kMaxRowsPerLaunch / pl->hg;
  if (pl->seqs_per_launch < 1) return B2D_ERR_TOO_LARGE;
  if (pl->seqs_per_launch > a->batch) pl->seqs_per_launch = a->batch > 0 ? a->batch : 1;
  pl->rows_per_launch = pl->seqs_per_launch * pl->hg;
  pl->smem = (size_t)pl->stages * 2 * pl->stage_bytes + 2 * pl->stages * sizeof(uint64_t) +
             (size_t)(pl->rows_per_launch + 1) * 4 + 32 * 4 + (pl->mma ? 1024 : 0);
  // Chunk indices are 32-bit in the kernel.
  const int64_t max_chunks_per_row =
      ((int64_t)a->max_pages_per_seq * a->page_size + pl->T - 1) / pl->T;
  if (max_chunks_per_row * pl->rows_per_launch > (int64_t)INT32_MAX) return B2D_ERR_TOO_LARGE;
  // num_ctas == 0: one resident wave, resolved at launch from the occupancy
  // of the selected kernel; the workspace is sized for the largest wave.
  int ctas = a->num_ctas;
  int ctas_cap = ctas;
  if (ctas <= 0) {
    int sms = 0;
    if (device_sm_count(&sms) != 0) return B2D_ERR_CUDA;
    ctas_cap = sms * plan_ctas_per_sm(*pl);
  }
  pl->ctas = ctas;
  const int hqc = pl->hk * group;
  const size_t segs = (size_t)pl->rows_per_launch + ctas_cap;
  pl->off_row_start = kWsHeaderBytes;
  pl->off_part_lse = align_up(pl->off_row_start + (size_t)(pl->rows_per_launch + 1) * 4, 256);
  pl->off_part_o = align_up(pl->off_part_lse + segs * hqc * 4, 256);
  pl->ws_bytes = align_up(pl->off_part_o + segs * hqc * (size_t)a->head_dim * 4, 256);
  return B2D_OK;
}

template <typename Kern>
static int launch_k(Kern kern, void (*combine)(const GqaParams, int, int), const GqaPlan& pl,
                    const CUtensorMap& tk, const CUtensorMap& tv, const GqaParams& p,
                    cudaStream_t st, int flags) {
  const int threads = 32 * (pl.nw + 1);
  if (ensure_dynamic_smem(reinterpret_cast<const void*>(kern), pl.smem)) return B2D_ERR_CUDA;
  int ctas = pl.ctas;
  if (ctas <= 0) {
    int sms = 0, per_sm = 0;
    if (device_sm_count(&sms) != 0) return B2D_ERR_CUDA;
    if (occupancy_per_sm(reinterpret_cast<const void*>(kern), threads, pl.smem, &per_sm))
      return B2D_ERR_CUDA;
    const int cap = plan_ctas_per_sm(pl);
    per_sm = per_sm < 1 ? 1 : (per_sm > cap ? cap : per_sm);
    ctas = sms * per_sm;
  }
  const int R = p.B * p.HG;
  // The split merge runs inside the split-KV kernel (the last warp to finish
  // a split row merges it) when rows are split over few CTAs each; with few
  // rows (small batches, rows over ~100 CTAs) the multi-warp combine kernel
  // spreads the merges instead.  B2D_GQA_FUSED_MERGE=0/1 forces either.
  static const int fused_env = env_int("B2D_GQA_FUSED_MERGE", -1);
  const bool fused = pl.mma && (fused_env >= 0 ? fused_env != 0 : (int64_t)R * 7 >= ctas) &&
                     (int64_t)R * p.NW <= kMergeCounters;
  if (pl.launch_count != nullptr) {
    *pl.launch_count += (flags & B2D_FLAG_COMBINE_ONLY) ? 0 : 1;
    if (!fused && !(flags & B2D_FLAG_SKIP_COMBINE) && R * pl.hk * pl.group > 0) ++*pl.launch_count;
    return B2D_OK;
  }
  if (!(flags & B2D_FLAG_COMBINE_ONLY)) {
    GqaParams pk = p;
    pk.merge_count = fused ? p.merge_count : nullptr;
    // Programmatic dependent launch (B2D_PDL=0 turns it off): the kernel's
    // prologue (barrier set-up, descriptor prefetch) overlaps the tail of
    // the previous kernel on the stream; the kernel waits for that kernel's
    // completion before it reads any input.
    static const int pdl = env_int("B2D_PDL", 1);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(ctas);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = pl.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    if (cudaLaunchKernelEx(&cfg, kern, tk, tv, pk) != cudaSuccess) return B2D_ERR_CUDA;
    if (cudaGetLastError() != cudaSuccess) return B2D_ERR_CUDA;
  }
  if (fused) return B2D_OK;
  const int64_t merges = (int64_t)R * pl.hk * pl.group;
  const int wpp = combine_warps_per_merge(merges);
  const int blocks = (int)((merges + 8 / wpp - 1) / (8 / wpp));
  if (blocks > 0 && !(flags & B2D_FLAG_SKIP_COMBINE)) {
    combine<<<blocks, 256, 0, st>>>(p, ctas, wpp);
    if (cudaGetLastError() != cudaSuccess) return B2D_ERR_CUDA;
  }
  return B2D_OK;
}

template <int D, int KIND, typename QT, int HQW>
static int launch_t(const GqaPlan& pl, const CUtensorMap& tk, const CUtensorMap& tv,
                    const GqaParams& p, cudaStream_t st, int flags) {
  return launch_k(gqa_decode_kernel<D, KIND, QT, HQW>, gqa_combine_kernel<D, QT>, pl, tk, tv, p,
                  st, flags);
}

template <int D, int KIND, typename QT, bool VL = false>
static int launch_mma(const GqaPlan& pl, const CUtensorMap& tk, const CUtensorMap& tv,
                      const GqaParams& p, cudaStream_t st, int flags) {
  if (pl.np == 2) {
    if constexpr (D >= 192) return B2D_ERR_UNSUPPORTED;
    else
      return launch_k(gqa_mma_kernel<D, KIND, QT, 2, VL>, gqa_combine_kernel<D, QT>, pl, tk, tv,
                      p, st, flags);
  }
  return launch_k(gqa_mma_kernel<D, KIND, QT, 1, VL>, gqa_combine_kernel<D, QT>, pl, tk, tv, p,
                  st, flags);
}

template <int D, int KIND, typename QT>
static int launch_hqw(const GqaPlan& pl, const CUtensorMap& tk, const CUtensorMap& tv,
                      const GqaParams& p, cudaStream_t st, int flags) {
  switch (pl.hqw) {
    case 4: return launch_t<D, KIND, QT, 4>(pl, tk, tv, p, st, flags);
    case 2: return launch_t<D, KIND, QT, 2>(pl, tk, tv, p, st, flags);
    default: return launch_t<D, KIND, QT, 1>(pl, tk, tv, p, st, flags);
  }
}

template <int D>
static int launch_d(const b2d_gqa_args* a, const GqaPlan& pl, const CUtensorMap& tk,
                    const CUtensorMap& tv, const GqaParams& p, cudaStream_t st) {
  const int flags = a->flags;
  const bool qbf = a->q_dtype == B2D_BF16;
  if (a->kv_layout == B2D_KV_VLLM)  // the plan admits only 16-bit caches here
    return qbf ? launch_mma<D, kKvBf16, __nv_bfloat16, true>(pl, tk, tv, p, st, flags)
               : launch_mma<D, kKvFp16, __half, true>(pl, tk, tv, p, st, flags);
  if constexpr (D == 192) {
    // the plan admits only the tensor-core path with 16-bit caches here
    return qbf ? launch_mma<D, kKvBf16, __nv_bfloat16>(pl, tk, tv, p, st, flags)
               : launch_mma<D, kKvFp16, __half>(pl, tk, tv, p, st, flags);
  } else {
    if (pl.mma) {
      if (a->kv_dtype == B2D_FP8_E4M3)
        return qbf ? launch_mma<D, kKvFp8, __nv_bfloat16>(pl, tk, tv, p, st, flags)
                   : launch_mma<D, kKvFp8, __half>(pl, tk, tv, p, st, flags);
      return qbf ? launch_mma<D, kKvBf16, __nv_bfloat16>(pl, tk, tv, p, st, flags)
                 : launch_mma<D, kKvFp16, __half>(pl, tk, tv, p, st, flags);
    }
    if (a->kv_dtype == B2D_FP8_E4M3) {
      return qbf ? launch_hqw<D, kKvFp8, __nv_bfloat16>(pl, tk, tv, p, st, flags)
                 : launch_hqw<D, kKvFp8, __half>(pl, tk, tv, p, st, flags);
    }
    return qbf ? launch_hqw<D, kKvBf16, __nv_bfloat16>(pl, tk, tv, p, st, flags)
               : launch_hqw<D, kKvFp16, __half>(pl, tk, tv, p, st, flags);
  }
}

static int encode_kv_map(CUtensorMap* map, const void* base, const b2d_gqa_args* a,
                         int64_t s_page, int64_t s_tok, int64_t s_head, const GqaPlan& pl,
                         bool is_v) {
  const int es = kv_elem_bytes(a->kv_dtype);
  const CUtensorMapDataType dt = es == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_UINT16;
  const uint64_t page_heads = (uint64_t)a->num_pages * (uint64_t)a->num_kv_heads;
  if (a->kv_layout == B2D_KV_VLLM && !is_v) {
    // K [blocks, Hkv, D/8, P, 8]: 16 tokens x 8 elements are one contiguous
    // 256-byte run, so the map is {P * 8 elements, 8-dim group, block * Hkv +
    // head} with a 128-element inner box; shared layout [HK][D / 8][16
    // tokens][8], no swizzle (an ldmatrix's 8 token rows are 16 bytes apart).
    const uint64_t P = (uint64_t)a->page_size;
    const uint64_t dims[3] = {P * 8, (uint64_t)a->head_dim / 8, page_heads};
    const uint64_t strides[2] = {P * 16, (uint64_t)(s_head * es)};
    const uint32_t box[3] = {128u, (uint32_t)(a->head_dim / 8), (uint32_t)pl.hk};
    return encode_tiled_map(map, dt, 3, base, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE);
  }
  if (a->kv_layout == B2D_KV_VLLM) {
    // V [blocks, Hkv, D, P]: shared layout [HK][D][16 tokens] (32-byte rows =
    // V^T), no swizzle.  With 16-token pages a head's block is one
    // contiguous run: {8 dims x 16 tokens, 8-dim group, block * Hkv + head};
    // otherwise {token, dim, block * Hkv + head} with 32-byte rows.
    const uint64_t P = (uint64_t)a->page_size;
    if (P == 16) {
      const uint64_t dims[3] = {128, (uint64_t)a->head_dim / 8, page_heads};
      const uint64_t strides[2] = {256, (uint64_t)(s_head * es)};
      const uint32_t box[3] = {128u, (uint32_t)(a->head_dim / 8), (uint32_t)pl.hk};
      return encode_tiled_map(map, dt, 3, base, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE);
    }
    const uint64_t dims[3] = {P, (uint64_t)a->head_dim, page_heads};
    const uint64_t strides[2] = {P * 2, (uint64_t)(s_head * es)};
    const uint32_t box[3] = {16u, (uint32_t)a->head_dim, (uint32_t)pl.hk};
    return encode_tiled_map(map, dt, 3, base, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE);
  }
  if (pl.mma) {
    // {128-byte line, token, line of the head row, head, page}; 128-byte
    // swizzle.  Shared layout: [HK][D / line][16 tokens][line].
    const uint64_t line = 128 / es;
    const uint64_t dims[5] = {line, (uint64_t)a->page_size, (uint64_t)a->head_dim / line,
                              (uint64_t)a->num_kv_heads, (uint64_t)a->num_pages};
    const uint64_t strides[4] = {(uint64_t)(s_tok * es), 128u, (uint64_t)(s_head * es),
                                 (uint64_t)(s_page * es)};
    const uint32_t box[5] = {(uint32_t)line, 16u, (uint32_t)(a->head_dim / line), (uint32_t)pl.hk,
                             1u};
    return encode_tiled_map(map, dt, 5, base, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  }
  const uint64_t dims[4] = {(uint64_t)a->head_dim, (uint64_t)a->num_kv_heads,
                            (uint64_t)a->page_size, (uint64_t)a->num_pages};
  const uint64_t strides[3] = {(uint64_t)(s_head * es), (uint64_t)(s_tok * es),
                               (uint64_t)(s_page * es)};
  const uint32_t box[4] = {(uint32_t)a->head_dim, (uint32_t)pl.hk, (uint32_t)pl.T, 1u};
  return encode_tiled_map(map, dt, 4, base, dims, strides, box);
}

}  // namespace b2d

using namespace b2d;

extern "C" int b2d_gqa_workspace_bytes(const b2d_gqa_args* a, size_t* bytes) {
  int rc = validate(a, false);
  if (rc) return rc;
  if (!bytes) return B2D_ERR_INVALID_ARG;
  GqaPlan pl{};
  rc = make_plan(a, &pl);
  if (rc) return rc;
  *bytes = pl.ws_bytes;
  return B2D_OK;
}

extern "C" int b2d_gqa_plan(const b2d_gqa_args* a, int32_t* num_ctas, int32_t* chunk_tokens,
                            int32_t* kv_heads_per_cta) {
  int rc = validate(a, false);
  if (rc) return rc;
  GqaPlan pl{};
  rc = make_plan(a, &pl);
  if (rc) return rc;
  if (num_ctas) *num_ctas = pl.ctas;
  if (chunk_tokens) *chunk_tokens = pl.T;
  if (kv_heads_per_cta) *kv_heads_per_cta = pl.hk;
  return B2D_OK;
}

static int decode_gqa(const b2d_gqa_args* a, void* stream, int* launch_count) {
  int rc = validate(a, launch_count == nullptr);
  if (rc) return rc;
  if (a->batch == 0) return B2D_OK;
  GqaPlan pl{};
  rc = make_plan(a, &pl);
  if (rc) return rc;
  pl.launch_count = launch_count;
  if (launch_count == nullptr) {
    if (!a->workspace || a->workspace_bytes < pl.ws_bytes) return B2D_ERR_WORKSPACE;
    if ((uintptr_t)a->workspace & 255) return B2D_ERR_ALIGNMENT;
  }
  CUtensorMap tk{}, tv{};
  if (launch_count == nullptr && (encode_kv_map(&tk, a->k_cache, a, a->k_stride_page, a->k_stride_tok, a->k_stride_head, pl,
                    false) ||
      encode_kv_map(&tv, a->v_cache, a, a->v_stride_page, a->v_stride_tok, a->v_stride_head, pl,
                    true)))
    return B2D_ERR_CUDA;
  uint8_t* ws = static_cast<uint8_t*>(a->workspace);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const float kLog2e = 1.4426950408889634f;
  for (int b0 = 0; b0 < a->batch; b0 += pl.seqs_per_launch) {
    const int nb = (a->batch - b0) < pl.seqs_per_launch ? (a->batch - b0) : pl.seqs_per_launch;
    const int qes = 2;
    GqaParams p{};
    p.q = static_cast<const uint8_t*>(a->q) + (size_t)b0 * a->q_stride_b * qes;
    p.q_sb = a->q_stride_b;
    p.q_sh = a->q_stride_h;
    p.out = static_cast<uint8_t*>(a->out) + (size_t)b0 * a->out_stride_b * qes;
    p.o_sb = a->out_stride_b;
    p.o_sh = a->out_stride_h;
    p.lse = a->lse ? a->lse + (size_t)b0 * a->lse_stride_b : nullptr;
    p.lse_sb = a->lse_stride_b;
    p.seqlens = a->cache_seqlens + b0;
    p.block_table = a->block_table + (size_t)b0 * a->block_table_stride;
    p.bt_stride = a->block_table_stride;
    p.k_scale = a->k_scale;
    p.v_scale = a->v_scale;
    p.status = reinterpret_cast<int*>(ws);
    p.merge_count = reinterpret_cast<int32_t*>(ws + kStatusBytes);
    p.wait_ns = a->wait_limit_us > 0 ? (unsigned long long)a->wait_limit_us * 1000ull : kWaitLimitNs;
    p.no_loads = (a->flags & B2D_FLAG_TEST_NO_LOADS) ? 1 : 0;
    p.row_start_g = reinterpret_cast<int32_t*>(ws + pl.off_row_start);
    p.part_lse = reinterpret_cast<float*>(ws + pl.off_part_lse);
    p.part_o = reinterpret_cast<float*>(ws + pl.off_part_o);
    p.B = nb;
    p.Hq = a->num_q_heads;
    p.Hkv = a->num_kv_heads;
    p.group = pl.group;
    p.HK = pl.hk;
    p.HG = pl.hg;
    p.P = a->page_size;
    p.T = pl.T;
    p.stages = pl.stages;
    p.NW = pl.nw;
    p.WPH = pl.wph;
    p.num_pages = (int)a->num_pages;
    p.max_pages = a->max_pages_per_seq;
    p.scale_log2 = a->softmax_scale * kLog2e;
    p.stage_bytes = pl.stage_bytes;
    switch (a->head_dim) {
      case 64: rc = launch_d<64>(a, pl, tk, tv, p, st); break;
      case 128: rc = launch_d<128>(a, pl, tk, tv, p, st); break;
      case 192: rc = launch_d<192>(a, pl, tk, tv, p, st); break;
      default: rc = launch_d<256>(a, pl, tk, tv, p, st); break;
    }
    if (rc) return rc;
  }
  return B2D_OK;
}

extern "C" int b2d_decode_gqa(const b2d_gqa_args* a, void* stream) {
  return decode_gqa(a, stream, nullptr);
}

extern "C" int b2d_gqa_launch_count(const b2d_gqa_args* a, int32_t* launches) {
  if (!launches) return B2D_ERR_INVALID_ARG;
  int n = 0;
  const int rc = decode_gqa(a, nullptr, &n);
  if (rc) return rc;
  *launches = n;
  return B2D_OK;
}
