// gqa_host.cu — host side of the GQA decode: argument validation, the split
// plan, TMA descriptor encoding, workspace layout and the two launches.
// Exposed through the C ABI in include/b2d_decode.h.
#include "b2d_decode.h"
#include "gqa_kernel.cuh"
#include "host_common.h"

namespace b2d {

// Rows (sequence x KV-head group) handled by one launch; larger batches are
// cut into slices of whole sequences that reuse the same workspace in order.
constexpr int kMaxRowsPerLaunch = 2048;
// Shared-memory budget for the K/V stage ring of one CTA (two CTAs per SM).
constexpr size_t kStageRingBytes = 96 * 1024;
constexpr size_t kStatusBytes = 256;

struct GqaPlan {
  int group, hqw, wph, hk, hg, nw, T, stages, ctas, rows_per_launch, seqs_per_launch;
  uint32_t stage_bytes;
  size_t smem;
  size_t off_row_start, off_part_lse, off_part_o, ws_bytes;
};

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
  if (a->head_dim != 64 && a->head_dim != 128 && a->head_dim != 256) return B2D_ERR_UNSUPPORTED;
  if (a->q_dtype != B2D_BF16 && a->q_dtype != B2D_FP16) return B2D_ERR_UNSUPPORTED;
  if (a->kv_dtype != a->q_dtype && a->kv_dtype != B2D_FP8_E4M3) return B2D_ERR_UNSUPPORTED;
  const int group = a->num_q_heads / a->num_kv_heads;
  if (group > 32) return B2D_ERR_UNSUPPORTED;
  if (a->page_size > (1 << 24)) return B2D_ERR_TOO_LARGE;
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
  for (int64_t s : strides)
    if (s <= 0 || (s * es) % 16 != 0) return B2D_ERR_ALIGNMENT;
  if ((a->q_stride_b * 2) % 16 || (a->q_stride_h * 2) % 16 || (a->out_stride_b * 2) % 16 ||
      (a->out_stride_h * 2) % 16)
    return B2D_ERR_ALIGNMENT;
  return B2D_OK;
}

static int make_plan(const b2d_gqa_args* a, GqaPlan* pl) {
  const int group = a->num_q_heads / a->num_kv_heads;
  pl->group = group;
  pl->hqw = (group % 4 == 0) ? 4 : (group % 2 == 0 ? 2 : 1);
  pl->wph = group / pl->hqw;
  if (pl->wph > 8) return B2D_ERR_UNSUPPORTED;
  pl->hk = largest_divisor_leq(a->num_kv_heads, 8 / pl->wph);
  pl->hg = a->num_kv_heads / pl->hk;
  pl->nw = pl->hk * pl->wph;
  const int es = kv_elem_bytes(a->kv_dtype);
  const int row_bytes = pl->hk * a->head_dim * es;
  // Chunk: the largest divisor of the page size that keeps one K tile at
  // <= 16 KB and the TMA box at <= 256 rows.
  int tmax = 16384 / row_bytes;
  if (tmax < 1) tmax = 1;
  if (tmax > 256) tmax = 256;
  pl->T = largest_divisor_leq(a->page_size, tmax);
  pl->stage_bytes = (uint32_t)(pl->T * row_bytes);
  int stages = (int)(kStageRingBytes / (2 * (size_t)pl->stage_bytes));
  pl->stages = stages < 2 ? 2 : (stages > 8 ? 8 : stages);
  pl->seqs_per_launch = kMaxRowsPerLaunch / pl->hg;
  if (pl->seqs_per_launch < 1) return B2D_ERR_TOO_LARGE;
  if (pl->seqs_per_launch > a->batch) pl->seqs_per_launch = a->batch > 0 ? a->batch : 1;
  pl->rows_per_launch = pl->seqs_per_launch * pl->hg;
  pl->smem = (size_t)pl->stages * 2 * pl->stage_bytes + 2 * pl->stages * sizeof(uint64_t) +
             (size_t)(pl->rows_per_launch + 1) * 4 + 32 * 4;
  int ctas = a->num_ctas;
  if (ctas <= 0) {
    int sms = 0;
    if (device_sm_count(&sms) != 0) return B2D_ERR_CUDA;
    const int per_sm = (2 * (pl->smem + 1024) <= 227 * 1024) ? 2 : 1;
    ctas = sms * per_sm;
  }
  pl->ctas = ctas;
  const int hqc = pl->hk * group;
  const size_t segs = (size_t)pl->rows_per_launch + ctas;
  pl->off_row_start = kStatusBytes;
  pl->off_part_lse = align_up(pl->off_row_start + (size_t)(pl->rows_per_launch + 1) * 4, 256);
  pl->off_part_o = align_up(pl->off_part_lse + segs * hqc * 4, 256);
  pl->ws_bytes = align_up(pl->off_part_o + segs * hqc * (size_t)a->head_dim * 4, 256);
  return B2D_OK;
}

template <int D, int KIND, typename QT, int HQW>
static int launch_t(const GqaPlan& pl, const CUtensorMap& tk, const CUtensorMap& tv,
                    const GqaParams& p, cudaStream_t st, int flags) {
  auto kern = gqa_decode_kernel<D, KIND, QT, HQW>;
  if (!(flags & B2D_FLAG_COMBINE_ONLY)) {
    if (ensure_dynamic_smem(reinterpret_cast<const void*>(kern), pl.smem)) return B2D_ERR_CUDA;
    kern<<<pl.ctas, 32 * (pl.nw + 1), pl.smem, st>>>(tk, tv, p);
    if (cudaGetLastError() != cudaSuccess) return B2D_ERR_CUDA;
  }
  const int R = p.B * p.HG;
  const int64_t warps = (int64_t)R * pl.hk * pl.group;
  const int blocks = (int)((warps * 32 + 255) / 256);
  if (blocks > 0 && !(flags & B2D_FLAG_SKIP_COMBINE)) {
    gqa_combine_kernel<D, QT><<<blocks, 256, 0, st>>>(p, pl.ctas);
    if (cudaGetLastError() != cudaSuccess) return B2D_ERR_CUDA;
  }
  return B2D_OK;
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
  if (a->kv_dtype == B2D_FP8_E4M3) {
    return qbf ? launch_hqw<D, kKvFp8, __nv_bfloat16>(pl, tk, tv, p, st, flags)
               : launch_hqw<D, kKvFp8, __half>(pl, tk, tv, p, st, flags);
  }
  return qbf ? launch_hqw<D, kKvBf16, __nv_bfloat16>(pl, tk, tv, p, st, flags)
             : launch_hqw<D, kKvFp16, __half>(pl, tk, tv, p, st, flags);
}

static int encode_kv_map(CUtensorMap* map, const void* base, const b2d_gqa_args* a,
                         int64_t s_page, int64_t s_tok, int64_t s_head, const GqaPlan& pl) {
  const int es = kv_elem_bytes(a->kv_dtype);
  const uint64_t dims[4] = {(uint64_t)a->head_dim, (uint64_t)a->num_kv_heads,
                            (uint64_t)a->page_size, (uint64_t)a->num_pages};
  const uint64_t strides[3] = {(uint64_t)(s_head * es), (uint64_t)(s_tok * es),
                               (uint64_t)(s_page * es)};
  const uint32_t box[4] = {(uint32_t)a->head_dim, (uint32_t)pl.hk, (uint32_t)pl.T, 1u};
  return encode_tiled_map(map, es == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_UINT16,
                          4, base, dims, strides, box);
}

}  // namespace b2d

using namespace b2d;

extern "C" int b2d_gqa_workspace_bytes(const b2d_gqa_args* a, size_t* bytes) {
  int rc = validate(a, false);
  if (rc) return rc;
  if (!bytes) return B2D_ERR_INVALID_ARG;
  GqaPlan pl;
  rc = make_plan(a, &pl);
  if (rc) return rc;
  *bytes = pl.ws_bytes;
  return B2D_OK;
}

extern "C" int b2d_gqa_plan(const b2d_gqa_args* a, int32_t* num_ctas, int32_t* chunk_tokens,
                            int32_t* kv_heads_per_cta) {
  int rc = validate(a, false);
  if (rc) return rc;
  GqaPlan pl;
  rc = make_plan(a, &pl);
  if (rc) return rc;
  if (num_ctas) *num_ctas = pl.ctas;
  if (chunk_tokens) *chunk_tokens = pl.T;
  if (kv_heads_per_cta) *kv_heads_per_cta = pl.hk;
  return B2D_OK;
}

extern "C" int b2d_decode_gqa(const b2d_gqa_args* a, void* stream) {
  int rc = validate(a, true);
  if (rc) return rc;
  if (a->batch == 0) return B2D_OK;
  GqaPlan pl;
  rc = make_plan(a, &pl);
  if (rc) return rc;
  if (!a->workspace || a->workspace_bytes < pl.ws_bytes) return B2D_ERR_WORKSPACE;
  if ((uintptr_t)a->workspace & 255) return B2D_ERR_ALIGNMENT;
  CUtensorMap tk, tv;
  if (encode_kv_map(&tk, a->k_cache, a, a->k_stride_page, a->k_stride_tok, a->k_stride_head, pl) ||
      encode_kv_map(&tv, a->v_cache, a, a->v_stride_page, a->v_stride_tok, a->v_stride_head, pl))
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
      default: rc = launch_d<256>(a, pl, tk, tv, p, st); break;
    }
    if (rc) return rc;
  }
  return B2D_OK;
}
