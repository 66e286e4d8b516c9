// mla_host.cu — host side of the absorbed-MLA decode: validation, TMA
// descriptors, workspace layout, and the split-KV + combine launches.
#include "b2d_decode.h"
#include "host_common.h"
#include "mla_kernel.cuh"

namespace b2d {

constexpr int kMlaMaxRows = 384;    // sequences per launch (row table in shared memory)

struct MlaPlan {
  int nr;            // CTA pairs (ranges)
  int seqs_per_launch;
  size_t smem, off_rows, off_part_lse, off_part_o, ws_bytes;
};

static int mla_validate(const b2d_mla_args* a, bool need_pointers) {
  if (!a) return B2D_ERR_INVALID_ARG;
  if (a->batch < 0 || a->page_size <= 0 || a->max_pages_per_seq <= 0) return B2D_ERR_INVALID_ARG;
  if (a->num_heads != 128 || a->head_dim_qk != 576 || a->head_dim_v != 512) return B2D_ERR_UNSUPPORTED;
  if (a->dtype != B2D_BF16) return B2D_ERR_UNSUPPORTED;
  if (a->page_size % mla::kT != 0) return B2D_ERR_UNSUPPORTED;
  // Token positions (max_pages_per_seq * page_size) are 32-bit in the kernel.
  if ((int64_t)a->max_pages_per_seq * a->page_size > (int64_t)INT32_MAX) return B2D_ERR_TOO_LARGE;
  if (a->wait_limit_us < 0) return B2D_ERR_INVALID_ARG;
  if (!need_pointers || a->batch == 0) return B2D_OK;
  if (!a->q || !a->kv_cache || !a->cache_seqlens || !a->block_table || !a->out)
    return B2D_ERR_INVALID_ARG;
  if (a->num_pages <= 0 || a->num_pages > (int64_t)INT32_MAX) return B2D_ERR_INVALID_ARG;
  if (((uintptr_t)a->q & 15) || ((uintptr_t)a->kv_cache & 15) || ((uintptr_t)a->out & 15))
    return B2D_ERR_ALIGNMENT;
  if ((a->q_stride_h * 2) % 16 || (a->q_stride_b * 2) % 16 || (a->kv_stride_tok * 2) % 16 ||
      (a->kv_stride_page * 2) % 16 || (a->out_stride_h * 2) % 16 || (a->out_stride_b * 2) % 16)
    return B2D_ERR_ALIGNMENT;
  return B2D_OK;
}

static int mla_make_plan(const b2d_mla_args* a, MlaPlan* pl) {
  int nr = a->num_ctas > 0 ? a->num_ctas / 2 : 0;
  if (nr <= 0) {
    int sms = 0;
    if (device_sm_count(&sms)) return B2D_ERR_CUDA;
    nr = sms / 2;  // 512 TMEM columns and ~200 KB of shared memory: one CTA per SM
  }
  if (nr < 1) nr = 1;
  pl->nr = nr;
  pl->seqs_per_launch = a->batch < kMlaMaxRows ? (a->batch > 0 ? a->batch : 1) : kMlaMaxRows;
  pl->smem = 1024 + mla::kOffRows + (size_t)(pl->seqs_per_launch + 1) * 4 + 32 * 4;
  const size_t segs = (size_t)pl->seqs_per_launch + nr;
  pl->off_rows = kWsHeaderBytes;
  pl->off_part_lse = align_up(pl->off_rows + (size_t)(pl->seqs_per_launch + 1) * 4, 256);
  pl->off_part_o = align_up(pl->off_part_lse + segs * 128 * 4, 256);
  pl->ws_bytes = align_up(pl->off_part_o + segs * 128 * 512 * 4, 256);
  return B2D_OK;
}

}  // namespace b2d

using namespace b2d;

extern "C" int b2d_mla_workspace_bytes(const b2d_mla_args* a, size_t* bytes) {
  int rc = mla_validate(a, false);
  if (rc) return rc;
  if (!bytes) return B2D_ERR_INVALID_ARG;
  MlaPlan pl;
  rc = mla_make_plan(a, &pl);
  if (rc) return rc;
  *bytes = pl.ws_bytes;
  return B2D_OK;
}

extern "C" int b2d_decode_mla(const b2d_mla_args* a, void* stream) {
  int rc = mla_validate(a, true);
  if (rc) return rc;
  if (a->batch == 0) return B2D_OK;
  MlaPlan pl;
  rc = mla_make_plan(a, &pl);
  if (rc) return rc;
  if (!a->workspace || a->workspace_bytes < pl.ws_bytes) return B2D_ERR_WORKSPACE;
  if ((uintptr_t)a->workspace & 255) return B2D_ERR_ALIGNMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  CUtensorMap tkv;
  {
    const uint64_t dims[5] = {64, (uint64_t)a->page_size, 9, (uint64_t)a->num_pages, 1};
    const uint64_t strides[4] = {(uint64_t)a->kv_stride_tok * 2, 128,
                                 (uint64_t)a->kv_stride_page * 2,
                                 (uint64_t)a->kv_stride_page * 2 * (uint64_t)a->num_pages};
    const uint32_t box[5] = {64, (uint32_t)mla::kT, 9, 1, 1};
    if (encode_tiled_map(&tkv, CU_TENSOR_MAP_DATA_TYPE_UINT16, 5, a->kv_cache, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_128B))
      return B2D_ERR_CUDA;
  }
  auto kern = mla_decode_kernel;
  if (ensure_dynamic_smem(reinterpret_cast<const void*>(kern), pl.smem)) return B2D_ERR_CUDA;
  uint8_t* ws = static_cast<uint8_t*>(a->workspace);
  const float kLog2e = 1.4426950408889634f;
  for (int b0 = 0; b0 < a->batch; b0 += pl.seqs_per_launch) {
    const int nb = (a->batch - b0) < pl.seqs_per_launch ? (a->batch - b0) : pl.seqs_per_launch;
    MlaParams p{};
    p.q = static_cast<const uint8_t*>(a->q) + (size_t)b0 * a->q_stride_b * 2;
    p.q_sb = a->q_stride_b;
    p.q_sh = a->q_stride_h;
    p.seqlens = a->cache_seqlens + b0;
    p.block_table = a->block_table + (size_t)b0 * a->block_table_stride;
    p.bt_stride = a->block_table_stride;
    p.out = static_cast<uint8_t*>(a->out) + (size_t)b0 * a->out_stride_b * 2;
    p.o_sb = a->out_stride_b;
    p.o_sh = a->out_stride_h;
    p.lse = a->lse ? a->lse + (size_t)b0 * a->lse_stride_b : nullptr;
    p.lse_sb = a->lse_stride_b;
    p.status = reinterpret_cast<int*>(ws);
    p.wait_ns = a->wait_limit_us > 0 ? (unsigned long long)a->wait_limit_us * 1000ull : kWaitLimitNs;
    p.row_start_g = reinterpret_cast<int32_t*>(ws + pl.off_rows);
    p.part_lse = reinterpret_cast<float*>(ws + pl.off_part_lse);
    p.part_o = reinterpret_cast<float*>(ws + pl.off_part_o);
    p.B = nb;
    p.P = a->page_size;
    p.num_pages = (int)a->num_pages;
    p.max_pages = a->max_pages_per_seq;
    p.scale_log2 = a->softmax_scale * kLog2e;
    if (!(a->flags & B2D_FLAG_COMBINE_ONLY)) {
      kern<<<2 * pl.nr, mla::kThreads, pl.smem, st>>>(tkv, p);
      if (cudaGetLastError() != cudaSuccess) return B2D_ERR_CUDA;
    }
    if (!(a->flags & B2D_FLAG_SKIP_COMBINE)) {
      GqaParams cp{};
      cp.out = p.out;
      cp.o_sb = p.o_sb;
      cp.o_sh = p.o_sh;
      cp.lse = p.lse;
      cp.lse_sb = p.lse_sb;
      cp.part_o = p.part_o;
      cp.part_lse = p.part_lse;
      cp.row_start_g = p.row_start_g;
      cp.B = nb;
      cp.HG = 1;
      cp.HK = 1;
      cp.group = 128;
      const int64_t merges = (int64_t)nb * 128;
      const int wpp = combine_warps_per_merge(merges);
      const int blocks = (int)((merges + 8 / wpp - 1) / (8 / wpp));
      gqa_combine_kernel<512, __nv_bfloat16><<<blocks, 256, 0, st>>>(cp, pl.nr, wpp);
      if (cudaGetLastError() != cudaSuccess) return B2D_ERR_CUDA;
    }
  }
  return B2D_OK;
}
