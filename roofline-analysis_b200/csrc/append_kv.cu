// append_kv.cu — KV-cache append with optional FP8-e4m3 quantisation: the
// write side of the paged cache (vLLM's reshape_and_cache, called by the
// reference at decodebench/vllm_paged_kernel.py:160-172).  HBM-bound copy:
// each thread moves 8 elements of one (token, head) row with one 16-byte
// load and one 16-byte (8-byte for FP8) store.
#include <type_traits>

#include "b2d_decode.h"
#include "common.cuh"

namespace b2d {

struct AppendParams {
  const void* key;
  const void* value;
  int64_t src_st, src_sh;
  void* kc;
  void* vc;
  int64_t k_sp, k_st, k_sh, v_sp, v_st, v_sh;
  int64_t k_sg;   // elements between consecutive 8-element groups of a K row (8, or P * 8 for vLLM)
  int64_t v_sd;   // elements between consecutive dims of a V row (1, or P for vLLM)
  const int64_t* slots;
  const float* k_scale;
  const float* v_scale;
  int* bad;
  int T, H, D, P;
  int64_t cap;  // num_pages * page_size
};

// Two fp32 -> two e4m3 bytes (lo in bits 0-7), round-to-nearest-even,
// saturated to the largest finite e4m3 value (the hardware cvt).
__device__ __forceinline__ uint16_t f2_to_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

template <typename ST, bool FP8>
__global__ void __launch_bounds__(256) append_kv_kernel(const AppendParams p) {
  const int lanes_per_row = p.D / 8;
  const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t rows = (int64_t)p.T * p.H;
  const int64_t row = gid / lanes_per_row;
  if (row >= rows) return;
  const int c = (int)(gid - row * lanes_per_row);
  const int t = (int)(row / p.H), h = (int)(row - (int64_t)t * p.H);
  const int64_t slot = p.slots[t];
  if (slot < 0) return;
  if (slot >= p.cap) {
    if (p.bad && c == 0 && h == 0) atomicAdd(p.bad, 1);
    return;
  }
  const int64_t page = slot / p.P, off = slot - page * p.P;
  const int64_t src = (int64_t)t * p.src_st + (int64_t)h * p.src_sh + c * 8;
  const uint4 kw = *reinterpret_cast<const uint4*>(static_cast<const ST*>(p.key) + src);
  const uint4 vw = *reinterpret_cast<const uint4*>(static_cast<const ST*>(p.value) + src);
  const int64_t kd = page * p.k_sp + off * p.k_st + (int64_t)h * p.k_sh + c * p.k_sg;
  const int64_t vd = page * p.v_sp + off * p.v_st + (int64_t)h * p.v_sh + c * 8 * p.v_sd;
  if constexpr (!FP8) {
    *reinterpret_cast<uint4*>(static_cast<ST*>(p.kc) + kd) = kw;
    if (p.v_sd == 1) {
      *reinterpret_cast<uint4*>(static_cast<ST*>(p.vc) + vd) = vw;
    } else {
      // vLLM's V is [blocks, Hkv, D, P]: the 8 dims of this row are P apart.
      const uint16_t* e = reinterpret_cast<const uint16_t*>(&vw);
      uint16_t* dst = reinterpret_cast<uint16_t*>(static_cast<ST*>(p.vc) + vd);
#pragma unroll
      for (int i = 0; i < 8; ++i) dst[i * p.v_sd] = e[i];
    }
  } else {
    const float ks = 1.f / (p.k_scale ? __ldg(p.k_scale + h) : 1.f);
    const float vs = 1.f / (p.v_scale ? __ldg(p.v_scale + h) : 1.f);
    const uint32_t kws[4] = {kw.x, kw.y, kw.z, kw.w};
    const uint32_t vws[4] = {vw.x, vw.y, vw.z, vw.w};
    uint16_t ko[4], vo[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 a, b;
      if constexpr (std::is_same<ST, __nv_bfloat16>::value) {
        a = bf16x2_to_f2(kws[i]);
        b = bf16x2_to_f2(vws[i]);
      } else {
        a = f16x2_to_f2(kws[i]);
        b = f16x2_to_f2(vws[i]);
      }
      ko[i] = f2_to_e4m3x2(a.x * ks, a.y * ks);
      vo[i] = f2_to_e4m3x2(b.x * vs, b.y * vs);
    }
    uint8_t* kdst = static_cast<uint8_t*>(p.kc) + kd;
    uint8_t* vdst = static_cast<uint8_t*>(p.vc) + vd;
    *reinterpret_cast<uint2*>(kdst) = make_uint2(ko[0] | ((uint32_t)ko[1] << 16), ko[2] | ((uint32_t)ko[3] << 16));
    *reinterpret_cast<uint2*>(vdst) = make_uint2(vo[0] | ((uint32_t)vo[1] << 16), vo[2] | ((uint32_t)vo[3] << 16));
  }
}

}  // namespace b2d

using namespace b2d;

extern "C" int b2d_append_kv(const b2d_append_args* a, void* stream) {
  if (!a) return B2D_ERR_INVALID_ARG;
  if (a->num_tokens < 0 || a->num_kv_heads <= 0 || a->page_size <= 0) return B2D_ERR_INVALID_ARG;
  if (a->head_dim != 64 && a->head_dim != 128 && a->head_dim != 256 && a->head_dim != 576 &&
      a->head_dim != 512)
    return B2D_ERR_UNSUPPORTED;
  if (a->src_dtype != B2D_BF16 && a->src_dtype != B2D_FP16) return B2D_ERR_UNSUPPORTED;
  if (a->cache_dtype != a->src_dtype && a->cache_dtype != B2D_FP8_E4M3) return B2D_ERR_UNSUPPORTED;
  if (a->kv_layout != B2D_KV_STRIDED && a->kv_layout != B2D_KV_VLLM) return B2D_ERR_INVALID_ARG;
  const bool vllm = a->kv_layout == B2D_KV_VLLM;
  if (vllm && a->cache_dtype == B2D_FP8_E4M3) return B2D_ERR_UNSUPPORTED;
  if (a->num_tokens == 0) return B2D_OK;
  if (!a->key || !a->value || !a->k_cache || !a->v_cache || !a->slot_mapping || a->num_pages <= 0)
    return B2D_ERR_INVALID_ARG;
  const int es = a->cache_dtype == B2D_FP8_E4M3 ? 1 : 2;
  if (((uintptr_t)a->key & 15) || ((uintptr_t)a->value & 15) || ((uintptr_t)a->k_cache & 15) ||
      ((uintptr_t)a->v_cache & 15))
    return B2D_ERR_ALIGNMENT;
  const int64_t cs[6] = {a->k_stride_page, a->k_stride_tok, a->k_stride_head,
                         a->v_stride_page, a->v_stride_tok, a->v_stride_head};
  for (int i = 0; i < 6; ++i) {
    if (vllm && (i == 1 || i == 4)) continue;  // token strides implied by the layout
    if (cs[i] <= 0 || (cs[i] * es) % 8 != 0) return B2D_ERR_ALIGNMENT;
  }
  if ((a->src_stride_t * 2) % 16 || (a->src_stride_h * 2) % 16) return B2D_ERR_ALIGNMENT;
  AppendParams p{};
  p.key = a->key;
  p.value = a->value;
  p.src_st = a->src_stride_t;
  p.src_sh = a->src_stride_h;
  p.kc = a->k_cache;
  p.vc = a->v_cache;
  p.k_sp = a->k_stride_page;
  p.k_st = a->k_stride_tok;
  p.k_sh = a->k_stride_head;
  p.v_sp = a->v_stride_page;
  p.v_st = a->v_stride_tok;
  p.v_sh = a->v_stride_head;
  p.k_sg = 8;
  p.v_sd = 1;
  if (vllm) {  // K [blocks, Hkv, D/8, P, 8], V [blocks, Hkv, D, P]
    p.k_st = 8;
    p.k_sg = (int64_t)a->page_size * 8;
    p.v_st = 1;
    p.v_sd = a->page_size;
  }
  p.slots = a->slot_mapping;
  p.k_scale = a->k_scale;
  p.v_scale = a->v_scale;
  p.bad = a->bad_slots;
  p.T = a->num_tokens;
  p.H = a->num_kv_heads;
  p.D = a->head_dim;
  p.P = a->page_size;
  p.cap = a->num_pages * (int64_t)a->page_size;
  const int64_t threads = (int64_t)a->num_tokens * a->num_kv_heads * (a->head_dim / 8);
  const int blocks = (int)((threads + 255) / 256);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool bf = a->src_dtype == B2D_BF16;
  if (a->cache_dtype == B2D_FP8_E4M3) {
    if (bf) append_kv_kernel<__nv_bfloat16, true><<<blocks, 256, 0, st>>>(p);
    else append_kv_kernel<__half, true><<<blocks, 256, 0, st>>>(p);
  } else {
    if (bf) append_kv_kernel<__nv_bfloat16, false><<<blocks, 256, 0, st>>>(p);
    else append_kv_kernel<__half, false><<<blocks, 256, 0, st>>>(p);
  }
  return cudaGetLastError() == cudaSuccess ? B2D_OK : B2D_ERR_CUDA;
}
