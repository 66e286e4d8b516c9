// UMMA issue-rate microbenchmark (sm_100a): cycles per tcgen05.mma
// (kind::f16, bf16 x bf16 -> fp32) for M x N x 16 shapes, A from shared
// memory (SS) or tensor memory (TS), B K-major or MN-major (128-byte swizzle).
// One CTA per SM, one issuing thread, NITER back-to-back MMAs into one
// accumulator, then a commit whose wait is bounded (~2 s of clock64).
// Operand data are zeros; every operand lies inside the CTA's own shared
// memory or TMEM.  It sizes the MLA decode kernel's instruction shapes.
// Build and run on one GPU:
//   nvcc -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 umma_rate.cu -o umma_rate
//   ./umma_rate
#include <cstdio>
#include <cstdint>
#include <cuda_runtime.h>

#define NITER 512

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}
__host__ __device__ constexpr uint32_t idesc(int M, int N, bool bmn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((bmn ? 1u : 0u) << 16) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

template <int M, int N, bool A_TMEM, bool B_MN>
__global__ void __launch_bounds__(128, 1) probe(unsigned long long* out, int* status) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  __shared__ uint64_t bar;
  __shared__ uint32_t tslot;
  const int warp = threadIdx.x >> 5;
  // zero A [M x 64] and B (K = 64 elements; K-major: one 128-byte line per N row,
  // MN-major: N/64 blocks of 64 K-rows x 128 bytes)
  for (int i = threadIdx.x; i < (M * 128 + (N / 64) * 8192) / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(smem)[i] = make_uint4(0, 0, 0, 0);
  if (threadIdx.x == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&bar)));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(&tslot)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tslot;
  if (threadIdx.x == 0) {
    const uint32_t a_s = smem_u32(smem), b_s = a_s + M * 128;
    const uint64_t ad = desc_sw128(a_s, 16, 1024);
    // MN-major B: 64-element N blocks of 64 K-rows x 128 bytes, 8 KB apart
    const uint64_t bd = B_MN ? desc_sw128(b_s, 64 * 128, 1024) : desc_sw128(b_s, 16, 1024);
    const uint32_t id = idesc(M, N, B_MN);
    const uint32_t d_t = tmem;                 // accumulator columns 0..N-1
    const uint32_t a_t = tmem + (N <= 256 ? 256 : 0);   // A in TMEM (same lanes as D)
    const unsigned long long t0 = clock64();
    for (int i = 0; i < NITER; ++i) {
      const uint32_t kk = (uint32_t)(i & 3);
      if (A_TMEM) {
        asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                     "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}"
                     ::"r"(d_t), "r"(a_t + kk * 8), "l"(bd + (((B_MN ? kk * 2048 : kk * 32)) >> 4)), "r"(id), "r"(1u),
                     "r"(0u), "r"(0u), "r"(0u), "r"(0u) : "memory");
      } else {
        asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                     "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
                     ::"r"(d_t), "l"(ad + ((kk * 32) >> 4)), "l"(bd + (((B_MN ? kk * 2048 : kk * 32)) >> 4)), "r"(id),
                     "r"(1u) : "memory");
      }
    }
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 ::"r"(smem_u32(&bar)) : "memory");
    // bounded wait: gives up after ~2 s (4e9 cycles at ~2 GHz)
    uint32_t done = 0;
    while (!done && clock64() - t0 < 4000000000ull) {
      asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0;\n\t"
                   "selp.u32 %0, 1, 0, p;\n\t}" : "=r"(done) : "r"(smem_u32(&bar)) : "memory");
    }
    const unsigned long long t1 = clock64();
    if (!done) atomicOr(status, 1);
    out[blockIdx.x] = t1 - t0;
  }
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
  }
}

template <int M, int N, bool A_TMEM, bool B_MN>
static void run(const char* name, int ctas) {
  unsigned long long* d;
  int* st;
  cudaMalloc(&d, ctas * sizeof(unsigned long long));
  cudaMalloc(&st, sizeof(int));
  cudaMemset(st, 0, sizeof(int));
  const size_t smem = 1024 + M * 128 + (N / 64) * 8192 + 1024;
  cudaFuncSetAttribute(probe<M, N, A_TMEM, B_MN>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  probe<M, N, A_TMEM, B_MN><<<ctas, 128, smem>>>(d, st);
  cudaError_t e = cudaDeviceSynchronize();
  unsigned long long h[256] = {0};
  int hs = 0;
  cudaMemcpy(h, d, ctas * sizeof(unsigned long long), cudaMemcpyDeviceToHost);
  cudaMemcpy(&hs, st, sizeof(int), cudaMemcpyDeviceToHost);
  unsigned long long mx = 0;
  for (int i = 0; i < ctas; ++i) mx = h[i] > mx ? h[i] : mx;
  const double cyc = (double)mx / NITER, flop = 2.0 * M * N * 16;
  printf("%-22s ctas=%3d  %7.1f cycles/mma  %6.0f flop/clk/SM  status=%d err=%s\n", name, ctas, cyc,
         flop / cyc, hs, cudaGetErrorString(e));
  cudaFree(d);
  cudaFree(st);
}

// One MLA decode chunk's MMA sequence, back to back, NCHUNK times: the QK
// step (36 x M64 N64 K16, A = Q from TMEM lane half 0 at 36 column offsets,
// B = a K-major 64-token tile over 9 column blocks) then the P.V step
// (4 k-steps x 2 output halves of M64 N256 K16, A = P K-major in shared
// memory, B = the tile read MN-major, D = O in lane half 1) -- the
// instruction mix of mla_decode_kernel.  COMMITS > 0 adds the kernel's
// per-chunk tcgen05.commit calls (1: after QK; 2: also two after P.V) to
// mbarriers nobody waits on, to see whether commits stall the pipe.
#define NCHUNK 64
template <int COMMITS>
__global__ void __launch_bounds__(128, 1) mla_chunk_probe(unsigned long long* out, int* status) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  __shared__ uint64_t bar, dummy[3];
  __shared__ uint32_t tslot;
  const int warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < (73728 + 8192) / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(smem)[i] = make_uint4(0, 0, 0, 0);
  if (threadIdx.x == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&bar)));
    for (int k = 0; k < 3; ++k)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&dummy[k])));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(&tslot)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tslot;
  if (threadIdx.x == 0) {
    const uint32_t kv = smem_u32(smem), pt = kv + 73728;
    const uint32_t id_qk = idesc(64, 64, false), id_pv = idesc(64, 256, true);
    const uint32_t t_s = tmem, t_q = tmem + 128, t_o = tmem + (16u << 16);
    const uint64_t bq0 = desc_sw128(kv, 16, 1024), bv0 = desc_sw128(kv, 64 * 128, 1024);
    const uint64_t pd0 = desc_sw128(pt, 16, 1024);
    const unsigned long long t0 = clock64();
    for (int c = 0; c < NCHUNK; ++c) {
      for (int kk = 0; kk < 36; ++kk) {
        const int cb = kk >> 2, ko = (kk & 3) * 32;
        const uint64_t bd = bq0 + (uint64_t)((cb * 8192 + ko) >> 4);
        asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                     "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}"
                     ::"r"(t_s), "r"(t_q + kk * 8), "l"(bd), "r"(id_qk), "r"((uint32_t)(kk > 0)),
                     "r"(0u), "r"(0u), "r"(0u), "r"(0u) : "memory");
      }
      if (COMMITS >= 1)
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                     ::"r"(smem_u32(&dummy[0])) : "memory");
      for (int j = 0; j < 8; ++j) {
        const int ks = j >> 1, hv = j & 1;
        const uint64_t ad = pd0 + (uint64_t)((ks * 32) >> 4);
        const uint64_t bd = bv0 + (uint64_t)((hv * 4 * 8192 + ks * 16 * 128) >> 4);
        asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                     "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
                     ::"r"(t_o + (uint32_t)(hv * 256)), "l"(ad), "l"(bd), "r"(id_pv), "r"(1u) : "memory");
      }
      if (COMMITS >= 2) {
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                     ::"r"(smem_u32(&dummy[1])) : "memory");
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                     ::"r"(smem_u32(&dummy[2])) : "memory");
      }
    }
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 ::"r"(smem_u32(&bar)) : "memory");
    uint32_t done = 0;
    while (!done && clock64() - t0 < 4000000000ull) {
      asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0;\n\t"
                   "selp.u32 %0, 1, 0, p;\n\t}" : "=r"(done) : "r"(smem_u32(&bar)) : "memory");
    }
    const unsigned long long t1 = clock64();
    if (!done) atomicOr(status, 1);
    out[blockIdx.x] = t1 - t0;
  }
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
  }
}

template <int COMMITS>
static void run_chunk(const char* name, int ctas) {
  unsigned long long* d;
  int* st;
  cudaMalloc(&d, ctas * sizeof(unsigned long long));
  cudaMalloc(&st, sizeof(int));
  cudaMemset(st, 0, sizeof(int));
  const size_t smem = 1024 + 73728 + 8192 + 1024;
  cudaFuncSetAttribute(mla_chunk_probe<COMMITS>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  mla_chunk_probe<COMMITS><<<ctas, 128, smem>>>(d, st);
  cudaError_t e = cudaDeviceSynchronize();
  unsigned long long h[256] = {0};
  int hs = 0;
  cudaMemcpy(h, d, ctas * sizeof(unsigned long long), cudaMemcpyDeviceToHost);
  cudaMemcpy(&hs, st, sizeof(int), cudaMemcpyDeviceToHost);
  unsigned long long mx = 0;
  for (int i = 0; i < ctas; ++i) mx = h[i] > mx ? h[i] : mx;
  printf("%-26s ctas=%3d  %7.1f cycles/chunk  status=%d err=%s\n", name, ctas,
         (double)mx / NCHUNK, hs, cudaGetErrorString(e));
  cudaFree(d);
  cudaFree(st);
}

int main() {
  run_chunk<0>("MLA chunk, no commits", 148);
  run_chunk<1>("MLA chunk, commit after QK", 148);
  run_chunk<2>("MLA chunk, 3 commits", 148);
  for (int ctas : {1, 148}) {
    run<64, 64, false, false>("M64 N64 SS Bk", ctas);
    run<64, 64, true, false>("M64 N64 TS Bk", ctas);
    run<64, 128, false, false>("M64 N128 SS Bk", ctas);
    run<64, 256, false, false>("M64 N256 SS Bk", ctas);
    run<64, 256, true, false>("M64 N256 TS Bk", ctas);
    run<64, 256, false, true>("M64 N256 SS Bmn", ctas);
    run<128, 64, false, false>("M128 N64 SS Bk", ctas);
    run<128, 64, true, false>("M128 N64 TS Bk", ctas);
    run<128, 64, false, true>("M128 N64 SS Bmn", ctas);
    run<128, 128, false, false>("M128 N128 SS Bk", ctas);
    run<128, 128, true, false>("M128 N128 TS Bk", ctas);
    run<128, 128, false, true>("M128 N128 SS Bmn", ctas);
    run<128, 256, false, false>("M128 N256 SS Bk", ctas);
    run<128, 256, true, false>("M128 N256 TS Bk", ctas);
    run<128, 256, false, true>("M128 N256 SS Bmn", ctas);
  }
  return 0;
}
