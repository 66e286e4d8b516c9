// common.cuh — sm_100a device helpers shared by the decode kernels:
// mbarrier pipeline primitives with bounded waits, TMA tile loads, packed
// conversions, and the workspace status word.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace b2d {

// Status bits OR-ed into the workspace status word by kernels.
constexpr int kStatusTimeout = 1;
constexpr int kStatusBounds = 2;

// By default a wait on an mbarrier gives up after this many nanoseconds of
// wall time (globaltimer).  No legitimate wait in these kernels comes near
// it: every wait is for a TMA copy already issued or for a stage the
// consumers release after a few microseconds of arithmetic.  Callers may
// pass a shorter limit per launch (b2d_gqa_args.wait_limit_us).
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

// Workspace header shared by every decode entry point: the status word
// (256 bytes), then the arrival counters of the in-kernel split merge
// (kMergeCounters int32, zero between calls).  Everything else follows.
constexpr size_t kStatusBytes = 256;
constexpr int kMergeCounters = 16384;
constexpr size_t kWsHeaderBytes = kStatusBytes + (size_t)kMergeCounters * 4;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: true when the phase with `parity` completed, false when the
// wall-time limit ran out (the caller then records kStatusTimeout and exits).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          unsigned long long limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > limit_ns) return false;
  }
  return true;
}

// Programmatic dependent launch.  A kernel launched with the
// programmatic-stream-serialization attribute may start while the previous
// kernel on the stream is still finishing; griddep_wait() blocks until that
// kernel has completed and its memory is visible, so it must come before
// the first read of any input or write of any output.  griddep_launch()
// lets the next such kernel start its own prologue early.  Both are no-ops
// for a kernel launched without the attribute.
__device__ __forceinline__ void griddep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void griddep_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}

// 4-D tiled TMA load (no multicast) into this CTA's shared memory; completion
// is signalled on `bar` as transaction bytes.  c0 (the innermost coordinate)
// is always 0 here, so the 16-byte rule on the x coordinate holds.
__device__ __forceinline__ void tma_load_4d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2, int c3, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cta.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar)),
      "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

__device__ __forceinline__ uint2 lds64(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}

// bf16x2 -> two fp32 (exact: bf16 is the top half of an fp32).
__device__ __forceinline__ float2 bf16x2_to_f2(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}

__device__ __forceinline__ float2 f16x2_to_f2(uint32_t w) {
  __half2 h = *reinterpret_cast<__half2*>(&w);
  return __half22float2(h);
}

// Two e4m3 bytes (in the low 16 bits of `w`, lowest byte first) -> fp16x2
// whose values are the e4m3 values times 2^-8.  e4m3 is s.eeee.mmm with bias
// 7, fp16 is s.eeeee.mmmmmmmmmm with bias 15: moving the 7 magnitude bits up
// by 7 and the sign up by 8 keeps every normal and subnormal e4m3 value
// exact, scaled by 2^(7-15) = 2^-8.  (The e4m3 NaN encoding maps to a
// finite value; caches written by a quantiser never hold it.)  The 2^8 is
// folded into the dequantisation scale by the caller.
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2_scaled(uint32_t w) {
  const uint32_t spread = __byte_perm(w, 0, 0x4140);  // (b1 << 16) | b0, as 16-bit lanes
  const uint32_t mag = (spread & 0x007f007fu) << 7;
  const uint32_t sgn = (spread & 0x00800080u) << 8;
  return mag | sgn;
}

// Two e4m3 bytes (low 16 bits of `w`) -> fp16x2 with the exact e4m3 values,
// by the hardware conversion instruction.
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2_cvt(uint32_t w) {
  uint32_t r;
  asm("{\n\t.reg .b16 lo;\n\tcvt.u16.u32 lo, %1;\n\tcvt.rn.f16x2.e4m3x2 %0, lo;\n\t}"
      : "=r"(r)
      : "r"(w));
  return r;
}

// atomicAdd with release + acquire semantics at GPU scope: writes this
// thread made before it (and, after a __syncwarp(), those of its warp) are
// visible to whoever observes the new value, and writes that the previous
// releasers made are visible to this thread afterwards.
__device__ __forceinline__ int atomic_add_acq_rel_gpu(int* addr, int v) {
  int old;
  asm volatile("atom.add.acq_rel.gpu.global.s32 %0, [%1], %2;" : "=r"(old) : "l"(addr), "r"(v)
               : "memory");
  return old;
}

__device__ __forceinline__ void record_status(int* status, int bits) {
  if (status != nullptr) atomicOr(status, bits);
}

}  // namespace b2d
