// Shared device helpers for the sm_100a stochastic-computing matmul.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "scmp_b200.h"

namespace scmp {

// Kernels launched by the library (scmp_launch_count); every launch site
// counts itself.
inline std::atomic<unsigned long long> g_launches{0};
inline void count_launch(unsigned long long n = 1) { g_launches.fetch_add(n, std::memory_order_relaxed); }

// ---------------------------------------------------------------------------
// IEEE float32, one rounding per operation. The intrinsics keep nvcc from
// contracting a multiply and an add into an FMA, which would change results
// relative to the reference (Triton interpreter / torch CPU kernels).
// ---------------------------------------------------------------------------
__device__ __forceinline__ float fmul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float fadd(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float fsub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float fdiv(float a, float b) { return __fdiv_rn(a, b); }
// round half to even (libdevice nearbyint / torch.round)
__device__ __forceinline__ float frint(float x) { return rintf(x); }
__device__ __forceinline__ float fclamp(float x, float lo, float hi) { return fminf(fmaxf(x, lo), hi); }

// Order-preserving map float -> int32 for atomicMax/atomicMin on floats.
__device__ __forceinline__ int f2ord(float f) {
  int i = __float_as_int(f);
  return i >= 0 ? i : i ^ 0x7FFFFFFF;
}
__device__ __forceinline__ float ord2f(int i) { return __int_as_float(i >= 0 ? i : i ^ 0x7FFFFFFF); }

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_min(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
// Sums of exact integers (< 2^24): any order gives the same float.
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Device-side error record (first error wins); read and cleared by
// scmp_device_error(). Kernels never trap: they record and return.
struct DeviceError {
  int code;
  int where;
};
// Defined here: the library is a single translation unit (scmp_b200.cu).
__device__ DeviceError g_device_error = {0, 0};

__device__ __forceinline__ void record_error(int code, int where) {
  if (atomicCAS(&g_device_error.code, 0, code) == 0) g_device_error.where = where;
}

// Longest legitimate device-side wait, in SM clock cycles (~2 s at 1.9 GHz).
constexpr long long kWaitLimitCycles = 4000000000LL;

// ---------------------------------------------------------------------------
// mbarrier helpers (shared::cta addresses as 32-bit integers)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(bar)
               : "memory");
}
// The waiting thread may be suspended until the phase completes or
// kSuspendHintNs nanoseconds pass, so that waiting warps do not take issue
// slots from the working ones.
constexpr uint32_t kSuspendHintNs = 1000000;
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "n"(kSuspendHintNs)
      : "memory");
  return ok != 0;
}
// Bounded wait: returns false (after recording SCMP_ERR_TIMEOUT) if the phase
// did not complete within kWaitLimitCycles or another role raised `abort`.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                          int where) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (clock64() - t0 > kWaitLimitCycles) {
      record_error(SCMP_ERR_TIMEOUT, where);
      *abort_flag = 1;
      return false;
    }
  }
}

__host__ __device__ __forceinline__ int cdiv(int a, int b) { return (a + b - 1) / b; }

}  // namespace scmp
