// Device-side building blocks shared by the attention kernels (sm_100a).
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "tla_api.h"

namespace tla {

// A bounded in-kernel wait gives up after this long and reports TLA_ERR_TIMEOUT.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void report_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

// Bounds-check builds (-DTLA_BOUNDS_CHECK): a guarded global index is checked
// against its buffer's extent; a bad one records TLA_ERR_BOUNDS and the access
// is skipped, with control flow and barriers unchanged. Other builds compile
// the guard to `true`.
#ifdef TLA_BOUNDS_CHECK
__device__ __forceinline__ bool in_bounds_checked(long long i, long long n, int* err) {
  if (i >= 0 && i < n) return true;
  report_error(err, TLA_ERR_BOUNDS);
  return false;
}
#define TLA_IN_BOUNDS(i, n, err) ::tla::in_bounds_checked(static_cast<long long>(i), static_cast<long long>(n), (err))
#else
#define TLA_IN_BOUNDS(i, n, err) true
#endif

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// try_wait suspends the thread until the phase completes or the hinted time
// (ns) passes, so waiting warps do not flood the shared-memory pipe.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u)
      : "memory");
  return ok != 0;
}
// Waits for the phase with the given parity; false (and TLA_ERR_TIMEOUT in
// *err) if it did not complete within kWaitLimitNs.
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity);
// The clock is read once every 64 polls: a waiting thread shares its
// sub-partition's issue slots with the compute warps, so its loop is kept short.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
  if (mbar_test_wait(bar, parity)) return true;  // already complete: no suspend round trip
  const unsigned long long t0 = globaltimer();
  for (;;) {
#pragma unroll 1
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer() - t0 > kWaitLimitNs) {
      report_error(err, TLA_ERR_TIMEOUT);
      return false;
    }
  }
}

// Non-blocking test of a phase (no suspension), and a bounded spin on it for
// the single-thread issuers whose next step is already due most of the time.
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_spin(uint64_t* bar, uint32_t parity, int* err) {
  if (mbar_test_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  for (;;) {
    if (mbar_test_wait(bar, parity)) return true;
    if (globaltimer() - t0 > kWaitLimitNs) {
      report_error(err, TLA_ERR_TIMEOUT);
      return false;
    }
  }
}

// Bounded poll with a short sleep between tests: for a single issuing thread
// whose sub-partition also runs issue-heavy warps.
__device__ __forceinline__ bool mbar_nap(uint64_t* bar, uint32_t parity, int* err) {
  if (mbar_test_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  for (;;) {
    __nanosleep(64);
    if (mbar_test_wait(bar, parity)) return true;
    if (globaltimer() - t0 > kWaitLimitNs) {
      report_error(err, TLA_ERR_TIMEOUT);
      return false;
    }
  }
}

// Programmatic dependent launch: wait for the preceding kernel in the stream
// (complete, memory visible); let the following kernel start its prologue.
// Both are no-ops for a kernel not launched with the PDL attribute.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- TMA (no multicast)
__device__ __forceinline__ void tma_prefetch(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------- warp-level MMA (decode)
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
// D = A(16x16, row) * B(16x8, col) + D, fp16 inputs, fp32 accumulators.
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// max(a, b, c) in one instruction (three-input max.f32, sm_100).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// 2^x with the hardware approximation (MUFU.EX2).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Byte offset of 16-byte chunk `chunk` (0..7) of row `row` in a tile written by
// TMA with CU_TENSOR_MAP_SWIZZLE_128B (128-byte rows, tile base 1024-aligned).
__device__ __forceinline__ uint32_t sw128(int row, int chunk) {
  return static_cast<uint32_t>(row * 128 + ((chunk ^ (row & 7)) << 4));
}

// ---------------------------------------------------------------- RoPE angle
// cos/sin of position * inv_freq. The product is exact in double (int32 x
// float32 fits in 53 bits), the reduction to [-pi, pi] is done in double, and
// only the reduced angle goes through sincosf, so large positions keep full
// float32 accuracy (the reference evaluates Math.cos/Math.sin in double).
__device__ __forceinline__ void rope_cos_sin(int position, float inv_freq, float* c, float* s) {
  const double a = static_cast<double>(position) * static_cast<double>(inv_freq);
  const double two_pi_hi = 6.283185307179586;             // 2*pi rounded to double
  const double two_pi_lo = 2.4492935982947064e-16;        // 2*pi - two_pi_hi
  const double k = rint(a * 0.15915494309189535);          // a / (2*pi)
  double r = fma(-k, two_pi_hi, a);
  r = fma(-k, two_pi_lo, r);
  sincosf(static_cast<float>(r), s, c);
}

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) {
  return __half2float(v);
}
template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) {
  return __float2half_rn(v);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ void named_barrier_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

}  // namespace tla
