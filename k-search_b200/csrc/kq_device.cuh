// Device-side helpers: block field extraction, mbarriers, bulk async copies,
// programmatic dependent launch. sm_100a only.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <utility>

namespace kq {

// Device error codes written to the error word (first writer wins).
enum DevErr : int { DEV_OK = 0, DEV_TIMEOUT_FULL = 1, DEV_TIMEOUT_EMPTY = 2, DEV_BAD_SHAPE = 3 };

__device__ __forceinline__ void record_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

// silu(g) * u as the MoE's SiLU quantiser forms it (kernels/activation/silu.cuh:97
// semantics); one definition so every kernel that needs h computes the same bits.
__device__ __forceinline__ float silu_mul(float g, float u) { return g / (1.0f + expf(-g)) * u; }

__device__ __forceinline__ float half_bits_to_float(uint32_t bits16) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16 & 0xFFFFu)));
}

__device__ __forceinline__ uint32_t float_to_half_bits(float f) {
  return static_cast<uint32_t>(__half_as_ushort(__float2half_rn(f)));
}

// ---- byte-window extraction ------------------------------------------------
// A lane holds a run of consecutive bytes in 32-bit words w[] (word 0 = bytes
// 0..3, little endian). These read a field at a compile-time byte offset.
template <int OFF, int NW>
__device__ __forceinline__ uint32_t get_u32(const uint32_t (&w)[NW]) {
  static_assert(OFF % 2 == 0, "fields are 2-byte aligned");
  if constexpr (OFF % 4 == 0) {
    return w[OFF / 4];
  } else {
    return __funnelshift_r(w[OFF / 4], w[OFF / 4 + 1], 16);
  }
}
template <int OFF, int NW>
__device__ __forceinline__ uint32_t get_u16(const uint32_t (&w)[NW]) {
  static_assert(OFF % 2 == 0, "fields are 2-byte aligned");
  if constexpr (OFF % 4 == 0) {
    return w[OFF / 4] & 0xFFFFu;
  } else {
    return w[OFF / 4] >> 16;
  }
}

// out[i] = 32-bit field at byte offset OFF + 4 i, i < N (compile-time offsets).
template <int OFF, int NW, int... I>
__device__ __forceinline__ void gather_u32_impl(const uint32_t (&w)[NW], uint32_t* out,
                                                std::integer_sequence<int, I...>) {
  ((out[I] = get_u32<OFF + 4 * I>(w)), ...);
}
template <int OFF, int N, int NW>
__device__ __forceinline__ void gather_u32(const uint32_t (&w)[NW], uint32_t (&out)[N]) {
  gather_u32_impl<OFF>(w, out, std::make_integer_sequence<int, N>{});
}

// ---- mbarrier --------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
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

// Non-suspending probe of a phase.
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

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait for the phase with the given parity to complete. Returns false
// (and records `code`) once kWaitLimitNs of wall time has passed: any legal
// wait in these kernels ends within microseconds. A short spin on the
// non-suspending probe comes first: a suspended try_wait resumes about 90
// cycles later than a spinning probe sees the phase complete, and most
// hand-offs here complete within a few hundred cycles.
constexpr uint64_t kWaitLimitNs = 2000000000ull;
constexpr int kSpinProbes = 32;
__device__ __forceinline__ bool mbar_wait_for(uint64_t* bar, uint32_t parity, int* err, int code,
                                              uint64_t limit_ns) {
#pragma unroll 1
  for (int i = 0; i < kSpinProbes; ++i)
    if (mbar_test_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 0 && globaltimer_ns() - t0 > limit_ns) {
      record_error(err, code);
      return false;
    }
  }
}
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
  return mbar_wait_for(bar, parity, err, code, kWaitLimitNs);
}

// Wait that never blocks again once one wait of this thread has timed out:
// after a timeout the kernel runs to completion on whatever data it has (the
// error word tells the host the output is invalid) instead of stalling at
// every later barrier.
__device__ __forceinline__ void mbar_wait_or_poison(uint64_t* bar, uint32_t parity, int* err, int code,
                                                    bool& dead) {
  if (!dead && !mbar_wait(bar, parity, err, code)) dead = true;
}

// The same bounded wait without the spinning probes: the thread suspends in
// try_wait from the start. For producer / issuer / converter threads that
// share an SM sub-partition with the warps doing the math: a spinning waiter
// takes issue slots from them.
__device__ __forceinline__ bool mbar_wait_idle(uint64_t* bar, uint32_t parity, int* err, int code) {
  if (mbar_try_wait(bar, parity)) return true;  // no timer read on the common path
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 0 && globaltimer_ns() - t0 > kWaitLimitNs) {
      record_error(err, code);
      return false;
    }
  }
}
__device__ __forceinline__ void mbar_wait_idle_or_poison(uint64_t* bar, uint32_t parity, int* err, int code,
                                                         bool& dead) {
  if (!dead && !mbar_wait_idle(bar, parity, err, code)) dead = true;
}

// Orders this thread's generic-proxy shared-memory accesses with later
// async-proxy ones (TMA / bulk copies, tensor-core operand reads): after
// writing an operand tile, and after reading a stage that a TMA refills once
// it is released.
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ---- bulk async copy global -> shared (this CTA only) -----------------------
// dst, src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Same, with an L2 eviction hint: streamed data that is read once.
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                              uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// ---- programmatic dependent launch -----------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- warp reductions ---------------------------------------------------------
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ---- named barriers ----------------------------------------------------------
__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

}  // namespace kq
