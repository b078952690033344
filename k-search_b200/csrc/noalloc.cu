// kq_gemm_f32act_noalloc: the fused fp32-activation GEMM without any device
// allocation.
//
// Who needs it: callers that may not call cudaMalloc at all, for example an
// inference server whose allocator has already reserved nearly all of HBM for
// its KV cache and weights (a cudaMalloc would fail or fragment its pool), a
// runtime that plans every byte of device memory before serving starts, or
// code running where a first-call allocation would synchronise the device in
// the middle of a latency-critical step. kq_gemm_f32act keeps its activation
// staging in a per-device buffer it grows with cudaMalloc; this entry point
// uses a fixed, statically sized array instead.
//
// The scratch below is a file-scope __device__ array, so every GPU that loads
// libkq holds it (kNoAllocScratchBytes plus one int) until the process exits.
// Host code cannot use the array's name as a device address (on the host it
// names a host-side stand-in), so the first call on each device, with that
// device current, resolves the device addresses with cudaGetSymbolAddress and
// caches them; make that first call before any stream capture. Every call
// shares the array and it keeps the last call's contents: the quantiser
// overwrites every staging byte a call reads, and the error word the kernels
// record timeouts in is cleared at the start of each call; two calls whose
// executions overlap on the GPU (different streams, no ordering between
// them) race on both.
#include <cstdio>
#include <mutex>

#include "kq_internal.h"

namespace kq {
namespace {

constexpr size_t kNoAllocScratchBytes = 1u << 20;  // activation staging limit (1 MiB)

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];
static __device__ int g_noalloc_error;  // device error word of the kernels launched from here

constexpr int kMaxDev = 64;
struct NoAllocPtrs {
  void* scratch = nullptr;
  int* err = nullptr;
};
NoAllocPtrs g_ptrs[kMaxDev];
std::mutex g_ptrs_mu;

kq_status_t device_ptrs(NoAllocPtrs* out) {
  int dev = 0;
  kq_status_t st = check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  if (st) return st;
  if (dev < 0 || dev >= kMaxDev) return fail(KQ_ERR_INVALID, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_ptrs_mu);
  NoAllocPtrs& p = g_ptrs[dev];
  if (!p.scratch) {
    void* s = nullptr;
    void* e = nullptr;
    st = check_cuda(cudaGetSymbolAddress(&s, g_noalloc_scratch), "cudaGetSymbolAddress(scratch)");
    if (st) return st;
    st = check_cuda(cudaGetSymbolAddress(&e, g_noalloc_error), "cudaGetSymbolAddress(error word)");
    if (st) return st;
    p.err = static_cast<int*>(e);
    p.scratch = s;
  }
  *out = p;
  return KQ_OK;
}

}  // namespace
}  // namespace kq

using namespace kq;

extern "C" kq_status_t kq_gemm_f32act_noalloc(int wtype, const void* w, const float* x, float* out, int M, int N,
                                              int K, int act_mode, kq_stream_t stream) {
  if (block_bytes(wtype) == 0) return fail(KQ_ERR_INVALID, "unknown weight type %d", wtype);
  if (M < 0 || N < 0 || K < 0 || K % 32 != 0)
    return fail(KQ_ERR_INVALID, "bad shape M=%d N=%d K=%d (K must be a multiple of 32)", M, N, K);
  if (act_mode < KQ_ACT_SUM_X || act_mode > KQ_ACT_F32) return fail(KQ_ERR_INVALID, "unknown activation mode %d", act_mode);
  if ((long long)M * N == 0 || K == 0) {
    if ((long long)M * N > 0)  // K == 0: the product is zero
      return check_cuda(cudaMemsetAsync(out, 0, sizeof(float) * (size_t)M * N, static_cast<cudaStream_t>(stream)),
                        "zero output");
    return KQ_OK;
  }
  if (!w || !x || !out) return fail(KQ_ERR_INVALID, "null pointer");
  if ((reinterpret_cast<uintptr_t>(x) & 15) != 0) return fail(KQ_ERR_INVALID, "activations must be 16-byte aligned");
  const size_t need = act8_bytes(M, K);
  if (need > kNoAllocScratchBytes)
    return fail(KQ_ERR_INVALID,
                "kq_gemm_f32act_noalloc: activation staging of %zu bytes (M=%d, K=%d) exceeds the fixed %zu-byte "
                "scratch; use kq_gemm_f32act",
                need, M, K, kNoAllocScratchBytes);
  NoAllocPtrs p;
  kq_status_t st = device_ptrs(&p);
  if (st) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  st = check_cuda(cudaMemsetAsync(p.err, 0, sizeof(int), s), "clear the no-alloc error word");
  if (st) return st;
  // one activation row with 4-bit weights: the single-launch GEMV needs no
  // staging at all (the same kernel kq_gemm_f32act runs for this shape)
  if (gemv1_supported(wtype, M, N, K, w, x)) return launch_gemv1(wtype, w, x, OutSpec::plain(out, N), N, K, act_mode, s, p.err);
  Act8 act = act8_view(p.scratch, M, K);
  st = launch_quantize_act(x, act, M, K, act_mode, s);
  if (st) return st;
  if (gemv_supported(wtype, M, N, K) && (reinterpret_cast<uintptr_t>(w) & 15) == 0)
    return launch_gemv(wtype, w, act, out, M, N, K, true, s, p.err);
  if (gemm_tc_supported(wtype, M, N, K, w, act)) return launch_gemm_tc(wtype, w, act, out, M, N, K, true, s, p.err);
  return launch_gemm_simt(wtype, w, act, out, M, N, K, s);
}

// The error word of kq_gemm_f32act_noalloc's kernels, read without any
// allocation (kq_device_error reads the library's own word, which it
// allocates on first use). Reads it on `stream`, synchronises that stream,
// and clears a non-zero word.
extern "C" kq_status_t kq_noalloc_device_error(int* code, kq_stream_t stream) {
  if (!code) return fail(KQ_ERR_INVALID, "null code pointer");
  NoAllocPtrs p;
  kq_status_t st = device_ptrs(&p);
  if (st) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int v = 0;
  st = check_cuda(cudaMemcpyAsync(&v, p.err, sizeof(int), cudaMemcpyDeviceToHost, s), "read the no-alloc error word");
  if (st) return st;
  st = check_cuda(cudaStreamSynchronize(s), "sync");
  if (st) return st;
  *code = v;
  if (v) return check_cuda(cudaMemsetAsync(p.err, 0, sizeof(int), s), "clear the no-alloc error word");
  return KQ_OK;
}
