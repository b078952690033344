// libkq C ABI: argument checks, dispatch, per-device workspace, error state.
#include <atomic>
#include <cstdlib>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "kq_internal.h"

namespace kq {

namespace {
thread_local std::string g_last_error;

constexpr int kMaxDevices = 64;
struct DeviceState {
  void* ws[WS_NSLOTS] = {};
  size_t ws_size[WS_NSLOTS] = {};
  int* err_word = nullptr;
  std::atomic<int> sms{0};  // read without g_mu
};
DeviceState g_dev[kMaxDevices];
std::mutex g_mu;
}  // namespace

kq_status_t fail(kq_status_t st, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return st;
}

kq_status_t check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return KQ_OK;
  return fail(KQ_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

kq_status_t check_launch(const char* what) { return check_cuda(cudaGetLastError(), what); }

int current_device() {
  int d = 0;
  cudaGetDevice(&d);
  return d;
}

int sm_count() {
  const int d = current_device();
  if (d < 0 || d >= kMaxDevices) return 148;
  int n = g_dev[d].sms.load(std::memory_order_relaxed);
  if (n == 0) {
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d);
    if (n <= 0) n = 148;
    g_dev[d].sms.store(n, std::memory_order_relaxed);
  }
  return n;
}

void* workspace(WsSlot slot, size_t bytes) {
  const int d = current_device();
  if (d < 0 || d >= kMaxDevices) {
    fail(KQ_ERR_INVALID, "device ordinal %d out of range", d);
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(g_mu);
  DeviceState& st = g_dev[d];
  if (bytes == 0) bytes = 256;
  if (st.ws_size[slot] >= bytes) return st.ws[slot];
  size_t grow = bytes + bytes / 4;
  grow = (grow + (1u << 20) - 1) & ~(size_t)((1u << 20) - 1);
  if (st.ws[slot]) {
    cudaFree(st.ws[slot]);  // implicitly synchronises the device
    st.ws[slot] = nullptr;
    st.ws_size[slot] = 0;
  }
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, grow);
  if (e != cudaSuccess) {
    cudaGetLastError();
    fail(KQ_ERR_NOMEM, "workspace allocation of %zu bytes failed: %s", grow, cudaGetErrorString(e));
    return nullptr;
  }
  st.ws[slot] = p;
  st.ws_size[slot] = grow;
  return p;
}

int* device_error_word() {
  const int d = current_device();
  if (d < 0 || d >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  DeviceState& st = g_dev[d];
  if (!st.err_word) {
    if (cudaMalloc(&st.err_word, sizeof(int)) != cudaSuccess) {
      cudaGetLastError();
      st.err_word = nullptr;
      return nullptr;
    }
    cudaMemset(st.err_word, 0, sizeof(int));
  }
  return st.err_word;
}

namespace {
struct SmemAttr {
  int dev;
  const void* func;
  int bytes;
};
std::vector<SmemAttr> g_smem_attrs;  // guarded by g_mu
}  // namespace

kq_status_t ensure_dynamic_smem(const void* func, int bytes, const char* what) {
  const int d = current_device();
  std::lock_guard<std::mutex> lk(g_mu);
  for (const SmemAttr& a : g_smem_attrs)
    if (a.dev == d && a.func == func && a.bytes >= bytes) return KQ_OK;
  kq_status_t st = check_cuda(cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes), what);
  if (st) return st;
  g_smem_attrs.push_back(SmemAttr{d, func, bytes});
  return KQ_OK;
}

void* tensor_map_encoder() {
  static void* fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* f = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = f;
    else
      cudaGetLastError();
  });
  return fn;
}

namespace {

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

kq_status_t check_gemm_args(int wtype, const void* w, const void* a, const float* out, int M, int N, int K) {
  if (block_bytes(wtype) == 0) return fail(KQ_ERR_INVALID, "unknown weight type %d", wtype);
  if (M < 0 || N < 0 || K < 0) return fail(KQ_ERR_INVALID, "negative dimension (M=%d N=%d K=%d)", M, N, K);
  if (K % 32 != 0) return fail(KQ_ERR_INVALID, "K=%d is not a multiple of 32", K);
  if ((long long)M * N > 0 && K > 0 && (!w || !a || !out)) return fail(KQ_ERR_INVALID, "null pointer");
  return KQ_OK;
}

// Quantised activations are staged; choose the GEMM kernel for the shape.
// M > 8 path: the warp-MMA skinny kernel for 8 < M <= 16 (measured faster
// than the split kernel there: 30.6 against 46.1 us at M=16, 30.5 against
// 57.6 at M=9, N=14336 K=4096 q4_0; from M=24 the split kernel is faster,
// 47 against 49 us), the exact split-fp16 tcgen05 kernel
// above; KQ_GEMM_PATH=int8 runs the int8 tcgen05 kernel (per-block int32
// sums rescaled on the FP32 pipe) for every M > 8, KQ_GEMM_PATH=skinny the
// skinny kernel up to its limit of 128 rows. Read once per process.
enum class GemmPath { kDefault, kSkinny, kInt8 };
GemmPath gemm_path() {
  static const GemmPath p = [] {
    const char* e = std::getenv("KQ_GEMM_PATH");
    if (e && std::string(e) == "int8") return GemmPath::kInt8;
    if (e && std::string(e) == "skinny") return GemmPath::kSkinny;
    return GemmPath::kDefault;
  }();
  return p;
}
constexpr int kSkinnyDefaultMaxM = 16;
bool use_skinny(int M) {
  const GemmPath p = gemm_path();
  return p == GemmPath::kSkinny || (p == GemmPath::kDefault && M <= kSkinnyDefaultMaxM);
}

// The tensor-core kernel for M > 8 with the given output destinations, or
// KQ_ERR_UNSUPPORTED when none fits the shape.
kq_status_t dispatch_gemm_tc(int wtype, const void* w, Act8 act, const OutSpec& out, int M, int N, int K,
                             cudaStream_t s, bool pdl) {
  const GemmPath path = gemm_path();
  if (use_skinny(M) && gemm_skinny_supported(wtype, M, N, K, w, act))
    return launch_gemm_skinny(wtype, w, act, out, M, N, K, s);
  if (path != GemmPath::kInt8 && gemm_split_supported(wtype, M, N, K, w, act))
    return launch_gemm_split(wtype, w, act, out, M, N, K, s);
  if (gemm_tc_supported(wtype, M, N, K, w, act)) return launch_gemm_tc(wtype, w, act, out, M, N, K, pdl, s);
  return fail(KQ_ERR_UNSUPPORTED, "no tensor-core GEMM for M=%d N=%d K=%d", M, N, K);
}

bool gemm_tc_any_supported(int wtype, int M, int N, int K, const void* w, Act8 act) {
  return (use_skinny(M) && gemm_skinny_supported(wtype, M, N, K, w, act)) ||
         (gemm_path() != GemmPath::kInt8 && gemm_split_supported(wtype, M, N, K, w, act)) ||
         gemm_tc_supported(wtype, M, N, K, w, act);
}

kq_status_t dispatch_gemm(int wtype, const void* w, Act8 act, float* out, int M, int N, int K, cudaStream_t s,
                          bool pdl) {
  if (gemv_supported(wtype, M, N, K) && aligned(w, 16)) return launch_gemv(wtype, w, act, out, M, N, K, pdl, s);
  if (gemm_tc_any_supported(wtype, M, N, K, w, act))
    return dispatch_gemm_tc(wtype, w, act, OutSpec::plain(out, N), M, N, K, s, pdl);
  return launch_gemm_simt(wtype, w, act, out, M, N, K, s);
}

}  // namespace

kq_status_t gemm_any(int wtype, const void* w, Act8 act, float* out, int M, int N, int K, cudaStream_t s) {
  return dispatch_gemm(wtype, w, act, out, M, N, K, s, false);
}

namespace {

kq_status_t zero_output(float* out, int M, int N, cudaStream_t s) {
  if ((long long)M * N == 0) return KQ_OK;
  return check_cuda(cudaMemsetAsync(out, 0, sizeof(float) * (size_t)M * N, s), "zero output");
}

}  // namespace
}  // namespace kq

using namespace kq;

extern "C" {

int kq_abi_version(void) { return 1; }

const char* kq_last_error(void) { return g_last_error.c_str(); }

size_t kq_block_bytes(int wtype) { return (size_t)block_bytes(wtype); }

kq_status_t kq_device_error(int* code, kq_stream_t stream) {
  if (!code) return fail(KQ_ERR_INVALID, "null code pointer");
  int* w = device_error_word();
  if (!w) return fail(KQ_ERR_NOMEM, "device error word unavailable");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int v = 0;
  kq_status_t st = check_cuda(cudaMemcpyAsync(&v, w, sizeof(int), cudaMemcpyDeviceToHost, s), "read error word");
  if (st) return st;
  st = check_cuda(cudaStreamSynchronize(s), "sync");
  if (st) return st;
  *code = v;
  if (v) return check_cuda(cudaMemsetAsync(w, 0, sizeof(int), s), "clear error word");
  return KQ_OK;
}

kq_status_t kq_quantize_q8_1(const float* x, void* y, int64_t M, int64_t K, int sum_mode, kq_stream_t stream) {
  if (M < 0 || K < 0 || K % 32 != 0) return fail(KQ_ERR_INVALID, "quantize_q8_1: bad shape M=%lld K=%lld", (long long)M, (long long)K);
  if (M * K == 0) return KQ_OK;
  if (!x || !y) return fail(KQ_ERR_INVALID, "quantize_q8_1: null pointer");
  if (!aligned(x, 16) || !aligned(y, 4)) return fail(KQ_ERR_INVALID, "quantize_q8_1: x must be 16-byte and y 4-byte aligned");
  return launch_quantize_q8_1_bytes(x, y, M, K, sum_mode, static_cast<cudaStream_t>(stream));
}

kq_status_t kq_quantize_rows(int wtype, const float* x, void* y, int64_t rows, int64_t K, kq_stream_t stream) {
  if (block_bytes(wtype) == 0) return fail(KQ_ERR_INVALID, "unknown weight type %d", wtype);
  if (rows < 0 || K < 0 || K % 32 != 0) return fail(KQ_ERR_INVALID, "quantize_rows: bad shape rows=%lld K=%lld", (long long)rows, (long long)K);
  if (rows * K == 0) return KQ_OK;
  if (!x || !y || !aligned(y, 2)) return fail(KQ_ERR_INVALID, "quantize_rows: null or misaligned pointer");
  return launch_quantize_rows(wtype, x, y, rows, K, static_cast<cudaStream_t>(stream));
}

kq_status_t kq_mul_mat_q(int wtype, const void* w, const void* a_q8_1, float* out, int M, int N, int K,
                         kq_stream_t stream) {
  kq_status_t st = check_gemm_args(wtype, w, a_q8_1, out, M, N, K);
  if (st) return st;
  if ((long long)M * N == 0) return KQ_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (K == 0) return zero_output(out, M, N, s);
  if (!aligned(a_q8_1, 4)) return fail(KQ_ERR_INVALID, "q8_1 activations must be 4-byte aligned");
  void* ws = workspace(WS_ACT, act8_bytes(M, K));
  if (!ws) return KQ_ERR_NOMEM;
  Act8 act = act8_view(ws, M, K);
  st = launch_q8_1_to_act(a_q8_1, act, M, K, s);
  if (st) return st;
  return dispatch_gemm(wtype, w, act, out, M, N, K, s, true);
}

kq_status_t kq_gemm_f32act(int wtype, const void* w, const float* x, float* out, int M, int N, int K, int act_mode,
                           kq_stream_t stream) {
  kq_status_t st = check_gemm_args(wtype, w, x, out, M, N, K);
  if (st) return st;
  if (act_mode < KQ_ACT_SUM_X || act_mode > KQ_ACT_F32) return fail(KQ_ERR_INVALID, "unknown activation mode %d", act_mode);
  if ((long long)M * N == 0) return KQ_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (K == 0) return zero_output(out, M, N, s);
  if (!aligned(x, 16)) return fail(KQ_ERR_INVALID, "activations must be 16-byte aligned");
  // one activation row, 4-bit weights: one launch that quantises the row itself
  if (gemv1_supported(wtype, M, N, K, w, x)) return launch_gemv1(wtype, w, x, OutSpec::plain(out, N), N, K, act_mode, s);
  void* ws = workspace(WS_ACT, act8_bytes(M, K));
  if (!ws) return KQ_ERR_NOMEM;
  Act8 act = act8_view(ws, M, K);
  st = launch_quantize_act(x, act, M, K, act_mode, s);
  if (st) return st;
  return dispatch_gemm(wtype, w, act, out, M, N, K, s, true);
}

kq_status_t kq_rms_norm_f32(const float* x, const float* weight, float* out, int M, int K, float eps,
                            kq_stream_t stream) {
  if (M < 0 || K < 0) return fail(KQ_ERR_INVALID, "rms_norm: negative dimension (M=%d K=%d)", M, K);
  if ((long long)M * K == 0) return KQ_OK;
  if (!x || !weight || !out) return fail(KQ_ERR_INVALID, "rms_norm: null pointer");
  if (!(eps >= 0.0f)) return fail(KQ_ERR_INVALID, "rms_norm: eps must be >= 0");
  return launch_rms_norm(x, weight, out, M, K, eps, static_cast<cudaStream_t>(stream));
}

namespace {
kq_status_t check_norm_quant_args(const float* x, const float* weight, int M, int K, float eps) {
  if (M < 0 || K < 0 || K % 32) return fail(KQ_ERR_INVALID, "rms_norm_quantize: bad shape M=%d K=%d (K %% 32 == 0)", M, K);
  if ((long long)M * K > 0 && (!x || !weight)) return fail(KQ_ERR_INVALID, "rms_norm_quantize: null pointer");
  if (!aligned(x, 16) || !aligned(weight, 16))
    return fail(KQ_ERR_INVALID, "rms_norm_quantize: x and weight must be 16-byte aligned");
  if (!(eps >= 0.0f)) return fail(KQ_ERR_INVALID, "rms_norm_quantize: eps must be >= 0");
  return KQ_OK;
}
}  // namespace

kq_status_t kq_rms_norm_quantize_q8_1(const float* x, const float* weight, void* y, int M, int K, float eps,
                                      int sum_mode, kq_stream_t stream) {
  kq_status_t st = check_norm_quant_args(x, weight, M, K, eps);
  if (st) return st;
  if (sum_mode != KQ_ACT_SUM_X && sum_mode != KQ_ACT_SUM_DQ)
    return fail(KQ_ERR_INVALID, "q8_1 bytes hold fp16 d and s: sum_mode must be KQ_ACT_SUM_X or KQ_ACT_SUM_DQ");
  if ((long long)M * K == 0) return KQ_OK;
  if (!y) return fail(KQ_ERR_INVALID, "rms_norm_quantize: null output");
  return launch_rms_norm_quantize(x, weight, eps, Act8{nullptr, nullptr}, y, M, K, sum_mode,
                                  static_cast<cudaStream_t>(stream));
}

kq_status_t kq_gemm_f32act_rmsnorm(int wtype, const void* w, const float* x, const float* norm_weight, float eps,
                                   float* out, int M, int N, int K, int act_mode, kq_stream_t stream) {
  kq_status_t st = check_gemm_args(wtype, w, x, out, M, N, K);
  if (st) return st;
  if (act_mode < KQ_ACT_SUM_X || act_mode > KQ_ACT_F32) return fail(KQ_ERR_INVALID, "unknown activation mode %d", act_mode);
  st = check_norm_quant_args(x, norm_weight, M, K, eps);
  if (st) return st;
  if ((long long)M * N == 0) return KQ_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (K == 0) return zero_output(out, M, N, s);
  void* ws = workspace(WS_ACT, act8_bytes(M, K));
  if (!ws) return KQ_ERR_NOMEM;
  Act8 act = act8_view(ws, M, K);
  st = launch_rms_norm_quantize(x, norm_weight, eps, act, nullptr, M, K, act_mode, s);
  if (st) return st;
  return dispatch_gemm(wtype, w, act, out, M, N, K, s, true);
}

kq_status_t kq_peer_alloc(size_t bytes, void** ptr, void* handle64) {
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  if (!ptr || !handle64 || bytes == 0) return fail(KQ_ERR_INVALID, "peer_alloc: bad arguments");
  *ptr = nullptr;
  void* p = nullptr;
  kq_status_t st = check_cuda(cudaMalloc(&p, bytes), "peer_alloc cudaMalloc");
  if (st) return st;
  cudaIpcMemHandle_t h;
  st = check_cuda(cudaIpcGetMemHandle(&h, p), "cudaIpcGetMemHandle");
  if (st) {
    cudaFree(p);
    return st;
  }
  std::memcpy(handle64, &h, sizeof(h));
  *ptr = p;
  return KQ_OK;
}

kq_status_t kq_peer_open(const void* handle64, void** ptr) {
  if (!ptr || !handle64) return fail(KQ_ERR_INVALID, "peer_open: bad arguments");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle64, sizeof(h));
  return check_cuda(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
}

kq_status_t kq_peer_close(void* ptr) { return check_cuda(cudaIpcCloseMemHandle(ptr), "cudaIpcCloseMemHandle"); }

kq_status_t kq_peer_free(void* ptr) { return check_cuda(cudaFree(ptr), "peer_free cudaFree"); }

kq_status_t kq_copy_2d(void* dst, size_t dst_pitch, const void* src, size_t src_pitch, size_t width_bytes,
                       size_t height, kq_stream_t stream) {
  if (width_bytes == 0 || height == 0) return KQ_OK;
  if (!dst || !src || width_bytes > dst_pitch || width_bytes > src_pitch) return fail(KQ_ERR_INVALID, "copy_2d: bad arguments");
  return check_cuda(cudaMemcpy2DAsync(dst, dst_pitch, src, src_pitch, width_bytes, height, cudaMemcpyDeviceToDevice,
                                      static_cast<cudaStream_t>(stream)),
                    "cudaMemcpy2DAsync");
}

kq_status_t kq_gemm_f32act_scatter(int wtype, const void* w, const float* x, float* const* outs, int n_out, int ldo,
                                   int col0, int M, int N, int K, int act_mode, kq_stream_t stream) {
  if (n_out < 1 || n_out > kMaxOut || !outs) return fail(KQ_ERR_INVALID, "scatter: n_out=%d (1..%d)", n_out, kMaxOut);
  kq_status_t st = check_gemm_args(wtype, w, x, outs[0], M, N, K);
  if (st) return st;
  if (act_mode < KQ_ACT_SUM_X || act_mode > KQ_ACT_F32) return fail(KQ_ERR_INVALID, "unknown activation mode %d", act_mode);
  if (col0 < 0 || ldo < col0 + N) return fail(KQ_ERR_INVALID, "scatter: ldo=%d col0=%d N=%d (ldo >= col0 + N)", ldo, col0, N);
  OutSpec o{};
  for (int d = 0; d < n_out; ++d) {
    if (!outs[d] || !aligned(outs[d], 16)) return fail(KQ_ERR_INVALID, "scatter: destination %d null or unaligned", d);
    o.ptr[d] = outs[d];
  }
  o.n_out = n_out;
  o.ld = ldo;
  o.col0 = col0;
  if ((long long)M * N == 0) return KQ_OK;
  if (K == 0) return fail(KQ_ERR_UNSUPPORTED, "scatter: K == 0");
  if (!aligned(x, 16)) return fail(KQ_ERR_INVALID, "activations must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (gemv1_supported(wtype, M, N, K, w, x)) return launch_gemv1(wtype, w, x, o, N, K, act_mode, s);
  void* ws = workspace(WS_ACT, act8_bytes(M, K));
  if (!ws) return KQ_ERR_NOMEM;
  Act8 act = act8_view(ws, M, K);
  const bool gemv = gemv_supported(wtype, M, N, K) && aligned(w, 16);
  const bool tc = !gemv && gemm_tc_any_supported(wtype, M, N, K, w, act);
  if (!gemv && !tc) return fail(KQ_ERR_UNSUPPORTED, "scatter: shape M=%d N=%d K=%d has no scatter epilogue", M, N, K);
  st = launch_quantize_act(x, act, M, K, act_mode, s);
  if (st) return st;
  return gemv ? launch_gemv(wtype, w, act, o, M, N, K, true, s) : dispatch_gemm_tc(wtype, w, act, o, M, N, K, s, true);
}

kq_status_t kq_mul_mat_q8x(int wtype, const void* w, const int8_t* a_qs, const float* a_ds, float* out, int M, int N,
                           int K, kq_stream_t stream) {
  kq_status_t st = check_gemm_args(wtype, w, a_qs, out, M, N, K);
  if (st) return st;
  if ((long long)M * N == 0) return KQ_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (K == 0) return zero_output(out, M, N, s);
  if (!a_ds || !aligned(a_qs, 16) || !aligned(a_ds, 8))
    return fail(KQ_ERR_INVALID, "staged activations: codes must be 16-byte and scales 8-byte aligned");
  Act8 act{const_cast<int8_t*>(a_qs), reinterpret_cast<float2*>(const_cast<float*>(a_ds))};
  return dispatch_gemm(wtype, w, act, out, M, N, K, s, false);
}

kq_status_t kq_moe_q4_0(const float* x, const float* router_logits, const void* w_gate, const void* w_up,
                       const void* w_down, int E, int topk, int T, int H, int I, int act_mode, float* out,
                       kq_stream_t stream) {
  if (T < 0 || H <= 0 || I <= 0 || H % 32 || I % 32) return fail(KQ_ERR_INVALID, "moe: bad shape T=%d H=%d I=%d", T, H, I);
  if (act_mode < KQ_ACT_SUM_X || act_mode > KQ_ACT_F32) return fail(KQ_ERR_INVALID, "unknown activation mode %d", act_mode);
  if (T == 0) return KQ_OK;
  if (!x || !router_logits || !w_gate || !w_up || !w_down || !out) return fail(KQ_ERR_INVALID, "moe: null pointer");
  if (!aligned(x, 16) || !aligned(out, 16)) return fail(KQ_ERR_INVALID, "moe: x and out must be 16-byte aligned");
  return launch_moe_q4_0(x, router_logits, w_gate, w_up, w_down, E, topk, T, H, I, act_mode, out,
                         static_cast<cudaStream_t>(stream));
}

kq_status_t kq_moe_route(const float* router_logits, int T, int E, int topk, int32_t* idx, float* wts,
                         kq_stream_t stream) {
  if (T < 0) return fail(KQ_ERR_INVALID, "moe route: T=%d", T);
  if (T == 0) return KQ_OK;
  if (!router_logits || !idx || !wts) return fail(KQ_ERR_INVALID, "moe route: null pointer");
  return launch_moe_route(router_logits, T, E, topk, idx, wts, static_cast<cudaStream_t>(stream));
}

kq_status_t kq_moe_experts_q4_0(const float* x_rows, const int32_t* expert_of_row, const void* w_gate,
                                const void* w_up, const void* w_down, int E, int P, int H, int I, int act_mode,
                                float* y_rows, kq_stream_t stream) {
  if (P < 0 || H <= 0 || I <= 0 || H % 32 || I % 32) return fail(KQ_ERR_INVALID, "moe experts: bad shape P=%d H=%d I=%d", P, H, I);
  if (act_mode < KQ_ACT_SUM_X || act_mode > KQ_ACT_F32) return fail(KQ_ERR_INVALID, "unknown activation mode %d", act_mode);
  if (P == 0) return KQ_OK;
  if (!x_rows || !expert_of_row || !w_gate || !w_up || !w_down || !y_rows)
    return fail(KQ_ERR_INVALID, "moe experts: null pointer");
  if (!aligned(x_rows, 16) || !aligned(y_rows, 16)) return fail(KQ_ERR_INVALID, "moe experts: rows must be 16-byte aligned");
  return launch_moe_experts_q4_0(x_rows, expert_of_row, w_gate, w_up, w_down, E, P, H, I, act_mode, y_rows,
                                 static_cast<cudaStream_t>(stream));
}

kq_status_t kq_moe_experts_q4_0_q8_1(const void* a_rows, const int32_t* expert_of_row, const void* w_gate,
                                     const void* w_up, const void* w_down, int E, int P, int H, int I, int act_mode,
                                     float* y_rows, kq_stream_t stream) {
  if (P < 0 || H <= 0 || I <= 0 || H % 32 || I % 32)
    return fail(KQ_ERR_INVALID, "moe experts q8_1: bad shape P=%d H=%d I=%d", P, H, I);
  if (act_mode < KQ_ACT_SUM_X || act_mode > KQ_ACT_F32) return fail(KQ_ERR_INVALID, "unknown activation mode %d", act_mode);
  if (P == 0) return KQ_OK;
  if (!a_rows || !expert_of_row || !w_gate || !w_up || !w_down || !y_rows)
    return fail(KQ_ERR_INVALID, "moe experts q8_1: null pointer");
  if (!aligned(a_rows, 4) || !aligned(y_rows, 16))
    return fail(KQ_ERR_INVALID, "moe experts q8_1: rows must be 4-byte (q8_1) / 16-byte (output) aligned");
  return launch_moe_experts_q4_0(nullptr, expert_of_row, w_gate, w_up, w_down, E, P, H, I, act_mode, y_rows,
                                 static_cast<cudaStream_t>(stream), nullptr, a_rows);
}

kq_status_t kq_moe_experts_stages_q4_0(const float* x_rows, const int32_t* expert_of_row, const void* w_gate,
                                       const void* w_up, const void* w_down, int E, int P, int H, int I, int act_mode,
                                       float* gate, float* up, float* h, int8_t* h_qs, float* h_ds, float* y_rows,
                                       kq_stream_t stream) {
  if (P < 0 || H <= 0 || I <= 0 || H % 32 || I % 32)
    return fail(KQ_ERR_INVALID, "moe stages: bad shape P=%d H=%d I=%d", P, H, I);
  if (act_mode < KQ_ACT_SUM_X || act_mode > KQ_ACT_F32) return fail(KQ_ERR_INVALID, "unknown activation mode %d", act_mode);
  if (P == 0) return KQ_OK;
  if (!x_rows || !expert_of_row || !w_gate || !w_up || !w_down || !y_rows || !gate || !up || !h || !h_qs || !h_ds)
    return fail(KQ_ERR_INVALID, "moe stages: null pointer");
  for (const void* p : {(const void*)x_rows, (const void*)y_rows, (const void*)gate, (const void*)up, (const void*)h,
                        (const void*)h_qs, (const void*)h_ds})
    if (!aligned(p, 16)) return fail(KQ_ERR_INVALID, "moe stages: buffers must be 16-byte aligned");
  MoeStages st{gate, up, h, h_qs, h_ds};
  return launch_moe_experts_q4_0(x_rows, expert_of_row, w_gate, w_up, w_down, E, P, H, I, act_mode, y_rows,
                                 static_cast<cudaStream_t>(stream), &st);
}

kq_status_t kq_moe_combine(const float* y, const float* wts, int T, int topk, int H, float* out, kq_stream_t stream) {
  if (T < 0 || topk < 1 || H <= 0 || H % 4) return fail(KQ_ERR_INVALID, "moe combine: bad shape T=%d topk=%d H=%d", T, topk, H);
  if (T == 0) return KQ_OK;
  if (!y || !wts || !out) return fail(KQ_ERR_INVALID, "moe combine: null pointer");
  if (!aligned(y, 16) || !aligned(out, 16)) return fail(KQ_ERR_INVALID, "moe combine: y and out must be 16-byte aligned");
  return launch_moe_combine(y, wts, T, topk, H, out, static_cast<cudaStream_t>(stream));
}

kq_status_t kq_block_sums_i32(int wtype, const void* w, const void* a_q8_1, int32_t* sumi, int M, int N, int K,
                              kq_stream_t stream) {
  if (block_bytes(wtype) == 0) return fail(KQ_ERR_INVALID, "unknown weight type %d", wtype);
  if (M < 0 || N < 0 || K < 0 || K % 32) return fail(KQ_ERR_INVALID, "block_sums: bad shape");
  if ((long long)M * N * K == 0) return KQ_OK;
  if (!w || !a_q8_1 || !sumi) return fail(KQ_ERR_INVALID, "block_sums: null pointer");
  return launch_block_sums(wtype, w, a_q8_1, sumi, M, N, K, static_cast<cudaStream_t>(stream));
}

kq_status_t kq_fa_decode_mha(int kv_format, const float* q, const void* k, const void* v, float* out, int B, int S,
                             int H, int D, kq_stream_t stream) {
  if (kv_format < KQ_KV_Q8_0 || kv_format > KQ_KV_F16) return fail(KQ_ERR_INVALID, "fa_mha: unknown KV format %d", kv_format);
  if (B < 0 || S < 0 || H < 0 || D <= 0 || D % 32 || D > 256)
    return fail(KQ_ERR_INVALID, "fa_mha: bad shape B=%d S=%d H=%d D=%d (D must be a multiple of 32, <= 256)", B, S, H, D);
  if ((long long)B * H == 0) return KQ_OK;
  if (!q || !out || (S > 0 && (!k || !v))) return fail(KQ_ERR_INVALID, "fa_mha: null pointer");
  if (!aligned(k, 2) || !aligned(v, 2)) return fail(KQ_ERR_INVALID, "fa_mha: caches must be 2-byte aligned");
  return launch_fa_mha(kv_format, q, k, v, out, B, S, H, D, static_cast<cudaStream_t>(stream));
}

kq_status_t kq_fa_decode_q8_0_mha(const float* q, const void* k, const void* v, float* out, int B, int S, int H,
                                  int D, kq_stream_t stream) {
  return kq_fa_decode_mha(KQ_KV_Q8_0, q, k, v, out, B, S, H, D, stream);
}

kq_status_t kq_fa_decode_q8_0_ragged(const void* q_f16, const void* k, const void* v, const int32_t* cu_seqlens,
                                     int B, int Hq, int Hkv, int D, int max_seqlen, int total_rows, float scale,
                                     void* out_f16, kq_stream_t stream) {
  if (B < 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv || D <= 0 || D % 32 || D > 256 || max_seqlen < 0 || total_rows < 0)
    return fail(KQ_ERR_INVALID, "fa_ragged: bad shape B=%d Hq=%d Hkv=%d D=%d", B, Hq, Hkv, D);
  if (B == 0) return KQ_OK;
  if (!q_f16 || !out_f16 || !cu_seqlens || !k || !v) return fail(KQ_ERR_INVALID, "fa_ragged: null pointer");
  if (!aligned(k, 2) || !aligned(v, 2)) return fail(KQ_ERR_INVALID, "fa_ragged: caches must be 2-byte aligned");
  return launch_fa_ragged(q_f16, k, v, cu_seqlens, B, Hq, Hkv, D, max_seqlen, total_rows, scale, out_f16,
                          static_cast<cudaStream_t>(stream));
}

// ---- KernelEvalPlus operator ABI --------------------------------------------

void kq_w4a32c8_q4_0_fp32_int8(const uint8_t* weight, const float* activation, float* output, int M, int N, int K) {
  g_last_error.clear();  // the harness shim reports a non-empty message as a failure
  kq_gemm_f32act(KQ_Q4_0, weight, activation, output, M, N, K, KQ_ACT_F32, nullptr);
}

void kq_w4a32c8_q4_1_fp32_int8(const uint8_t* weight, const float* activation, float* output, int M, int N, int K) {
  g_last_error.clear();  // the harness shim reports a non-empty message as a failure
  kq_gemm_f32act(KQ_Q4_1, weight, activation, output, M, N, K, KQ_ACT_F32, nullptr);
}

void kq_w8a32c8_q8_0_fp32_int8(const uint8_t* weight, const float* activation, float* output, int M, int N, int K) {
  g_last_error.clear();  // the harness shim reports a non-empty message as a failure
  kq_gemm_f32act(KQ_Q8_0, weight, activation, output, M, N, K, KQ_ACT_F32, nullptr);
}

void kq_w4a8_q4_0_q8_1(const uint8_t* weight, const uint8_t* activation, float* output, int M, int N, int K) {
  g_last_error.clear();  // the harness shim reports a non-empty message as a failure
  kq_mul_mat_q(KQ_Q4_0, weight, activation, output, M, N, K, nullptr);
}

void kq_flash_attn_q8_0(const float* query, const void* key_cache, const void* value_cache, float* output,
                        int batch_size, int seq_len, int num_heads, int head_dim) {
  g_last_error.clear();  // the harness shim reports a non-empty message as a failure
  kq_fa_decode_q8_0_mha(query, key_cache, value_cache, output, batch_size, seq_len, num_heads, head_dim, nullptr);
}

void kq_rms_norm(const float* input, const float* weight, float* output, int batch_size, int hidden_size) {
  g_last_error.clear();
  kq_rms_norm_f32(input, weight, output, batch_size, hidden_size, 1e-6f, nullptr);
}

void kq_flash_attn_q4_0(const float* query, const void* key_cache, const void* value_cache, float* output,
                        int batch_size, int seq_len, int num_heads, int head_dim) {
  g_last_error.clear();
  kq_fa_decode_mha(KQ_KV_Q4_0, query, key_cache, value_cache, output, batch_size, seq_len, num_heads, head_dim,
                   nullptr);
}

void kq_flash_attn_f16(const float* query, const void* key_cache, const void* value_cache, float* output,
                       int batch_size, int seq_len, int num_heads, int head_dim) {
  g_last_error.clear();
  kq_fa_decode_mha(KQ_KV_F16, query, key_cache, value_cache, output, batch_size, seq_len, num_heads, head_dim,
                   nullptr);
}

}  // extern "C"
