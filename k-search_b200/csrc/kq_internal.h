// Internal host-side declarations shared by the libkq translation units.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>

#include <cstddef>
#include <cstdint>

#include "kq.h"

namespace kq {

// ---- errors ---------------------------------------------------------------
// Records `msg` as the calling thread's last error and returns `st`.
kq_status_t fail(kq_status_t st, const char* fmt, ...);
// Turns a pending launch / runtime error into KQ_ERR_CUDA.
kq_status_t check_cuda(cudaError_t e, const char* what);
kq_status_t check_launch(const char* what);

// ---- device properties ----------------------------------------------------
int current_device();
int sm_count();

// ---- driver entry points ----------------------------------------------------
// cuTensorMapEncodeTiled resolved through the runtime (no link-time libcuda
// dependency, so the library loads on hosts without a driver). Returns
// nullptr if unavailable.
void* tensor_map_encoder();

// ---- kernel attributes ------------------------------------------------------
// Raises `func`'s dynamic shared-memory limit to `bytes` on the current
// device, once per (device, kernel); thread-safe. `what` names the kernel in
// the error message.
kq_status_t ensure_dynamic_smem(const void* func, int bytes, const char* what);

// ---- workspace ------------------------------------------------------------
// Per-device cached scratch, one buffer per slot, grown on demand (never
// shrunk). The buffer is ordered on `stream`: growing it synchronises the
// device before the old buffer is freed. Returns nullptr (and records the
// error) on allocation failure.
enum WsSlot { WS_ACT = 0, WS_FA = 1, WS_MOE = 2, WS_MOE2 = 3, WS_A16 = 4, WS_NSLOTS = 8 };
void* workspace(WsSlot slot, size_t bytes);
// Device error word of the current device (zeroed at allocation).
int* device_error_word();

// ---- activation staging ---------------------------------------------------
// Quantised activations as the kernels consume them: int8 codes row-major
// [M, K] (row stride K bytes) and one float2 (d, s) per 32-block [M, K/32].
// Output destinations of a GEMM epilogue: element (m, n) goes to
// ptr[d][m * ld + col0 + n] for every d < n_out. One destination is the plain
// case; several are the N-sharded multi-GPU case (this rank's columns written
// into every rank's full-width output over peer mappings).
constexpr int kMaxOut = 8;
struct OutSpec {
  float* ptr[kMaxOut];
  int n_out;
  int ld;
  int col0;
  static OutSpec plain(float* out, int N) {
    OutSpec o{};
    o.ptr[0] = out;
    o.n_out = 1;
    o.ld = N;
    o.col0 = 0;
    return o;
  }
};

struct Act8 {
  int8_t* qs;
  float2* ds;
};
inline size_t act8_bytes(int M, int K) {
  const size_t q = ((size_t)M * K + 255) & ~(size_t)255;
  return q + (size_t)M * (K / 32) * sizeof(float2);
}
inline Act8 act8_view(void* base, int M, int K) {
  const size_t q = ((size_t)M * K + 255) & ~(size_t)255;
  return Act8{static_cast<int8_t*>(base), reinterpret_cast<float2*>(static_cast<char*>(base) + q)};
}

inline int block_bytes(int wtype) {
  return wtype == KQ_Q4_0 ? 18 : wtype == KQ_Q4_1 ? 20 : wtype == KQ_Q8_0 ? 34 : 0;
}

// ---- kernel launchers (one per translation unit family) -------------------
// quantize.cu
kq_status_t launch_quantize_act(const float* x, Act8 act, int M, int K, int mode, cudaStream_t s);
kq_status_t launch_quantize_q8_1_bytes(const float* x, void* y, int64_t M, int64_t K, int mode, cudaStream_t s);
kq_status_t launch_quantize_rows(int wtype, const float* x, void* y, int64_t rows, int64_t K, cudaStream_t s);
kq_status_t launch_q8_1_to_act(const void* a_q8_1, Act8 act, int M, int K, cudaStream_t s);
// Row r of the staging takes q8_1 row rowmap[r] (K/32 blocks of 36 B per row).
kq_status_t launch_q8_1_to_act_gather(const void* a_q8_1, const int* rowmap, Act8 act, int M, int K, cudaStream_t s);
// out = x / sqrt(mean(x^2) + eps) * w per row of x fp32 [M, K]
kq_status_t launch_rms_norm(const float* x, const float* w, float* out, int M, int K, float eps, cudaStream_t s);
// RMSNorm then q8_1: into the staging `act` (q81 == nullptr) or as q8_1 bytes
// q81 [M, K/32, 36]. K % 32 == 0; x, w 16-byte aligned.
kq_status_t launch_rms_norm_quantize(const float* x, const float* w, float eps, Act8 act, void* q81, int M, int K,
                                     int mode, cudaStream_t s);
// staging row r <- quantise(x row rowmap[r] / div)
kq_status_t launch_quantize_act_gather(const float* x, const int* rowmap, int div, Act8 act, int M, int K, int mode,
                                       cudaStream_t s);
// staging <- quantise(silu(gate) * up), gate/up fp32 [M, K]
kq_status_t launch_silu_mul_quantize(const float* gate, const float* up, Act8 act, int M, int K, int mode,
                                     cudaStream_t s);
// gemv.cu (M <= 8, K % 256 == 0); `pdl` = launched as a programmatic
// dependent of the preceding kernel on `s` (the activation producer).
bool gemv_supported(int wtype, int M, int N, int K);
kq_status_t launch_gemv(int wtype, const void* w, Act8 act, const OutSpec& out, int M, int N, int K, bool pdl,
                        cudaStream_t s, int* err = nullptr);
kq_status_t launch_gemv(int wtype, const void* w, Act8 act, float* out, int M, int N, int K, bool pdl,
                        cudaStream_t s, int* err = nullptr);
// gemv1.cu: one launch for M = 1 (q4_0 / q4_1 / q8_0 weights): quantises
// the fp32 row itself (bit-identical codes), no workspace. K % 256 == 0,
// K <= 32768, w and x 16-byte aligned.
bool gemv1_supported(int wtype, int M, int N, int K, const void* w, const float* x);
kq_status_t launch_gemv1(int wtype, const void* w, const float* x, const OutSpec& out, int N, int K, int mode,
                         cudaStream_t s, int* err = nullptr);
// gemm_tc.cu (M > 8, K % 256 == 0, 16-byte aligned operands): tcgen05 int8 MMA
bool gemm_tc_supported(int wtype, int M, int N, int K, const void* w, Act8 act);
kq_status_t launch_gemm_tc(int wtype, const void* w, Act8 act, const OutSpec& out, int M, int N, int K, bool pdl,
                           cudaStream_t s, int* err = nullptr);
kq_status_t launch_gemm_tc(int wtype, const void* w, Act8 act, float* out, int M, int N, int K, bool pdl,
                           cudaStream_t s, int* err = nullptr);
// gemm_split.cu (M > 8, K % 256 == 0): exact split-fp16 operands, tcgen05 kind::f16
bool gemm_split_supported(int wtype, int M, int N, int K, const void* w, Act8 act);
kq_status_t launch_gemm_split(int wtype, const void* w, Act8 act, const OutSpec& out, int M, int N, int K,
                              cudaStream_t s, int* err = nullptr);
// gemm_skinny.cu (8 < M <= 128, K % 256 == 0, 16-byte aligned weights and
// staging): weights streamed once, mma.sync int8 per 32-block, fp32 epilogue
bool gemm_skinny_supported(int wtype, int M, int N, int K, const void* w, Act8 act);
kq_status_t launch_gemm_skinny(int wtype, const void* w, Act8 act, const OutSpec& out, int M, int N, int K,
                               cudaStream_t s, int* err = nullptr);
// gemm_simt.cu (any shape; the generic path)
kq_status_t launch_gemm_simt(int wtype, const void* w, Act8 act, float* out, int M, int N, int K, cudaStream_t s);
// any shape: GEMV (M <= 8), tcgen05 GEMM, else the generic kernel (no PDL)
kq_status_t gemm_any(int wtype, const void* w, Act8 act, float* out, int M, int N, int K, cudaStream_t s);
// moe.cu
size_t moe_workspace_bytes(int P, int E, int H, int I);
kq_status_t launch_moe_route(const float* logits, int T, int E, int topk, int* idx, float* wts, cudaStream_t s);
// Intermediates of the expert FFNs in the input row order (parity debugging):
// gate / up / h = silu(gate) * up fp32 [P, I], h's staged codes [P, I] and
// (d, s) pairs [P, I/32].
struct MoeStages {
  float* gate;
  float* up;
  float* h;
  int8_t* h_qs;
  float* h_ds;
};
kq_status_t launch_moe_experts_q4_0(const float* x_rows, const int* expert_of_row, const void* w_gate,
                                    const void* w_up, const void* w_down, int E, int P, int H, int I, int act_mode,
                                    float* y_rows, cudaStream_t s, const MoeStages* stages = nullptr,
                                    const void* a_q8_1 = nullptr);  // a_q8_1: q8_1 rows replace x_rows
kq_status_t launch_moe_combine(const float* y, const float* wts, int T, int topk, int H, float* out, cudaStream_t s);
kq_status_t launch_moe_q4_0(const float* x, const float* logits, const void* w_gate, const void* w_up,
                            const void* w_down, int E, int topk, int T, int H, int I, int act_mode, float* out,
                            cudaStream_t s);
kq_status_t launch_block_sums(int wtype, const void* w, const void* a_q8_1, int32_t* sumi, int M, int N, int K,
                              cudaStream_t s);
// fa_decode.cu
// kv_format: KQ_KV_Q8_0 / KQ_KV_Q4_0 / KQ_KV_F16
kq_status_t launch_fa_mha(int kv_format, const float* q, const void* k, const void* v, float* out, int B, int S, int H,
                          int D, cudaStream_t s);
// fa_stream.cu: the tensor-core decode with the balanced persistent schedule
// (q8_0 caches, D = 128, KV heads in groups of 8, <= 4 queries per KV head,
// <= 512 ragged sequences, 16-byte aligned q, k, v and out)
bool fa_stream_supported(const void* q, const void* k, const void* v, const void* out, int D, int Hkv,
                         int queries_per_kv_head, int nseq_ragged);
kq_status_t launch_fa_stream_ragged(const void* q, const void* k, const void* v, const int32_t* cu, int B, int Hq,
                                    int Hkv, int total_rows, float scale, void* out, cudaStream_t s);
kq_status_t launch_fa_stream_mha(const float* q, const void* k, const void* v, float* out, int B, int S, int H,
                                 cudaStream_t s);
// fa_small.cu: the small-batch decode (D = 128, <= 4 queries per KV head,
// 16-byte aligned q, k, v and out; q8_0 or q4_0 caches with an even number
// of KV heads, or fp16 caches; the ragged form q8_0 only): every warp streams
// one KV head's token chunk by itself
bool fa_small_supported(int kv_format, const void* q, const void* k, const void* v, const void* out, int D,
                        int Hkv, int queries_per_unit);
kq_status_t launch_fa_small_mha(int kv_format, const float* q, const void* k, const void* v, float* out, int B,
                                int S, int H, cudaStream_t s);
kq_status_t launch_fa_small_ragged(const void* q, const void* k, const void* v, const int32_t* cu, int B, int Hq,
                                   int Hkv, int max_seqlen, int total_rows, float scale, void* out, cudaStream_t s);
// fa_batch.cu: the harness form with many queries per head (q8_0, q4_0 or
// fp16 caches, D = 128, an even head count for the block formats,
// ceil(B / 64) * H >= SMs, 16-byte aligned q, k, v and out): tensor-core
// flash attention, 64 queries per CTA
bool fa_batch_supported(int kv_format, const void* q, const void* k, const void* v, const void* out, int B, int S,
                        int H, int D);
kq_status_t launch_fa_batch_mha(int kv_format, const float* q, const void* k, const void* v, float* out, int B,
                                int S, int H, cudaStream_t s);
kq_status_t launch_fa_ragged(const void* q, const void* k, const void* v, const int32_t* cu, int B, int Hq, int Hkv,
                             int D, int max_seqlen, int total_rows, float scale, void* out, cudaStream_t s);

}  // namespace kq
