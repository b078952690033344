/*
 * kq.h - C ABI of libkq.so, the B200 (sm_100a) kernels for the GGML
 * block-quantized inference path that KernelEvalPlus (inside qhy991/K-Search)
 * defines.
 *
 * Plain pointers and sizes only. All pointers are DEVICE pointers unless a
 * comment says otherwise; buffers belong to the caller. Streams are passed as
 * an opaque cudaStream_t (NULL = legacy default stream).
 *
 * Two families of entry points:
 *
 *  1. The KernelEvalPlus operator ABI, signature for signature. The harness
 *     binds the first `extern "C" void` of an attempt's kernel.cu
 *     (kernelevalplus-main/llm_kernel_test/op_test_handler.py:305-349 for
 *     quant_gemm, llm_kernel_test/unified_test_runner.py:295-324 for
 *     flash_attention). These return void, run on the legacy default stream
 *     (as the harness's candidate kernels do) and record failures for
 *     kq_last_error(); the harness-side shim (k-search_b200/harness/) turns a
 *     failure into a C++ exception.
 *
 *  2. Status-returning entry points with an explicit stream (kq_status_t,
 *     KQ_OK == 0). These are what the Python package and the benchmarks call.
 *
 * Block layouts are the reference's (kernelevalplus-main/include/quant_types.h:
 * 59-152): q4_0 = fp16 d | 16 B nibbles (18 B), q4_1 = fp16 d | fp16 m |
 * 16 B (20 B), q8_0 = fp16 d | 32 x int8 (34 B), q8_1 = fp16 d | fp16 s |
 * 32 x int8 (36 B); a weight matrix [N, K] is N rows of K/32 blocks.
 */
#ifndef KQ_H
#define KQ_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int kq_status_t;
#define KQ_OK 0
#define KQ_ERR_INVALID 1     /* bad argument: shape, type, null pointer, alignment */
#define KQ_ERR_UNSUPPORTED 2 /* valid input this build does not handle */
#define KQ_ERR_CUDA 3        /* CUDA runtime error (launch, memory) */
#define KQ_ERR_NOMEM 4       /* library workspace could not be allocated */
#define KQ_ERR_TIMEOUT 5     /* a bounded device-side wait gave up */
#define KQ_ERR_DEVICE 6      /* a device-side check recorded an error */

/* weight block types */
#define KQ_Q4_0 0
#define KQ_Q4_1 1
#define KQ_Q8_0 2

/* On-the-fly activation quantisation modes. The int8 codes are the same in
 * all three (q = round_half_even(x / d), d = amax/127, d = 1 when amax == 0;
 * llm_kernel_test/reference/quantize.py:181-191); they differ in the block
 * scale d and sum s used by the fp32 epilogue:
 *   KQ_ACT_SUM_X  fp16 d, fp16 s = sum(x)        (quantize.py:193-209, q8_1 bytes)
 *   KQ_ACT_SUM_DQ fp16 d, fp16 s = fp16(d)*sum(q) (benchmark configurations)
 *   KQ_ACT_F32    fp32 d, fp32 s = sum(x)         (per-definition W4A32C8 reference,
 *                 core/operators/quant_gemm/variants/deepseek_v2/w4a32c8_q4_0_fp32_int8/reference.py:50-90) */
#define KQ_ACT_SUM_X 0
#define KQ_ACT_SUM_DQ 1
#define KQ_ACT_F32 2

/* KV cache formats of the flash_attention definitions, as the harness builds
 * them from fp32 [S, H, D] (op_test_handler.py:485-534): q8_0 blocks of each
 * D-long row (quantize_to_q8_0), q4_0 blocks (quantize_to_q4_0, quantize.py:56-102:
 * d = amax/7, value d (q - 8)), or fp16. */
#define KQ_KV_Q8_0 0
#define KQ_KV_Q4_0 1
#define KQ_KV_F16 2

typedef void* kq_stream_t; /* cudaStream_t */

/* ---- library ------------------------------------------------------------ */

/* ABI version (bumped on any signature change). */
int kq_abi_version(void);
/* Message of the last failure on the calling host thread ("" if none). */
const char* kq_last_error(void);
/* Bytes per block of a weight type (18, 20, 34), 0 for an unknown type. */
size_t kq_block_bytes(int wtype);
/* Reads and clears the device error word of the current device (synchronises
 * the given stream). *code receives the first recorded device error (0 = none). */
kq_status_t kq_device_error(int* code, kq_stream_t stream);
/* Failure-detection self-test (no counterpart in the reference, which has no
 * device-side waits): runs the library's bounded mbarrier wait on a barrier
 * that nothing ever arrives at, with a wait limit of limit_ns (0 < limit_ns <=
 * 2e9; the kernels use 2e9). The wait gives up, records DEV_TIMEOUT_FULL (1)
 * in the device error word (first writer wins; read and cleared with
 * kq_device_error) and the kernel returns. Synchronises the stream; returns
 * KQ_ERR_TIMEOUT when the error word holds a timeout code. */
kq_status_t kq_selftest_wait_timeout(int64_t limit_ns, kq_stream_t stream);

/* ---- 1. KernelEvalPlus operator ABI (void, legacy default stream) -------- */

/* quant_gemm, fp32 activations quantised on the fly (W4A32C8 / W8A32C8):
 * output[M, N] = activation[M, K] x dequant(weight[N, K/32 blocks])^T with the
 * llama.cpp per-block formula. Activation mode KQ_ACT_F32.
 * Replaces the attempt entry bound by op_test_handler.py:315-320
 * (`extern "C" void <entry>(const uint8_t*, const float*, float*, int, int, int)`)
 * for definitions with weight dtype block_q4_0 / block_q4_1 / block_q8_0 and
 * activation dtype float32 (e.g. definitions/quant_gemm/.../w4a32c8_q4_0_fp32_int8_*.json). */
void kq_w4a32c8_q4_0_fp32_int8(const uint8_t* weight, const float* activation, float* output, int M, int N, int K);
void kq_w4a32c8_q4_1_fp32_int8(const uint8_t* weight, const float* activation, float* output, int M, int N, int K);
void kq_w8a32c8_q8_0_fp32_int8(const uint8_t* weight, const float* activation, float* output, int M, int N, int K);

/* quant_gemm with pre-quantised q8_1 activations (activation dtype block_q8_1;
 * op_test_handler.py:311-313 switches the activation pointer to uint8_t).
 * Replaces the same attempt entry for W4A8 definitions. */
void kq_w4a8_q4_0_q8_1(const uint8_t* weight, const uint8_t* activation, float* output, int M, int N, int K);

/* flash_attention decode with a q8_0 KV cache: query fp32 [B, H, D];
 * key_cache / value_cache = q8_0 blocks of the [S, H, D] cache (row (s, h) is
 * D/32 blocks, op_test_handler.py:489-508); all B queries attend to the same
 * cache; scale 1/sqrt(D); output fp32 [B, H, D].
 * Replaces `extern "C" void flash_attn_kernel(...)` bound by
 * unified_test_runner.py:298-303. */
void kq_flash_attn_q8_0(const float* query, const void* key_cache, const void* value_cache, float* output,
                        int batch_size, int seq_len, int num_heads, int head_dim);
/* The same operator for the q4_0-cache definitions
 * (definitions/flash_attention/<model>/fp32_flash_attention_*_q4_0_cache*.json):
 * key_cache / value_cache = q4_0 blocks (18 B) of the [S, H, D] rows. */
void kq_flash_attn_q4_0(const float* query, const void* key_cache, const void* value_cache, float* output,
                        int batch_size, int seq_len, int num_heads, int head_dim);
/* The same operator for the f16-cache definitions
 * (definitions/flash_attention/<model>/fp32_flash_attention_*_f16_cache*.json):
 * key_cache / value_cache = fp16 [S, H, D]. */
void kq_flash_attn_f16(const float* query, const void* key_cache, const void* value_cache, float* output,
                       int batch_size, int seq_len, int num_heads, int head_dim);

/* rms_norm: output[b, :] = input[b, :] / sqrt(mean(input[b, :]^2) + 1e-6) * weight
 * (fp32; RMSNormHandler op_test_handler.py:641-690, every rms_norm definition
 * has epsilon 1e-6 and the bound signature carries none).
 * Replaces `extern "C" void rms_norm_kernel(const float* input, const float* weight,
 * float* output, int batch_size, int hidden_size)` bound by unified_test_runner.py:330-350. */
void kq_rms_norm(const float* input, const float* weight, float* output, int batch_size, int hidden_size);

/* ---- 2. Status-returning entry points ------------------------------------ */

/* fp32 x[M, K] -> q8_1 blocks y[M, K/32] (36 B each), sum_mode KQ_ACT_SUM_X
 * or KQ_ACT_SUM_DQ. Bit-exact with quantize_to_q8_1 (quantize.py:165-214) for
 * KQ_ACT_SUM_X, including the fp32 summation order of s.
 * GPU form of quantize_q8_1_kernel (include/quantize.h:302-340). */
kq_status_t kq_quantize_q8_1(const float* x, void* y, int64_t M, int64_t K, int sum_mode, kq_stream_t stream);

/* fp32 rows x[rows, K] -> q4_0 / q4_1 / q8_0 blocks y (weights, KV caches).
 * Bit-exact with quantize_to_q4_0 / _q4_1 / _q8_0 (quantize.py:12-162); GPU
 * form of quantize_q4_0_kernel / quantize_q8_0_kernel (include/quantize.h:221-294). */
kq_status_t kq_quantize_rows(int wtype, const float* x, void* y, int64_t rows, int64_t K, kq_stream_t stream);

/* Weights x pre-quantised q8_1 activations a[M, K/32] -> fp32 out[M, N]
 * (reference_q4_0_q8_1_gemm gemm_ref.py:100-153, reference_q4_1_q8_1_gemm
 * gemm_ref.py:274-331, vec_dot_q8_0_q8_1 gemm_reference.h:311-336). */
kq_status_t kq_mul_mat_q(int wtype, const void* w, const void* a_q8_1, float* out, int M, int N, int K,
                         kq_stream_t stream);

/* RMSNorm with an explicit epsilon: out[M, K] from x[M, K] and weight[K]
 * (the status form of kq_rms_norm). */
kq_status_t kq_rms_norm_f32(const float* x, const float* weight, float* out, int M, int K, float eps,
                            kq_stream_t stream);

/* RMSNorm fused into quantize_q8_1: y = q8_1 blocks [M, K/32] (36 B) of
 * x[m] / sqrt(mean(x[m]^2) + eps) * weight, sum_mode KQ_ACT_SUM_X or
 * KQ_ACT_SUM_DQ. The normalised fp32 row never goes to memory. K % 32 == 0;
 * x and weight 16-byte aligned. No reference counterpart: the reference runs
 * rms_norm and quantize_q8_1 as separate operators. */
kq_status_t kq_rms_norm_quantize_q8_1(const float* x, const float* weight, void* y, int M, int K, float eps,
                                      int sum_mode, kq_stream_t stream);

/* kq_gemm_f32act on RMSNorm(x): out[M, N] = q8_1(x / rms(x) * norm_weight) x W^T
 * in one call (the normalised activation is quantised as it is produced).
 * No reference counterpart: rms_norm followed by the quant_gemm operator. */
kq_status_t kq_gemm_f32act_rmsnorm(int wtype, const void* w, const float* x, const float* norm_weight, float eps,
                                   float* out, int M, int N, int K, int act_mode, kq_stream_t stream);

/* Weights x fp32 activations quantised on the fly (the harness operator).
 * act_mode is one of KQ_ACT_*; the status form of the void entries above. */
kq_status_t kq_gemm_f32act(int wtype, const void* w, const float* x, float* out, int M, int N, int K,
                           int act_mode, kq_stream_t stream);

/* kq_gemm_f32act without device allocation. No counterpart in the reference:
 * it exists for callers that cannot call cudaMalloc (a serving runtime whose
 * allocator already owns nearly all of HBM, or code that must not synchronise
 * the device on a first-call allocation). The activation staging lives in a
 * fixed 1 MiB file-scope __device__ array held by every GPU that loads libkq:
 * calls whose staging, round_up(M*K, 256) + M*(K/32)*8 bytes, is above 1 MiB
 * are rejected with KQ_ERR_INVALID. Device-side wait timeouts of these calls
 * go to a word of their own, read with kq_noalloc_device_error (which, unlike
 * kq_device_error, allocates nothing). The first call on a device
 * resolves the array's device address (cudaGetSymbolAddress) and should come
 * before any stream capture. All calls share the array: calls that overlap on
 * the GPU race. Same arguments as kq_gemm_f32act; for M > 8 it runs the int8
 * tensor-core kernel (no fp16 operand workspace), whose results agree with
 * kq_gemm_f32act's to the parity bar rather than bit for bit. For M = 1 both
 * entry points run the same single-launch GEMV,
 * which quantises the row in shared memory and touches no staging. */
kq_status_t kq_gemm_f32act_noalloc(int wtype, const void* w, const float* x, float* out, int M, int N, int K,
                                   int act_mode, kq_stream_t stream);
/* Reads and clears the device error word of kq_gemm_f32act_noalloc's kernels
 * on the current device (synchronises `stream`); *code = 0 when no wait timed
 * out. Allocates nothing. No reference counterpart. */
kq_status_t kq_noalloc_device_error(int* code, kq_stream_t stream);

/* The fused fp32-activation GEMM writing each output element to several
 * destinations: element (m, n) goes to outs[d][m * ldo + col0 + n] for every
 * d < n_out (1 <= n_out <= 8). For N-sharded multi-GPU use: a rank computes
 * its columns and stores them straight into every rank's full-width output
 * (pointers to peer memory mapped with CUDA IPC); the epilogue ends with a
 * system-scope fence, so a barrier after the call (stream-ordered) makes the
 * peers' data visible. Supported on the GEMV (M <= 8) and tensor-core
 * (M > 8, K % 256 == 0) paths; other shapes return KQ_ERR_UNSUPPORTED. ldo,
 * col0 and every pointer must keep 16-byte alignment for the vector stores
 * (ldo and col0 multiples of 4). No reference counterpart: the reference is
 * single-device. */
kq_status_t kq_gemm_f32act_scatter(int wtype, const void* w, const float* x, float* const* outs, int n_out, int ldo,
                                   int col0, int M, int N, int K, int act_mode, kq_stream_t stream);

/* Peer-mapped buffers for kq_gemm_f32act_scatter (CUDA IPC, one process per
 * GPU on one node). kq_peer_alloc allocates `bytes` on the current device and
 * writes its 64-byte IPC handle; another process opens it with kq_peer_open
 * (the mapping is usable from that process's current device) and releases it
 * with kq_peer_close; the owner frees it with kq_peer_free. */
kq_status_t kq_peer_alloc(size_t bytes, void** ptr, void* handle64);
kq_status_t kq_peer_open(const void* handle64, void** ptr);
kq_status_t kq_peer_close(void* ptr);
kq_status_t kq_peer_free(void* ptr);
/* Strided device copy (rows of `width_bytes`, `height` rows), either side may
 * be a peer mapping: the push of one rank's column block into a peer's
 * full-width output. Stream-ordered on `stream`. */
kq_status_t kq_copy_2d(void* dst, size_t dst_pitch, const void* src, size_t src_pitch, size_t width_bytes,
                       size_t height, kq_stream_t stream);

/* Weights x activations already in the kernels' staging layout: int8 codes
 * a_qs[M, K] (row stride K bytes, 16-byte aligned) and one (d, s) fp32 pair
 * per 32-block a_ds[M, K/32, 2]. For callers that quantise inside their own
 * producer kernel; the same per-block formulas as kq_mul_mat_q. */
kq_status_t kq_mul_mat_q8x(int wtype, const void* w, const int8_t* a_qs, const float* a_ds, float* out, int M, int N,
                           int K, kq_stream_t stream);

/* Grouped q4_0 MoE expert FFN (benchmark configuration 4). x fp32 [T, H];
 * router_logits fp32 [T, E]; per expert, contiguous q4_0 weights: w_gate and
 * w_up [E][I rows][H/32 blocks], w_down [E][H rows][I/32 blocks]. Routing:
 * softmax over E, top-k (ties -> lower expert index), weights renormalised
 * over the k chosen. Per expert: h = silu(x Wg^T) * (x Wu^T), y = h Wd^T, with
 * activations quantised (act_mode) before each GEMM; out fp32 [T, H] =
 * sum_k w[t,k] y_k[t]. No grouped MoE operator exists in the reference; each
 * expert GEMM is the W4A32C8 operator
 * (definitions/quant_gemm/mixtral8x7b/w4a32c8_q4_0_fp32_int8_mixtral8x7b_moe_up_n14336_k4096.json).
 * Reads the per-expert token counts back to the host once per call. */
kq_status_t kq_moe_q4_0(const float* x, const float* router_logits, const void* w_gate, const void* w_up,
                       const void* w_down, int E, int topk, int T, int H, int I, int act_mode, float* out,
                       kq_stream_t stream);

/* The three stages of kq_moe_q4_0 as separate calls, for expert parallelism
 * (routed rows cross ranks between them). No reference counterpart: the
 * reference has no MoE operator; the math is exactly kq_moe_q4_0's.
 *
 * kq_moe_route: idx int32 [T, topk] and wts fp32 [T, topk] from router_logits
 * fp32 [T, E] (softmax, top-k with ties to the lower index, renormalised). */
kq_status_t kq_moe_route(const float* router_logits, int T, int E, int topk, int32_t* idx, float* wts,
                         kq_stream_t stream);

/* Expert FFNs of P routed rows: row p of x_rows fp32 [P, H] goes through
 * expert expert_of_row[p] (0 <= e < E; int32, device) of this call's weights
 * (same layout as kq_moe_q4_0); y_rows fp32 [P, H] keeps the row order. Reads
 * the per-expert row counts back to the host once per call. */
kq_status_t kq_moe_experts_q4_0(const float* x_rows, const int32_t* expert_of_row, const void* w_gate,
                                const void* w_up, const void* w_down, int E, int P, int H, int I, int act_mode,
                                float* y_rows, kq_stream_t stream);
/* kq_moe_experts_q4_0 on rows that arrive already quantised: a_rows are P
 * rows of q8_1 blocks (H/32 blocks of 36 bytes each, the layout
 * kq_quantize_q8_1 writes), for instance received from another rank in an
 * expert-parallel dispatch (a third of the bytes of fp32 rows). act_mode
 * applies to the re-quantisation of silu(gate) * up. Same results as
 * kq_moe_experts_q4_0 on the fp32 rows those bytes were quantised from in the
 * same mode (KQ_ACT_SUM_X or KQ_ACT_SUM_DQ). No counterpart in the reference
 * (it has no MoE operator). */
kq_status_t kq_moe_experts_q4_0_q8_1(const void* a_rows, const int32_t* expert_of_row, const void* w_gate,
                                     const void* w_up, const void* w_down, int E, int P, int H, int I, int act_mode,
                                     float* y_rows, kq_stream_t stream);

/* Parity debugging: kq_moe_experts_q4_0 that also writes the pipeline's own
 * intermediates in the input row order: gate = x W_gate^T and up = x W_up^T
 * fp32 [P, I], h = silu(gate) * up fp32 [P, I] exactly as the quantiser forms
 * it, and h's quantised codes h_qs int8 [P, I] with (d, s) fp32 pairs
 * h_ds [P, I/32, 2] (the down projection's input). All buffers 16-byte
 * aligned. No reference counterpart (the reference has no MoE operator). */
kq_status_t kq_moe_experts_stages_q4_0(const float* x_rows, const int32_t* expert_of_row, const void* w_gate,
                                       const void* w_up, const void* w_down, int E, int P, int H, int I, int act_mode,
                                       float* gate, float* up, float* h, int8_t* h_qs, float* h_ds, float* y_rows,
                                       kq_stream_t stream);

/* out[t] = sum_k wts[t, k] * y[t * topk + k]  (fp32, slots in order k = 0..topk-1). */
kq_status_t kq_moe_combine(const float* y, const float* wts, int T, int topk, int H, float* out, kq_stream_t stream);

/* Debug / parity: int32 sumi[m, n, b] = sum_i q_w[n, b, i] * q_a[m, b, i] with
 * q_w the stored code (0..15 for q4_0/q4_1, int8 for q8_0), as the reference
 * forms it (gemm_ref.py:146, gemm_reference.h:200-211). */
kq_status_t kq_block_sums_i32(int wtype, const void* w, const void* a_q8_1, int32_t* sumi, int M, int N, int K,
                              kq_stream_t stream);

/* Flash-attention decode, harness semantics (see kq_flash_attn_q8_0). */
kq_status_t kq_fa_decode_q8_0_mha(const float* q, const void* k, const void* v, float* out, int B, int S, int H,
                                  int D, kq_stream_t stream);
/* The same for any KV format (KQ_KV_*): the status form of kq_flash_attn_q8_0,
 * kq_flash_attn_q4_0 and kq_flash_attn_f16. */
kq_status_t kq_fa_decode_mha(int kv_format, const float* q, const void* k, const void* v, float* out, int B, int S,
                             int H, int D, kq_stream_t stream);

/* Ragged GQA flash-decode over a q8_0 KV cache (benchmark configuration 3).
 * q fp16 [B, Hq, D]; k, v = q8_0 blocks of [total_rows, Hkv, D] (total_rows =
 * token rows allocated in the cache, >= cu_seqlens[B]); sequence b owns cache
 * rows cu_seqlens[b] .. cu_seqlens[b+1]-1 (int32, device); query head h reads
 * KV head h / (Hq / Hkv); fp32 softmax and accumulation; out fp16 [B, Hq, D].
 * max_seqlen bounds the per-sequence length (it sizes the split-KV grid).
 * An empty sequence yields zeros. */
kq_status_t kq_fa_decode_q8_0_ragged(const void* q_f16, const void* k, const void* v, const int32_t* cu_seqlens,
                                     int B, int Hq, int Hkv, int D, int max_seqlen, int total_rows, float scale,
                                     void* out_f16, kq_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* KQ_H */
