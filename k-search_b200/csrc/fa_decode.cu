// Flash-attention decode over a q8_0 KV cache (split-KV "flash decoding").
//
// Semantics: the harness flash_attention operator
// (kernelevalplus-main/llm_kernel_test/op_test_handler.py:543-563):
// out = softmax(q . K^T / sqrt(D)) . V per (query, head), with K and V stored
// as q8_0 blocks along head_dim (op_test_handler.py:489-508), dequantised as
// x = q * d. The ragged GQA form (one KV stream per (sequence, KV head),
// shared by Hq/Hkv query heads) follows the same arithmetic.
//
// Structure: pass 1 gives every (KV stream, token chunk, query group) to one
// CTA, one warp per query; each warp keeps an online-softmax state (running
// max in the log2 domain, running sum, fp32 accumulator) and writes it as a
// partial. Pass 2 merges the partials of each query. Lanes own head-dim
// elements {32 j + lane}, so every q8_0 block row is read as 32 consecutive
// bytes by the warp.
#include <algorithm>
#include <cmath>

#include "kq_internal.h"
#include "kq_device.cuh"

namespace kq {
namespace {

constexpr int kQPerCta = 4;  // queries (warps) per CTA
constexpr int kMaxDJ = 8;    // head_dim <= 256

struct FaParams {
  const void* q;
  const uint8_t* k;
  const uint8_t* v;
  const int32_t* cu;  // ragged only
  float* pm;          // [Q][NC] running max (log2 domain)
  float* pl;          // [Q][NC] running sum
  float* pacc;        // [Q][NC][D]
  void* out;
  int B, H, Hkv, D, S, NC, chunk;
  float qscale;  // softmax scale * log2(e)
};

__device__ __forceinline__ float load_q(const float* q, size_t i) { return q[i]; }
__device__ __forceinline__ float load_q(const __half* q, size_t i) { return __half2float(q[i]); }
__device__ __forceinline__ void store_o(float* o, size_t i, float v) { o[i] = v; }
__device__ __forceinline__ void store_o(__half* o, size_t i, float v) { o[i] = __float2half_rn(v); }

// RAGGED = false: grid (NC, H, ceil(B/4)); queries b of head h share KV head h.
// RAGGED = true:  grid (NC, B*Hkv, ceil(g/4)); query heads of KV head hk.
template <typename QT, bool RAGGED>
__global__ void __launch_bounds__(32 * kQPerCta) fa_partial_kernel(FaParams p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x;
  const int dj = p.D / 32;
  const size_t row_bytes = (size_t)dj * 34;

  int qg, L, row0, row_stride;  // query index, stream length, first KV row, rows per token
  if (!RAGGED) {
    const int h = blockIdx.y;
    const int b = blockIdx.z * kQPerCta + warp;
    if (b >= p.B) return;
    qg = b * p.H + h;
    L = p.S;
    row0 = h;
    row_stride = p.H;
  } else {
    const int b = blockIdx.y / p.Hkv, hk = blockIdx.y % p.Hkv;
    const int g = p.H / p.Hkv;
    const int j = blockIdx.z * kQPerCta + warp;
    if (j >= g) return;
    qg = b * p.H + hk * g + j;
    const int s0 = p.cu[b];
    L = p.cu[b + 1] - s0;
    row0 = s0 * p.Hkv + hk;
    row_stride = p.Hkv;
  }

  float qv[kMaxDJ], acc[kMaxDJ];
  const QT* q = static_cast<const QT*>(p.q) + (size_t)qg * p.D;
#pragma unroll
  for (int j = 0; j < kMaxDJ; ++j) {
    qv[j] = (j < dj) ? load_q(q, (size_t)j * 32 + lane) * p.qscale : 0.0f;
    acc[j] = 0.0f;
  }
  float m = -INFINITY, l = 0.0f;
  const int t0 = c * p.chunk, t1 = min(L, t0 + p.chunk);
  for (int t = t0; t < t1; ++t) {
    const size_t row = (size_t)row0 + (size_t)t * row_stride;
    const uint8_t* kb = p.k + row * row_bytes;
    const uint8_t* vb = p.v + row * row_bytes;
    float s = 0.0f;
#pragma unroll
    for (int j = 0; j < kMaxDJ; ++j) {
      if (j < dj) {
        const float d = half_bits_to_float(*reinterpret_cast<const uint16_t*>(kb + j * 34));
        const float kq = (float)(int8_t)kb[j * 34 + 2 + lane];
        s = fmaf(d, qv[j] * kq, s);
      }
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mn = fmaxf(m, s);
    const float corr = exp2f(m - mn);
    const float pr = exp2f(s - mn);
    l = fmaf(l, corr, pr);
#pragma unroll
    for (int j = 0; j < kMaxDJ; ++j) {
      if (j < dj) {
        const float d = half_bits_to_float(*reinterpret_cast<const uint16_t*>(vb + j * 34));
        const float vq = (float)(int8_t)vb[j * 34 + 2 + lane];
        acc[j] = fmaf(acc[j], corr, pr * d * vq);
      }
    }
    m = mn;
  }
  const size_t pi = (size_t)qg * p.NC + c;
  if (lane == 0) {
    p.pm[pi] = m;
    p.pl[pi] = l;
  }
#pragma unroll
  for (int j = 0; j < kMaxDJ; ++j)
    if (j < dj) p.pacc[pi * p.D + j * 32 + lane] = acc[j];
}

// One warp per query: merge the NC partial states.
template <typename OT>
__global__ void __launch_bounds__(128) fa_combine_kernel(FaParams p, int Q) {
  const int qg = blockIdx.x * 4 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (qg >= Q) return;
  const int dj = p.D / 32;
  float M = -INFINITY;
  for (int c = 0; c < p.NC; ++c) M = fmaxf(M, p.pm[(size_t)qg * p.NC + c]);
  float acc[kMaxDJ] = {};
  float L = 0.0f;
  if (M != -INFINITY) {
    for (int c = 0; c < p.NC; ++c) {
      const size_t pi = (size_t)qg * p.NC + c;
      const float mc = p.pm[pi];
      if (mc == -INFINITY) continue;
      const float w = exp2f(mc - M);
      L = fmaf(p.pl[pi], w, L);
#pragma unroll
      for (int j = 0; j < kMaxDJ; ++j)
        if (j < dj) acc[j] = fmaf(p.pacc[pi * p.D + j * 32 + lane], w, acc[j]);
    }
  }
  const float inv = L > 0.0f ? 1.0f / L : 0.0f;
  OT* o = static_cast<OT*>(p.out) + (size_t)qg * p.D;
#pragma unroll
  for (int j = 0; j < kMaxDJ; ++j)
    if (j < dj) store_o(o, (size_t)j * 32 + lane, acc[j] * inv);
}

// Choose the number of chunks so the partial buffers stay within `budget`.
int choose_chunks(long long Q, int D, int max_len, size_t budget, int* chunk) {
  int nc = std::max(1, (max_len + 255) / 256);
  const long long per = (long long)Q * (D + 2) * 4;
  const long long cap = std::max<long long>(1, (long long)budget / std::max<long long>(per, 1));
  nc = (int)std::min<long long>(nc, cap);
  nc = std::min(nc, 65535);
  *chunk = std::max(1, (max_len + nc - 1) / nc);
  nc = std::max(1, (max_len + *chunk - 1) / *chunk);
  return nc;
}

constexpr size_t kPartialBudget = 64ull << 20;

}  // namespace

kq_status_t launch_fa_mha(const float* q, const void* k, const void* v, float* out, int B, int S, int H, int D,
                          cudaStream_t s) {
  const long long Q = (long long)B * H;
  if (Q == 0) return KQ_OK;
  int chunk = 0;
  const int NC = choose_chunks(Q, D, std::max(S, 1), kPartialBudget, &chunk);
  const size_t bytes = (size_t)Q * NC * (D + 2) * sizeof(float);
  float* ws = static_cast<float*>(workspace(WS_FA, bytes));
  if (!ws) return KQ_ERR_NOMEM;
  FaParams p{};
  p.q = q; p.k = static_cast<const uint8_t*>(k); p.v = static_cast<const uint8_t*>(v); p.cu = nullptr;
  p.pm = ws; p.pl = ws + Q * NC; p.pacc = ws + 2 * Q * NC; p.out = out;
  p.B = B; p.H = H; p.Hkv = H; p.D = D; p.S = S; p.NC = NC; p.chunk = chunk;
  p.qscale = (float)(1.0 / std::sqrt((double)D) * 1.4426950408889634);
  dim3 grid(NC, H, (B + kQPerCta - 1) / kQPerCta);
  if (grid.z > 65535 || grid.y > 65535) return fail(KQ_ERR_UNSUPPORTED, "fa_mha: grid too large");
  fa_partial_kernel<float, false><<<grid, 32 * kQPerCta, 0, s>>>(p);
  kq_status_t st = check_launch("fa_partial(mha)");
  if (st) return st;
  fa_combine_kernel<float><<<(unsigned)((Q + 3) / 4), 128, 0, s>>>(p, (int)Q);
  return check_launch("fa_combine(mha)");
}

kq_status_t launch_fa_ragged(const void* q, const void* k, const void* v, const int32_t* cu, int B, int Hq, int Hkv,
                             int D, int max_seqlen, float scale, void* out, cudaStream_t s) {
  const long long Q = (long long)B * Hq;
  if (Q == 0) return KQ_OK;
  int chunk = 0;
  const int NC = choose_chunks(Q, D, std::max(max_seqlen, 1), kPartialBudget, &chunk);
  const size_t bytes = (size_t)Q * NC * (D + 2) * sizeof(float);
  float* ws = static_cast<float*>(workspace(WS_FA, bytes));
  if (!ws) return KQ_ERR_NOMEM;
  FaParams p{};
  p.q = q; p.k = static_cast<const uint8_t*>(k); p.v = static_cast<const uint8_t*>(v); p.cu = cu;
  p.pm = ws; p.pl = ws + Q * NC; p.pacc = ws + 2 * Q * NC; p.out = out;
  p.B = B; p.H = Hq; p.Hkv = Hkv; p.D = D; p.S = max_seqlen; p.NC = NC; p.chunk = chunk;
  p.qscale = (float)((double)scale * 1.4426950408889634);
  const int g = Hq / Hkv;
  dim3 grid(NC, (unsigned)((long long)B * Hkv), (g + kQPerCta - 1) / kQPerCta);
  if (grid.y > 65535) return fail(KQ_ERR_UNSUPPORTED, "fa_ragged: B*Hkv too large");
  fa_partial_kernel<__half, true><<<grid, 32 * kQPerCta, 0, s>>>(p);
  kq_status_t st = check_launch("fa_partial(ragged)");
  if (st) return st;
  fa_combine_kernel<__half><<<(unsigned)((Q + 3) / 4), 128, 0, s>>>(p, (int)Q);
  return check_launch("fa_combine(ragged)");
}

}  // namespace kq
