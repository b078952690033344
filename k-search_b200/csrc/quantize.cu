// Activation quantisation: fp32 rows -> q8_1 (reference byte layout) or the
// kernels' staging layout (int8 codes [M, K] + float2 (d, s) per block).
//
// Semantics follow llm_kernel_test/reference/quantize.py:165-214 exactly:
//   amax = max |x|, d = amax / 127 (IEEE fp32 division), d = 1 if amax == 0,
//   q = round_half_even(x / d) clamped to [-128, 127],
//   s = fp32 sum of the 32 values in numpy's pairwise order (8 strided
//       partial sums r[j] = x[j] + x[j+8] + x[j+16] + x[j+24], then
//       ((r0+r1)+(r2+r3)) + ((r4+r5)+(r6+r7)), then added to +0.0).
// The reference's GPU kernel (include/quantize.h:302-340) uses one thread per
// block, x * (1/d) and a serial sum; this one uses 8 lanes per block with
// 16-byte loads and reproduces the Python oracle bit for bit instead.
//
// Also RMSNorm (the harness's rms_norm operator, op_test_handler.py:641-690:
// out = x / sqrt(mean(x^2) + eps) * weight in fp32), alone and fused in front
// of the quantiser so a normalised activation row goes straight to q8_1.
#include <algorithm>

#include "kq_internal.h"
#include "kq_device.cuh"
#include "kq_quant.cuh"

namespace kq {
namespace {

// Where a block's 32 input values come from.
enum Src : int {
  SRC_X = 0,       // x[blk * 32 ..]
  SRC_GATHER = 1,  // row r of the output reads row rowmap[r] / div of x (K values per row)
  SRC_SILU = 2,    // silu(x[..]) * y[..] (x = gate, y = up), same indexing as SRC_X
};

template <int SRC>
__device__ __forceinline__ float4 load_octet(const float* __restrict__ x, const float* __restrict__ y,
                                             const int* __restrict__ rowmap, int div, int nb, long long blk,
                                             int sub) {
  if constexpr (SRC == SRC_GATHER) {
    const long long r = blk / nb, b = blk % nb;
    const long long src = (long long)(rowmap[r] / div) * nb + b;
    return __ldg(reinterpret_cast<const float4*>(x + src * 32) + sub);
  } else if constexpr (SRC == SRC_SILU) {
    const float4 g = __ldg(reinterpret_cast<const float4*>(x + blk * 32) + sub);
    const float4 u = __ldg(reinterpret_cast<const float4*>(y + blk * 32) + sub);
    return make_float4(silu_mul(g.x, u.x), silu_mul(g.y, u.y), silu_mul(g.z, u.z), silu_mul(g.w, u.w));
  } else {
    return __ldg(reinterpret_cast<const float4*>(x + blk * 32) + sub);
  }
}

// One warp quantises 4 consecutive blocks per step (grid-stride).
template <int MODE, bool BYTES, int SRC = SRC_X>
__global__ void __launch_bounds__(256) quantize_kernel(const float* __restrict__ x, int8_t* __restrict__ qs,
                                                       float2* __restrict__ ds, uint8_t* __restrict__ q81,
                                                       long long total_blocks, const float* __restrict__ y = nullptr,
                                                       const int* __restrict__ rowmap = nullptr, int div = 1,
                                                       int nb = 1) {
  const int lane = threadIdx.x & 31;
  const int grp = lane >> 3;
  const int sub = lane & 7;
  const long long nwarps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long b0 = ((long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * 4; b0 < total_blocks;
       b0 += nwarps * 4) {
    const long long blk = b0 + grp;
    const bool valid = blk < total_blocks;
    const long long src = valid ? blk : b0;  // keep all lanes in the shuffles
    const float4 v = load_octet<SRC>(x, y, rowmap, div, nb, src, sub);
    const BlockQ r = quantize_octet<MODE>(v, lane);
    if (!valid) continue;
    if (BYTES) {
      uint8_t* dst = q81 + blk * 36;
      reinterpret_cast<uint32_t*>(dst + 4)[sub] = r.qs;
      if (sub == 0) {
        const uint32_t ds16 = float_to_half_bits(r.d) | (float_to_half_bits(r.s) << 16);
        *reinterpret_cast<uint32_t*>(dst) = ds16;
      }
    } else {
      reinterpret_cast<uint32_t*>(qs + blk * 32)[sub] = r.qs;
      if (sub == 0) ds[blk] = staging_ds<MODE>(r);
    }
  }
  // Let a programmatic dependent (the GEMV) start its weight prefetch; it
  // reads these results only after griddepcontrol.wait.
  pdl_launch_dependents();
}

// q8_1 bytes [blocks, 36] -> staging layout. One thread per block.
// q8_1 bytes (36-byte blocks) -> staging. With a row map, output row r
// reads row rowmap[r] of a (nb blocks per row): the MoE expert pipeline's
// grouping of received q8_1 rows.
__global__ void __launch_bounds__(256) q8_1_to_act_kernel(const uint8_t* __restrict__ a, int8_t* __restrict__ qs,
                                                          float2* __restrict__ ds, long long total_blocks,
                                                          const int* __restrict__ rowmap = nullptr, int nb = 1) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < total_blocks) {
    const long long si = rowmap ? (long long)rowmap[i / nb] * nb + i % nb : i;
    const uint32_t* src = reinterpret_cast<const uint32_t*>(a + si * 36);
    const uint32_t h = src[0];
    uint4 lo = make_uint4(src[1], src[2], src[3], src[4]);
    uint4 hi = make_uint4(src[5], src[6], src[7], src[8]);
    uint4* dst = reinterpret_cast<uint4*>(qs + i * 32);
    dst[0] = lo;
    dst[1] = hi;
    ds[i] = make_float2(half_bits_to_float(h), half_bits_to_float(h >> 16));
  }
  pdl_launch_dependents();
}

// Weight / KV-cache quantisers, one warp per 32-value block, lane = element.
// Bit-exact with quantize.py:12-162 (division and round-half-even, not the
// reciprocal-multiply of include/quantize.h:221-294).
template <int WT>
__global__ void __launch_bounds__(256) quantize_rows_kernel(const float* __restrict__ x, uint8_t* __restrict__ y,
                                                            long long total_blocks) {
  const unsigned full = 0xffffffffu;
  const int lane = threadIdx.x & 31;
  const long long nwarps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long blk = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); blk < total_blocks;
       blk += nwarps) {
    const float v = x[blk * 32 + lane];
    if (WT == KQ_Q8_0) {
      float amax = fabsf(v);
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(full, amax, o));
      const float d = amax > 0.0f ? __fdiv_rn(amax, 127.0f) : 1.0f;
      const int q = max(-128, min(127, __float2int_rn(__fdiv_rn(v, d))));
      uint8_t* b = y + blk * 34;
      b[2 + lane] = (uint8_t)(q & 0xff);
      if (lane == 0) *reinterpret_cast<uint16_t*>(b) = (uint16_t)float_to_half_bits(d);
    } else {
      float lo = v, hi = v;
      if (WT == KQ_Q4_0) {
        lo = fabsf(v);
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) lo = fmaxf(lo, __shfl_xor_sync(full, lo, o));
      } else {
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) {
          lo = fminf(lo, __shfl_xor_sync(full, lo, o));
          hi = fmaxf(hi, __shfl_xor_sync(full, hi, o));
        }
      }
      float d;
      int q;
      if (WT == KQ_Q4_0) {
        d = lo > 0.0f ? __fdiv_rn(lo, 7.0f) : 1.0f;  // lo holds amax here
        q = max(0, min(15, __float2int_rn(__fadd_rn(__fdiv_rn(v, d), 8.0f))));
      } else {
        d = hi > lo ? __fdiv_rn(__fsub_rn(hi, lo), 15.0f) : 1.0f;
        q = max(0, min(15, __float2int_rn(__fdiv_rn(__fsub_rn(v, lo), d))));
      }
      const int qhi = __shfl_down_sync(full, q, 16);
      const int hdr = (WT == KQ_Q4_0) ? 2 : 4;
      uint8_t* b = y + blk * (WT == KQ_Q4_0 ? 18 : 20);
      if (lane < 16) b[hdr + lane] = (uint8_t)((q & 0x0F) | ((qhi & 0x0F) << 4));
      if (lane == 0) {
        reinterpret_cast<uint16_t*>(b)[0] = (uint16_t)float_to_half_bits(d);
        if (WT == KQ_Q4_1) reinterpret_cast<uint16_t*>(b)[1] = (uint16_t)float_to_half_bits(lo);
      }
    }
  }
}

int grid_for(long long total_blocks) {
  const long long warps = (total_blocks + 3) / 4;
  const long long ctas = (warps + 7) / 8;
  const long long cap = (long long)sm_count() * 8;
  return (int)std::max(1LL, std::min(ctas, cap));
}

// ---- RMSNorm -------------------------------------------------------------
// One CTA per row. rms = sqrt(sum(x^2) / K + eps) (fp32, correctly rounded
// divide and square root; the sum in this kernel's order), then x / rms * w
// with the harness's two roundings.
constexpr int kNormThreads = 256;

__device__ __forceinline__ float block_sum(float v, float* red) {
  const unsigned full = 0xffffffffu;
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(full, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.0f;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(full, v, o);
    if (lane == 0) red[32] = v;
  }
  __syncthreads();
  return red[32];
}

// VEC: K % 4 == 0 and 16-byte aligned rows (float4 loads).
template <bool VEC>
__device__ __forceinline__ float row_rms(const float* __restrict__ xr, int K, float eps, float* red) {
  float ss = 0.0f;
  if (VEC) {
    const float4* x4 = reinterpret_cast<const float4*>(xr);
    for (int i = threadIdx.x; i < K / 4; i += blockDim.x) {
      const float4 v = __ldg(x4 + i);
      ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, ss))));
    }
  } else {
    for (int i = threadIdx.x; i < K; i += blockDim.x) ss = fmaf(xr[i], xr[i], ss);
  }
  ss = block_sum(ss, red);
  return __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), eps));
}

__device__ __forceinline__ float norm1(float x, float rms, float w) { return __fmul_rn(__fdiv_rn(x, rms), w); }
__device__ __forceinline__ float4 norm4(float4 v, float rms, float4 w) {
  return make_float4(norm1(v.x, rms, w.x), norm1(v.y, rms, w.y), norm1(v.z, rms, w.z), norm1(v.w, rms, w.w));
}

template <bool VEC>
__global__ void __launch_bounds__(kNormThreads) rms_norm_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                                float* __restrict__ out, int K, float eps) {
  __shared__ float red[33];
  const size_t off = (size_t)blockIdx.x * K;
  const float rms = row_rms<VEC>(x + off, K, eps, red);
  if (VEC) {
    const float4* x4 = reinterpret_cast<const float4*>(x + off);
    const float4* w4 = reinterpret_cast<const float4*>(w);
    float4* o4 = reinterpret_cast<float4*>(out + off);
    for (int i = threadIdx.x; i < K / 4; i += blockDim.x) o4[i] = norm4(__ldg(x4 + i), rms, __ldg(w4 + i));
  } else {
    for (int i = threadIdx.x; i < K; i += blockDim.x) out[off + i] = norm1(x[off + i], rms, w[i]);
  }
}

// RMSNorm then q8_1 of the normalised row: staging layout (BYTES = false) or
// q8_1 bytes. K % 32 == 0, x and w 16-byte aligned. Each warp quantises 4
// blocks per step with the same per-block arithmetic as quantize_kernel.
template <int MODE, bool BYTES>
__global__ void __launch_bounds__(kNormThreads) rms_norm_quantize_kernel(const float* __restrict__ x,
                                                                         const float* __restrict__ w, float eps, int K,
                                                                         int8_t* __restrict__ qs,
                                                                         float2* __restrict__ ds,
                                                                         uint8_t* __restrict__ q81) {
  __shared__ float red[33];
  const size_t row = blockIdx.x;
  const float* xr = x + row * K;
  const float rms = row_rms<true>(xr, K, eps, red);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int grp = lane >> 3, sub = lane & 7;
  const int nb = K / 32;
  const int nwarps = blockDim.x >> 5;
  const float4* x4 = reinterpret_cast<const float4*>(xr);
  const float4* w4 = reinterpret_cast<const float4*>(w);
  for (int b0 = warp * 4; b0 < nb; b0 += nwarps * 4) {
    const int b = b0 + grp;
    const bool valid = b < nb;
    const int src = valid ? b : b0;  // keep all lanes in the shuffles
    const float4 v = norm4(__ldg(x4 + src * 8 + sub), rms, __ldg(w4 + src * 8 + sub));
    const BlockQ r = quantize_octet<MODE>(v, lane);
    if (!valid) continue;
    const long long blk = (long long)row * nb + b;
    if (BYTES) {
      uint8_t* dst = q81 + blk * 36;
      reinterpret_cast<uint32_t*>(dst + 4)[sub] = r.qs;
      if (sub == 0) *reinterpret_cast<uint32_t*>(dst) = float_to_half_bits(r.d) | (float_to_half_bits(r.s) << 16);
    } else {
      reinterpret_cast<uint32_t*>(qs + blk * 32)[sub] = r.qs;
      if (sub == 0) ds[blk] = staging_ds<MODE>(r);
    }
  }
  pdl_launch_dependents();
}

}  // namespace

kq_status_t launch_quantize_act(const float* x, Act8 act, int M, int K, int mode, cudaStream_t s) {
  const long long nb = (long long)M * (K / 32);
  if (nb == 0) return KQ_OK;
  const int grid = grid_for(nb);
  switch (mode) {
    case KQ_ACT_SUM_X:
      quantize_kernel<KQ_ACT_SUM_X, false><<<grid, 256, 0, s>>>(x, act.qs, act.ds, nullptr, nb);
      break;
    case KQ_ACT_SUM_DQ:
      quantize_kernel<KQ_ACT_SUM_DQ, false><<<grid, 256, 0, s>>>(x, act.qs, act.ds, nullptr, nb);
      break;
    case KQ_ACT_F32:
      quantize_kernel<KQ_ACT_F32, false><<<grid, 256, 0, s>>>(x, act.qs, act.ds, nullptr, nb);
      break;
    default:
      return fail(KQ_ERR_INVALID, "unknown activation mode %d", mode);
  }
  return check_launch("quantize_act");
}

kq_status_t launch_quantize_q8_1_bytes(const float* x, void* y, int64_t M, int64_t K, int mode, cudaStream_t s) {
  const long long nb = (long long)M * (K / 32);
  if (nb == 0) return KQ_OK;
  const int grid = grid_for(nb);
  uint8_t* out = static_cast<uint8_t*>(y);
  switch (mode) {
    case KQ_ACT_SUM_X:
      quantize_kernel<KQ_ACT_SUM_X, true><<<grid, 256, 0, s>>>(x, nullptr, nullptr, out, nb);
      break;
    case KQ_ACT_SUM_DQ:
      quantize_kernel<KQ_ACT_SUM_DQ, true><<<grid, 256, 0, s>>>(x, nullptr, nullptr, out, nb);
      break;
    default:
      return fail(KQ_ERR_INVALID, "q8_1 bytes hold fp16 d and s: sum_mode must be KQ_ACT_SUM_X or KQ_ACT_SUM_DQ");
  }
  return check_launch("quantize_q8_1");
}

kq_status_t launch_quantize_rows(int wtype, const float* x, void* y, int64_t rows, int64_t K, cudaStream_t s) {
  const long long nb = (long long)rows * (K / 32);
  if (nb == 0) return KQ_OK;
  const int grid = (int)std::min<long long>((nb + 7) / 8, (long long)sm_count() * 16);
  uint8_t* out = static_cast<uint8_t*>(y);
  switch (wtype) {
    case KQ_Q4_0: quantize_rows_kernel<KQ_Q4_0><<<grid, 256, 0, s>>>(x, out, nb); break;
    case KQ_Q4_1: quantize_rows_kernel<KQ_Q4_1><<<grid, 256, 0, s>>>(x, out, nb); break;
    case KQ_Q8_0: quantize_rows_kernel<KQ_Q8_0><<<grid, 256, 0, s>>>(x, out, nb); break;
    default: return fail(KQ_ERR_INVALID, "unknown weight type %d", wtype);
  }
  return check_launch("quantize_rows");
}

template <int SRC>
kq_status_t launch_staging(const float* x, const float* y, const int* rowmap, int div, Act8 act, int M, int K, int mode,
                           cudaStream_t s) {
  const long long nb = (long long)M * (K / 32);
  if (nb == 0) return KQ_OK;
  const int grid = grid_for(nb);
  const int nbr = K / 32;
  switch (mode) {
    case KQ_ACT_SUM_X:
      quantize_kernel<KQ_ACT_SUM_X, false, SRC><<<grid, 256, 0, s>>>(x, act.qs, act.ds, nullptr, nb, y, rowmap, div, nbr);
      break;
    case KQ_ACT_SUM_DQ:
      quantize_kernel<KQ_ACT_SUM_DQ, false, SRC><<<grid, 256, 0, s>>>(x, act.qs, act.ds, nullptr, nb, y, rowmap, div, nbr);
      break;
    case KQ_ACT_F32:
      quantize_kernel<KQ_ACT_F32, false, SRC><<<grid, 256, 0, s>>>(x, act.qs, act.ds, nullptr, nb, y, rowmap, div, nbr);
      break;
    default:
      return fail(KQ_ERR_INVALID, "unknown activation mode %d", mode);
  }
  return check_launch("quantize_staging");
}

kq_status_t launch_quantize_act_gather(const float* x, const int* rowmap, int div, Act8 act, int M, int K, int mode,
                                       cudaStream_t s) {
  return launch_staging<SRC_GATHER>(x, nullptr, rowmap, div, act, M, K, mode, s);
}

kq_status_t launch_silu_mul_quantize(const float* gate, const float* up, Act8 act, int M, int K, int mode,
                                     cudaStream_t s) {
  return launch_staging<SRC_SILU>(gate, up, nullptr, 1, act, M, K, mode, s);
}

kq_status_t launch_q8_1_to_act(const void* a_q8_1, Act8 act, int M, int K, cudaStream_t s) {
  const long long nb = (long long)M * (K / 32);
  if (nb == 0) return KQ_OK;
  const int grid = (int)((nb + 255) / 256);
  q8_1_to_act_kernel<<<grid, 256, 0, s>>>(static_cast<const uint8_t*>(a_q8_1), act.qs, act.ds, nb);
  return check_launch("q8_1_to_act");
}

kq_status_t launch_q8_1_to_act_gather(const void* a_q8_1, const int* rowmap, Act8 act, int M, int K, cudaStream_t s) {
  const long long total = (long long)M * (K / 32);
  if (total == 0) return KQ_OK;
  const int grid = (int)((total + 255) / 256);
  q8_1_to_act_kernel<<<grid, 256, 0, s>>>(static_cast<const uint8_t*>(a_q8_1), act.qs, act.ds, total, rowmap,
                                          K / 32);
  return check_launch("q8_1_to_act_gather");
}

kq_status_t launch_rms_norm(const float* x, const float* w, float* out, int M, int K, float eps, cudaStream_t s) {
  if ((long long)M * K == 0) return KQ_OK;
  const bool vec = K % 4 == 0 && ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) |
                                   reinterpret_cast<uintptr_t>(out)) & 15) == 0;
  if (vec)
    rms_norm_kernel<true><<<M, kNormThreads, 0, s>>>(x, w, out, K, eps);
  else
    rms_norm_kernel<false><<<M, kNormThreads, 0, s>>>(x, w, out, K, eps);
  return check_launch("rms_norm");
}

kq_status_t launch_rms_norm_quantize(const float* x, const float* w, float eps, Act8 act, void* q81, int M, int K,
                                     int mode, cudaStream_t s) {
  if ((long long)M * K == 0) return KQ_OK;
  uint8_t* y = static_cast<uint8_t*>(q81);
  const bool bytes = y != nullptr;
  switch (mode) {
    case KQ_ACT_SUM_X:
      if (bytes)
        rms_norm_quantize_kernel<KQ_ACT_SUM_X, true><<<M, kNormThreads, 0, s>>>(x, w, eps, K, nullptr, nullptr, y);
      else
        rms_norm_quantize_kernel<KQ_ACT_SUM_X, false><<<M, kNormThreads, 0, s>>>(x, w, eps, K, act.qs, act.ds, nullptr);
      break;
    case KQ_ACT_SUM_DQ:
      if (bytes)
        rms_norm_quantize_kernel<KQ_ACT_SUM_DQ, true><<<M, kNormThreads, 0, s>>>(x, w, eps, K, nullptr, nullptr, y);
      else
        rms_norm_quantize_kernel<KQ_ACT_SUM_DQ, false><<<M, kNormThreads, 0, s>>>(x, w, eps, K, act.qs, act.ds, nullptr);
      break;
    case KQ_ACT_F32:
      if (bytes) return fail(KQ_ERR_INVALID, "q8_1 bytes hold fp16 d and s: sum_mode must be KQ_ACT_SUM_X or KQ_ACT_SUM_DQ");
      rms_norm_quantize_kernel<KQ_ACT_F32, false><<<M, kNormThreads, 0, s>>>(x, w, eps, K, act.qs, act.ds, nullptr);
      break;
    default:
      return fail(KQ_ERR_INVALID, "unknown activation mode %d", mode);
  }
  return check_launch("rms_norm_quantize");
}

}  // namespace kq
