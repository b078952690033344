// Generic quantised GEMM (any M, N; K % 32 == 0; weights 2-byte aligned) and
// the int32 block-sum parity kernel. CUDA cores, dp4a.
//
// This is the shape-generic path (odd K, unaligned weight slices) and the
// cross-check for the tensor-core GEMMs; the hot paths are gemv.cu (M <= 8)
// and gemm_split.cu (M > 8, tcgen05; gemm_tc.cu is the int8 alternative).
// Formulas: gemm_ref.py:100-153 (q4_0), :274-331 (q4_1),
// gemm_reference.h:311-336 (q8_0).
#include <algorithm>

#include "kq_internal.h"
#include "kq_device.cuh"

namespace kq {
namespace {

constexpr int BM = 32, BN = 64;

// Unpack one weight block (BB bytes at a 2-byte aligned address) into 8 code
// words matched to the activation words (word k pairs with activation word
// k): q8_0 -> the 8 int8 words; q4_x -> words 0..3 = low nibbles (elements
// 0..15), words 4..7 = high nibbles (elements 16..31).
template <int WT>
__device__ __forceinline__ void unpack_block(const uint8_t* p, uint32_t (&q)[8], float& d, float& m) {
  const uint16_t* h = reinterpret_cast<const uint16_t*>(p);
  d = half_bits_to_float(h[0]);
  m = 0.0f;
  if constexpr (WT == KQ_Q8_0) {
#pragma unroll
    for (int k = 0; k < 8; ++k) q[k] = (uint32_t)h[1 + 2 * k] | ((uint32_t)h[2 + 2 * k] << 16);
  } else {
    const int o = (WT == KQ_Q4_0) ? 1 : 2;
    if constexpr (WT == KQ_Q4_1) m = half_bits_to_float(h[1]);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t v = (uint32_t)h[o + 2 * k] | ((uint32_t)h[o + 2 * k + 1] << 16);
      q[k] = v & 0x0F0F0F0Fu;
      q[k + 4] = (v >> 4) & 0x0F0F0F0Fu;
    }
  }
}

template <int WT>
__global__ void __launch_bounds__(256) gemm_simt_kernel(const uint8_t* __restrict__ w, const int8_t* __restrict__ aqs,
                                                        const float2* __restrict__ ads, float* __restrict__ out, int M,
                                                        int N, int K) {
  constexpr int BB = (WT == KQ_Q4_0) ? 18 : (WT == KQ_Q4_1) ? 20 : 34;
  __shared__ uint32_t sa[BM][9];
  __shared__ float sad[BM], sas[BM];
  __shared__ uint32_t sw[BN][9];
  __shared__ float swd[BN], swm[BN];
  const int nb = K / 32;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  const int tid = threadIdx.x;
  const int ty = tid / 16, tx = tid % 16;
  float acc[2][4] = {};
  for (int b = 0; b < nb; ++b) {
    {
      const int r = tid / 8, k = tid % 8;
      const int m = m0 + r;
      sa[r][k] = (m < M) ? reinterpret_cast<const uint32_t*>(aqs + (size_t)m * K + (size_t)b * 32)[k] : 0u;
      if (tid < BM) {
        const float2 v = (m0 + tid < M) ? ads[(size_t)(m0 + tid) * nb + b] : make_float2(0.f, 0.f);
        sad[tid] = v.x;
        sas[tid] = v.y;
      }
    }
    if (tid < BN) {
      const int n = n0 + tid;
      uint32_t q[8] = {};
      float d = 0.f, mm = 0.f;
      if (n < N) unpack_block<WT>(w + ((size_t)n * nb + b) * BB, q, d, mm);
#pragma unroll
      for (int k = 0; k < 8; ++k) sw[tid][k] = q[k];
      swd[tid] = d;
      swm[tid] = mm;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int r = ty + 16 * i;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c = tx + 16 * j;
        int s = 0;
#pragma unroll
        for (int k = 0; k < 8; ++k) s = __dp4a((int)sw[c][k], (int)sa[r][k], s);
        if (WT == KQ_Q4_0) {
          acc[i][j] = fmaf(swd[c], fmaf(sad[r], (float)s, -8.0f * sas[r]), acc[i][j]);
        } else if (WT == KQ_Q4_1) {
          acc[i][j] = fmaf(swd[c] * sad[r], (float)s, fmaf(swm[c], sas[r], acc[i][j]));
        } else {
          acc[i][j] = fmaf(swd[c] * sad[r], (float)s, acc[i][j]);
        }
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int m = m0 + ty + 16 * i;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx + 16 * j;
      if (m < M && n < N) out[(size_t)m * N + n] = acc[i][j];
    }
  }
}

// sumi[m, n, b]: one thread per output, straight from the reference byte layouts.
template <int WT>
__global__ void __launch_bounds__(256) block_sums_kernel(const uint8_t* __restrict__ w, const uint8_t* __restrict__ a,
                                                         int32_t* __restrict__ sumi, int M, int N, int K) {
  constexpr int BB = (WT == KQ_Q4_0) ? 18 : (WT == KQ_Q4_1) ? 20 : 34;
  const int nb = K / 32;
  const long long total = (long long)M * N * nb;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int b = (int)(i % nb);
    const long long mn = i / nb;
    const int n = (int)(mn % N);
    const int m = (int)(mn / N);
    uint32_t q[8];
    float d, mm;
    unpack_block<WT>(w + ((size_t)n * nb + b) * BB, q, d, mm);
    const uint32_t* av = reinterpret_cast<const uint32_t*>(a + ((size_t)m * nb + b) * 36 + 4);
    int s = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) s = __dp4a((int)q[k], (int)av[k], s);
    sumi[i] = s;
  }
}

}  // namespace

kq_status_t launch_gemm_simt(int wtype, const void* w, Act8 act, float* out, int M, int N, int K, cudaStream_t s) {
  if (reinterpret_cast<uintptr_t>(w) % 2 != 0) return fail(KQ_ERR_INVALID, "weight pointer must be 2-byte aligned");
  dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM);
  if (grid.y > 65535) return fail(KQ_ERR_UNSUPPORTED, "M too large for the generic GEMM (%d)", M);
  const uint8_t* wp = static_cast<const uint8_t*>(w);
  switch (wtype) {
    case KQ_Q4_0: gemm_simt_kernel<KQ_Q4_0><<<grid, 256, 0, s>>>(wp, act.qs, act.ds, out, M, N, K); break;
    case KQ_Q4_1: gemm_simt_kernel<KQ_Q4_1><<<grid, 256, 0, s>>>(wp, act.qs, act.ds, out, M, N, K); break;
    case KQ_Q8_0: gemm_simt_kernel<KQ_Q8_0><<<grid, 256, 0, s>>>(wp, act.qs, act.ds, out, M, N, K); break;
    default: return fail(KQ_ERR_INVALID, "unknown weight type %d", wtype);
  }
  return check_launch("gemm_simt");
}

kq_status_t launch_block_sums(int wtype, const void* w, const void* a_q8_1, int32_t* sumi, int M, int N, int K,
                              cudaStream_t s) {
  if (reinterpret_cast<uintptr_t>(w) % 2 != 0 || reinterpret_cast<uintptr_t>(a_q8_1) % 4 != 0)
    return fail(KQ_ERR_INVALID, "block_sums: weight must be 2-byte and activation 4-byte aligned");
  const long long total = (long long)M * N * (K / 32);
  if (total == 0) return KQ_OK;
  const int grid = (int)std::min<long long>((total + 255) / 256, (long long)sm_count() * 16);
  const uint8_t* wp = static_cast<const uint8_t*>(w);
  const uint8_t* ap = static_cast<const uint8_t*>(a_q8_1);
  switch (wtype) {
    case KQ_Q4_0: block_sums_kernel<KQ_Q4_0><<<grid, 256, 0, s>>>(wp, ap, sumi, M, N, K); break;
    case KQ_Q4_1: block_sums_kernel<KQ_Q4_1><<<grid, 256, 0, s>>>(wp, ap, sumi, M, N, K); break;
    case KQ_Q8_0: block_sums_kernel<KQ_Q8_0><<<grid, 256, 0, s>>>(wp, ap, sumi, M, N, K); break;
    default: return fail(KQ_ERR_INVALID, "unknown weight type %d", wtype);
  }
  return check_launch("block_sums");
}

}  // namespace kq
