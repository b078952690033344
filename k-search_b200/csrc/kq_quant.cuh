// The activation quantiser's per-block step, shared by every kernel that
// quantises fp32 activations to q8_1 (the quantiser kernels, and the
// single-launch GEMV that quantises its own copy of the row): one definition,
// so every path produces the same codes and sums bit for bit.
//
// Semantics follow llm_kernel_test/reference/quantize.py:165-214 exactly:
//   amax = max |x|, d = amax / 127 (IEEE fp32 division), d = 1 if amax == 0,
//   q = round_half_even(x / d) clamped to [-128, 127],
//   s = fp32 sum of the 32 values in numpy's pairwise order.
#pragma once

#include "kq_device.cuh"
#include "kq.h"

namespace kq {

struct BlockQ {
  uint32_t qs;  // this lane's 4 codes, packed little endian
  float d;      // fp32 scale (unrounded)
  float s;      // fp32 sum per mode (unrounded)
};

// 8 lanes (an aligned octet of the warp) quantise one 32-value block per
// element of v[]; lane `sub` holds values 4*sub .. 4*sub+3 of each. All 32
// lanes must call this. The U blocks go through each step together, so their
// independent shuffle / divide chains overlap; each block's arithmetic is the
// same whatever U is.
template <int MODE, int U>
__device__ __forceinline__ void quantize_octets(const float4 (&v)[U], int lane, BlockQ (&r)[U]) {
  const unsigned full = 0xffffffffu;
  const int sub = lane & 7;
  const int base = lane & ~7;

  float amax[U], d[U];
#pragma unroll
  for (int u = 0; u < U; ++u)
    amax[u] = fmaxf(fmaxf(fabsf(v[u].x), fabsf(v[u].y)), fmaxf(fabsf(v[u].z), fabsf(v[u].w)));
#pragma unroll
  for (int o = 1; o <= 4; o <<= 1) {
#pragma unroll
    for (int u = 0; u < U; ++u) amax[u] = fmaxf(amax[u], __shfl_xor_sync(full, amax[u], o));
  }
#pragma unroll
  for (int u = 0; u < U; ++u) d[u] = amax[u] > 0.0f ? __fdiv_rn(amax[u], 127.0f) : 1.0f;

  int q[U][4];
#pragma unroll
  for (int u = 0; u < U; ++u) {
    q[u][0] = max(-128, min(127, __float2int_rn(__fdiv_rn(v[u].x, d[u]))));
    q[u][1] = max(-128, min(127, __float2int_rn(__fdiv_rn(v[u].y, d[u]))));
    q[u][2] = max(-128, min(127, __float2int_rn(__fdiv_rn(v[u].z, d[u]))));
    q[u][3] = max(-128, min(127, __float2int_rn(__fdiv_rn(v[u].w, d[u]))));
    r[u].qs = (uint32_t)(q[u][0] & 0xff) | ((uint32_t)(q[u][1] & 0xff) << 8) | ((uint32_t)(q[u][2] & 0xff) << 16) |
              ((uint32_t)(q[u][3] & 0xff) << 24);
    r[u].d = d[u];
  }

  if (MODE == KQ_ACT_SUM_DQ) {
    int sq[U];
#pragma unroll
    for (int u = 0; u < U; ++u) sq[u] = q[u][0] + q[u][1] + q[u][2] + q[u][3];
#pragma unroll
    for (int o = 1; o <= 4; o <<= 1) {
#pragma unroll
      for (int u = 0; u < U; ++u) sq[u] += __shfl_xor_sync(full, sq[u], o);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const float dh = __half2float(__float2half_rn(d[u]));
      r[u].s = __fmul_rn(dh, (float)sq[u]);
    }
  } else {
    // numpy pairwise order. Value j of the block is lane j/4, component j%4.
    // Lanes sub=0 and sub=1 build r[4*sub + c] = x[4sub+c] + x[4sub+c+8]
    // + x[4sub+c+16] + x[4sub+c+24] (lanes sub, sub+2, sub+4, sub+6).
    const int a = sub & 1;
    float t[U][4];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      t[u][0] = v[u].x;
      t[u][1] = v[u].y;
      t[u][2] = v[u].z;
      t[u][3] = v[u].w;
    }
#pragma unroll
    for (int k = 1; k < 4; ++k) {
      const int src = base + a + 2 * k;
#pragma unroll
      for (int u = 0; u < U; ++u) {
        t[u][0] = __fadd_rn(t[u][0], __shfl_sync(full, v[u].x, src));
        t[u][1] = __fadd_rn(t[u][1], __shfl_sync(full, v[u].y, src));
        t[u][2] = __fadd_rn(t[u][2], __shfl_sync(full, v[u].z, src));
        t[u][3] = __fadd_rn(t[u][3], __shfl_sync(full, v[u].w, src));
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const float p = __fadd_rn(__fadd_rn(t[u][0], t[u][1]), __fadd_rn(t[u][2], t[u][3]));
      const float other = __shfl_xor_sync(full, p, 1);
      // lane sub=0 holds the left half of the final addition, sub=1 the right.
      const float res = (a == 0) ? __fadd_rn(p, other) : __fadd_rn(other, p);
      r[u].s = __shfl_sync(full, __fadd_rn(res, 0.0f), base);
    }
  }
}

// One block per call (see quantize_octets).
template <int MODE>
__device__ __forceinline__ BlockQ quantize_octet(float4 v, int lane) {
  const float4 vv[1] = {v};
  BlockQ r[1];
  quantize_octets<MODE, 1>(vv, lane, r);
  return r[0];
}

// The staging layout's (d, s) pair for a quantised block: fp32 in the
// KQ_ACT_F32 mode, else rounded through fp16 as the q8_1 bytes hold them.
template <int MODE>
__device__ __forceinline__ float2 staging_ds(const BlockQ& r) {
  if (MODE == KQ_ACT_F32) return make_float2(r.d, r.s);
  return make_float2(__half2float(__float2half_rn(r.d)), __half2float(__float2half_rn(r.s)));
}

}  // namespace kq
