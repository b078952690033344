// Flash attention for the harness form with many queries per head over a
// q8_0 KV cache (D = 128): the harness flash_attention operator
// (kernelevalplus-main/llm_kernel_test/op_test_handler.py:543-563) shares one
// [S, H, D] cache across all B queries of a head, so at B = 512 a head is a
// GEMM pair (S = Q K^T, O = softmax(S) V) rather than a stream of the cache.
//
// CTA = 4 warps over 64 queries of one head (16 per warp); it walks the
// cache in 64-token tiles:
//  * a TMA ring (two stages) brings the raw q8_0 rows of the head (boxes of
//    64 rows x 144 bytes: the head's 136-byte row 0 or 8 bytes in);
//  * QK is exact on the raw K codes (mma.m16n8k32 s8, one MMA per 32-dim
//    block and query level): the query q * scale * log2(e) is held as two int8
//    levels (q ~ s1 c1 + s2 c2, s2 = s1 / 127, so 127 dot1 + dot2 is the exact
//    block dot at scale s2), and the fp32 epilogue applies each (token, block)
//    K scale, as the decode kernels do;
//  * the CTA dequantises each V tile once into fp16 in shared memory, as a
//    high part and its fp16 remainder (hi + lo carries ~22 bits of code * d);
//  * online softmax per query row in registers (exp2), and P = p as fp16
//    plus its fp16 remainder, taken straight from the S accumulators as the
//    A operand of the PV products: O += P_hi V_hi + P_lo V_hi + P_hi V_lo.
// Precision, from an fp64 emulation of each arithmetic against the oracle
// (worst |error| / per-element bar): fp16 Q, K, P and V each rounded once
// misses the bar on a few elements; with fp16 remainders on three of the four
// operands 0.71-0.78 (still 1 miss in 2.1 M elements on the GPU), on all four
// 0.003 (three f16 products per GEMM); this kernel's int8 QK with P and V
// split 0.15-0.20.
#include <cuda.h>

#include <algorithm>
#include <cmath>

#include "kq_internal.h"
#include "kq_device.cuh"

namespace kq {
namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

constexpr int kWarps = 4;
constexpr int kQTile = 16 * kWarps;      // queries per CTA
constexpr int kTTile = 64;               // tokens per tile
constexpr int kStages = 2;
constexpr int kRawRow = 144;             // raw smem row: 136 bytes of the head (+8 before or after)
constexpr int kRawTile = kTTile * kRawRow;          // 9216 bytes
constexpr int kHPitch = 272;             // fp16 tile row: 256 bytes + 16 (ldmatrix rows in distinct banks)
constexpr int kHTile = kTTile * kHPitch;            // 17408 bytes
constexpr int kOffRawV = kStages * kRawTile;
constexpr int kOffVh = 2 * kStages * kRawTile;
constexpr int kOffVl = kOffVh + kHTile;
constexpr int kOffDk = kOffVl + kHTile;               // K block scales of the tile, fp32 [4 blocks][64 tokens]
constexpr int kOffBar = kOffDk + 4 * kTTile * 4;
constexpr int kSmem = kOffBar + kStages * 8 + 128;  // + base alignment slack
static_assert(kRawTile % 128 == 0 && kOffVh % 128 == 0 && kHTile % 128 == 0, "aligned tiles");

struct BatchParams {
  const float* q;   // [B, H, 128]
  float* out;       // [B, H, 128]
  int* err;
  int B, H, S;
  float qscale;     // softmax scale * log2(e)
};

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mma_f16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%10, %10, %10, %10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0));
}

__device__ __forceinline__ uint32_t pack_s8x4(int a, int b, int c, int d) {
  return (uint32_t)(a & 0xFF) | ((uint32_t)(b & 0xFF) << 8) | ((uint32_t)(c & 0xFF) << 16) | ((uint32_t)d << 24);
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], uint32_t saddr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(saddr));
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// fp16x2 of (lo, hi) and the fp16x2 of their rounding remainders
__device__ __forceinline__ void split_half2(float lo, float hi, uint32_t& h, uint32_t& r) {
  const __half2 a = __floats2half2_rn(lo, hi);
  const float2 f = __half22float2(a);
  const __half2 b = __floats2half2_rn(lo - f.x, hi - f.y);
  h = *reinterpret_cast<const uint32_t*>(&a);
  r = *reinterpret_cast<const uint32_t*>(&b);
}

// 32-bit word at a 2-byte aligned shared address
__device__ __forceinline__ uint32_t lds_u32_a2(const uint8_t* b) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(b);
  const uint32_t* q = reinterpret_cast<const uint32_t*>(a & ~(uintptr_t)3);
  return __funnelshift_r(q[0], q[1], (a & 2) ? 16u : 0u);
}

// Four int8 codes -> two f16x2 holding them exactly (elements 0, 1 and 2, 3):
// byte b ^ 0x80 under the exponent bits 0x64 is 1024 + 128 + code.
__device__ __forceinline__ void codes_f16(uint32_t w, __half2& c01, __half2& c23) {
  const uint32_t x = w ^ 0x80808080u;
  const uint32_t lo = __byte_perm(x, 0x64646464u, 0x4140), hi = __byte_perm(x, 0x64646464u, 0x4342);
  const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));
  c01 = __hsub2(*reinterpret_cast<const __half2*>(&lo), bias);
  c23 = __hsub2(*reinterpret_cast<const __half2*>(&hi), bias);
}
__device__ __forceinline__ uint32_t h2u(__half2 x) { return *reinterpret_cast<const uint32_t*>(&x); }

__global__ void __launch_bounds__(32 * kWarps, 2)
    fa_batch_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                    BatchParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~(uintptr_t)127);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kOffBar);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int h = blockIdx.y;
  const int q0 = blockIdx.x * kQTile + warp * 16;  // this warp's first query
  const int ntiles = (p.S + kTTile - 1) / kTTile;
  const int xoff = (h & 1) * 8;                    // the head's first byte inside a raw row
  const int bx = 17 * h - (h & 1);                 // box start in 8-byte units (16-byte aligned)
  const uint32_t vh_s = smem_u32(smem + kOffVh), vl_s = smem_u32(smem + kOffVl);
  float* dks = reinterpret_cast<float*>(smem + kOffDk);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
  }
  __syncthreads();
  auto issue = [&](int i) {
    const int s = i % kStages;
    mbar_arrive_expect_tx(&full[s], 2 * kRawTile);
    tma_load_2d(smem + s * kRawTile, &kmap, bx, i * kTTile, &full[s]);
    tma_load_2d(smem + kOffRawV + s * kRawTile, &vmap, bx, i * kTTile, &full[s]);
  };
  if (threadIdx.x == 0)
    for (int i = 0; i < min(kStages, ntiles); ++i) issue(i);

  // ---- Q as two int8 levels (A operand of m16n8k32, rows g and g + 8): thread
  // (g, t) holds dims 32 b + 4 t .. + 3 and 32 b + 16 + 4 t .. + 3 of each row ----
  uint32_t qc[2][4][4];  // [level][block][A register]
  float s2a, s2b;        // level-2 scales of rows g and g + 8
  {
    float v[2][4][8];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int row = q0 + g + 8 * r;
      const float* pr = p.q + ((size_t)row * p.H + h) * 128;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        float4 x0 = make_float4(0.f, 0.f, 0.f, 0.f), x1 = x0;
        if (row < p.B) {
          x0 = *reinterpret_cast<const float4*>(pr + 32 * b + 4 * t);
          x1 = *reinterpret_cast<const float4*>(pr + 32 * b + 16 + 4 * t);
        }
        v[r][b][0] = x0.x * p.qscale; v[r][b][1] = x0.y * p.qscale; v[r][b][2] = x0.z * p.qscale;
        v[r][b][3] = x0.w * p.qscale; v[r][b][4] = x1.x * p.qscale; v[r][b][5] = x1.y * p.qscale;
        v[r][b][6] = x1.z * p.qscale; v[r][b][7] = x1.w * p.qscale;
      }
    }
    float s2[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      float a = 0.0f;
#pragma unroll
      for (int b = 0; b < 4; ++b)
#pragma unroll
        for (int e = 0; e < 8; ++e) a = fmaxf(a, fabsf(v[r][b][e]));
      a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 1));  // the row's 4 threads
      a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 2));
      const float s1 = a > 0.0f ? a / 127.0f : 1.0f;
      const float inv1 = a > 0.0f ? 127.0f / a : 0.0f;
      const float inv2 = 127.0f * inv1;
      s2[r] = s1 * (1.0f / 127.0f);
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        int c1[8], c2[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          c1[e] = max(-127, min(127, __float2int_rn(v[r][b][e] * inv1)));
          c2[e] = max(-127, min(127, __float2int_rn(fmaf(-s1, (float)c1[e], v[r][b][e]) * inv2)));
        }
        // A registers: 0 = (row g, k 4t..), 1 = (row g + 8, k 4t..), 2 = (row g, k 16 + 4t..), 3 = (row g + 8, ..)
        qc[0][b][r] = pack_s8x4(c1[0], c1[1], c1[2], c1[3]);
        qc[0][b][2 + r] = pack_s8x4(c1[4], c1[5], c1[6], c1[7]);
        qc[1][b][r] = pack_s8x4(c2[0], c2[1], c2[2], c2[3]);
        qc[1][b][2 + r] = pack_s8x4(c2[4], c2[5], c2[6], c2[7]);
      }
    }
    s2a = s2[0];
    s2b = s2[1];
  }

  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.0f, l_b = 0.0f;  // rows g and g + 8
  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
  bool dead = false;
  // ldmatrix row addresses: matrix mi = lane / 8, row r = lane % 8
  const int mi = lane >> 3, r8 = lane & 7;
  const uint32_t v_off = (uint32_t)(((mi & 1) * 8 + r8) * kHPitch + (mi >> 1) * 16);   // V: tokens x dims, .trans

  for (int i = 0; i < ntiles; ++i) {
    const int s = i % kStages;
    mbar_wait_or_poison(&full[s], (i / kStages) & 1, p.err, DEV_TIMEOUT_FULL, dead);
    // ---- dequantise: thread = (token, pair of 32-dim blocks) ----
    {
      const int tok = threadIdx.x >> 1, hb = threadIdx.x & 1;
      const uint8_t* rk = smem + s * kRawTile + tok * kRawRow + xoff;
      const uint8_t* rv = smem + kOffRawV + s * kRawTile + tok * kRawRow + xoff;
      uint8_t* dvh = smem + kOffVh + tok * kHPitch;
      uint8_t* dvl = smem + kOffVl + tok * kHPitch;
#pragma unroll
      for (int bi = 0; bi < 2; ++bi) {
        const int blk = 2 * hb + bi;
        // V: code * d rounded once to fp16 (mul.rn) and its remainder (fma.rn
        // of the exact product minus the high part): the bits of rounding the
        // exact fp32 product, in fp16 arithmetic; K: its block scales only
        dks[blk * kTTile + tok] = __half2float(*reinterpret_cast<const __half*>(rk + 34 * blk));
        const __half sdv = *reinterpret_cast<const __half*>(rv + 34 * blk);
        const __half2 dv2 = __halves2half2(sdv, sdv);
#pragma unroll
        for (int pr = 0; pr < 4; ++pr) {  // 8 codes
          const int co = 34 * blk + 2 + 8 * pr;
          const uint32_t v0 = lds_u32_a2(rv + co), v1 = lds_u32_a2(rv + co + 4);
          __half2 e[4];
          codes_f16(v0, e[0], e[1]);
          codes_f16(v1, e[2], e[3]);
          __half2 g2[4];
#pragma unroll
          for (int x = 0; x < 4; ++x) g2[x] = __hmul2(e[x], dv2);
          const uint4 vv = make_uint4(h2u(g2[0]), h2u(g2[1]), h2u(g2[2]), h2u(g2[3]));
          const uint4 vl = make_uint4(h2u(__hfma2(e[0], dv2, __hneg2(g2[0]))), h2u(__hfma2(e[1], dv2, __hneg2(g2[1]))),
                                      h2u(__hfma2(e[2], dv2, __hneg2(g2[2]))), h2u(__hfma2(e[3], dv2, __hneg2(g2[3]))));
          const int d = (32 * blk + 8 * pr) * 2;
          *reinterpret_cast<uint4*>(dvh + d) = vv;
          *reinterpret_cast<uint4*>(dvl + d) = vl;
        }
      }
    }
    __syncthreads();  // V tiles and K scales complete

    // ---- S: 16 queries x 64 tokens per warp; per 32-dim block two s8 MMAs
    // (query levels) on the raw K codes, then the block's K scale ----
    float sc[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.0f;
    {
      const uint8_t* kraw = smem + s * kRawTile + xoff + 2 + 4 * t;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint8_t* krow = kraw + (8 * j + g) * kRawRow;  // B column = token 8 j + g
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const uint32_t b0 = lds_u32_a2(krow + 34 * b), b1 = lds_u32_a2(krow + 34 * b + 16);
          int d1[4], d2[4];
          mma_s8(d1, qc[0][b], b0, b1);
          mma_s8(d2, qc[1][b], b0, b1);
          const float2 dk = *reinterpret_cast<const float2*>(dks + b * kTTile + 8 * j + 2 * t);
          sc[j][0] = fmaf((float)(127 * d1[0] + d2[0]), dk.x, sc[j][0]);
          sc[j][1] = fmaf((float)(127 * d1[1] + d2[1]), dk.y, sc[j][1]);
          sc[j][2] = fmaf((float)(127 * d1[2] + d2[2]), dk.x, sc[j][2]);
          sc[j][3] = fmaf((float)(127 * d1[3] + d2[3]), dk.y, sc[j][3]);
        }
        sc[j][0] *= s2a;
        sc[j][1] *= s2a;
        sc[j][2] *= s2b;
        sc[j][3] *= s2b;
      }
    }
    // the raw stage is no longer read: refill it once every warp is past QK
    fence_proxy_async_smem();
    __syncthreads();
    if (threadIdx.x == 0 && i + kStages < ntiles) issue(i + kStages);
    // tokens past the cache end (the last tile) weigh nothing
    const int tbase = i * kTTile + 2 * t;
    if (i * kTTile + kTTile > p.S) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (tbase + 8 * j >= p.S) sc[j][0] = sc[j][2] = -INFINITY;
        if (tbase + 8 * j + 1 >= p.S) sc[j][1] = sc[j][3] = -INFINITY;
      }
    }
    // ---- online softmax, rows g (a) and g + 8 (b) ----
    float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      mx_a = fmaxf(mx_a, fmaxf(sc[j][0], sc[j][1]));
      mx_b = fmaxf(mx_b, fmaxf(sc[j][2], sc[j][3]));
    }
    mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 1));
    mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 2));
    mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 1));
    mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 2));
    const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);
    const float ca = m_a == -INFINITY ? 0.0f : ex2(m_a - mn_a);
    const float cb = m_b == -INFINITY ? 0.0f : ex2(m_b - mn_b);
    m_a = mn_a;
    m_b = mn_b;
    float sa = 0.0f, sb = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      sc[j][0] = ex2(sc[j][0] - mn_a);
      sc[j][1] = ex2(sc[j][1] - mn_a);
      sc[j][2] = ex2(sc[j][2] - mn_b);
      sc[j][3] = ex2(sc[j][3] - mn_b);
      sa += sc[j][0] + sc[j][1];
      sb += sc[j][2] + sc[j][3];
    }
    l_a = fmaf(l_a, ca, sa);
    l_b = fmaf(l_b, cb, sb);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      o[j][0] *= ca;
      o[j][1] *= ca;
      o[j][2] *= cb;
      o[j][3] *= cb;
    }
    // ---- O += P_hi V_hi + P_lo V_hi + P_hi V_lo: k-steps of 16 tokens, P from the S accumulators ----
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t ph[4], pl[4];
      split_half2(sc[2 * kk][0], sc[2 * kk][1], ph[0], pl[0]);
      split_half2(sc[2 * kk][2], sc[2 * kk][3], ph[1], pl[1]);
      split_half2(sc[2 * kk + 1][0], sc[2 * kk + 1][1], ph[2], pl[2]);
      split_half2(sc[2 * kk + 1][2], sc[2 * kk + 1][3], ph[3], pl[3]);
#pragma unroll
      for (int np = 0; np < 8; ++np) {
        uint32_t vb[4], vr[4];
        const uint32_t off = v_off + (uint32_t)(16 * kk * kHPitch + 32 * np);
        ldsm_x4_trans(vb, vh_s + off);
        ldsm_x4_trans(vr, vl_s + off);
        mma_f16(o[2 * np], ph[0], ph[1], ph[2], ph[3], vb[0], vb[1]);
        mma_f16(o[2 * np + 1], ph[0], ph[1], ph[2], ph[3], vb[2], vb[3]);
        mma_f16(o[2 * np], pl[0], pl[1], pl[2], pl[3], vb[0], vb[1]);
        mma_f16(o[2 * np + 1], pl[0], pl[1], pl[2], pl[3], vb[2], vb[3]);
        mma_f16(o[2 * np], ph[0], ph[1], ph[2], ph[3], vr[0], vr[1]);
        mma_f16(o[2 * np + 1], ph[0], ph[1], ph[2], ph[3], vr[2], vr[3]);
      }
    }
    __syncthreads();  // the V tiles and K scales are rewritten by the next tile
  }

  // ---- out = O / l ----
  l_a += __shfl_xor_sync(0xffffffffu, l_a, 1);
  l_a += __shfl_xor_sync(0xffffffffu, l_a, 2);
  l_b += __shfl_xor_sync(0xffffffffu, l_b, 1);
  l_b += __shfl_xor_sync(0xffffffffu, l_b, 2);
  const float ia = l_a > 0.0f ? 1.0f / l_a : 0.0f, ib = l_b > 0.0f ? 1.0f / l_b : 0.0f;
  const int ra = q0 + g, rb = q0 + g + 8;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int c = 8 * j + 2 * t;
    if (ra < p.B)
      *reinterpret_cast<float2*>(p.out + ((size_t)ra * p.H + h) * 128 + c) = make_float2(o[j][0] * ia, o[j][1] * ia);
    if (rb < p.B)
      *reinterpret_cast<float2*>(p.out + ((size_t)rb * p.H + h) * 128 + c) = make_float2(o[j][2] * ib, o[j][3] * ib);
  }
}

bool encode_raw_map(CUtensorMap* map, const void* base, uint64_t rows, int heads) {
  // [rows][heads * 136 bytes] as 8-byte elements; boxes of 64 rows x 18
  // elements (one head's 136 bytes plus 8 before or after, so every box
  // starts on a 16-byte boundary; past the last row the fill is zero)
  auto fn = reinterpret_cast<EncodeTiledFn>(tensor_map_encoder());
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)heads * 17, rows};
  cuuint64_t strides[1] = {(cuuint64_t)heads * 136};
  cuuint32_t box[2] = {kRawRow / 8, kTTile};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

bool fa_batch_supported(const void* q, const void* k, const void* v, const void* out, int B, int S, int H, int D) {
  auto al = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; };
  // an even head count keeps every head's 16-byte aligned box inside the rows;
  // enough (query tile, head) CTAs to fill the GPU without splitting the cache
  return D == 128 && H >= 2 && H % 2 == 0 && S >= 1 && al(q) && al(k) && al(v) && al(out) &&
         (long long)((B + kQTile - 1) / kQTile) * H >= sm_count() && (B + kQTile - 1) / kQTile <= 65535 &&
         H <= 65535;
}

kq_status_t launch_fa_batch_mha(const float* q, const void* k, const void* v, float* out, int B, int S, int H,
                                cudaStream_t s) {
  CUtensorMap km, vm;
  if (!encode_raw_map(&km, k, (uint64_t)S, H) || !encode_raw_map(&vm, v, (uint64_t)S, H))
    return fail(KQ_ERR_CUDA, "fa_batch: KV tensor map rejected");
  kq_status_t st = ensure_dynamic_smem(reinterpret_cast<const void*>(fa_batch_kernel), kSmem,
                                       "fa_batch smem attribute");
  if (st) return st;
  BatchParams p;
  p.q = q;
  p.out = out;
  p.err = device_error_word();
  p.B = B;
  p.H = H;
  p.S = S;
  p.qscale = (float)(1.0 / std::sqrt(128.0) * 1.4426950408889634);
  dim3 grid((unsigned)((B + kQTile - 1) / kQTile), (unsigned)H);
  fa_batch_kernel<<<grid, 32 * kWarps, kSmem, s>>>(km, vm, p);
  return check_launch("fa_batch");
}

}  // namespace kq
