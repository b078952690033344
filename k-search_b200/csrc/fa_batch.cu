// Flash attention for the harness form with many queries per head (D = 128)
// over a q8_0, q4_0 or fp16 KV cache: the harness flash_attention operator
// (kernelevalplus-main/llm_kernel_test/op_test_handler.py:543-563, cache
// built at :489-534) shares one [S, H, D] cache across all B queries of a
// head, so at B = 512 a head is a GEMM pair (S = Q K^T, O = softmax(S) V)
// rather than a stream of the cache.
//
// CTA = 4 warps over 64 queries of one head (16 per warp); it walks the
// cache (or one token chunk of it) in 64-token tiles brought by a two-stage
// TMA ring. When (query tile, head) CTAs alone would leave the last wave
// short, each is split into token chunks that write their partial softmax
// state (m, l, O), and fa_batch_combine_kernel merges them per row.
//
// Block-quantised caches (fa_batch_kernel<KVF>, q8_0 and q4_0):
//  * the boxes hold the raw rows of the head (64 rows x 144 bytes for q8_0,
//    x 80 for q4_0: the head's 136- or 72-byte row sits 0 or 8 bytes in, so
//    every box starts on a 16-byte boundary);
//  * QK is exact on the raw K codes (mma.m16n8k32 s8, one MMA per 32-dim
//    block and query level; q4_0 nibbles become the int8 codes q - 8): the
//    query q * scale * log2(e) is held as two int8 levels (q ~ s1 c1 + s2 c2,
//    s2 = s1 / 127, so 127 dot1 + dot2 is the exact block dot at scale s2),
//    and the fp32 epilogue applies each (token, block) K scale, as the decode
//    kernels do;
//  * the CTA turns each V tile's codes into fp16 once (exact: |code| <= 127)
//    and keeps the V block scales apart; per 32-dim block b,
//    PV_b = P'_hi C + P'_lo C (mma.m16n8k16 f16) with P' = p * d_v(token, b)
//    split into an fp16 high part and remainder.
// fp16 caches (fa_batch_f16_kernel): K and V are exact in fp16, so the TMA
// boxes (two 64-dim halves, 128-byte swizzled) are read by ldmatrix in place;
// the query is an fp16 high part plus its remainder in shared memory, and
// QK = Q_hi K + Q_lo K, PV = P_hi V + P_lo V.
// Both: online softmax per query row in registers (exp2); P (or P') as fp16
// plus its fp16 remainder, taken straight from the S accumulators as the A
// operand of the PV products.
// Precision, from an fp64 emulation of each arithmetic against the oracle
// (worst |error| / per-element bar): fp16 Q, K, P and V each rounded once
// misses the bar on a few elements; with fp16 remainders on three of the four
// operands 0.71-0.78 (still 1 miss in 2.1 M elements on the GPU), on all four
// 0.003 (three f16 products per GEMM); the int8 QK with P and V split
// 0.15-0.20. Both forms here have every operand exact or split.
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
constexpr int kHPitch = 272;             // fp16 tile row: 256 bytes + 16 (ldmatrix rows in distinct banks)
constexpr int kHTile = kTTile * kHPitch;            // 17408 bytes

// Shared-memory plan of the block-quantised kernels: the raw K and V rings,
// the V codes of the current tile as fp16 and the K and V block scales.
template <int KVF>
struct RawFmt {
  static constexpr int kBlk = KVF == KQ_KV_Q8_0 ? 34 : 18;  // bytes per 32-dim block
  static constexpr int kUnits = 4 * kBlk / 8;                // the head's row in 8-byte units (17, 9)
  static constexpr int kRawRow = 8 * (kUnits + 1);           // box row: 144, 80 bytes
  static constexpr int kRawTile = kTTile * kRawRow;
  static constexpr int kOffRawV = kStages * kRawTile;
  static constexpr int kOffVc = 2 * kStages * kRawTile;      // V codes as fp16 (exact) [64 tokens][kHPitch]
  static constexpr int kOffDk = kOffVc + kHTile;             // K block scales, fp32 [4 blocks][64 tokens]
  static constexpr int kOffDv = kOffDk + 4 * kTTile * 4;     // V block scales, fp32 [4 blocks][64 tokens]
  static constexpr int kOffBar = kOffDv + 4 * kTTile * 4;
  static constexpr int kSmem = kOffBar + kStages * 8 + 128;  // + base alignment slack
  static_assert(kRawTile % 128 == 0 && kOffVc % 128 == 0 && kHTile % 128 == 0, "aligned tiles");
};

// Shared-memory plan of the fp16-cache kernel: per stage K then V, each two
// 64-token x 128-byte swizzled halves (dims 0-63, 64-127; 1024-byte aligned
// for the 128-byte swizzle), then per warp the query's high parts and
// remainders [2][16 rows][kHPitch].
constexpr int kF16Half = kTTile * 128;               // 8192 bytes
constexpr int kF16Tile = 2 * kF16Half;               // one operand tile
constexpr int kF16Stage = 2 * kF16Tile;              // K and V
constexpr int kF16OffQ = kStages * kF16Stage;
constexpr int kF16QWarp = 2 * 16 * kHPitch;
constexpr int kF16OffBar = kF16OffQ + kWarps * kF16QWarp;
constexpr int kF16Smem = kF16OffBar + kStages * 8 + 1024;  // + base alignment slack

struct BatchParams {
  const float* q;   // [B, H, 128]
  float* out;       // [B, H, 128]
  int* err;
  int B, H, S;
  float qscale;     // softmax scale * log2(e)
  // token chunks (grid z): chunk c takes tiles [c ct, (c + 1) ct); with
  // nc > 1 each writes its unnormalised partial state, [B * H][nc] maxima and
  // sums and [B * H][nc][128] accumulators, and a combine kernel merges them
  int nc, ct;
  float* pm;
  float* pl;
  float* pacc;
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

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t saddr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(saddr));
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
// Four nibbles (one per byte, 0-15) -> two f16x2 of q - 8, exactly: 1024 + q
// under the exponent bits 0x64, minus 1032.
__device__ __forceinline__ void nibbles_f16(uint32_t x, __half2& c01, __half2& c23) {
  const uint32_t lo = __byte_perm(x, 0x64646464u, 0x4140), hi = __byte_perm(x, 0x64646464u, 0x4342);
  const __half2 bias = __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408));
  c01 = __hsub2(*reinterpret_cast<const __half2*>(&lo), bias);
  c23 = __hsub2(*reinterpret_cast<const __half2*>(&hi), bias);
}
// Four nibbles (one per byte) -> four int8 codes q - 8 (no borrow between
// bytes: every byte is at least 0x80 before the subtraction)
__device__ __forceinline__ uint32_t nibbles_s8(uint32_t x) {
  return ((x | 0x80808080u) - 0x08080808u) ^ 0x80808080u;
}
__device__ __forceinline__ uint32_t h2u(__half2 x) { return *reinterpret_cast<const uint32_t*>(&x); }

// Online softmax over one 64-token tile for rows g (a) and g + 8 (b) of the
// warp's 16 queries: masks tokens at or past S (tile starting at token tok0),
// turns the scores into p = exp2(s - m), updates the running maxima and sums
// and rescales the O accumulators.
__device__ __forceinline__ void softmax_tile(float (&sc)[8][4], int tok0, int S, int t, float& m_a, float& m_b,
                                             float& l_a, float& l_b, float (&o)[16][4]) {
  if (tok0 + kTTile > S) {
    const int tbase = tok0 + 2 * t;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (tbase + 8 * j >= S) sc[j][0] = sc[j][2] = -INFINITY;
      if (tbase + 8 * j + 1 >= S) sc[j][1] = sc[j][3] = -INFINITY;
    }
  }
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
}

// P of k-step kk (16 tokens) as the A operand of m16n8k16: high parts and
// remainders, straight from the S accumulators
__device__ __forceinline__ void p_operand(const float (&sc)[8][4], int kk, uint32_t (&ph)[4], uint32_t (&pl)[4]) {
  split_half2(sc[2 * kk][0], sc[2 * kk][1], ph[0], pl[0]);
  split_half2(sc[2 * kk][2], sc[2 * kk][3], ph[1], pl[1]);
  split_half2(sc[2 * kk + 1][0], sc[2 * kk + 1][1], ph[2], pl[2]);
  split_half2(sc[2 * kk + 1][2], sc[2 * kk + 1][3], ph[3], pl[3]);
}

// The warp's rows g and g + 8 (queries past B are not written): out = O / l
// with one token chunk, else chunk c's partial state (m, l, O).
__device__ __forceinline__ void store_rows(const float (&o)[16][4], float m_a, float m_b, float l_a, float l_b,
                                           const BatchParams& p, int q0, int g, int t, int h, int c) {
  l_a += __shfl_xor_sync(0xffffffffu, l_a, 1);
  l_a += __shfl_xor_sync(0xffffffffu, l_a, 2);
  l_b += __shfl_xor_sync(0xffffffffu, l_b, 1);
  l_b += __shfl_xor_sync(0xffffffffu, l_b, 2);
  const int ra = q0 + g, rb = q0 + g + 8;
  if (p.nc > 1) {
    const size_t pa = ((size_t)ra * p.H + h) * p.nc + c, pb = ((size_t)rb * p.H + h) * p.nc + c;
    if (t == 0 && ra < p.B) {
      p.pm[pa] = m_a;
      p.pl[pa] = l_a;
    }
    if (t == 0 && rb < p.B) {
      p.pm[pb] = m_b;
      p.pl[pb] = l_b;
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int d = 8 * j + 2 * t;
      if (ra < p.B) *reinterpret_cast<float2*>(p.pacc + pa * 128 + d) = make_float2(o[j][0], o[j][1]);
      if (rb < p.B) *reinterpret_cast<float2*>(p.pacc + pb * 128 + d) = make_float2(o[j][2], o[j][3]);
    }
    return;
  }
  const float ia = l_a > 0.0f ? 1.0f / l_a : 0.0f, ib = l_b > 0.0f ? 1.0f / l_b : 0.0f;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int d = 8 * j + 2 * t;
    if (ra < p.B)
      *reinterpret_cast<float2*>(p.out + ((size_t)ra * p.H + h) * 128 + d) = make_float2(o[j][0] * ia, o[j][1] * ia);
    if (rb < p.B)
      *reinterpret_cast<float2*>(p.out + ((size_t)rb * p.H + h) * 128 + d) = make_float2(o[j][2] * ib, o[j][3] * ib);
  }
}

// One warp per (query, head) row: out = sum_c 2^(m_c - M) O_c / sum_c 2^(m_c - M) l_c
// over the row's token chunks. Lane = 4 dims.
__global__ void __launch_bounds__(128) fa_batch_combine_kernel(BatchParams p, int rows) {
  const int r = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (r >= rows) return;
  const size_t base = (size_t)r * p.nc;
  float M = -INFINITY;
  for (int c = 0; c < p.nc; ++c) M = fmaxf(M, p.pm[base + c]);
  float L = 0.0f;
  float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
  if (M != -INFINITY) {
    for (int c = 0; c < p.nc; ++c) {
      const float mc = p.pm[base + c];
      const float w = mc == -INFINITY ? 0.0f : ex2(mc - M);
      L = fmaf(p.pl[base + c], w, L);
      const float4 x = reinterpret_cast<const float4*>(p.pacc + (base + c) * 128)[lane];
      a.x = fmaf(x.x, w, a.x);
      a.y = fmaf(x.y, w, a.y);
      a.z = fmaf(x.z, w, a.z);
      a.w = fmaf(x.w, w, a.w);
    }
  }
  const float inv = L > 0.0f ? 1.0f / L : 0.0f;
  reinterpret_cast<float4*>(p.out + (size_t)r * 128)[lane] = make_float4(a.x * inv, a.y * inv, a.z * inv, a.w * inv);
}

template <int KVF>
__global__ void __launch_bounds__(32 * kWarps, 2)
    fa_batch_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                    BatchParams p) {
  using F = RawFmt<KVF>;
  constexpr int kBlk = F::kBlk, kRawRow = F::kRawRow, kRawTile = F::kRawTile;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~(uintptr_t)127);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + F::kOffBar);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int h = blockIdx.y;
  const int q0 = blockIdx.x * kQTile + warp * 16;  // this warp's first query
  const int c = blockIdx.z;  // token chunk
  const int tile0 = c * p.ct;
  const int ntiles = max(0, min((p.S + kTTile - 1) / kTTile, tile0 + p.ct) - tile0);
  const int xoff = (h & 1) * 8;                    // the head's first byte inside a raw row
  const int bx = F::kUnits * h - (h & 1);          // box start in 8-byte units (16-byte aligned)
  const uint32_t vc_s = smem_u32(smem + F::kOffVc);
  float* dks = reinterpret_cast<float*>(smem + F::kOffDk);
  float* dvs = reinterpret_cast<float*>(smem + F::kOffDv);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
  }
  __syncthreads();

  auto issue = [&](int i) {
    const int s = i % kStages;
    mbar_arrive_expect_tx(&full[s], 2 * kRawTile);
    tma_load_2d(smem + s * kRawTile, &kmap, bx, (tile0 + i) * kTTile, &full[s]);
    tma_load_2d(smem + F::kOffRawV + s * kRawTile, &vmap, bx, (tile0 + i) * kTTile, &full[s]);
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
    // ---- V codes to fp16 (exact) and the K and V block scales: two (token,
    // block) items per thread; a quarter-warp holds 8 consecutive tokens of
    // one block, so its 16-byte stores fall in distinct banks ----
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int item = threadIdx.x + 128 * r;
      const int tok = (item & 7) + 8 * (item >> 5), blk = (item >> 3) & 3;
      const uint8_t* rk = smem + s * kRawTile + tok * kRawRow + xoff + kBlk * blk;
      const uint8_t* rv = smem + F::kOffRawV + s * kRawTile + tok * kRawRow + xoff + kBlk * blk;
      uint8_t* dvc = smem + F::kOffVc + tok * kHPitch + 64 * blk;
      dks[blk * kTTile + tok] = __half2float(*reinterpret_cast<const __half*>(rk));
      dvs[blk * kTTile + tok] = __half2float(*reinterpret_cast<const __half*>(rv));
      if constexpr (KVF == KQ_KV_Q8_0) {
#pragma unroll
        for (int pr = 0; pr < 4; ++pr) {  // codes 8 pr .. 8 pr + 7
          __half2 e[4];
          codes_f16(lds_u32_a2(rv + 2 + 8 * pr), e[0], e[1]);
          codes_f16(lds_u32_a2(rv + 6 + 8 * pr), e[2], e[3]);
          *reinterpret_cast<uint4*>(dvc + 16 * pr) = make_uint4(h2u(e[0]), h2u(e[1]), h2u(e[2]), h2u(e[3]));
        }
      } else {
        // q4_0: byte e of the 16 holds element e (low nibble) and e + 16
#pragma unroll
        for (int wp = 0; wp < 2; ++wp) {  // bytes 8 wp .. 8 wp + 7
          const uint32_t x0 = lds_u32_a2(rv + 2 + 8 * wp), x1 = lds_u32_a2(rv + 6 + 8 * wp);
          __half2 lo[4], hi[4];
          nibbles_f16(x0 & 0x0F0F0F0Fu, lo[0], lo[1]);
          nibbles_f16(x1 & 0x0F0F0F0Fu, lo[2], lo[3]);
          nibbles_f16((x0 >> 4) & 0x0F0F0F0Fu, hi[0], hi[1]);
          nibbles_f16((x1 >> 4) & 0x0F0F0F0Fu, hi[2], hi[3]);
          *reinterpret_cast<uint4*>(dvc + 16 * wp) = make_uint4(h2u(lo[0]), h2u(lo[1]), h2u(lo[2]), h2u(lo[3]));
          *reinterpret_cast<uint4*>(dvc + 32 + 16 * wp) =
              make_uint4(h2u(hi[0]), h2u(hi[1]), h2u(hi[2]), h2u(hi[3]));
        }
      }
    }
    __syncthreads();  // V codes and block scales complete

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
          uint32_t b0, b1;
          if constexpr (KVF == KQ_KV_Q8_0) {
            b0 = lds_u32_a2(krow + kBlk * b);
            b1 = lds_u32_a2(krow + kBlk * b + 16);
          } else {  // dims 4t .. 4t + 3 are the low nibbles of bytes 4t .., dims 16 + 4t .. their high ones
            const uint32_t x = lds_u32_a2(krow + kBlk * b);
            b0 = nibbles_s8(x & 0x0F0F0F0Fu);
            b1 = nibbles_s8((x >> 4) & 0x0F0F0F0Fu);
          }
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
    softmax_tile(sc, (tile0 + i) * kTTile, p.S, t, m_a, m_b, l_a, l_b, o);
    // ---- O += P'_hi C + P'_lo C per 32-dim block b: C = the exact V codes,
    // P' = p * d_v(token, b) split into fp16 high part and remainder; k-steps
    // of 16 tokens (this thread's A columns: tokens 16 kk + 2 t, + 1, + 8, + 9) ----
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const int t0 = 16 * kk + 2 * t;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const float2 d01 = *reinterpret_cast<const float2*>(dvs + b * kTTile + t0);
        const float2 d89 = *reinterpret_cast<const float2*>(dvs + b * kTTile + t0 + 8);
        uint32_t ph[4], pl[4];
        split_half2(sc[2 * kk][0] * d01.x, sc[2 * kk][1] * d01.y, ph[0], pl[0]);
        split_half2(sc[2 * kk][2] * d01.x, sc[2 * kk][3] * d01.y, ph[1], pl[1]);
        split_half2(sc[2 * kk + 1][0] * d89.x, sc[2 * kk + 1][1] * d89.y, ph[2], pl[2]);
        split_half2(sc[2 * kk + 1][2] * d89.x, sc[2 * kk + 1][3] * d89.y, ph[3], pl[3]);
#pragma unroll
        for (int np = 2 * b; np < 2 * b + 2; ++np) {  // dims 16 np .. + 15
          uint32_t vb[4];
          ldsm_x4_trans(vb, vc_s + v_off + (uint32_t)(16 * kk * kHPitch + 32 * np));
          mma_f16(o[2 * np], ph[0], ph[1], ph[2], ph[3], vb[0], vb[1]);
          mma_f16(o[2 * np + 1], ph[0], ph[1], ph[2], ph[3], vb[2], vb[3]);
          mma_f16(o[2 * np], pl[0], pl[1], pl[2], pl[3], vb[0], vb[1]);
          mma_f16(o[2 * np + 1], pl[0], pl[1], pl[2], pl[3], vb[2], vb[3]);
        }
      }
    }
    __syncthreads();  // the V codes and block scales are rewritten by the next tile
  }
  store_rows(o, m_a, m_b, l_a, l_b, p, q0, g, t, h, c);
}

__global__ void __launch_bounds__(32 * kWarps, 2)
    fa_batch_f16_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                        BatchParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kF16OffBar);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int h = blockIdx.y;
  const int q0 = blockIdx.x * kQTile + warp * 16;  // this warp's first query
  const int c = blockIdx.z;  // token chunk
  const int tile0 = c * p.ct;
  const int ntiles = max(0, min((p.S + kTTile - 1) / kTTile, tile0 + p.ct) - tile0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
  }
  __syncthreads();

  auto issue = [&](int i) {
    const int s = i % kStages;
    uint8_t* st = smem + s * kF16Stage;
    mbar_arrive_expect_tx(&full[s], kF16Stage);
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      tma_load_2d(st + hf * kF16Half, &kmap, 128 * h + 64 * hf, (tile0 + i) * kTTile, &full[s]);
      tma_load_2d(st + kF16Tile + hf * kF16Half, &vmap, 128 * h + 64 * hf, (tile0 + i) * kTTile, &full[s]);
    }
  };
  if (threadIdx.x == 0)
    for (int i = 0; i < min(kStages, ntiles); ++i) issue(i);

  // ---- the warp's 16 queries * scale * log2(e): fp16 high parts (rows 0-15)
  // and remainders (rows 16-31); lane = 4 dims of each row ----
  uint8_t* qsm = smem + kF16OffQ + warp * kF16QWarp;
#pragma unroll 4
  for (int r = 0; r < 16; ++r) {
    const int row = q0 + r;
    float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
    if (row < p.B) x = *reinterpret_cast<const float4*>(p.q + ((size_t)row * p.H + h) * 128 + 4 * lane);
    uint32_t h0, l0, h1, l1;
    split_half2(x.x * p.qscale, x.y * p.qscale, h0, l0);
    split_half2(x.z * p.qscale, x.w * p.qscale, h1, l1);
    *reinterpret_cast<uint2*>(qsm + r * kHPitch + 8 * lane) = make_uint2(h0, h1);
    *reinterpret_cast<uint2*>(qsm + (16 + r) * kHPitch + 8 * lane) = make_uint2(l0, l1);
  }
  __syncwarp();

  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.0f, l_b = 0.0f;  // rows g and g + 8
  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
  bool dead = false;
  // ldmatrix row addresses: matrix mi = lane / 8, row r8 = lane % 8. In the
  // swizzled K / V halves, 16-byte chunk c of token row r sits at chunk
  // c ^ (r % 8), and r % 8 = r8 for every row a lane addresses.
  const int mi = lane >> 3, r8 = lane & 7;
  const uint32_t q_s = smem_u32(qsm) + (uint32_t)(((mi & 1) * 8 + r8) * kHPitch + (mi >> 1) * 16);

  for (int i = 0; i < ntiles; ++i) {
    const int s = i % kStages;
    mbar_wait_or_poison(&full[s], (i / kStages) & 1, p.err, DEV_TIMEOUT_FULL, dead);
    const uint32_t k_s = smem_u32(smem + s * kF16Stage), v_s = k_s + kF16Tile;

    // ---- S = Q_hi K + Q_lo K: k-steps of 16 dims; B = K rows (tokens) ----
    float sc[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.0f;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      uint32_t qh[4], ql[4];
      ldsm_x4(qh, q_s + 32 * ks);
      ldsm_x4(ql, q_s + 16 * kHPitch + 32 * ks);
      const uint32_t kc = (uint32_t)(((((2 * ks) & 7) + (mi & 1)) ^ r8) << 4);
      const uint32_t kbase = k_s + (uint32_t)((ks >> 2) * kF16Half) + kc;
#pragma unroll
      for (int jp = 0; jp < 4; ++jp) {  // tokens 16 jp .. + 15
        uint32_t kb[4];
        ldsm_x4(kb, kbase + (uint32_t)((16 * jp + (mi >> 1) * 8 + r8) * 128));
        mma_f16(sc[2 * jp], qh[0], qh[1], qh[2], qh[3], kb[0], kb[1]);
        mma_f16(sc[2 * jp], ql[0], ql[1], ql[2], ql[3], kb[0], kb[1]);
        mma_f16(sc[2 * jp + 1], qh[0], qh[1], qh[2], qh[3], kb[2], kb[3]);
        mma_f16(sc[2 * jp + 1], ql[0], ql[1], ql[2], ql[3], kb[2], kb[3]);
      }
    }
    softmax_tile(sc, (tile0 + i) * kTTile, p.S, t, m_a, m_b, l_a, l_b, o);
    // ---- O += P_hi V + P_lo V: k-steps of 16 tokens, V by ldmatrix.trans ----
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t ph[4], pl[4];
      p_operand(sc, kk, ph, pl);
      const uint32_t vrow = v_s + (uint32_t)((16 * kk + (mi & 1) * 8 + r8) * 128);
#pragma unroll
      for (int np = 0; np < 8; ++np) {  // dims 16 np .. + 15
        const uint32_t vc = (uint32_t)(((((2 * np) & 7) + (mi >> 1)) ^ r8) << 4);
        uint32_t vb[4];
        ldsm_x4_trans(vb, vrow + (uint32_t)((np >> 2) * kF16Half) + vc);
        mma_f16(o[2 * np], ph[0], ph[1], ph[2], ph[3], vb[0], vb[1]);
        mma_f16(o[2 * np + 1], ph[0], ph[1], ph[2], ph[3], vb[2], vb[3]);
        mma_f16(o[2 * np], pl[0], pl[1], pl[2], pl[3], vb[0], vb[1]);
        mma_f16(o[2 * np + 1], pl[0], pl[1], pl[2], pl[3], vb[2], vb[3]);
      }
    }
    // the stage is no longer read: refill it once every warp is past PV
    fence_proxy_async_smem();
    __syncthreads();
    if (threadIdx.x == 0 && i + kStages < ntiles) issue(i + kStages);
  }
  store_rows(o, m_a, m_b, l_a, l_b, p, q0, g, t, h, c);
}

bool encode_raw_map(CUtensorMap* map, const void* base, uint64_t rows, int heads, int units) {
  // [rows][heads * units 8-byte elements]; boxes of 64 rows x (units + 1)
  // elements (one head's row plus 8 bytes before or after, so every box
  // starts on a 16-byte boundary; past the last row the fill is zero)
  auto fn = reinterpret_cast<EncodeTiledFn>(tensor_map_encoder());
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)heads * units, rows};
  cuuint64_t strides[1] = {(cuuint64_t)heads * units * 8};
  cuuint32_t box[2] = {(cuuint32_t)units + 1, kTTile};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool encode_f16_map(CUtensorMap* map, const void* base, uint64_t rows, int heads) {
  // [rows][heads * 128] fp16; boxes of 64 rows x 64 elements (128 bytes)
  // with the 128-byte swizzle (past the last row the fill is zero)
  auto fn = reinterpret_cast<EncodeTiledFn>(tensor_map_encoder());
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)heads * 128, rows};
  cuuint64_t strides[1] = {(cuuint64_t)heads * 256};
  cuuint32_t box[2] = {64, kTTile};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int KVF>
kq_status_t launch_raw(const CUtensorMap& km, const CUtensorMap& vm, const BatchParams& p, dim3 grid, cudaStream_t s) {
  kq_status_t st = ensure_dynamic_smem(reinterpret_cast<const void*>(fa_batch_kernel<KVF>), RawFmt<KVF>::kSmem,
                                       "fa_batch smem attribute");
  if (st) return st;
  fa_batch_kernel<KVF><<<grid, 32 * kWarps, RawFmt<KVF>::kSmem, s>>>(km, vm, p);
  return check_launch("fa_batch");
}

// Token chunks per (query tile, head): the block scheduler fills the GPU's
// 2 CTAs per SM from a grid of ctas * nc CTAs. Modelled time: waves x (tiles
// per chunk + 2), the 2 being a CTA's set-up, pipeline fill and partial
// write in tile times (fitted to CUDA-event timings at B = 512, H = 32,
// S = 4096 and 8192 with 1 and 8 chunks: 1.4-2.4 across the three cache
// formats). The cheapest count of at most 16, with chunks of at least 4
// tiles; one chunk unless a split is cheaper. B = 512: H = 32, S = 8192
// takes 8 chunks (365 -> 356 us fp16, 603 -> 589 q8_0, 560 -> 527 q4_0);
// S = 4096 stays whole (8 chunks were 4-10% slower); H = 28, whose 224
// CTAs leave a quarter of the slots idle, splits (S = 8192 with 9 chunks:
// fp16 366 -> 325 us, q4_0 569 -> 467).
int choose_token_chunks(long long ctas, int ntiles) {
  const long long slots = 2LL * sm_count();
  auto cost = [&](int nc) {
    const int ct = (ntiles + nc - 1) / nc;
    const long long u = ctas * ((ntiles + ct - 1) / ct), waves = (u + slots - 1) / slots;
    return (double)waves * (ct + 2.0);
  };
  int best = 1;
  double bc = cost(1);
  for (int nc = 2; nc <= 16 && ntiles / nc >= 4; ++nc) {
    const double c = cost(nc);
    if (c < bc) {
      best = nc;
      bc = c;
    }
  }
  return best;
}

}  // namespace

bool fa_batch_supported(int kv_format, const void* q, const void* k, const void* v, const void* out, int B, int S,
                        int H, int D) {
  auto al = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; };
  // block-quantised caches: an even head count keeps every head's 16-byte
  // aligned box inside the rows; enough (query tile, head) CTAs to fill the
  // GPU without splitting the cache
  const bool heads = kv_format == KQ_KV_F16 ? H >= 1
                                            : (kv_format == KQ_KV_Q8_0 || kv_format == KQ_KV_Q4_0) && H >= 2 &&
                                                  H % 2 == 0;
  return heads && D == 128 && S >= 1 && al(q) && al(k) && al(v) && al(out) &&
         (long long)((B + kQTile - 1) / kQTile) * H >= sm_count() && (B + kQTile - 1) / kQTile <= 65535 &&
         H <= 65535;
}

kq_status_t launch_fa_batch_mha(int kv_format, const float* q, const void* k, const void* v, float* out, int B,
                                int S, int H, cudaStream_t s) {
  CUtensorMap km, vm;
  const bool ok = kv_format == KQ_KV_F16
                      ? encode_f16_map(&km, k, (uint64_t)S, H) && encode_f16_map(&vm, v, (uint64_t)S, H)
                      : encode_raw_map(&km, k, (uint64_t)S, H, kv_format == KQ_KV_Q8_0 ? 17 : 9) &&
                            encode_raw_map(&vm, v, (uint64_t)S, H, kv_format == KQ_KV_Q8_0 ? 17 : 9);
  if (!ok) return fail(KQ_ERR_CUDA, "fa_batch: KV tensor map rejected");
  BatchParams p;
  p.q = q;
  p.out = out;
  p.err = device_error_word();
  p.B = B;
  p.H = H;
  p.S = S;
  p.qscale = (float)(1.0 / std::sqrt(128.0) * 1.4426950408889634);
  const int qtiles = (B + kQTile - 1) / kQTile;
  const int ntiles = (S + kTTile - 1) / kTTile;
  const int nc0 = choose_token_chunks((long long)qtiles * H, ntiles);
  p.ct = (ntiles + nc0 - 1) / nc0;
  p.nc = (ntiles + p.ct - 1) / p.ct;  // no empty chunk
  p.pm = p.pl = p.pacc = nullptr;
  const long long rows = (long long)B * H;
  if (p.nc > 1) {
    float* ws = static_cast<float*>(workspace(WS_FA, (size_t)rows * p.nc * (2 + 128) * sizeof(float)));
    if (!ws) return KQ_ERR_NOMEM;
    p.pm = ws;
    p.pl = ws + rows * p.nc;
    p.pacc = ws + 2 * rows * p.nc;
  }
  dim3 grid((unsigned)qtiles, (unsigned)H, (unsigned)p.nc);
  kq_status_t st = KQ_OK;
  switch (kv_format) {
    case KQ_KV_Q8_0: st = launch_raw<KQ_KV_Q8_0>(km, vm, p, grid, s); break;
    case KQ_KV_Q4_0: st = launch_raw<KQ_KV_Q4_0>(km, vm, p, grid, s); break;
    case KQ_KV_F16: {
      st = ensure_dynamic_smem(reinterpret_cast<const void*>(fa_batch_f16_kernel), kF16Smem,
                               "fa_batch smem attribute");
      if (st) return st;
      fa_batch_f16_kernel<<<grid, 32 * kWarps, kF16Smem, s>>>(km, vm, p);
      st = check_launch("fa_batch(f16)");
      break;
    }
    default: return fail(KQ_ERR_INVALID, "fa_batch: unknown KV format %d", kv_format);
  }
  if (st || p.nc == 1) return st;
  fa_batch_combine_kernel<<<(unsigned)((rows + 3) / 4), 128, 0, s>>>(p, (int)rows);
  return check_launch("fa_batch_combine");
}

}  // namespace kq
