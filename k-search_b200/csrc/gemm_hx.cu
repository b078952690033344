// Tensor-core quantised GEMM for M > 8 activation rows, dequantise-and-matmul
// form (the reference's own gemm_ref.py:100-153 / :274-331 path): both
// operands are dequantised to fp16 and one tcgen05.mma.kind::f16 chain
// accumulates the whole K range in an fp32 TMEM accumulator.
//
//   A'[m, k] = fp16(q_a[m, k] * d_a[m, k/32])            (activations, prep kernel)
//   W'[n, k] = fp16((q_w[n, k] - 8) * d_w[n, k/32])      q4_0
//            = fp16(q_w[n, k] * d_w[n, k/32] + m_w)      q4_1
//            = fp16(q_w[n, k] * d_w[n, k/32])            q8_0
//   out[m, n] = sum_k A'[m, k] W'[n, k] + sum_b X_a[m, b] X_w[n, b]
//
// W' is the dequantised weight (zero-centred, so the sum has no cancellation).
// The second sum carries what separates the reference's per-block formulas
// from the plain product, the residual X_a = s_a - d_a * sum_i q_a (s as the
// activation block stores it), as extra K columns:
//   q4_0: X_w = -8 d_w -> d_w (d_a sumi - 8 s_a)          (gemm_ref.py:100-153)
//   q4_1: X_w = m_w    -> d_w d_a sumi + m_w s_a          (gemm_ref.py:274-331)
//   q8_0: no extra columns -> d_w d_a sumi                (gemm_reference.h:311-336)
// The only departures from exact per-block arithmetic are the fp16 roundings
// of A' and W' (relative 2^-11 per element, unbiased) and the fp32
// accumulation order; the int32 block sums themselves are served by
// kq_block_sums_i32.
//
// Why not int8 MMA per block: every 32-wide K block has its own scales, so an
// int8 kind::i8 pipeline must rescale a fresh 128x128 int32 tile per block on
// the FP32 pipe (at least 2 FMAs per element and block), which caps it near
// 35% of the int8 tensor rate; the dequantised form keeps the tensor pipe
// busy instead (kind::f16 runs at half the int8 rate, with no per-block
// epilogue).
//
// CTA: 128 x 128 output tile (tokens x weight rows), persistent over tiles,
// tokens fastest so co-running CTAs share weight tiles in L2. 14 warps:
//   warp 0      TMA producer: A' chunks (fp16, 128B-swizzled boxes of 128 rows
//               x 64 K) and raw weight rows (unchanged AoS q-blocks, 128 rows x
//               8 blocks per box)
//   warp 1      MMA issuer (one thread), owns the TMEM allocation
//   warps 2-9   converters: two threads per weight row, each turns 4 raw blocks
//               into two 128B-swizzled fp16 K-chunks (and the X_w column)
//   warps 10-13 epilogue: TMEM -> registers -> global fp32, double-buffered
//               accumulators so the next tile's MMAs overlap the stores
#include <cuda_fp16.h>

#include <algorithm>
#include <type_traits>

#include "kq_internal.h"
#include "kq_device.cuh"
#include "kq_tc.cuh"

namespace kq {
namespace {

using namespace tc;

constexpr int HM = 128;          // tokens per tile (TMEM lanes)
constexpr int HN = 128;          // weight rows per tile (TMEM columns per accumulator)
constexpr int CK = 64;           // K elements per chunk: one 128-byte swizzle atom of fp16
constexpr int RB = 8;            // blocks per raw weight stage (= 4 chunks)
constexpr int GRP = 32;          // main chunks per extra chunk (64 blocks)
constexpr int SA = 4;            // A' chunk stages
constexpr int SW = 4;            // converted weight chunk stages
constexpr int SR = 2;            // raw weight stages
constexpr int NACC = 2;          // TMEM accumulators
constexpr int kWarpTma = 0, kWarpMma = 1, kWarpConv = 2, kConvWarps = 8, kWarpEpi = kWarpConv + kConvWarps,
              kEpiWarps = 4;
constexpr int kWarps = kWarpEpi + kEpiWarps;
constexpr int kThreads = kWarps * 32;
constexpr int kTmemCols = NACC * HN;  // 256
constexpr int CHUNK_BYTES = 128 * 128;  // 128 rows x 128 B

template <int WT>
struct HxTraits {
  static constexpr int BB = WT == KQ_Q4_0 ? 18 : WT == KQ_Q4_1 ? 20 : 34;
  static constexpr bool kExtra = WT != KQ_Q8_0;
  static constexpr int RAW_ROW = RB * BB;                  // 144 / 160 / 272 bytes
  static constexpr int RAW_STAGE = HN * RAW_ROW;
  static constexpr int HALF = RAW_ROW / 2;                 // 4 blocks
  static constexpr int WIN1 = HALF & ~15;                  // 16-byte aligned window start of the second half
  static constexpr int NV4 = (RAW_ROW - WIN1 + 15) / 16;   // 16-byte loads per thread (5 / 5 / 9)
  static constexpr int D1 = HALF - WIN1;                   // data offset of the second half inside its window
  static_assert((HALF + 15) / 16 <= NV4, "first-half window");
  static constexpr int OFF_A = 0;
  static constexpr int OFF_W = OFF_A + SA * CHUNK_BYTES;
  static constexpr int OFF_X = OFF_W + SW * CHUNK_BYTES;
  static constexpr int OFF_RAW = OFF_X + (kExtra ? 2 * CHUNK_BYTES : 0);
  static constexpr int OFF_BAR = OFF_RAW + SR * RAW_STAGE;
  static constexpr int NBARS = 2 * SA + 2 * SW + 2 * SR + 2 * NACC + 2;
  static constexpr int OFF_TMEM = OFF_BAR + NBARS * 8;
  static constexpr int SMEM = OFF_TMEM + 16 + 1024;
  static_assert(RAW_ROW % 16 == 0, "raw rows must stay 16-byte aligned");
  static_assert(SMEM <= 232448, "shared memory budget");
};

__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}

// Instruction descriptor, kind::f16: D f32, A = B = f16, both K-major.
__host__ __device__ constexpr uint32_t idesc_f16() {
  return (1u << 4) | ((uint32_t)(HN >> 3) << 17) | ((uint32_t)(HM >> 4) << 24);
}

__device__ __forceinline__ uint32_t hsub2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t hfma2(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// Four byte-codes c (one per byte of `bytes`, each < 256) -> two f16x2 words
// holding (M + c) exactly, M = 1024 (fp16 exponent 10: unit spacing).
__device__ __forceinline__ void magic4(uint32_t bytes, uint32_t& lo, uint32_t& hi) {
  lo = __byte_perm(bytes, 0x64646464u, 0x4140);
  hi = __byte_perm(bytes, 0x64646464u, 0x4342);
}

// Per-thread 32-bit word at compile-time byte offset OFF (even) of the loaded window.
template <int OFF, int N>
__device__ __forceinline__ uint32_t win32(const uint32_t (&w)[N]) {
  static_assert(OFF % 2 == 0 && OFF / 4 + 1 < N + 1, "window offset");
  if constexpr ((OFF & 3) == 0) {
    return w[OFF / 4];
  } else {
    return __funnelshift_r(w[OFF / 4], w[OFF / 4 + 1], 16);
  }
}
template <int OFF, int N>
__device__ __forceinline__ uint32_t win16(const uint32_t (&w)[N]) {
  if constexpr ((OFF & 3) == 0) {
    return w[OFF / 4] & 0xFFFFu;
  } else {
    return w[OFF / 4] >> 16;
  }
}

// Converts the 4 blocks at data offset D of the window into 4 x 32 fp16
// values: out[j][0..15] = packed pairs (k = 2i, 2i+1) of block j, and the X_w
// value of each block.
template <int WT, int D, int N>
__device__ __forceinline__ void convert4(const uint32_t (&w)[N], uint32_t (&out)[4][16], uint32_t (&xw)[4]) {
  using T = HxTraits<WT>;
  // one instantiation per block: every field offset is a compile-time constant
  auto blk = [&](auto jc) {
    constexpr int j = decltype(jc)::value;
    constexpr int o = D + j * T::BB;
    const uint32_t dh = win16<o>(w);
    const uint32_t d2 = dh | (dh << 16);
    if constexpr (WT == KQ_Q8_0) {
      // codes: 32 int8 at o + 2; c ^ 0x80 = c + 128 in 0..255 -> M + c + 128
      const uint32_t c0 = win32<o + 2>(w), c1 = win32<o + 6>(w), c2 = win32<o + 10>(w), c3 = win32<o + 14>(w);
      const uint32_t c4 = win32<o + 18>(w), c5 = win32<o + 22>(w), c6 = win32<o + 26>(w), c7 = win32<o + 30>(w);
      const uint32_t cs[8] = {c0, c1, c2, c3, c4, c5, c6, c7};
      constexpr uint32_t kOff = 0x64806480u;  // (1152, 1152)
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        uint32_t lo, hi;
        magic4(cs[q] ^ 0x80808080u, lo, hi);
        out[j][2 * q] = hmul2(hsub2(lo, kOff), d2);
        out[j][2 * q + 1] = hmul2(hsub2(hi, kOff), d2);
      }
      xw[j] = 0;
    } else {
      constexpr int qo = o + (WT == KQ_Q4_0 ? 2 : 4);
      uint32_t m2 = 0;
      if constexpr (WT == KQ_Q4_1) {
        const uint32_t mh = win16<o + 2>(w);
        m2 = mh | (mh << 16);
      }
      const uint32_t a0 = win32<qo>(w), a1 = win32<qo + 4>(w), a2 = win32<qo + 8>(w), a3 = win32<qo + 12>(w);
      const uint32_t as[4] = {a0, a1, a2, a3};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint32_t l0, l1, h0, h1;
        magic4(as[q] & 0x0F0F0F0Fu, l0, l1);          // elements 4q .. 4q+3
        magic4((as[q] >> 4) & 0x0F0F0F0Fu, h0, h1);   // elements 16+4q .. 16+4q+3
        if constexpr (WT == KQ_Q4_0) {
          constexpr uint32_t k1032 = 0x64086408u;  // (1032, 1032): M + c - 1032 = c - 8 exactly
          out[j][2 * q] = hmul2(hsub2(l0, k1032), d2);
          out[j][2 * q + 1] = hmul2(hsub2(l1, k1032), d2);
          out[j][8 + 2 * q] = hmul2(hsub2(h0, k1032), d2);
          out[j][8 + 2 * q + 1] = hmul2(hsub2(h1, k1032), d2);
        } else {
          // the dequantised weight c d + m, one rounding (c exact after M + c - M)
          constexpr uint32_t k1024 = 0x64006400u;
          out[j][2 * q] = hfma2(hsub2(l0, k1024), d2, m2);
          out[j][2 * q + 1] = hfma2(hsub2(l1, k1024), d2, m2);
          out[j][8 + 2 * q] = hfma2(hsub2(h0, k1024), d2, m2);
          out[j][8 + 2 * q + 1] = hfma2(hsub2(h1, k1024), d2, m2);
        }
      }
      if constexpr (WT == KQ_Q4_0) {
        xw[j] = hmul2(dh, 0xC800u) & 0xFFFFu;  // -8 d (exact)
      } else {
        xw[j] = win16<o + 2>(w);  // m
      }
    }
  };
  blk(std::integral_constant<int, 0>{});
  blk(std::integral_constant<int, 1>{});
  blk(std::integral_constant<int, 2>{});
  blk(std::integral_constant<int, 3>{});
}

struct HxParams {
  int M, N, K, Kp;
  int nmain, ngrp, nb;
  int num_m_tiles, num_tiles;
  float* out;
  const float* rscale;  // per activation row: 2^e undoing the prep kernel's scaling
  int* err;
};

// position of main chunk c's extra chunk, if one follows it
__device__ __forceinline__ bool extra_after(int c, int nmain) { return (c % GRP) == GRP - 1 || c == nmain - 1; }

template <int WT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_hx_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_raw,
                   HxParams p) {
  using T = HxTraits<WT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + T::OFF_BAR);
  uint64_t* a_full = bars;
  uint64_t* a_empty = a_full + SA;
  uint64_t* w_full = a_empty + SA;
  uint64_t* w_empty = w_full + SW;
  uint64_t* raw_full = w_empty + SW;
  uint64_t* raw_empty = raw_full + SR;
  uint64_t* tm_full = raw_empty + SR;
  uint64_t* tm_empty = tm_full + NACC;
  uint64_t* x_empty = tm_empty + NACC;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + T::OFF_TMEM);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nraw = p.nmain / 4;
  const int my_tiles = (p.num_tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;

  if (threadIdx.x == 0) {
    for (int i = 0; i < SA; ++i) {
      mbar_init(&a_full[i], 1);
      mbar_init(&a_empty[i], 1);
    }
    for (int i = 0; i < SW; ++i) {
      mbar_init(&w_full[i], kConvWarps / 2);  // one converter half writes a given chunk
      mbar_init(&w_empty[i], 1);
    }
    for (int i = 0; i < SR; ++i) {
      mbar_init(&raw_full[i], 1);
      mbar_init(&raw_empty[i], kConvWarps);
    }
    for (int i = 0; i < NACC; ++i) {
      mbar_init(&tm_full[i], 1);
      mbar_init(&tm_empty[i], kEpiWarps);
    }
    mbar_init(&x_empty[0], 1);
    mbar_init(&x_empty[1], 1);
    fence_mbar_init();
  }
  if constexpr (T::kExtra) {
    // X tiles start zeroed: columns past the last block stay finite (x 0 in A')
    for (int i = threadIdx.x; i < 2 * CHUNK_BYTES / 16; i += kThreads)
      reinterpret_cast<uint4*>(smem + T::OFF_X)[i] = make_uint4(0, 0, 0, 0);
    fence_proxy_async_smem();
  }
  if (warp == kWarpMma) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  bool dead = false;
  if (warp == kWarpTma) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tmap(&map_a);
      prefetch_tmap(&map_raw);
      int ia = 0, ir = 0;
      bool waited_pdl = false;
      for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x) {
        const int m0 = (t % p.num_m_tiles) * HM, n0 = (t / p.num_m_tiles) * HN;
        for (int r = 0; r < nraw; ++r, ++ir) {
          const int rs = ir % SR;
          if (ir >= SR) mbar_wait_or_poison(&raw_empty[rs], ((ir / SR) - 1) & 1, p.err, DEV_TIMEOUT_EMPTY, dead);
          mbar_arrive_expect_tx(&raw_full[rs], T::RAW_STAGE);
          tma_load_2d(smem + T::OFF_RAW + rs * T::RAW_STAGE, &map_raw, r * (T::RAW_ROW / 2), n0, &raw_full[rs]);
          if (!waited_pdl) {  // A' is produced by the preceding kernel
            pdl_wait();
            waited_pdl = true;
          }
          for (int c = 4 * r; c < 4 * r + 4; ++c) {
            const int nx = (T::kExtra && extra_after(c, p.nmain)) ? 2 : 1;
            for (int e = 0; e < nx; ++e, ++ia) {
              const int as = ia % SA;
              if (ia >= SA) mbar_wait_or_poison(&a_empty[as], ((ia / SA) - 1) & 1, p.err, DEV_TIMEOUT_EMPTY, dead);
              const int x = e == 0 ? c * CK : p.K + (c / GRP) * CK;
              mbar_arrive_expect_tx(&a_full[as], CHUNK_BYTES);
              tma_load_2d(smem + T::OFF_A + as * CHUNK_BYTES, &map_a, x, m0, &a_full[as]);
            }
          }
        }
      }
    }
  } else if (warp == kWarpMma) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16();
      const uint32_t a_base = smem_u32(smem + T::OFF_A);
      const uint32_t w_base = smem_u32(smem + T::OFF_W);
      const uint32_t x_base = smem_u32(smem + T::OFF_X);
      int ia = 0, iw = 0, ix = 0;
      for (int it = 0; it < my_tiles; ++it) {
        const int acc = it % NACC;
        if (it >= NACC) mbar_wait_or_poison(&tm_empty[acc], ((it / NACC) - 1) & 1, p.err, DEV_TIMEOUT_EMPTY, dead);
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * HN;
        for (int c = 0; c < p.nmain; ++c, ++ia, ++iw) {
          const int as = ia % SA, ws = iw % SW;
          mbar_wait_or_poison(&a_full[as], (ia / SA) & 1, p.err, DEV_TIMEOUT_FULL, dead);
          mbar_wait_or_poison(&w_full[ws], (iw / SW) & 1, p.err, DEV_TIMEOUT_FULL, dead);
          tc_fence_after();
          const uint64_t ad = sw128_desc(a_base + as * CHUNK_BYTES);
          const uint64_t bd = sw128_desc(w_base + ws * CHUNK_BYTES);
#pragma unroll
          for (int j = 0; j < CK / 16; ++j)
            mma_f16(d_tmem, ad + (uint64_t)(2 * j), bd + (uint64_t)(2 * j), idesc, (c | j) ? 1u : 0u);
          mma_commit(&a_empty[as]);
          mma_commit(&w_empty[ws]);
          if (T::kExtra && extra_after(c, p.nmain)) {
            ++ia;
            const int as2 = ia % SA;
            mbar_wait_or_poison(&a_full[as2], (ia / SA) & 1, p.err, DEV_TIMEOUT_FULL, dead);
            tc_fence_after();
            const uint64_t ad2 = sw128_desc(a_base + as2 * CHUNK_BYTES);
            const uint64_t xd = sw128_desc(x_base + (ix & 1) * CHUNK_BYTES);
#pragma unroll
            for (int j = 0; j < CK / 16; ++j)
              mma_f16(d_tmem, ad2 + (uint64_t)(2 * j), xd + (uint64_t)(2 * j), idesc, 1u);
            mma_commit(&a_empty[as2]);
            mma_commit(&x_empty[ix & 1]);
            ++ix;
          }
        }
        mma_commit(&tm_full[acc]);
      }
    }
  } else if (warp < kWarpEpi) {
    // ------------------------------------------------------------ converters
    const int cw = warp - kWarpConv;
    const int h = cw / (kConvWarps / 2);          // which 4 blocks of the raw stage
    const int row = (cw % (kConvWarps / 2)) * 32 + lane;
    const int off0 = sw128_off(row, 0);
    int irr = 0, ic = 0, ixg = 0;
    for (int it = 0; it < my_tiles; ++it) {
      for (int r = 0; r < nraw; ++r, ++irr) {
        const int rs = irr % SR;
        mbar_wait_or_poison(&raw_full[rs], (irr / SR) & 1, p.err, DEV_TIMEOUT_FULL, dead);
        uint32_t win[T::NV4 * 4];
        {
          const uint4* src = reinterpret_cast<const uint4*>(smem + T::OFF_RAW + rs * T::RAW_STAGE + row * T::RAW_ROW +
                                                            (h ? T::WIN1 : 0));
#pragma unroll
          for (int i = 0; i < T::NV4; ++i) {
            const uint4 v = src[i];
            win[4 * i] = v.x;
            win[4 * i + 1] = v.y;
            win[4 * i + 2] = v.z;
            win[4 * i + 3] = v.w;
          }
        }
        fence_proxy_async_smem();  // generic reads of a TMA-refilled stage, before its release
        __syncwarp();
        if (lane == 0) mbar_arrive(&raw_empty[rs]);
        uint32_t vals[4][16];
        uint32_t xw[4];
        if (h == 0) {
          convert4<WT, 0>(win, vals, xw);
        } else {
          convert4<WT, T::D1>(win, vals, xw);
        }
        // this thread's two chunks: 4r + 2h, 4r + 2h + 1 (global chunk counter ic + ...)
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const int gc = ic + 4 * r + 2 * h + q;
          const int ws = gc % SW;
          if (gc >= SW) mbar_wait_or_poison(&w_empty[ws], ((gc / SW) - 1) & 1, p.err, DEV_TIMEOUT_EMPTY, dead);
          uint8_t* tile = smem + T::OFF_W + ws * CHUNK_BYTES;
          // chunk q holds blocks 2q, 2q+1 of this thread's four: 8 x 16-byte pieces
#pragma unroll
          for (int jj = 0; jj < 2; ++jj) {
#pragma unroll
            for (int pc = 0; pc < 4; ++pc) {
              const int piece = jj * 4 + pc;  // 16-byte piece index inside the 128-byte row
              *reinterpret_cast<uint4*>(tile + (off0 ^ (piece << 4))) =
                  make_uint4(vals[2 * q + jj][4 * pc], vals[2 * q + jj][4 * pc + 1], vals[2 * q + jj][4 * pc + 2],
                             vals[2 * q + jj][4 * pc + 3]);
            }
          }
        }
        if constexpr (T::kExtra) {
          const int b0 = 8 * r + 4 * h;  // first block (tile-local) of this thread's four
          const int g = b0 / 64;
          const int xgc = ixg + g;
          if ((b0 & 63) < 8 && xgc >= 2)  // first write of group g: the MMA must be done with the buffer
            mbar_wait_or_poison(&x_empty[xgc & 1], ((xgc / 2) - 1) & 1, p.err, DEV_TIMEOUT_EMPTY, dead);
          uint8_t* xt = smem + T::OFF_X + (xgc & 1) * CHUNK_BYTES;
          const int col = b0 & 63;  // multiple of 4: one 8-byte store
          *reinterpret_cast<uint2*>(xt + (off0 ^ ((col >> 3) << 4)) + (col & 7) * 2) =
              make_uint2(xw[0] | (xw[1] << 16), xw[2] | (xw[3] << 16));
        }
        fence_proxy_async_smem();  // generic-proxy writes -> tensor-core reads
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&w_full[(ic + 4 * r + 2 * h) % SW]);
          mbar_arrive(&w_full[(ic + 4 * r + 2 * h + 1) % SW]);
        }
      }
      ic += p.nmain;
      ixg += p.ngrp;
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    int it = 0;
    for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x, ++it) {
      const int acc = it % NACC;
      mbar_wait_or_poison(&tm_full[acc], (it / NACC) & 1, p.err, DEV_TIMEOUT_FULL, dead);
      tc_fence_after();
      const int m0 = (t % p.num_m_tiles) * HM, n0 = (t / p.num_m_tiles) * HN;
      const int m = m0 + row;
      float* orow = p.out + (size_t)m * p.N;
      const float rs = m < p.M ? p.rscale[m] : 1.0f;
      const bool full_cols = (n0 + HN <= p.N) && (p.N & 3) == 0;
#pragma unroll 1
      for (int half = 0; half < 2; ++half) {
        uint32_t v0[32], v1[32];
        const uint32_t ta = tmem_base + lane_addr + acc * HN + half * 64;
        tmem_ld32(ta, v0);
        tmem_ld32(ta + 32, v1);
        tmem_ld_wait();
        auto v = [&](int c) { return c < 32 ? v0[c] : v1[c - 32]; };
        if (half == 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tm_empty[acc]);
        }
        if (m < p.M) {
          const int c0 = n0 + half * 64;
          if (full_cols) {
#pragma unroll
            for (int c = 0; c < 64; c += 4)
              *reinterpret_cast<float4*>(orow + c0 + c) =
                  make_float4(__uint_as_float(v(c)) * rs, __uint_as_float(v(c + 1)) * rs,
                              __uint_as_float(v(c + 2)) * rs, __uint_as_float(v(c + 3)) * rs);
          } else {
#pragma unroll
            for (int c = 0; c < 64; ++c)
              if (c0 + c < p.N) orow[c0 + c] = __uint_as_float(v(c)) * rs;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kWarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// A'[m, k] = fp16(q * d * 2^-e_m) from the staging layout, plus the extra
// columns (scaled alike); rscale[m] = 2^e_m. One CTA per activation row. The
// per-row power of two puts the row's largest magnitude in [2^14, 2^15), so no
// element overflows fp16 and small rows do not fall into fp16 subnormals; the
// GEMM epilogue multiplies row m by rscale[m] (exact). Extra blocks nb .. KX-1
// are zero.
template <int WT>
__global__ void __launch_bounds__(128) act16_kernel(Act8 act, int M, int K, int Kp, __half* __restrict__ a16,
                                                    float* __restrict__ rscale) {
  const int nb = K / 32;
  const int nbx = Kp - K;  // extra columns (0 for q8_0)
  const int m = blockIdx.x;
  if (m >= M) return;
  const float2* ds = act.ds + (size_t)m * nb;
  // pass 1: largest magnitude of the row (|q| <= 127; the residual column
  // s - d sum q stays below 127 d: 32 rounding residuals of at most d / 2 each,
  // plus the fp16 rounding of s)
  float amax = 0.0f;
  for (int b = threadIdx.x; b < nb; b += blockDim.x) amax = fmaxf(amax, 127.0f * fabsf(ds[b].x));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  __shared__ float wmax[4];
  if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = amax;
  __syncthreads();
  amax = fmaxf(fmaxf(wmax[0], wmax[1]), fmaxf(wmax[2], wmax[3]));
  int e = 0;  // amax in [2^E, 2^(E+1)) -> e = E - 14
  if (amax > 0.0f && isfinite(amax)) e = max(-100, min(100, (int)((__float_as_uint(amax) >> 23) & 0xFF) - 127 - 14));
  const float down = __uint_as_float((uint32_t)(127 - e) << 23);  // 2^-e
  if (threadIdx.x == 0) rscale[m] = __uint_as_float((uint32_t)(127 + e) << 23);
  __half* arow = a16 + (size_t)m * Kp;
  for (int b = threadIdx.x; b < nb; b += blockDim.x) {
    const float2 v = ds[b];
    const float d = v.x * down;  // exact (power-of-two scaling)
    const int4* src = reinterpret_cast<const int4*>(act.qs + (size_t)m * K + 32 * b);
    const int4 c01 = src[0], c23 = src[1];
    const int cw[8] = {c01.x, c01.y, c01.z, c01.w, c23.x, c23.y, c23.z, c23.w};
    uint32_t outw[16];
    int qsum = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
#pragma unroll
      for (int e2 = 0; e2 < 4; e2 += 2) {
        const int q0 = (int)(int8_t)((cw[i] >> (8 * e2)) & 0xFF);
        const int q1 = (int)(int8_t)((cw[i] >> (8 * e2 + 8)) & 0xFF);
        qsum += q0 + q1;
        const __half2 hv = __floats2half2_rn((float)q0 * d, (float)q1 * d);  // q * d exact in fp32
        outw[2 * i + e2 / 2] = *reinterpret_cast<const uint32_t*>(&hv);
      }
    }
    uint4* dst = reinterpret_cast<uint4*>(arow + 32 * b);
#pragma unroll
    for (int i = 0; i < 4; ++i) dst[i] = make_uint4(outw[4 * i], outw[4 * i + 1], outw[4 * i + 2], outw[4 * i + 3]);
    if constexpr (WT != KQ_Q8_0) arow[K + b] = __float2half_rn((v.y - v.x * (float)qsum) * down);
  }
  for (int b = nb + threadIdx.x; b < nbx; b += blockDim.x) arow[K + b] = __float2half_rn(0.0f);
}

template <int WT>
kq_status_t launch_hx(const void* w, Act8 act, float* out, int M, int N, int K, bool pdl, cudaStream_t s, int* err) {
  using T = HxTraits<WT>;
  const int nb = K / 32;
  const int nmain = K / CK;
  const int ngrp = T::kExtra ? (nmain + GRP - 1) / GRP : 0;
  const int Kp = K + ngrp * CK;
  const size_t a16_bytes = ((size_t)M * Kp * sizeof(__half) + 255) & ~(size_t)255;
  uint8_t* ws = static_cast<uint8_t*>(workspace(WS_A16, a16_bytes + (size_t)M * sizeof(float)));
  if (!ws) return KQ_ERR_NOMEM;
  __half* a16 = reinterpret_cast<__half*>(ws);
  float* rscale = reinterpret_cast<float*>(ws + a16_bytes);
  {
    act16_kernel<WT><<<M, 128, 0, s>>>(act, M, K, Kp, a16, rscale);
    kq_status_t st = check_launch("act16");
    if (st) return st;
  }
  CUtensorMap m_a, m_raw;
  if (!encode_map(&m_a, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a16, (uint64_t)Kp, (uint64_t)M, (uint64_t)Kp * 2, CK, HM,
                  CU_TENSOR_MAP_SWIZZLE_128B))
    return fail(KQ_ERR_CUDA, "tensor map (fp16 activations) rejected");
  const uint64_t rowbytes = (uint64_t)nb * T::BB;
  if (!encode_map(&m_raw, CU_TENSOR_MAP_DATA_TYPE_UINT16, w, rowbytes / 2, (uint64_t)N, rowbytes, T::RAW_ROW / 2, HN,
                  CU_TENSOR_MAP_SWIZZLE_NONE))
    return fail(KQ_ERR_CUDA, "tensor map (weights) rejected");

  auto kern = gemm_hx_kernel<WT>;
  if (kq_status_t st = ensure_dynamic_smem(reinterpret_cast<const void*>(kern), T::SMEM, "gemm_hx smem attribute"))
    return st;
  HxParams p;
  p.M = M; p.N = N; p.K = K; p.Kp = Kp;
  p.nmain = nmain; p.ngrp = ngrp; p.nb = nb;
  p.num_m_tiles = (M + HM - 1) / HM;
  p.num_tiles = p.num_m_tiles * ((N + HN - 1) / HN);
  p.out = out;
  p.rscale = rscale;
  p.err = err ? err : device_error_word();
  const int grid = std::max(1, std::min(sm_count(), p.num_tiles));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = T::SMEM;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  (void)pdl;  // the prep kernel always precedes the GEMM on this stream
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, m_a, m_raw, p);
  if (e != cudaSuccess) return check_cuda(e, "gemm_hx launch");
  return check_launch("gemm_hx");
}

}  // namespace

bool gemm_hx_supported(int wtype, int M, int N, int K, const void* w, Act8 act) {
  (void)wtype;
  (void)act;
  return M > 8 && N >= 1 && K >= 256 && K % 256 == 0 && (reinterpret_cast<uintptr_t>(w) & 15) == 0;
}

kq_status_t launch_gemm_hx(int wtype, const void* w, Act8 act, float* out, int M, int N, int K, bool pdl,
                           cudaStream_t s, int* err) {
  switch (wtype) {
    case KQ_Q4_0: return launch_hx<KQ_Q4_0>(w, act, out, M, N, K, pdl, s, err);
    case KQ_Q4_1: return launch_hx<KQ_Q4_1>(w, act, out, M, N, K, pdl, s, err);
    case KQ_Q8_0: return launch_hx<KQ_Q8_0>(w, act, out, M, N, K, pdl, s, err);
    default: return fail(KQ_ERR_INVALID, "unknown weight type %d", wtype);
  }
}

}  // namespace kq
