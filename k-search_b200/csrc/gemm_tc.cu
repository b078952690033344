// Tensor-core quantised GEMM for M > 8 activation rows (llama.cpp's
// mul_mat_q family) on sm_100a: tcgen05.mma.kind::i8 with TMEM accumulators.
//
//   out[m, n] = sum_b scale(m, n, b) * sumi[m, n, b]
//   sumi[m, n, b] = sum_{i<32} q_a[m, 32b+i] * q_w[n, b, i]      (exact int32)
//   q8_0: scale term d_w * d_a * sumi                   (gemm_reference.h:311-336)
//   q4_0: d_w * (d_a * sumi - 8 s_a)   (codes 0..15)    (gemm_ref.py:100-153)
//   q4_1: d_w * d_a * sumi + m_w * s_a                  (gemm_ref.py:274-331)
//
// Every 32-wide K block has its own scales, so each block's product is a
// separate MMA (K = 32, one instruction) into a fresh TMEM buffer; the fp32
// accumulation across blocks happens in the epilogue warps' registers.
//
// CTA = 20 warps, one CTA per SM, persistent over 128 x 128 output tiles
// (tokens x weight rows), tokens fastest so co-running CTAs share weights in L2:
//   warp 0      TMA producer: activation codes (int8 [M, K], 128B-swizzled
//               boxes of 128 rows x 128 B = 4 blocks), activation (d, s)
//               pairs, and raw weight rows (the unchanged AoS q-blocks,
//               128 rows x 8 blocks per box); every CTA loads its own tiles.
//   warp 1      MMA issuer (one thread), owns the TMEM allocation. Per block:
//               a kind::f16 MMA writes the bias words (see kBias), then the
//               block's kind::i8 MMA accumulates onto them; one commit.
//   warps 2-3   converters: two weight rows per thread, the 4 blocks of a stage
//               into int8 codes in the UMMA K-major SWIZZLE_128B layout plus
//               fp32 scale rows, running ahead of the MMA by up to SWS stages.
//   warps 4-19  epilogue: read each block's result from TMEM (tcgen05.ld,
//               32 columns per thread, one half-load ahead), hand the buffer
//               back, apply the block's scales and accumulate in fp32 registers.
//               4 TMEM buffers of 128 columns let the MMA run a stage ahead.
// Every hand-off is an mbarrier; every wait is bounded (kq_device.cuh).
#include <cuda.h>

#include <algorithm>
#include <mutex>

#include "kq_internal.h"
#include "kq_device.cuh"
#include "kq_tc.cuh"

namespace kq {
namespace {

using namespace tc;


constexpr int TM = 128;        // tokens per tile (TMEM lanes)
constexpr int TN = 128;        // weight rows per tile (TMEM columns per buffer)
constexpr int KSUB = 4;        // blocks per activation / converted-weight stage (128 B of K)
constexpr int KRAW = 8;        // blocks per raw weight stage (16-byte aligned for all block sizes)
constexpr int SA = 4;          // activation stages (codes + scales)
constexpr int SWS = 4;         // converted weight stages (codes + scales)
constexpr int SRAW = 2;        // raw weight stages
constexpr int NBUF = 4;        // TMEM buffers (one per block of a stage)
constexpr int kWarpTma = 0, kWarpMma = 1, kWarpConv = 2, kConvWarps = 2, kWarpEpi = kWarpConv + kConvWarps,
              kEpiWarps = 8;
constexpr int kEpiCols = TN / (kEpiWarps / 4);  // columns per epilogue thread (64)
constexpr int kChunk = 16;                      // columns per TMEM load
constexpr int kChunks = kEpiCols / kChunk;      // loads per block (4)
constexpr int kWarps = kWarpEpi + kEpiWarps;
constexpr int kThreads = kWarps * 32;
constexpr int kTmemCols = NBUF * TN;  // 512
static_assert(NBUF == KSUB, "one TMEM buffer per K block of a stage");
constexpr int kConvRows = TN / (kConvWarps * 32);  // weight rows per converter thread (2)

template <int WT>
struct TcTraits {
  static constexpr int BB = WT == KQ_Q4_0 ? 18 : WT == KQ_Q4_1 ? 20 : 34;
  static constexpr bool kHasMin = WT == KQ_Q4_1;
  static constexpr bool kSignedW = WT == KQ_Q8_0;
  static constexpr int RAW_ROW = KRAW * BB;                 // bytes per raw row per stage
  static constexpr int RAW_STAGE = TN * RAW_ROW;
  static constexpr int ACT_TILE = TM * 128;                 // 16 KB, 1024-aligned
  static constexpr int W_TILE = TN * 128;                   // 16 KB
  static constexpr int ASC_STAGE = TM * KSUB * 8;           // (d, s) per row and block
  static constexpr int WSC_STAGE = KSUB * TN * 4 * (kHasMin ? 2 : 1);
  static constexpr int PRE_TILE = 8 * 128;   // one 8-row swizzle atom, repeated over 128 rows (SBO 0)
  // byte offsets in dynamic shared memory (base aligned to 1024)
  static constexpr int OFF_ACT = 0;
  static constexpr int OFF_W = OFF_ACT + SA * ACT_TILE;
  static constexpr int OFF_RAW = OFF_W + SWS * W_TILE;
  static constexpr int OFF_ASC = OFF_RAW + SRAW * RAW_STAGE;
  static constexpr int OFF_WSC = OFF_ASC + SA * ASC_STAGE;
  static constexpr int OFF_PRE = (OFF_WSC + SWS * WSC_STAGE + 1023) / 1024 * 1024;  // bias-preset operands
  static constexpr int OFF_BAR = OFF_PRE + 2 * PRE_TILE;
  static constexpr int NBARS = 2 * SA + 2 * SWS + 2 * SRAW + 2 * NBUF;
  static constexpr int OFF_TMEM = OFF_BAR + NBARS * 8;
  static constexpr int SMEM = OFF_TMEM + 16 + 1024;  // + alignment slack
  static_assert(RAW_ROW % 16 == 0, "raw rows must stay 16-byte aligned");
  static_assert(SMEM <= 232448, "shared memory budget");
};


__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}



// Packed fp32 pairs (one instruction, two lanes of math each).
__device__ __forceinline__ uint64_t pk2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ uint64_t pk2u(uint32_t lo, uint32_t hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo), "r"(hi));
  return r;
}
__device__ __forceinline__ float2 upk2(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// Integer -> float without a conversion instruction: every TMEM accumulator
// word is preset to kBias = bits of 12582912.0f (1.5 * 2^23) and the MMA
// accumulates the block's int32 sum onto it; for |sumi| < 2^22 the result
// (kBias + sumi) is the fp32 bit pattern of 12582912 + sumi exactly. Then
// d * sumi = fma(f, d, -12582912 d), exact before the final rounding when
// 12582912 d is exact (d with <= 22 significant bits; fp16 scales always
// are, fp32 scales are rounded to 22 bits, a relative change below 2^-22).
constexpr uint32_t kBias = 0x4B400000u;
constexpr float kBiasF = 12582912.0f;

// The bias is written by the tensor core itself: before each block's int8 MMA
// a kind::f16 MMA with accumulate off computes A_pre x B_pre^T, where every row
// of A_pre is (3072, 0, ..., 0) and every row of B_pre is (4096, 0, ..., 0):
// 3072 * 4096 = 12582912 exactly, so each fp32 word becomes kBias. The int8
// MMA then accumulates (integer add) onto those bits.
constexpr uint16_t kPreA = 0x6A00;  // fp16 3072
constexpr uint16_t kPreB = 0x6C00;  // fp16 4096

__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ float round22(float d) {
  return __uint_as_float((__float_as_uint(d) + 2u) & ~3u);
}

// Instruction descriptor, kind::i8: D s32, A = activations (signed),
// B = weights (signed for q8_0, unsigned codes 0..15 for q4_x), both K-major.
__host__ __device__ constexpr uint32_t idesc_i8(bool b_signed) {
  return (2u << 4)                        // D format S32
         | (1u << 7)                      // A signed 8-bit
         | ((b_signed ? 1u : 0u) << 10)   // B signed / unsigned 8-bit
         | ((uint32_t)(TN >> 3) << 17)    // N
         | ((uint32_t)(TM >> 4) << 24);   // M
}

// Instruction descriptor, kind::f16: D f32, A = B = f16, both K-major.
__host__ __device__ constexpr uint32_t idesc_f16() {
  return (1u << 4) | ((uint32_t)(TN >> 3) << 17) | ((uint32_t)(TM >> 4) << 24);
}

template <int NC>
__device__ __forceinline__ void tmem_ldh(uint32_t taddr, uint32_t (&v)[NC]) {
  if constexpr (NC == 32) {
    tmem_ld32(taddr, v);
  } else {
    static_assert(NC == 16, "TMEM load width");
    tmem_ld16(taddr, v);
  }
}

struct TcParams {
  int M, N, K, nb;
  int num_m_tiles, num_tiles;
  OutSpec out;
  int* err;
};

// SWIZZLE_128B K-major descriptor whose 8-row groups all alias one 1 KB atom
// (SBO = 0): 128 identical-pattern rows from 8 stored ones.
__device__ __forceinline__ uint64_t sw128_desc_rep8(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;    // LBO (unused for swizzled K-major)
  d |= (uint64_t)1 << 46;    // version
  d |= (uint64_t)2 << 61;    // SWIZZLE_128B
  return d;
}

template <int WT, bool SCATTER>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap map_act, const __grid_constant__ CUtensorMap map_asc,
                   const __grid_constant__ CUtensorMap map_raw, const __grid_constant__ TcParams p) {
  using T = TcTraits<WT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + T::OFF_BAR);
  uint64_t* act_full = bars;
  uint64_t* act_empty = act_full + SA;
  uint64_t* w_full = act_empty + SA;
  uint64_t* w_empty = w_full + SWS;
  uint64_t* raw_full = w_empty + SWS;
  uint64_t* raw_empty = raw_full + SRAW;
  uint64_t* tm_full = raw_empty + SRAW;
  uint64_t* tm_empty = tm_full + NBUF;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + T::OFF_TMEM);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkb8 = p.nb / KRAW;
  const int spt = p.nb / KSUB;  // K stages per tile (even: nb % 8 == 0)
  const int my_tiles = (p.num_tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
  const int total = my_tiles * spt;  // K stages this CTA runs

  if (threadIdx.x == 0) {
    for (int i = 0; i < SA; ++i) {
      mbar_init(&act_full[i], 1);
      mbar_init(&act_empty[i], 1 + kEpiWarps);  // MMA commit + epilogue warps (they read the scales)
    }
    for (int i = 0; i < SWS; ++i) {
      mbar_init(&w_full[i], kConvWarps);
      mbar_init(&w_empty[i], 1 + kEpiWarps);
    }
    for (int i = 0; i < SRAW; ++i) {
      mbar_init(&raw_full[i], 1);
      mbar_init(&raw_empty[i], kConvWarps);
    }
    for (int i = 0; i < NBUF; ++i) {
      mbar_init(&tm_full[i], 1);
      mbar_init(&tm_empty[i], kEpiWarps);
    }
    fence_mbar_init();
  }
  {
    // bias-preset operands: rows (c, 0, ..., 0), c = 3072 (A) / 4096 (B);
    // logical chunk 0 of row r sits in physical chunk r (128B swizzle)
    uint4* pre = reinterpret_cast<uint4*>(smem + T::OFF_PRE);
    for (int i = threadIdx.x; i < 2 * T::PRE_TILE / 16; i += kThreads) {
      const int tile = i / (T::PRE_TILE / 16), r = (i % (T::PRE_TILE / 16)) / 8, c = i % 8;
      pre[i] = make_uint4(c == r ? (uint32_t)(tile == 0 ? kPreA : kPreB) : 0u, 0u, 0u, 0u);
    }
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
      prefetch_tmap(&map_act);
      prefetch_tmap(&map_asc);
      prefetch_tmap(&map_raw);
      int ia = 0, ir = 0;
      bool waited_pdl = false;
      for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x) {
        const int m0 = (t % p.num_m_tiles) * TM, n0 = (t / p.num_m_tiles) * TN;
        for (int k8 = 0; k8 < nkb8; ++k8, ++ir) {
          const int rs = ir % SRAW;
          if (ir >= SRAW) mbar_wait_idle_or_poison(&raw_empty[rs], ((ir / SRAW) - 1) & 1, p.err, DEV_TIMEOUT_EMPTY, dead);
          mbar_arrive_expect_tx(&raw_full[rs], T::RAW_STAGE);
          tma_load_2d(smem + T::OFF_RAW + rs * T::RAW_STAGE, &map_raw, k8 * (T::RAW_ROW / 2), n0, &raw_full[rs]);
          if (!waited_pdl) {  // activations are produced by the preceding kernel
            pdl_wait();
            waited_pdl = true;
          }
          for (int sub = 0; sub < KRAW / KSUB; ++sub, ++ia) {
            const int as = ia % SA;
            if (ia >= SA) mbar_wait_idle_or_poison(&act_empty[as], ((ia / SA) - 1) & 1, p.err, DEV_TIMEOUT_EMPTY, dead);
            const int kb = k8 * KRAW + sub * KSUB;  // first block of this stage
            mbar_arrive_expect_tx(&act_full[as], T::ACT_TILE + T::ASC_STAGE);
            tma_load_2d(smem + T::OFF_ACT + as * T::ACT_TILE, &map_act, kb * 32, m0, &act_full[as]);
            tma_load_2d(smem + T::OFF_ASC + as * T::ASC_STAGE, &map_asc, kb * 2, m0, &act_full[as]);
          }
        }
      }
    }
  } else if (warp == kWarpMma) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_i8(T::kSignedW);
      constexpr uint32_t idesc_pre = idesc_f16();
      const uint32_t act_base = smem_u32(smem + T::OFF_ACT);
      const uint32_t w_base = smem_u32(smem + T::OFF_W);
      const uint64_t pre_a = sw128_desc_rep8(smem_u32(smem + T::OFF_PRE));
      const uint64_t pre_b = sw128_desc_rep8(smem_u32(smem + T::OFF_PRE + T::PRE_TILE));
      for (int gs = 0; gs < total; ++gs) {
        const int as = gs % SA, ws = gs % SWS;
        mbar_wait_idle_or_poison(&act_full[as], (gs / SA) & 1, p.err, DEV_TIMEOUT_FULL, dead);
        mbar_wait_idle_or_poison(&w_full[ws], (gs / SWS) & 1, p.err, DEV_TIMEOUT_FULL, dead);
        const uint64_t adesc = sw128_desc(act_base + as * T::ACT_TILE);
        const uint64_t bdesc = sw128_desc(w_base + ws * T::W_TILE);
#pragma unroll
        for (int j = 0; j < KSUB; ++j) {
          if (gs > 0) mbar_wait_idle_or_poison(&tm_empty[j], (gs - 1) & 1, p.err, DEV_TIMEOUT_EMPTY, dead);
          tc_fence_after();
          // bias words from the tensor core, then K block j of the stage
          // (+32 bytes inside the 128-byte swizzle atom) accumulated onto them
          mma_f16(tmem_base + j * TN, pre_a, pre_b, idesc_pre, 0u);
          mma_i8(tmem_base + j * TN, adesc + (uint64_t)(2 * j), bdesc + (uint64_t)(2 * j), idesc, 1u);
          mma_commit(&tm_full[j]);
        }
        mma_commit(&act_empty[as]);
        mma_commit(&w_empty[ws]);
      }
    }
  } else if (warp < kWarpEpi) {
    // ------------------------------------------------------------ converters
    const int crow0 = (warp - kWarpConv) * 32 + lane;  // rows crow0 + kConvWarps * 32 * r are converted here
    constexpr int SB = KSUB * T::BB;                  // bytes of one stage of a raw row
    constexpr int HB = 2 * T::BB;                     // two blocks (36 / 40 / 68 bytes: 4-byte aligned)
    constexpr int NW = HB / 4;
    for (int gs = 0; gs < total; ++gs) {
      const int irr = gs >> 1, sub = gs & 1;
      const int rs = irr % SRAW;
      mbar_wait_idle_or_poison(&raw_full[rs], (irr / SRAW) & 1, p.err, DEV_TIMEOUT_FULL, dead);
      const int ws = gs % SWS;
      if (gs >= SWS) mbar_wait_idle_or_poison(&w_empty[ws], ((gs / SWS) - 1) & 1, p.err, DEV_TIMEOUT_EMPTY, dead);
      uint8_t* wt = smem + T::OFF_W + ws * T::W_TILE;
      float* wsc = reinterpret_cast<float*>(smem + T::OFF_WSC + ws * T::WSC_STAGE);
#pragma unroll 1
      for (int rr = 0; rr < kConvRows; ++rr) {
      const int crow = crow0 + rr * kConvWarps * 32;
      const uint32_t* src =
          reinterpret_cast<const uint32_t*>(smem + T::OFF_RAW + rs * T::RAW_STAGE + crow * T::RAW_ROW + sub * SB);
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {  // blocks 2hh, 2hh + 1 of the stage
        uint32_t w[NW + 1];
#pragma unroll
        for (int i = 0; i < NW; ++i) w[i] = src[hh * NW + i];
        w[NW] = 0;
        auto u32 = [&](int off) -> uint32_t {
          return (off & 3) ? __funnelshift_r(w[off >> 2], w[(off >> 2) + 1], 16) : w[off >> 2];
        };
        auto u16 = [&](int off) -> uint32_t { return (off & 3) ? (w[off >> 2] >> 16) : (w[off >> 2] & 0xFFFFu); };
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
          const int o = jj * T::BB;  // compile-time after unrolling
          const int j = 2 * hh + jj;
          uint4 c0, c1;
          float mn = 0.0f;
          const float d = half_bits_to_float(u16(o));
          if constexpr (WT == KQ_Q8_0) {
            c0 = make_uint4(u32(o + 2), u32(o + 6), u32(o + 10), u32(o + 14));
            c1 = make_uint4(u32(o + 18), u32(o + 22), u32(o + 26), u32(o + 30));
          } else {
            const int q = o + (WT == KQ_Q4_0 ? 2 : 4);
            if constexpr (WT == KQ_Q4_1) mn = half_bits_to_float(u16(o + 2));
            const uint32_t a0 = u32(q), a1 = u32(q + 4), a2 = u32(q + 8), a3 = u32(q + 12);
            c0 = make_uint4(a0 & 0x0F0F0F0Fu, a1 & 0x0F0F0F0Fu, a2 & 0x0F0F0F0Fu, a3 & 0x0F0F0F0Fu);
            c1 = make_uint4((a0 >> 4) & 0x0F0F0F0Fu, (a1 >> 4) & 0x0F0F0F0Fu, (a2 >> 4) & 0x0F0F0F0Fu,
                            (a3 >> 4) & 0x0F0F0F0Fu);
          }
          // block j = bytes 32j .. 32j+31 of the 128-byte row: chunks 2j, 2j+1
          *reinterpret_cast<uint4*>(wt + sw128_off(crow, 2 * j)) = c0;
          *reinterpret_cast<uint4*>(wt + sw128_off(crow, 2 * j + 1)) = c1;
          wsc[j * TN + crow] = d;
          if constexpr (T::kHasMin) wsc[KSUB * TN + j * TN + crow] = mn;
        }
      }
      }

      // generic-proxy writes -> tensor-core reads, and generic reads of the
      // TMA-refilled raw stage before its release
      fence_proxy_async_smem();
      __syncwarp();
      if (sub == 1 && lane == 0) mbar_arrive(&raw_empty[rs]);  // both stages of the raw box are read
      if (lane == 0) mbar_arrive(&w_full[ws]);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int ew = warp - kWarpEpi;          // 0..15
    const int quarter = warp & 3;            // TMEM lane quarter this warp may access
    const int cg = ew >> 2;                  // column group of kEpiCols
    const int row = quarter * 32 + lane;     // token row in the tile
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    // fp32 accumulators as packed pairs. TMEM is read in chunks of kChunk
    // columns, one chunk ahead: the load of the next chunk (of this block, or
    // the first chunk of the next block) is in flight while the current
    // chunk's math runs; a buffer goes back to the MMA as soon as all its
    // chunks are in registers. Eight warps of 64 columns each (not sixteen of
    // 32): the math needs ~170 registers per thread without moves, and fewer
    // warps have to release every buffer before the MMA can refill it.
    constexpr int NP = kEpiCols / 2;
    uint64_t acc[NP];
    uint32_t vbuf[2][kChunk];
    // Stage es (counted over all tiles) fills TMEM buffer j with its block j,
    // so buffer j's phase parity at stage es is es & 1 (NBUF == KSUB).
    const uint32_t tm_row = tmem_base + lane_addr + (uint32_t)(cg * kEpiCols);
    if (total > 0) {
      mbar_wait_idle_or_poison(&tm_full[0], 0, p.err, DEV_TIMEOUT_FULL, dead);
      tc_fence_after();
      tmem_ldh(tm_row, vbuf[0]);
      tmem_ld_wait();
    }
    int es = 0;
    for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x) {
#pragma unroll
      for (int c = 0; c < NP; ++c) acc[c] = 0ull;
      const bool last_tile = t + (int)gridDim.x >= p.num_tiles;
      for (int s = 0; s < spt; ++s, ++es) {
        const int as = es % SA, ws = es % SWS;  // compile-time powers of two
        const uint32_t par = (uint32_t)es & 1u;
        mbar_wait_idle_or_poison(&act_full[as], (es / SA) & 1, p.err, DEV_TIMEOUT_FULL, dead);
        mbar_wait_idle_or_poison(&w_full[ws], (es / SWS) & 1, p.err, DEV_TIMEOUT_FULL, dead);
        const float2* dsp = reinterpret_cast<const float2*>(smem + T::OFF_ASC + as * T::ASC_STAGE) + row * KSUB;
        const float* wsc = reinterpret_cast<const float*>(smem + T::OFF_WSC + ws * T::WSC_STAGE);
        const bool last_stage = last_tile && s == spt - 1;
#pragma unroll 1
        for (int j = 0; j < KSUB; ++j) {
          const float2 dsj = dsp[j];
          const float dx = dsj.x, dy = dsj.y;
          const float d = round22(dx);
          const uint64_t d2 = pk2(d, d);
          const uint64_t c2 = pk2(-kBiasF * d, -kBiasF * d);
          const uint64_t ms8 = pk2(-8.0f * dy, -8.0f * dy);
          const uint64_t sy2 = pk2(dy, dy);
          const ulonglong2* dw = reinterpret_cast<const ulonglong2*>(wsc + j * TN + cg * kEpiCols);
          const ulonglong2* mw = reinterpret_cast<const ulonglong2*>(wsc + KSUB * TN + j * TN + cg * kEpiCols);
#pragma unroll
          for (int h = 0; h < kChunks; ++h) {
            uint32_t(&cur)[kChunk] = vbuf[h & 1];
            uint32_t(&nxt)[kChunk] = vbuf[(h + 1) & 1];
            if (h + 1 < kChunks) {
              tmem_ldh(tm_row + (uint32_t)(j * TN + kChunk * (h + 1)), nxt);
            } else if (!(last_stage && j == KSUB - 1)) {
              // the next block's first chunk (buffer j + 1 of this stage, or 0 of the next)
              const int jn = (j + 1) & (KSUB - 1);
              const uint32_t pn = j == KSUB - 1 ? (par ^ 1u) : par;
              mbar_wait_idle_or_poison(&tm_full[jn], pn, p.err, DEV_TIMEOUT_FULL, dead);
              tc_fence_after();
              tmem_ldh(tm_row + (uint32_t)(jn * TN), nxt);
            }
#pragma unroll
            for (int q = 0; q < kChunk / 4; ++q) {  // 4 columns per step
              const ulonglong2 w4 = dw[(kChunk / 4) * h + q];
              const int c = (kChunk / 2) * h + 2 * q;  // pair index
              uint64_t u0 = fma2(pk2u(cur[4 * q], cur[4 * q + 1]), d2, c2);  // d_a * sumi (exact)
              uint64_t u1 = fma2(pk2u(cur[4 * q + 2], cur[4 * q + 3]), d2, c2);
              if constexpr (WT == KQ_Q4_0) {
                u0 = add2(u0, ms8);  // d_a sumi - 8 s_a
                u1 = add2(u1, ms8);
              }
              acc[c] = fma2(u0, w4.x, acc[c]);
              acc[c + 1] = fma2(u1, w4.y, acc[c + 1]);
              if constexpr (WT == KQ_Q4_1) {
                const ulonglong2 m4 = mw[(kChunk / 4) * h + q];
                acc[c] = fma2(m4.x, sy2, acc[c]);  // + m_w s_a
                acc[c + 1] = fma2(m4.y, sy2, acc[c + 1]);
              }
            }
            tmem_ld_wait();
            if (h == kChunks - 2) {
              // every chunk of block j is in registers: hand buffer j back
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(&tm_empty[j]);
            }
          }
        }
        fence_proxy_async_smem();  // generic reads of the TMA-refilled scale stage, before its release
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&act_empty[as]);
          mbar_arrive(&w_empty[ws]);
        }
      }
      // ---- store this tile's rows ----
      {
        const int m0 = (t % p.num_m_tiles) * TM, n0 = (t / p.num_m_tiles) * TN;
        const int m = m0 + row;
        const int nc0 = n0 + cg * kEpiCols;
        if (m < p.M) {
          if constexpr (!SCATTER) {
            float* o = p.out.ptr[0] + (size_t)m * p.N + nc0;
            // float4 stores only when every row start is 16-byte aligned
            // (an offset output view falls back to scalar stores)
            if (nc0 + kEpiCols <= p.N && (p.N & 3) == 0 && (reinterpret_cast<uintptr_t>(p.out.ptr[0]) & 15) == 0) {
#pragma unroll
              for (int c = 0; c < NP; c += 2) {
                const float2 a = upk2(acc[c]), b = upk2(acc[c + 1]);
                *reinterpret_cast<float4*>(o + 2 * c) = make_float4(a.x, a.y, b.x, b.y);
              }
            } else {
#pragma unroll
              for (int c = 0; c < NP; ++c) {
                const float2 a = upk2(acc[c]);
                if (nc0 + 2 * c < p.N) o[2 * c] = a.x;
                if (nc0 + 2 * c + 1 < p.N) o[2 * c + 1] = a.y;
              }
            }
          } else {
            const size_t off = (size_t)m * p.out.ld + p.out.col0 + nc0;
            const bool vec = nc0 + kEpiCols <= p.N && ((p.out.ld | p.out.col0) & 3) == 0;
            for (int dd = 0; dd < p.out.n_out; ++dd) {
              float* o = p.out.ptr[dd] + off;
              if (vec) {
#pragma unroll
                for (int c = 0; c < NP; c += 2) {
                  const float2 a = upk2(acc[c]), b = upk2(acc[c + 1]);
                  *reinterpret_cast<float4*>(o + 2 * c) = make_float4(a.x, a.y, b.x, b.y);
                }
              } else {
#pragma unroll
                for (int c = 0; c < NP; ++c) {
                  const float2 a = upk2(acc[c]);
                  if (nc0 + 2 * c < p.N) o[2 * c] = a.x;
                  if (nc0 + 2 * c + 1 < p.N) o[2 * c + 1] = a.y;
                }
              }
            }
          }
        }
      }
    }
    if constexpr (SCATTER) __threadfence_system();  // peer stores visible before the host-side barrier
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kWarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ---- host side -----------------------------------------------------------------

template <int WT>
kq_status_t launch_tc(const void* w, Act8 act, const OutSpec& out, int M, int N, int K, bool pdl, cudaStream_t s,
                      int* err) {
  using T = TcTraits<WT>;
  const int nb = K / 32;
  CUtensorMap m_act, m_asc, m_raw;
  if (!encode_map(&m_act, CU_TENSOR_MAP_DATA_TYPE_UINT8, act.qs, (uint64_t)K, (uint64_t)M, (uint64_t)K, 128, TM,
                  CU_TENSOR_MAP_SWIZZLE_128B))
    return fail(KQ_ERR_CUDA, "tensor map (activation codes) rejected");
  if (!encode_map(&m_asc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, act.ds, (uint64_t)nb * 2, (uint64_t)M, (uint64_t)nb * 8,
                  KSUB * 2, TM, CU_TENSOR_MAP_SWIZZLE_NONE))
    return fail(KQ_ERR_CUDA, "tensor map (activation scales) rejected");
  const uint64_t rowbytes = (uint64_t)nb * T::BB;
  if (!encode_map(&m_raw, CU_TENSOR_MAP_DATA_TYPE_UINT16, w, rowbytes / 2, (uint64_t)N, rowbytes, T::RAW_ROW / 2, TN,
                  CU_TENSOR_MAP_SWIZZLE_NONE))
    return fail(KQ_ERR_CUDA, "tensor map (weights) rejected");

  const bool scatter = out.n_out > 1 || out.ld != N || out.col0 != 0;
  auto kern = scatter ? gemm_tc_kernel<WT, true> : gemm_tc_kernel<WT, false>;
  if (kq_status_t st = ensure_dynamic_smem(reinterpret_cast<const void*>(kern), T::SMEM, "gemm_tc smem attribute"))
    return st;
  TcParams p;
  p.M = M; p.N = N; p.K = K; p.nb = nb;
  p.num_m_tiles = (M + TM - 1) / TM;
  p.num_tiles = p.num_m_tiles * ((N + TN - 1) / TN);
  p.out = out;
  p.err = err ? err : device_error_word();
  const int grid = std::max(1, std::min(sm_count(), p.num_tiles));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = T::SMEM;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, m_act, m_asc, m_raw, p);
  if (e != cudaSuccess) return check_cuda(e, "gemm_tc launch");
  return check_launch("gemm_tc");
}

}  // namespace

bool gemm_tc_supported(int wtype, int M, int N, int K, const void* w, Act8 act) {
  (void)wtype;
  const int nb = K / 32;
  return M > 8 && N >= 1 && K >= 256 && nb % KRAW == 0 && (reinterpret_cast<uintptr_t>(w) & 15) == 0 &&
         (reinterpret_cast<uintptr_t>(act.qs) & 15) == 0 && (reinterpret_cast<uintptr_t>(act.ds) & 15) == 0;
}

kq_status_t launch_gemm_tc(int wtype, const void* w, Act8 act, float* out, int M, int N, int K, bool pdl,
                           cudaStream_t s, int* err) {
  return launch_gemm_tc(wtype, w, act, OutSpec::plain(out, N), M, N, K, pdl, s, err);
}

kq_status_t launch_gemm_tc(int wtype, const void* w, Act8 act, const OutSpec& out, int M, int N, int K, bool pdl,
                           cudaStream_t s, int* err) {
  switch (wtype) {
    case KQ_Q4_0: return launch_tc<KQ_Q4_0>(w, act, out, M, N, K, pdl, s, err);
    case KQ_Q4_1: return launch_tc<KQ_Q4_1>(w, act, out, M, N, K, pdl, s, err);
    case KQ_Q8_0: return launch_tc<KQ_Q8_0>(w, act, out, M, N, K, pdl, s, err);
    default: return fail(KQ_ERR_INVALID, "unknown weight type %d", wtype);
  }
}

}  // namespace kq
