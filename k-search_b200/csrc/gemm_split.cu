// Tensor-core quantised GEMM for M > 8 activation rows in exact split-fp16
// form: the reference's per-block integer formulas (gemm_ref.py:100-153
// q4_0, :274-331 q4_1; include/gemm_reference.h:311-336 q8_0) evaluated as
// fp16 tensor-core products whose operands carry every bit of the
// dequantised values.
//
// Both operands are dequantised and split into a high fp16 part and a
// low fp16 part scaled by 2^11 (so it never falls into fp16 subnormals):
//   a = q_a * d_a * 2^-e_m          (per activation row, e_m puts the row's
//                                     largest |a| in [2^14, 2^15))
//   A_hi = fp16(a),  A_lo = fp16((a - A_hi) * 2^11)         exact: a has 19 bits
//   W    = (q_w - 8) d_w  (q4_0),  q_w d_w + m_w  (q4_1),  q_w d_w  (q8_0)
//   W_hi = fp16(W),  W_lo = fp16((W - W_hi) * 2^11)          exact for q4_0 / q8_0
// and tcgen05.mma.kind::f16 accumulates in fp32 TMEM, per weight row n and
// token m:
//   main = sum_k W_hi A_hi (+ the extra columns below)
//   corr = sum_k W_hi A_lo + W_lo A_hi
//   out[m, n] = 2^e_m (main + 2^-11 corr)
// The dropped W_lo A_lo term is 2^-22 of the products, so the result equals
// the exact per-block sum up to fp32 accumulation order. For q4_0 / q4_1 the
// difference between the plain product and the reference's formulas (its
// stored block sum s_a instead of d_a sum q_a) rides in extra K columns:
//   X_a = (s_a - d_a sum_i q_a) 2^-e_m,  X_w = -8 d_w (q4_0) | m_w (q4_1).
//
// Why this form: an int8 kind::i8 pipeline has to rescale a fresh int32 tile
// per 32-wide K block on the FP32 pipe (at least two FMAs per element and
// block); a single fp16 rounding of each operand is 2x faster but leaves a
// relative error of ~3e-4 per element, outside the parity bar.
//
// Operand placement: shared-memory bandwidth, not the tensor pipe, limits a
// split GEMM whose operands all live in shared memory (every MMA re-reads
// both operands there, and the converted weights are written there first).
// Here the weights are the MMA's A operand and live in TMEM: converter
// threads write W_hi / W_lo straight from registers with tcgen05.st, so they
// never touch shared memory. The activations are the B operand (TMA into
// 128B-swizzled shared memory, A_hi and A_lo tiles adjacent), so per 16-wide
// K step two MMAs cover all three products:
//   D[:, 0:256]   (+)= W_hi x [A_hi; A_lo]^T    main | first corr term
//   D[:, 128:256]  += W_lo x A_hi^T             second corr term
//
// CTA: 128 weight rows (TMEM lanes, MMA M) x 128 tokens per tile, one
// persistent CTA per SM; each CTA runs an equal share of all tiles' K groups
// (stream-K, see for_items), so a tile can be split between CTAs and summed
// by its owner from the others' partials. Warps (each loop runs on the whole
// warp; lane 0 issues):
//   0       activation producer: A_hi + A_lo chunks (128 tokens x 64 K each)
//   1       raw weight producer: unchanged AoS q-blocks, 128 rows x 8 blocks
//   2       MMA issuer, owns the TMEM allocation
//   3..10   converters: warp w serves the TMEM lane quarter w % 4 (32 weight
//           rows) and one 32-block of each 64-wide K chunk
//   11..18  epilogue: TMEM -> registers -> global fp32, two warps per lane
//           quarter (64 tokens each)
// TMEM: D = 256 columns (main 0..127, corr 128..255); four weight stages of
// 64 columns (W_hi 32 | W_lo 32) behind it.
#include <cuda_fp16.h>

#include <algorithm>

#include "kq_internal.h"
#include "kq_device.cuh"
#include "kq_tc.cuh"

namespace kq {
namespace {

using namespace tc;

constexpr int TW = 128;                  // weight rows per tile (TMEM lanes, MMA M)
constexpr int TT = 128;                  // tokens per tile
constexpr int CK = 64;                   // K elements per chunk: one 128-byte swizzle atom of fp16
constexpr int RB = 8;                    // blocks per raw weight stage (= 4 chunks)
constexpr int GRP = 32;                  // main chunks per extra chunk (64 blocks)
constexpr int UNIT = 4;                  // chunks per schedule unit (one raw weight stage)
constexpr int SS = 4;                    // chunk stages: activations (shared memory) + weights (TMEM), paired
constexpr int A_PART = TT * 128;         // one 128-token x 128-byte tile
constexpr int A_STAGE = 2 * A_PART;
constexpr int kSmemLimit = 232448;

constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColD = 0;            // main 0..127, corr 128..255
constexpr uint32_t kColW = 2 * TT;       // weight stage s at kColW + 64 s: W_hi 32 | W_lo 32
constexpr int kWarpA = 0, kWarpRaw = 1, kWarpMma = 2, kWarpConv = 3, kConvWarps = 8, kWarpEpi = 11;
constexpr int kEpiWarps = 8;             // two per TMEM lane quarter
constexpr int kEpiTok = TT / 2;          // tokens per epilogue warp
constexpr int kWarps = kWarpEpi + kEpiWarps;
constexpr int kThreads = kWarps * 32;

template <int WT>
struct SxTraits {
  static constexpr int BB = WT == KQ_Q4_0 ? 18 : WT == KQ_Q4_1 ? 20 : 34;
  static constexpr bool kExtra = WT != KQ_Q8_0;
  static constexpr int RAW_ROW = RB * BB;  // 144 / 160 / 272 bytes
  static constexpr int RAW_STAGE = TW * RAW_ROW;
  static constexpr int X_BYTES = kExtra ? TW * 128 : 0;   // X_w tile (converters)
  static constexpr int XA_BYTES = kExtra ? A_PART : 0;    // X_a tile of the activations (TMA)
  // 32-bit words a converter reads for one block: from the 4-byte boundary at
  // or below the block start (blocks are 2-byte aligned) to its end
  static constexpr int NW = WT == KQ_Q4_1 ? 5 : (BB + 2 + 3) / 4;
  // 16-byte loads per block window (from the 16-byte boundary at or below the
  // block start): the block's words start at word ((start & 15) >> 2) < 4
  static constexpr int NV = (3 + NW + 3) / 4;
  // two raw stages keep a weight box in flight while the other is converted
  static constexpr int SR = 2;
  static constexpr int OFF_A = 0;
  static constexpr int OFF_X = OFF_A + SS * A_STAGE;
  static constexpr int OFF_XA = OFF_X + X_BYTES;
  static constexpr int OFF_RAW = OFF_XA + XA_BYTES;
  static constexpr int OFF_BAR = OFF_RAW + SR * RAW_STAGE;
  static constexpr int NBARS = 2 * SS + 2 * SR + 2 + 2;
  static constexpr int OFF_TMEM = OFF_BAR + NBARS * 8;
  static constexpr int SMEM = OFF_TMEM + 16 + 1024;
  static_assert(RAW_ROW % 16 == 0 && RAW_STAGE % 16 == 0, "raw stages stay 16-byte aligned");
  static_assert(OFF_RAW % 1024 == 0, "swizzled tiles stay 1024-byte aligned");
  static_assert(SMEM <= kSmemLimit, "shared memory budget");
  static_assert(kColW + 64 * SS <= kTmemCols, "TMEM budget");
};

// D (+)= A x B^T, A from shared memory (descriptor)
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}

// D (+)= A x B^T, A from TMEM (lane = row, two fp16 per 32-bit column)
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}

// Instruction descriptor, kind::f16: D f32, A = B = f16, both K-major, M = 128.
template <int N>
__host__ __device__ constexpr uint32_t idesc_f16() {
  static_assert(N % 16 == 0 && N >= 16 && N <= 256, "MMA N");
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(TW >> 4) << 24);
}

// 16 consecutive 32-bit TMEM columns of this thread's lane <- v
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
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

// Bounded spin on the non-suspending probe (the hand-offs in this kernel
// complete within a few hundred cycles; a suspended wait resumes later).
// Gives up after kWaitLimitNs, records `code` and poisons the caller.
__device__ __forceinline__ void spin_wait(uint64_t* bar, uint32_t parity, int* err, int code, bool& dead) {
  if (dead) return;
  const uint64_t t0 = globaltimer_ns();
#pragma unroll 1
  for (uint32_t i = 1;; ++i) {
    if (mbar_test_wait(bar, parity)) return;
    if ((i & 1023u) == 0 && globaltimer_ns() - t0 > kWaitLimitNs) {
      record_error(err, code);
      dead = true;
      return;
    }
  }
}

// Bounded wait on the suspending probe, for waits that usually last long
// (a role idle until a whole tile or stage ring has moved on): the warp
// yields its issue slots to the warps doing the work instead of spinning.
__device__ __forceinline__ void sleep_wait(uint64_t* bar, uint32_t parity, int* err, int code, bool& dead) {
  if (dead) return;
  const uint64_t t0 = globaltimer_ns();
#pragma unroll 1
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return;
    if ((i & 63u) == 0 && globaltimer_ns() - t0 > kWaitLimitNs) {
      record_error(err, code);
      dead = true;
      return;
    }
  }
}

// One weight block -> 16 packed fp16 pairs of W_hi and of W_lo (element pairs
// 2i, 2i+1 in K order) and the block's X_w. `w` holds the block's bytes from
// the 4-byte boundary at or below its start; `sh` = 8 * (start & 3).
//
// W_lo exactness for q4_0 / q8_0: c and d are fp16 (c an integer of at most 8
// bits), so c*d is a multiple of d's unit in the last place and so is
// r = c*d - fp16(c*d); |r| is at most half an ulp of fp16(c*d), hence r is an
// fp16 value (normal or subnormal) and the fma below returns it exactly.
// Scaling by -2^11 is exact (|r| * 2^11 <= 2^15).
template <int WT, int NW>
__device__ __forceinline__ void convert_block(const uint32_t (&w)[NW], uint32_t sh, uint32_t (&hi)[16],
                                              uint32_t (&lo)[16], uint16_t& xw) {
  constexpr uint32_t kNeg2048 = 0xE800E800u;  // (-2048, -2048)
  const uint32_t dh = __funnelshift_r(w[0], w[1], sh) & 0xFFFFu;
  const uint32_t d2 = dh | (dh << 16);
  if constexpr (WT == KQ_Q8_0) {
    const uint32_t nd2 = d2 ^ 0x80008000u;
    constexpr uint32_t kOff = 0x64806480u;  // (1152, 1152): M + (c ^ 0x80) - 1152 = c
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const uint32_t cw = __funnelshift_rc(w[k], w[k + 1], sh + 16) ^ 0x80808080u;
      const uint32_t c01 = hsub2(__byte_perm(cw, 0x64646464u, 0x4140), kOff);
      const uint32_t c23 = hsub2(__byte_perm(cw, 0x64646464u, 0x4342), kOff);
      const uint32_t h01 = hmul2(c01, d2), h23 = hmul2(c23, d2);
      hi[2 * k] = h01;
      hi[2 * k + 1] = h23;
      lo[2 * k] = hmul2(hfma2(c01, nd2, h01), kNeg2048);      // (h - c d) * -2^11 = r * 2^11
      lo[2 * k + 1] = hmul2(hfma2(c23, nd2, h23), kNeg2048);
    }
    xw = 0;
  } else if constexpr (WT == KQ_Q4_0) {
    const uint32_t nd2 = d2 ^ 0x80008000u;
    constexpr uint32_t k1032 = 0x64086408u;  // (1032, 1032): M + c - 1032 = c - 8
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t cw = __funnelshift_rc(w[k], w[k + 1], sh + 16);
      const uint32_t lw = cw & 0x0F0F0F0Fu, hw = (cw >> 4) & 0x0F0F0F0Fu;
      uint32_t c[4];
      c[0] = hsub2(__byte_perm(lw, 0x64646464u, 0x4140), k1032);  // elements 4k, 4k+1
      c[1] = hsub2(__byte_perm(lw, 0x64646464u, 0x4342), k1032);  // 4k+2, 4k+3
      c[2] = hsub2(__byte_perm(hw, 0x64646464u, 0x4140), k1032);  // 16+4k, 16+4k+1
      c[3] = hsub2(__byte_perm(hw, 0x64646464u, 0x4342), k1032);
      const int idx[4] = {2 * k, 2 * k + 1, 8 + 2 * k, 8 + 2 * k + 1};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t h = hmul2(c[i], d2);
        hi[idx[i]] = h;
        lo[idx[i]] = hmul2(hfma2(c[i], nd2, h), kNeg2048);
      }
    }
    xw = (uint16_t)(hmul2(dh, 0xC800u) & 0xFFFFu);  // -8 d (exact)
  } else {
    // q4_1: W = c d + m (one rounding for W_hi); the residual in fp32, where
    // c d + m is exact whenever it fits 24 bits
    const uint32_t mh = w[0] >> 16;
    const uint32_t m2 = mh | (mh << 16);
    const float df = __half2float(__ushort_as_half((uint16_t)dh));
    const float mf = __half2float(__ushort_as_half((uint16_t)mh));
    constexpr uint32_t k1024 = 0x64006400u;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t cw = w[k + 1];
      const uint32_t lw = cw & 0x0F0F0F0Fu, hw = (cw >> 4) & 0x0F0F0F0Fu;
      uint32_t c[4];
      c[0] = hsub2(__byte_perm(lw, 0x64646464u, 0x4140), k1024);
      c[1] = hsub2(__byte_perm(lw, 0x64646464u, 0x4342), k1024);
      c[2] = hsub2(__byte_perm(hw, 0x64646464u, 0x4140), k1024);
      c[3] = hsub2(__byte_perm(hw, 0x64646464u, 0x4342), k1024);
      const int idx[4] = {2 * k, 2 * k + 1, 8 + 2 * k, 8 + 2 * k + 1};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t h = hfma2(c[i], d2, m2);
        hi[idx[i]] = h;
        const float2 cf = __half22float2(*reinterpret_cast<const __half2*>(&c[i]));
        const float2 hf = __half22float2(*reinterpret_cast<const __half2*>(&h));
        const __half2 l = __floats2half2_rn((fmaf(cf.x, df, mf) - hf.x) * 2048.0f, (fmaf(cf.y, df, mf) - hf.y) * 2048.0f);
        lo[idx[i]] = *reinterpret_cast<const uint32_t*>(&l);
      }
    }
    xw = (uint16_t)mh;
  }
}

struct SxParams {
  int M, N, K;
  int nmain, ngrp;
  int num_t_tiles, num_tiles;
  int upt, num_units;   // K units (UNIT chunks each) per tile, units in all
  OutSpec out;
  const float* rscale;  // per activation row: 2^e undoing the prep kernel's scaling
  int* flags;           // per CTA: epilogue warps done writing its partial tile (zeroed by the prep kernel)
  float* partial;       // per CTA: [TT tokens][TW rows] partial sums of the tile it starts inside
  int* err;
};

// Work schedule (stream-K): every tile's K range is cut into units of UNIT
// chunks; CTA b takes units [U b / G, U (b + 1) / G) in order, so the SMs
// get equal work whatever the tile count. A work item is the part of one
// tile inside a CTA's range. The CTA holding a tile's first unit owns the
// tile; the others (whose ranges start inside it: each CTA at most once, on
// its first item) write partial sums that the owner adds, in CTA order,
// after its own part. The extra columns follow the same split: a CTA applies
// them for the blocks it converted, at the end of each group segment of an
// item (its X tile holds zero for the group's other blocks).
__device__ __forceinline__ int unit_begin(const SxParams& p, int b) {
  return (int)(((long long)p.num_units * b) / (long long)gridDim.x);
}
struct Item {
  int t, c0, c1;  // tile, chunk range [c0, c1)
};
// Calls f(item) for each work item of this CTA, in order.
template <typename F>
__device__ __forceinline__ void for_items(const SxParams& p, F&& f) {
  const int ue = unit_begin(p, blockIdx.x + 1);
  for (int u = unit_begin(p, blockIdx.x); u < ue;) {
    const int t = u / p.upt;
    const int uend = min(ue, (t + 1) * p.upt);
    f(Item{t, (u - t * p.upt) * UNIT, min((uend - t * p.upt) * UNIT, p.nmain)});
    u = uend;
  }
}

// main chunk c of an item ending at chunk c1 is followed by an extra chunk:
// the last chunk of its group of GRP, or of the item
__device__ __forceinline__ bool x_after(int c, int c1) { return (c % GRP) == GRP - 1 || c == c1 - 1; }

template <int WT, bool SCATTER>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_split_kernel(const __grid_constant__ CUtensorMap map_hi, const __grid_constant__ CUtensorMap map_lo,
                      const __grid_constant__ CUtensorMap map_raw, const __grid_constant__ SxParams p) {
  using T = SxTraits<WT>;
  constexpr int SR = T::SR;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + T::OFF_BAR);
  // chunk stage s: full[s] completes when the activation tiles have landed
  // (TMA bytes) and every converter warp has written the weight stage;
  // empty[s] when the MMAs that read both are done (one commit)
  uint64_t* full = bars;
  uint64_t* empty = full + SS;
  uint64_t* raw_full = empty + SS;
  uint64_t* raw_empty = raw_full + SR;
  uint64_t* d_full = raw_empty + SR;
  uint64_t* d_empty = d_full + 1;
  uint64_t* x_empty = d_empty + 1;   // the X MMA of a group segment is done (X_w and X_a tiles free)
  uint64_t* xa_full = x_empty + 1;   // the X_a tile has landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + T::OFF_TMEM);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < SS; ++i) {
      mbar_init(&full[i], kConvWarps + 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < SR; ++i) {
      mbar_init(&raw_full[i], 1);
      mbar_init(&raw_empty[i], kConvWarps);
    }
    mbar_init(d_full, 1);
    mbar_init(d_empty, kEpiWarps);
    mbar_init(x_empty, 1);
    mbar_init(xa_full, 1);
    fence_mbar_init();
  }
  if constexpr (T::kExtra) {
    // the X tile starts zeroed: columns past the last block stay finite (x 0 in A_hi)
    for (int i = threadIdx.x; i < T::X_BYTES / 16; i += kThreads)
      reinterpret_cast<uint4*>(smem + T::OFF_X)[i] = make_uint4(0, 0, 0, 0);
    fence_proxy_async_smem();
  }
  if (warp == kWarpMma) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  bool dead = false;
  if (warp == kWarpA) {
    // ------------------------------------------------------------ activation producer
    if (lane == 0) {
      prefetch_tmap(&map_hi);
      prefetch_tmap(&map_lo);
      pdl_wait();  // A_hi / A_lo come from the preceding prep kernel
    }
    __syncwarp();
    int k = 0, gxa = 0;
    for_items(p, [&](const Item& w) {
      const int m0 = (w.t % p.num_t_tiles) * TT;
      for (int c = w.c0; c < w.c1; ++c, ++k) {
        const int st = k % SS;
        if (k >= SS) spin_wait(&empty[st], ((k / SS) - 1) & 1, p.err, DEV_TIMEOUT_EMPTY, dead);
        if (lane == 0) {
          uint8_t* dst = smem + T::OFF_A + st * A_STAGE;
          mbar_arrive_expect_tx(&full[st], A_STAGE);
          tma_load_2d(dst, &map_hi, c * CK, m0, &full[st]);
          tma_load_2d(dst + A_PART, &map_lo, c * CK, m0, &full[st]);
        }
        __syncwarp();
        if (T::kExtra && x_after(c, w.c1)) {  // the group's X_a columns, once the previous X MMA is done
          if (gxa >= 1) spin_wait(x_empty, (gxa - 1) & 1, p.err, DEV_TIMEOUT_EMPTY, dead);
          if (lane == 0) {
            mbar_arrive_expect_tx(xa_full, A_PART);
            tma_load_2d(smem + T::OFF_XA, &map_hi, p.K + (c / GRP) * CK, m0, xa_full);
          }
          __syncwarp();
          ++gxa;
        }
      }
    });
  } else if (warp == kWarpRaw) {
    // ------------------------------------------------------------ raw weight producer
    if (lane == 0) prefetch_tmap(&map_raw);
    __syncwarp();
    int ir = 0;
    for_items(p, [&](const Item& w) {
      const int n0 = (w.t / p.num_t_tiles) * TW;
      for (int r = w.c0 / 4; r < w.c1 / 4; ++r, ++ir) {
        const int rs = ir % SR;
        if (ir >= SR) spin_wait(&raw_empty[rs], ((ir / SR) - 1) & 1, p.err, DEV_TIMEOUT_EMPTY, dead);
        if (lane == 0) {
          mbar_arrive_expect_tx(&raw_full[rs], T::RAW_STAGE);
          tma_load_2d(smem + T::OFF_RAW + rs * T::RAW_STAGE, &map_raw, r * (T::RAW_ROW / 2), n0, &raw_full[rs]);
        }
        __syncwarp();
      }
    });
  } else if (warp == kWarpMma) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc2 = idesc_f16<2 * TT>();  // B = [A_hi; A_lo]: 256 rows, adjacent in the stage
    constexpr uint32_t idesc1 = idesc_f16<TT>();
    const uint32_t a_base = smem_u32(smem + T::OFF_A);
    const uint32_t x_base = smem_u32(smem + T::OFF_X);
    const uint32_t xa_base = smem_u32(smem + T::OFF_XA);
    const uint32_t d_main = tmem_base + kColD, d_corr = tmem_base + kColD + TT;
    int k = 0, gx = 0, it = 0;
    for_items(p, [&](const Item& w) {
      if (it >= 1) spin_wait(d_empty, (it - 1) & 1, p.err, DEV_TIMEOUT_EMPTY, dead);
      tc_fence_after();
      for (int c = w.c0; c < w.c1; ++c, ++k) {
        const int st = k % SS;
        spin_wait(&full[st], (k / SS) & 1, p.err, DEV_TIMEOUT_FULL, dead);
        tc_fence_after();
        if (lane == 0) {
          const uint64_t bdesc = sw128_desc(a_base + st * A_STAGE);  // A_hi rows, then A_lo rows
          const uint32_t whi = tmem_base + kColW + 64 * st, wlo = whi + 32;
#pragma unroll
          for (int j = 0; j < CK / 16; ++j) {
            mma_ts(d_main, whi + 8 * j, bdesc + (uint64_t)(2 * j), idesc2, (c > w.c0 || j > 0) ? 1u : 0u);
            mma_ts(d_corr, wlo + 8 * j, bdesc + (uint64_t)(2 * j), idesc1, 1u);
          }
          mma_commit(&empty[st]);
        }
        __syncwarp();
        if (T::kExtra && x_after(c, w.c1)) {
          // the segment's X_w columns are complete: every converter arrived on
          // full[] for the segment's chunks after writing them
          spin_wait(xa_full, gx & 1, p.err, DEV_TIMEOUT_FULL, dead);
          tc_fence_after();
          if (lane == 0) {
            const uint64_t xd = sw128_desc(x_base);
            const uint64_t bx = sw128_desc(xa_base);
#pragma unroll
            for (int j = 0; j < CK / 16; ++j)
              mma_ss(d_main, xd + (uint64_t)(2 * j), bx + (uint64_t)(2 * j), idesc1, 1u);
            mma_commit(x_empty);
          }
          __syncwarp();
          ++gx;
        }
      }
      if (lane == 0) mma_commit(d_full);
      __syncwarp();
      ++it;
    });
  } else if (warp < kWarpEpi) {
    // ------------------------------------------------------------ converters
    const int cw = warp - kWarpConv;                 // 0..7
    const int quarter = warp & 3;                    // TMEM lane quarter this warp may access
    const int row = quarter * 32 + lane;             // weight row within the tile
    const int b = cw >> 2;                           // which 32-block of each 64-wide chunk
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    const int offx = (row >> 3) * 1024 + (row & 7) * 128;  // X tile row (128B-swizzled, K-major)
    const uint32_t sh = (uint32_t)((b * T::BB) & 3) * 8;  // 16 * b for q4_0 / q8_0, 0 for q4_1
    int ir = 0, gc = 0, gx = 0;
    for_items(p, [&](const Item& wi) {
      for (int r = wi.c0 / 4; r < wi.c1 / 4; ++r, ++ir) {
        const int rs = ir % SR;
        spin_wait(&raw_full[rs], (ir / SR) & 1, p.err, DEV_TIMEOUT_FULL, dead);
        const uint8_t* src = smem + T::OFF_RAW + rs * T::RAW_STAGE + row * T::RAW_ROW;
#pragma unroll
        for (int j = 0; j < 4; ++j, ++gc) {
          const int c = 4 * r + j;  // chunk within the tile
          // this chunk's block: a 16-byte window load (rows are 16-byte
          // multiples apart, so eight consecutive rows read eight distinct
          // bank groups)
          uint32_t w[T::NW];
          {
            const int o = (2 * j + b) * T::BB;
            const uint4* s4 = reinterpret_cast<const uint4*>(src + (o & ~15));
            uint32_t win[4 * T::NV];
#pragma unroll
            for (int v = 0; v < T::NV; ++v) {
              const uint4 q = s4[v];
              win[4 * v] = q.x;
              win[4 * v + 1] = q.y;
              win[4 * v + 2] = q.z;
              win[4 * v + 3] = q.w;
            }
            const int wo0 = (((2 * j) * T::BB) & 15) >> 2;      // compile-time after unrolling
            const int wo1 = (((2 * j + 1) * T::BB) & 15) >> 2;
#pragma unroll
            for (int i = 0; i < T::NW; ++i) w[i] = b ? win[wo1 + i] : win[wo0 + i];
          }
          if (j == 3) {
            // the stage is refilled by TMA (async proxy): order these generic
            // reads before the release, or a late read can see the next stage
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&raw_empty[rs]);
          }
          uint32_t hi[16], lo[16];
          uint16_t xw;
          convert_block<WT, T::NW>(w, sh, hi, lo, xw);
          const int ws = gc % SS;
          if (gc >= SS) spin_wait(&empty[ws], ((gc / SS) - 1) & 1, p.err, DEV_TIMEOUT_EMPTY, dead);
          tc_fence_after();
          const uint32_t wcol = tmem_base + lane_addr + kColW + 64 * ws + 16 * b;
          tmem_st16(wcol, hi);
          tmem_st16(wcol + 32, lo);
          if constexpr (T::kExtra) {
            if (c % GRP == 0 || c == wi.c0) {
              // first chunk of a group segment: once the MMA is done with the X
              // tile, clear this thread's columns (those of parity b: the
              // blocks 2c + b it converts), so blocks of the group that other
              // CTAs convert count zero here
              if (gx >= 1) spin_wait(x_empty, (gx - 1) & 1, p.err, DEV_TIMEOUT_EMPTY, dead);
              ++gx;
#pragma unroll 4
              for (int z = b; z < 64; z += 2)
                *reinterpret_cast<uint16_t*>(smem + T::OFF_X + (offx + (((z >> 3) ^ (row & 7)) << 4)) + (z & 7) * 2) = 0;
            }
            const int col = (2 * c + b) & 63;
            *reinterpret_cast<uint16_t*>(smem + T::OFF_X + (offx + ((((col >> 3) ^ (row & 7))) << 4)) + (col & 7) * 2) =
                xw;
            fence_proxy_async_smem();  // generic-proxy write -> tensor-core read
          }
          tmem_st_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&full[ws]);
        }
      }
    });
  } else {
    // ------------------------------------------------------------ epilogue
    // two warps per TMEM lane quarter, one half of the tile's tokens each: a
    // warp pulls its 64 tokens of D into registers and releases D to the next
    // item's MMAs before any global traffic
    const int ew = warp - kWarpEpi;             // 0..7
    const int quarter = warp & 3;
    const int half = ew >> 2;
    const int row = quarter * 32 + lane;        // weight row within the tile
    const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + kColD + (uint32_t)(half * kEpiTok);
    pdl_wait();  // rscale and the zeroed flags come from the prep kernel
    int it = 0;
    for_items(p, [&](const Item& w) {
      sleep_wait(d_full, it & 1, p.err, DEV_TIMEOUT_FULL, dead);
      tc_fence_after();
      // main straight into the output registers, then corr 16 columns at a time
      uint32_t ov[kEpiTok / 16][16];
#pragma unroll
      for (int g = 0; g < kEpiTok / 16; ++g) tmem_ld16(taddr + 16 * g, ov[g]);
      tmem_ld_wait();
      float o[kEpiTok];
#pragma unroll
      for (int g = 0; g < kEpiTok / 16; ++g) {
        uint32_t u[16];
        tmem_ld16(taddr + TT + 16 * g, u);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; ++i) o[16 * g + i] = fmaf(__uint_as_float(u[i]), 1.0f / 2048.0f, __uint_as_float(ov[g][i]));
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(d_empty);
      ++it;

      const int m0 = (w.t % p.num_t_tiles) * TT + half * kEpiTok, n0 = (w.t / p.num_t_tiles) * TW;
      const int n = n0 + row;
      const int tokens = min(kEpiTok, p.M - m0);
      const int tbase = half * kEpiTok;           // token offset inside the tile
      // per-token row scales (powers of two): two per lane, broadcast by shuffle
      const int last = max(tokens - 1, 0);
      const float rs_a = tokens > 0 ? p.rscale[m0 + min(lane, last)] : 1.0f;
      const float rs_b = tokens > 0 ? p.rscale[m0 + min(32 + lane, last)] : 1.0f;
      const int tile_u0 = w.t * p.upt, tile_end = (w.t + 1) * p.upt;
      // A split tile with exactly two contributors skips the partial buffer:
      // the helper, which finishes its part early in its run, stores its
      // scaled sums into the output; the owner adds its own with
      // red.global.add after the helper's flag. The scale is a power of two,
      // so this equals scaling the two-term sum once.
      const bool pair_helper = !SCATTER && w.c0 > 0 && w.c1 == p.nmain && blockIdx.x >= 1 &&
                               unit_begin(p, (int)blockIdx.x - 1) <= tile_u0;
      auto signal = [&]() {  // this warp's rows are written
        __threadfence();
        __syncwarp();
        if (lane == 0) atomicAdd(p.flags + blockIdx.x, 1);
      };
      if (w.c0 > 0 && !pair_helper) {             // helper: partial sums for the tile's owner
        float* part = p.partial + (size_t)blockIdx.x * (TT * TW);
#pragma unroll
        for (int j = 0; j < kEpiTok; ++j) __stcg(part + (tbase + j) * TW + row, o[j]);
        signal();
        return;
      }
      bool pair_owner = false;
      if (w.c0 == 0 && w.c1 < p.nmain) {          // owner of a split tile
        int h_end = (int)blockIdx.x + 1;          // helpers: CTAs blockIdx.x + 1 .. h_end - 1
        while (h_end < (int)gridDim.x && unit_begin(p, h_end) < tile_end) ++h_end;
        pair_owner = !SCATTER && h_end == (int)blockIdx.x + 2;
        for (int k = (int)blockIdx.x + 1; k < h_end; ++k) {
          const uint64_t t0 = globaltimer_ns();
          for (uint32_t i = 1;; ++i) {  // written early in the helper's run: normally already complete
            uint32_t v;
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p.flags + k) : "memory");
            if (v >= (uint32_t)kEpiWarps || dead) break;
            if ((i & 255u) == 0 && globaltimer_ns() - t0 > kWaitLimitNs) {
              record_error(p.err, DEV_TIMEOUT_FULL);
              dead = true;
              break;
            }
          }
          if (!pair_owner) {
            const float* hp = p.partial + (size_t)k * (TT * TW);
#pragma unroll
            for (int j = 0; j < kEpiTok; ++j) o[j] += __ldcg(hp + (tbase + j) * TW + row);
          }
        }
      }
#pragma unroll
      for (int j = 0; j < kEpiTok; ++j) o[j] *= __shfl_sync(0xffffffffu, j < 32 ? rs_a : rs_b, j & 31);
      if (n < p.N) {
        const size_t ld = (size_t)p.out.ld;
        if (pair_owner) {
          float* dst = p.out.ptr[0] + (size_t)m0 * ld + p.out.col0 + n;
#pragma unroll
          for (int j = 0; j < kEpiTok; ++j)
            if (j < tokens) atomicAdd(dst + j * ld, o[j]);
        } else {
          const int nd = SCATTER ? p.out.n_out : 1;
#pragma unroll
          for (int dd = 0; dd < (SCATTER ? kMaxOut : 1); ++dd) {  // destinations outermost, static indices
            if (dd < nd) {
              float* dst = p.out.ptr[dd] + (size_t)m0 * ld + p.out.col0 + n;
#pragma unroll
              for (int j = 0; j < kEpiTok; ++j)
                if (j < tokens) dst[j * ld] = o[j];
            }
          }
        }
      }
      if (pair_helper) signal();
    });
    if constexpr (SCATTER) __threadfence_system();  // peer stores visible before the host-side barrier
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kWarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// A_hi[m, k] = fp16(a), A_lo[m, k] = fp16((a - A_hi) 2^11) with
// a = q * d * 2^-e_m from the staging layout, plus the extra columns of
// A_hi (scaled alike; zero past the last block); rscale[m] = 2^e_m. One CTA
// per activation row. The per-row power of two puts the row's largest
// magnitude in [2^14, 2^15), so nothing overflows fp16 and A_lo stays clear
// of fp16 subnormals except for elements below 2^-17 of the row maximum.
template <int WT>
__global__ void __launch_bounds__(128) split_act_kernel(Act8 act, int M, int K, int Kp, __half* __restrict__ a_hi,
                                                        __half* __restrict__ a_lo, float* __restrict__ rscale,
                                                        int* __restrict__ flags, int nflags) {
  pdl_launch_dependents();
  pdl_wait();  // the staged activations come from the preceding quantiser
  if (blockIdx.x == 0)  // the GEMM's partial-tile flags start at zero every call
    for (int i = threadIdx.x; i < nflags; i += blockDim.x) flags[i] = 0;
  const int nb = K / 32;
  const int m = blockIdx.x;
  if (m >= M) return;
  const float2* ds = act.ds + (size_t)m * nb;
  // block sum of the codes (the residual column's d sum q)
  auto code_sum = [&](int b) {
    const int4* src = reinterpret_cast<const int4*>(act.qs + (size_t)m * K + 32 * b);
    const int4 c01 = src[0], c23 = src[1];
    int q = 0;
    q = __dp4a(c01.x, 0x01010101, q); q = __dp4a(c01.y, 0x01010101, q);
    q = __dp4a(c01.z, 0x01010101, q); q = __dp4a(c01.w, 0x01010101, q);
    q = __dp4a(c23.x, 0x01010101, q); q = __dp4a(c23.y, 0x01010101, q);
    q = __dp4a(c23.z, 0x01010101, q); q = __dp4a(c23.w, 0x01010101, q);
    return q;
  };
  // largest magnitude of the row: |q d| <= 127 |d|, and the residual column
  // s - d sum q (usually below 32 |d|, but not when the stored fp16 d is a
  // coarse subnormal far from the d the codes were quantised with)
  float amax = 0.0f;
  for (int b = threadIdx.x; b < nb; b += blockDim.x) {
    const float2 v = ds[b];
    amax = fmaxf(amax, 127.0f * fabsf(v.x));
    if constexpr (WT != KQ_Q8_0) amax = fmaxf(amax, fabsf(v.y - v.x * (float)code_sum(b)));
  }
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
  __half* hrow = a_hi + (size_t)m * Kp;
  __half* lrow = a_lo + (size_t)m * K;
  for (int b = threadIdx.x; b < nb; b += blockDim.x) {
    const float2 v = ds[b];
    const float d = v.x * down;  // exact (power-of-two scaling)
    const int4* src = reinterpret_cast<const int4*>(act.qs + (size_t)m * K + 32 * b);
    const int4 c01 = src[0], c23 = src[1];
    const int cw[8] = {c01.x, c01.y, c01.z, c01.w, c23.x, c23.y, c23.z, c23.w};
    uint32_t hw[16], lw[16];
    int qsum = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
#pragma unroll
      for (int e2 = 0; e2 < 4; e2 += 2) {
        const int q0 = (int)(int8_t)((cw[i] >> (8 * e2)) & 0xFF);
        const int q1 = (int)(int8_t)((cw[i] >> (8 * e2 + 8)) & 0xFF);
        qsum += q0 + q1;
        const float a0 = (float)q0 * d, a1 = (float)q1 * d;  // exact for an fp16 d
        const __half2 h = __floats2half2_rn(a0, a1);
        const float2 hf = __half22float2(h);
        const __half2 l = __floats2half2_rn((a0 - hf.x) * 2048.0f, (a1 - hf.y) * 2048.0f);
        hw[2 * i + e2 / 2] = *reinterpret_cast<const uint32_t*>(&h);
        lw[2 * i + e2 / 2] = *reinterpret_cast<const uint32_t*>(&l);
      }
    }
    uint4* dh = reinterpret_cast<uint4*>(hrow + 32 * b);
    uint4* dl = reinterpret_cast<uint4*>(lrow + 32 * b);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      dh[i] = make_uint4(hw[4 * i], hw[4 * i + 1], hw[4 * i + 2], hw[4 * i + 3]);
      dl[i] = make_uint4(lw[4 * i], lw[4 * i + 1], lw[4 * i + 2], lw[4 * i + 3]);
    }
    if constexpr (WT != KQ_Q8_0) hrow[K + b] = __float2half_rn((v.y - v.x * (float)qsum) * down);
  }
  for (int b = nb + threadIdx.x; b < Kp - K; b += blockDim.x) hrow[K + b] = __float2half_rn(0.0f);
}

template <int WT>
kq_status_t launch_split(const void* w, Act8 act, const OutSpec& out, int M, int N, int K, cudaStream_t s, int* err) {
  using T = SxTraits<WT>;
  const int nb = K / 32;
  const int nmain = K / CK;
  const int ngrp = T::kExtra ? (nmain + GRP - 1) / GRP : 0;
  const int Kp = K + ngrp * CK;
  const int num_t_tiles = (M + TT - 1) / TT;
  const int num_tiles = num_t_tiles * ((N + TW - 1) / TW);
  const int upt = nmain / UNIT;
  const int num_units = num_tiles * upt;
  const int grid = std::max(1, std::min(sm_count(), num_units));
  auto up = [](size_t b) { return (b + 255) & ~(size_t)255; };
  const size_t hi_bytes = up((size_t)M * Kp * sizeof(__half));
  const size_t lo_bytes = up((size_t)M * K * sizeof(__half));
  const size_t rs_bytes = up((size_t)M * sizeof(float));
  const size_t fl_bytes = up((size_t)grid * sizeof(int));
  const size_t pt_bytes = (size_t)grid * TT * TW * sizeof(float);
  uint8_t* ws = static_cast<uint8_t*>(workspace(WS_A16, hi_bytes + lo_bytes + rs_bytes + fl_bytes + pt_bytes));
  if (!ws) return KQ_ERR_NOMEM;
  __half* a_hi = reinterpret_cast<__half*>(ws);
  __half* a_lo = reinterpret_cast<__half*>(ws + hi_bytes);
  float* rscale = reinterpret_cast<float*>(ws + hi_bytes + lo_bytes);
  int* flags = reinterpret_cast<int*>(ws + hi_bytes + lo_bytes + rs_bytes);
  float* partial = reinterpret_cast<float*>(ws + hi_bytes + lo_bytes + rs_bytes + fl_bytes);
  {
    // a programmatic dependent of the quantiser that usually precedes it: its
    // launch overlaps the quantiser's tail, its reads wait for its results
    cudaLaunchConfig_t pc = {};
    pc.gridDim = dim3(M);
    pc.blockDim = dim3(128);
    pc.stream = s;
    cudaLaunchAttribute pa[1];
    pa[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    pa[0].val.programmaticStreamSerializationAllowed = 1;
    pc.attrs = pa;
    pc.numAttrs = 1;
    cudaError_t pe = cudaLaunchKernelEx(&pc, split_act_kernel<WT>, act, M, K, Kp, a_hi, a_lo, rscale, flags, grid);
    if (pe != cudaSuccess) return check_cuda(pe, "split_act launch");
  }
  kq_status_t st = check_launch("split_act");
  if (st) return st;
  CUtensorMap m_hi, m_lo, m_raw;
  if (!encode_map(&m_hi, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a_hi, (uint64_t)Kp, (uint64_t)M, (uint64_t)Kp * 2, CK, TT,
                  CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_map(&m_lo, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a_lo, (uint64_t)K, (uint64_t)M, (uint64_t)K * 2, CK, TT,
                  CU_TENSOR_MAP_SWIZZLE_128B))
    return fail(KQ_ERR_CUDA, "tensor map (split activations) rejected");
  const uint64_t rowbytes = (uint64_t)nb * T::BB;
  if (!encode_map(&m_raw, CU_TENSOR_MAP_DATA_TYPE_UINT16, w, rowbytes / 2, (uint64_t)N, rowbytes, T::RAW_ROW / 2, TW,
                  CU_TENSOR_MAP_SWIZZLE_NONE))
    return fail(KQ_ERR_CUDA, "tensor map (weights) rejected");

  const bool scatter = out.n_out > 1 || out.ld != N || out.col0 != 0;
  auto kern = scatter ? gemm_split_kernel<WT, true> : gemm_split_kernel<WT, false>;
  if (kq_status_t st = ensure_dynamic_smem(reinterpret_cast<const void*>(kern), T::SMEM, "gemm_split smem attribute"))
    return st;
  SxParams p;
  p.M = M; p.N = N; p.K = K;
  p.nmain = nmain; p.ngrp = ngrp;
  p.num_t_tiles = num_t_tiles;
  p.num_tiles = num_tiles;
  p.upt = upt;
  p.num_units = num_units;
  p.out = out;
  p.rscale = rscale;
  p.flags = flags;
  p.partial = partial;
  p.err = err ? err : device_error_word();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = T::SMEM;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;  // the prep kernel precedes on this stream
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, m_hi, m_lo, m_raw, p);
  if (e != cudaSuccess) return check_cuda(e, "gemm_split launch");
  return check_launch("gemm_split");
}

}  // namespace

bool gemm_split_supported(int wtype, int M, int N, int K, const void* w, Act8 act) {
  (void)act;
  return (wtype == KQ_Q4_0 || wtype == KQ_Q4_1 || wtype == KQ_Q8_0) && M > 8 && N >= 1 && K >= 256 &&
         K % 256 == 0 && (reinterpret_cast<uintptr_t>(w) & 15) == 0;
}

kq_status_t launch_gemm_split(int wtype, const void* w, Act8 act, const OutSpec& out, int M, int N, int K,
                              cudaStream_t s, int* err) {
  switch (wtype) {
    case KQ_Q4_0: return launch_split<KQ_Q4_0>(w, act, out, M, N, K, s, err);
    case KQ_Q4_1: return launch_split<KQ_Q4_1>(w, act, out, M, N, K, s, err);
    case KQ_Q8_0: return launch_split<KQ_Q8_0>(w, act, out, M, N, K, s, err);
    default: return fail(KQ_ERR_INVALID, "unknown weight type %d", wtype);
  }
}

}  // namespace kq
