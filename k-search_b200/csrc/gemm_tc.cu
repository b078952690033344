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
// CTA = 11 warps, one CTA per SM, persistent over 128 x 128 output tiles
// (tokens x weight rows), tokens fastest so co-running CTAs share weights in L2:
//   warp 0      TMA producer: activation codes (int8 [M, K], 128B-swizzled
//               boxes of 128 rows x 128 B = 4 blocks), activation (d, s)
//               pairs, and raw weight rows (the unchanged AoS q-blocks,
//               128 rows x 8 blocks per box); every CTA loads its own tiles.
//   warps 1-2   MMA issuers (one thread each): warp 1+i issues K blocks
//               i, i+2 of every stage into TMEM buffers i, i+2, so two
//               issue/commit latency chains run side by side; warp 1 also
//               owns the TMEM allocation.
//   warps 3-10  workers. For K stage s they first convert the raw weight
//               blocks of stage s+1 (two blocks of one row per thread) into
//               int8 codes in the UMMA K-major SWIZZLE_128B layout plus fp32
//               scale rows (then fence.proxy.async and release it to the MMA),
//               then run the epilogue of stage s: read each block's int32
//               result from TMEM (tcgen05.ld 32x32b, 64 columns per thread),
//               apply the block's scales and accumulate in fp32 registers.
//               4 TMEM buffers of 128 columns let the MMA run ahead.
#include <cuda.h>

#include <algorithm>
#include <mutex>

#include "kq_internal.h"
#include "kq_device.cuh"

namespace kq {
namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

CUresult encode_tiled(CUtensorMap* map, CUtensorMapDataType dt, cuuint32_t rank, void* base, const cuuint64_t* dims,
                      const cuuint64_t* strides, const cuuint32_t* box, const cuuint32_t* estr,
                      CUtensorMapInterleave il, CUtensorMapSwizzle sw, CUtensorMapL2promotion l2,
                      CUtensorMapFloatOOBfill oob) {
  auto fn = reinterpret_cast<EncodeTiledFn>(tensor_map_encoder());
  if (!fn) return CUDA_ERROR_NOT_SUPPORTED;
  return fn(map, dt, rank, base, dims, strides, box, estr, il, sw, l2, oob);
}

constexpr int TM = 128;        // tokens per tile (TMEM lanes)
constexpr int TN = 128;        // weight rows per tile (TMEM columns per buffer)
constexpr int KSUB = 4;        // blocks per activation / converted-weight stage (128 B of K)
constexpr int KRAW = 8;        // blocks per raw weight stage (16-byte aligned for all block sizes)
constexpr int SA = 3;          // activation stages
constexpr int SWS = 3;         // converted weight stages
constexpr int SRAW = 2;        // raw weight stages
constexpr int NBUF = 4;        // TMEM buffers
constexpr int kWarpTma = 0, kWarpMma = 1, kMmaWarps = 2, kWarpWork = kWarpMma + kMmaWarps, kWorkWarps = 8;
constexpr int kEpiCols = TN / (kWorkWarps / 4);  // columns per worker thread in the epilogue (32)
constexpr int kWarps = kWarpWork + kWorkWarps;
constexpr int kThreads = kWarps * 32;
constexpr int kTmemCols = NBUF * TN;  // 512
static_assert(NBUF == KSUB && NBUF % kMmaWarps == 0, "one TMEM buffer per K block of a stage, split over the issuers");

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
  // byte offsets in dynamic shared memory (base aligned to 1024)
  static constexpr int OFF_ACT = 0;
  static constexpr int OFF_W = OFF_ACT + SA * ACT_TILE;
  static constexpr int OFF_RAW = OFF_W + SWS * W_TILE;
  static constexpr int OFF_ASC = OFF_RAW + SRAW * RAW_STAGE;
  static constexpr int OFF_WSC = OFF_ASC + SA * ASC_STAGE;
  static constexpr int OFF_BAR = (OFF_WSC + SWS * WSC_STAGE + 15) / 16 * 16;
  static constexpr int NBARS = 2 * SA + 2 * SWS + 2 * SRAW + 2 * NBUF;
  static constexpr int OFF_TMEM = OFF_BAR + NBARS * 8;
  static constexpr int SMEM = OFF_TMEM + 16 + 1024;  // + alignment slack
  static_assert(RAW_ROW % 16 == 0, "raw rows must stay 16-byte aligned");
  static_assert(SMEM <= 232448, "shared memory budget");
};

// ---- tcgen05 / TMA primitives ---------------------------------------------
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
        "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
      "[%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Writes the same 32-bit value to 32 consecutive columns of this thread's lane.
__device__ __forceinline__ void tmem_st32_const(uint32_t taddr, uint32_t v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, "
      "%1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1};" ::"r"(taddr),
      "r"(v)
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

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
__device__ __forceinline__ float round22(float d) {
  return __uint_as_float((__float_as_uint(d) + 2u) & ~3u);
}

__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// UMMA shared-memory descriptor: K-major, SWIZZLE_128B, 8-row groups 1024 B
// apart (SBO), version 1 (sm_100).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;                 // LBO (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;       // SBO
  d |= (uint64_t)1 << 46;                 // version
  d |= (uint64_t)2 << 61;                 // SWIZZLE_128B
  return d;
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

// byte offset of (row r, 16-byte chunk c) in a 128B-swizzled K-major tile
__device__ __forceinline__ int sw128_off(int r, int c) { return (r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4); }

struct TcParams {
  int M, N, K, nb;
  int num_m_tiles, num_tiles;
  float* out;
  int* err;
};

template <int WT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap map_act, const __grid_constant__ CUtensorMap map_asc,
                   const __grid_constant__ CUtensorMap map_raw, TcParams p) {
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

  if (threadIdx.x == 0) {
    for (int i = 0; i < SA; ++i) {
      mbar_init(&act_full[i], 1);
      mbar_init(&act_empty[i], kMmaWarps + kWorkWarps);  // MMA commits + workers (they read the scales)
    }
    for (int i = 0; i < SWS; ++i) {
      mbar_init(&w_full[i], kWorkWarps);
      mbar_init(&w_empty[i], kMmaWarps + kWorkWarps);
    }
    for (int i = 0; i < SRAW; ++i) {
      mbar_init(&raw_full[i], 1);
      mbar_init(&raw_empty[i], kWorkWarps);
    }
    for (int i = 0; i < NBUF; ++i) {
      mbar_init(&tm_full[i], 1);
      mbar_init(&tm_empty[i], kWorkWarps);
    }
    fence_mbar_init();
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
          if (ir >= SRAW) mbar_wait_or_poison(&raw_empty[rs], ((ir / SRAW) - 1) & 1, p.err, DEV_TIMEOUT_EMPTY, dead);
          mbar_arrive_expect_tx(&raw_full[rs], T::RAW_STAGE);
          tma_load_2d(smem + T::OFF_RAW + rs * T::RAW_STAGE, &map_raw, k8 * (T::RAW_ROW / 2), n0, &raw_full[rs]);
          if (!waited_pdl) {  // activations are produced by the preceding kernel
            pdl_wait();
            waited_pdl = true;
          }
          for (int sub = 0; sub < KRAW / KSUB; ++sub, ++ia) {
            const int as = ia % SA;
            if (ia >= SA) mbar_wait_or_poison(&act_empty[as], ((ia / SA) - 1) & 1, p.err, DEV_TIMEOUT_EMPTY, dead);
            const int kb = k8 * KRAW + sub * KSUB;  // first block of this stage
            mbar_arrive_expect_tx(&act_full[as], T::ACT_TILE + T::ASC_STAGE);
            tma_load_2d(smem + T::OFF_ACT + as * T::ACT_TILE, &map_act, kb * 32, m0, &act_full[as]);
            tma_load_2d(smem + T::OFF_ASC + as * T::ASC_STAGE, &map_asc, kb * 2, m0, &act_full[as]);
          }
        }
      }
    }
  } else if (warp < kWarpWork) {
    // ------------------------------------------------------------ MMA issuers
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_i8(T::kSignedW);
      const int i0 = warp - kWarpMma;  // this thread issues K blocks i0, i0 + kMmaWarps, ... of every stage
      const uint32_t act_base = smem_u32(smem + T::OFF_ACT);
      const uint32_t w_base = smem_u32(smem + T::OFF_W);
      int ia = 0;
      for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x) {
        for (int s = 0; s < p.nb / KSUB; ++s, ++ia) {
          const int as = ia % SA, ws = ia % SWS;
          mbar_wait_or_poison(&act_full[as], (ia / SA) & 1, p.err, DEV_TIMEOUT_FULL, dead);
          mbar_wait_or_poison(&w_full[ws], (ia / SWS) & 1, p.err, DEV_TIMEOUT_FULL, dead);
          const uint64_t adesc = sw128_desc(act_base + as * T::ACT_TILE);
          const uint64_t bdesc = sw128_desc(w_base + ws * T::W_TILE);
#pragma unroll
          for (int j = i0; j < KSUB; j += kMmaWarps) {
            mbar_wait_or_poison(&tm_empty[j], ia & 1, p.err, DEV_TIMEOUT_EMPTY, dead);
            tc_fence_after();
            // K block j of the stage: +32 bytes inside the 128-byte swizzle atom;
            // accumulate onto the bias words the workers left in the buffer.
            mma_i8(tmem_base + j * TN, adesc + (uint64_t)(2 * j), bdesc + (uint64_t)(2 * j), idesc, 1u);
            mma_commit(&tm_full[j]);
          }
          mma_commit(&act_empty[as]);
          mma_commit(&w_empty[ws]);
        }
      }
    }
  } else {
    // ------------------------------------------------------------ workers
    const int wi = warp - kWarpWork;        // 0..7
    const int quarter = warp & 3;           // TMEM lane quarter this warp may access
    const int cg = wi >> 2;                 // column half of the epilogue
    const int row = quarter * 32 + lane;    // token row in the tile (epilogue)
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    const int crow = (wi * 32 + lane) >> 1; // weight row converted by this thread
    const int chalf = lane & 1;             // blocks 2*chalf, 2*chalf+1 of the 4-block stage
    const int coff0 = sw128_off(crow, 4 * chalf), coff1 = sw128_off(crow, 4 * chalf + 1);
    const int coff2 = sw128_off(crow, 4 * chalf + 2), coff3 = sw128_off(crow, 4 * chalf + 3);
    const int spt = p.nb / KSUB;            // K stages per tile (even: nb % 8 == 0)
    const int my_tiles = (p.num_tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
    const int total = my_tiles * spt;

    // Convert global stage gs: blocks 2*chalf, 2*chalf+1 of row crow.
    auto convert = [&](int gs) {
      const int irr = gs >> 1, sub = gs & 1;
      const int rs = irr % SRAW;
      mbar_wait_or_poison(&raw_full[rs], (irr / SRAW) & 1, p.err, DEV_TIMEOUT_FULL, dead);
      constexpr int HB = 2 * T::BB;  // 36 / 40 / 68 bytes, 4-byte aligned
      const uint32_t* src = reinterpret_cast<const uint32_t*>(smem + T::OFF_RAW + rs * T::RAW_STAGE +
                                                              crow * T::RAW_ROW + (sub * KSUB + 2 * chalf) * T::BB);
      uint32_t w[HB / 4 + 1];
#pragma unroll
      for (int i = 0; i < HB / 4; ++i) w[i] = src[i];
      w[HB / 4] = 0;
      const int ws = gs % SWS;
      if (gs >= SWS) mbar_wait_or_poison(&w_empty[ws], ((gs / SWS) - 1) & 1, p.err, DEV_TIMEOUT_EMPTY, dead);
      uint8_t* wt = smem + T::OFF_W + ws * T::W_TILE;
      float* wsc = reinterpret_cast<float*>(smem + T::OFF_WSC + ws * T::WSC_STAGE);
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
        const int o = jj * T::BB;  // compile-time after unrolling
        auto u32 = [&](int off) -> uint32_t {
          return (off & 3) ? __funnelshift_r(w[off >> 2], w[(off >> 2) + 1], 16) : w[off >> 2];
        };
        auto u16 = [&](int off) -> uint32_t { return (off & 3) ? (w[off >> 2] >> 16) : (w[off >> 2] & 0xFFFFu); };
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
        *reinterpret_cast<uint4*>(wt + (jj == 0 ? coff0 : coff2)) = c0;
        *reinterpret_cast<uint4*>(wt + (jj == 0 ? coff1 : coff3)) = c1;
        const int j = 2 * chalf + jj;
        wsc[j * TN + crow] = d;
        if constexpr (T::kHasMin) wsc[KSUB * TN + j * TN + crow] = mn;
      }
      fence_proxy_async_smem();  // generic-proxy writes -> tensor-core reads
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&w_full[ws]);
        if (sub == 1) mbar_arrive(&raw_empty[rs]);  // both halves of the raw stage are converted
      }
    };

    // every TMEM buffer starts free, preset to the bias
    for (int b = 0; b < NBUF; ++b)
      for (int c32 = 0; c32 < kEpiCols / 32; ++c32)
        tmem_st32_const(tmem_base + lane_addr + b * TN + cg * kEpiCols + 32 * c32, kBias);
    tmem_st_wait();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) {
      for (int b = 0; b < NBUF; ++b) mbar_arrive(&tm_empty[b]);
    }

    if (total > 0) convert(0);
    float acc[kEpiCols];  // fp32 accumulators
    int ib = 0;
    for (int es = 0; es < total; ++es) {
      if (es + 1 < total) convert(es + 1);
      const int s = es % spt;
      const int t = (int)blockIdx.x + (es / spt) * (int)gridDim.x;
      if (s == 0) {
#pragma unroll
        for (int c = 0; c < kEpiCols; ++c) acc[c] = 0.0f;
      }
      const int as = es % SA, ws = es % SWS;
      mbar_wait_or_poison(&act_full[as], (es / SA) & 1, p.err, DEV_TIMEOUT_FULL, dead);
      mbar_wait_or_poison(&w_full[ws], (es / SWS) & 1, p.err, DEV_TIMEOUT_FULL, dead);
      const float2* asc = reinterpret_cast<const float2*>(smem + T::OFF_ASC + as * T::ASC_STAGE) + row * KSUB;
      const float* wsc = reinterpret_cast<const float*>(smem + T::OFF_WSC + ws * T::WSC_STAGE);
#pragma unroll 1
      for (int j = 0; j < KSUB; ++j, ++ib) {
        const int buf = ib % NBUF;
        const float2 dsj = asc[j];
        const float d = round22(dsj.x);
        const float ncs = -kBiasF * d;
        const float ms8 = -8.0f * dsj.y;
        const float sy = dsj.y;
        const float* dw = wsc + j * TN + cg * kEpiCols;
        const float* mw = wsc + KSUB * TN + j * TN + cg * kEpiCols;
        mbar_wait_or_poison(&tm_full[buf], (ib / NBUF) & 1, p.err, DEV_TIMEOUT_FULL, dead);
        tc_fence_after();
        const uint32_t taddr = tmem_base + lane_addr + buf * TN + cg * kEpiCols;
        // 16 columns per TMEM round trip; re-arm the bias (asynchronously) and
        // hand the buffer back after the math
#pragma unroll
        for (int h = 0; h < kEpiCols / 16; ++h) {
          uint32_t v[16];
          tmem_ld16(taddr + 16 * h, v);
          tmem_ld_wait();
          if (h == kEpiCols / 16 - 1) {
#pragma unroll
            for (int c32 = 0; c32 < kEpiCols / 32; ++c32) tmem_st32_const(taddr + 32 * c32, kBias);
          }
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float4 w4 = reinterpret_cast<const float4*>(dw + 16 * h)[q];  // scales of 4 columns (broadcast)
            const float wv[4] = {w4.x, w4.y, w4.z, w4.w};
            float mv[4] = {0.f, 0.f, 0.f, 0.f};
            if constexpr (WT == KQ_Q4_1) {
              const float4 m4 = reinterpret_cast<const float4*>(mw + 16 * h)[q];
              mv[0] = m4.x; mv[1] = m4.y; mv[2] = m4.z; mv[3] = m4.w;
            }
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int c = 16 * h + 4 * q + e;
              const float pr = fmaf(__uint_as_float(v[4 * q + e]), d, ncs);  // d_a * sumi
              if constexpr (WT == KQ_Q8_0) {
                acc[c] = fmaf(pr, wv[e], acc[c]);
              } else if constexpr (WT == KQ_Q4_0) {
                acc[c] = fmaf(pr + ms8, wv[e], acc[c]);  // d_w * (d_a sumi - 8 s_a)
              } else {
                acc[c] = fmaf(mv[e], sy, fmaf(pr, wv[e], acc[c]));  // d_w d_a sumi + m_w s_a
              }
            }
          }
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tm_empty[buf]);
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&act_empty[as]);
        mbar_arrive(&w_empty[ws]);
      }
      if (s == spt - 1) {
        // ---- store this tile's rows ----
        const int m0 = (t % p.num_m_tiles) * TM, n0 = (t / p.num_m_tiles) * TN;
        const int m = m0 + row;
        const int nc0 = n0 + cg * kEpiCols;
        if (m < p.M) {
          float* o = p.out + (size_t)m * p.N + nc0;
          if (nc0 + kEpiCols <= p.N && (p.N & 3) == 0) {
#pragma unroll
            for (int c = 0; c < kEpiCols; c += 4)
              *reinterpret_cast<float4*>(o + c) = make_float4(acc[c], acc[c + 1], acc[c + 2], acc[c + 3]);
          } else {
#pragma unroll
            for (int c = 0; c < kEpiCols; ++c)
              if (nc0 + c < p.N) o[c] = acc[c];
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

// ---- host side -----------------------------------------------------------------
bool encode_map(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t dim0, uint64_t dim1,
                uint64_t stride1_bytes, uint32_t box0, uint32_t box1, CUtensorMapSwizzle swz) {
  cuuint64_t dims[2] = {dim0, dim1};
  cuuint64_t strides[1] = {stride1_bytes};
  cuuint32_t box[2] = {box0, box1};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_tiled(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                                      CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <int WT>
kq_status_t launch_tc(const void* w, Act8 act, float* out, int M, int N, int K, bool pdl, cudaStream_t s, int* err) {
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

  auto kern = gemm_tc_kernel<WT>;
  static unsigned attr_done = 0;
  const int dev = current_device();
  if (!(attr_done & (1u << (dev & 31)))) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, T::SMEM);
    if (e != cudaSuccess) return check_cuda(e, "gemm_tc smem attribute");
    attr_done |= 1u << (dev & 31);
  }
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
  switch (wtype) {
    case KQ_Q4_0: return launch_tc<KQ_Q4_0>(w, act, out, M, N, K, pdl, s, err);
    case KQ_Q4_1: return launch_tc<KQ_Q4_1>(w, act, out, M, N, K, pdl, s, err);
    case KQ_Q8_0: return launch_tc<KQ_Q8_0>(w, act, out, M, N, K, pdl, s, err);
    default: return fail(KQ_ERR_INVALID, "unknown weight type %d", wtype);
  }
}

}  // namespace kq
