// Quantised GEMM for 8 < M <= 128 activation rows ("skinny": the weight
// stream dominates). Formulas: the reference's per-block integer sums
// (llm_kernel_test/reference/gemm_ref.py:100-153 q4_0, :274-331 q4_1;
// include/gemm_reference.h:311-336 q8_0):
//   q4_0  out[m, n] = sum_b d_w (d_a sumi - 8 s_a)
//   q4_1  out[m, n] = sum_b d_w d_a sumi + m_w s_a
//   q8_0  out[m, n] = sum_b d_w d_a sumi
// with sumi the int32 dot of the stored weight codes (nibbles 0..15, or int8)
// and the q8_1 activation codes of block b.
//
// Design (B200): the weights are read from HBM exactly once. Each CTA (one
// per SM) owns up to 8 groups of 16 weight rows; a producer warp streams
// 256-wide K chunks of those rows (the unchanged AoS blocks, one TMA box per
// 16 rows) together with the whole activation chunk (int8 codes in a
// 128-byte-swizzled tile and the (d, s) pairs) into a shared-memory ring.
// Eight compute warps tile (row group, 8-token group) pairs and run
// mma.sync.m16n8k32 with the weight codes as A (u8 nibbles or s8) and the
// activation codes as B (s8): one MMA is one 32-wide block, so D is exactly
// the reference's sumi for 16 rows x 8 tokens. Its accumulator input is
// preset to 0x4B400000, so D is the fp32 bit pattern of 1.5 * 2^23 + sumi
// (|sumi| < 2^22) and the scale epilogue needs no conversion instruction;
// it runs on fp32 pairs (two tokens per instruction).
#include <algorithm>

#include "kq_internal.h"
#include "kq_device.cuh"
#include "kq_tc.cuh"

namespace kq {
namespace {

using namespace tc;

constexpr int kRowsPerGroup = 16;
constexpr int kMaxGroups = 8;            // row groups per CTA
constexpr int kMaxTok = 128;             // activation rows
constexpr int kChunkK = 256;             // K elements per stage (8 blocks)
constexpr int kComputeWarps = 8;   // per K half
constexpr int threads_of(int ks) { return 32 * (kComputeWarps * ks + 1); }
constexpr uint32_t kMagic = 0x4B400000u; // bits of 12582912.0f = 1.5 * 2^23
constexpr float kMagicF = 12582912.0f;

template <int WT>
struct SkTraits {
  static constexpr int BB = WT == KQ_Q4_0 ? 18 : WT == KQ_Q4_1 ? 20 : 34;
  static constexpr int ROW = 8 * BB;      // bytes of one weight row per chunk (144 / 160 / 272)
};

struct SkParams {
  OutSpec out;
  int M, N, K;
  int Mp;             // M rounded up to 8 (the activation box height)
  int RG;             // row groups ceil(N / 16)
  int stages;
  int stage_bytes;    // one ring stage: A codes | scales | weights
  int off_x;          // K split: partial-sum exchange buffer (after the ring and its barriers)
  int off_s, off_w;   // offsets of the scales and weights inside a stage
  int* err;
};

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
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// D = A (16 x 32) B (32 x 8) + 0x4B400000, A = weight codes, B = activation codes (s8)
template <int WT>
__device__ __forceinline__ void mma_block(uint32_t (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (WT == KQ_Q8_0) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%10, %10, %10, %10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(kMagic));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%10, %10, %10, %10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(kMagic));
  }
}

// 32-bit word at a shared address that is 4-byte aligned (ALIGNED) or 2-byte aligned
template <bool ALIGNED>
__device__ __forceinline__ uint32_t lds_word(const uint8_t* b) {
  if constexpr (ALIGNED) {
    return *reinterpret_cast<const uint32_t*>(b);
  } else {
    const uint32_t* q = reinterpret_cast<const uint32_t*>(b - 2);
    return __funnelshift_r(q[0], q[1], 16);
  }
}

__device__ __forceinline__ float lds_half(const uint8_t* b) {
  return __half2float(__ushort_as_half(*reinterpret_cast<const uint16_t*>(b)));
}

// A fragment of block BLK for rows g and g + 8 of a 16-row group (row stride
// ROW bytes), plus the rows' scales: a[0] = row g codes 4 tid .. +3,
// a[1] = row g + 8 same, a[2] = row g codes 16 + 4 tid .., a[3] = row g + 8.
template <int WT, int BLK>
__device__ __forceinline__ void load_a(const uint8_t* grp, int gid, int tid, uint32_t (&a)[4], uint64_t& dw2g,
                                       uint64_t& dw2h, uint64_t& mw2g, uint64_t& mw2h) {
  using T = SkTraits<WT>;
  const uint8_t* r0 = grp + gid * T::ROW + BLK * T::BB;
  const uint8_t* r1 = r0 + 8 * T::ROW;
  const float d0 = lds_half(r0), d1 = lds_half(r1);
  dw2g = pk2(d0, d0);
  dw2h = pk2(d1, d1);
  if constexpr (WT == KQ_Q8_0) {
    constexpr bool AL = ((BLK * T::BB + 2) & 3) == 0;  // ROW is a multiple of 4
    a[0] = lds_word<AL>(r0 + 2 + 4 * tid);
    a[1] = lds_word<AL>(r1 + 2 + 4 * tid);
    a[2] = lds_word<AL>(r0 + 18 + 4 * tid);
    a[3] = lds_word<AL>(r1 + 18 + 4 * tid);
  } else {
    constexpr int QO = WT == KQ_Q4_0 ? 2 : 4;
    constexpr bool AL = ((BLK * T::BB + QO) & 3) == 0;
    // byte i of a block holds element i (low nibble) and element i + 16 (high)
    const uint32_t w0 = lds_word<AL>(r0 + QO + 4 * tid), w1 = lds_word<AL>(r1 + QO + 4 * tid);
    a[0] = w0 & 0x0F0F0F0Fu;
    a[1] = w1 & 0x0F0F0F0Fu;
    a[2] = (w0 >> 4) & 0x0F0F0F0Fu;
    a[3] = (w1 >> 4) & 0x0F0F0F0Fu;
    if constexpr (WT == KQ_Q4_1) {
      const float m0 = lds_half(r0 + 2), m1 = lds_half(r1 + 2);
      mw2g = pk2(m0, m0);
      mw2h = pk2(m1, m1);
    }
  }
}

// one output element to every destination of the epilogue
__device__ __forceinline__ void put_out(const OutSpec& o, int m, int n, float v) {
  const size_t off = (size_t)m * o.ld + o.col0 + n;
  o.ptr[0][off] = v;
  for (int d = 1; d < o.n_out; ++d) o.ptr[d][off] = v;
}

// Warps form a WR x WTOK grid over (row group, token group): warp (wr, wt)
// takes row groups wr, wr + WR, ... and token groups wt, wt + WTOK, ...;
// TPW (token groups per warp) is a template parameter sized to the launch's
// token count, so the unrolled block loop holds only the token groups that
// exist (an instantiation for 128 tokens run at 16 missed the instruction
// cache on the guarded-off copies). KS = 2 splits every chunk's 8 blocks
// between two warps per (row group, token group) - blocks 0-3 and 4-7 - so
// twice as many warps hide the MMA -> FMA latency when there are few token
// groups; the two partial sums meet in shared memory at the end.
template <int WT, int WTOK, int TPW, int KS>
__global__ void __launch_bounds__(threads_of(KS), 1)
    gemm_skinny_kernel(const __grid_constant__ CUtensorMap m_w, const __grid_constant__ CUtensorMap m_a,
                       const __grid_constant__ CUtensorMap m_s, const __grid_constant__ SkParams p) {
  using T = SkTraits<WT>;
  constexpr int CW = kComputeWarps * KS;  // compute warps
  constexpr int BPW = 8 / KS;             // blocks of a chunk per warp
  constexpr int WR = kComputeWarps / WTOK;
  constexpr int RPW = (kMaxGroups + WR - 1) / WR;  // row groups per warp (at most)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.stages * p.stage_bytes);
  uint64_t* empty = full + p.stages;

  const int rg0 = (int)((long long)p.RG * blockIdx.x / gridDim.x);
  const int rg1 = (int)((long long)p.RG * (blockIdx.x + 1) / gridDim.x);
  const int GC = rg1 - rg0;
  if (GC <= 0) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nch = p.K / kChunkK;
  const int ntg = p.Mp / 8;

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], CW);
    }
    fence_mbar_init();
  }
  __syncthreads();

  bool dead = false;
  if (warp == CW) {
    // ---------------- producer ----------------
    if (lane == 0) {
      const uint32_t wbytes = (uint32_t)(GC * kRowsPerGroup * T::ROW);
      const uint32_t abytes = (uint32_t)(p.Mp * kChunkK + p.Mp * 64);
      auto load_w = [&](int k) {
        uint8_t* st = smem + (k % p.stages) * p.stage_bytes;
        for (int g = 0; g < GC; ++g)
          tma_load_2d(st + p.off_w + g * kRowsPerGroup * T::ROW, &m_w, k * T::BB, (rg0 + g) * kRowsPerGroup,
                      &full[k % p.stages]);
      };
      auto load_act = [&](int k) {
        uint8_t* st = smem + (k % p.stages) * p.stage_bytes;
        tma_load_2d(st, &m_a, k * kChunkK, 0, &full[k % p.stages]);
        tma_load_2d(st + p.Mp * 128, &m_a, k * kChunkK + 128, 0, &full[k % p.stages]);
        tma_load_2d(st + p.off_s, &m_s, k * 16, 0, &full[k % p.stages]);
      };
      const int pre = min(p.stages, nch);
      for (int k = 0; k < pre; ++k) {  // weights do not depend on the preceding kernel
        mbar_arrive_expect_tx(&full[k], wbytes + abytes);
        load_w(k);
      }
      pdl_wait();  // the activations are the preceding kernel's output
      for (int k = 0; k < pre; ++k) load_act(k);
      for (int k = pre; k < nch; ++k) {
        const int s = k % p.stages;
        mbar_wait_or_poison(&empty[s], ((k / p.stages) - 1) & 1, p.err, DEV_TIMEOUT_EMPTY, dead);
        mbar_arrive_expect_tx(&full[s], wbytes + abytes);
        load_w(k);
        load_act(k);
      }
      for (int k = max(0, nch - p.stages); k < nch; ++k)
        mbar_wait_or_poison(&empty[k % p.stages], (k / p.stages) & 1, p.err, DEV_TIMEOUT_EMPTY, dead);
    }
    return;
  }

  // ---------------- compute warp ----------------
  const int kh = warp / kComputeWarps, w8 = warp % kComputeWarps;  // K half, warp within it
  const int wr = w8 % WR, wt = w8 / WR;
  const int gid = lane >> 2, tid = lane & 3;
  uint64_t acc[RPW][TPW][2];  // [row group][token group][row g | row g + 8] x tokens 2 tid, 2 tid + 1
#pragma unroll
  for (int i = 0; i < RPW; ++i)
#pragma unroll
    for (int j = 0; j < TPW; ++j) acc[i][j][0] = acc[i][j][1] = 0ull;
  const uint64_t neg_magic2 = pk2(-kMagicF, -kMagicF);

  for (int k = 0; k < nch; ++k) {
    const int s = k % p.stages;
    mbar_wait_or_poison(&full[s], (k / p.stages) & 1, p.err, DEV_TIMEOUT_FULL, dead);
    const uint8_t* st = smem + s * p.stage_bytes;
    const float2* sc = reinterpret_cast<const float2*>(st + p.off_s);   // [Mp][8] (d, s)
    const uint8_t* wst = st + p.off_w;
#pragma unroll
    for (int bi = 0; bi < BPW; ++bi) {
      const int blk = bi + kh * BPW;
      uint32_t a[RPW][4];
      uint64_t dwg[RPW], dwh[RPW], mwg[RPW] = {}, mwh[RPW] = {};
#pragma unroll
      for (int i = 0; i < RPW; ++i) {
        const int r = wr + i * WR;
        if (r < GC) {
          const uint8_t* grp = wst + r * kRowsPerGroup * T::ROW;
          switch (blk) {  // compile-time block index after unrolling
            case 0: load_a<WT, 0>(grp, gid, tid, a[i], dwg[i], dwh[i], mwg[i], mwh[i]); break;
            case 1: load_a<WT, 1>(grp, gid, tid, a[i], dwg[i], dwh[i], mwg[i], mwh[i]); break;
            case 2: load_a<WT, 2>(grp, gid, tid, a[i], dwg[i], dwh[i], mwg[i], mwh[i]); break;
            case 3: load_a<WT, 3>(grp, gid, tid, a[i], dwg[i], dwh[i], mwg[i], mwh[i]); break;
            case 4: load_a<WT, 4>(grp, gid, tid, a[i], dwg[i], dwh[i], mwg[i], mwh[i]); break;
            case 5: load_a<WT, 5>(grp, gid, tid, a[i], dwg[i], dwh[i], mwg[i], mwh[i]); break;
            case 6: load_a<WT, 6>(grp, gid, tid, a[i], dwg[i], dwh[i], mwg[i], mwh[i]); break;
            default: load_a<WT, 7>(grp, gid, tid, a[i], dwg[i], dwh[i], mwg[i], mwh[i]); break;
          }
        }
      }
      // activation codes: 128-byte swizzled rows; block blk lies in half blk / 4
      const uint8_t* ah = st + (blk >> 2) * (p.Mp * 128);
      const int c0 = 2 * (blk & 3);
#pragma unroll
      for (int j = 0; j < TPW; ++j) {
        const int t = wt + j * WTOK;
        if (t < ntg) {
          const int row = 8 * t + gid;
          const uint8_t* ar = ah + row * 128 + 4 * tid;
          const uint32_t b0 = *reinterpret_cast<const uint32_t*>(ar + ((c0 ^ (row & 7)) << 4));
          const uint32_t b1 = *reinterpret_cast<const uint32_t*>(ar + (((c0 + 1) ^ (row & 7)) << 4));
          const float2 s0 = sc[(8 * t + 2 * tid) * 8 + blk], s1 = sc[(8 * t + 2 * tid + 1) * 8 + blk];
          const uint64_t da2 = pk2(s0.x, s1.x);
          uint64_t cst2 = 0;
          if constexpr (WT == KQ_Q4_0) cst2 = pk2(-8.0f * s0.y, -8.0f * s1.y);
          if constexpr (WT == KQ_Q4_1) cst2 = pk2(s0.y, s1.y);
#pragma unroll
          for (int i = 0; i < RPW; ++i) {
            const int r = wr + i * WR;
            if (r < GC) {
              uint32_t d[4];
              mma_block<WT>(d, a[i], b0, b1);
              // f = sumi exactly (the preset bias removed), then the block's scales
              const uint64_t fg = add2(pk2u(d[0], d[1]), neg_magic2);
              const uint64_t fh = add2(pk2u(d[2], d[3]), neg_magic2);
              if constexpr (WT == KQ_Q4_0) {
                acc[i][j][0] = fma2(dwg[i], fma2(da2, fg, cst2), acc[i][j][0]);
                acc[i][j][1] = fma2(dwh[i], fma2(da2, fh, cst2), acc[i][j][1]);
              } else if constexpr (WT == KQ_Q8_0) {
                acc[i][j][0] = fma2(dwg[i], mul2(da2, fg), acc[i][j][0]);
                acc[i][j][1] = fma2(dwh[i], mul2(da2, fh), acc[i][j][1]);
              } else {
                acc[i][j][0] = fma2(dwg[i], mul2(da2, fg), fma2(mwg[i], cst2, acc[i][j][0]));
                acc[i][j][1] = fma2(dwh[i], mul2(da2, fh), fma2(mwh[i], cst2, acc[i][j][1]));
              }
            }
          }
        }
      }
    }
    fence_proxy_async_smem();  // generic reads of the TMA-refilled stage, before its release
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }

  if constexpr (KS == 2) {
    // the second K half hands its partial sums to the first
    uint64_t* xb = reinterpret_cast<uint64_t*>(smem + p.off_x) + ((size_t)w8 * 32 + lane) * (RPW * TPW * 2);
    if (kh == 1) {
#pragma unroll
      for (int i = 0; i < RPW; ++i)
#pragma unroll
        for (int j = 0; j < TPW; ++j) {
          xb[(i * TPW + j) * 2] = acc[i][j][0];
          xb[(i * TPW + j) * 2 + 1] = acc[i][j][1];
        }
    }
    named_bar_sync(1, CW * 32);
    if (kh == 1) return;
#pragma unroll
    for (int i = 0; i < RPW; ++i)
#pragma unroll
      for (int j = 0; j < TPW; ++j) {
        acc[i][j][0] = add2(acc[i][j][0], xb[(i * TPW + j) * 2]);
        acc[i][j][1] = add2(acc[i][j][1], xb[(i * TPW + j) * 2 + 1]);
      }
  }

  // ---- store: rows 16 (rg0 + r) + gid (+ 8), tokens 8 t + 2 tid (+ 1) ----
#pragma unroll
  for (int i = 0; i < RPW; ++i) {
    const int r = wr + i * WR;
    if (r >= GC) continue;
#pragma unroll
    for (int j = 0; j < TPW; ++j) {
      const int t = wt + j * WTOK;
      if (t >= ntg) continue;
      const int m = 8 * t + 2 * tid;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int n = (rg0 + r) * kRowsPerGroup + gid + 8 * h;
        const float2 v = upk2(acc[i][j][h]);
        if (n < p.N) {
          if (m < p.M) put_out(p.out, m, n, v.x);
          if (m + 1 < p.M) put_out(p.out, m + 1, n, v.y);
        }
      }
    }
  }
  if (p.out.n_out > 1) __threadfence_system();  // peer stores visible before the host-side barrier
}

template <int WT, int WTOK, int TPW, int KS>
kq_status_t launch_cfg(const CUtensorMap& mw, const CUtensorMap& ma, const CUtensorMap& ms, const SkParams& p,
                       int grid, size_t smem, cudaStream_t s) {
  auto kern = gemm_skinny_kernel<WT, WTOK, TPW, KS>;
  if (kq_status_t st = ensure_dynamic_smem(reinterpret_cast<const void*>(kern), (int)smem, "gemm_skinny smem attribute"))
    return st;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(threads_of(KS));
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;  // the activation quantiser precedes on this stream
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, mw, ma, ms, p);
  if (e != cudaSuccess) return check_cuda(e, "gemm_skinny launch");
  return check_launch("gemm_skinny");
}

template <int WT>
kq_status_t launch_wt(const void* w, Act8 act, const OutSpec& out, int M, int N, int K, cudaStream_t s, int* err) {
  using T = SkTraits<WT>;
  SkParams p{};
  p.out = out;
  p.M = M;
  p.N = N;
  p.K = K;
  p.Mp = (M + 7) & ~7;
  p.RG = (N + kRowsPerGroup - 1) / kRowsPerGroup;
  const int grid = std::max(std::min(sm_count(), p.RG), (p.RG + kMaxGroups - 1) / kMaxGroups);
  const int gc = (p.RG + grid - 1) / grid;  // row groups of the largest CTA
  // stage: A codes (two 128-byte halves, 1024-aligned) | scales (Mp x 64 B) | weights
  p.off_s = 2 * p.Mp * 128;
  p.off_w = p.off_s + p.Mp * 64;
  p.stage_bytes = (p.off_w + gc * kRowsPerGroup * T::ROW + 1023) & ~1023;
  p.err = err ? err : device_error_word();

  const int nb = K / 32;
  const uint64_t rowbytes = (uint64_t)nb * T::BB;
  CUtensorMap mw, ma, ms;
  if (!encode_map(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT64, w, rowbytes / 8, (uint64_t)N, rowbytes, T::ROW / 8,
                  kRowsPerGroup, CU_TENSOR_MAP_SWIZZLE_NONE))
    return fail(KQ_ERR_CUDA, "gemm_skinny: weight tensor map rejected");
  if (!encode_map(&ma, CU_TENSOR_MAP_DATA_TYPE_UINT8, act.qs, (uint64_t)K, (uint64_t)M, (uint64_t)K, 128, p.Mp,
                  CU_TENSOR_MAP_SWIZZLE_128B))
    return fail(KQ_ERR_CUDA, "gemm_skinny: activation tensor map rejected");
  if (!encode_map(&ms, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, act.ds, (uint64_t)nb * 2, (uint64_t)M, (uint64_t)nb * 8, 16,
                  p.Mp, CU_TENSOR_MAP_SWIZZLE_NONE))
    return fail(KQ_ERR_CUDA, "gemm_skinny: scale tensor map rejected");

  // warp grid: the fewest (row group, token group) tiles per warp, then the
  // fewest weight-fragment loads (row groups) per warp
  const int ntg = p.Mp / 8;
  int best = 1, best_cost = 1 << 30;
  for (int wtok : {1, 2, 4}) {
    const int wr = kComputeWarps / wtok;
    const int rpw = (gc + wr - 1) / wr, tpw = (ntg + wtok - 1) / wtok;
    const int cost = rpw * tpw * 64 + rpw;
    if (cost < best_cost) {
      best_cost = cost;
      best = wtok;
    }
  }
  // token groups per warp, rounded up to the instantiated sizes
  const int tpw = (ntg + best - 1) / best;
  const int tp = tpw <= 1 ? 1 : tpw <= 2 ? 2 : tpw <= 4 ? 4 : tpw <= 8 ? 8 : 16;
  // few token groups: split each chunk's blocks between two warps
  const int ks = (best == 1 && tp <= 2) ? 2 : 1;
  const int rpw_max = (kMaxGroups + kComputeWarps / best - 1) / (kComputeWarps / best);
  const size_t xbytes = ks == 2 ? (size_t)kComputeWarps * 32 * rpw_max * tp * 2 * 8 : 0;
  const size_t budget = 227 * 1024 - 1024 - 256 - xbytes;
  p.stages = (int)std::min<size_t>(4, budget / p.stage_bytes);
  if (p.stages < 2) return fail(KQ_ERR_UNSUPPORTED, "gemm_skinny: stage of %d bytes does not fit twice", p.stage_bytes);
  p.off_x = (p.stages * p.stage_bytes + 2 * p.stages * 8 + 15) & ~15;
  const size_t smem = (size_t)p.off_x + xbytes + 1024;
  switch (ks * 1000 + best * 100 + tp) {
    case 2101: return launch_cfg<WT, 1, 1, 2>(mw, ma, ms, p, grid, smem, s);
    case 2102: return launch_cfg<WT, 1, 2, 2>(mw, ma, ms, p, grid, smem, s);
    case 1104: return launch_cfg<WT, 1, 4, 1>(mw, ma, ms, p, grid, smem, s);
    case 1108: return launch_cfg<WT, 1, 8, 1>(mw, ma, ms, p, grid, smem, s);
    case 1116: return launch_cfg<WT, 1, 16, 1>(mw, ma, ms, p, grid, smem, s);
    case 1201: return launch_cfg<WT, 2, 1, 1>(mw, ma, ms, p, grid, smem, s);
    case 1202: return launch_cfg<WT, 2, 2, 1>(mw, ma, ms, p, grid, smem, s);
    case 1204: return launch_cfg<WT, 2, 4, 1>(mw, ma, ms, p, grid, smem, s);
    case 1208: return launch_cfg<WT, 2, 8, 1>(mw, ma, ms, p, grid, smem, s);
    case 1401: return launch_cfg<WT, 4, 1, 1>(mw, ma, ms, p, grid, smem, s);
    case 1402: return launch_cfg<WT, 4, 2, 1>(mw, ma, ms, p, grid, smem, s);
    case 1404: return launch_cfg<WT, 4, 4, 1>(mw, ma, ms, p, grid, smem, s);
    default: return fail(KQ_ERR_UNSUPPORTED, "gemm_skinny: no instantiation for %d token groups", ntg);
  }
}

}  // namespace

bool gemm_skinny_supported(int wtype, int M, int N, int K, const void* w, Act8 act) {
  return (wtype == KQ_Q4_0 || wtype == KQ_Q4_1 || wtype == KQ_Q8_0) && M > 8 && M <= kMaxTok && N >= 1 &&
         K >= kChunkK && K % kChunkK == 0 && (reinterpret_cast<uintptr_t>(w) & 15) == 0 &&
         (reinterpret_cast<uintptr_t>(act.qs) & 15) == 0 && (reinterpret_cast<uintptr_t>(act.ds) & 15) == 0;
}

kq_status_t launch_gemm_skinny(int wtype, const void* w, Act8 act, const OutSpec& out, int M, int N, int K,
                               cudaStream_t s, int* err) {
  switch (wtype) {
    case KQ_Q4_0: return launch_wt<KQ_Q4_0>(w, act, out, M, N, K, s, err);
    case KQ_Q4_1: return launch_wt<KQ_Q4_1>(w, act, out, M, N, K, s, err);
    case KQ_Q8_0: return launch_wt<KQ_Q8_0>(w, act, out, M, N, K, s, err);
    default: return fail(KQ_ERR_INVALID, "unknown weight type %d", wtype);
  }
}

}  // namespace kq
