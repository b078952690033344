// Decode GEMV: out[m, n] = sum_b f(weight block (n, b), activation block (m, b))
// for M <= 8 activation rows (llama.cpp's mul_mat_vec_q family; the
// per-block formulas are vec_dot_q4_0_q8_1 / vec_dot_q8_0_q8_1 in
// kernelevalplus-main/include/gemm_reference.h:276-336 and
// reference_q4_1_q8_1_gemm in llm_kernel_test/reference/gemm_ref.py:274-331).
//
// HBM-streaming design (B200):
//  * Persistent grid, one CTA per SM, each CTA owns a contiguous range of
//    weight rows. A producer warp streams the raw AoS rows (18/20/34-byte
//    blocks, unchanged layout) into a 4-deep shared-memory ring with
//    cp.async.bulk (no register staging, L2 evict-first), one bulk copy per
//    row slice, completion tracked by mbarrier transaction counts.
//  * 8 consumer warps read their lanes' block runs from shared memory with
//    the widest aligned vector loads the block size allows (conflict-free:
//    a lane's run is BPL consecutive blocks, so lane strides are 72/36/80/40/
//    136/68 bytes), unpack nibbles, run dp4a against the int8 activation codes
//    held in registers, and apply the per-block fp32 scale epilogue.
//  * Per-lane partial sums are reduced with a transpose-halving warp
//    reduction (V values in 31 + V/32 shuffles per lane instead of 5V), then
//    across the K-split warps through shared memory.
//  * The kernel is launched as a programmatic dependent of the activation
//    quantiser: weight streaming starts before the activations exist;
//    consumers call griddepcontrol.wait before touching them.
#include <algorithm>

#include "kq_internal.h"
#include "kq_device.cuh"

namespace kq {
namespace {

constexpr int kConsumerWarps = 8;
constexpr int kStages = 4;

template <int WT>
struct WTraits;
template <>
struct WTraits<KQ_Q4_0> {
  static constexpr int BB = 18;
};
template <>
struct WTraits<KQ_Q4_1> {
  static constexpr int BB = 20;
};
template <>
struct WTraits<KQ_Q8_0> {
  static constexpr int BB = 34;
};

// Load CB bytes starting at shared address p into w[] (normalised so that
// w[0] holds bytes 0..3 of the run). The run's alignment is the largest power
// of two dividing CB (runs start at multiples of CB from a 16-aligned base).
template <int CB>
struct Chunk {
  static constexpr int NW = (CB + 3) / 4 + 1;
  uint32_t w[NW];
  __device__ __forceinline__ void load(const uint8_t* p) {
    if constexpr (CB % 16 == 0) {
#pragma unroll
      for (int i = 0; i < CB / 16; ++i) {
        const uint4 v = reinterpret_cast<const uint4*>(p)[i];
        w[4 * i] = v.x; w[4 * i + 1] = v.y; w[4 * i + 2] = v.z; w[4 * i + 3] = v.w;
      }
    } else if constexpr (CB % 8 == 0) {
#pragma unroll
      for (int i = 0; i < CB / 8; ++i) {
        const uint2 v = reinterpret_cast<const uint2*>(p)[i];
        w[2 * i] = v.x; w[2 * i + 1] = v.y;
      }
    } else if constexpr (CB % 4 == 0) {
#pragma unroll
      for (int i = 0; i < CB / 4; ++i) w[i] = reinterpret_cast<const uint32_t*>(p)[i];
    } else {
      // 2-byte aligned run: read the covering aligned words, shift by 16 if needed.
      const uint32_t* q = reinterpret_cast<const uint32_t*>(reinterpret_cast<uintptr_t>(p) & ~(uintptr_t)3);
      const uint32_t sh = (reinterpret_cast<uintptr_t>(p) & 2) ? 16u : 0u;
      uint32_t raw[NW];
#pragma unroll
      for (int i = 0; i < NW; ++i) raw[i] = q[i];
#pragma unroll
      for (int i = 0; i < NW - 1; ++i) w[i] = __funnelshift_r(raw[i], raw[i + 1], sh);
      w[NW - 1] = 0;
    }
  }
};

// Per-block dot product and scale epilogue for one weight block (fields at
// byte offset OFF of the lane's run) against MR activation blocks.
template <int WT, int OFF, int MR, int NW>
__device__ __forceinline__ void block_dot(const uint32_t (&w)[NW], const uint32_t (&aq)[MR][8],
                                          const float (&ad)[MR], const float (&as)[MR], float (&acc)[MR],
                                          int mvalid) {
  const float dw = half_bits_to_float(get_u16<OFF>(w));
  if constexpr (WT == KQ_Q8_0) {
    uint32_t q[8];
    gather_u32<OFF + 2>(w, q);
#pragma unroll
    for (int m = 0; m < MR; ++m) {
      if (m < mvalid) {
        int s = 0;
#pragma unroll
        for (int k = 0; k < 8; ++k) s = __dp4a((int)q[k], (int)aq[m][k], s);
        acc[m] = fmaf(dw * ad[m], (float)s, acc[m]);
      }
    }
  } else {
    constexpr int QOFF = (WT == KQ_Q4_0) ? OFF + 2 : OFF + 4;
    uint32_t raw[4], lo[4], hi[4];
    gather_u32<QOFF>(w, raw);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      lo[k] = raw[k] & 0x0F0F0F0Fu;
      hi[k] = (raw[k] >> 4) & 0x0F0F0F0Fu;
    }
    float mw = 0.0f;
    if constexpr (WT == KQ_Q4_1) mw = half_bits_to_float(get_u16<OFF + 2>(w));
#pragma unroll
    for (int m = 0; m < MR; ++m) {
      if (m < mvalid) {
        int s = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          s = __dp4a((int)lo[k], (int)aq[m][k], s);
          s = __dp4a((int)hi[k], (int)aq[m][k + 4], s);
        }
        if constexpr (WT == KQ_Q4_0) {
          // d_w * (d_a * sumi - 8 * s_a); as[] holds -8 * s_a.
          acc[m] = fmaf(dw, fmaf(ad[m], (float)s, as[m]), acc[m]);
        } else {
          // d_w * d_a * sumi + m_w * s_a
          acc[m] = fmaf(dw * ad[m], (float)s, fmaf(mw, as[m], acc[m]));
        }
      }
    }
  }
}

template <int WT, int OFF, int J, int BPL, int MR, int NW>
__device__ __forceinline__ void run_blocks(const uint32_t (&w)[NW], const uint32_t (&aq)[BPL][MR][8],
                                           const float (&ad)[BPL][MR], const float (&as)[BPL][MR], float (&acc)[MR],
                                           int mvalid, int jvalid) {
  if constexpr (J < BPL) {
    if (J < jvalid) block_dot<WT, OFF + J * WTraits<WT>::BB, MR>(w, aq[J], ad[J], as[J], acc, mvalid);
    run_blocks<WT, OFF, J + 1, BPL, MR>(w, aq, ad, as, acc, mvalid, jvalid);
  }
}

// Transpose-halving reduction of V (power of two) per-lane values across the
// warp. Afterwards lane l holds the sums of indices [l*C, l*C + C) for V >= 32
// (C = V/32); for V < 32 lanes l with (l & (32/V - 1)) == 0 hold index
// l / (32/V) (C = 1).
template <int V>
__device__ __forceinline__ void warp_transpose_reduce(float (&v)[V], int lane) {
  int c = V;
#pragma unroll
  for (int mask = 16; mask >= 1; mask >>= 1) {
    if (c >= 2) {
      const int half = c / 2;
      const bool upper = (lane & mask) != 0;
#pragma unroll
      for (int i = 0; i < V / 2; ++i) {
        if (i < half) {
          const float send = upper ? v[i] : v[i + half];
          const float keep = upper ? v[i + half] : v[i];
          v[i] = keep + __shfl_xor_sync(0xffffffffu, send, mask);
        }
      }
      c = half;
    } else {
      v[0] += __shfl_xor_sync(0xffffffffu, v[0], mask);
    }
  }
}

template <int WT, int MR, int BPL, int KW, int SR>
struct GemvCfg {
  static constexpr int BB = WTraits<WT>::BB;
  static constexpr int RG = kConsumerWarps / KW;       // row groups
  static constexpr int RPW = (SR + RG - 1) / RG;        // rows per warp per stage
  static constexpr int KS = KW * 32 * BPL;              // blocks per stage (K slice)
  static constexpr int SB = ((SR * KS * BB + 16) + 127) / 128 * 128;  // stage bytes (+ over-read pad)
  static constexpr int V = RPW * MR;                    // partials per lane
  static constexpr int VPOW = V <= 1 ? 1 : V <= 2 ? 2 : V <= 4 ? 4 : V <= 8 ? 8 : V <= 16 ? 16 : V <= 32 ? 32 : 64;
  static constexpr int RED_FLOATS = 2 * RG * KW * VPOW;  // cross-warp reduction buffer
  static constexpr size_t SMEM = (size_t)kStages * SB + RED_FLOATS * sizeof(float) + 2 * kStages * sizeof(uint64_t);
  static_assert(RG * KW == kConsumerWarps, "warp split");
  static_assert(KS % 8 == 0, "K slice must keep 16-byte alignment");
};

// one output element to every destination of the epilogue
__device__ __forceinline__ void put_out(const OutSpec& o, int m, int n, float v) {
  const size_t off = (size_t)m * o.ld + o.col0 + n;
  o.ptr[0][off] = v;
  for (int d = 1; d < o.n_out; ++d) o.ptr[d][off] = v;
}

template <int WT, int MR, int BPL, int KW, int SR>
__global__ void __launch_bounds__(32 * (kConsumerWarps + 1), 1)
    gemv_kernel(const uint8_t* __restrict__ w, const int8_t* __restrict__ aqs, const float2* __restrict__ ads,
                const __grid_constant__ OutSpec out, int M, int N, int K, int* __restrict__ err) {
  using C = GemvCfg<WT, MR, BPL, KW, SR>;
  constexpr int BB = C::BB;
  extern __shared__ __align__(128) uint8_t smem[];
  float* red = reinterpret_cast<float*>(smem + kStages * C::SB);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * C::SB + C::RED_FLOATS * sizeof(float));
  uint64_t* empty = full + kStages;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nb = K / 32;
  const size_t rowbytes = (size_t)nb * BB;
  const int nits = (nb + C::KS - 1) / C::KS;
  const int n_begin = (int)(((long long)N * blockIdx.x) / gridDim.x);
  const int n_end = (int)(((long long)N * (blockIdx.x + 1)) / gridDim.x);
  const int nrb = (n_end - n_begin + SR - 1) / SR;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    // ---------------- producer ----------------
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      bool dead = false;
      int sidx = 0;
      for (int rb = 0; rb < nrb; ++rb) {
        const int n0 = n_begin + rb * SR;
        const int rows = min(SR, n_end - n0);
        for (int it = 0; it < nits; ++it, ++sidx) {
          const int slot = sidx % kStages;
          const int fill = sidx / kStages;
          if (fill > 0) mbar_wait_or_poison(&empty[slot], (fill - 1) & 1, err, DEV_TIMEOUT_EMPTY, dead);
          if (dead) continue;  // consumers will time out on `full` and finish
          const int ks = min(C::KS, nb - it * C::KS);
          const uint32_t pitch = (uint32_t)ks * BB;
          mbar_arrive_expect_tx(&full[slot], pitch * rows);
          uint8_t* dst = smem + slot * C::SB;
          const uint8_t* src = w + (size_t)n0 * rowbytes + (size_t)it * C::KS * BB;
          if (nits == 1) {
            // whole rows: the stage is one contiguous byte range
            bulk_g2s_hint(dst, src, pitch * rows, &full[slot], pol);
          } else {
            for (int r = 0; r < rows; ++r) bulk_g2s_hint(dst + r * pitch, src + r * rowbytes, pitch, &full[slot], pol);
          }
        }
      }
      // Drain: every filled slot must be released by the consumers (who
      // wait for its bytes to land) before the CTA may exit.
      for (int s = max(0, sidx - kStages); s < sidx; ++s)
        mbar_wait_or_poison(&empty[s % kStages], (s / kStages) & 1, err, DEV_TIMEOUT_EMPTY, dead);
    }
    return;
  }

  // ---------------- consumers ----------------
  const int kw = warp % KW;
  const int rg = warp / KW;
  const int mvalid = min(M, MR);
  pdl_wait();  // activations come from the preceding kernel

  uint32_t aq[BPL][MR][8];
  float ad[BPL][MR], as[BPL][MR];
  int loaded_it = -1;
  int jvalid = 0;
  bool dead = false;

  int sidx = 0;
  for (int rb = 0; rb < nrb; ++rb) {
    const int n0 = n_begin + rb * SR;
    const int rows = min(SR, n_end - n0);
    float part[C::VPOW];
#pragma unroll
    for (int i = 0; i < C::VPOW; ++i) part[i] = 0.0f;

    for (int it = 0; it < nits; ++it, ++sidx) {
      const int slot = sidx % kStages;
      const int ks = min(C::KS, nb - it * C::KS);
      const int blk0 = kw * 32 * BPL + lane * BPL;  // first block of this lane in the slice
      if (it != loaded_it) {
        jvalid = max(0, min(BPL, ks - blk0));
#pragma unroll
        for (int j = 0; j < BPL; ++j) {
#pragma unroll
          for (int m = 0; m < MR; ++m) {
            if (j < jvalid && m < mvalid) {
              const int b = it * C::KS + blk0 + j;
              const uint4* src = reinterpret_cast<const uint4*>(aqs + (size_t)m * K + (size_t)b * 32);
              const uint4 v0 = __ldg(src), v1 = __ldg(src + 1);
              aq[j][m][0] = v0.x; aq[j][m][1] = v0.y; aq[j][m][2] = v0.z; aq[j][m][3] = v0.w;
              aq[j][m][4] = v1.x; aq[j][m][5] = v1.y; aq[j][m][6] = v1.z; aq[j][m][7] = v1.w;
              const float2 dsv = __ldg(ads + (size_t)m * nb + b);
              ad[j][m] = dsv.x;
              as[j][m] = (WT == KQ_Q4_0) ? -8.0f * dsv.y : dsv.y;
            } else {
#pragma unroll
              for (int k = 0; k < 8; ++k) aq[j][m][k] = 0;
              ad[j][m] = 0.0f;
              as[j][m] = 0.0f;
            }
          }
        }
        loaded_it = (nits == 1) ? it : -1;
      }

      mbar_wait_or_poison(&full[slot], (sidx / kStages) & 1, err, DEV_TIMEOUT_FULL, dead);
      const uint8_t* stage = smem + slot * C::SB;
      const uint32_t pitch = (uint32_t)ks * BB;
#pragma unroll
      for (int rr = 0; rr < C::RPW; ++rr) {
        const int r = rg + rr * C::RG;
        if (r < rows && jvalid > 0) {
          Chunk<BPL * BB> ch;
          ch.load(stage + r * pitch + blk0 * BB);
          float acc[MR];
#pragma unroll
          for (int m = 0; m < MR; ++m) acc[m] = 0.0f;
          run_blocks<WT, 0, 0, BPL, MR>(ch.w, aq, ad, as, acc, mvalid, jvalid);
#pragma unroll
          for (int m = 0; m < MR; ++m) part[rr * MR + m] += acc[m];
        }
      }
      fence_proxy_async_smem();  // generic reads of the bulk-copy-refilled stage, before its release
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
    }

    // ---- reduce and write this row block ----
    warp_transpose_reduce<C::VPOW>(part, lane);
    constexpr int CNT = C::VPOW >= 32 ? C::VPOW / 32 : 1;
    constexpr int STRIDE = C::VPOW >= 32 ? 1 : 32 / C::VPOW;  // lanes per index when V < 32
    const bool holder = (lane % STRIDE) == 0;
    const int idx0 = C::VPOW >= 32 ? lane * CNT : lane / STRIDE;
    if constexpr (KW == 1) {
      if (holder) {
#pragma unroll
        for (int c = 0; c < CNT; ++c) {
          const int idx = idx0 + c;
          const int rr = idx / MR, m = idx % MR;
          const int r = rg + rr * C::RG;
          if (idx < C::V && r < rows && m < mvalid) put_out(out, m, n0 + r, part[c]);
        }
      }
    } else {
      float* rbuf = red + (rb & 1) * (C::RG * KW * C::VPOW) + rg * (KW * C::VPOW);
      if (holder) {
#pragma unroll
        for (int c = 0; c < CNT; ++c) rbuf[kw * C::VPOW + idx0 + c] = part[c];
      }
      named_bar_sync(1 + rg, KW * 32);
      if (kw == 0) {
        for (int idx = lane; idx < C::V; idx += 32) {
          float s = 0.0f;
#pragma unroll
          for (int q = 0; q < KW; ++q) s += rbuf[q * C::VPOW + idx];
          const int rr = idx / MR, m = idx % MR;
          const int r = rg + rr * C::RG;
          if (r < rows && m < mvalid) put_out(out, m, n0 + r, s);
        }
      }
    }
  }
  if (out.n_out > 1) __threadfence_system();  // peer stores visible before the host-side barrier
}

template <int WT, int MR, int BPL, int KW, int SR>
kq_status_t launch_cfg(const void* w, Act8 act, const OutSpec& out, int M, int N, int K, bool pdl, cudaStream_t s,
                       int* err, int per_sm = 1) {
  using C = GemvCfg<WT, MR, BPL, KW, SR>;
  auto kern = gemv_kernel<WT, MR, BPL, KW, SR>;
  if (kq_status_t st = ensure_dynamic_smem(reinterpret_cast<const void*>(kern), (int)C::SMEM, "gemv smem attribute"))
    return st;
  const int grid = std::max(1, std::min(per_sm * sm_count(), (N + SR - 1) / SR));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(32 * (kConsumerWarps + 1));
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, static_cast<const uint8_t*>(w), (const int8_t*)act.qs,
                                     (const float2*)act.ds, out, M, N, K, err ? err : device_error_word());
  if (e != cudaSuccess) return check_cuda(e, "gemv launch");
  return check_launch("gemv");
}

template <int WT>
kq_status_t launch_wt(const void* w, Act8 act, const OutSpec& out, int M, int N, int K, bool pdl, cudaStream_t s,
                      int* err) {
  constexpr int SR = (WT == KQ_Q8_0) ? 8 : 16;
  if (M <= 1) {
    // Many 4-bit rows: two CTAs per SM with 8-row stages (twice the consumer
    // warps, half the wait for a stage's first byte): 10.5 -> 9.4 us at
    // N = 14336, K = 4096; at N = 4096 the single-CTA form is faster.
    if (WT != KQ_Q8_0 && N >= 8192) return launch_cfg<WT, 1, 4, 1, SR / 2>(w, act, out, M, N, K, pdl, s, err, 2);
    return launch_cfg<WT, 1, 4, 1, SR>(w, act, out, M, N, K, pdl, s, err);
  }
  if (M <= 2) return launch_cfg<WT, 2, 4, 1, SR>(w, act, out, M, N, K, pdl, s, err);
  if (M <= 4) return launch_cfg<WT, 4, 2, 2, SR>(w, act, out, M, N, K, pdl, s, err);
  return launch_cfg<WT, 8, 1, 4, SR>(w, act, out, M, N, K, pdl, s, err);
}

}  // namespace

bool gemv_supported(int wtype, int M, int N, int K) {
  (void)wtype;
  return M >= 1 && M <= 8 && N >= 1 && K >= 256 && K % 256 == 0;
}

kq_status_t launch_gemv(int wtype, const void* w, Act8 act, float* out, int M, int N, int K, bool pdl,
                        cudaStream_t s, int* err) {
  return launch_gemv(wtype, w, act, OutSpec::plain(out, N), M, N, K, pdl, s, err);
}

kq_status_t launch_gemv(int wtype, const void* w, Act8 act, const OutSpec& out, int M, int N, int K, bool pdl,
                        cudaStream_t s, int* err) {
  if (reinterpret_cast<uintptr_t>(w) % 16 != 0) return fail(KQ_ERR_INVALID, "gemv: weight pointer must be 16-byte aligned");
  switch (wtype) {
    case KQ_Q4_0: return launch_wt<KQ_Q4_0>(w, act, out, M, N, K, pdl, s, err);
    case KQ_Q4_1: return launch_wt<KQ_Q4_1>(w, act, out, M, N, K, pdl, s, err);
    case KQ_Q8_0: return launch_wt<KQ_Q8_0>(w, act, out, M, N, K, pdl, s, err);
    default: return fail(KQ_ERR_INVALID, "unknown weight type %d", wtype);
  }
}

}  // namespace kq
