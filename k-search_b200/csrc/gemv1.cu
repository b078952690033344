// Single-launch GEMV for one fp32 activation row over q4_0 / q4_1 / q8_0
// weight rows: out[n] = sum_b f(weight block (n, b), q8_1(x) block b). This
// is the W4A32C8 / W8A32C8 operator at M = 1 (the harness quant_gemm op,
// llm_kernel_test/op_test_handler.py:128-458, with the per-block formulas of
// vec_dot_q4_0_q8_1 and vec_dot_q8_0_q8_1, kernelevalplus-main/include/
// gemm_reference.h:276-336, and reference_q4_1_q8_1_gemm,
// llm_kernel_test/reference/gemm_ref.py:274-331).
//
// At M = 1 the operator is one HBM stream of the weights (9.4 MB at
// N = K = 4096), and its time is mostly fixed costs: a quantiser launch in
// front of the GEMV, and each CTA's wait for its first weight bytes. So this
// kernel
//  * requests the activation row, then starts every warp's first weight item
//    on its way (one bulk copy per item into the warp's shared-memory slot,
//    on the TMA engine, so the copies in flight do not hold up the
//    quantiser's shuffles and shared stores);
//  * quantises the activation row itself, once per CTA, into shared memory
//    while those copies are in flight (the quantiser kernels' octet step, so
//    codes and (d, s) pairs are bit-identical to theirs);
//  * then walks its rows with the next item's copies in flight while the
//    current item is computed (two shared-memory slots per warp).
// An item is the contiguous byte range a warp computes in one step: RPW
// whole rows when a row has at most 32 chunks (8 blocks of q4_0 / q4_1, 144 /
// 160 bytes; 4 blocks of q8_0, 136 bytes),
// else 32 chunks of one row. The LPR lanes of a row (a power of two <= 32)
// each take one chunk of it, read it from the warp's slot with 16-byte loads
// (lane stride 144 / 160 / 136 bytes: conflict-free), sum their blocks in order and
// reduce with an xor tree, so results are deterministic.
// Activation codes sit in shared memory as 16-byte pieces ordered
// [block-in-chunk j][half h][chunk c]: the LPR lanes of a row read chunks
// c .. c+LPR-1 at the same (j, h), i.e. consecutive 16-byte words (no bank
// conflicts), and lanes of the warp's other rows read the same words.
// Tasks are dealt to warps CTA-minor so every SM gets an equal share.
#include <algorithm>

#include "kq_internal.h"
#include "kq_device.cuh"
#include "kq_quant.cuh"

namespace kq {
namespace {

constexpr int kG1Threads = 512;
constexpr int kG1Warps = kG1Threads / 32;
constexpr int kG1MaxK = 32768;  // shared memory: K code bytes + 8 bytes per block + the warps' slots

template <int WT>
struct G1Traits;
// BB: bytes per block; CB: blocks per lane chunk (8 for the 4-bit formats,
// 144 / 160 bytes; 4 for q8_0, 136 bytes, so an item keeps the same size)
template <>
struct G1Traits<KQ_Q4_0> {
  static constexpr int BB = 18, CB = 8;
};
template <>
struct G1Traits<KQ_Q4_1> {
  static constexpr int BB = 20, CB = 8;
};
template <>
struct G1Traits<KQ_Q8_0> {
  static constexpr int BB = 34, CB = 4;
};

constexpr int kSlots = 2;  // weight slots per warp
template <int WT>
constexpr int kSlotBytes = 32 * G1Traits<WT>::CB * G1Traits<WT>::BB;  // one item: 32 chunks

// Item q of a warp's sequence: task T = gw + (q / cpl) * tw, iteration
// i = q % cpl. Its bytes are the contiguous range [start, start + len):
// rows [T * RPW, T * RPW + RPW) whole when cpl == 1, else chunks
// [32 i, 32 i + 32) of row T (then RPW = 1, LPR = 32). Lane (row-in-task
// rho = lane / LPR, sub = lane % LPR) computes chunk c = sub + 32 i of row
// r = T * RPW + rho, found at slot offset rho * rowbytes + sub * CB * BB.
// `last` marks the task's final item.
struct Item {
  size_t start;
  uint32_t len;
  int r;
  int c0;
  bool valid;
  bool last;
};

struct G1Geom {
  int N, C, lpr_log, cpl, gw, tw, sub;
  uint32_t rowbytes, chunkbytes;
  __device__ __forceinline__ Item item(int q, int lane) const {
    const int t = q / cpl, i = q - t * cpl;
    const int row0 = (gw + t * tw) << (5 - lpr_log);
    Item it;
    it.start = (size_t)row0 * rowbytes + (size_t)i * 32 * chunkbytes;
    if (cpl == 1) {
      it.len = (uint32_t)min(32 >> lpr_log, N - row0) * rowbytes;
    } else {
      it.len = (uint32_t)min(32, C - 32 * i) * chunkbytes;
    }
    it.r = row0 + (lane >> lpr_log);
    it.c0 = 32 * i;
    it.valid = it.r < N && sub + 32 * i < C;
    it.last = i == cpl - 1;
    return it;
  }
};

// Start an item's copy into a warp slot: one bulk copy (the TMA engine, not
// the load/store pipe the quantiser's shuffles and shared stores use) that
// completes on the slot's mbarrier. Called by one lane.
__device__ __forceinline__ void issue_item(uint8_t* slot, uint64_t* bar, const uint8_t* __restrict__ w,
                                           const Item& it, uint64_t pol) {
  mbar_arrive_expect_tx(bar, it.len);
  bulk_g2s_hint(slot, w + it.start, it.len, bar, pol);
}

// Blocks J .. CB - 1 of a chunk held in w[] against the activation pieces at
// aq (chunk c's column; piece (j, h) at aq + (2j + h) * c16) and the (d, s')
// pairs at ads[j * C].
template <int WT, int J, int NW>
__device__ __forceinline__ void chunk_dot(const uint32_t (&w)[NW], const uint8_t* aq, int c16, const float2* ads,
                                          int C, float& acc) {
  if constexpr (J < G1Traits<WT>::CB) {
    constexpr int OFF = J * G1Traits<WT>::BB;
    const uint4 alo = *reinterpret_cast<const uint4*>(aq + (2 * J) * c16);
    const uint4 ahi = *reinterpret_cast<const uint4*>(aq + (2 * J + 1) * c16);
    const float2 ds = ads[J * C];
    if constexpr (WT == KQ_Q8_0) {
      // d_w * d_a * sumi over the block's 32 int8 codes
      uint32_t q[8];
      gather_u32<OFF + 2>(w, q);
      int s0 = __dp4a((int)q[0], (int)alo.x, 0);
      int s1 = __dp4a((int)q[4], (int)ahi.x, 0);
      s0 = __dp4a((int)q[1], (int)alo.y, s0);
      s1 = __dp4a((int)q[5], (int)ahi.y, s1);
      s0 = __dp4a((int)q[2], (int)alo.z, s0);
      s1 = __dp4a((int)q[6], (int)ahi.z, s1);
      s0 = __dp4a((int)q[3], (int)alo.w, s0);
      s1 = __dp4a((int)q[7], (int)ahi.w, s1);
      const float dw = half_bits_to_float(get_u16<OFF>(w));
      acc = fmaf(dw * ds.x, (float)(s0 + s1), acc);
    } else {
    constexpr int QOFF = (WT == KQ_Q4_0) ? OFF + 2 : OFF + 4;
    uint32_t raw[4];
    gather_u32<QOFF>(w, raw);
    // two independent dp4a chains (low and high nibbles), exact int32 sums
    int sl = __dp4a((int)(raw[0] & 0x0F0F0F0Fu), (int)alo.x, 0);
    int sh = __dp4a((int)((raw[0] >> 4) & 0x0F0F0F0Fu), (int)ahi.x, 0);
    sl = __dp4a((int)(raw[1] & 0x0F0F0F0Fu), (int)alo.y, sl);
    sh = __dp4a((int)((raw[1] >> 4) & 0x0F0F0F0Fu), (int)ahi.y, sh);
    sl = __dp4a((int)(raw[2] & 0x0F0F0F0Fu), (int)alo.z, sl);
    sh = __dp4a((int)((raw[2] >> 4) & 0x0F0F0F0Fu), (int)ahi.z, sh);
    sl = __dp4a((int)(raw[3] & 0x0F0F0F0Fu), (int)alo.w, sl);
    sh = __dp4a((int)((raw[3] >> 4) & 0x0F0F0F0Fu), (int)ahi.w, sh);
    const int s = sl + sh;
    const float dw = half_bits_to_float(get_u16<OFF>(w));
    if constexpr (WT == KQ_Q4_0) {
      // d_w * (d_a * sumi - 8 * s_a); ds.y holds -8 * s_a
      acc = fmaf(dw, fmaf(ds.x, (float)s, ds.y), acc);
    } else {
      // d_w * d_a * sumi + m_w * s_a
      const float mw = half_bits_to_float(get_u16<OFF + 2>(w));
      acc = fmaf(dw * ds.x, (float)s, fmaf(mw, ds.y, acc));
    }
    }
    chunk_dot<WT, J + 1>(w, aq, c16, ads, C, acc);
  }
}

// One step of the activation quantisation: lane (grp, osub) of the warp loads
// values 4 osub .. 4 osub + 3 of blocks b0 + u * step + grp, u < 4.
__device__ __forceinline__ void load_x_step(float4 (&v)[4], const float* __restrict__ x, int b0, int nb, int step,
                                            int grp, int osub) {
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int blk = b0 + u * step + grp;
    v[u] = blk < nb ? __ldg(reinterpret_cast<const float4*>(x + (size_t)blk * 32) + osub)
                    : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  }
}

template <int WT>
__device__ __forceinline__ void compute_item(const uint8_t* slot, const Item& it, const G1Geom& g, int lane,
                                             const uint8_t* sq, const float2* sds, const OutSpec& out, float& acc) {
  constexpr int CBYTES = G1Traits<WT>::CB * G1Traits<WT>::BB;  // a lane's chunk (its stride in the slot)
  constexpr int NW = CBYTES / 4;
  if (it.valid) {
    const uint8_t* src = slot + (lane >> g.lpr_log) * g.rowbytes + g.sub * CBYTES;
    uint32_t w[NW];
    if constexpr (CBYTES % 16 == 0) {
#pragma unroll
      for (int i = 0; i < NW / 4; ++i) {
        const uint4 v = reinterpret_cast<const uint4*>(src)[i];
        w[4 * i] = v.x;
        w[4 * i + 1] = v.y;
        w[4 * i + 2] = v.z;
        w[4 * i + 3] = v.w;
      }
    } else {  // q8_0: 136-byte chunks, 8-byte aligned (lane stride 34 words: conflict-free 8-byte loads)
#pragma unroll
      for (int i = 0; i < NW / 2; ++i) {
        const uint2 v = reinterpret_cast<const uint2*>(src)[i];
        w[2 * i] = v.x;
        w[2 * i + 1] = v.y;
      }
    }
    const int c = it.c0 + g.sub;
    chunk_dot<WT, 0>(w, sq + c * 16, g.C * 16, sds + c, g.C, acc);
  }
  if (it.last) {  // warp-uniform: every lane is at the same item
    for (int o = (1 << g.lpr_log) >> 1; o >= 1; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (g.sub == 0 && it.r < g.N) {
      const size_t off = (size_t)out.col0 + it.r;
      out.ptr[0][off] = acc;
      for (int d = 1; d < out.n_out; ++d) out.ptr[d][off] = acc;
    }
    acc = 0.0f;
  }
}

template <int WT, int MODE>
__global__ void __launch_bounds__(kG1Threads, 1)
    gemv1_kernel(const uint8_t* __restrict__ w, const float* __restrict__ x, const __grid_constant__ OutSpec out,
                 int N, int K, int lpr_log, int* __restrict__ err) {
  constexpr int BB = G1Traits<WT>::BB;
  extern __shared__ __align__(16) uint8_t smem[];
  const int nb = K >> 5;
  constexpr int CB = G1Traits<WT>::CB;
  const int C = nb / CB;
  uint8_t* sq = smem;                                  // piece (j, h, c) at ((2j + h) * C + c) * 16
  float2* sds = reinterpret_cast<float2*>(smem + K);  // (d_a, s') of block CB c + j at j * C + c

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  G1Geom g;
  g.N = N;
  g.C = C;
  g.lpr_log = lpr_log;
  g.cpl = (C + (1 << lpr_log) - 1) >> lpr_log;
  g.gw = warp * gridDim.x + blockIdx.x;
  g.tw = gridDim.x * kG1Warps;
  g.sub = lane & ((1 << lpr_log) - 1);
  g.chunkbytes = CB * BB;
  g.rowbytes = (uint32_t)nb * BB;
  const int tasks = (N + (32 >> lpr_log) - 1) / (32 >> lpr_log);
  const int nitems = (g.gw < tasks ? (tasks - 1 - g.gw) / g.tw + 1 : 0) * g.cpl;
  const uint64_t pol = policy_evict_first();
  uint8_t* slots = smem + K + nb * sizeof(float2) + warp * (kSlots * kSlotBytes<WT>);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + K + nb * sizeof(float2) + kG1Warps * kSlots * kSlotBytes<WT>) +
                   warp * kSlots;
  if (lane == 0) {
    for (int i = 0; i < kSlots; ++i) mbar_init(&bars[i], 1);
    fence_mbar_init();
  }
  __syncwarp();
  // Launched as a programmatic dependent: the set-up above overlaps the
  // preceding kernel, and nothing in global memory is read before that
  // kernel has completed (its output may be this call's row or weights).
  // The next kernel may be scheduled now; it waits for this one likewise.
  pdl_wait();
  pdl_launch_dependents();

  // ---- q8_1 of the activation row into shared memory ----
  // The row's first values are requested before any weight byte: behind the
  // weight stream they would wait for most of it at DRAM.
  const int grp = lane >> 3, osub = lane & 7;
  constexpr int kStep = kG1Warps * 4;  // blocks per warp-wide step of the CTA
  float4 v[4];
  load_x_step(v, x, warp * 4, nb, kStep, grp, osub);
  // the first item's bytes are on their way during the quantisation
  if (lane == 0 && nitems > 0) issue_item(slots, &bars[0], w, g.item(0, lane), pol);
  for (int b0 = warp * 4; b0 < nb; b0 += 4 * kStep) {
    if (b0 != warp * 4) load_x_step(v, x, b0, nb, kStep, grp, osub);
    BlockQ r[4];
    // steps past the row's end are skipped (warp-uniform: nb % 8 == 0)
    if (b0 + kStep >= nb) {
      quantize_octets<MODE, 1>(reinterpret_cast<const float4(&)[1]>(v), lane, reinterpret_cast<BlockQ(&)[1]>(r));
    } else if (b0 + 2 * kStep >= nb) {
      quantize_octets<MODE, 2>(reinterpret_cast<const float4(&)[2]>(v), lane, reinterpret_cast<BlockQ(&)[2]>(r));
    } else {
      quantize_octets<MODE, 4>(v, lane, r);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int blk = b0 + u * kStep + grp;
      if (blk < nb) {
        const int c = blk / CB, j = blk % CB, h = osub >> 2;
        *reinterpret_cast<uint32_t*>(sq + ((2 * j + h) * C + c) * 16 + (osub & 3) * 4) = r[u].qs;
        if (osub == 0) {
          float2 ds = staging_ds<MODE>(r[u]);
          if (WT == KQ_Q4_0) ds.y = -8.0f * ds.y;
          sds[j * C + c] = ds;
        }
      }
    }
  }
  __syncthreads();

  // ---- dot products: item q + 1's copy in flight while item q is computed ----
  float acc = 0.0f;
  bool dead = false;
  for (int q = 0; q < nitems; ++q) {
    // slot (q + 1) % kSlots was last read for item q - 1: every lane fenced
    // its reads and passed the __syncwarp below before this refill
    if (lane == 0 && q + 1 < nitems)
      issue_item(slots + ((q + 1) % kSlots) * kSlotBytes<WT>, &bars[(q + 1) % kSlots], w, g.item(q + 1, lane), pol);
    mbar_wait_or_poison(&bars[q % kSlots], (q / kSlots) & 1, err, DEV_TIMEOUT_FULL, dead);
    compute_item<WT>(slots + (q % kSlots) * kSlotBytes<WT>, g.item(q, lane), g, lane, sq, sds, out, acc);
    fence_proxy_async_smem();  // generic reads of the slot, before a bulk copy refills it
    __syncwarp();
  }
  if (out.n_out > 1) __threadfence_system();  // peer stores visible before the host-side barrier
}

template <int WT, int MODE>
kq_status_t launch_mode(const void* w, const float* x, const OutSpec& out, int N, int K, cudaStream_t s, int* err) {
  auto kern = gemv1_kernel<WT, MODE>;
  const int smem = K + (K / 32) * (int)sizeof(float2) + kG1Warps * kSlots * (kSlotBytes<WT> + (int)sizeof(uint64_t));
  if (kq_status_t st = ensure_dynamic_smem(reinterpret_cast<const void*>(kern), smem, "gemv1 smem attribute"))
    return st;
  const int C = K / (32 * G1Traits<WT>::CB);
  int lpr_log = 0;
  while ((1 << lpr_log) < C && lpr_log < 5) ++lpr_log;
  const int rpw = 32 >> lpr_log;
  const int tasks = (N + rpw - 1) / rpw;
  const int grid = std::max(1, std::min(sm_count(), tasks));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kG1Threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, static_cast<const uint8_t*>(w), x, out, N, K, lpr_log,
                                     err ? err : device_error_word());
  if (e != cudaSuccess) return check_cuda(e, "gemv1 launch");
  return check_launch("gemv1");
}

template <int WT>
kq_status_t launch_wt(const void* w, const float* x, const OutSpec& out, int N, int K, int mode, cudaStream_t s,
                      int* err) {
  switch (mode) {
    case KQ_ACT_SUM_X: return launch_mode<WT, KQ_ACT_SUM_X>(w, x, out, N, K, s, err);
    case KQ_ACT_SUM_DQ: return launch_mode<WT, KQ_ACT_SUM_DQ>(w, x, out, N, K, s, err);
    case KQ_ACT_F32: return launch_mode<WT, KQ_ACT_F32>(w, x, out, N, K, s, err);
    default: return fail(KQ_ERR_INVALID, "unknown activation mode %d", mode);
  }
}

}  // namespace

bool gemv1_supported(int wtype, int M, int N, int K, const void* w, const float* x) {
  return M == 1 && (wtype == KQ_Q4_0 || wtype == KQ_Q4_1 || wtype == KQ_Q8_0) && N >= 1 && K >= 256 && K % 256 == 0 && K <= kG1MaxK &&
         reinterpret_cast<uintptr_t>(w) % 16 == 0 && reinterpret_cast<uintptr_t>(x) % 16 == 0;
}

kq_status_t launch_gemv1(int wtype, const void* w, const float* x, const OutSpec& out, int N, int K, int mode,
                         cudaStream_t s, int* err) {
  switch (wtype) {
    case KQ_Q4_0: return launch_wt<KQ_Q4_0>(w, x, out, N, K, mode, s, err);
    case KQ_Q4_1: return launch_wt<KQ_Q4_1>(w, x, out, N, K, mode, s, err);
    case KQ_Q8_0: return launch_wt<KQ_Q8_0>(w, x, out, N, K, mode, s, err);
    default: return fail(KQ_ERR_INVALID, "gemv1: unknown weight type %d", wtype);
  }
}

}  // namespace kq
