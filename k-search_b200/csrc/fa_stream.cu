// Flash-attention decode over a q8_0 KV cache on the tensor pipe, with a
// persistent, balanced ("stream") schedule. The default kernel for head_dim
// 128 and KV heads in groups of 8 with at most 4 queries per KV head: the
// ragged GQA decode and the harness MHA form.
//
// Semantics: the harness flash_attention operator
// (kernelevalplus-main/llm_kernel_test/op_test_handler.py:543-563):
// out = softmax(q . K^T / sqrt(D)) . V per (query, head), with K and V stored
// as q8_0 blocks along head_dim (op_test_handler.py:489-508), dequantised as
// x = q * d. In the ragged form sequence b owns cache rows cu[b] .. cu[b+1]-1
// and query head h reads KV head h / (Hq / Hkv).
//
// Work: an "item" is (sequence or query group, group of 8 KV heads); its
// tokens are cut into 16-token tiles, and the tiles of all items form one
// ordered list that the grid (two CTAs per SM) splits into equal contiguous
// ranges, so every SM streams the same number of KV bytes whatever the
// sequence lengths. A CTA's range crosses items; at each item boundary its
// warps write their online-softmax state as a partial (slot = CTA + item,
// unique because ranges are contiguous), and the combine kernel merges the
// partials of each query.
//
// CTA (two per SM): warp 0's lane 0 streams K and V tiles by TMA (16 token
// rows x 8 heads, the cache's own 1088-byte rows, landing at a 1104-byte
// pitch so that fragment loads from different rows fall in different banks)
// into a two-stage ring, refilling a stage once all warps released it; 8 compute warps each own one KV head and its (up to 4)
// queries:
//   QK  mma.m16n8k32 s8: A = the raw K codes of 16 tokens x one 32-dim block
//       (all 16 rows used), B = the queries as two int8 levels
//       (q ~ s1 q1 + s2 q2, s2 = s1 / 127; the columns are query x level), so
//       127 dot1 + dot2 is the exact int32 block dot at scale s2; the fp32
//       epilogue applies the per-(token, block) K scale.
//   PV  mma.m16n8k16 f16: A = V^T (16 dims x 16 tokens) read with
//       ldmatrix.trans from a per-warp fp16 copy of the tile's V codes (exact
//       small integers), B = p * d_v (16 tokens x 4 queries) per 32-dim block
//       as fp16 in columns 0-3 and its fp16 rounding remainder in columns 4-7,
//       fp32 accumulation. 8 MMAs per tile cover 128 dims.
// The running maximum moves only when a tile exceeds it (the accumulator is
// rescaled then), so p <= 1 and p * d_v stays inside the fp16 range.
#include <cuda.h>

#include <algorithm>
#include <atomic>
#include <cmath>

#include "kq_internal.h"
#include "kq_device.cuh"

namespace kq {
namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

constexpr int kTok = 16;                    // tokens per tile
constexpr int kHeads = 8;                   // KV heads per item (one compute warp each)
constexpr int kQ = 4;                       // queries per KV head per item (at most)
constexpr int kStages = 2;
constexpr int kHeadBytes = 136;             // one head's row: 4 q8_0 blocks of 34 B
constexpr int kBoxU64 = 138;                // TMA box width in 8-byte units: 1088 B of row + 16 B
constexpr int kPitch = kBoxU64 * 8;         // 1104: smem row pitch (276 words = 20 mod 32 banks)
constexpr int kTile = kTok * kPitch;        // 17664 bytes per K (or V) tile
// 8 warps, no separate producer warp: two CTAs per SM then fit the register
// file of each SM sub-partition (a 9-warp CTA puts 3 warps on one, and two of
// those at 112 registers do not fit), doubling the warps that hide the
// per-tile latency chain. Warp 0's lane 0 issues the TMA loads.
constexpr int kThreads = 32 * kHeads;
constexpr int kMaxSeq = 512;                // ragged sequences the schedule table holds
constexpr int kVhPitch = 272;               // fp16 V tile row: 256 B + 16 (ldmatrix rows in distinct banks)

constexpr int kOffV = kStages * kTile;
constexpr int kOffVh = 2 * kStages * kTile;               // fp16 V tiles: [warp][16 tokens][kVhPitch]
constexpr int kOffP = kOffVh + kHeads * kTok * kVhPitch;  // p transposition: [warp][4 queries][16 tokens] fp32
constexpr int kOffD = kOffP + kHeads * kQ * kTok * 4;     // scales: [warp][32] float4 (dk tokens 0-15, dv 0-15)
constexpr int kOffT = kOffD + kHeads * 32 * 16;           // schedule prefix table (kMaxSeq + 1 ints)
constexpr int kOffBar = kOffT + ((kMaxSeq + 1) * 4 + 15) / 16 * 16;
constexpr size_t kSmem = kOffBar + 4 * kStages * 8 + 128; // + base alignment slack
static_assert(kOffV % 128 == 0 && kOffVh % 128 == 0 && kTile % 128 == 0, "TMA destinations stay 128-byte aligned");

struct StreamParams {
  const void* q;          // ragged: fp16 [B, Hq, 128]; MHA: fp32 [B, H, 128]
  const int32_t* cu;      // ragged: cu_seqlens [B + 1]; MHA: nullptr
  int* tprefix;           // [nseq + 1] tile prefix written by CTA 0 for the combine (ragged)
  float* pm;              // [slot][8 heads][4 queries]
  float* pl;
  float* pacc;            // [slot][8][4][128]
  void* out;
  int* err;
  int nseq;               // ragged: B; MHA: query groups ceil(B / 4)
  int B, H, Hkv;          // batch, query heads, KV heads
  int S;                  // MHA: cache length (every item)
  int n_hg;               // Hkv / 8
  float qscale;           // softmax scale * log2(e)
};

// The tile list: item (b, hg) holds nt(b) = ceil(L_b / 16) tiles; items are
// ordered by b then hg; tprefix(b) = sum of nt over sequences before b.
struct Sched {
  const int* T;  // smem prefix (ragged) or nullptr (uniform nt)
  int nt_uni;
  int nseq;
  int n_hg;
  __device__ __forceinline__ int pre(int b) const { return T ? T[b] : b * nt_uni; }
  __device__ __forceinline__ int nt(int b) const { return pre(b + 1) - pre(b); }
  __device__ __forceinline__ long long total() const { return (long long)n_hg * pre(nseq); }
  // position of global tile t (< total()): sequence, head group, tile within the item
  __device__ void locate(long long t, int& b, int& hg, int& j) const {
    int lo = 0, hi = nseq - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if ((long long)n_hg * pre(mid) <= t) lo = mid;
      else hi = mid - 1;
    }
    b = lo;
    const long long local = t - (long long)n_hg * pre(b);
    const int n = nt(b);
    hg = (int)(local / n);
    j = (int)(local % n);
  }
  __device__ __forceinline__ void next(int& b, int& hg, int& j) const {
    if (++j < nt(b)) return;
    j = 0;
    if (++hg < n_hg) return;
    hg = 0;
    do {
      ++b;
    } while (b < nseq && nt(b) == 0);
  }
};

// CTA whose contiguous range [TT i / G, TT (i+1) / G) holds tile t
__host__ __device__ __forceinline__ int owner_of(long long t, long long TT, int G) {
  return (int)(((t + 1) * (long long)G - 1) / TT);
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// 32-bit word at a 2-byte aligned shared address
__device__ __forceinline__ uint32_t lds_u32_a2(const uint8_t* b) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(b);
  const uint32_t* q = reinterpret_cast<const uint32_t*>(a & ~(uintptr_t)3);
  return __funnelshift_r(q[0], q[1], (a & 2) ? 16u : 0u);
}

__device__ __forceinline__ float lds_half(const uint8_t* b) {
  return __half2float(__ushort_as_half(*reinterpret_cast<const uint16_t*>(b)));
}

__device__ __forceinline__ void mma_s8_16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%10, %10, %10, %10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

__device__ __forceinline__ void mma_f16_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], uint32_t saddr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(saddr));
}

// 2^x by the hardware approximation (ex2.approx: relative error ~2^-22)
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// 4 consecutive query elements starting at i (i % 4 == 0)
__device__ __forceinline__ float4 load_q4(const float* q, size_t i) { return *reinterpret_cast<const float4*>(q + i); }
__device__ __forceinline__ float4 load_q4(const __half* q, size_t i) {
  const uint2 u = *reinterpret_cast<const uint2*>(q + i);
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
  return make_float4(a.x, a.y, b.x, b.y);
}

__device__ __forceinline__ uint32_t pack_s8x4(int a, int b, int c, int d) {
  return (uint32_t)(a & 0xFF) | ((uint32_t)(b & 0xFF) << 8) | ((uint32_t)(c & 0xFF) << 16) | ((uint32_t)d << 24);
}

// query index of (item sequence b, KV head hk, query j)
template <bool RAGGED>
__device__ __forceinline__ size_t query_index(const StreamParams& p, int b, int hk, int j) {
  if (RAGGED) return (size_t)b * p.H + (size_t)hk * (p.H / p.Hkv) + j;
  return (size_t)(b * kQ + j) * p.H + hk;
}

template <bool RAGGED>
__device__ __forceinline__ int queries_of(const StreamParams& p, int b) {
  return RAGGED ? p.H / p.Hkv : min(kQ, p.B - b * kQ);
}

template <typename QT, bool RAGGED>
__global__ void __maxnreg__(112)
    fa_stream_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                     StreamParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~(uintptr_t)127);
  int* sT = reinterpret_cast<int*>(smem + kOffT);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* empty = full + kStages;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // launched as a programmatic dependent: no global read before the
  // preceding kernel (the previous call's merge, or the queries' producer) ends
  pdl_wait();

  // ---- schedule: tile prefix over the sequences ----
  Sched sc;
  sc.nseq = p.nseq;
  sc.n_hg = p.n_hg;
  if (RAGGED) {
    for (int i = threadIdx.x; i < p.nseq; i += blockDim.x) sT[i + 1] = (p.cu[i + 1] - p.cu[i] + kTok - 1) / kTok;
    if (threadIdx.x == 0) sT[0] = 0;
    __syncthreads();
    if (warp == 0) {
      const int per = (p.nseq + 31) / 32;
      const int i0 = 1 + lane * per, i1 = min(p.nseq + 1, i0 + per);
      int s = 0;
      for (int i = i0; i < i1; ++i) s += sT[i];
      int incl = s;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      int run = incl - s;
      for (int i = i0; i < i1; ++i) {
        run += sT[i];
        sT[i] = run;
      }
    }
    __syncthreads();
    if (blockIdx.x == 0)
      for (int i = threadIdx.x; i <= p.nseq; i += blockDim.x) p.tprefix[i] = sT[i];
    sc.T = sT;
    sc.nt_uni = 0;
  } else {
    sc.T = nullptr;
    sc.nt_uni = (p.S + kTok - 1) / kTok;
  }
  const long long TT = sc.total();
  const long long t_begin = TT * blockIdx.x / gridDim.x, t_end = TT * (blockIdx.x + 1) / gridDim.x;
  if (t_begin >= t_end) return;  // no tiles for this CTA (uniform exit: nothing initialised yet)
  // the combine may launch now: it waits (griddepcontrol.wait) for this whole
  // grid to finish, but its launch latency overlaps the decode
  pdl_launch_dependents();

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kHeads);
    }
    fence_mbar_init();
  }
  __syncthreads();

  bool dead = false;
  // ---- TMA issue (warp 0, lane 0): tile k goes to stage k % kStages ----
  int pb = 0, phg = 0, pj = 0;  // position of the next tile to issue
  const int ntiles = (int)(t_end - t_begin);
  auto issue = [&](int s) {
    mbar_arrive_expect_tx(&full[s], 2 * kTile);
    const int row0 = RAGGED ? p.cu[pb] : 0;
    const int y = row0 + pj * kTok;
    tma_load_2d(smem + s * kTile, &kmap, phg * (kHeads * kHeadBytes / 8), y, &full[s]);
    tma_load_2d(smem + kOffV + s * kTile, &vmap, phg * (kHeads * kHeadBytes / 8), y, &full[s]);
    sc.next(pb, phg, pj);
  };
  if (warp == 0 && lane == 0) {
    sc.locate(t_begin, pb, phg, pj);
    for (int k = 0; k < min(kStages, ntiles); ++k) issue(k);
  }

  // ---------------- compute warp w: KV head hg * 8 + w ----------------
  const int w = warp;
  const int gid = lane >> 2, tid = lane & 3;
  uint8_t* vh = smem + kOffVh + w * (kTok * kVhPitch);
  const uint32_t vh_s = smem_u32(vh);
  float* pbuf = reinterpret_cast<float*>(smem + kOffP) + w * (kQ * kTok);
  float4* dkv = reinterpret_cast<float4*>(smem + kOffD) + w * 32;

  uint32_t qb[4][2];  // B fragments: column gid = (query gid / 2, level gid % 2)
  float s2t = 0.0f;   // level-2 scale of query tid (score scale of the D columns this lane holds)
  float m_run = -INFINITY, l_run = 0.0f;  // query tid
  float o[8][4];      // D: dims 16 mt + gid (+8) x columns 2 tid, 2 tid + 1 (queries; tid < 2)
  int nq = 0, cur_item = -1, cur_b = 0, cur_hg = 0, L = 0;

  auto start_item = [&](int b, int hg) {
    cur_b = b;
    cur_hg = hg;
    cur_item = b * p.n_hg + hg;
    nq = queries_of<RAGGED>(p, b);
    L = RAGGED ? p.cu[b + 1] - p.cu[b] : p.S;
    const int hk = hg * kHeads + w;
    const int jq = gid >> 1, lvl = gid & 1;
    float v[4][2][4];
    if (jq < nq) {
      const QT* qp = static_cast<const QT*>(p.q) + query_index<RAGGED>(p, b, hk, jq) * 128;
#pragma unroll
      for (int bb = 0; bb < 4; ++bb)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const float4 t = load_q4(qp, 32 * bb + 16 * h + 4 * tid);
          v[bb][h][0] = t.x * p.qscale; v[bb][h][1] = t.y * p.qscale;
          v[bb][h][2] = t.z * p.qscale; v[bb][h][3] = t.w * p.qscale;
        }
    } else {
#pragma unroll
      for (int bb = 0; bb < 4; ++bb)
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int i = 0; i < 4; ++i) v[bb][h][i] = 0.0f;
    }
    float a = 0.0f;
#pragma unroll
    for (int bb = 0; bb < 4; ++bb)
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int i = 0; i < 4; ++i) a = fmaxf(a, fabsf(v[bb][h][i]));
    a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 1));
    a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 2));
    const float s1 = a > 0.0f ? a / 127.0f : 1.0f;
    const float inv1 = a > 0.0f ? 127.0f / a : 0.0f;
    const float inv2 = 127.0f * inv1;
#pragma unroll
    for (int bb = 0; bb < 4; ++bb)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        int c[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int c1 = max(-127, min(127, __float2int_rn(v[bb][h][i] * inv1)));
          const int c2 = max(-127, min(127, __float2int_rn(fmaf(-s1, (float)c1, v[bb][h][i]) * inv2)));
          c[i] = lvl ? c2 : c1;
        }
        qb[bb][h] = pack_s8x4(c[0], c[1], c[2], c[3]);
      }
    // query tid's level-2 scale: lane 8 tid holds query tid at level 1
    s2t = __shfl_sync(0xffffffffu, s1, 8 * tid) * (1.0f / 127.0f);
    m_run = -INFINITY;
    l_run = 0.0f;
#pragma unroll
    for (int mt = 0; mt < 8; ++mt)
#pragma unroll
      for (int i = 0; i < 4; ++i) o[mt][i] = 0.0f;
  };

  auto flush_item = [&]() {
    const size_t base = ((size_t)(blockIdx.x + cur_item) * kHeads + w) * kQ;
    if (lane < kQ && lane < nq) {  // lane q = (gid 0, tid q) holds query q's state
      p.pm[base + lane] = m_run;
      p.pl[base + lane] = l_run;
    }
    // columns 4-7 (lanes tid 2, 3) hold the fp16 remainders of queries 0-3
#pragma unroll
    for (int mt = 0; mt < 8; ++mt)
#pragma unroll
      for (int i = 0; i < 4; ++i) o[mt][i] += __shfl_xor_sync(0xffffffffu, o[mt][i], 2);
    if (tid < 2) {
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int q = 2 * tid + c;
        if (q < nq) {
          float* acc = p.pacc + (base + q) * 128;
#pragma unroll
          for (int mt = 0; mt < 8; ++mt) {
            acc[16 * mt + gid] = o[mt][c];
            acc[16 * mt + gid + 8] = o[mt][2 + c];
          }
        }
      }
    }
  };

  int b, hg, j;
  sc.locate(t_begin, b, hg, j);
  for (int k = 0; k < ntiles; ++k) {
    if (b * p.n_hg + hg != cur_item) {
      if (cur_item >= 0) flush_item();
      start_item(b, hg);
    }
    const int s = k % kStages;
    const int nvalid = min(kTok, L - j * kTok);  // >= 1
    mbar_wait_or_poison(&full[s], (k / kStages) & 1, p.err, DEV_TIMEOUT_FULL, dead);
    const uint8_t* kt = smem + s * kTile + w * kHeadBytes;
    const uint8_t* vt = smem + kOffV + s * kTile + w * kHeadBytes;

    // ---- per-token block scales: lanes 0-15 d_k of token lane, 16-31 d_v of token lane-16 ----
    {
      const int t = lane & 15;
      const uint8_t* row = (lane < 16 ? kt : vt) + t * kPitch;
      float4 d = make_float4(lds_half(row), lds_half(row + 34), lds_half(row + 68), lds_half(row + 102));
      if (lane >= 16 && t >= nvalid) d = make_float4(0.f, 0.f, 0.f, 0.f);  // masked tokens weigh nothing
      dkv[lane] = d;
    }
    // ---- V codes -> fp16 (exact), lane = 4 dims ----
    {
      const uint8_t* src = vt + (lane >> 3) * 34 + 2 + 4 * (lane & 7);
      uint8_t* dst = vh + 8 * lane;
#pragma unroll
      for (int t = 0; t < kTok; ++t) {
        const uint32_t cw = lds_u32_a2(src + t * kPitch) ^ 0x80808080u;
        const uint32_t lo = __byte_perm(cw, 0x64646464u, 0x4140), hi = __byte_perm(cw, 0x64646464u, 0x4342);
        uint32_t l2, h2;
        asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(l2) : "r"(lo), "r"(0x64806480u));
        asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(h2) : "r"(hi), "r"(0x64806480u));
        *reinterpret_cast<uint2*>(dst + t * kVhPitch) = make_uint2(l2, h2);
      }
    }
    __syncwarp();

    // ---- QK: 4 blocks; D rows = tokens gid, gid + 8; columns = query tid x level ----
    float sc0, sc1;
    {
      const float4 dka = dkv[gid], dkb = dkv[gid + 8];
      const float dk0[4] = {dka.x, dka.y, dka.z, dka.w}, dk1[4] = {dkb.x, dkb.y, dkb.z, dkb.w};
      const uint8_t* r0 = kt + gid * kPitch + 2 + 4 * tid;
      const uint8_t* r1 = r0 + 8 * kPitch;
      float acc0 = 0.0f, acc1 = 0.0f;
#pragma unroll
      for (int bb = 0; bb < 4; ++bb) {
        uint32_t a0, a1, a2, a3;
        if (bb & 1) {  // odd blocks: codes 4-byte aligned
          a0 = *reinterpret_cast<const uint32_t*>(r0 + 34 * bb);
          a1 = *reinterpret_cast<const uint32_t*>(r1 + 34 * bb);
          a2 = *reinterpret_cast<const uint32_t*>(r0 + 34 * bb + 16);
          a3 = *reinterpret_cast<const uint32_t*>(r1 + 34 * bb + 16);
        } else {
          a0 = lds_u32_a2(r0 + 34 * bb);
          a1 = lds_u32_a2(r1 + 34 * bb);
          a2 = lds_u32_a2(r0 + 34 * bb + 16);
          a3 = lds_u32_a2(r1 + 34 * bb + 16);
        }
        int d[4];
        mma_s8_16832(d, a0, a1, a2, a3, qb[bb][0], qb[bb][1]);
        acc0 = fmaf(dk0[bb], (float)(127 * d[0] + d[1]), acc0);
        acc1 = fmaf(dk1[bb], (float)(127 * d[2] + d[3]), acc1);
      }
      sc0 = gid < nvalid ? acc0 * s2t : -INFINITY;
      sc1 = gid + 8 < nvalid ? acc1 * s2t : -INFINITY;
    }
    // the TMA stage is no longer read: release it for the next tile
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    if (warp == 0 && lane == 0 && k + kStages < ntiles) {
      // refill this stage once every warp has released it
      mbar_wait_or_poison(&empty[s], (k / kStages) & 1, p.err, DEV_TIMEOUT_EMPTY, dead);
      issue(s);
    }

    // ---- online softmax for query tid ----
    float mx = fmaxf(sc0, sc1);
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
    if (__any_sync(0xffffffffu, mx > m_run)) {
      const float m_new = fmaxf(m_run, mx);
      const float corr = (m_run == -INFINITY) ? 0.0f : ex2(m_run - m_new);
      m_run = m_new;
      l_run *= corr;
      const float ca = __shfl_sync(0xffffffffu, corr, (2 * tid) & 3);
      const float cb = __shfl_sync(0xffffffffu, corr, (2 * tid + 1) & 3);
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        o[mt][0] *= ca;
        o[mt][1] *= cb;
        o[mt][2] *= ca;
        o[mt][3] *= cb;
      }
    }
    const float p0 = sc0 == -INFINITY ? 0.0f : ex2(sc0 - m_run);
    const float p1 = sc1 == -INFINITY ? 0.0f : ex2(sc1 - m_run);
    float ls = p0 + p1;
    ls += __shfl_xor_sync(0xffffffffu, ls, 4);
    ls += __shfl_xor_sync(0xffffffffu, ls, 8);
    ls += __shfl_xor_sync(0xffffffffu, ls, 16);
    l_run += ls;
    pbuf[tid * kTok + gid] = p0;
    pbuf[tid * kTok + gid + 8] = p1;
    __syncwarp();

    // ---- PV: B = p * d_v, tokens 2 tid, 2 tid + 1, 2 tid + 8, 2 tid + 9; column gid < 4
    // holds query gid rounded to fp16, column gid + 4 the rounding remainder
    // (so the product carries about 22 bits of p * d_v) ----
    uint32_t bf[4][2];
    {
      const float4 v0 = dkv[16 + 2 * tid], v1 = dkv[16 + 2 * tid + 1], v8 = dkv[16 + 2 * tid + 8],
                   v9 = dkv[16 + 2 * tid + 9];
      const float dv0[4] = {v0.x, v0.y, v0.z, v0.w}, dv1[4] = {v1.x, v1.y, v1.z, v1.w};
      const float dv8[4] = {v8.x, v8.y, v8.z, v8.w}, dv9[4] = {v9.x, v9.y, v9.z, v9.w};
      const float2 pa = *reinterpret_cast<const float2*>(pbuf + (gid & 3) * kTok + 2 * tid);
      const float2 pb = *reinterpret_cast<const float2*>(pbuf + (gid & 3) * kTok + 2 * tid + 8);
      const bool rem = gid >= kQ;
#pragma unroll
      for (int bb = 0; bb < 4; ++bb) {
        const float x0 = pa.x * dv0[bb], x1 = pa.y * dv1[bb], x2 = pb.x * dv8[bb], x3 = pb.y * dv9[bb];
        uint32_t h0 = pack_half2(x0, x1), h1 = pack_half2(x2, x3);
        if (rem) {
          const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&h0));
          const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&h1));
          h0 = pack_half2(x0 - f0.x, x1 - f0.y);
          h1 = pack_half2(x2 - f1.x, x3 - f1.y);
        }
        bf[bb][0] = h0;
        bf[bb][1] = h1;
      }
    }
    {
      const int mi = lane >> 3, r = lane & 7;
      const int tok = (mi >> 1) * 8 + r;
      const uint32_t row = vh_s + tok * kVhPitch + (mi & 1) * 16;
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        uint32_t af[4];
        ldsm_x4_trans(af, row + mt * 32);
        mma_f16_16816(o[mt], af, bf[mt >> 1][0], bf[mt >> 1][1]);
      }
    }
    __syncwarp();  // vh and pbuf are rewritten by the next tile
    sc.next(b, hg, j);
  }
  if (cur_item >= 0) flush_item();
}

// One warp per query: merge the partials of its item (slots owner(first tile)
// + item .. owner(last tile) + item). Lane = 4 dims.
template <typename OT, bool RAGGED>
__global__ void __launch_bounds__(128) fa_stream_combine_kernel(StreamParams p, int Q, int G) {
  pdl_wait();  // the decode grid's partials
  pdl_launch_dependents();  // a following decode waits for this grid in turn
  const int qg = blockIdx.x * 4 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (qg >= Q) return;
  int b, hk, j;
  if (RAGGED) {
    const int g = p.H / p.Hkv;
    b = qg / p.H;
    const int rem = qg % p.H;
    hk = rem / g;
    j = rem % g;
  } else {
    const int bq = qg / p.H;
    hk = qg % p.H;
    b = bq / kQ;
    j = bq % kQ;
  }
  const int hg = hk / kHeads, w = hk % kHeads;
  const int item = b * p.n_hg + hg;
  int pre_b, pre_b1, pre_n;
  if (RAGGED) {
    pre_b = p.tprefix[b];
    pre_b1 = p.tprefix[b + 1];
    pre_n = p.tprefix[p.nseq];
  } else {
    const int nt = (p.S + kTok - 1) / kTok;
    pre_b = b * nt;
    pre_b1 = pre_b + nt;
    pre_n = p.nseq * nt;
  }
  const int nt = pre_b1 - pre_b;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  float L = 0.0f;
  if (nt > 0) {
    const long long TT = (long long)p.n_hg * pre_n;
    const long long f = (long long)p.n_hg * pre_b + (long long)hg * nt;
    const int c0 = owner_of(f, TT, G), c1 = owner_of(f + nt - 1, TT, G);
    // CTAs between the owners of the first and last tile whose ranges are
    // empty (fewer tiles than CTAs) wrote no partial
    auto has_tiles = [&](int c) { return TT * c / G < TT * (c + 1) / G; };
    auto slot = [&](int c) { return ((size_t)(c + item) * kHeads + w) * kQ + j; };
    const int np = c1 - c0 + 1;
    // Lane i holds partial c0 + base + i: all maxima and sums arrive in one
    // round of loads instead of a dependent chain per partial.
    float M = -INFINITY;
    for (int base = 0; base < np; base += 32) {
      const int c = c0 + base + lane;
      const float mc = (base + lane < np && has_tiles(c)) ? p.pm[slot(c)] : -INFINITY;
      M = fmaxf(M, warp_max(mc));
    }
    if (M != -INFINITY) {
      for (int base = 0; base < np; base += 32) {
        const int c = c0 + base + lane;
        const bool valid = base + lane < np && has_tiles(c);
        const float mc = valid ? p.pm[slot(c)] : -INFINITY;
        const float lc = valid ? p.pl[slot(c)] : 0.0f;
        const float wgt = mc == -INFINITY ? 0.0f : exp2f(mc - M);
        const int cnt = min(32, np - base);
        // in partial order, as a sequential merge would: four accumulator
        // loads in flight ahead of their FMAs
        for (int k0 = 0; k0 < cnt; k0 += 4) {
          float4 a[4];
          float wk[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int k = k0 + u;
            wk[u] = __shfl_sync(0xffffffffu, wgt, k & 31);
            a[u] = (k < cnt && wk[u] != 0.0f)
                       ? *reinterpret_cast<const float4*>(p.pacc + slot(c0 + base + k) * 128 + 4 * lane)
                       : make_float4(0.f, 0.f, 0.f, 0.f);
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int k = k0 + u;
            const float lk = __shfl_sync(0xffffffffu, lc, k & 31);
            if (k < cnt && wk[u] != 0.0f) {
              L = fmaf(lk, wk[u], L);
              acc.x = fmaf(a[u].x, wk[u], acc.x);
              acc.y = fmaf(a[u].y, wk[u], acc.y);
              acc.z = fmaf(a[u].z, wk[u], acc.z);
              acc.w = fmaf(a[u].w, wk[u], acc.w);
            }
          }
        }
      }
    }
  }
  const float inv = L > 0.0f ? 1.0f / L : 0.0f;
  if constexpr (RAGGED) {
    __half2* o = reinterpret_cast<__half2*>(static_cast<__half*>(p.out) + (size_t)qg * 128 + 4 * lane);
    o[0] = __floats2half2_rn(acc.x * inv, acc.y * inv);
    o[1] = __floats2half2_rn(acc.z * inv, acc.w * inv);
  } else {
    *reinterpret_cast<float4*>(static_cast<float*>(p.out) + (size_t)qg * 128 + 4 * lane) =
        make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
  }
}

bool encode_map(CUtensorMap* map, const void* base, uint64_t rows, int heads) {
  // [rows][heads * 136 bytes] as 8-byte elements; boxes of 16 rows x 138
  // elements (8 heads' 1088 bytes plus 16 bytes that land in the padding of
  // the smem row pitch: the next head group's first bytes or the out-of-bounds
  // fill past the last one)
  auto fn = reinterpret_cast<EncodeTiledFn>(tensor_map_encoder());
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)heads * 17, rows};
  cuuint64_t strides[1] = {(cuuint64_t)heads * 136};
  cuuint32_t box[2] = {kBoxU64, kTok};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Resident CTAs of a decode kernel on the current device, after asking for
// the largest shared-memory carveout (two CTAs per SM need it). Cached per
// (device, kernel): the answer depends on nothing else.
int grid_size(const void* kern, int slot) {
  static std::atomic<int> cache[64][2];
  const int d = current_device();
  if (d < 0 || d >= 64) return sm_count();
  int g = cache[d][slot].load(std::memory_order_relaxed);
  if (g == 0) {
    int per_sm = 0;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, kSmem) != cudaSuccess || per_sm < 1) {
      cudaGetLastError();
      per_sm = 1;
    }
    g = std::min(per_sm, 2) * sm_count();
    cache[d][slot].store(g, std::memory_order_relaxed);
  }
  return g;
}

// Tiles per SM below which one CTA per SM is faster than two (the start of
// the two-stage ring and each item's query setup are paid per CTA). Harness
// form, CUDA-graph device time with the current combine: ~14 tiles per SM
// (S = 8192 B = 1, S = 4096 B = 8) one CTA 41.7 / 37.2 us, two 46.6 / 39.4;
// ~28 tiles per SM (S = 8192 B = 8) one 62.3, two 56.2; the ragged configs[3]
// workload (~59 tiles per SM) and B = 512 run faster with two.
constexpr long long kTwoCtaMinTilesPerSm = 20;

template <typename QT, typename OT, bool RAGGED>
kq_status_t launch(StreamParams p, const void* k, const void* v, uint64_t rows, int heads, long long Q,
                   long long tiles_estimate, cudaStream_t s) {
  CUtensorMap km, vm;
  if (!encode_map(&km, k, rows, heads) || !encode_map(&vm, v, rows, heads))
    return fail(KQ_ERR_CUDA, "fa_stream: KV tensor map rejected");
  auto kern = fa_stream_kernel<QT, RAGGED>;
  kq_status_t st = ensure_dynamic_smem(reinterpret_cast<const void*>(kern), (int)kSmem, "fa_stream smem attribute");
  if (st) return st;
  // one wave of resident CTAs (two per SM when the carveout allows it): the
  // schedule splits the tiles evenly over exactly the CTAs that run at once
  int G = grid_size(reinterpret_cast<const void*>(kern), RAGGED ? 0 : 1);
  if (tiles_estimate < kTwoCtaMinTilesPerSm * sm_count()) G = std::min(G, sm_count());
  {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(G);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, km, vm, p);
    if (e != cudaSuccess) return check_cuda(e, "fa_stream launch");
  }
  if ((st = check_launch("fa_stream"))) return st;
  // a programmatic dependent of the decode kernel
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((Q + 3) / 4));
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, fa_stream_combine_kernel<OT, RAGGED>, p, (int)Q, G);
  if (e != cudaSuccess) return check_cuda(e, "fa_stream_combine launch");
  return check_launch("fa_stream_combine");
}

size_t scratch_bytes(int nseq, long long items, int G) {
  const size_t table = ((size_t)(nseq + 1) * sizeof(int) + 255) & ~(size_t)255;
  const size_t slots = (size_t)G + (size_t)items;
  return table + slots * kHeads * kQ * (2 + 128) * sizeof(float);
}

StreamParams carve(void* ws, int nseq, long long items, int G) {
  StreamParams p{};
  const size_t table = ((size_t)(nseq + 1) * sizeof(int) + 255) & ~(size_t)255;
  const size_t slots = (size_t)G + (size_t)items;
  char* base = static_cast<char*>(ws);
  p.tprefix = reinterpret_cast<int*>(base);
  p.pm = reinterpret_cast<float*>(base + table);
  p.pl = p.pm + slots * kHeads * kQ;
  p.pacc = p.pl + slots * kHeads * kQ;
  return p;
}

}  // namespace

bool fa_stream_supported(const void* q, const void* k, const void* v, const void* out, int D, int Hkv,
                         int queries_per_kv_head, int nseq_ragged) {
  auto al = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; };
  return D == 128 && Hkv % kHeads == 0 && queries_per_kv_head >= 1 && queries_per_kv_head <= kQ &&
         nseq_ragged <= kMaxSeq && al(q) && al(k) && al(v) && al(out);
}

kq_status_t launch_fa_stream_ragged(const void* q, const void* k, const void* v, const int32_t* cu, int B, int Hq,
                                    int Hkv, int total_rows, float scale, void* out, cudaStream_t s) {
  const int G = 2 * sm_count();  // slots for up to two CTAs per SM
  const int n_hg = Hkv / kHeads;
  const long long items = (long long)B * n_hg;
  void* ws = workspace(WS_FA, scratch_bytes(B, items, G));
  if (!ws) return KQ_ERR_NOMEM;
  StreamParams p = carve(ws, B, items, G);
  p.q = q;
  p.cu = cu;
  p.out = out;
  p.err = device_error_word();
  p.nseq = B;
  p.B = B;
  p.H = Hq;
  p.Hkv = Hkv;
  p.S = 0;
  p.n_hg = n_hg;
  p.qscale = (float)((double)scale * 1.4426950408889634);
  const long long tiles = ((long long)total_rows + (long long)B * (kTok - 1)) / kTok * n_hg;  // upper bound
  return launch<__half, __half, true>(p, k, v, (uint64_t)std::max(total_rows, 1), Hkv, (long long)B * Hq, tiles, s);
}

kq_status_t launch_fa_stream_mha(const float* q, const void* k, const void* v, float* out, int B, int S, int H,
                                 cudaStream_t s) {
  const int G = 2 * sm_count();  // slots for up to two CTAs per SM
  const int n_hg = H / kHeads;
  const int nseq = (B + kQ - 1) / kQ;
  const long long items = (long long)nseq * n_hg;
  void* ws = workspace(WS_FA, scratch_bytes(nseq, items, G));
  if (!ws) return KQ_ERR_NOMEM;
  StreamParams p = carve(ws, nseq, items, G);
  p.q = q;
  p.cu = nullptr;
  p.out = out;
  p.err = device_error_word();
  p.nseq = nseq;
  p.B = B;
  p.H = H;
  p.Hkv = H;
  p.S = S;
  p.n_hg = n_hg;
  p.qscale = (float)(1.0 / std::sqrt(128.0) * 1.4426950408889634);
  const long long tiles = (long long)items * ((S + kTok - 1) / kTok);
  return launch<float, float, false>(p, k, v, (uint64_t)std::max(S, 1), H, (long long)B * H, tiles, s);
}

}  // namespace kq
