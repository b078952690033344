// Flash-attention decode over a q8_0, q4_0 or fp16 KV cache (split-KV "flash
// decoding").
//
// Semantics: the harness flash_attention operator
// (kernelevalplus-main/llm_kernel_test/op_test_handler.py:543-563):
// out = softmax(q . K^T / sqrt(D)) . V per (query, head), with K and V stored
// as q8_0 blocks along head_dim (op_test_handler.py:489-508), dequantised as
// x = q * d, as q4_0 blocks (x = d (q - 8)) or as fp16. The ragged GQA form (one KV stream per (sequence, KV head),
// shared by Hq/Hkv query heads) follows the same arithmetic.
//
// Fast path (head_dim 128, KV heads in groups of 8, <= 4 queries per KV
// head): one CTA per (sequence or query group, token chunk, group of 8 KV
// heads). A producer warp streams 32-token tiles of K and V for the 8 heads
// (1088 contiguous bytes per token row: the cache's own layout) with 2D TMA
// boxes into a double-buffered ring; each of 8 compute warps owns one KV head
// and its queries, lanes own 4 head dims. Scores are partial dot products
// reduced with a transpose-halving warp reduction (8 tokens x 4 queries per
// step); q8_0 bytes become fp32 exactly through a signed bit-field extract
// and the 1.5 * 2^23 bias (x = fma(f, d, -12582912 d)), no conversion op.
//
// Generic path: pass 1 gives every (KV stream, token chunk, query group) to one
// CTA, one warp per query; each warp keeps an online-softmax state (running
// max in the log2 domain, running sum, fp32 accumulator) and writes it as a
// partial; it takes 8 tokens per step (independent loads, interleaved
// reductions, one rescale). Pass 2 merges the partials of each query. For
// head_dim 64, 128 or 256 a lane owns D/32 consecutive elements (one vector
// load of fp16, or 2-byte loads of codes inside one block plus its scale);
// otherwise lanes own elements {32 j + lane}.
#include <cuda.h>

#include <algorithm>
#include <cmath>

#include <cstdlib>
#include <string>

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

constexpr int kQPerCta = 4;  // queries (warps) per CTA
constexpr int kMaxDJ = 8;    // head_dim <= 256
constexpr int kTokU = 8;     // tokens per step of the generic kernel

struct FaParams {
  const void* q;
  const uint8_t* k;
  const uint8_t* v;
  const int32_t* cu;  // ragged only
  float* pm;          // [Q][NC] running max (log2 domain)
  float* pl;          // [Q][NC] running sum
  float* pacc;        // [Q][NC][D]
  void* out;
  int B, H, Hkv, D, S, NC, chunk;
  float qscale;  // softmax scale * log2(e)
};

__device__ __forceinline__ float load_q(const float* q, size_t i) { return q[i]; }
__device__ __forceinline__ float load_q(const __half* q, size_t i) { return __half2float(q[i]); }
__device__ __forceinline__ void store_o(float* o, size_t i, float v) { o[i] = v; }
__device__ __forceinline__ void store_o(__half* o, size_t i, float v) { o[i] = __float2half_rn(v); }

// KV cache element (dimension 32 j + lane) of one cache row, per format:
//   q8_0: D/32 blocks of 34 B (fp16 d, 32 int8), value d q
//   q4_0: D/32 blocks of 18 B (fp16 d, byte i = q[i] | q[i+16] << 4), value d (q - 8)
//         (op_test_handler.py:502-516 builds it with quantize_to_q4_0, quantize.py:56-102)
//   f16:  D halves
template <int KVF>
__device__ __forceinline__ float kv_elem(const uint8_t* row, int j, int lane) {
  if constexpr (KVF == KQ_KV_Q8_0) {
    const uint8_t* b = row + j * 34;
    return half_bits_to_float(*reinterpret_cast<const uint16_t*>(b)) * (float)(int8_t)b[2 + lane];
  } else if constexpr (KVF == KQ_KV_Q4_0) {
    const uint8_t* b = row + j * 18;
    const uint32_t byte = b[2 + (lane & 15)];
    const int q = (int)(lane < 16 ? (byte & 15u) : (byte >> 4)) - 8;
    return half_bits_to_float(*reinterpret_cast<const uint16_t*>(b)) * (float)q;
  } else {
    return __half2float(reinterpret_cast<const __half*>(row)[j * 32 + lane]);
  }
}
__host__ __device__ constexpr int kv_block_bytes(int kvf) { return kvf == KQ_KV_Q8_0 ? 34 : kvf == KQ_KV_Q4_0 ? 18 : 64; }

// Elements DJ*lane .. DJ*lane + DJ - 1 of a cache row with D = 32 DJ,
// DJ in {2, 4, 8}: they lie in one 32-element block. fp16 rows need 2 DJ-byte
// alignment; block codes start at an even offset (2-byte loads).
template <int KVF, int DJ>
__device__ __forceinline__ void kv_lane(const uint8_t* row, int lane, float (&x)[DJ]) {
  static_assert(DJ == 2 || DJ == 4 || DJ == 8, "DJ");
  const int e0 = DJ * lane;
  if constexpr (KVF == KQ_KV_F16) {
    const uint8_t* p = row + 2 * e0;
    auto cvt = [](uint32_t w, float& a, float& b) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w));
      a = f.x;
      b = f.y;
    };
    if constexpr (DJ == 8) {
      const uint4 u = *reinterpret_cast<const uint4*>(p);
      cvt(u.x, x[0], x[1]); cvt(u.y, x[2], x[3]); cvt(u.z, x[4], x[5]); cvt(u.w, x[6], x[7]);
    } else if constexpr (DJ == 4) {
      const uint2 u = *reinterpret_cast<const uint2*>(p);
      cvt(u.x, x[0], x[1]); cvt(u.y, x[2], x[3]);
    } else {
      cvt(*reinterpret_cast<const uint32_t*>(p), x[0], x[1]);
    }
  } else {
    const int o = e0 & 31;
    const uint8_t* blk = row + (e0 >> 5) * kv_block_bytes(KVF);
    const float d = half_bits_to_float(*reinterpret_cast<const uint16_t*>(blk));
    if constexpr (KVF == KQ_KV_Q8_0) {
      const uint16_t* c = reinterpret_cast<const uint16_t*>(blk + 2 + o);
#pragma unroll
      for (int i = 0; i < DJ / 2; ++i) {
        const uint32_t v = c[i];
        x[2 * i] = d * (float)(int8_t)(v & 0xffu);
        x[2 * i + 1] = d * (float)(int8_t)(v >> 8);
      }
    } else {
      // byte i of a block holds element i (low nibble) and i + 16 (high)
      const int sh = o < 16 ? 0 : 4;
      const uint16_t* c = reinterpret_cast<const uint16_t*>(blk + 2 + (o & 15));
#pragma unroll
      for (int i = 0; i < DJ / 2; ++i) {
        const uint32_t v = c[i];
        x[2 * i] = d * (float)((int)((v >> sh) & 15u) - 8);
        x[2 * i + 1] = d * (float)((int)((v >> (8 + sh)) & 15u) - 8);
      }
    }
  }
}

// RAGGED = false: grid (NC, H, ceil(B/4)); queries b of head h share KV head h.
// RAGGED = true:  grid (NC, B*Hkv, ceil(g/4)); query heads of KV head hk.
// This warp's query of a generic-path CTA: query index, stream length, first
// KV row, rows per token. False when the warp has no query.
template <bool RAGGED>
__device__ __forceinline__ bool fa_query(const FaParams& p, int warp, int& qg, int& L, int& row0, int& row_stride) {
  if (!RAGGED) {
    const int h = blockIdx.y;
    const int b = blockIdx.z * kQPerCta + warp;
    if (b >= p.B) return false;
    qg = b * p.H + h;
    L = p.S;
    row0 = h;
    row_stride = p.H;
  } else {
    const int b = blockIdx.y / p.Hkv, hk = blockIdx.y % p.Hkv;
    const int g = p.H / p.Hkv;
    const int j = blockIdx.z * kQPerCta + warp;
    if (j >= g) return false;
    qg = b * p.H + hk * g + j;
    const int s0 = p.cu[b];
    L = p.cu[b + 1] - s0;
    row0 = s0 * p.Hkv + hk;
    row_stride = p.Hkv;
  }
  return true;
}

template <typename QT, bool RAGGED, int KVF>
__global__ void __launch_bounds__(32 * kQPerCta) fa_partial_kernel(FaParams p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x;
  const int dj = p.D / 32;
  const size_t row_bytes = (size_t)dj * kv_block_bytes(KVF);

  int qg, L, row0, row_stride;
  if (!fa_query<RAGGED>(p, warp, qg, L, row0, row_stride)) return;

  float qv[kMaxDJ], acc[kMaxDJ];
  const QT* q = static_cast<const QT*>(p.q) + (size_t)qg * p.D;
#pragma unroll
  for (int j = 0; j < kMaxDJ; ++j) {
    qv[j] = (j < dj) ? load_q(q, (size_t)j * 32 + lane) * p.qscale : 0.0f;
    acc[j] = 0.0f;
  }
  // Tokens in groups of kTokU. Loads are unconditional (a token past the
  // chunk re-reads its last row and is masked out of the softmax), so the
  // group's loads issue back to back instead of one round trip per token;
  // then kTokU score reductions interleave, one rescale per group, V likewise.
  float m = -INFINITY, l = 0.0f;
  const int t0 = c * p.chunk, t1 = min(L, t0 + p.chunk);
  for (int t = t0; t < t1; t += kTokU) {
    float sc[kTokU];
#pragma unroll
    for (int u = 0; u < kTokU; ++u) {
      const uint8_t* kb = p.k + ((size_t)row0 + (size_t)min(t + u, t1 - 1) * row_stride) * row_bytes;
      sc[u] = 0.0f;
#pragma unroll
      for (int j = 0; j < kMaxDJ; ++j)
        if (j < dj) sc[u] = fmaf(qv[j], kv_elem<KVF>(kb, j, lane), sc[u]);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1)
#pragma unroll
      for (int u = 0; u < kTokU; ++u) sc[u] += __shfl_xor_sync(0xffffffffu, sc[u], o);
    float mn = m;
#pragma unroll
    for (int u = 0; u < kTokU; ++u) {
      if (t + u >= t1) sc[u] = -INFINITY;
      mn = fmaxf(mn, sc[u]);
    }
    const float corr = exp2f(m - mn);  // 0 on the first group (m = -inf, mn finite)
    l *= corr;
#pragma unroll
    for (int j = 0; j < kMaxDJ; ++j) acc[j] *= corr;
#pragma unroll
    for (int u = 0; u < kTokU; ++u) {
      const float pr = exp2f(sc[u] - mn);  // 0 for a masked token
      l += pr;
      const uint8_t* vb = p.v + ((size_t)row0 + (size_t)min(t + u, t1 - 1) * row_stride) * row_bytes;
#pragma unroll
      for (int j = 0; j < kMaxDJ; ++j)
        if (j < dj) acc[j] = fmaf(pr, kv_elem<KVF>(vb, j, lane), acc[j]);
    }
    m = mn;
  }
  const size_t pi = (size_t)qg * p.NC + c;
  if (lane == 0) {
    p.pm[pi] = m;
    p.pl[pi] = l;
  }
#pragma unroll
  for (int j = 0; j < kMaxDJ; ++j)
    if (j < dj) p.pacc[pi * p.D + j * 32 + lane] = acc[j];
}

// The same pass with lanes owning DJ consecutive elements (D = 32 DJ).
template <typename QT, bool RAGGED, int KVF, int DJ>
__global__ void __launch_bounds__(32 * kQPerCta, 4) fa_partial_vec_kernel(FaParams p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x;
  const size_t row_bytes = (size_t)DJ * kv_block_bytes(KVF);

  int qg, L, row0, row_stride;
  if (!fa_query<RAGGED>(p, warp, qg, L, row0, row_stride)) return;

  float qv[DJ], acc[DJ];
  const QT* q = static_cast<const QT*>(p.q) + (size_t)qg * p.D + DJ * lane;
#pragma unroll
  for (int i = 0; i < DJ; ++i) {
    qv[i] = load_q(q, i) * p.qscale;
    acc[i] = 0.0f;
  }
  float m = -INFINITY, l = 0.0f;
  const int t0 = c * p.chunk, t1 = min(L, t0 + p.chunk);
  for (int t = t0; t < t1; t += kTokU) {
    float kx[kTokU][DJ];
#pragma unroll
    for (int u = 0; u < kTokU; ++u)
      kv_lane<KVF, DJ>(p.k + ((size_t)row0 + (size_t)min(t + u, t1 - 1) * row_stride) * row_bytes, lane, kx[u]);
    float sc[kTokU];
#pragma unroll
    for (int u = 0; u < kTokU; ++u) {
      sc[u] = 0.0f;
#pragma unroll
      for (int i = 0; i < DJ; ++i) sc[u] = fmaf(qv[i], kx[u][i], sc[u]);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1)
#pragma unroll
      for (int u = 0; u < kTokU; ++u) sc[u] += __shfl_xor_sync(0xffffffffu, sc[u], o);
    float mn = m;
#pragma unroll
    for (int u = 0; u < kTokU; ++u) {
      if (t + u >= t1) sc[u] = -INFINITY;
      mn = fmaxf(mn, sc[u]);
    }
    const float corr = exp2f(m - mn);
    l *= corr;
#pragma unroll
    for (int i = 0; i < DJ; ++i) acc[i] *= corr;
#pragma unroll
    for (int u = 0; u < kTokU; ++u)
      kv_lane<KVF, DJ>(p.v + ((size_t)row0 + (size_t)min(t + u, t1 - 1) * row_stride) * row_bytes, lane, kx[u]);
#pragma unroll
    for (int u = 0; u < kTokU; ++u) {
      const float pr = exp2f(sc[u] - mn);  // 0 for a masked token
      l += pr;
#pragma unroll
      for (int i = 0; i < DJ; ++i) acc[i] = fmaf(pr, kx[u][i], acc[i]);
    }
    m = mn;
  }
  const size_t pi = (size_t)qg * p.NC + c;
  if (lane == 0) {
    p.pm[pi] = m;
    p.pl[pi] = l;
  }
  float* pa = p.pacc + pi * p.D + DJ * lane;
#pragma unroll
  for (int i = 0; i < DJ; ++i) pa[i] = acc[i];
}

// One warp per query: merge the NC partial states.
// One warp per query: merge the NC partial states. The lanes take the
// partials' maxima and sums 32 at a time; the accumulator pass selects (no
// branch) so its loads do not wait on the scale loads. A partial with
// m = -inf (no tokens) weighs 0 whatever its accumulator holds.
template <typename OT>
__global__ void __launch_bounds__(128) fa_combine_kernel(FaParams p, int Q) {
  const int qg = blockIdx.x * 4 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (qg >= Q) return;
  const int dj = p.D / 32;
  const float* pm = p.pm + (size_t)qg * p.NC;
  const float* pl = p.pl + (size_t)qg * p.NC;
  float M = -INFINITY;
  for (int c = lane; c < p.NC; c += 32) M = fmaxf(M, pm[c]);
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
  float acc[kMaxDJ] = {};
  float L = 0.0f;
  if (M != -INFINITY) {
    for (int c = lane; c < p.NC; c += 32) {
      const float mc = pm[c];
      L += mc == -INFINITY ? 0.0f : pl[c] * exp2f(mc - M);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
    const float* pa = p.pacc + (size_t)qg * p.NC * p.D + lane;
#pragma unroll 4
    for (int c = 0; c < p.NC; ++c) {
      const float mc = pm[c];
      const float w = mc == -INFINITY ? 0.0f : exp2f(mc - M);
#pragma unroll
      for (int j = 0; j < kMaxDJ; ++j)
        if (j < dj) {
          const float a = pa[(size_t)c * p.D + j * 32];
          acc[j] = fmaf(w == 0.0f ? 0.0f : a, w, acc[j]);
        }
    }
  }
  const float inv = L > 0.0f ? 1.0f / L : 0.0f;
  OT* o = static_cast<OT*>(p.out) + (size_t)qg * p.D;
#pragma unroll
  for (int j = 0; j < kMaxDJ; ++j)
    if (j < dj) store_o(o, (size_t)j * 32 + lane, acc[j] * inv);
}

// ---------------------------------------------------------------------------
// Fast path
// ---------------------------------------------------------------------------
constexpr int kHpc = 8;        // KV heads per CTA (one compute warp each)
constexpr int kG = 4;          // queries per KV head per CTA
constexpr int kStages = 2;
constexpr int kRowBytes = kHpc * 136;  // one token row of 8 heads x (4 q8_0 blocks of 34 B)
constexpr int kFastThreads = (kHpc + 1) * 32;
// 16-token tiles, so two CTAs (18 warps) fit on an SM.
constexpr int kStF = 16;
constexpr int kTileF = kStF * kRowBytes;
constexpr int kGrpF = kStF / 8;  // 8-token score groups per tile
constexpr size_t kFastSmem = 2 * kStages * kTileF + kHpc * kG * 128 * 4 + kHpc * kStF * kG * 4 + 4 * kStages * 8 + 128;

struct FastParams {
  const void* q;
  const int32_t* cu;  // ragged only
  float* pm;
  float* pl;
  float* pacc;
  int B, H, Hkv, S, NC, chunk;
  int n_hg;           // KV head groups (Hkv / 8)
  float qscale;
};

__device__ __forceinline__ void tma_load_2d_u64(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Transpose-halving warp reduction of 32 per-lane values: lane l ends with the
// sum over lanes of value index l.
__device__ __forceinline__ float warp_reduce32_transpose(float (&v)[32], int lane) {
#pragma unroll
  for (int mask = 16, half = 16; mask >= 1; mask >>= 1, half >>= 1) {
    const bool upper = (lane & mask) != 0;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      if (i < half) {
        const float send = upper ? v[i] : v[i + half];
        const float keep = upper ? v[i + half] : v[i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, mask);
      }
    }
  }
  return v[0];
}

// Signed byte i of w as int32 (bit-field extract with sign extension).
__device__ __forceinline__ int sbyte(uint32_t w, int i) {
  int r;
  asm("bfe.s32 %0, %1, %2, 8;" : "=r"(r) : "r"(w), "r"(8 * i));
  return r;
}

// 4 signed bytes of w -> fp32 values d * byte (exact before the final rounding).
__device__ __forceinline__ void dequant4(uint32_t w, float d, float (&o)[4]) {
  const float nc = -12582912.0f * d;  // exact: fp16 d times 1.5 * 2^23
#pragma unroll
  for (int i = 0; i < 4; ++i) o[i] = fmaf(__int_as_float(sbyte(w, i) + 0x4B400000), d, nc);
}

// Read the 4 code bytes (head dims 4l..4l+3) and the block scale of one token
// row for KV head `w`; rows are 4-byte aligned, blocks 2-byte aligned.
__device__ __forceinline__ uint32_t row_codes(const uint8_t* row, int w, int lane, float& d) {
  const int blk = lane >> 3;
  const uint8_t* b = row + w * 136 + blk * 34;
  d = __half2float(__ushort_as_half(*reinterpret_cast<const uint16_t*>(b)));
  const uintptr_t a = reinterpret_cast<uintptr_t>(b + 2 + 4 * (lane & 7));
  const uint32_t* p = reinterpret_cast<const uint32_t*>(a & ~(uintptr_t)3);
  return __funnelshift_r(p[0], p[1], (a & 2) ? 16u : 0u);
}

template <typename QT, bool RAGGED>
__global__ void __launch_bounds__(kFastThreads, 2)
    fa_fast_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap, FastParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~(uintptr_t)127);
  uint8_t* ktile = smem;
  uint8_t* vtile = smem + kStages * kTileF;
  float* qs = reinterpret_cast<float*>(smem + 2 * kStages * kTileF);      // [8][4][128]
  float* ps = qs + kHpc * kG * 128;                                       // [8][kStF tokens][4]
  uint64_t* full = reinterpret_cast<uint64_t*>(ps + kHpc * kStF * kG);
  uint64_t* empty = full + kStages;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x;
  const int item = blockIdx.y;
  const int hg = item % p.n_hg;
  const int grp = item / p.n_hg;  // RAGGED: sequence b; else query group
  int L, row0, nq;
  if (RAGGED) {
    row0 = p.cu[grp];
    L = p.cu[grp + 1] - row0;
    nq = p.H / p.Hkv;
  } else {
    row0 = 0;
    L = p.S;
    nq = min(kG, p.B - grp * kG);
  }
  const int t0 = c * p.chunk, t1 = min(L, t0 + p.chunk);
  const int nsub = t1 > t0 ? (t1 - t0 + kStF - 1) / kStF : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kHpc);
    }
    fence_mbar_init();
  }
  // queries of this CTA into shared memory, pre-scaled by scale * log2(e)
  for (int i = threadIdx.x; i < kHpc * kG * 128; i += blockDim.x) {
    const int w = i / (kG * 128), j = (i / 128) % kG, dim = i % 128;
    const int hk = hg * kHpc + w;
    float v = 0.0f;
    if (j < nq) {
      size_t qi;
      if (RAGGED) qi = ((size_t)grp * p.H + (size_t)hk * (p.H / p.Hkv) + j) * 128 + dim;
      else qi = ((size_t)(grp * kG + j) * p.H + hk) * 128 + dim;
      v = load_q(static_cast<const QT*>(p.q), qi) * p.qscale;
    }
    qs[i] = v;
  }
  __syncthreads();

  bool dead = false;
  if (warp == kHpc) {
    // ---------------- producer ----------------
    if (lane == 0) {
      for (int i = 0; i < nsub; ++i) {
        const int s = i % kStages;
        if (i >= kStages) mbar_wait_or_poison(&empty[s], ((i / kStages) - 1) & 1, nullptr, 0, dead);
        mbar_arrive_expect_tx(&full[s], 2 * kTileF);
        const int y = row0 + t0 + i * kStF;
        tma_load_2d_u64(ktile + s * kTileF, &kmap, hg * (kRowBytes / 8), y, &full[s]);
        tma_load_2d_u64(vtile + s * kTileF, &vmap, hg * (kRowBytes / 8), y, &full[s]);
      }
      // drain: every issued tile must be consumed before the CTA exits
      for (int i = max(0, nsub - kStages); i < nsub; ++i)
        mbar_wait_or_poison(&empty[i % kStages], (i / kStages) & 1, nullptr, 0, dead);
    }
    return;
  }

  // ---------------- compute warp: KV head hg*8 + warp ----------------
  const int w = warp;
  float qv[kG][4];
#pragma unroll
  for (int j = 0; j < kG; ++j) {
    const float4 t = reinterpret_cast<const float4*>(qs + (w * kG + j) * 128)[lane];
    qv[j][0] = t.x; qv[j][1] = t.y; qv[j][2] = t.z; qv[j][3] = t.w;
  }
  float acc[kG][4];
#pragma unroll
  for (int j = 0; j < kG; ++j)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[j][i] = 0.0f;
  float m_run = -INFINITY, l_run = 0.0f;  // for query (lane & 3)
  float* pw = ps + w * kStF * kG;

  for (int it = 0; it < nsub; ++it) {
    const int s = it % kStages;
    mbar_wait_or_poison(&full[s], (it / kStages) & 1, nullptr, 0, dead);
    const uint8_t* kt = ktile + s * kTileF;
    const uint8_t* vt = vtile + s * kTileF;
    const int tb = t0 + it * kStF;  // first token of the tile

    // ---- scores: kGrpF groups of 8 tokens x 4 queries ----
    float sc[kGrpF];
#pragma unroll 1
    for (int g = 0; g < kGrpF; ++g) {
      float part[32];
#pragma unroll
      for (int tt = 0; tt < 8; ++tt) {
        float d;
        const uint32_t cw = row_codes(kt + (8 * g + tt) * kRowBytes, w, lane, d);
        float kf[4];
        dequant4(cw, d, kf);
#pragma unroll
        for (int j = 0; j < kG; ++j)
          part[tt * kG + j] = fmaf(qv[j][0], kf[0], fmaf(qv[j][1], kf[1], fmaf(qv[j][2], kf[2], qv[j][3] * kf[3])));
      }
      const float sv = warp_reduce32_transpose(part, lane);  // token 8g + lane/4, query lane%4
      const int tok = tb + 8 * g + (lane >> 2);
      sc[g] = (tok < t1 && (lane & 3) < nq) ? sv : -INFINITY;
    }
    // ---- online softmax for query (lane & 3) ----
    float mx = sc[0];
#pragma unroll
    for (int g = 1; g < kGrpF; ++g) mx = fmaxf(mx, sc[g]);
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
    const float m_new = fmaxf(m_run, mx);
    float pr[kGrpF], ls = 0.0f;
#pragma unroll
    for (int g = 0; g < kGrpF; ++g) {
      pr[g] = (m_new == -INFINITY) ? 0.0f : exp2f(sc[g] - m_new);
      ls += pr[g];
    }
    ls += __shfl_xor_sync(0xffffffffu, ls, 4);
    ls += __shfl_xor_sync(0xffffffffu, ls, 8);
    ls += __shfl_xor_sync(0xffffffffu, ls, 16);
    const float corr = (m_run == -INFINITY) ? 0.0f : exp2f(m_run - m_new);
    l_run = fmaf(l_run, corr, ls);
    m_run = m_new;
#pragma unroll
    for (int g = 0; g < kGrpF; ++g) pw[(8 * g + (lane >> 2)) * kG + (lane & 3)] = pr[g];
    __syncwarp();
    // ---- rescale and accumulate P . V ----
#pragma unroll
    for (int j = 0; j < kG; ++j) {
      const float cj = __shfl_sync(0xffffffffu, corr, j);
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[j][i] *= cj;
    }
#pragma unroll 4
    for (int tt = 0; tt < kStF; ++tt) {
      float d;
      const uint32_t cw = row_codes(vt + tt * kRowBytes, w, lane, d);
      float vf[4];
      dequant4(cw, d, vf);
      const float4 pj = reinterpret_cast<const float4*>(pw)[tt];
      const float pv[4] = {pj.x, pj.y, pj.z, pj.w};
#pragma unroll
      for (int j = 0; j < kG; ++j)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[j][i] = fmaf(pv[j], vf[i], acc[j][i]);
    }
    fence_proxy_async_smem();  // generic reads of the TMA-refilled tile, before its release
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }

  // ---- partial state of each query of this warp ----
  const int hk = hg * kHpc + w;
#pragma unroll
  for (int j = 0; j < kG; ++j) {
    if (j >= nq) break;
    size_t qg;
    if (RAGGED) qg = (size_t)grp * p.H + (size_t)hk * (p.H / p.Hkv) + j;
    else qg = (size_t)(grp * kG + j) * p.H + hk;
    const size_t pi = qg * p.NC + c;
    const float mj = __shfl_sync(0xffffffffu, m_run, j);
    const float lj = __shfl_sync(0xffffffffu, l_run, j);
    if (lane == 0) {
      p.pm[pi] = mj;
      p.pl[pi] = lj;
    }
    reinterpret_cast<float4*>(p.pacc + pi * 128)[lane] = make_float4(acc[j][0], acc[j][1], acc[j][2], acc[j][3]);
  }
}

bool encode_kv_map(CUtensorMap* map, const void* base, uint64_t rows, uint64_t heads, uint32_t box_rows) {
  // [rows][heads * 136 bytes] as uint64 elements; boxes of box_rows rows x 8
  // heads (the kernel's tile: its expected transaction bytes match the box)
  cuuint64_t dims[2] = {heads * 17, rows};
  cuuint64_t strides[1] = {heads * 136};
  cuuint32_t box[2] = {kRowBytes / 8, box_rows};
  cuuint32_t estr[2] = {1, 1};
  return encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(base), dims, strides, box,
                                estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Decode kernel family, read once per process from KQ_FA_PATH: by default
// the tensor-pipe kernels (fa_stream.cu, fa_small.cu, fa_batch.cu) where
// their shapes allow; "tma" = the TMA CUDA-core kernel for q8_0 caches in the
// TMA-able shapes; "generic" = the split-KV kernel every other shape uses,
// for every shape and cache format.
enum class FaPath { kStream, kTma, kGeneric };
FaPath fa_path() {
  static const FaPath p = [] {
    const char* e = std::getenv("KQ_FA_PATH");
    if (e && std::string(e) == "tma") return FaPath::kTma;
    if (e && std::string(e) == "generic") return FaPath::kGeneric;
    return FaPath::kStream;
  }();
  return p;
}

template <typename QT, bool RAGGED>
kq_status_t launch_fast(const FastParams& p, const void* k, const void* v, uint64_t rows, int heads, int items,
                        cudaStream_t s) {
  CUtensorMap km, vm;
  if (!encode_kv_map(&km, k, rows, heads, kStF) || !encode_kv_map(&vm, v, rows, heads, kStF))
    return fail(KQ_ERR_CUDA, "fa: KV tensor map rejected");
  auto kern = fa_fast_kernel<QT, RAGGED>;
  kq_status_t st = ensure_dynamic_smem(reinterpret_cast<const void*>(kern), (int)kFastSmem, "fa smem attribute");
  if (st) return st;
  dim3 grid(p.NC, items);
  kern<<<grid, kFastThreads, kFastSmem, s>>>(km, vm, p);
  return check_launch("fa_fast");
}

bool fast_ok(const void* k, const void* v, int D, int Hkv, int g) {
  return (fa_path() == FaPath::kTma || fa_path() == FaPath::kStream) && D == 128 &&
         Hkv % kHpc == 0 && g <= kG &&
         (reinterpret_cast<uintptr_t>(k) & 15) == 0 && (reinterpret_cast<uintptr_t>(v) & 15) == 0;
}

constexpr size_t kPartialBudget = 64ull << 20;

// The small-batch kernel (fa_small.cu) takes workloads with few stream tiles
// (16 tokens x 8 KV heads) per SM, where the stream kernel runs one CTA per
// SM through a long per-tile chain. With one or two queries per KV head it
// wins below 20 tiles per SM; with three or four its CUDA-core QK / PV per
// query cost more, and it wins below 4. CUDA-graph device time, q8_0, D = 128
// (small vs stream): harness S = 8192 B = 1 28.2 vs 42.9 us, B = 2 32.6 vs
// 46.2, B = 3 56.3 vs 46.4; S = 512 B = 4 10.0 vs 18.4; one ragged sequence
// of 8192 tokens (Hq 32, Hkv 8) 21.7 vs 42.0; four of 8192 55.3 vs 41.8.
// Shapes the stream kernel does not take (KV heads not in groups of 8) and
// the batch kernel does not either go to the small-batch kernel at any size:
// the generic split-KV kernel is about 3x slower there (harness H = 28,
// B = 8, S = 8192: 250 vs 74 us; ragged Hkv = 4, 8 x 4096 tokens: 83 vs 33).
bool small_batch(long long stream_tiles, int queries_per_kv_head) {
  const long long per_sm = queries_per_kv_head <= 2 ? 20 : 4;
  return stream_tiles < per_sm * sm_count();
}

// Chunks for the TMA kernels: 256-token chunks, more (down to one tile each)
// when `items` CTAs per chunk would leave the GPU short of two CTAs per SM.
int choose_chunks_fast(long long Q, int D, int max_len, size_t budget, int items, int* chunk) {
  long long nc = std::max(1, (max_len + 255) / 256);
  nc = std::max<long long>(nc, (2LL * sm_count() + items - 1) / std::max(items, 1));
  nc = std::min<long long>(nc, std::max(1, (max_len + kStF - 1) / kStF));
  const long long per = (long long)Q * (D + 2) * 4;
  nc = std::min<long long>(nc, std::max<long long>(1, (long long)budget / std::max<long long>(per, 1)));
  nc = std::min<long long>(nc, 65535);
  *chunk = (int)std::max<long long>(1, (max_len + nc - 1) / nc);
  return std::max(1, (max_len + *chunk - 1) / *chunk);
}

// Pass 1 of the generic path: the lane-vector kernel when head_dim is 64, 128
// or 256 (and fp16 caches are aligned for its vector loads), else the
// per-element one. `qpc` = queries per CTA (warps; fewer than kQPerCta when
// there are fewer queries per KV stream).
template <typename QT, bool RAGGED, int KVF>
void launch_partial(const FaParams& p, dim3 grid, int qpc, cudaStream_t s) {
  const int dj = p.D / 32;
  const int threads = 32 * std::max(1, std::min(qpc, kQPerCta));
  const uintptr_t al = reinterpret_cast<uintptr_t>(p.k) | reinterpret_cast<uintptr_t>(p.v);
  auto fits = [&](int DJ) { return dj == DJ && (KVF != KQ_KV_F16 || al % (2 * DJ) == 0); };
  if (fits(8))
    fa_partial_vec_kernel<QT, RAGGED, KVF, 8><<<grid, threads, 0, s>>>(p);
  else if (fits(4))
    fa_partial_vec_kernel<QT, RAGGED, KVF, 4><<<grid, threads, 0, s>>>(p);
  else if (fits(2))
    fa_partial_vec_kernel<QT, RAGGED, KVF, 2><<<grid, threads, 0, s>>>(p);
  else
    fa_partial_kernel<QT, RAGGED, KVF><<<grid, threads, 0, s>>>(p);
}

// Chunks for the generic kernel: about one resident wave of (query, chunk)
// warps (16 per SM at its ~100-128 registers per thread), at least 4 token
// groups per chunk, partials within `budget`.
int choose_chunks_generic(long long Q, int D, int max_len, size_t budget, int* chunk) {
  const long long target = (long long)sm_count() * 16;
  long long nc = std::max<long long>(1, (target + Q - 1) / Q);
  nc = std::min<long long>(nc, std::max(1, max_len / (4 * kTokU)));
  const long long per = (long long)Q * (D + 2) * 4;
  nc = std::min<long long>(nc, std::max<long long>(1, (long long)budget / std::max<long long>(per, 1)));
  nc = std::min<long long>(nc, 65535);
  *chunk = (int)std::max<long long>(1, (max_len + nc - 1) / nc);
  return std::max(1, (max_len + *chunk - 1) / *chunk);
}

}  // namespace

kq_status_t launch_fa_mha(int kvf, const float* q, const void* k, const void* v, float* out, int B, int S, int H,
                          int D, cudaStream_t s) {
  const long long Q = (long long)B * H;
  if (Q == 0) return KQ_OK;
  if (kvf == KQ_KV_Q8_0 && fa_path() == FaPath::kStream && S > 0) {
    const long long tiles = (long long)((B + 3) / 4) * (H / 8) * ((S + 15) / 16);
    const bool batch = fa_batch_supported(KQ_KV_Q8_0, q, k, v, out, B, S, H, D);
    const bool stream = fa_stream_supported(q, k, v, out, D, H, 1, 0);
    // the small-batch kernel also takes what neither other kernel does (head
    // counts not in groups of 8): the generic kernel is ~3x slower there
    if ((small_batch(tiles, std::min(B, 4)) || (!batch && !stream)) &&
        fa_small_supported(KQ_KV_Q8_0, q, k, v, out, D, H, std::min(B, 4)))
      return launch_fa_small_mha(KQ_KV_Q8_0, q, k, v, out, B, S, H, s);
    if (batch) return launch_fa_batch_mha(KQ_KV_Q8_0, q, k, v, out, B, S, H, s);
    if (stream) return launch_fa_stream_mha(q, k, v, out, B, S, H, s);
  }
  // q4_0 / fp16 caches: the tensor-core batch kernel when its CTAs fill the
  // GPU, else the small-batch kernel (each K / V tile read once for up to 4
  // queries; the generic kernel reads it once per query)
  if (kvf != KQ_KV_Q8_0 && fa_path() == FaPath::kStream && S > 0) {
    if (fa_batch_supported(kvf, q, k, v, out, B, S, H, D)) return launch_fa_batch_mha(kvf, q, k, v, out, B, S, H, s);
    if (fa_small_supported(kvf, q, k, v, out, D, H, std::min(B, 4)))
      return launch_fa_small_mha(kvf, q, k, v, out, B, S, H, s);
  }
  const bool fast = kvf == KQ_KV_Q8_0 && fast_ok(k, v, D, H, 1) && S > 0 &&
                    (long long)((B + kG - 1) / kG) * (H / kHpc) <= 65535;
  int chunk = 0;
  const int NC = fast ? choose_chunks_fast(Q, D, std::max(S, 1), kPartialBudget, ((B + kG - 1) / kG) * (H / kHpc),
                                           &chunk)
                      : choose_chunks_generic(Q, D, std::max(S, 1), kPartialBudget, &chunk);
  const size_t bytes = (size_t)Q * NC * (D + 2) * sizeof(float);
  float* ws = static_cast<float*>(workspace(WS_FA, bytes));
  if (!ws) return KQ_ERR_NOMEM;
  FaParams p{};
  p.q = q; p.k = static_cast<const uint8_t*>(k); p.v = static_cast<const uint8_t*>(v); p.cu = nullptr;
  p.pm = ws; p.pl = ws + Q * NC; p.pacc = ws + 2 * Q * NC; p.out = out;
  p.B = B; p.H = H; p.Hkv = H; p.D = D; p.S = S; p.NC = NC; p.chunk = chunk;
  p.qscale = (float)(1.0 / std::sqrt((double)D) * 1.4426950408889634);
  if (fast) {
    FastParams f{q, nullptr, p.pm, p.pl, p.pacc, B, H, H, S, NC, chunk, H / kHpc, p.qscale};
    const int items = ((B + kG - 1) / kG) * (H / kHpc);
    kq_status_t st = launch_fast<float, false>(f, k, v, (uint64_t)S, H, items, s);
    if (st) return st;
    fa_combine_kernel<float><<<(unsigned)((Q + 3) / 4), 128, 0, s>>>(p, (int)Q);
    return check_launch("fa_combine(mha)");
  }
  dim3 grid(NC, H, (B + kQPerCta - 1) / kQPerCta);
  if (grid.z > 65535 || grid.y > 65535) return fail(KQ_ERR_UNSUPPORTED, "fa_mha: grid too large");
  switch (kvf) {
    case KQ_KV_Q8_0: launch_partial<float, false, KQ_KV_Q8_0>(p, grid, B, s); break;
    case KQ_KV_Q4_0: launch_partial<float, false, KQ_KV_Q4_0>(p, grid, B, s); break;
    case KQ_KV_F16: launch_partial<float, false, KQ_KV_F16>(p, grid, B, s); break;
    default: return fail(KQ_ERR_INVALID, "fa_mha: unknown KV format %d", kvf);
  }
  kq_status_t st = check_launch("fa_partial(mha)");
  if (st) return st;
  fa_combine_kernel<float><<<(unsigned)((Q + 3) / 4), 128, 0, s>>>(p, (int)Q);
  return check_launch("fa_combine(mha)");
}

kq_status_t launch_fa_ragged(const void* q, const void* k, const void* v, const int32_t* cu, int B, int Hq, int Hkv,
                             int D, int max_seqlen, int total_rows, float scale, void* out, cudaStream_t s) {
  const long long Q = (long long)B * Hq;
  if (Q == 0) return KQ_OK;
  const int g = Hq / Hkv;
  if (fa_path() == FaPath::kStream) {
    const long long tiles = (long long)B * std::max(1, Hkv / 8) * ((std::max(max_seqlen, 1) + 15) / 16);
    const bool stream = fa_stream_supported(q, k, v, out, D, Hkv, g, B);
    if ((small_batch(tiles, g) || !stream) && fa_small_supported(KQ_KV_Q8_0, q, k, v, out, D, Hkv, g))
      return launch_fa_small_ragged(q, k, v, cu, B, Hq, Hkv, max_seqlen, total_rows, scale, out, s);
    if (stream) return launch_fa_stream_ragged(q, k, v, cu, B, Hq, Hkv, total_rows, scale, out, s);
  }
  const bool fast = fast_ok(k, v, D, Hkv, g) && total_rows > 0 && (long long)B * (Hkv / kHpc) <= 65535;
  int chunk = 0;
  const int NC = fast ? choose_chunks_fast(Q, D, std::max(max_seqlen, 1), kPartialBudget, B * (Hkv / kHpc), &chunk)
                      : choose_chunks_generic(Q, D, std::max(max_seqlen, 1), kPartialBudget, &chunk);
  const size_t bytes = (size_t)Q * NC * (D + 2) * sizeof(float);
  float* ws = static_cast<float*>(workspace(WS_FA, bytes));
  if (!ws) return KQ_ERR_NOMEM;
  FaParams p{};
  p.q = q; p.k = static_cast<const uint8_t*>(k); p.v = static_cast<const uint8_t*>(v); p.cu = cu;
  p.pm = ws; p.pl = ws + Q * NC; p.pacc = ws + 2 * Q * NC; p.out = out;
  p.B = B; p.H = Hq; p.Hkv = Hkv; p.D = D; p.S = max_seqlen; p.NC = NC; p.chunk = chunk;
  p.qscale = (float)((double)scale * 1.4426950408889634);
  if (fast) {
    // total_rows bounds the TMA map: no tile reads past the cache allocation
    FastParams f{q, cu, p.pm, p.pl, p.pacc, B, Hq, Hkv, max_seqlen, NC, chunk, Hkv / kHpc, p.qscale};
    kq_status_t st = launch_fast<__half, true>(f, k, v, (uint64_t)total_rows, Hkv, B * (Hkv / kHpc), s);
    if (st) return st;
    fa_combine_kernel<__half><<<(unsigned)((Q + 3) / 4), 128, 0, s>>>(p, (int)Q);
    return check_launch("fa_combine(ragged)");
  }
  dim3 grid(NC, (unsigned)((long long)B * Hkv), (g + kQPerCta - 1) / kQPerCta);
  if (grid.y > 65535) return fail(KQ_ERR_UNSUPPORTED, "fa_ragged: B*Hkv too large");
  launch_partial<__half, true, KQ_KV_Q8_0>(p, grid, g, s);
  kq_status_t st = check_launch("fa_partial(ragged)");
  if (st) return st;
  fa_combine_kernel<__half><<<(unsigned)((Q + 3) / 4), 128, 0, s>>>(p, (int)Q);
  return check_launch("fa_combine(ragged)");
}

}  // namespace kq
