// Flash-attention decode for small batches over a q8_0, q4_0 or fp16 KV
// cache (D = 128): at most 4 queries per KV head and too few tiles for the
// balanced stream kernel (fa_stream.cu) to fill the GPU (a single sequence,
// or a harness batch of 1-8 queries); for q4_0 and fp16 caches every harness
// batch the tensor-core batch kernel (fa_batch.cu) does not take. Semantics
// as the harness flash_attention operator
// (kernelevalplus-main/llm_kernel_test/op_test_handler.py:543-563):
// out = softmax(q . K^T * scale) . V per (query, head), K and V stored as
// q8_0 or q4_0 blocks along head_dim or as fp16 (op_test_handler.py:489-534).
// In the ragged form (q8_0) sequence b owns cache rows cu[b] .. cu[b+1]-1
// and query head h reads KV head h / (Hq / Hkv).
//
// Why a separate kernel: the stream kernel's CTA is 8 warps over a tile of
// 16 tokens x 8 KV heads, so one sequence gives ~14 tiles per SM, processed
// one after another by a single CTA with a long per-tile chain. Here every
// warp is independent: a "unit" is (sequence or group of 4 harness queries,
// KV head) and a warp takes one contiguous token chunk of one unit. It
// streams that head's 16-token K and V tiles through its own two-stage TMA
// ring (boxes of 16 rows x 144 bytes: the head's 136-byte row starts 0 or 8
// bytes in, keeping the box 16-byte aligned), so 20 warps per SM stream
// independently.
//   QK  lanes = (token t, half): each lane forms the int32 block dots of its
//       token's two 32-dim blocks with the query held as two int8 levels
//       (q ~ s1 c1 + s2 c2, s2 = s1 / 127, so 127 dot1 + dot2 is the exact
//       block dot at scale s2), applies the per-(token, block) K scale, and
//       the halves are added with one shuffle.
//   softmax  online, per query, in log2 units (scale * log2 e folded into q).
//   PV  lanes = 4 dims: for each token, its V codes times p * d_v accumulate
//       in fp32 (no conversion to a second operand format).
// q4_0: the box row is the head's 72 bytes plus 8; QK turns the nibbles into
// the int8 codes q - 8 for the same dp4a dots, PV decodes them. fp16: the
// row is the head's 256 bytes as two 128-byte-swizzled boxes (rows of a
// half tile in distinct banks); QK is an fp32 dot of the fp32 query with
// the fp16 row, PV takes the fp16 values with weight p.
// Each warp writes its chunk's (m, l, acc) per query; a merge kernel combines
// the chunks of each query.
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

constexpr int kTok = 16;                  // tokens per tile
constexpr int kWarps = 4;                 // warps per CTA (independent tasks)
constexpr int kStages = 2;                // TMA ring depth per warp
constexpr int kQ = 4;                     // queries per unit (at most)

// Per-warp shared memory by cache format: K and V rings, the queries (int8
// codes [4 queries][2 levels][128] for the block formats, fp32 [4][128] for
// fp16), barriers. Block formats: a smem row is the head's 136- (q8_0) or
// 72-byte (q4_0) row plus 8 bytes before or after it. fp16: a row is the
// head's 256 bytes as two 128-byte halves, each half tile (16 rows) stored
// with the 128-byte swizzle (1024-byte aligned).
template <int KVF>
struct SmallFmt {
  static constexpr int kBlk = KVF == KQ_KV_Q8_0 ? 34 : 18;     // block formats: bytes per 32 dims
  static constexpr int kUnits = 4 * kBlk / 8;                   // the head's row in 8-byte units (17, 9)
  static constexpr int kRow = KVF == KQ_KV_F16 ? 256 : 8 * (kUnits + 1);
  static constexpr int kTile = kTok * kRow;                     // 2304, 1280, 4096 bytes
  static constexpr int kOffV = kStages * kTile;
  static constexpr int kOffQ = 2 * kStages * kTile;
  static constexpr int kOffBar = kOffQ + (KVF == KQ_KV_F16 ? kQ * 128 * 4 : kQ * 2 * 128);
  static constexpr int kAlign = KVF == KQ_KV_F16 ? 1024 : 128;
  static constexpr int kWarpSmem = (kOffBar + kStages * 8 + kAlign - 1) / kAlign * kAlign;
  static constexpr int kSmem = kWarps * kWarpSmem + kAlign;    // + base alignment slack
  static_assert(kTile % kAlign == 0 && kWarpSmem % kAlign == 0, "TMA destinations stay aligned");
};

struct SmallParams {
  const void* q;          // ragged: fp16 [B, Hq, 128]; MHA: fp32 [B, H, 128]
  const int32_t* cu;      // ragged: cu_seqlens [B + 1]; MHA: nullptr
  float* pm;              // [unit][chunk / 4][4]: one partial per CTA (4 chunks)
  float* pl;
  float* pacc;            // [unit][chunk / 4][4][128]
  void* out;
  int* err;
  int nunits;             // groups x KV heads
  int nchunk;             // chunks per unit (token chunks of `chunk` tokens), a multiple of 4
  int chunk;              // tokens per chunk (multiple of 16)
  int B, H, Hkv;          // MHA: B queries, H heads (= KV heads); ragged: B sequences, H = Hq
  int S;                  // MHA: cache length
  float qscale;           // softmax scale * log2(e)
};

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

// 2^x by the hardware approximation (ex2.approx: relative error ~2^-22)
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float4 load_q4(const float* q, size_t i) { return *reinterpret_cast<const float4*>(q + i); }
__device__ __forceinline__ float4 load_q4(const __half* q, size_t i) {
  const uint2 u = *reinterpret_cast<const uint2*>(q + i);
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
  return make_float4(a.x, a.y, b.x, b.y);
}

// Four nibbles (one per byte) -> four int8 codes q - 8 (no borrow between
// bytes: every byte is at least 0x80 before the subtraction)
__device__ __forceinline__ uint32_t nibbles_s8(uint32_t x) {
  return ((x | 0x80808080u) - 0x08080808u) ^ 0x80808080u;
}

__device__ __forceinline__ uint32_t pack_s8x4(int a, int b, int c, int d) {
  return (uint32_t)(a & 0xFF) | ((uint32_t)(b & 0xFF) << 8) | ((uint32_t)(c & 0xFF) << 16) | ((uint32_t)d << 24);
}

// Unit u = (group, KV head): its token rows, queries and KV head.
template <bool RAGGED>
__device__ __forceinline__ void unit_of(const SmallParams& p, int u, int& grp, int& hk, int& row0, int& len,
                                        int& nq) {
  grp = u / p.Hkv;
  hk = u % p.Hkv;
  if (RAGGED) {
    row0 = p.cu[grp];
    len = p.cu[grp + 1] - row0;
    nq = p.H / p.Hkv;
  } else {
    row0 = 0;
    len = p.S;
    nq = min(kQ, p.B - grp * kQ);
  }
}

template <bool RAGGED>
__device__ __forceinline__ size_t query_index(const SmallParams& p, int grp, int hk, int j) {
  if (RAGGED) return (size_t)grp * p.H + (size_t)hk * (p.H / p.Hkv) + j;
  return (size_t)(grp * kQ + j) * p.H + hk;
}

template <typename QT, bool RAGGED, int NQ, int KVF>
__global__ void __launch_bounds__(32 * kWarps)
    fa_small_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                    SmallParams p) {
  using F = SmallFmt<KVF>;
  constexpr int kRow = F::kRow, kTile = F::kTile, kBlk = F::kBlk;
  extern __shared__ uint8_t smem_raw[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* cta = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + F::kAlign - 1) &
                                            ~(uintptr_t)(F::kAlign - 1));
  uint8_t* ws = cta + warp * F::kWarpSmem;
  uint64_t* full = reinterpret_cast<uint64_t*>(ws + F::kOffBar);
  int8_t* qc = reinterpret_cast<int8_t*>(ws + F::kOffQ);   // block formats: [query][level][128]
  float* qf = reinterpret_cast<float*>(ws + F::kOffQ);     // fp16: [query][128]
  // launched as a programmatic dependent: no global read before the
  // preceding kernel (the previous call's merge, or the queries' producer) ends
  pdl_wait();

  // the grid covers exactly nunits * nchunk tasks (nchunk % kWarps == 0), so
  // the CTA's warps hold consecutive chunks of one unit and all reach the
  // merge barrier at the end
  const int task = blockIdx.x * kWarps + warp;
  const int u = task / p.nchunk, c = task % p.nchunk;
  int grp, hk, row0, len, nq;
  unit_of<RAGGED>(p, u, grp, hk, row0, len, nq);
  const int t0 = c * p.chunk, t1 = min(len, t0 + p.chunk);
  const int ntiles = t1 > t0 ? (t1 - t0 + kTok - 1) / kTok : 0;
  const int xoff = KVF == KQ_KV_F16 ? 0 : (hk & 1) * 8;  // block formats: the head's first byte in a row
  const int bx = F::kUnits * hk - (hk & 1);              // block formats: box start in 8-byte units

  if (lane == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
  }
  __syncwarp();
  auto issue = [&](int i) {
    const int s = i % kStages;
    const int y = row0 + t0 + i * kTok;
    mbar_arrive_expect_tx(&full[s], 2 * kTile);
    if constexpr (KVF == KQ_KV_F16) {
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        tma_load_2d(ws + s * kTile + hf * (kTile / 2), &kmap, 128 * hk + 64 * hf, y, &full[s]);
        tma_load_2d(ws + F::kOffV + s * kTile + hf * (kTile / 2), &vmap, 128 * hk + 64 * hf, y, &full[s]);
      }
    } else {
      tma_load_2d(ws + s * kTile, &kmap, bx, y, &full[s]);
      tma_load_2d(ws + F::kOffV + s * kTile, &vmap, bx, y, &full[s]);
    }
  };
  if (lane == 0)
    for (int i = 0; i < min(kStages, ntiles); ++i) issue(i);

  // ---- queries (lane = dims 4 lane .. 4 lane + 3): fp32 for fp16 caches,
  // else two int8 levels ----
  float s2[NQ];  // level-2 scale of each query: score = s2 * sum_b d_k (127 dot1 + dot2)
#pragma unroll
  for (int j = 0; j < NQ; ++j) {
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (j < nq) {
      const QT* qp = static_cast<const QT*>(p.q) + query_index<RAGGED>(p, grp, hk, j) * 128;
      const float4 t = load_q4(qp, 4 * lane);
      v[0] = t.x * p.qscale; v[1] = t.y * p.qscale; v[2] = t.z * p.qscale; v[3] = t.w * p.qscale;
    }
    if constexpr (KVF == KQ_KV_F16) {
      reinterpret_cast<float4*>(qf + j * 128)[lane] = make_float4(v[0], v[1], v[2], v[3]);
      s2[j] = 1.0f;
    } else {
      const float a = warp_max(fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3]))));
      const float s1 = a > 0.0f ? a / 127.0f : 1.0f;
      const float inv1 = a > 0.0f ? 127.0f / a : 0.0f;
      const float inv2 = 127.0f * inv1;
      int c1[4], c2[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        c1[i] = max(-127, min(127, __float2int_rn(v[i] * inv1)));
        c2[i] = max(-127, min(127, __float2int_rn(fmaf(-s1, (float)c1[i], v[i]) * inv2)));
      }
      reinterpret_cast<uint32_t*>(qc + (j * 2) * 128)[lane] = pack_s8x4(c1[0], c1[1], c1[2], c1[3]);
      reinterpret_cast<uint32_t*>(qc + (j * 2 + 1) * 128)[lane] = pack_s8x4(c2[0], c2[1], c2[2], c2[3]);
      s2[j] = s1 * (1.0f / 127.0f);
    }
  }
  __syncwarp();

  float m_run[NQ], l_run[NQ], acc[NQ][4];
#pragma unroll
  for (int j = 0; j < NQ; ++j) {
    m_run[j] = -INFINITY;
    l_run[j] = 0.0f;
    acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.0f;
  }
  const int tq = lane & 15, half = lane >> 4;  // QK: token, block pair {2 half, 2 half + 1} (dims 64 half ..)
  const int vb = lane >> 3;                     // PV: block of this lane's 4 dims
  // PV: this lane's 4 codes. q8_0: bytes 4 (lane % 8) .. of block vb; q4_0:
  // element e = 4 (lane % 8) of the block is the low nibble of byte e for
  // e < 16, else the high nibble of byte e - 16; fp16: bytes 8 lane .. of
  // the row, in half lane / 16 at swizzled chunk ((lane % 16) / 2) ^ (row % 8)
  const int voff = KVF == KQ_KV_Q8_0   ? xoff + vb * kBlk + 2 + 4 * (lane & 7)
                   : KVF == KQ_KV_Q4_0 ? xoff + vb * kBlk + 2 + 4 * (lane & 3)
                                       : (lane >> 4) * (kTile / 2) + 8 * (lane & 1);
  const int vshift = (lane & 4) ? 4 : 0;        // q4_0: high nibbles for elements 16-31
  bool dead = false;

  for (int i = 0; i < ntiles; ++i) {
    const int s = i % kStages;
    const int nvalid = min(kTok, t1 - (t0 + i * kTok));
    mbar_wait_or_poison(&full[s], (i / kStages) & 1, p.err, DEV_TIMEOUT_FULL, dead);
    const uint8_t* kt = ws + s * kTile;
    const uint8_t* vt = ws + F::kOffV + s * kTile;

    // ---- QK: token tq, blocks 2 half and 2 half + 1 ----
    float sc[NQ];
    {
      float part[NQ];
#pragma unroll
      for (int j = 0; j < NQ; ++j) part[j] = 0.0f;
      if constexpr (KVF == KQ_KV_F16) {
        // dims 64 half .. + 63: the row's half `half`, 16-byte chunk c at c ^ (tq % 8)
        const uint8_t* row = kt + half * (kTile / 2) + tq * 128;
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
          const uint4 kw = *reinterpret_cast<const uint4*>(row + ((cc ^ (tq & 7)) << 4));
          const float2 k0 = __half22float2(*reinterpret_cast<const __half2*>(&kw.x));
          const float2 k1 = __half22float2(*reinterpret_cast<const __half2*>(&kw.y));
          const float2 k2 = __half22float2(*reinterpret_cast<const __half2*>(&kw.z));
          const float2 k3 = __half22float2(*reinterpret_cast<const __half2*>(&kw.w));
#pragma unroll
          for (int j = 0; j < NQ; ++j) {
            const float4* qv = reinterpret_cast<const float4*>(qf + j * 128 + 64 * half + 8 * cc);
            const float4 a = qv[0], b = qv[1];
            float x = part[j];
            x = fmaf(a.x, k0.x, x); x = fmaf(a.y, k0.y, x); x = fmaf(a.z, k1.x, x); x = fmaf(a.w, k1.y, x);
            x = fmaf(b.x, k2.x, x); x = fmaf(b.y, k2.y, x); x = fmaf(b.z, k3.x, x); x = fmaf(b.w, k3.y, x);
            part[j] = x;
          }
        }
      } else {
        const uint8_t* row = kt + tq * kRow + xoff;
        int d1[NQ], d2[NQ];
#pragma unroll
        for (int bi = 0; bi < 2; ++bi) {
          const int blk = 2 * half + bi;
          const uint8_t* b = row + kBlk * blk;
          const float dk = lds_half(b);
          uint32_t kw[8];  // codes of dims 4 w .. 4 w + 3 of the block
          if constexpr (KVF == KQ_KV_Q8_0) {
#pragma unroll
            for (int w = 0; w < 8; ++w) kw[w] = lds_u32_a2(b + 2 + 4 * w);
          } else {
#pragma unroll
            for (int w = 0; w < 4; ++w) {
              const uint32_t x = lds_u32_a2(b + 2 + 4 * w);
              kw[w] = nibbles_s8(x & 0x0F0F0F0Fu);
              kw[4 + w] = nibbles_s8((x >> 4) & 0x0F0F0F0Fu);
            }
          }
#pragma unroll
          for (int j = 0; j < NQ; ++j) {
            const uint4* q1 = reinterpret_cast<const uint4*>(qc + (j * 2) * 128 + 32 * blk);
            const uint4* q2 = reinterpret_cast<const uint4*>(qc + (j * 2 + 1) * 128 + 32 * blk);
            const uint4 a0 = q1[0], a1 = q1[1], b0 = q2[0], b1 = q2[1];
            d1[j] = __dp4a((int)kw[0], (int)a0.x, 0);
            d1[j] = __dp4a((int)kw[1], (int)a0.y, d1[j]);
            d1[j] = __dp4a((int)kw[2], (int)a0.z, d1[j]);
            d1[j] = __dp4a((int)kw[3], (int)a0.w, d1[j]);
            d1[j] = __dp4a((int)kw[4], (int)a1.x, d1[j]);
            d1[j] = __dp4a((int)kw[5], (int)a1.y, d1[j]);
            d1[j] = __dp4a((int)kw[6], (int)a1.z, d1[j]);
            d1[j] = __dp4a((int)kw[7], (int)a1.w, d1[j]);
            d2[j] = __dp4a((int)kw[0], (int)b0.x, 0);
            d2[j] = __dp4a((int)kw[1], (int)b0.y, d2[j]);
            d2[j] = __dp4a((int)kw[2], (int)b0.z, d2[j]);
            d2[j] = __dp4a((int)kw[3], (int)b0.w, d2[j]);
            d2[j] = __dp4a((int)kw[4], (int)b1.x, d2[j]);
            d2[j] = __dp4a((int)kw[5], (int)b1.y, d2[j]);
            d2[j] = __dp4a((int)kw[6], (int)b1.z, d2[j]);
            d2[j] = __dp4a((int)kw[7], (int)b1.w, d2[j]);
            part[j] = fmaf(dk, (float)(127 * d1[j] + d2[j]), part[j]);
          }
        }
      }
#pragma unroll
      for (int j = 0; j < NQ; ++j) {
        const float tot = part[j] + __shfl_xor_sync(0xffffffffu, part[j], 16);
        sc[j] = tq < nvalid ? tot * s2[j] : -INFINITY;
      }
    }

    // ---- online softmax per query (lanes 0-15 and 16-31 hold the same scores) ----
    float pj[NQ];
#pragma unroll
    for (int j = 0; j < NQ; ++j) {
      float mx = sc[j];
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
      const float m_new = fmaxf(m_run[j], mx);
      const float corr = (m_run[j] == -INFINITY) ? 0.0f : ex2(m_run[j] - m_new);
      m_run[j] = m_new;
      pj[j] = sc[j] == -INFINITY ? 0.0f : ex2(sc[j] - m_new);
      float ls = pj[j];
      ls += __shfl_xor_sync(0xffffffffu, ls, 1);
      ls += __shfl_xor_sync(0xffffffffu, ls, 2);
      ls += __shfl_xor_sync(0xffffffffu, ls, 4);
      ls += __shfl_xor_sync(0xffffffffu, ls, 8);
      l_run[j] = fmaf(l_run[j], corr, ls);
      acc[j][0] *= corr; acc[j][1] *= corr; acc[j][2] *= corr; acc[j][3] *= corr;
    }

    // ---- PV: lane = dims 4 lane .. 4 lane + 3 (block vb) ----
#pragma unroll 4
    for (int t = 0; t < kTok; ++t) {
      float dv, v0, v1, v2, v3;
      if constexpr (KVF == KQ_KV_F16) {
        const uint2 w = *reinterpret_cast<const uint2*>(vt + voff + t * 128 + ((((lane & 15) >> 1) ^ (t & 7)) << 4));
        const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&w.x));
        const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&w.y));
        dv = t < nvalid ? 1.0f : 0.0f;  // masked tokens weigh nothing
        v0 = a.x; v1 = a.y; v2 = b.x; v3 = b.y;
      } else {
        const uint8_t* row = vt + t * kRow;
        dv = t < nvalid ? lds_half(row + xoff + kBlk * vb) : 0.0f;  // masked tokens weigh nothing
        const uint32_t w = lds_u32_a2(row + voff);
        if constexpr (KVF == KQ_KV_Q8_0) {
          v0 = (float)(int8_t)(w & 0xFF); v1 = (float)(int8_t)((w >> 8) & 0xFF);
          v2 = (float)(int8_t)((w >> 16) & 0xFF); v3 = (float)(int8_t)(w >> 24);
        } else {
          const uint32_t x = (w >> vshift) & 0x0F0F0F0Fu;
          v0 = (float)((int)(x & 0xF) - 8); v1 = (float)((int)((x >> 8) & 0xF) - 8);
          v2 = (float)((int)((x >> 16) & 0xF) - 8); v3 = (float)((int)(x >> 24) - 8);
        }
      }
#pragma unroll
      for (int j = 0; j < NQ; ++j) {
        const float wt = __shfl_sync(0xffffffffu, pj[j], t) * dv;
        acc[j][0] = fmaf(wt, v0, acc[j][0]);
        acc[j][1] = fmaf(wt, v1, acc[j][1]);
        acc[j][2] = fmaf(wt, v2, acc[j][2]);
        acc[j][3] = fmaf(wt, v3, acc[j][3]);
      }
    }
    // the stage is no longer read: refill it with tile i + kStages
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0 && i + kStages < ntiles) issue(i + kStages);
  }

  // ---- merge the CTA's kWarps chunks per query in shared memory (each warp
  // writes its state into its own ring, which its TMA no longer fills) ----
  float* mine = reinterpret_cast<float*>(ws);  // [NQ][132]: m, l, 2 spare, acc[128] (16-byte aligned)
#pragma unroll
  for (int j = 0; j < NQ; ++j) {
    if (lane == 0) {
      mine[j * 132] = m_run[j];
      mine[j * 132 + 1] = l_run[j];
    }
    *reinterpret_cast<float4*>(mine + j * 132 + 4 + 4 * lane) = make_float4(acc[j][0], acc[j][1], acc[j][2], acc[j][3]);
  }
  __syncthreads();
  if (warp != 0) return;
  const size_t base = ((size_t)u * (p.nchunk / kWarps) + c / kWarps) * kQ;
#pragma unroll
  for (int j = 0; j < NQ; ++j) {
    if (j >= nq) continue;
    float mw[kWarps], M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      mw[w] = reinterpret_cast<const float*>(cta + w * F::kWarpSmem)[j * 132];
      M = fmaxf(M, mw[w]);
    }
    float L = 0.0f;
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        const float* st = reinterpret_cast<const float*>(cta + w * F::kWarpSmem) + j * 132;
        const float wg = mw[w] == -INFINITY ? 0.0f : ex2(mw[w] - M);
        L = fmaf(st[1], wg, L);
        const float4 x = *reinterpret_cast<const float4*>(st + 4 + 4 * lane);
        a.x = fmaf(x.x, wg, a.x);
        a.y = fmaf(x.y, wg, a.y);
        a.z = fmaf(x.z, wg, a.z);
        a.w = fmaf(x.w, wg, a.w);
      }
    }
    if (lane == 0) {
      p.pm[base + j] = M;
      p.pl[base + j] = L;
    }
    reinterpret_cast<float4*>(p.pacc + (base + j) * 128)[lane] = a;
  }
}

// One warp per query: merge the chunk partials of its unit. Lane = 4 dims.
template <typename OT, bool RAGGED>
__global__ void __launch_bounds__(128) fa_small_combine_kernel(SmallParams p, int Q) {
  pdl_wait();  // the decode grid's partials
  pdl_launch_dependents();  // a following decode waits for this grid in turn
  const int qg = blockIdx.x * 4 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (qg >= Q) return;
  int grp, hk, j;
  if (RAGGED) {
    const int g = p.H / p.Hkv;
    grp = qg / p.H;
    const int rem = qg % p.H;
    hk = rem / g;
    j = rem % g;
  } else {
    const int b = qg / p.H;
    hk = qg % p.H;
    grp = b / kQ;
    j = b % kQ;
  }
  const int np = p.nchunk / kWarps;  // partials per unit (one per CTA)
  const size_t base = ((size_t)(grp * p.Hkv + hk) * np) * kQ + j;  // partial c at base + 4 c
  float M = -INFINITY;
  for (int c0 = 0; c0 < np; c0 += 32)
    if (c0 + lane < np) M = fmaxf(M, p.pm[base + (size_t)(c0 + lane) * kQ]);
  M = warp_max(M);
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  float L = 0.0f;
  if (M != -INFINITY) {
    for (int c0 = 0; c0 < np; c0 += 32) {
      const int cnt = min(32, np - c0);
      const size_t pi = base + (size_t)(c0 + lane) * kQ;
      const float mc = lane < cnt ? p.pm[pi] : -INFINITY;
      const float lc = lane < cnt ? p.pl[pi] : 0.0f;
      const float wgt = mc == -INFINITY ? 0.0f : ex2(mc - M);
      for (int k0 = 0; k0 < cnt; k0 += 8) {
        float4 a[8];
        float wk[8];
#pragma unroll
        for (int x = 0; x < 8; ++x) {
          const int k = k0 + x;
          wk[x] = __shfl_sync(0xffffffffu, wgt, k & 31);
          a[x] = (k < cnt && wk[x] != 0.0f)
                     ? reinterpret_cast<const float4*>(p.pacc + (base + (size_t)(c0 + k) * kQ) * 128)[lane]
                     : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int x = 0; x < 8; ++x) {
          const int k = k0 + x;
          const float lk = __shfl_sync(0xffffffffu, lc, k & 31);
          if (k < cnt && wk[x] != 0.0f) {
            L = fmaf(lk, wk[x], L);
            acc.x = fmaf(a[x].x, wk[x], acc.x);
            acc.y = fmaf(a[x].y, wk[x], acc.y);
            acc.z = fmaf(a[x].z, wk[x], acc.z);
            acc.w = fmaf(a[x].w, wk[x], acc.w);
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

bool encode_head_map(CUtensorMap* map, const void* base, uint64_t rows, int heads, int kv_format) {
  auto fn = reinterpret_cast<EncodeTiledFn>(tensor_map_encoder());
  if (!fn) return false;
  cuuint32_t estr[2] = {1, 1};
  if (kv_format == KQ_KV_F16) {
    // [rows][heads * 128] fp16; boxes of 16 rows x 64 elements (one half of
    // a head's row) with the 128-byte swizzle; past the last row the fill is zero
    cuuint64_t dims[2] = {(cuuint64_t)heads * 128, rows};
    cuuint64_t strides[1] = {(cuuint64_t)heads * 256};
    cuuint32_t box[2] = {64, kTok};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
  }
  // [rows][heads * units 8-byte elements] (units = 17 for q8_0's 136-byte
  // head rows, 9 for q4_0's 72); boxes of 16 rows x (units + 1) elements
  // (one head's row plus 8 bytes before or after it, so every box starts on
  // a 16-byte boundary; past the last row the fill is zero)
  const int units = kv_format == KQ_KV_Q8_0 ? 17 : 9;
  cuuint64_t dims[2] = {(cuuint64_t)heads * units, rows};
  cuuint64_t strides[1] = {(cuuint64_t)heads * units * 8};
  cuuint32_t box[2] = {(cuuint32_t)units + 1, kTok};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Token chunks per unit: about 20 resident warps per SM in total (five
// 4-warp CTAs), each chunk a whole number of 16-token tiles, the count a
// multiple of the CTA's 4 warps and at most 128 (32 partials per query after
// the in-CTA merge).
void choose_chunks(int nunits, int max_len, int* nchunk, int* chunk) {
  const long long target = 20LL * sm_count();
  const int max_tiles = std::max(1, (max_len + kTok - 1) / kTok);
  long long nc = std::max<long long>(1, (target + nunits - 1) / nunits);
  nc = std::min<long long>(nc, std::min(max_tiles, 128));
  const int tiles_per = (int)((max_tiles + nc - 1) / nc);
  *chunk = tiles_per * kTok;
  const int used = (max_len + *chunk - 1) / *chunk;
  *nchunk = std::max(kWarps, (used + kWarps - 1) / kWarps * kWarps);
}

template <typename QT, typename OT, bool RAGGED, int NQ, int KVF>
kq_status_t launch(SmallParams p, const void* k, const void* v, uint64_t rows, int heads, long long Q,
                   cudaStream_t s) {
  CUtensorMap km, vm;
  if (!encode_head_map(&km, k, rows, heads, KVF) || !encode_head_map(&vm, v, rows, heads, KVF))
    return fail(KQ_ERR_CUDA, "fa_small: KV tensor map rejected");
  auto kern = fa_small_kernel<QT, RAGGED, NQ, KVF>;
  constexpr int kSmem = SmallFmt<KVF>::kSmem;
  kq_status_t st = ensure_dynamic_smem(reinterpret_cast<const void*>(kern), kSmem, "fa_small smem attribute");
  if (st) return st;
  const long long tasks = (long long)p.nunits * p.nchunk;
  {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((tasks + kWarps - 1) / kWarps));
    cfg.blockDim = dim3(32 * kWarps);
    cfg.dynamicSmemBytes = kSmem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, km, vm, p);
    if (e != cudaSuccess) return check_cuda(e, "fa_small launch");
  }
  if ((st = check_launch("fa_small"))) return st;
  // a programmatic dependent of the decode kernel: its launch overlaps the decode
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
  cudaError_t e = cudaLaunchKernelEx(&cfg, fa_small_combine_kernel<OT, RAGGED>, p, (int)Q);
  if (e != cudaSuccess) return check_cuda(e, "fa_small_combine launch");
  return check_launch("fa_small_combine");
}

template <typename QT, typename OT, bool RAGGED, int KVF>
kq_status_t launch_nq(int nq, SmallParams p, const void* k, const void* v, uint64_t rows, int heads, long long Q,
                      cudaStream_t s) {
  if (nq <= 1) return launch<QT, OT, RAGGED, 1, KVF>(p, k, v, rows, heads, Q, s);
  if (nq <= 2) return launch<QT, OT, RAGGED, 2, KVF>(p, k, v, rows, heads, Q, s);
  return launch<QT, OT, RAGGED, 4, KVF>(p, k, v, rows, heads, Q, s);
}

SmallParams carve(void* ws, int nunits, int nchunk) {
  SmallParams p{};
  const size_t n = (size_t)nunits * (nchunk / kWarps) * kQ;
  float* f = static_cast<float*>(ws);
  p.pm = f;
  p.pl = f + n;
  p.pacc = f + 2 * n;
  p.nunits = nunits;
  p.nchunk = nchunk;
  return p;
}

size_t scratch_bytes(int nunits, int nchunk) {
  return (size_t)nunits * (nchunk / kWarps) * kQ * (2 + 128) * sizeof(float);
}

}  // namespace

bool fa_small_supported(int kv_format, const void* q, const void* k, const void* v, const void* out, int D,
                        int Hkv, int queries_per_unit) {
  auto al = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; };
  // block formats: an even head count keeps every head's 16-byte aligned box inside the rows
  const bool heads = kv_format == KQ_KV_F16 ? Hkv >= 1
                                            : (kv_format == KQ_KV_Q8_0 || kv_format == KQ_KV_Q4_0) && Hkv >= 2 &&
                                                  Hkv % 2 == 0;
  return heads && D == 128 && queries_per_unit >= 1 && queries_per_unit <= kQ && al(q) && al(k) && al(v) &&
         al(out);
}

kq_status_t launch_fa_small_mha(int kv_format, const float* q, const void* k, const void* v, float* out, int B,
                                int S, int H, cudaStream_t s) {
  const int ngrp = (B + kQ - 1) / kQ;
  const int nunits = ngrp * H;
  int nchunk = 1, chunk = kTok;
  choose_chunks(nunits, S, &nchunk, &chunk);
  void* ws = workspace(WS_FA, scratch_bytes(nunits, nchunk));
  if (!ws) return KQ_ERR_NOMEM;
  SmallParams p = carve(ws, nunits, nchunk);
  p.q = q;
  p.cu = nullptr;
  p.out = out;
  p.err = device_error_word();
  p.chunk = chunk;
  p.B = B;
  p.H = H;
  p.Hkv = H;
  p.S = S;
  p.qscale = (float)(1.0 / std::sqrt(128.0) * 1.4426950408889634);
  const int nq = std::min(B, kQ);
  const uint64_t rows = (uint64_t)std::max(S, 1);
  switch (kv_format) {
    case KQ_KV_Q8_0: return launch_nq<float, float, false, KQ_KV_Q8_0>(nq, p, k, v, rows, H, (long long)B * H, s);
    case KQ_KV_Q4_0: return launch_nq<float, float, false, KQ_KV_Q4_0>(nq, p, k, v, rows, H, (long long)B * H, s);
    case KQ_KV_F16: return launch_nq<float, float, false, KQ_KV_F16>(nq, p, k, v, rows, H, (long long)B * H, s);
    default: return fail(KQ_ERR_INVALID, "fa_small: unknown KV format %d", kv_format);
  }
}

kq_status_t launch_fa_small_ragged(const void* q, const void* k, const void* v, const int32_t* cu, int B, int Hq,
                                   int Hkv, int max_seqlen, int total_rows, float scale, void* out, cudaStream_t s) {
  const int nunits = B * Hkv;
  int nchunk = 1, chunk = kTok;
  choose_chunks(nunits, std::max(max_seqlen, 1), &nchunk, &chunk);
  void* ws = workspace(WS_FA, scratch_bytes(nunits, nchunk));
  if (!ws) return KQ_ERR_NOMEM;
  SmallParams p = carve(ws, nunits, nchunk);
  p.q = q;
  p.cu = cu;
  p.out = out;
  p.err = device_error_word();
  p.chunk = chunk;
  p.B = B;
  p.H = Hq;
  p.Hkv = Hkv;
  p.S = max_seqlen;
  p.qscale = (float)((double)scale * 1.4426950408889634);
  return launch_nq<__half, __half, true, KQ_KV_Q8_0>(Hq / Hkv, p, k, v, (uint64_t)std::max(total_rows, 1), Hkv,
                                                     (long long)B * Hq, s);
}

}  // namespace kq
