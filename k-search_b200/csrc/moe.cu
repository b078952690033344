// Grouped q4_0 MoE expert FFN (benchmark configuration 4):
//
//   route:   p = softmax(logits[t, :]), top-k experts (ties -> lower index),
//            weights renormalised over the k chosen
//   per expert e and its routed tokens X_e:
//            h = silu(X_e W_gate[e]^T) * (X_e W_up[e]^T)      (activations q8_1-quantised)
//            y = h W_down[e]^T                               (h q8_1-quantised)
//   combine: out[t] = sum_k w[t, k] * y[pair(t, k)]          (fixed slot order)
//
// The reference has no grouped MoE operator; each expert GEMM is the
// per-definition W4A32C8 operator (e.g. definitions/quant_gemm/mixtral8x7b/
// w4a32c8_q4_0_fp32_int8_mixtral8x7b_moe_up_n14336_k4096.json), and SiLU
// follows kernels/activation/silu.cuh:97 (silu(g) * u).
//
// Pipeline (all on one stream): route_kernel -> expert_rank_kernel (a stable
// counting sort of (token, slot) pairs by expert) -> gather_quantize (routed
// rows of x into the GEMM staging layout, expert-contiguous) -> per-expert
// gate / up GEMMs (tcgen05 / GEMV / generic by size, on row ranges of the
// shared staging) -> silu_mul_quantize (h straight into staging) -> per-expert
// down GEMMs -> combine_kernel. Expert row counts come back to the host once
// per call to size the per-expert launches.
#include <algorithm>
#include <cmath>

#include "kq_internal.h"
#include "kq_device.cuh"

namespace kq {
namespace {

constexpr int kMaxExperts = 64;
constexpr int kMaxTopk = 8;

// One thread per token: softmax over E logits, top-k, renormalised weights.
__global__ void route_kernel(const float* __restrict__ logits, int T, int E, int topk, int* __restrict__ idx,
                             float* __restrict__ wts, int* __restrict__ counts) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  const float* l = logits + (size_t)t * E;
  float mx = -INFINITY;
  for (int e = 0; e < E; ++e) mx = fmaxf(mx, l[e]);
  float den = 0.0f;
  for (int e = 0; e < E; ++e) den += expf(l[e] - mx);
  int chosen[kMaxTopk];
  float pw[kMaxTopk];
  float tot = 0.0f;
  for (int k = 0; k < topk; ++k) {
    int best = -1;
    float bv = -INFINITY;
    for (int e = 0; e < E; ++e) {
      bool used = false;
      for (int q = 0; q < k; ++q) used |= (chosen[q] == e);
      if (!used && (best < 0 || l[e] > bv)) {
        best = e;
        bv = l[e];
      }
    }
    chosen[k] = best;
    pw[k] = expf(bv - mx) / den;
    tot += pw[k];
  }
  for (int k = 0; k < topk; ++k) {
    idx[(size_t)t * topk + k] = chosen[k];
    wts[(size_t)t * topk + k] = pw[k] / tot;
    atomicAdd(&counts[chosen[k]], 1);
  }
}

// Block e lists the pairs routed to expert e in (token, slot) order: a stable
// counting sort. row_of_pair[t * topk + k] = row of that pair in the grouped
// layout; pair_of_row[row] = t * topk + k.
__global__ void __launch_bounds__(1024) expert_rank_kernel(const int* __restrict__ idx, const int* __restrict__ counts,
                                                           int P, int E, int* __restrict__ row_of_pair,
                                                           int* __restrict__ pair_of_row) {
  const int e = blockIdx.x;
  __shared__ int base;
  __shared__ int warp_tot[32];
  if (threadIdx.x == 0) {
    int b = 0;
    for (int q = 0; q < e; ++q) b += counts[q];
    base = b;
  }
  __syncthreads();
  int running = base;
  for (int c0 = 0; c0 < P; c0 += blockDim.x) {
    const int i = c0 + threadIdx.x;
    const int flag = (i < P && idx[i] == e) ? 1 : 0;
    // block-wide exclusive scan of flags
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    int v = flag;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += n;
    }
    if (lane == 31) warp_tot[wid] = v;
    __syncthreads();
    if (wid == 0) {
      int w = (lane < (int)(blockDim.x >> 5)) ? warp_tot[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += n;
      }
      warp_tot[lane] = w;  // inclusive prefix over warps
    }
    __syncthreads();
    const int before = (wid > 0 ? warp_tot[wid - 1] : 0) + v - flag;
    if (flag) {
      const int row = running + before;
      row_of_pair[i] = row;
      pair_of_row[row] = i;
    }
    const int chunk_total = warp_tot[(blockDim.x >> 5) - 1];
    __syncthreads();
    running += chunk_total;
  }
}

// y[t] = sum_k w[t,k] * Y[row_of_pair[t*topk+k]]   (fp32, fixed slot order;
// row_of_pair == nullptr: Y is already in (token, slot) order)
__global__ void combine_kernel(const float* __restrict__ Y, const int* __restrict__ row_of_pair,
                               const float* __restrict__ wts, int T, int topk, int H, float* __restrict__ out) {
  const int t = blockIdx.x;
  for (int h = threadIdx.x * 4; h < H; h += blockDim.x * 4) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k = 0; k < topk; ++k) {
      const float w = wts[(size_t)t * topk + k];
      const size_t pr = (size_t)t * topk + k;
      const size_t r = row_of_pair ? (size_t)row_of_pair[pr] : pr;
      const float4 y = *reinterpret_cast<const float4*>(Y + r * H + h);
      acc.x = fmaf(w, y.x, acc.x);
      acc.y = fmaf(w, y.y, acc.y);
      acc.z = fmaf(w, y.z, acc.z);
      acc.w = fmaf(w, y.w, acc.w);
    }
    *reinterpret_cast<float4*>(out + (size_t)t * H + h) = acc;
  }
}

// Per-row unsort: y[p] = Y[row_of_pair[p]].
__global__ void unsort_kernel(const float* __restrict__ Y, const int* __restrict__ row_of_pair, int H,
                              float* __restrict__ y) {
  const int p = blockIdx.x;
  const float* src = Y + (size_t)row_of_pair[p] * H;
  float* dst = y + (size_t)p * H;
  for (int h = threadIdx.x * 4; h < H; h += blockDim.x * 4)
    *reinterpret_cast<float4*>(dst + h) = *reinterpret_cast<const float4*>(src + h);
}

// Row unsort of any row width (16-byte multiple): dst row p = src row row_of_pair[p].
__global__ void unsort_rows_kernel(const uint8_t* __restrict__ src, const int* __restrict__ row_of_pair,
                                   size_t row_bytes, uint8_t* __restrict__ dst) {
  const int p = blockIdx.x;
  const uint4* s = reinterpret_cast<const uint4*>(src + (size_t)row_of_pair[p] * row_bytes);
  uint4* d = reinterpret_cast<uint4*>(dst + (size_t)p * row_bytes);
  for (size_t i = threadIdx.x; i < row_bytes / 16; i += blockDim.x) d[i] = s[i];
}

// h = silu(gate) * up elementwise, the value the SiLU quantiser quantises.
__global__ void silu_mul_kernel(const float* __restrict__ g, const float* __restrict__ u, long long n,
                                float* __restrict__ h) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    h[i] = silu_mul(g[i], u[i]);
}

__global__ void count_kernel(const int* __restrict__ expert_of_pair, int P, int* __restrict__ counts) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < P) atomicAdd(&counts[expert_of_pair[i]], 1);
}

}  // namespace

// ---------------------------------------------------------------------------
size_t moe_workspace_bytes(int P, int E, int H, int I) {
  size_t b = 0;
  auto add = [&](size_t n) { b += (n + 255) & ~(size_t)255; };
  add(E * sizeof(int));                 // counts
  add((size_t)P * sizeof(int));         // idx (routing) / expert of pair
  add((size_t)P * sizeof(float));       // wts
  add((size_t)P * sizeof(int));         // row_of_pair
  add((size_t)P * sizeof(int));         // pair_of_row
  add(act8_bytes(P, H));                // staged x rows
  add((size_t)P * I * sizeof(float));   // gate
  add((size_t)P * I * sizeof(float));   // up
  add(act8_bytes(P, I));                // staged h
  add((size_t)P * H * sizeof(float));   // y (grouped)
  return b;
}

namespace {

struct MoeWs {
  int* counts;
  int* idx;
  float* wts;
  int* row_of_pair;
  int* pair_of_row;
  Act8 ax;
  float* G;
  float* U;
  Act8 ah;
  float* Y;
};

bool moe_ws(int P, int E, int H, int I, MoeWs* w) {
  uint8_t* ws = static_cast<uint8_t*>(workspace(WS_MOE, moe_workspace_bytes(P, E, H, I)));
  if (!ws) return false;
  size_t off = 0;
  auto take = [&](size_t n) {
    uint8_t* q = ws + off;
    off += (n + 255) & ~(size_t)255;
    return q;
  };
  w->counts = reinterpret_cast<int*>(take(E * sizeof(int)));
  w->idx = reinterpret_cast<int*>(take((size_t)P * sizeof(int)));
  w->wts = reinterpret_cast<float*>(take((size_t)P * sizeof(float)));
  w->row_of_pair = reinterpret_cast<int*>(take((size_t)P * sizeof(int)));
  w->pair_of_row = reinterpret_cast<int*>(take((size_t)P * sizeof(int)));
  w->ax = act8_view(take(act8_bytes(P, H)), P, H);
  w->G = reinterpret_cast<float*>(take((size_t)P * I * sizeof(float)));
  w->U = reinterpret_cast<float*>(take((size_t)P * I * sizeof(float)));
  w->ah = act8_view(take(act8_bytes(P, I)), P, I);
  w->Y = reinterpret_cast<float*>(take((size_t)P * H * sizeof(float)));
  return true;
}

// Expert FFNs of P routed rows. Row p reads x row p / div (or, with a_q8_1,
// row p of those pre-quantised q8_1 rows) and goes to expert
// expert_of_pair[p] (w.counts already holds the per-expert row counts). The
// result for row p lands in w.Y[w.row_of_pair[p]].
kq_status_t moe_core(const float* x, int div, const int* expert_of_pair, int P, int E, const void* w_gate,
                     const void* w_up, const void* w_down, int H, int I, int act_mode, MoeWs& w, cudaStream_t s,
                     const void* a_q8_1 = nullptr) {
  expert_rank_kernel<<<E, 1024, 0, s>>>(expert_of_pair, w.counts, P, E, w.row_of_pair, w.pair_of_row);
  kq_status_t st = check_launch("moe rank");
  if (st) return st;
  int hc[kMaxExperts];
  if ((st = check_cuda(cudaMemcpyAsync(hc, w.counts, E * sizeof(int), cudaMemcpyDeviceToHost, s), "moe counts d2h")))
    return st;
  if ((st = check_cuda(cudaStreamSynchronize(s), "moe counts sync"))) return st;
  if (a_q8_1) {
    if ((st = launch_q8_1_to_act_gather(a_q8_1, w.pair_of_row, w.ax, P, H, s))) return st;
  } else if ((st = launch_quantize_act_gather(x, w.pair_of_row, div, w.ax, P, H, act_mode, s))) {
    return st;
  }
  const size_t gate_bytes = (size_t)I * (H / 32) * 18, down_bytes = (size_t)H * (I / 32) * 18;
  auto rows = [](Act8 a, int r0, int K) { return Act8{a.qs + (size_t)r0 * K, a.ds + (size_t)r0 * (K / 32)}; };
  int r0 = 0;
  for (int e = 0; e < E; ++e) {
    const int m = hc[e];
    if (m > 0) {
      const Act8 a = rows(w.ax, r0, H);
      if ((st = gemm_any(KQ_Q4_0, static_cast<const uint8_t*>(w_gate) + e * gate_bytes, a, w.G + (size_t)r0 * I, m,
                         I, H, s)))
        return st;
      if ((st = gemm_any(KQ_Q4_0, static_cast<const uint8_t*>(w_up) + e * gate_bytes, a, w.U + (size_t)r0 * I, m, I,
                         H, s)))
        return st;
    }
    r0 += m;
  }
  if ((st = launch_silu_mul_quantize(w.G, w.U, w.ah, P, I, act_mode, s))) return st;
  r0 = 0;
  for (int e = 0; e < E; ++e) {
    const int m = hc[e];
    if (m > 0) {
      if ((st = gemm_any(KQ_Q4_0, static_cast<const uint8_t*>(w_down) + e * down_bytes, rows(w.ah, r0, I),
                         w.Y + (size_t)r0 * H, m, H, I, s)))
        return st;
    }
    r0 += m;
  }
  return KQ_OK;
}

kq_status_t check_moe(int E, int topk, int H, int I) {
  if (E < 1 || E > kMaxExperts || topk < 1 || topk > kMaxTopk || topk > E)
    return fail(KQ_ERR_INVALID, "moe: unsupported E=%d topk=%d", E, topk);
  if (H % 32 || I % 32) return fail(KQ_ERR_INVALID, "moe: H and I must be multiples of 32");
  return KQ_OK;
}

}  // namespace

kq_status_t launch_moe_route(const float* logits, int T, int E, int topk, int* idx, float* wts, cudaStream_t s) {
  kq_status_t st = check_moe(E, topk, 32, 32);
  if (st || T == 0) return st;
  int* counts = static_cast<int*>(workspace(WS_MOE2, E * sizeof(int)));
  if (!counts) return KQ_ERR_NOMEM;
  if ((st = check_cuda(cudaMemsetAsync(counts, 0, E * sizeof(int), s), "moe counts"))) return st;
  route_kernel<<<(T + 127) / 128, 128, 0, s>>>(logits, T, E, topk, idx, wts, counts);
  return check_launch("moe route");
}

kq_status_t launch_moe_combine(const float* y, const float* wts, int T, int topk, int H, float* out, cudaStream_t s) {
  if (T == 0) return KQ_OK;
  combine_kernel<<<T, 256, 0, s>>>(y, nullptr, wts, T, topk, H, out);
  return check_launch("moe combine");
}

kq_status_t launch_moe_experts_q4_0(const float* x_rows, const int* expert_of_row, const void* w_gate,
                                    const void* w_up, const void* w_down, int E, int P, int H, int I, int act_mode,
                                    float* y_rows, cudaStream_t s, const MoeStages* stages, const void* a_q8_1) {
  kq_status_t st = check_moe(E, 1, H, I);
  if (st || P == 0) return st;
  MoeWs w;
  if (!moe_ws(P, E, H, I, &w)) return KQ_ERR_NOMEM;
  if ((st = check_cuda(cudaMemsetAsync(w.counts, 0, E * sizeof(int), s), "moe counts"))) return st;
  count_kernel<<<(P + 255) / 256, 256, 0, s>>>(expert_of_row, P, w.counts);
  if ((st = check_launch("moe count"))) return st;
  if ((st = moe_core(x_rows, 1, expert_of_row, P, E, w_gate, w_up, w_down, H, I, act_mode, w, s, a_q8_1)))
    return st;
  unsort_kernel<<<P, 256, 0, s>>>(w.Y, w.row_of_pair, H, y_rows);
  if ((st = check_launch("moe unsort"))) return st;
  if (stages) {
    // the pipeline's own intermediates, back in the input row order
    const size_t fbytes = (size_t)I * sizeof(float);
    auto unsort = [&](const void* src, size_t row_bytes, void* dst) {
      unsort_rows_kernel<<<P, 128, 0, s>>>(static_cast<const uint8_t*>(src), w.row_of_pair, row_bytes,
                                           static_cast<uint8_t*>(dst));
      return check_launch("moe stage unsort");
    };
    if ((st = unsort(w.G, fbytes, stages->gate)) || (st = unsort(w.U, fbytes, stages->up))) return st;
    // h of the grouped rows, formed by the same function as the quantiser, into the gate buffer's
    // successor (the grouped G is no longer needed once it has been copied out)
    silu_mul_kernel<<<std::min<long long>(4096, ((long long)P * I + 255) / 256), 256, 0, s>>>(w.G, w.U,
                                                                                            (long long)P * I, w.G);
    if ((st = check_launch("moe stage silu"))) return st;
    if ((st = unsort(w.G, fbytes, stages->h))) return st;
    if ((st = unsort(w.ah.qs, (size_t)I, stages->h_qs))) return st;
    if ((st = unsort(w.ah.ds, (size_t)(I / 32) * sizeof(float2), stages->h_ds))) return st;
  }
  return KQ_OK;
}

kq_status_t launch_moe_q4_0(const float* x, const float* logits, const void* w_gate, const void* w_up,
                            const void* w_down, int E, int topk, int T, int H, int I, int act_mode, float* out,
                            cudaStream_t s) {
  kq_status_t st = check_moe(E, topk, H, I);
  if (st) return st;
  const int P = T * topk;
  MoeWs w;
  if (!moe_ws(P, E, H, I, &w)) return KQ_ERR_NOMEM;
  if ((st = check_cuda(cudaMemsetAsync(w.counts, 0, E * sizeof(int), s), "moe counts"))) return st;
  route_kernel<<<(T + 127) / 128, 128, 0, s>>>(logits, T, E, topk, w.idx, w.wts, w.counts);
  if ((st = check_launch("moe route"))) return st;
  if ((st = moe_core(x, topk, w.idx, P, E, w_gate, w_up, w_down, H, I, act_mode, w, s))) return st;
  combine_kernel<<<T, 256, 0, s>>>(w.Y, w.row_of_pair, w.wts, T, topk, H, out);
  return check_launch("moe combine");
}

}  // namespace kq
