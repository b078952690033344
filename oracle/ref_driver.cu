// Thin C-ABI driver around the reference's own CPU GEMM / quantize routines.
//
// TEST INFRASTRUCTURE ONLY. Built by oracle/Makefile from the reference
// headers where they lie in the qhy991/K-Search checkout
// (kernelevalplus-main/include/{quant_types.h,quantize.h,gemm_reference.h});
// the output goes to oracle/_ref/libkqref.so, which is git-ignored. The
// shipped library never links or loads it: bench.py's cpu_baseline leg and
// the tests use it as the reference CPU path.
//
// Each entry splits rows across host threads and calls the reference routine
// unchanged on each slice:
//   quantize_row_q8_1_ref   include/quantize.h:165-193
//   gemm_w4a8_reference     include/gemm_reference.h:175-222
//   gemm_w8a8_reference     include/gemm_reference.h:233-267
#include "quant_types.h"
#include "quantize.h"
#include "gemm_reference.h"

#include <algorithm>
#include <cstdint>
#include <thread>
#include <vector>

namespace {
template <class F>
void parallel_rows(int rows, int threads, F&& f) {
  threads = std::max(1, std::min(threads, rows));
  std::vector<std::thread> pool;
  const int per = (rows + threads - 1) / threads;
  for (int t = 0; t < threads; ++t) {
    const int r0 = t * per, r1 = std::min(rows, r0 + per);
    if (r0 >= r1) break;
    pool.emplace_back([=, &f] { f(r0, r1); });
  }
  for (auto& th : pool) th.join();
}

// gemm_w{4,8}a8_reference write C[i*N + j] for their own N, so a slice of
// the weight rows gets its own output buffer that is scattered back.
template <class WBlock, class G>
void gemm_split(const block_q8_1* A, const WBlock* B, float* C, int M, int N, int K, int threads, G gemm) {
  const int nb = K / 32;
  if (M >= threads || N < 2 * threads) {
    parallel_rows(M, threads, [&](int m0, int m1) {
      gemm(A + (size_t)m0 * nb, B, C + (size_t)m0 * N, m1 - m0, N, K);
    });
    return;
  }
  parallel_rows(N, threads, [&](int n0, int n1) {
    std::vector<float> tmp((size_t)M * (n1 - n0));
    gemm(A, B + (size_t)n0 * nb, tmp.data(), M, n1 - n0, K);
    for (int m = 0; m < M; ++m)
      std::copy(tmp.begin() + (size_t)m * (n1 - n0), tmp.begin() + (size_t)(m + 1) * (n1 - n0), C + (size_t)m * N + n0);
  });
}
}  // namespace

extern "C" {

int kqref_quantize_q8_1(const float* x, void* y, int M, int K, int threads) {
  if (K % 32) return 1;
  const int nb = K / 32;
  block_q8_1* out = static_cast<block_q8_1*>(y);
  parallel_rows(M, threads, [&](int m0, int m1) {
    for (int m = m0; m < m1; ++m) quantize_row_q8_1_ref(x + (size_t)m * K, out + (size_t)m * nb, K);
  });
  return 0;
}

int kqref_gemm_w4a8(const void* a_q8_1, const void* w_q4_0, float* c, int M, int N, int K, int threads) {
  if (K % 32) return 1;
  gemm_split(static_cast<const block_q8_1*>(a_q8_1), static_cast<const block_q4_0*>(w_q4_0), c, M, N, K, threads,
             [](const block_q8_1* A, const block_q4_0* B, float* C, int m, int n, int k) { gemm_w4a8_reference(A, B, C, m, n, k); });
  return 0;
}

int kqref_gemm_w8a8(const void* a_q8_1, const void* w_q8_0, float* c, int M, int N, int K, int threads) {
  if (K % 32) return 1;
  gemm_split(static_cast<const block_q8_1*>(a_q8_1), static_cast<const block_q8_0*>(w_q8_0), c, M, N, K, threads,
             [](const block_q8_1* A, const block_q8_0* B, float* C, int m, int n, int k) { gemm_w8a8_reference(A, B, C, m, n, k); });
  return 0;
}

}  // extern "C"
