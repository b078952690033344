// KernelEvalPlus attempt file for quant_gemm definitions with block_q4_1 weights and fp32
// activations (W4A32C8) (copy to kernel.cu in the attempt
// directory). The harness binds the first `extern "C" void` in kernel.cu
// through its generated PyTorch wrapper
// (kernelevalplus-main/llm_kernel_test/op_test_handler.py:298-349) and
// compiles the file for compute_100/sm_100, which cannot hold tcgen05 code;
// this host-only forwarder calls kq_w4a32c8_q4_1_fp32_int8 in the prebuilt sm_100a library
// libkq.so (path in $KQ_LIB, else the loader's search path).
#include <cstdint>
#include <cstdlib>
#include <dlfcn.h>
#include <stdexcept>
#include <string>

namespace {
using entry_t = void (*)(const uint8_t*, const float*, float*, int, int, int);
using err_t = const char* (*)();

struct KqLib {
  entry_t fn = nullptr;
  err_t last_error = nullptr;
  KqLib() {
    const char* path = std::getenv("KQ_LIB");
    void* h = dlopen(path ? path : "libkq.so", RTLD_NOW | RTLD_LOCAL);
    if (!h) throw std::runtime_error(std::string("cannot load libkq: ") + dlerror());
    fn = reinterpret_cast<entry_t>(dlsym(h, "kq_w4a32c8_q4_1_fp32_int8"));
    last_error = reinterpret_cast<err_t>(dlsym(h, "kq_last_error"));
    if (!fn || !last_error) throw std::runtime_error("libkq entry point kq_w4a32c8_q4_1_fp32_int8 not found");
  }
};
}  // namespace

extern "C" void quant_gemm_q4_1(const uint8_t* weight, const float* activation, float* output, int M, int N, int K) {
  static KqLib lib;
  lib.fn(weight, activation, output, M, N, K);
  const char* e = lib.last_error();
  if (e && *e) throw std::runtime_error(std::string("libkq: ") + e);
}
