// ref_cuda_capi.cu -- C shim over the reference engine's OWN CUDA launchers,
// compiled unmodified from the reference tree for sm_100a (oracle/Makefile,
// target `refcuda`, output oracle/_ref/libref_cuda.so).
//
// Test and benchmark infrastructure only: bench.py's baseline leg times these
// sm_89-design kernels beside the library's on the same B200 (the same-box "old
// kernel" comparison); nothing in the product path loads this library.  Each
// entry catches the reference's engine::EngineError and returns 1 (0 = ok), so
// a C caller never sees a C++ exception.
//
// Wrapped launchers (namespace engine::cuda, include/engine/kernels.hpp of the
// reference): matmul_register_tiled :80, matmul_tiled :74, gemv :85,
// gemv_fp16 :120, rmsnorm_linear :97.
#include <cstdint>
#include <cstdio>
#include <exception>

#include <engine/kernels.hpp>

namespace {
template <class F>
int guarded(F&& f) {
  try {
    f();
    return 0;
  } catch (const std::exception& e) {
    std::fprintf(stderr, "ref_cuda: %s\n", e.what());
    return 1;
  }
}
}  // namespace

extern "C" {

int refcuda_matmul_register_tiled(const float* A, const float* B, float* C, int64_t M, int64_t N,
                                  int64_t K, void* stream) {
  return guarded([&] {
    engine::cuda::matmul_register_tiled(A, B, C, M, N, K, static_cast<cudaStream_t>(stream));
  });
}

int refcuda_matmul_tiled(const float* A, const float* B, float* C, int64_t M, int64_t N,
                         int64_t K, void* stream) {
  return guarded(
      [&] { engine::cuda::matmul_tiled(A, B, C, M, N, K, static_cast<cudaStream_t>(stream)); });
}

int refcuda_gemv(const float* A, const float* x, float* out, int64_t N, int64_t K, void* stream) {
  return guarded([&] { engine::cuda::gemv(A, x, out, N, K, static_cast<cudaStream_t>(stream)); });
}

int refcuda_gemv_fp16(const void* A, const void* x, void* out, int64_t N, int64_t K,
                      void* stream) {
  return guarded([&] {
    engine::cuda::gemv_fp16(static_cast<const engine::half*>(A),
                            static_cast<const engine::half*>(x), static_cast<engine::half*>(out),
                            N, K, static_cast<cudaStream_t>(stream));
  });
}

int refcuda_rmsnorm_linear(const float* in, const float* w, const float* W, float* out, int64_t M,
                           int64_t N, int64_t K, float eps, void* stream) {
  return guarded([&] {
    engine::cuda::rmsnorm_linear(in, w, W, out, M, N, K, eps, static_cast<cudaStream_t>(stream));
  });
}

}  // extern "C"
