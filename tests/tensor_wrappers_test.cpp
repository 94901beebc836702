// The Tensor-typed overloads (include/engine/kernels_b200_tensor.hpp) against
// the engine's own Tensor (include/engine/tensor.hpp, src/tensor.cpp of the
// reference, built unmodified by oracle/Makefile's `tensor` target).
//
//   tensor_wrappers_test cpu   every argument check throws engine::EngineError
//                              with the expected message; no GPU is touched
//   tensor_wrappers_test gpu   each overload's output equals, bit for bit, the
//                              pointer launcher's output on the same inputs
//
// Exit status 0 when every check passes; one line per failure otherwise.
#include <cuda_runtime.h>

#include <engine/kernels_b200.hpp>

#include <cstdio>
#include <cstring>
#include <functional>
#include <random>
#include <string>
#include <vector>

using engine::Device;
using engine::DType;
using engine::Tensor;
namespace ec = engine::cuda;

namespace {

int g_checks = 0, g_failures = 0;

void fail(const std::string& what) {
  ++g_failures;
  std::printf("FAIL: %s\n", what.c_str());
}

void expect_throw(const std::function<void()>& f, const std::string& substr) {
  ++g_checks;
  try {
    f();
    fail("no error, expected '" + substr + "'");
  } catch (const engine::EngineError& e) {
    if (std::string(e.what()).find(substr) == std::string::npos)
      fail("error '" + std::string(e.what()) + "' lacks '" + substr + "'");
  }
}

Tensor cpu(std::vector<std::int64_t> shape, DType dt) { return Tensor(shape, dt, Device::CPU); }

void run_cpu_checks() {
  const Tensor A = cpu({4, 8}, DType::F32), B = cpu({8, 3}, DType::F32);
  Tensor C = cpu({4, 3}, DType::F32);
  expect_throw([&] { ec::matmul_register_tiled(A, B, C); }, "A must be on the CUDA device");
  expect_throw([&] { ec::matmul_naive(A, cpu({7, 3}, DType::F32), C); },
               "B has shape [7, 3], expected [8, 3]");
  expect_throw([&] { ec::matmul_tiled(cpu({4, 8}, DType::F16), B, C); }, "A has dtype");
  expect_throw([&] { ec::matmul_tiled(cpu({8, 4}, DType::F32).transpose(0, 1), B, C); },
               "A must be contiguous");
  expect_throw([&] { ec::matmul_tiled(Tensor(), B, C); }, "A is an undefined tensor");
  expect_throw([&] { ec::matmul_tiled(cpu({32}, DType::F32), B, C); }, "A has 1 dims");
  Tensor y = cpu({3}, DType::F32);
  expect_throw([&] { ec::gemv(cpu({8, 3}, DType::F32), cpu({7}, DType::F32), y); },
               "x has shape [7], expected [8]");
  Tensor n = cpu({4, 8}, DType::F32);
  expect_throw([&] { ec::rmsnorm(A, cpu({7}, DType::F32), n, 1e-5f); }, "weight has shape");
  expect_throw([&] { ec::rmsnorm(A, Tensor(), n, 1e-5f); }, "in must be on the CUDA device");
  Tensor s = cpu({4, 8}, DType::F32);
  expect_throw([&] { ec::residual_rmsnorm(A, cpu({4, 7}, DType::F32), Tensor(), n, s, 1e-5f); },
               "residual has shape [4, 7], expected [4, 8]");
  Tensor o = cpu({4, 2}, DType::F32);
  expect_throw([&] { ec::rmsnorm_linear(A, Tensor(), cpu({8, 2}, DType::F32), o, -1.0f); },
               "in must be on the CUDA device");
  // FP16 / BF16 entry points
  const Tensor X = cpu({16, 64}, DType::F16), W = cpu({32, 64}, DType::F16);
  Tensor Y = cpu({16, 32}, DType::F16);
  expect_throw([&] { ec::linear(X, cpu({32, 63}, DType::F16), Tensor(), Y); },
               "W has shape [32, 63], expected [32, 64]");
  expect_throw([&] { ec::linear(X, W, cpu({16, 31}, DType::F16), Y); }, "residual has shape");
  expect_throw([&] { ec::linear(X, cpu({32, 64}, DType::BF16), Tensor(), Y); }, "W has dtype");
  expect_throw([&] { ec::linear(X, W, Tensor(), Y); }, "X must be on the CUDA device");
  Tensor Cm = cpu({16, 32}, DType::BF16);
  expect_throw([&] { ec::matmul(cpu({16, 64}, DType::BF16), cpu({64, 32}, DType::F16), Cm); },
               "B has dtype");
  Tensor yv = cpu({32}, DType::F16);
  expect_throw([&] { ec::gemv_f16_nk(W, cpu({63}, DType::F16), Tensor(), yv); },
               "x has shape [63], expected [64]");
  expect_throw([&] { ec::rmsnorm_linear_f16(X, cpu({65}, DType::F16), W, Tensor(), Y, 1e-5f); },
               "gamma has shape");
  Tensor Ys = cpu({16, 16}, DType::F16);
  expect_throw([&] { ec::rmsnorm_linear_swiglu_fp16(X, Tensor(), cpu({33, 64}, DType::F16), Ys,
                                                    1e-5f); },
               "even number of rows");
  expect_throw([&] { ec::rmsnorm_linear_swiglu_fp16(X, Tensor(), W, Y, 1e-5f); },
               "Y has shape [16, 32], expected [16, 16]");
}

// ------------------------------------------------------------------ GPU mode

Tensor dev(std::vector<std::int64_t> shape, DType dt, std::mt19937& rng, float scale = 1.0f) {
  Tensor t(shape, dt, Device::CUDA);
  const std::size_t n = static_cast<std::size_t>(t.numel());
  std::normal_distribution<float> nd(0.0f, scale);
  if (dt == DType::F32) {
    std::vector<float> h(n);
    for (auto& v : h) v = nd(rng);
    cudaMemcpy(t.data(), h.data(), n * 4, cudaMemcpyHostToDevice);
  } else {
    std::vector<std::uint16_t> h(n);
    for (auto& v : h) {
      const float f = nd(rng);
      v = dt == DType::F16 ? __half_as_ushort(__float2half(f))
                           : __bfloat16_as_ushort(__float2bfloat16(f));
    }
    cudaMemcpy(t.data(), h.data(), n * 2, cudaMemcpyHostToDevice);
  }
  return t;
}

Tensor like(const Tensor& t) { return Tensor(t.shape(), t.dtype(), Device::CUDA); }

void same(const char* what, const Tensor& a, const Tensor& b) {
  ++g_checks;
  if (cudaDeviceSynchronize() != cudaSuccess) return fail(std::string(what) + ": CUDA error");
  std::vector<unsigned char> ha(a.nbytes()), hb(b.nbytes());
  cudaMemcpy(ha.data(), a.data(), ha.size(), cudaMemcpyDeviceToHost);
  cudaMemcpy(hb.data(), b.data(), hb.size(), cudaMemcpyDeviceToHost);
  if (ha != hb) fail(std::string(what) + ": Tensor overload differs from the pointer launcher");
}

template <class T>
T* P(const Tensor& t) {
  return static_cast<T*>(const_cast<void*>(t.data()));
}

void run_gpu_checks() {
  std::mt19937 rng(20260826);
  {  // FP32 launchers
    Tensor A = dev({64, 96}, DType::F32, rng), B = dev({96, 80}, DType::F32, rng);
    Tensor C1 = like(Tensor({64, 80}, DType::F32, Device::CUDA)), C2 = like(C1);
    ec::matmul_register_tiled(A, B, C1);
    ec::matmul_register_tiled(P<float>(A), P<float>(B), P<float>(C2), 64, 80, 96);
    same("matmul_register_tiled", C1, C2);
    ec::matmul_naive(A, B, C1);
    ec::matmul_naive(P<float>(A), P<float>(B), P<float>(C2), 64, 80, 96);
    same("matmul_naive", C1, C2);
    Tensor x = dev({64}, DType::F32, rng), y1({96}, DType::F32, Device::CUDA), y2 = like(y1);
    ec::gemv(A, x, y1);
    ec::gemv(P<float>(A), P<float>(x), P<float>(y2), 96, 64);
    same("gemv", y1, y2);
    Tensor w = dev({96}, DType::F32, rng), n1 = like(A), n2 = like(A), s1 = like(A), s2 = like(A);
    ec::rmsnorm(A, w, n1, 1e-5f);
    ec::rmsnorm(P<float>(A), P<float>(w), P<float>(n2), 64, 96, 1e-5f);
    same("rmsnorm", n1, n2);
    Tensor R = dev({64, 96}, DType::F32, rng);
    ec::residual_rmsnorm(A, R, Tensor(), n1, s1, 1e-5f);
    ec::residual_rmsnorm(P<float>(A), P<float>(R), nullptr, P<float>(n2), P<float>(s2), 64, 96,
                         1e-5f);
    same("residual_rmsnorm norm", n1, n2);
    same("residual_rmsnorm sum", s1, s2);
    Tensor Wl = dev({96, 40}, DType::F32, rng), o1({64, 40}, DType::F32, Device::CUDA), o2 = like(o1);
    ec::rmsnorm_linear(A, w, Wl, o1, 1e-5f);
    ec::rmsnorm_linear(P<float>(A), P<float>(w), P<float>(Wl), P<float>(o2), 64, 40, 96, 1e-5f);
    same("rmsnorm_linear", o1, o2);
    ec::vector_add(A, R, s1);
    ec::vector_add(P<float>(A), P<float>(R), P<float>(s2), 64 * 96);
    same("vector_add", s1, s2);
  }
  {  // FP16 legacy layout
    Tensor A = dev({256, 128}, DType::F16, rng, 0.05f), x = dev({256}, DType::F16, rng);
    Tensor y1({128}, DType::F16, Device::CUDA), y2 = like(y1);
    ec::gemv_fp16(A, x, y1);
    ec::gemv_fp16(P<__half>(A), P<__half>(x), P<__half>(y2), 128, 256);
    same("gemv_fp16", y1, y2);
    Tensor g = dev({64, 32}, DType::F16, rng), u = dev({64, 32}, DType::F16, rng);
    Tensor o1 = like(g), o2 = like(g);
    ec::swiglu_fp16(g, u, o1);
    ec::swiglu_fp16(P<__half>(g), P<__half>(u), P<__half>(o2), 64 * 32);
    same("swiglu_fp16", o1, o2);
  }
  for (DType dt : {DType::F16, DType::BF16}) {  // tcgen05 entry points
    Tensor A = dev({256, 384}, dt, rng), B = dev({384, 512}, dt, rng);
    Tensor C1({256, 512}, dt, Device::CUDA), C2 = like(C1);
    ec::matmul(A, B, C1);
    if (dt == DType::F16) {
      ec::matmul_f16(P<__half>(A), P<__half>(B), P<__half>(C2), 256, 512, 384);
    } else {
      ec::matmul_bf16(P<__nv_bfloat16>(A), P<__nv_bfloat16>(B), P<__nv_bfloat16>(C2), 256, 512, 384);
    }
    same(dt == DType::F16 ? "matmul f16" : "matmul bf16", C1, C2);
    Tensor X = dev({16, 384}, dt, rng), W = dev({512, 384}, dt, rng, 0.02f), R = dev({16, 512}, dt, rng);
    Tensor Y1({16, 512}, dt, Device::CUDA), Y2 = like(Y1);
    ec::linear(X, W, R, Y1);
    if (dt == DType::F16) {
      ec::linear_f16(P<__half>(X), P<__half>(W), P<__half>(R), P<__half>(Y2), 16, 512, 384);
    } else {
      ec::linear_bf16(P<__nv_bfloat16>(X), P<__nv_bfloat16>(W), P<__nv_bfloat16>(R),
                      P<__nv_bfloat16>(Y2), 16, 512, 384);
    }
    same(dt == DType::F16 ? "linear f16" : "linear bf16", Y1, Y2);
  }
  {  // decode GEMV and fused norm projections
    Tensor W = dev({1024, 2048}, DType::F16, rng, 0.02f), x = dev({2048}, DType::F16, rng);
    Tensor r = dev({1024}, DType::F16, rng), y1({1024}, DType::F16, Device::CUDA), y2 = like(y1);
    ec::gemv_f16_nk(W, x, r, y1);
    ec::gemv_f16_nk(P<__half>(W), P<__half>(x), P<__half>(r), P<__half>(y2), 1024, 2048);
    same("gemv_f16_nk", y1, y2);
    Tensor g = dev({2048}, DType::F16, rng, 0.1f);
    for (std::int64_t M : {1, 16}) {
      Tensor xs = dev({M, 2048}, DType::F16, rng), Y1({M, 1024}, DType::F16, Device::CUDA);
      Tensor Y2 = like(Y1);
      ec::rmsnorm_linear_f16(xs, g, W, Tensor(), Y1, 1e-5f);
      ec::rmsnorm_linear_f16(P<__half>(xs), P<__half>(g), P<__half>(W), nullptr, P<__half>(Y2), M,
                             1024, 2048, 1e-5f);
      same("rmsnorm_linear_f16", Y1, Y2);
      Tensor S1({M, 512}, DType::F16, Device::CUDA), S2 = like(S1);
      ec::rmsnorm_linear_swiglu_fp16(xs, g, W, S1, 1e-5f);
      ec::rmsnorm_linear_swiglu_fp16(P<__half>(xs), P<__half>(g), P<__half>(W), P<__half>(S2), M,
                                     512, 2048, 1e-5f);
      same("rmsnorm_linear_swiglu_fp16", S1, S2);
    }
  }
}

}  // namespace

int main(int argc, char** argv) {
  const std::string mode = argc > 1 ? argv[1] : "cpu";
  try {
    if (mode == "gpu") {
      run_gpu_checks();
    } else {
      run_cpu_checks();
    }
  } catch (const std::exception& e) {
    fail(std::string("unexpected exception: ") + e.what());
  }
  std::printf("tensor_wrappers %s: %d checks, %d failures\n", mode.c_str(), g_checks, g_failures);
  return g_failures == 0 ? 0 : 1;
}
