#pragma once
//===----------------------------------------------------------------------===//
// engine/kernels_b200_tensor.hpp -- Tensor-typed overloads of the B200 launchers.
//
// The engine keeps raw pointers at the kernel boundary and plans Tensor-aware
// overloads "as thin wrappers that unpack .data() and .shape() and forward"
// (include/engine/kernels.hpp:16-17, ADR 0003).  These are those wrappers for
// the GEMM, GEMV, norm, norm->projection, SwiGLU and vector-add launchers of
// this library: same names, the engine's Tensor (include/engine/tensor.hpp) in
// place of pointer + dims, stream last.
//
// Each wrapper checks its tensors before forwarding: for every argument in
// turn, defined (an undefined Tensor is allowed only where the pointer API
// takes null), dtype, contiguity and shape; then that all are on the CUDA
// device.  A failure throws
// engine::EngineError naming the function, the argument and what was
// expected.  Shapes are row-major, outermost first: W[N,K] for the [N,K]
// entry points, A[K,N] for the engine's legacy gemv / gemv_fp16.
//
// Included by kernels_b200.hpp when <engine/tensor.hpp> is on the include path.
//===----------------------------------------------------------------------===//

#include <engine/tensor.hpp>

#include <cstdint>
#include <initializer_list>
#include <string>
#include <utility>
#include <vector>

namespace engine::cuda {

namespace b200_detail {

inline std::string shape_str(const std::vector<std::int64_t>& s) {
  std::string out = "[";
  for (std::size_t i = 0; i < s.size(); ++i) out += (i ? ", " : "") + std::to_string(s[i]);
  return out + "]";
}

[[noreturn]] inline void fail(const char* fn, const std::string& msg) {
  throw ::engine::EngineError(std::string("[engine] ") + fn + ": " + msg);
}

/// Checks one tensor argument.  `want` lists the expected extents; -1 accepts
/// any extent there.  Returns the device pointer (null for an allowed
/// undefined tensor).
inline const void* arg(const char* fn, const char* name, const Tensor& t, DType dt,
                       const std::vector<std::int64_t>& want, bool optional = false) {
  if (!t.defined()) {
    if (optional) return nullptr;
    fail(fn, std::string(name) + " is an undefined tensor");
  }
  if (t.dtype() != dt)
    fail(fn, std::string(name) + " has dtype " + dtype_name(t.dtype()) + ", expected " +
                 dtype_name(dt));
  if (!t.is_contiguous()) fail(fn, std::string(name) + " must be contiguous");
  bool ok = t.shape().size() == want.size();
  for (std::size_t i = 0; ok && i < want.size(); ++i) ok = want[i] < 0 || t.shape()[i] == want[i];
  if (!ok)
    fail(fn, std::string(name) + " has shape " + shape_str(t.shape()) + ", expected " +
                 shape_str(want));
  return t.data();
}

/// The device check, run after every argument's dtype and shape were checked.
inline void cuda_all(const char* fn,
                     std::initializer_list<std::pair<const char*, const Tensor*>> args) {
  for (const auto& a : args)
    if (a.second->defined() && a.second->device() != Device::CUDA)
      fail(fn, std::string(a.first) + " must be on the CUDA device");
}

inline void* dst(const char* fn, const char* name, Tensor& t, DType dt,
                 const std::vector<std::int64_t>& want) {
  return const_cast<void*>(arg(fn, name, t, dt, want));
}

inline std::int64_t extent(const char* fn, const char* name, const Tensor& t, int axis) {
  if (!t.defined()) fail(fn, std::string(name) + " is an undefined tensor");
  if (axis < 0 || t.dim() <= axis)
    fail(fn, std::string(name) + " has " + std::to_string(t.dim()) + " dims, expected " +
                 std::to_string(axis < 0 ? 1 : axis + 1) + " or more");
  return t.shape()[static_cast<std::size_t>(axis)];
}

template <typename T>
T* as(const void* p) {
  return static_cast<T*>(const_cast<void*>(p));
}

}  // namespace b200_detail

// -- legacy FP32 / [K,N] launchers (kernels.hpp:62-121) ------------------------

/// in[rows, cols] (any leading dims are rows), weight[cols] or undefined.
inline void rmsnorm(const Tensor& in, const Tensor& weight, Tensor& out, float eps,
                    cudaStream_t stream = 0) {
  using namespace b200_detail;
  const char* fn = "rmsnorm";
  const std::int64_t cols = extent(fn, "in", in, static_cast<int>(in.dim()) - 1);
  const std::int64_t rows = cols > 0 ? in.numel() / cols : 0;
  const void* x = arg(fn, "in", in, DType::F32, in.shape());
  const void* w = arg(fn, "weight", weight, DType::F32, {cols}, true);
  void* y = dst(fn, "out", out, DType::F32, in.shape());
  cuda_all(fn, {{"in", &in}, {"weight", &weight}, {"out", &out}});
  rmsnorm(as<float>(x), as<float>(w), as<float>(y), rows, cols, eps, stream);
}

/// sum_out = x + residual; norm_out = rmsnorm(sum_out) * weight (weight may be undefined).
inline void residual_rmsnorm(const Tensor& x, const Tensor& residual, const Tensor& weight,
                             Tensor& norm_out, Tensor& sum_out, float eps,
                             cudaStream_t stream = 0) {
  using namespace b200_detail;
  const char* fn = "residual_rmsnorm";
  const std::int64_t cols = extent(fn, "x", x, static_cast<int>(x.dim()) - 1);
  const std::int64_t rows = cols > 0 ? x.numel() / cols : 0;
  const void* px = arg(fn, "x", x, DType::F32, x.shape());
  const void* pr = arg(fn, "residual", residual, DType::F32, x.shape());
  const void* pw = arg(fn, "weight", weight, DType::F32, {cols}, true);
  void* pn = dst(fn, "norm_out", norm_out, DType::F32, x.shape());
  void* ps = dst(fn, "sum_out", sum_out, DType::F32, x.shape());
  cuda_all(fn, {{"x", &x}, {"residual", &residual}, {"weight", &weight}, {"norm_out", &norm_out}, {"sum_out", &sum_out}});
  residual_rmsnorm(as<float>(px), as<float>(pr), as<float>(pw), as<float>(pn), as<float>(ps),
                   rows, cols, eps, stream);
}

#define ENGINE_B200_TENSOR_MATMUL(NAME)                                                    \
  inline void NAME(const Tensor& A, const Tensor& B, Tensor& C, cudaStream_t stream = 0) { \
    using namespace b200_detail;                                                           \
    const char* fn = #NAME;                                                                \
    const std::int64_t M = extent(fn, "A", A, 0), K = extent(fn, "A", A, 1);              \
    const std::int64_t N = extent(fn, "B", B, 1);                                          \
    const void* a = arg(fn, "A", A, DType::F32, {M, K});                                   \
    const void* b = arg(fn, "B", B, DType::F32, {K, N});                                   \
    void* c = dst(fn, "C", C, DType::F32, {M, N});                                         \
    cuda_all(fn, {{"A", &A}, {"B", &B}, {"C", &C}});                                        \
    NAME(as<float>(a), as<float>(b), as<float>(c), M, N, K, stream);                      \
  }
ENGINE_B200_TENSOR_MATMUL(matmul_naive)
ENGINE_B200_TENSOR_MATMUL(matmul_tiled)
ENGINE_B200_TENSOR_MATMUL(matmul_register_tiled)
#undef ENGINE_B200_TENSOR_MATMUL

/// out[N] = x[K] * A[K,N] (the engine's [K,N] layout), FP32.
inline void gemv(const Tensor& A, const Tensor& x, Tensor& out, cudaStream_t stream = 0) {
  using namespace b200_detail;
  const char* fn = "gemv";
  const std::int64_t K = extent(fn, "A", A, 0), N = extent(fn, "A", A, 1);
  const void* pa = arg(fn, "A", A, DType::F32, {K, N});
  const void* px = arg(fn, "x", x, DType::F32, {K});
  void* py = dst(fn, "out", out, DType::F32, {N});
  cuda_all(fn, {{"A", &A}, {"x", &x}, {"out", &out}});
  gemv(as<float>(pa), as<float>(px), as<float>(py), N, K, stream);
}

/// out[N] = x[K] * A[K,N], FP16.
inline void gemv_fp16(const Tensor& A, const Tensor& x, Tensor& out, cudaStream_t stream = 0) {
  using namespace b200_detail;
  const char* fn = "gemv_fp16";
  const std::int64_t K = extent(fn, "A", A, 0), N = extent(fn, "A", A, 1);
  const void* pa = arg(fn, "A", A, DType::F16, {K, N});
  const void* px = arg(fn, "x", x, DType::F16, {K});
  void* py = dst(fn, "out", out, DType::F16, {N});
  cuda_all(fn, {{"A", &A}, {"x", &x}, {"out", &out}});
  gemv_fp16(as<__half>(pa), as<__half>(px), as<__half>(py), N, K, stream);
}

/// out[M,N] = rmsnorm(in[M,K], rms_weight[K] or undefined) * W[K,N], FP32.
inline void rmsnorm_linear(const Tensor& in, const Tensor& rms_weight, const Tensor& W,
                           Tensor& out, float eps, cudaStream_t stream = 0) {
  using namespace b200_detail;
  const char* fn = "rmsnorm_linear";
  const std::int64_t M = extent(fn, "in", in, 0), K = extent(fn, "in", in, 1);
  const std::int64_t N = extent(fn, "W", W, 1);
  const void* px = arg(fn, "in", in, DType::F32, {M, K});
  const void* pg = arg(fn, "rms_weight", rms_weight, DType::F32, {K}, true);
  const void* pw = arg(fn, "W", W, DType::F32, {K, N});
  void* py = dst(fn, "out", out, DType::F32, {M, N});
  cuda_all(fn, {{"in", &in}, {"rms_weight", &rms_weight}, {"W", &W}, {"out", &out}});
  rmsnorm_linear(as<float>(px), as<float>(pg), as<float>(pw), as<float>(py), M, N, K, eps,
                 stream);
}

inline void vector_add(const Tensor& a, const Tensor& b, Tensor& out, cudaStream_t stream = 0) {
  using namespace b200_detail;
  const char* fn = "vector_add";
  const void* pa = arg(fn, "a", a, DType::F32, a.shape());
  const void* pb = arg(fn, "b", b, DType::F32, a.shape());
  void* po = dst(fn, "out", out, DType::F32, a.shape());
  cuda_all(fn, {{"a", &a}, {"b", &b}, {"out", &out}});
  vector_add(as<float>(pa), as<float>(pb), as<float>(po), a.numel(), stream);
}

inline void swiglu_fp16(const Tensor& gate, const Tensor& up, Tensor& out,
                        cudaStream_t stream = 0) {
  using namespace b200_detail;
  const char* fn = "swiglu_fp16";
  const void* pg = arg(fn, "gate", gate, DType::F16, gate.shape());
  const void* pu = arg(fn, "up", up, DType::F16, gate.shape());
  void* po = dst(fn, "out", out, DType::F16, gate.shape());
  cuda_all(fn, {{"gate", &gate}, {"up", &up}, {"out", &out}});
  swiglu_fp16(as<__half>(pg), as<__half>(pu), as<__half>(po), gate.numel(), stream);
}

// -- B200 entry points: FP16 / BF16, [N,K] weights -----------------------------

/// C[M,N] = A[M,K] * B[K,N] on tcgen05; F16 or BF16 (all three the same).
inline void matmul(const Tensor& A, const Tensor& B, Tensor& C, cudaStream_t stream = 0) {
  using namespace b200_detail;
  const char* fn = "matmul";
  const DType dt = A.defined() && A.dtype() == DType::BF16 ? DType::BF16 : DType::F16;
  const std::int64_t M = extent(fn, "A", A, 0), K = extent(fn, "A", A, 1);
  const std::int64_t N = extent(fn, "B", B, 1);
  const void* pa = arg(fn, "A", A, dt, {M, K});
  const void* pb = arg(fn, "B", B, dt, {K, N});
  void* pc = dst(fn, "C", C, dt, {M, N});
  cuda_all(fn, {{"A", &A}, {"B", &B}, {"C", &C}});
  if (dt == DType::BF16) {
    matmul_bf16(as<__nv_bfloat16>(pa), as<__nv_bfloat16>(pb), as<__nv_bfloat16>(pc), M, N, K,
                stream);
  } else {
    matmul_f16(as<__half>(pa), as<__half>(pb), as<__half>(pc), M, N, K, stream);
  }
}

/// Y[M,N] = X[M,K] * W[N,K]^T (+ residual[M,N], or undefined); F16 or BF16.
inline void linear(const Tensor& X, const Tensor& W, const Tensor& residual, Tensor& Y,
                   cudaStream_t stream = 0) {
  using namespace b200_detail;
  const char* fn = "linear";
  const DType dt = X.defined() && X.dtype() == DType::BF16 ? DType::BF16 : DType::F16;
  const std::int64_t M = extent(fn, "X", X, 0), K = extent(fn, "X", X, 1);
  const std::int64_t N = extent(fn, "W", W, 0);
  const void* px = arg(fn, "X", X, dt, {M, K});
  const void* pw = arg(fn, "W", W, dt, {N, K});
  const void* pr = arg(fn, "residual", residual, dt, {M, N}, true);
  void* py = dst(fn, "Y", Y, dt, {M, N});
  cuda_all(fn, {{"X", &X}, {"W", &W}, {"residual", &residual}, {"Y", &Y}});
  if (dt == DType::BF16) {
    linear_bf16(as<__nv_bfloat16>(px), as<__nv_bfloat16>(pw), as<__nv_bfloat16>(pr),
                as<__nv_bfloat16>(py), M, N, K, stream);
  } else {
    linear_f16(as<__half>(px), as<__half>(pw), as<__half>(pr), as<__half>(py), M, N, K, stream);
  }
}

/// y[N] = W[N,K] x[K] (+ residual[N], or undefined), FP16: the decode GEMV.
inline void gemv_f16_nk(const Tensor& W, const Tensor& x, const Tensor& residual, Tensor& y,
                        cudaStream_t stream = 0) {
  using namespace b200_detail;
  const char* fn = "gemv_f16_nk";
  const std::int64_t N = extent(fn, "W", W, 0), K = extent(fn, "W", W, 1);
  const void* pw = arg(fn, "W", W, DType::F16, {N, K});
  const void* px = arg(fn, "x", x, DType::F16, {K});
  const void* pr = arg(fn, "residual", residual, DType::F16, {N}, true);
  void* py = dst(fn, "y", y, DType::F16, {N});
  cuda_all(fn, {{"W", &W}, {"x", &x}, {"residual", &residual}, {"y", &y}});
  gemv_f16_nk(as<__half>(pw), as<__half>(px), as<__half>(pr), as<__half>(py), N, K, stream);
}

/// Y[M,N] = rmsnorm(x[M,K], gamma[K] or undefined) * W[N,K]^T (+ residual), FP16.
inline void rmsnorm_linear_f16(const Tensor& x, const Tensor& gamma, const Tensor& W,
                               const Tensor& residual, Tensor& Y, float eps,
                               cudaStream_t stream = 0) {
  using namespace b200_detail;
  const char* fn = "rmsnorm_linear_f16";
  const std::int64_t M = extent(fn, "x", x, 0), K = extent(fn, "x", x, 1);
  const std::int64_t N = extent(fn, "W", W, 0);
  const void* px = arg(fn, "x", x, DType::F16, {M, K});
  const void* pg = arg(fn, "gamma", gamma, DType::F16, {K}, true);
  const void* pw = arg(fn, "W", W, DType::F16, {N, K});
  const void* pr = arg(fn, "residual", residual, DType::F16, {M, N}, true);
  void* py = dst(fn, "Y", Y, DType::F16, {M, N});
  cuda_all(fn, {{"x", &x}, {"gamma", &gamma}, {"W", &W}, {"residual", &residual}, {"Y", &Y}});
  rmsnorm_linear_f16(as<__half>(px), as<__half>(pg), as<__half>(pw), as<__half>(pr),
                     as<__half>(py), M, N, K, eps, stream);
}

/// Y[M,F] = swiglu(rmsnorm(x) * W_gu[2F,K]^T), W_gu = gate rows then up rows, FP16.
inline void rmsnorm_linear_swiglu_fp16(const Tensor& x, const Tensor& gamma, const Tensor& W_gu,
                                       Tensor& Y, float eps, cudaStream_t stream = 0) {
  using namespace b200_detail;
  const char* fn = "rmsnorm_linear_swiglu_fp16";
  const std::int64_t M = extent(fn, "x", x, 0), K = extent(fn, "x", x, 1);
  const std::int64_t F2 = extent(fn, "W_gu", W_gu, 0);
  if (F2 % 2 != 0) fail(fn, "W_gu must have an even number of rows (gate, then up)");
  const void* px = arg(fn, "x", x, DType::F16, {M, K});
  const void* pg = arg(fn, "gamma", gamma, DType::F16, {K}, true);
  const void* pw = arg(fn, "W_gu", W_gu, DType::F16, {F2, K});
  void* py = dst(fn, "Y", Y, DType::F16, {M, F2 / 2});
  cuda_all(fn, {{"x", &x}, {"gamma", &gamma}, {"W_gu", &W_gu}, {"Y", &Y}});
  rmsnorm_linear_swiglu_fp16(as<__half>(px), as<__half>(pg), as<__half>(pw), as<__half>(py), M,
                             F2 / 2, K, eps, stream);
}

}  // namespace engine::cuda
