// linear.cu -- entry points of the FP16/BF16 projections and their dispatch:
//
//   matmul_{f16,bf16}      C = A[M,K] B[K,N]                 -> tcgen05 GEMM (MN-major B)
//   linear_{f16,bf16}      Y = X[M,K] W[N,K]^T (+ residual)  -> M <= 4 (FP16): decode GEMV
//                                                               M <= 64: swap-AB tcgen05 + split-K
//                                                               else    : persistent tcgen05 GEMM
//   rmsnorm_linear_f16     Y = rmsnorm(x) W^T (+ residual)   -> M <= 4: GEMV with the norm fused
//                                                               M <= 32: hi/lo normalised rows +
//                                                                        swap-AB tcgen05 (HILO)
//                                                               else   : FP16 normalised rows +
//                                                                        persistent tcgen05 GEMM
//
// The hi/lo pre-pass writes, for each activation row, t = (x * scale) * gamma in
// float (the reference's temp, rmsnorm_linear_cpu.cpp:38-41), its FP16 rounding
// hi = fp16(t) and the FP16 rounding of the remainder lo = fp16(t - hi); the
// tensor cores then form W.hi + W.lo in FP32, which carries t to ~2^-22 relative
// instead of the 2^-11 of a plain FP16 activation.
#include "common.cuh"
#include "kernels.cuh"

namespace b200 {
namespace {

// Block (r, s) of a (hb x P) grid: activation row r, K slice s of P.  Output
// rows [0, M) = hi, [hb, hb + M) = lo; the padding rows [M, hb) and
// [hb + M, 2 hb) are written as zeros.  Every block of a row forms the row's
// scale from the whole row (the same threads and order, so the same scale); it
// then converts only its slice, 8 elements per 16-byte access.
__global__ void __launch_bounds__(256) rmsnorm_hilo_kernel(const __half* __restrict__ x,
                                                           const __half* __restrict__ gamma,
                                                           __half* __restrict__ out, int64_t M,
                                                           int64_t K, int hb, float eps) {
  __shared__ double s_part[8];
  __shared__ float s_scale;
  pdl_trigger();
  pdl_wait();
  const int64_t r = blockIdx.x;  // 0 .. hb-1
  const int64_t P = gridDim.y;
  const int64_t s = blockIdx.y;
  __half* hi = out + r * K;
  __half* lo = out + (r + hb) * K;
  const bool vec = (K % 8 == 0) && (reinterpret_cast<uintptr_t>(x) % 16 == 0) &&
                   (gamma == nullptr || reinterpret_cast<uintptr_t>(gamma) % 16 == 0) &&
                   (reinterpret_cast<uintptr_t>(out) % 16 == 0);
  // This block's slice, in 8-element chunks when vectorised.
  const int64_t units = vec ? K / 8 : K;
  const int64_t u0 = units * s / P;
  const int64_t u1 = units * (s + 1) / P;
  if (r >= M) {
    if (vec) {
      for (int64_t u = u0 + threadIdx.x; u < u1; u += blockDim.x) {
        reinterpret_cast<uint4*>(hi)[u] = make_uint4(0, 0, 0, 0);
        reinterpret_cast<uint4*>(lo)[u] = make_uint4(0, 0, 0, 0);
      }
    } else {
      for (int64_t k = u0 + threadIdx.x; k < u1; k += blockDim.x) {
        hi[k] = __float2half_rn(0.0f);
        lo[k] = __float2half_rn(0.0f);
      }
    }
    return;
  }
  const __half* src = x + r * K;
  double ss = 0.0;
  if (vec) {  // 16-byte loads: one pass over the row in a few iterations
    for (int64_t k8 = threadIdx.x; k8 < K / 8; k8 += blockDim.x) {
      const uint4 raw = *reinterpret_cast<const uint4*>(src + 8 * k8);
      const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(h[i]);
        const double a = static_cast<double>(f.x), b = static_cast<double>(f.y);
        ss = __dadd_rn(ss, __dmul_rn(a, a));
        ss = __dadd_rn(ss, __dmul_rn(b, b));
      }
    }
  } else {
    for (int64_t k = threadIdx.x; k < K; k += blockDim.x) {
      const double v = static_cast<double>(__half2float(src[k]));
      ss = __dadd_rn(ss, __dmul_rn(v, v));
    }
  }
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) s_part[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int i = 0; i < static_cast<int>(blockDim.x >> 5); ++i) t += s_part[i];
    s_scale = static_cast<float>(1.0 / sqrt(t / static_cast<double>(K) + static_cast<double>(eps)));
  }
  __syncthreads();
  const float scale = s_scale;
  auto split = [&](float xv, float g, __half& h, __half& l) {
    const float t = __fmul_rn(__fmul_rn(xv, scale), g);
    h = __float2half_rn(t);
    l = __float2half_rn(__fsub_rn(t, __half2float(h)));
  };
  if (vec) {
    for (int64_t u = u0 + threadIdx.x; u < u1; u += blockDim.x) {
      const uint4 xr = reinterpret_cast<const uint4*>(src)[u];
      const uint4 gr = gamma ? reinterpret_cast<const uint4*>(gamma)[u]
                             : make_uint4(0x3c003c00u, 0x3c003c00u, 0x3c003c00u, 0x3c003c00u);
      const __half* xh = reinterpret_cast<const __half*>(&xr);
      const __half* gh = reinterpret_cast<const __half*>(&gr);
      uint4 ho, lo4;
      __half* hp = reinterpret_cast<__half*>(&ho);
      __half* lp = reinterpret_cast<__half*>(&lo4);
#pragma unroll
      for (int i = 0; i < 8; ++i) split(__half2float(xh[i]), __half2float(gh[i]), hp[i], lp[i]);
      reinterpret_cast<uint4*>(hi)[u] = ho;
      reinterpret_cast<uint4*>(lo)[u] = lo4;
    }
  } else {
    for (int64_t k = u0 + threadIdx.x; k < u1; k += blockDim.x) {
      const float g = gamma ? __half2float(gamma[k]) : 1.0f;
      split(__half2float(src[k]), g, hi[k], lo[k]);
    }
  }
}

// Y[m, i] = swiglu(GU[m, i], GU[m, F + i]) over the [M, 2F] gate/up rows.
__global__ void swiglu_rows_kernel(const __half* __restrict__ gu, __half* __restrict__ y,
                                   int64_t M, int64_t F) {
  pdl_trigger();
  pdl_wait();
  const int64_t n = M * F;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t m = i / F;
    const int64_t c = i - m * F;
    y[i] = swiglu_h(gu[m * 2 * F + c], gu[m * 2 * F + F + c]);
  }
}

int linear_impl(const void* X, const void* W, const void* R, void* Y, int64_t M, int64_t N,
                int64_t K, bool bf16, cudaStream_t stream) {
  if (!bf16 && M <= 4) {
    return gemv_nk_f16(static_cast<const __half*>(W), static_cast<const __half*>(X), nullptr, 0.f,
                       false, static_cast<const __half*>(R), static_cast<__half*>(Y), M, N, K,
                       stream);
  }
  return gemm_tc(X, W, R, Y, M, N, K, bf16, /*b_kmajor=*/true, stream);
}

}  // namespace

int rmsnorm_hilo(const __half* x, const __half* gamma, __half* out, int64_t M, int64_t K, int hb,
                 float eps, cudaStream_t stream) {
  // Slices of >= 2048 elements per block, at most 8 per row.
  const unsigned P = static_cast<unsigned>(K >= 16384 ? 8 : (K + 2047) / 2048);
  B200_CUDA(launch_pdl(rmsnorm_hilo_kernel, dim3(hb, P > 0 ? P : 1), dim3(256), 0, stream, x,
                       gamma, out, M, K,
                       hb, eps));
  return check_launch("rmsnorm_linear_f16 (normalise)");
}

}  // namespace b200

using namespace b200;

namespace {

int check_mm_args(const std::string& n, const void* A, const void* B, const void* C, int64_t M,
                  int64_t N, int64_t K) {
  B200_REQUIRE(A != nullptr, n + ": A is null");
  B200_REQUIRE(B != nullptr, n + ": B is null");
  B200_REQUIRE(C != nullptr, n + ": C is null");
  B200_REQUIRE(M >= 0, n + ": M must be non-negative");
  B200_REQUIRE(N >= 0, n + ": N must be non-negative");
  B200_REQUIRE(K >= 0, n + ": K must be non-negative");
  B200_REQUIRE(M <= 0x7fffffffLL * 128 && N <= 0x7fffffffLL, n + ": dimension too large");
  return ENGINE_OK;
}

int matmul16_entry(const char* name, const void* A, const void* B, void* C, int64_t M,
                   int64_t N, int64_t K, bool bf16, cudaStream_t stream) {
  const int rc = check_mm_args(name, A, B, C, M, N, K);
  if (rc != ENGINE_OK) return rc;
  if (M == 0 || N == 0) return ENGINE_OK;
  if (K == 0) {
    B200_CUDA(cudaMemsetAsync(C, 0, static_cast<size_t>(M) * static_cast<size_t>(N) * 2, stream));
    return ENGINE_OK;
  }
  return gemm_tc(A, B, nullptr, C, M, N, K, bf16, /*b_kmajor=*/false, stream);
}

int linear16_entry(const char* name, const void* X, const void* W, const void* R, void* Y,
                   int64_t M, int64_t N, int64_t K, bool bf16, cudaStream_t stream) {
  const std::string n(name);
  B200_REQUIRE(X != nullptr, n + ": X is null");
  B200_REQUIRE(W != nullptr, n + ": W is null");
  B200_REQUIRE(Y != nullptr, n + ": Y is null");
  B200_REQUIRE(M >= 0, n + ": M must be non-negative");
  B200_REQUIRE(N >= 0, n + ": N must be non-negative");
  B200_REQUIRE(K >= 0, n + ": K must be non-negative");
  if (M == 0 || N == 0) return ENGINE_OK;
  if (K == 0 && R == nullptr) {
    B200_CUDA(cudaMemsetAsync(Y, 0, static_cast<size_t>(M) * static_cast<size_t>(N) * 2, stream));
    return ENGINE_OK;
  }
  if (K == 0) {  // Y = residual: the empty product is zero
    B200_CUDA(cudaMemcpyAsync(Y, R, static_cast<size_t>(M) * static_cast<size_t>(N) * 2,
                              cudaMemcpyDeviceToDevice, stream));
    return ENGINE_OK;
  }
  return linear_impl(X, W, R, Y, M, N, K, bf16, stream);
}

}  // namespace

extern "C" {

int engine_cuda_matmul_f16(const engine_half_t* A, const engine_half_t* B, engine_half_t* C,
                           int64_t M, int64_t N, int64_t K, engine_stream_t stream) {
  B200_ENTRY_BEGIN
  return matmul16_entry("matmul_f16", A, B, C, M, N, K, false, stream);
  B200_ENTRY_END
}

int engine_cuda_matmul_bf16(const engine_bf16_t* A, const engine_bf16_t* B, engine_bf16_t* C,
                            int64_t M, int64_t N, int64_t K, engine_stream_t stream) {
  B200_ENTRY_BEGIN
  return matmul16_entry("matmul_bf16", A, B, C, M, N, K, true, stream);
  B200_ENTRY_END
}

int engine_cuda_linear_f16(const engine_half_t* X, const engine_half_t* W,
                           const engine_half_t* residual, engine_half_t* Y, int64_t M,
                           int64_t N, int64_t K, engine_stream_t stream) {
  B200_ENTRY_BEGIN
  return linear16_entry("linear_f16", X, W, residual, Y, M, N, K, false, stream);
  B200_ENTRY_END
}

int engine_cuda_linear_bf16(const engine_bf16_t* X, const engine_bf16_t* W,
                            const engine_bf16_t* residual, engine_bf16_t* Y, int64_t M,
                            int64_t N, int64_t K, engine_stream_t stream) {
  B200_ENTRY_BEGIN
  return linear16_entry("linear_bf16", X, W, residual, Y, M, N, K, true, stream);
  B200_ENTRY_END
}

int engine_cuda_rmsnorm_linear_f16(const engine_half_t* x, const engine_half_t* gamma,
                                   const engine_half_t* W, const engine_half_t* residual,
                                   engine_half_t* Y, int64_t M, int64_t N, int64_t K,
                                   float eps, engine_stream_t stream) {
  B200_ENTRY_BEGIN
  B200_REQUIRE(M >= 0 && N >= 0 && K >= 0, "rmsnorm_linear_f16: negative dimension");
  B200_REQUIRE(x != nullptr && W != nullptr && Y != nullptr,
               "rmsnorm_linear_f16: null device pointer");
  B200_REQUIRE(eps >= 0.0f, "rmsnorm_linear_f16: eps must be non-negative");
  if (M == 0 || N == 0 || K == 0) return ENGINE_OK;
  const __half* xh = reinterpret_cast<const __half*>(x);
  const __half* gh = reinterpret_cast<const __half*>(gamma);
  const __half* wh = reinterpret_cast<const __half*>(W);
  const __half* rh = reinterpret_cast<const __half*>(residual);
  __half* yh = reinterpret_cast<__half*>(Y);
  if (M <= 4) return gemv_nk_f16(wh, xh, gh, eps, true, rh, yh, M, N, K, stream);

  const bool aligned = (K % 8 == 0) && (reinterpret_cast<uintptr_t>(W) % 16 == 0);
  if (M <= 32 && aligned) {
    int hb = 8;
    while (hb < M) hb <<= 1;
    const size_t bytes = static_cast<size_t>(2 * hb) * static_cast<size_t>(K) * 2;
    __half* x2 = static_cast<__half*>(scratch_alloc(bytes, stream));
    if (x2 == nullptr) return ENGINE_ERR_CUDA;
    int rc = rmsnorm_hilo(xh, gh, x2, M, K, hb, eps, stream);
    if (rc == ENGINE_OK) {
      rc = gemm_tc_general(x2, wh, rh, yh, M, N, K, false, true, true, hb, stream);
    }
    scratch_free(x2, stream);
    return rc;
  }
  const size_t bytes = static_cast<size_t>(M) * static_cast<size_t>(K) * 2;
  __half* xn = static_cast<__half*>(scratch_alloc(bytes, stream));
  if (xn == nullptr) return ENGINE_ERR_CUDA;
  int rc = rmsnorm_f16(xh, gh, xn, M, K, eps, stream);
  if (rc == ENGINE_OK) rc = linear_impl(xn, wh, rh, yh, M, N, K, false, stream);
  scratch_free(xn, stream);
  return rc;
  B200_ENTRY_END
}

}  // extern "C"

extern "C" int engine_cuda_rmsnorm_linear_swiglu_f16(const engine_half_t* x,
                                                     const engine_half_t* gamma,
                                                     const engine_half_t* W_gu, engine_half_t* Y,
                                                     int64_t M, int64_t F, int64_t K, float eps,
                                                     engine_stream_t stream) {
  B200_ENTRY_BEGIN
  B200_REQUIRE(M >= 0 && F >= 0 && K >= 0, "rmsnorm_linear_swiglu_f16: negative dimension");
  B200_REQUIRE(x != nullptr && W_gu != nullptr && Y != nullptr,
               "rmsnorm_linear_swiglu_f16: null device pointer");
  B200_REQUIRE(eps >= 0.0f, "rmsnorm_linear_swiglu_f16: eps must be non-negative");
  if (M == 0 || F == 0) return ENGINE_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (K == 0) {  // empty projections: swiglu(0, 0) = 0
    B200_CUDA(cudaMemsetAsync(Y, 0, static_cast<size_t>(M * F) * sizeof(engine_half_t), st));
    return ENGINE_OK;
  }
  const __half* xh = reinterpret_cast<const __half*>(x);
  const __half* gh = reinterpret_cast<const __half*>(gamma);
  const __half* wh = reinterpret_cast<const __half*>(W_gu);
  __half* yh = reinterpret_cast<__half*>(Y);
  if (M == 1) {
    const int rc = gemv_nk_norm1_swiglu_f16(wh, xh, gh, eps, yh, F, K, st);
    if (rc != ENGINE_ERR_UNSUPPORTED) return rc;
  }
  // Otherwise: the projection into stream-ordered scratch, then the SwiGLU.
  const size_t bytes = static_cast<size_t>(M) * static_cast<size_t>(2 * F) * sizeof(__half);
  __half* gu = static_cast<__half*>(scratch_alloc(bytes, st));
  if (gu == nullptr) return ENGINE_ERR_CUDA;
  int rc = engine_cuda_rmsnorm_linear_f16(x, gamma, W_gu, nullptr,
                                          reinterpret_cast<engine_half_t*>(gu), M, 2 * F, K, eps,
                                          stream);
  if (rc == ENGINE_OK) {
    const int64_t n = M * F;
    const int64_t blocks64 = (n + 255) / 256;
    const unsigned blocks = static_cast<unsigned>(blocks64 < 4096 ? blocks64 : 4096);
    const cudaError_t e =
        launch_pdl(swiglu_rows_kernel, dim3(blocks), dim3(256), 0, st, gu, yh, M, F);
    rc = (e == cudaSuccess) ? check_launch("rmsnorm_linear_swiglu_f16")
                            : set_cuda_error(e, "rmsnorm_linear_swiglu_f16");
  }
  scratch_free(gu, st);
  return rc;
  B200_ENTRY_END
}
