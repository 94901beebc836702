// gemv.cu -- HBM-streaming matrix-vector products.
//
// 1. gemv_nk_kernel: y[m, n] = sum_k X[m, k] * W[n, k] for a handful of rows of X
//    (batch-1 and tiny-batch decode) over weights stored [N,K], K contiguous --
//    the layout of the B200 decode configuration.  One warp owns RPW weight rows;
//    each lane streams 16-byte (8 x FP16) chunks of those rows with
//    L1::no_allocate loads, U chunks in flight per row, multiplies them with the
//    matching chunks of X (L1-resident after the first warp) and reduces with warp
//    shuffles.  No shared memory, no split-K: N=4096 already gives 1024 CTAs.
//    Optional fused RMSNorm (the warp accumulates sum(x^2) in the same pass and
//    applies the scale after the dot product) and residual epilogue.
// 2. gemv_kn_kernel: out[n] = sum_k x[k] * A[k, n] over the reference's legacy
//    [K,N] layout (engine::cuda::gemv / gemv_fp16, kernels/gemv*.cu).  A warp
//    covers 32 x 16 bytes of one row of A per k, eight warps split K inside the
//    CTA, and up to eight CTAs of a thread-block cluster split it further,
//    reducing through distributed shared memory (no global scratch).
// 3. rmsnorm_f16_kernel: row RMSNorm FP16 -> FP16 for the tensor-core path of
//    rmsnorm_linear_f16.
#include <cooperative_groups.h>

#include <cstdlib>

#include "common.cuh"
#include "kernels.cuh"

namespace cg = cooperative_groups;

namespace b200 {
namespace {

__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ void h8_to_f8(const uint4& v, float (&f)[8]) {
  const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __half22float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

// ---------------------------------------------------------------- [N,K] GEMV

constexpr int kNkWarps = 4;

template <int MR, int RPW, int U, bool NORM, bool RESID>
__global__ void __launch_bounds__(kNkWarps * 32) gemv_nk_vec_kernel(
    const __half* __restrict__ W, const __half* __restrict__ X, const __half* __restrict__ gamma,
    const __half* __restrict__ R, __half* __restrict__ Y, int64_t N, int64_t K, float eps) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int64_t row0 = (static_cast<int64_t>(blockIdx.x) * kNkWarps + warp) * RPW;
  if (row0 >= N) return;
  const int64_t nchunk = K >> 3;  // 8 halves per 16-byte chunk

  float acc[MR][RPW];
  float ss[MR];
#pragma unroll
  for (int m = 0; m < MR; ++m) {
    ss[m] = 0.0f;
#pragma unroll
    for (int r = 0; r < RPW; ++r) acc[m][r] = 0.0f;
  }
  const __half* wrow[RPW];
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    const int64_t n = (row0 + r < N) ? row0 + r : N - 1;  // clamp: duplicate rows are not stored
    wrow[r] = W + n * K;
  }

  for (int64_t c0 = lane; c0 < nchunk; c0 += 32 * U) {
    uint4 wv[U][RPW];
    uint4 xv[U][MR];
    uint4 gv[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t c = c0 + 32 * u;
      if (c < nchunk) {
#pragma unroll
        for (int r = 0; r < RPW; ++r) wv[u][r] = ld_stream_v4(wrow[r] + 8 * c);
#pragma unroll
        for (int m = 0; m < MR; ++m) xv[u][m] = __ldg(reinterpret_cast<const uint4*>(X + m * K + 8 * c));
        if constexpr (NORM) {
          gv[u] = gamma ? __ldg(reinterpret_cast<const uint4*>(gamma + 8 * c))
                        : make_uint4(0x3c003c00u, 0x3c003c00u, 0x3c003c00u, 0x3c003c00u);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t c = c0 + 32 * u;
      if (c < nchunk) {
        float g[8];
        if constexpr (NORM) h8_to_f8(gv[u], g);
#pragma unroll
        for (int m = 0; m < MR; ++m) {
          float xf[8];
          h8_to_f8(xv[u][m], xf);
          if constexpr (NORM) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              ss[m] = fmaf(xf[i], xf[i], ss[m]);
              xf[i] *= g[i];
            }
          }
#pragma unroll
          for (int r = 0; r < RPW; ++r) {
            float wf[8];
            h8_to_f8(wv[u][r], wf);
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[m][r] = fmaf(xf[i], wf[i], acc[m][r]);
          }
        }
      }
    }
  }

#pragma unroll
  for (int m = 0; m < MR; ++m) {
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc[m][r] += __shfl_xor_sync(0xffffffffu, acc[m][r], o);
    }
    if constexpr (NORM) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss[m] += __shfl_xor_sync(0xffffffffu, ss[m], o);
    }
  }
  if (lane < RPW * MR) {
    // Lane l writes row r = l % RPW of batch row m = l / RPW.
#pragma unroll
    for (int m = 0; m < MR; ++m) {
#pragma unroll
      for (int r = 0; r < RPW; ++r) {
        if (lane == m * RPW + r && row0 + r < N) {
          float v = acc[m][r];
          if constexpr (NORM) {
            const float scale = static_cast<float>(
                1.0 / sqrt(static_cast<double>(ss[m]) / static_cast<double>(K) +
                           static_cast<double>(eps)));
            v = v * scale;
          }
          if constexpr (RESID) v = v + __half2float(R[m * N + row0 + r]);
          Y[m * N + row0 + r] = __float2half_rn(v);
        }
      }
    }
  }
}

// Any K / alignment: one weight row per warp, scalar loads.
template <bool NORM, bool RESID>
__global__ void __launch_bounds__(kNkWarps * 32) gemv_nk_scalar_kernel(
    const __half* __restrict__ W, const __half* __restrict__ X, const __half* __restrict__ gamma,
    const __half* __restrict__ R, __half* __restrict__ Y, int64_t M, int64_t N, int64_t K,
    float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t n = static_cast<int64_t>(blockIdx.x) * kNkWarps + (threadIdx.x >> 5);
  if (n >= N) return;
  for (int64_t m = 0; m < M; ++m) {
    float acc = 0.0f, ss = 0.0f;
    for (int64_t k = lane; k < K; k += 32) {
      float xf = __half2float(X[m * K + k]);
      if constexpr (NORM) {
        ss = fmaf(xf, xf, ss);
        xf *= gamma ? __half2float(gamma[k]) : 1.0f;
      }
      acc = fmaf(xf, __half2float(W[n * K + k]), acc);
    }
    for (int o = 16; o > 0; o >>= 1) {
      acc += __shfl_xor_sync(0xffffffffu, acc, o);
      ss += __shfl_xor_sync(0xffffffffu, ss, o);
    }
    if (lane == 0) {
      float v = acc;
      if constexpr (NORM) {
        v = v * static_cast<float>(1.0 / sqrt(static_cast<double>(ss) / static_cast<double>(K) +
                                              static_cast<double>(eps)));
      }
      if constexpr (RESID) v = v + __half2float(R[m * N + n]);
      Y[m * N + n] = __float2half_rn(v);
    }
  }
}

int env_int(const char* name, int dflt) {
  const char* e = std::getenv(name);
  if (e == nullptr || e[0] == '\0') return dflt;
  return static_cast<int>(std::strtol(e, nullptr, 10));
}

template <int MR, int RPW, bool NORM, bool RESID>
void launch_nk_vec(const __half* W, const __half* X, const __half* gamma, const __half* R,
                   __half* Y, int64_t N, int64_t K, float eps, cudaStream_t stream) {
  constexpr int U = (MR >= 4) ? 2 : 4;
  const int64_t rows_per_cta = static_cast<int64_t>(kNkWarps) * RPW;
  const unsigned grid = static_cast<unsigned>((N + rows_per_cta - 1) / rows_per_cta);
  gemv_nk_vec_kernel<MR, RPW, U, NORM, RESID>
      <<<grid, kNkWarps * 32, 0, stream>>>(W, X, gamma, R, Y, N, K, eps);
}

template <int MR, bool NORM, bool RESID>
void dispatch_rpw(int rpw, const __half* W, const __half* X, const __half* gamma,
                  const __half* R, __half* Y, int64_t N, int64_t K, float eps,
                  cudaStream_t stream) {
  if (rpw >= 2) {
    launch_nk_vec<MR, 2, NORM, RESID>(W, X, gamma, R, Y, N, K, eps, stream);
  } else {
    launch_nk_vec<MR, 1, NORM, RESID>(W, X, gamma, R, Y, N, K, eps, stream);
  }
}

template <bool NORM, bool RESID>
void dispatch_mr(int64_t mr, int rpw, const __half* W, const __half* X, const __half* gamma,
                 const __half* R, __half* Y, int64_t N, int64_t K, float eps,
                 cudaStream_t stream) {
  switch (mr) {
    case 1: dispatch_rpw<1, NORM, RESID>(rpw, W, X, gamma, R, Y, N, K, eps, stream); break;
    case 2: dispatch_rpw<2, NORM, RESID>(rpw, W, X, gamma, R, Y, N, K, eps, stream); break;
    case 3: dispatch_rpw<3, NORM, RESID>(rpw, W, X, gamma, R, Y, N, K, eps, stream); break;
    default: dispatch_rpw<4, NORM, RESID>(rpw, W, X, gamma, R, Y, N, K, eps, stream); break;
  }
}

// ---------------------------------------------------------------- [K,N] GEMV

constexpr int kKnWarps = 8;

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }

template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }

template <typename T, bool VEC, bool NORM>
__global__ void __launch_bounds__(kKnWarps * 32) gemv_kn_kernel(
    const T* __restrict__ A, const T* __restrict__ x, T* __restrict__ out, int64_t N, int64_t K,
    int64_t kchunk, int S, const float* __restrict__ rms_w, float eps) {
  constexpr int VW = VEC ? static_cast<int>(16 / sizeof(T)) : 1;
  constexpr int CPB = 32 * VW;
  __shared__ __align__(16) float red[kKnWarps][CPB];
  __shared__ float part[CPB];
  __shared__ double s_part[kKnWarps];
  __shared__ float s_scale;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t n0 = static_cast<int64_t>(blockIdx.x) * CPB;
  const int z = static_cast<int>(blockIdx.z);
  const int64_t kbeg = static_cast<int64_t>(z) * kchunk;
  const int64_t kend = (kbeg + kchunk < K) ? kbeg + kchunk : K;

  float scale = 1.0f;
  if constexpr (NORM) {
    double ss = 0.0;
    for (int64_t k = tid; k < K; k += blockDim.x) {
      const double v = static_cast<double>(to_f<T>(x[k]));
      ss = __dadd_rn(ss, __dmul_rn(v, v));
    }
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) s_part[warp] = ss;
    __syncthreads();
    if (tid == 0) {
      double t = 0.0;
      for (int i = 0; i < kKnWarps; ++i) t += s_part[i];
      s_scale = static_cast<float>(1.0 / sqrt(t / static_cast<double>(K) + static_cast<double>(eps)));
    }
    __syncthreads();
    scale = s_scale;
  }

  float acc[VW];
#pragma unroll
  for (int v = 0; v < VW; ++v) acc[v] = 0.0f;
  const int64_t ncol = n0 + static_cast<int64_t>(lane) * VW;
  const bool col_ok = ncol < N;
  constexpr int U = 4;
  for (int64_t kb = kbeg + warp; kb < kend; kb += kKnWarps * U) {
    float xk[U];
    T av[U][VW];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t k = kb + static_cast<int64_t>(kKnWarps) * u;
      const bool ok = k < kend;
      float xv = ok ? to_f<T>(x[k]) : 0.0f;
      if constexpr (NORM) {
        if (ok) xv = __fmul_rn(__fmul_rn(xv, scale), rms_w ? rms_w[k] : 1.0f);
      }
      xk[u] = xv;
      if constexpr (VEC) {
        if (ok && col_ok) {
          const uint4 raw = __ldg(reinterpret_cast<const uint4*>(A + k * N + ncol));
          const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
          for (int v = 0; v < VW; ++v) av[u][v] = e[v];
        } else {
#pragma unroll
          for (int v = 0; v < VW; ++v) av[u][v] = from_f<T>(0.0f);
        }
      } else {
        av[u][0] = (ok && col_ok) ? A[k * N + ncol] : from_f<T>(0.0f);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u)
#pragma unroll
      for (int v = 0; v < VW; ++v) acc[v] = fmaf(xk[u], to_f<T>(av[u][v]), acc[v]);
  }

#pragma unroll
  for (int v = 0; v < VW; ++v) red[warp][lane * VW + v] = acc[v];
  __syncthreads();
  for (int t = tid; t < CPB; t += blockDim.x) {
    float s = 0.0f;
#pragma unroll
    for (int w = 0; w < kKnWarps; ++w) s += red[w][t];
    part[t] = s;
  }
  if (S == 1) {
    __syncthreads();
    for (int t = tid; t < CPB; t += blockDim.x) {
      if (n0 + t < N) out[n0 + t] = from_f<T>(part[t]);
    }
    return;
  }
  cg::cluster_group cluster = cg::this_cluster();
  cluster.sync();
  for (int t = tid; t < CPB; t += blockDim.x) {
    if (t % S != z) continue;
    float s = 0.0f;
    for (int q = 0; q < S; ++q) s += cluster.map_shared_rank(part, q)[t];
    if (n0 + t < N) out[n0 + t] = from_f<T>(s);
  }
  cluster.sync();
}

template <typename T, bool VEC, bool NORM>
int launch_kn(const T* A, const T* x, T* out, int64_t N, int64_t K, const float* rms_w,
              float eps, cudaStream_t stream) {
  constexpr int VW = VEC ? static_cast<int>(16 / sizeof(T)) : 1;
  constexpr int CPB = 32 * VW;
  const int64_t cols = (N + CPB - 1) / CPB;
  B200_REQUIRE(cols <= 0x7fffffff, "gemv: N too large");
  const int sms = sm_count();
  int S = 1;
  if (cols < 2 * sms) {
    S = static_cast<int>((2 * sms) / cols);
    if (S > 8) S = 8;
    const int64_t kmax = K / (kKnWarps * 4);
    if (S > kmax) S = static_cast<int>(kmax > 0 ? kmax : 1);
    if (S < 1) S = 1;
  }
  const int64_t kchunk = (K + S - 1) / S;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(cols), 1, static_cast<unsigned>(S));
  cfg.blockDim = dim3(kKnWarps * 32);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = static_cast<unsigned>(S);
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  B200_CUDA(cudaLaunchKernelEx(&cfg, gemv_kn_kernel<T, VEC, NORM>, A, x, out, N, K, kchunk, S,
                               rms_w, eps));
  return ENGINE_OK;
}

// ---------------------------------------------------------------- RMSNorm FP16

__global__ void __launch_bounds__(256) rmsnorm_f16_kernel(const __half* __restrict__ in,
                                                          const __half* __restrict__ w,
                                                          __half* __restrict__ out,
                                                          int64_t rows, int64_t cols,
                                                          float eps) {
  __shared__ double s_part[8];
  __shared__ float s_scale;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const __half* src = in + r * cols;
    double ss = 0.0;
    for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
      const double v = static_cast<double>(__half2float(src[c]));
      ss = __dadd_rn(ss, __dmul_rn(v, v));
    }
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) s_part[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
      double t = 0.0;
      for (int i = 0; i < static_cast<int>(blockDim.x >> 5); ++i) t += s_part[i];
      s_scale = static_cast<float>(1.0 / sqrt(t / static_cast<double>(cols) + static_cast<double>(eps)));
    }
    __syncthreads();
    const float scale = s_scale;
    __half* dst = out + r * cols;
    for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
      const float wv = w ? __half2float(w[c]) : 1.0f;
      dst[c] = __float2half_rn(__fmul_rn(__fmul_rn(__half2float(src[c]), scale), wv));
    }
    __syncthreads();
  }
}

}  // namespace

int gemv_nk_f16(const __half* W, const __half* X, const __half* gamma, float eps, bool norm,
                const __half* residual, __half* Y, int64_t M, int64_t N, int64_t K,
                cudaStream_t stream) {
  const bool vec = (K % 8 == 0) && (reinterpret_cast<uintptr_t>(W) % 16 == 0) &&
                   (reinterpret_cast<uintptr_t>(X) % 16 == 0) &&
                   (gamma == nullptr || reinterpret_cast<uintptr_t>(gamma) % 16 == 0);
  B200_REQUIRE(N <= (static_cast<int64_t>(1) << 36), "gemv: N too large");
  if (!vec) {
    const unsigned grid = static_cast<unsigned>((N + kNkWarps - 1) / kNkWarps);
    if (norm) {
      if (residual) gemv_nk_scalar_kernel<true, true><<<grid, kNkWarps * 32, 0, stream>>>(W, X, gamma, residual, Y, M, N, K, eps);
      else gemv_nk_scalar_kernel<true, false><<<grid, kNkWarps * 32, 0, stream>>>(W, X, gamma, residual, Y, M, N, K, eps);
    } else {
      if (residual) gemv_nk_scalar_kernel<false, true><<<grid, kNkWarps * 32, 0, stream>>>(W, X, gamma, residual, Y, M, N, K, eps);
      else gemv_nk_scalar_kernel<false, false><<<grid, kNkWarps * 32, 0, stream>>>(W, X, gamma, residual, Y, M, N, K, eps);
    }
    return check_launch("gemv_f16_nk");
  }
  static const int rpw_env = env_int("ENGINE_GEMV_RPW", 0);
  const int rpw = rpw_env > 0 ? rpw_env : (N >= 8192 ? 2 : 1);
  for (int64_t m0 = 0; m0 < M; m0 += 4) {
    const int64_t mr = (M - m0 < 4) ? M - m0 : 4;
    const __half* Xm = X + m0 * K;
    const __half* Rm = residual ? residual + m0 * N : nullptr;
    __half* Ym = Y + m0 * N;
    if (norm) {
      if (residual) dispatch_mr<true, true>(mr, rpw, W, Xm, gamma, Rm, Ym, N, K, eps, stream);
      else dispatch_mr<true, false>(mr, rpw, W, Xm, gamma, Rm, Ym, N, K, eps, stream);
    } else {
      if (residual) dispatch_mr<false, true>(mr, rpw, W, Xm, gamma, Rm, Ym, N, K, eps, stream);
      else dispatch_mr<false, false>(mr, rpw, W, Xm, gamma, Rm, Ym, N, K, eps, stream);
    }
  }
  return check_launch("gemv_f16_nk");
}

int gemv_kn_f32(const float* A, const float* x, float* out, int64_t N, int64_t K,
                const float* rms_w, float eps, bool norm, cudaStream_t stream) {
  const bool vec = (N % 4 == 0) && (reinterpret_cast<uintptr_t>(A) % 16 == 0);
  int rc;
  if (norm) {
    rc = vec ? launch_kn<float, true, true>(A, x, out, N, K, rms_w, eps, stream)
             : launch_kn<float, false, true>(A, x, out, N, K, rms_w, eps, stream);
  } else {
    rc = vec ? launch_kn<float, true, false>(A, x, out, N, K, nullptr, 0.f, stream)
             : launch_kn<float, false, false>(A, x, out, N, K, nullptr, 0.f, stream);
  }
  if (rc != ENGINE_OK) return rc;
  return check_launch(norm ? "rmsnorm_linear" : "gemv");
}

int gemv_kn_f16(const __half* A, const __half* x, __half* out, int64_t N, int64_t K,
                cudaStream_t stream) {
  const bool vec = (N % 8 == 0) && (reinterpret_cast<uintptr_t>(A) % 16 == 0);
  const int rc = vec ? launch_kn<__half, true, false>(A, x, out, N, K, nullptr, 0.f, stream)
                     : launch_kn<__half, false, false>(A, x, out, N, K, nullptr, 0.f, stream);
  if (rc != ENGINE_OK) return rc;
  return check_launch("gemv_fp16");
}

int rmsnorm_f16(const __half* x, const __half* gamma, __half* out, int64_t rows, int64_t cols,
                float eps, cudaStream_t stream) {
  const int64_t cap = static_cast<int64_t>(sm_count()) * 32;
  const int grid = static_cast<int>(rows < cap ? rows : cap);
  rmsnorm_f16_kernel<<<grid, 256, 0, stream>>>(x, gamma, out, rows, cols, eps);
  return check_launch("rmsnorm_f16");
}

}  // namespace b200

using namespace b200;

extern "C" {

int engine_cuda_gemv(const float* A, const float* x, float* out, int64_t N, int64_t K,
                     engine_stream_t stream) {
  B200_ENTRY_BEGIN
  B200_REQUIRE(A != nullptr, "gemv: A is null");
  B200_REQUIRE(x != nullptr, "gemv: x is null");
  B200_REQUIRE(out != nullptr, "gemv: out is null");
  B200_REQUIRE(N >= 0, "gemv: N must be non-negative");
  B200_REQUIRE(K >= 0, "gemv: K must be non-negative");
  if (N == 0) return ENGINE_OK;
  if (K == 0) {
    B200_CUDA(cudaMemsetAsync(out, 0, static_cast<size_t>(N) * sizeof(float), stream));
    return ENGINE_OK;
  }
  return gemv_kn_f32(A, x, out, N, K, nullptr, 0.f, false, stream);
  B200_ENTRY_END
}

int engine_cuda_gemv_fp16(const engine_half_t* A, const engine_half_t* x, engine_half_t* out,
                          int64_t N, int64_t K, engine_stream_t stream) {
  B200_ENTRY_BEGIN
  B200_REQUIRE(A != nullptr, "gemv_fp16: A is null");
  B200_REQUIRE(x != nullptr, "gemv_fp16: x is null");
  B200_REQUIRE(out != nullptr, "gemv_fp16: out is null");
  B200_REQUIRE(N >= 0, "gemv_fp16: N must be non-negative");
  B200_REQUIRE(K >= 0, "gemv_fp16: K must be non-negative");
  if (N == 0) return ENGINE_OK;
  if (K == 0) {
    B200_CUDA(cudaMemsetAsync(out, 0, static_cast<size_t>(N) * sizeof(engine_half_t), stream));
    return ENGINE_OK;
  }
  return gemv_kn_f16(reinterpret_cast<const __half*>(A), reinterpret_cast<const __half*>(x),
                     reinterpret_cast<__half*>(out), N, K, stream);
  B200_ENTRY_END
}

int engine_cuda_gemv_f16_nk(const engine_half_t* W, const engine_half_t* x,
                            const engine_half_t* residual, engine_half_t* y, int64_t N,
                            int64_t K, engine_stream_t stream) {
  B200_ENTRY_BEGIN
  B200_REQUIRE(W != nullptr, "gemv_f16_nk: W is null");
  B200_REQUIRE(x != nullptr, "gemv_f16_nk: x is null");
  B200_REQUIRE(y != nullptr, "gemv_f16_nk: y is null");
  B200_REQUIRE(N >= 0, "gemv_f16_nk: N must be non-negative");
  B200_REQUIRE(K >= 0, "gemv_f16_nk: K must be non-negative");
  if (N == 0) return ENGINE_OK;
  if (K == 0 && residual == nullptr) {
    B200_CUDA(cudaMemsetAsync(y, 0, static_cast<size_t>(N) * sizeof(engine_half_t), stream));
    return ENGINE_OK;
  }
  return gemv_nk_f16(reinterpret_cast<const __half*>(W), reinterpret_cast<const __half*>(x),
                     nullptr, 0.f, false, reinterpret_cast<const __half*>(residual),
                     reinterpret_cast<__half*>(y), 1, N, K, stream);
  B200_ENTRY_END
}

}  // extern "C"
