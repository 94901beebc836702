// gemm_simt.cu -- FP32 GEMM C[M,N] = A[M,K] * B[K,N] on the CUDA cores, and the
// fused FP32 RMSNorm -> linear built on it.
//
// Replaces engine::cuda::matmul_naive / matmul_tiled / matmul_register_tiled
// (reference kernels/matmul_*.cu, launchers at matmul_register_tiled.cu:176-199)
// and rmsnorm_linear / rmsnorm_linear_fused_direct (rmsnorm_linear.cu:145-201).
//
// Why CUDA cores: the FP32 configuration is held to the FP32 error bound
// K * u32 * sum|a||b| (u32 = 2^-24), which a TF32 tensor-core product cannot meet.
//
// Design for B200 (148 SMs):
//   * 64x64 output tile per 256-thread CTA, 4x4 register tile per thread, BK=16,
//     two shared-memory stages with register prefetch of the next k-tile;
//   * when the tile grid is too small to fill the SMs (512^3 has 64 tiles), the
//     K dimension is split over S <= 8 CTAs of one thread-block CLUSTER; each CTA
//     parks its 64x64 FP32 partial in its own shared memory and, after a cluster
//     barrier, CTA z sums rows z, z+S, ... over the S partials read through
//     distributed shared memory in fixed rank order (deterministic, no global
//     scratch, one launch);
//   * the fused RMSNorm prologue computes each tile row's scale from the FULL row
//     (squares summed in double, scale = float(1/sqrt(mean + eps)) -- the
//     reference's arithmetic, rmsnorm_linear_cpu.cpp:18-51), and the A loader
//     forms temp = (x * scale) * w in float on the way into shared memory, so the
//     normalised activation never touches global memory.
#include <cooperative_groups.h>

#include <cstdlib>

#include "common.cuh"
#include "kernels.cuh"

namespace cg = cooperative_groups;

namespace b200 {
namespace {

constexpr int kBM = 64;
constexpr int kBN = 64;
constexpr int kBK = 16;
constexpr int kThreads = 256;
constexpr int kApad = kBM + 4;  // padded A^T row (floats): spreads the transposed stores
constexpr int kSmemFloats = 2 * kBK * kApad + 2 * kBK * kBN;  // >= kBM*kBN partial buffer

static_assert(kSmemFloats >= kBM * kBN, "split-K partial must fit in the tile buffers");

template <bool VEC, bool NORM>
__global__ void __launch_bounds__(kThreads) sgemm_kernel(const float* __restrict__ A,
                                                         const float* __restrict__ B,
                                                         float* __restrict__ C, int64_t M,
                                                         int64_t N, int64_t K, int64_t kchunk,
                                                         int S, const float* __restrict__ rms_w,
                                                         float eps) {
  __shared__ __align__(16) float smem[kSmemFloats];
  __shared__ float s_scale[kBM];
  float* As = smem;                        // [2][kBK][kApad], A tile transposed (k-major)
  float* Bs = smem + 2 * kBK * kApad;      // [2][kBK][kBN]

  const int tid = threadIdx.x;
  const int tx = tid & 15;   // output columns tx*4 .. tx*4+3
  const int ty = tid >> 4;   // output rows    ty*4 .. ty*4+3
  const int64_t m0 = static_cast<int64_t>(blockIdx.y) * kBM;
  const int64_t n0 = static_cast<int64_t>(blockIdx.x) * kBN;
  const int z = static_cast<int>(blockIdx.z);
  const int64_t kbeg = static_cast<int64_t>(z) * kchunk;
  const int64_t kend = (kbeg + kchunk < K) ? kbeg + kchunk : K;

  if constexpr (NORM) {
    const int warp = tid >> 5, lane = tid & 31;
    for (int r = warp; r < kBM; r += kThreads / 32) {
      const int64_t m = m0 + r;
      double ss = 0.0;
      if (m < M) {
        const float* row = A + m * K;
        for (int64_t k = lane; k < K; k += 32) {
          const double v = static_cast<double>(row[k]);
          ss = __dadd_rn(ss, __dmul_rn(v, v));
        }
      }
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if (lane == 0) {
        s_scale[r] = (m < M) ? static_cast<float>(1.0 / sqrt(ss / static_cast<double>(K) +
                                                              static_cast<double>(eps)))
                             : 0.0f;
      }
    }
    __syncthreads();
  }

  // Loader roles: A tile 64x16 (row ar, cols kc..kc+3), B tile 16x64 (row br, cols nc..nc+3).
  const int ar = tid >> 2, kc = (tid & 3) * 4;
  const int br = tid >> 4, nc = (tid & 15) * 4;
  float ra[4], rb[4];

  auto load_tile = [&](int64_t k0) {
    const int64_t am = m0 + ar;
    const int64_t ak = k0 + kc;
    if constexpr (VEC) {
      if (am < M && ak < kend) {
        const float4 v = *reinterpret_cast<const float4*>(A + am * K + ak);
        ra[0] = v.x; ra[1] = v.y; ra[2] = v.z; ra[3] = v.w;
      } else {
        ra[0] = ra[1] = ra[2] = ra[3] = 0.0f;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) ra[i] = (am < M && ak + i < kend) ? A[am * K + ak + i] : 0.0f;
    }
    if constexpr (NORM) {
      const float sc = s_scale[ar];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float w = (rms_w != nullptr && ak + i < kend) ? rms_w[ak + i] : 1.0f;
        ra[i] = __fmul_rn(__fmul_rn(ra[i], sc), w);
      }
    }
    const int64_t bk = k0 + br;
    const int64_t bn = n0 + nc;
    if constexpr (VEC) {
      if (bk < kend && bn < N) {
        const float4 v = *reinterpret_cast<const float4*>(B + bk * N + bn);
        rb[0] = v.x; rb[1] = v.y; rb[2] = v.z; rb[3] = v.w;
      } else {
        rb[0] = rb[1] = rb[2] = rb[3] = 0.0f;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) rb[i] = (bk < kend && bn + i < N) ? B[bk * N + bn + i] : 0.0f;
    }
  };
  auto store_tile = [&](int buf) {
    float* as = As + buf * kBK * kApad;
#pragma unroll
    for (int i = 0; i < 4; ++i) as[(kc + i) * kApad + ar] = ra[i];
    *reinterpret_cast<float4*>(Bs + buf * kBK * kBN + br * kBN + nc) =
        make_float4(rb[0], rb[1], rb[2], rb[3]);
  };

  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;

  const int64_t ntiles = (kend > kbeg) ? (kend - kbeg + kBK - 1) / kBK : 0;
  if (ntiles > 0) {
    load_tile(kbeg);
    store_tile(0);
    __syncthreads();
    for (int64_t t = 0; t < ntiles; ++t) {
      const int buf = static_cast<int>(t & 1);
      if (t + 1 < ntiles) load_tile(kbeg + (t + 1) * kBK);
      const float* as = As + buf * kBK * kApad;
      const float* bs = Bs + buf * kBK * kBN;
#pragma unroll
      for (int kk = 0; kk < kBK; ++kk) {
        const float4 a = *reinterpret_cast<const float4*>(as + kk * kApad + ty * 4);
        const float4 b = *reinterpret_cast<const float4*>(bs + kk * kBN + tx * 4);
        const float av[4] = {a.x, a.y, a.z, a.w};
        const float bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
      }
      if (t + 1 < ntiles) store_tile(buf ^ 1);
      __syncthreads();
    }
  }

  if (S == 1) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t m = m0 + ty * 4 + i;
      if (m >= M) continue;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int64_t n = n0 + tx * 4 + j;
        if (n < N) C[m * N + n] = acc[i][j];
      }
    }
    return;
  }

  // Split-K: reduce the S partials of this tile through distributed shared memory.
  cg::cluster_group cluster = cg::this_cluster();
  float* P = smem;  // [kBM][kBN]; the k-loop ended with a __syncthreads
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    *reinterpret_cast<float4*>(P + (ty * 4 + i) * kBN + tx * 4) =
        make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
  }
  cluster.sync();
  const int my_rows = (kBM - z + S - 1) / S;
  for (int e = tid; e < my_rows * kBN; e += kThreads) {
    const int r = z + S * (e / kBN);
    const int c = e % kBN;
    float v = 0.0f;
    for (int q = 0; q < S; ++q) {
      const float* peer = cluster.map_shared_rank(P, q);
      v += peer[r * kBN + c];
    }
    const int64_t m = m0 + r, n = n0 + c;
    if (m < M && n < N) C[m * N + n] = v;
  }
  cluster.sync();  // peers' shared memory must outlive every remote read
}

template <bool VEC, bool NORM>
int launch_sgemm(const float* A, const float* B, float* C, int64_t M, int64_t N, int64_t K,
                 const float* rms_w, float eps, cudaStream_t stream) {
  const int64_t gx = (N + kBN - 1) / kBN;
  const int64_t gy = (M + kBM - 1) / kBM;
  B200_REQUIRE(gy <= 65535, "matmul: M too large for the FP32 tile grid");
  B200_REQUIRE(gx <= 0x7fffffff, "matmul: N too large");
  const int sms = sm_count();
  const int64_t tiles = gx * gy;
  // Split K over a cluster of S CTAs while the tiles alone cannot fill `waves`
  // CTAs per SM.  The kernel is small (48 registers, 16 KB static shared
  // memory), so four fit per SM; on B200 waves = 4 took 512^3 from 27.7 to
  // 19.0 us per launch (S = 8, 512 CTAs).  ENGINE_SGEMM_WAVES overrides.
  static const int waves_env = [] {
    const char* e = std::getenv("ENGINE_SGEMM_WAVES");
    return (e && e[0]) ? static_cast<int>(std::strtol(e, nullptr, 10)) : 4;
  }();
  const int64_t slots = static_cast<int64_t>(sms) * (waves_env > 0 ? waves_env : 1);
  int S = 1;
  if (tiles < slots) {
    S = static_cast<int>(slots / tiles);
    if (S > 8) S = 8;
    const int64_t kmax = (K + 63) / 64;  // keep at least 64 of K per split
    if (S > kmax) S = static_cast<int>(kmax);
    if (S < 1) S = 1;
  }
  int64_t kchunk = (K + S - 1) / S;
  kchunk = (kchunk + kBK - 1) / kBK * kBK;

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(gx), static_cast<unsigned>(gy), static_cast<unsigned>(S));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = static_cast<unsigned>(S);
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  B200_CUDA(cudaLaunchKernelEx(&cfg, sgemm_kernel<VEC, NORM>, A, B, C, M, N, K, kchunk, S,
                               rms_w, eps));
  return ENGINE_OK;
}

}  // namespace

int sgemm(const float* A, const float* B, float* C, int64_t M, int64_t N, int64_t K,
          const float* rms_w, float eps, bool norm, cudaStream_t stream) {
  const bool vec = (K % 4 == 0) && (N % 4 == 0) &&
                   (reinterpret_cast<uintptr_t>(A) % 16 == 0) &&
                   (reinterpret_cast<uintptr_t>(B) % 16 == 0);
  int rc;
  if (norm) {
    rc = vec ? launch_sgemm<true, true>(A, B, C, M, N, K, rms_w, eps, stream)
             : launch_sgemm<false, true>(A, B, C, M, N, K, rms_w, eps, stream);
  } else {
    rc = vec ? launch_sgemm<true, false>(A, B, C, M, N, K, nullptr, 0.f, stream)
             : launch_sgemm<false, false>(A, B, C, M, N, K, nullptr, 0.f, stream);
  }
  if (rc != ENGINE_OK) return rc;
  return check_launch(norm ? "rmsnorm_linear" : "matmul");
}

}  // namespace b200

using namespace b200;

namespace {

int matmul_f32_entry(const char* name, const float* A, const float* B, float* C, int64_t M,
                     int64_t N, int64_t K, cudaStream_t stream) {
  const std::string n(name);
  B200_REQUIRE(A != nullptr, n + ": A is null");
  B200_REQUIRE(B != nullptr, n + ": B is null");
  B200_REQUIRE(C != nullptr, n + ": C is null");
  B200_REQUIRE(M >= 0, n + ": M must be non-negative");
  B200_REQUIRE(N >= 0, n + ": N must be non-negative");
  B200_REQUIRE(K >= 0, n + ": K must be non-negative");
  if (M == 0 || N == 0) return ENGINE_OK;
  if (K == 0) {  // an Mx0 times 0xN product is the MxN zero matrix
    B200_CUDA(cudaMemsetAsync(C, 0, static_cast<size_t>(M) * static_cast<size_t>(N) * sizeof(float),
                              stream));
    return ENGINE_OK;
  }
  return sgemm(A, B, C, M, N, K, nullptr, 0.f, false, stream);
}

int rmsnorm_linear_entry(const float* in, const float* rms_weight, const float* W, float* out,
                         int64_t M, int64_t N, int64_t K, float eps, cudaStream_t stream) {
  B200_REQUIRE(M >= 0 && N >= 0 && K >= 0, "rmsnorm_linear: negative dimension");
  B200_REQUIRE(in != nullptr && W != nullptr && out != nullptr,
               "rmsnorm_linear: null device pointer");
  B200_REQUIRE(eps >= 0.0f, "rmsnorm_linear: eps must be non-negative");
  if (M == 0 || N == 0 || K == 0) return ENGINE_OK;
  if (M == 1) return gemv_kn_f32(W, in, out, N, K, rms_weight, eps, true, stream);
  return sgemm(in, W, out, M, N, K, rms_weight, eps, true, stream);
}

}  // namespace

extern "C" {

int engine_cuda_matmul_naive(const float* A, const float* B, float* C, int64_t M, int64_t N,
                             int64_t K, engine_stream_t stream) {
  B200_ENTRY_BEGIN
  return matmul_f32_entry("matmul_naive", A, B, C, M, N, K, stream);
  B200_ENTRY_END
}

int engine_cuda_matmul_tiled(const float* A, const float* B, float* C, int64_t M, int64_t N,
                             int64_t K, engine_stream_t stream) {
  B200_ENTRY_BEGIN
  return matmul_f32_entry("matmul_tiled", A, B, C, M, N, K, stream);
  B200_ENTRY_END
}

int engine_cuda_matmul_register_tiled(const float* A, const float* B, float* C, int64_t M,
                                      int64_t N, int64_t K, engine_stream_t stream) {
  B200_ENTRY_BEGIN
  return matmul_f32_entry("matmul_register_tiled", A, B, C, M, N, K, stream);
  B200_ENTRY_END
}

int engine_cuda_rmsnorm_linear(const float* in, const float* rms_weight, const float* W,
                               float* out, int64_t M, int64_t N, int64_t K, float eps,
                               engine_stream_t stream) {
  B200_ENTRY_BEGIN
  return rmsnorm_linear_entry(in, rms_weight, W, out, M, N, K, eps, stream);
  B200_ENTRY_END
}

int engine_cuda_rmsnorm_linear_fused_direct(const float* in, const float* rms_weight,
                                            const float* W, float* out, int64_t M, int64_t N,
                                            int64_t K, float eps, engine_stream_t stream) {
  B200_ENTRY_BEGIN
  return rmsnorm_linear_entry(in, rms_weight, W, out, M, N, K, eps, stream);
  B200_ENTRY_END
}

}  // extern "C"
