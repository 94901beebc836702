// gemv.cu -- HBM-streaming matrix-vector products.
//
// 1. gemv_nk_vec_kernel: y[m, n] = sum_k X[m, k] * W[n, k] for up to four rows
//    of X (batch-1 and tiny-batch decode) over weights stored [N,K], K
//    contiguous -- the layout of the B200 decode configuration.  A group of SK
//    warps owns RPW weight rows; each lane streams 16-byte (8 x FP16) chunks of
//    those rows with L1::no_allocate loads, software-pipelined so 2*U chunks per
//    row are in flight, multiplies them with the matching chunks of X
//    (L1-resident after the first warp) and reduces with warp shuffles, then
//    across the SK warps through shared memory.  SK is chosen so that about 8k
//    warps stream W at once (N=4096 -> SK=2).  Optional fused RMSNorm (sum(x^2)
//    is accumulated in the same pass, the scale applied after the dot product)
//    and residual epilogue.
// 2. gemv_kn_kernel: out[n] = sum_k x[k] * A[k, n] over the reference's legacy
//    [K,N] layout (engine::cuda::gemv / gemv_fp16, kernels/gemv*.cu).  A warp
//    covers 32 x 16 bytes of one row of A per k, eight warps split K inside the
//    CTA, and up to eight CTAs of a thread-block cluster split it further,
//    reducing through distributed shared memory (no global scratch).
// 3. rmsnorm_f16_kernel: row RMSNorm FP16 -> FP16 for the tensor-core path of
//    rmsnorm_linear_f16.
#include <cooperative_groups.h>

#include <atomic>
#include <cstdlib>

#include "common.cuh"
#include "gemv_core.cuh"
#include "kernels.cuh"

namespace cg = cooperative_groups;

namespace b200 {
namespace {

// ---------------------------------------------------------------- [N,K] GEMV

constexpr int kNkWarps = 4;     // scalar fallback: one row per warp

// Decode GEMV kernel: one row block per CTA (nk_block_dots), then the SK
// partial sums of each row are added in fixed order, scaled by the RMS factor
// when NORM, plus the residual, rounded once to FP16.
template <int MR, int RPW, int SK, int U, bool NORM, bool RESID>
__global__ void __launch_bounds__(kNkVecWarps * 32) gemv_nk_vec_kernel(
    const __half* __restrict__ W, const __half* __restrict__ X, const __half* __restrict__ gamma,
    const __half* __restrict__ R, __half* __restrict__ Y, int64_t N, int64_t K, float eps) {
  constexpr int GROUPS = kNkVecWarps / SK;
  constexpr int NACC = MR * RPW + (NORM ? MR : 0);
  __shared__ float red[kNkVecWarps][NACC];
  pdl_trigger();
  nk_block_prefetch<RPW, SK, U>(W, N, K, blockIdx.x);
  pdl_wait();
  nk_block_dots<MR, RPW, SK, U, NORM>(W, X, gamma, N, K, blockIdx.x, red);
  for (int o = threadIdx.x; o < GROUPS * MR * RPW; o += blockDim.x) {
    const int g = o / (MR * RPW);
    const int rem = o % (MR * RPW);
    const int m = rem / RPW;
    const int r = rem % RPW;
    const int64_t row = (static_cast<int64_t>(blockIdx.x) * GROUPS + g) * RPW + r;
    if (row >= N) continue;
    float v = 0.0f;
#pragma unroll
    for (int q = 0; q < SK; ++q) v += red[g * SK + q][m * RPW + r];
    if constexpr (NORM) {
      float s2 = 0.0f;
#pragma unroll
      for (int q = 0; q < SK; ++q) s2 += red[g * SK + q][MR * RPW + m];
      v = v * static_cast<float>(1.0 / sqrt(static_cast<double>(s2) / static_cast<double>(K) +
                                            static_cast<double>(eps)));
    }
    if constexpr (RESID) v = v + __half2float(R[m * N + row]);
    Y[m * N + row] = __float2half_rn(v);
  }
}

// KV-cache scatter of the batch-1 norm projection (engine_cuda_rmsnorm_linear_kv_f16):
// output rows [n0, n0 + nkv) are the new token's K row and [n0 + nkv, n0 + 2 nkv)
// its V row; each is also stored at position `pos` of its head in the caches
// ([heads][max_len][d]: element c of head h at h * head_stride + pos_off + c).
struct KvScatter {
  __half* k = nullptr;
  __half* v = nullptr;
  int64_t n0 = 0, nkv = 0, d = 1, head_stride = 0, pos_off = 0;
};

// Batch-1 fused RMSNorm -> GEMV.  Persistent: each CTA forms t = x * gamma
// (FP32) in shared memory and the sum of squares of x with one block reduction
// -- once per CTA, not once per row block -- then streams row block after row
// block (blockIdx.x, + gridDim.x, ...) against t.  The RMS scale multiplies each
// finished dot product: y = scale * sum_k t_k W_nk (+ residual).  The first row
// block's first weight chunks are prefetched into L2 before griddepcontrol.wait
// and loaded before the prologue, so HBM is busy while t is formed.
//
// PAIR (the SwiGLU projection): W holds 2N rows, gate rows [0, N) then up rows
// [N, 2N).  Warp group j streams the pair (j, N + j) -- each row accumulated
// exactly as without PAIR -- and writes swiglu(fp16(gate_j), fp16(up_j)).
// With kv.k set, the store loop also writes the K / V rows into the caches.
template <int RPW, int SK, int U, bool RESID, bool PAIR = false>
__global__ void __launch_bounds__(kNkVecWarps * 32) gemv_nk_norm1_kernel(
    const __half* __restrict__ W, const __half* __restrict__ X, const __half* __restrict__ gamma,
    const __half* __restrict__ R, __half* __restrict__ Y, int64_t N, int64_t K, float eps,
    const KvScatter kv) {
  constexpr int GROUPS = kNkVecWarps / SK;
  static_assert(!PAIR || (RPW == 2 && !RESID), "PAIR streams one gate/up row pair per group");
  constexpr int64_t ROWS = static_cast<int64_t>(GROUPS) * (PAIR ? 1 : RPW);  // outputs per block
  extern __shared__ __align__(16) float s_t[];  // K floats
  __shared__ float red[kNkVecWarps][RPW];
  __shared__ float s_ss[kNkVecWarps];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int grp = warp / SK;
  const int sub = warp % SK;
  const int64_t nchunk = K >> 3;
  const int64_t nblocks = (N + ROWS - 1) / ROWS;
  constexpr int64_t kStride = 32 * SK;

  const __half* wrow[RPW];
  auto set_rows = [&](int64_t b) {
    if constexpr (PAIR) {
      const int64_t j = b * GROUPS + grp;
      const int64_t jc = (j < N) ? j : N - 1;  // clamp: never stored
      wrow[0] = W + jc * K;
      wrow[1] = W + (N + jc) * K;
      return j < N;
    } else {
      const int64_t row0 = (b * GROUPS + grp) * RPW;
#pragma unroll
      for (int r = 0; r < RPW; ++r) {
        const int64_t n = (row0 + r < N) ? row0 + r : N - 1;  // clamp: never stored
        wrow[r] = W + n * K;
      }
      return row0 < N;
    }
  };
  uint4 wa[U][RPW], wb[U][RPW];
  auto load = [&](int64_t c0, uint4 (&w)[U][RPW]) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t c = c0 + kStride * u;
      if (c < nchunk) {
#pragma unroll
        for (int r = 0; r < RPW; ++r) w[u][r] = ld_stream_v4(wrow[r] + 8 * c);
      }
    }
  };
  const int64_t cstart = sub * 32 + lane;
  bool active = set_rows(blockIdx.x);
  pdl_trigger();
  if (active) {  // warm L2 with the first weight chunks while the preceding kernel drains
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t c = cstart + kStride * u;
      if (c < nchunk) {
#pragma unroll
        for (int r = 0; r < RPW; ++r) prefetch_l2(wrow[r] + 8 * c);
      }
    }
  }
  pdl_wait();
  if (active) load(cstart, wa);

  // Prologue: t = x * gamma into shared memory, sum of squares of x.
  float ss = 0.0f;
  for (int64_t k8 = threadIdx.x; k8 < nchunk; k8 += blockDim.x) {
    float xf[8], gf[8];
    h8_to_f8(__ldg(reinterpret_cast<const uint4*>(X + 8 * k8)), xf);
    if (gamma != nullptr) {
      h8_to_f8(__ldg(reinterpret_cast<const uint4*>(gamma + 8 * k8)), gf);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) gf[i] = 1.0f;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      ss = fmaf(xf[i], xf[i], ss);
      xf[i] *= gf[i];
    }
    // Two planes (elements 0-3 and 4-7 of each 8-element chunk): the lanes of a
    // warp then read 16-byte words at a 16-byte stride, free of bank conflicts.
    *reinterpret_cast<float4*>(s_t + 4 * k8) = make_float4(xf[0], xf[1], xf[2], xf[3]);
    *reinterpret_cast<float4*>(s_t + 4 * (nchunk + k8)) = make_float4(xf[4], xf[5], xf[6], xf[7]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (lane == 0) s_ss[warp] = ss;
  __syncthreads();
  float total = 0.0f;
#pragma unroll
  for (int w = 0; w < kNkVecWarps; ++w) total += s_ss[w];
  const float scale = static_cast<float>(
      1.0 / sqrt(static_cast<double>(total) / static_cast<double>(K) + static_cast<double>(eps)));

  for (int64_t b = blockIdx.x; b < nblocks; b += gridDim.x) {
    if (b != blockIdx.x) {
      active = set_rows(b);
      if (active) load(cstart, wa);
    }
    float acc[RPW];
#pragma unroll
    for (int r = 0; r < RPW; ++r) acc[r] = 0.0f;
    auto compute = [&](int64_t cc, uint4 (&w)[U][RPW]) {
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t c = cc + kStride * u;
        if (c < nchunk) {
          const float4 t0 = *reinterpret_cast<const float4*>(s_t + 4 * c);
          const float4 t1 = *reinterpret_cast<const float4*>(s_t + 4 * (nchunk + c));
          const float tf[8] = {t0.x, t0.y, t0.z, t0.w, t1.x, t1.y, t1.z, t1.w};
#pragma unroll
          for (int r = 0; r < RPW; ++r) {
            float wf[8];
            h8_to_f8(w[u][r], wf);
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[r] = fmaf(tf[i], wf[i], acc[r]);
          }
        }
      }
    };
    if (active) {
      for (int64_t c0 = cstart; c0 < nchunk; c0 += 2 * kStride * U) {
        const int64_t c1 = c0 + kStride * U;
        load(c1, wb);
        compute(c0, wa);
        load(c1 + kStride * U, wa);
        compute(c1, wb);
      }
    }
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
    }
    if (lane == 0) {
#pragma unroll
      for (int r = 0; r < RPW; ++r) red[warp][r] = acc[r];
    }
    __syncthreads();
    if constexpr (PAIR) {
      for (int o = threadIdx.x; o < GROUPS; o += blockDim.x) {
        const int64_t j = b * GROUPS + o;
        if (j >= N) continue;
        float vg = 0.0f, vu = 0.0f;
#pragma unroll
        for (int q = 0; q < SK; ++q) {
          vg += red[o * SK + q][0];
          vu += red[o * SK + q][1];
        }
        Y[j] = swiglu_h(__float2half_rn(vg * scale), __float2half_rn(vu * scale));
      }
    } else {
      for (int o = threadIdx.x; o < GROUPS * RPW; o += blockDim.x) {
        const int g = o / RPW;
        const int r = o % RPW;
        const int64_t row = (b * GROUPS + g) * RPW + r;
        if (row >= N) continue;
        float v = 0.0f;
#pragma unroll
        for (int q = 0; q < SK; ++q) v += red[g * SK + q][r];
        v = v * scale;
        if constexpr (RESID) v = v + __half2float(R[row]);
        const __half h = __float2half_rn(v);
        Y[row] = h;
        if (kv.k != nullptr) {
          const int64_t e = row - kv.n0;
          if (e >= 0 && e < 2 * kv.nkv) {
            const bool is_v = e >= kv.nkv;
            const int64_t f = is_v ? e - kv.nkv : e;
            (is_v ? kv.v : kv.k)[(f / kv.d) * kv.head_stride + kv.pos_off + f % kv.d] = h;
          }
        }
      }
    }
    __syncthreads();  // `red` is reused by the next row block
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

template <int MR, int RPW, int SK, bool NORM, bool RESID>
void launch_nk_vec(const __half* W, const __half* X, const __half* gamma, const __half* R,
                   __half* Y, int64_t N, int64_t K, float eps, cudaStream_t stream) {
  constexpr int U = (MR >= 3) ? 2 : 4;
  constexpr int64_t rows_per_cta = static_cast<int64_t>(kNkVecWarps / SK) * RPW;
  const unsigned grid = static_cast<unsigned>((N + rows_per_cta - 1) / rows_per_cta);
  launch_pdl(gemv_nk_vec_kernel<MR, RPW, SK, U, NORM, RESID>, dim3(grid), dim3(kNkVecWarps * 32),
             0, stream, W, X, gamma, R, Y, N, K, eps);
}

template <int RPW, int SK, bool RESID, bool PAIR = false>
int launch_nk_norm1(const __half* W, const __half* X, const __half* gamma, const __half* R,
                    __half* Y, int64_t N, int64_t K, float eps, cudaStream_t stream,
                    const KvScatter& kv = KvScatter{}) {
  constexpr int64_t rows_per_cta = static_cast<int64_t>(kNkVecWarps / SK) * (PAIR ? 1 : RPW);
  const int64_t nblocks = (N + rows_per_cta - 1) / rows_per_cta;
  const size_t smem = static_cast<size_t>(K) * sizeof(float);
  auto kern = gemv_nk_norm1_kernel<RPW, SK, 4, RESID, PAIR>;
  int dev = 0;
  B200_CUDA(cudaGetDevice(&dev));
  if (smem > 48 * 1024) {  // opt in once per device to the largest size the dispatch allows
    static std::atomic<uint64_t> configured{0};
    const uint64_t bit = 1ull << (dev & 63);
    if ((configured.load() & bit) == 0) {
      B200_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(40960 * sizeof(float))));
      configured.fetch_or(bit);
    }
  }
  // Persistent grid: as many CTAs as are resident at once (the prologue runs
  // once per CTA), never more than there are row blocks.  When every CTA gets
  // only a few row blocks, the grid shrinks so that all get the same number:
  // a CTA with one block more than the others is the launch's tail (W[6144,4096]:
  // 768 blocks as 256 CTAs x 3 instead of 296 CTAs with 2 or 3, 11.7 -> 11.2 us;
  // W[4096,4096]: 8.5 -> 8.1 us; at 50+ blocks per CTA it does not pay).
  int per_sm = 0;
  B200_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kNkVecWarps * 32, smem));
  if (per_sm < 1) per_sm = 1;
  const int64_t resident = static_cast<int64_t>(per_sm) * sm_count();
  int64_t g = nblocks < resident ? nblocks : resident;
  if (g > 0) {
    const int64_t per = (nblocks + g - 1) / g;
    if (per <= 4) g = (nblocks + per - 1) / per;
  }
  const unsigned grid = static_cast<unsigned>(g);
  B200_CUDA(launch_pdl(kern, dim3(grid), dim3(kNkVecWarps * 32), smem, stream, W, X, gamma, R, Y,
                       N, K, eps, kv));
  return ENGINE_OK;
}

template <int MR, int RPW, bool NORM, bool RESID>
void dispatch_sk(int sk, const __half* W, const __half* X, const __half* gamma, const __half* R,
                 __half* Y, int64_t N, int64_t K, float eps, cudaStream_t stream) {
  if (sk >= 4) {
    launch_nk_vec<MR, RPW, 4, NORM, RESID>(W, X, gamma, R, Y, N, K, eps, stream);
  } else if (sk == 2) {
    launch_nk_vec<MR, RPW, 2, NORM, RESID>(W, X, gamma, R, Y, N, K, eps, stream);
  } else {
    launch_nk_vec<MR, RPW, 1, NORM, RESID>(W, X, gamma, R, Y, N, K, eps, stream);
  }
}

template <bool NORM, bool RESID>
void dispatch_mr(int64_t mr, int rpw, int sk, const __half* W, const __half* X,
                 const __half* gamma, const __half* R, __half* Y, int64_t N, int64_t K, float eps,
                 cudaStream_t stream) {
  switch (mr) {
    case 1:
      if (rpw >= 2) dispatch_sk<1, 2, NORM, RESID>(sk, W, X, gamma, R, Y, N, K, eps, stream);
      else dispatch_sk<1, 1, NORM, RESID>(sk, W, X, gamma, R, Y, N, K, eps, stream);
      break;
    case 2: dispatch_sk<2, 1, NORM, RESID>(sk, W, X, gamma, R, Y, N, K, eps, stream); break;
    case 3: dispatch_sk<3, 1, NORM, RESID>(sk, W, X, gamma, R, Y, N, K, eps, stream); break;
    default: dispatch_sk<4, 1, NORM, RESID>(sk, W, X, gamma, R, Y, N, K, eps, stream); break;
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
  // Defaults from a sweep over the B200 decode shapes (CUDA-graph timing, cold
  // L2): two weight rows per warp group; each row split over two warps unless K
  // is long enough (> 8192) to keep one warp busy.  The fused-norm variant keeps
  // one row per group (its per-chunk x-side work doubles the register load).
  // ENGINE_GEMV_RPW / ENGINE_GEMV_SK override them for tuning sweeps.
  static const int rpw_env = env_int("ENGINE_GEMV_RPW", 0);
  static const int sk_env = env_int("ENGINE_GEMV_SK", 0);
  const int rpw = rpw_env > 0 ? rpw_env : (norm ? 1 : 2);
  int sk = sk_env > 0 ? sk_env : ((norm || K <= 8192) ? 2 : 1);
  sk = sk >= 4 ? 4 : (sk >= 2 ? 2 : 1);
  static const int norm1_env = env_int("ENGINE_GEMV_NORM1", 1);
  if (norm && M == 1 && norm1_env != 0 && K <= 40960) {
    // Batch-1 fused norm: x * gamma formed once per CTA in shared memory.
    const int nsk = sk_env > 0 ? sk : 2;
    const int nrpw = rpw_env > 0 ? rpw : 2;
    int rc;
    if (residual) {
      rc = (nrpw >= 2) ? (nsk >= 2 ? launch_nk_norm1<2, 2, true>(W, X, gamma, residual, Y, N, K, eps, stream)
                                   : launch_nk_norm1<2, 1, true>(W, X, gamma, residual, Y, N, K, eps, stream))
                       : (nsk >= 2 ? launch_nk_norm1<1, 2, true>(W, X, gamma, residual, Y, N, K, eps, stream)
                                   : launch_nk_norm1<1, 1, true>(W, X, gamma, residual, Y, N, K, eps, stream));
    } else {
      rc = (nrpw >= 2) ? (nsk >= 2 ? launch_nk_norm1<2, 2, false>(W, X, gamma, residual, Y, N, K, eps, stream)
                                   : launch_nk_norm1<2, 1, false>(W, X, gamma, residual, Y, N, K, eps, stream))
                       : (nsk >= 2 ? launch_nk_norm1<1, 2, false>(W, X, gamma, residual, Y, N, K, eps, stream)
                                   : launch_nk_norm1<1, 1, false>(W, X, gamma, residual, Y, N, K, eps, stream));
    }
    if (rc != ENGINE_OK) return rc;
    return check_launch("rmsnorm_linear_f16 (batch-1 GEMV)");
  }
  for (int64_t m0 = 0; m0 < M; m0 += 4) {
    const int64_t mr = (M - m0 < 4) ? M - m0 : 4;
    const __half* Xm = X + m0 * K;
    const __half* Rm = residual ? residual + m0 * N : nullptr;
    __half* Ym = Y + m0 * N;
    if (norm) {
      if (residual) dispatch_mr<true, true>(mr, rpw, sk, W, Xm, gamma, Rm, Ym, N, K, eps, stream);
      else dispatch_mr<true, false>(mr, rpw, sk, W, Xm, gamma, Rm, Ym, N, K, eps, stream);
    } else {
      if (residual) dispatch_mr<false, true>(mr, rpw, sk, W, Xm, gamma, Rm, Ym, N, K, eps, stream);
      else dispatch_mr<false, false>(mr, rpw, sk, W, Xm, gamma, Rm, Ym, N, K, eps, stream);
    }
  }
  return check_launch("gemv_f16_nk");
}

int gemv_nk_norm1_swiglu_f16(const __half* W, const __half* X, const __half* gamma, float eps,
                             __half* Y, int64_t F, int64_t K, cudaStream_t stream) {
  const bool vec = (K % 8 == 0) && (reinterpret_cast<uintptr_t>(W) % 16 == 0) &&
                   (reinterpret_cast<uintptr_t>(X) % 16 == 0) &&
                   (gamma == nullptr || reinterpret_cast<uintptr_t>(gamma) % 16 == 0);
  static const int norm1_env = env_int("ENGINE_GEMV_NORM1", 1);
  if (!vec || K > 40960 || norm1_env == 0) return ENGINE_ERR_UNSUPPORTED;
  // Same warps per row as the unfused batch-1 norm GEMV, so each gate / up row
  // is accumulated identically.
  static const int sk_env = env_int("ENGINE_GEMV_SK", 0);
  const int rc = (sk_env == 1)
                     ? launch_nk_norm1<2, 1, false, true>(W, X, gamma, nullptr, Y, F, K, eps, stream)
                     : launch_nk_norm1<2, 2, false, true>(W, X, gamma, nullptr, Y, F, K, eps, stream);
  if (rc != ENGINE_OK) return rc;
  return check_launch("rmsnorm_linear_swiglu_f16 (batch-1 GEMV)");
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

int engine_cuda_rmsnorm_linear_kv_f16(const engine_half_t* x, const engine_half_t* gamma,
                                      const engine_half_t* W, const engine_half_t* residual,
                                      engine_half_t* Y, int64_t N, int64_t K, float eps,
                                      engine_half_t* k_cache, engine_half_t* v_cache,
                                      int64_t kv_row0, int64_t n_kv_heads, int64_t head_dim,
                                      int64_t max_len, int64_t pos, engine_stream_t stream) {
  B200_ENTRY_BEGIN
  B200_REQUIRE(N >= 0 && K >= 0, "rmsnorm_linear_kv_f16: negative dimension");
  B200_REQUIRE(x != nullptr && W != nullptr && Y != nullptr,
               "rmsnorm_linear_kv_f16: null device pointer");
  B200_REQUIRE(k_cache != nullptr && v_cache != nullptr, "rmsnorm_linear_kv_f16: cache is null");
  B200_REQUIRE(eps >= 0.0f, "rmsnorm_linear_kv_f16: eps must be non-negative");
  B200_REQUIRE(n_kv_heads > 0 && head_dim > 0, "rmsnorm_linear_kv_f16: n_kv_heads and head_dim must be positive");
  B200_REQUIRE(kv_row0 >= 0 && kv_row0 + 2 * n_kv_heads * head_dim <= N,
               "rmsnorm_linear_kv_f16: the K and V rows must lie inside the N output rows");
  B200_REQUIRE(pos >= 0 && pos < max_len, "rmsnorm_linear_kv_f16: pos must lie in [0, max_len)");
  B200_REQUIRE(K > 0 && K % 8 == 0 && K <= 40960, "rmsnorm_linear_kv_f16: K must be a positive multiple of 8, at most 40960");
  B200_REQUIRE(((reinterpret_cast<uintptr_t>(W) | reinterpret_cast<uintptr_t>(x) |
                 reinterpret_cast<uintptr_t>(gamma)) % 16) == 0,
               "rmsnorm_linear_kv_f16: W, x and gamma must be 16-byte aligned");
  if (N == 0) return ENGINE_OK;
  KvScatter kv;
  kv.k = reinterpret_cast<__half*>(k_cache);
  kv.v = reinterpret_cast<__half*>(v_cache);
  kv.n0 = kv_row0;
  kv.nkv = n_kv_heads * head_dim;
  kv.d = head_dim;
  kv.head_stride = max_len * head_dim;
  kv.pos_off = pos * head_dim;
  const auto* wh = reinterpret_cast<const __half*>(W);
  const auto* xh = reinterpret_cast<const __half*>(x);
  const auto* gh = reinterpret_cast<const __half*>(gamma);
  const auto* rh = reinterpret_cast<const __half*>(residual);
  auto* yh = reinterpret_cast<__half*>(Y);
  // The batch-1 configuration of engine_cuda_rmsnorm_linear_f16 (two rows per
  // warp group, K split over two warps), so Y is bit-identical to it.
  const int rc = rh ? launch_nk_norm1<2, 2, true>(wh, xh, gh, rh, yh, N, K, eps, stream, kv)
                    : launch_nk_norm1<2, 2, false>(wh, xh, gh, rh, yh, N, K, eps, stream, kv);
  if (rc != ENGINE_OK) return rc;
  return check_launch("rmsnorm_linear_kv_f16");
  B200_ENTRY_END
}

}  // extern "C"
