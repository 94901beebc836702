// gemv_core.cuh -- the [N,K] GEMV row-block dot products shared by the decode
// GEMV kernels (gemv.cu) and the fused projection + all-reduce (tp_comm.cu).
#pragma once

#include "common.cuh"

namespace b200 {
namespace {

constexpr int kNkVecWarps = 8;  // vector kernels: 8 warps per CTA

__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
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

// Prefetches into L2 the first weight chunks that nk_block_dots<.., RPW, SK, U>
// will load for row block `block`.  Kernels launched as programmatic dependents
// call it before griddepcontrol.wait: weights are streamed from HBM while the
// preceding kernel drains.  L2 is the device's point of coherence, so this
// cannot return stale data even if the preceding kernel writes W (every load
// still happens after the wait).
template <int RPW, int SK, int U>
__device__ __forceinline__ void nk_block_prefetch(const __half* __restrict__ W, int64_t N,
                                                  int64_t K, int64_t block) {
  constexpr int GROUPS = kNkVecWarps / SK;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int64_t row0 = (block * GROUPS + warp / SK) * RPW;
  const int64_t c0 = (warp % SK) * 32 + lane;
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    if (row0 + r >= N) break;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t c = c0 + 32 * SK * u;
      if (c < (K >> 3)) prefetch_l2(W + (row0 + r) * K + 8 * c);
    }
  }
}

// Row block `block` of y[m, n] = sum_k X[m, k] W[n, k] (m < MR): the CTA's
// kNkVecWarps / SK warp groups own RPW consecutive weight rows each, and the SK
// warps of a group share its rows: lane l of warp `sub` streams the
// 16-byte chunks c = sub*32 + l + i*32*SK of every row, so the SK warps of a
// group read 512*SK contiguous bytes per step.  Loads are software-pipelined
// (two register buffers of U chunks per row: the next U chunks are in flight
// while the current ones are multiplied).  Each warp's partial sums (and, with
// NORM, its sums of x^2) end in red[warp][m * RPW + r] (red[warp][MR*RPW + m]);
// the caller reduces them across the SK warps in fixed order after the
// __syncthreads() this function ends with.
template <int MR, int RPW, int SK, int U, bool NORM>
__device__ __forceinline__ void nk_block_dots(const __half* __restrict__ W,
                                              const __half* __restrict__ X,
                                              const __half* __restrict__ gamma, int64_t N,
                                              int64_t K, int64_t block,
                                              float (*red)[MR * RPW + (NORM ? MR : 0)]) {
  constexpr int GROUPS = kNkVecWarps / SK;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int grp = warp / SK;
  const int sub = warp % SK;
  const int64_t row0 = (block * GROUPS + grp) * RPW;
  const int64_t nchunk = K >> 3;  // 8 halves per 16-byte chunk
  constexpr int64_t kStride = 32 * SK;

  float acc[MR][RPW];
  float ss[MR];
#pragma unroll
  for (int m = 0; m < MR; ++m) {
    ss[m] = 0.0f;
#pragma unroll
    for (int r = 0; r < RPW; ++r) acc[m][r] = 0.0f;
  }
  if (row0 < N) {
    const __half* wrow[RPW];
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
      const int64_t n = (row0 + r < N) ? row0 + r : N - 1;  // clamp: never stored
      wrow[r] = W + n * K;
    }
    uint4 wa[U][RPW], xa[U][MR], ga[U];
    uint4 wb[U][RPW], xb[U][MR], gb[U];
    auto load_w = [&](int64_t c0, uint4 (&w)[U][RPW]) {
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t c = c0 + kStride * u;
        if (c < nchunk) {
#pragma unroll
          for (int r = 0; r < RPW; ++r) w[u][r] = ld_stream_v4(wrow[r] + 8 * c);
        }
      }
    };
    auto load_xg = [&](int64_t c0, uint4 (&x)[U][MR], uint4 (&g)[U]) {
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t c = c0 + kStride * u;
        if (c < nchunk) {
#pragma unroll
          for (int m = 0; m < MR; ++m)
            x[u][m] = __ldg(reinterpret_cast<const uint4*>(X + m * K + 8 * c));
          if constexpr (NORM) {
            g[u] = gamma ? __ldg(reinterpret_cast<const uint4*>(gamma + 8 * c))
                         : make_uint4(0x3c003c00u, 0x3c003c00u, 0x3c003c00u, 0x3c003c00u);
          }
        }
      }
    };
    auto load = [&](int64_t c0, uint4 (&w)[U][RPW], uint4 (&x)[U][MR], uint4 (&g)[U]) {
      load_w(c0, w);
      load_xg(c0, x, g);
    };
    auto compute = [&](int64_t c0, uint4 (&w)[U][RPW], uint4 (&x)[U][MR], uint4 (&g)[U]) {
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t c = c0 + kStride * u;
        if (c < nchunk) {
          float gf[8];
          if constexpr (NORM) h8_to_f8(g[u], gf);
#pragma unroll
          for (int m = 0; m < MR; ++m) {
            float xf[8];
            h8_to_f8(x[u][m], xf);
            if constexpr (NORM) {
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                ss[m] = fmaf(xf[i], xf[i], ss[m]);
                xf[i] *= gf[i];
              }
            }
#pragma unroll
            for (int r = 0; r < RPW; ++r) {
              float wf[8];
              h8_to_f8(w[u][r], wf);
#pragma unroll
              for (int i = 0; i < 8; ++i) acc[m][r] = fmaf(xf[i], wf[i], acc[m][r]);
            }
          }
        }
      }
    };
    int64_t c0 = sub * 32 + lane;
    load(c0, wa, xa, ga);
    for (; c0 < nchunk; c0 += 2 * kStride * U) {
      const int64_t c1 = c0 + kStride * U;
      load(c1, wb, xb, gb);
      compute(c0, wa, xa, ga);
      load(c1 + kStride * U, wa, xa, ga);
      compute(c1, wb, xb, gb);
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
  if (lane == 0) {
#pragma unroll
    for (int m = 0; m < MR; ++m) {
#pragma unroll
      for (int r = 0; r < RPW; ++r) red[warp][m * RPW + r] = acc[m][r];
      if constexpr (NORM) red[warp][MR * RPW + m] = ss[m];
    }
  }
  __syncthreads();
}

}  // namespace
}  // namespace b200
