// gemv_quant.cu -- decode GEMV over block-quantised weights (Q8_0 / Q4_0).
//
// Format (GGUF's, as declared by the engine: include/engine/dtype.hpp:95-125,
// kQuantBlockSize = 32).  A row of K weights is K/32 blocks, each with one FP16
// scale d:
//   Q8_0 block: { half d; int8  q[32]; }        34 bytes, w[i] = d * q[i]
//   Q4_0 block: { half d; uint8 nib[16]; }      18 bytes, w[j] = d * (lo(nib[j]) - 8),
//                                                         w[j+16] = d * (hi(nib[j]) - 8)
// GGUF stores these blocks packed back to back (34- and 18-byte strides), which
// is not 16-byte aligned.  engine_cuda_quant_repack() converts them once, at load
// time, into the layout the GEMV streams:
//   payload  [N][K] int8 (Q8_0) or [N][K/2] nibble bytes (Q4_0, each block's 16
//            bytes kept in the GGUF order), 16-byte aligned rows;
//   scales   [N][K/32] FP16.
//
// GEMV: y[n] = sum_b d[n,b] * (sum_{i<32} q[n,32b+i] * x[32b+i]) (+ residual).
// - Each lane owns whole blocks; the 32 lanes of a warp cover 32 consecutive
//   blocks of a row: 1 KB of Q8_0 or 512 B of Q4_0 payload per warp step.
//   A warp group (one warp, or two splitting K) owns four rows, so each x chunk
//   it loads from L1 is multiplied into four rows' payload.
// - Payload loads are 16-byte `ld.global.nc.L1::no_allocate`; scales (64 B per
//   warp step) and x come through L1.
// - Weights are widened to exact FP16 values by bit arithmetic (no int->float
//   conversion); the 32 products of a block are exact in FP32 (a half times a
//   half) and are summed in FP32 by mixed-precision fma, multiplied by d and
//   accumulated per lane.
// - The warp shuffle and the cross-warp sum run in fixed order.
// HBM bytes per weight: 1.0625 (Q8_0) or 0.5625 (Q4_0), against 2 for FP16.
#include "common.cuh"
#include "gemv_core.cuh"
#include "kernels.cuh"

namespace b200 {
namespace {

constexpr int kQWarps = 8;

// One GGUF block -> the split layout.  One thread per block.
template <int QT>
__global__ void quant_repack_kernel(const uint8_t* __restrict__ blocks, uint8_t* __restrict__ q,
                                    __half* __restrict__ d, int64_t N, int64_t nblk) {
  constexpr int PAY = QT == 8 ? 32 : 16;
  constexpr int BLK = 2 + PAY;
  pdl_trigger();
  pdl_wait();
  const int64_t total = N * nblk;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint8_t* src = blocks + i * BLK;
    const uint16_t bits = static_cast<uint16_t>(src[0] | (src[1] << 8));
    d[i] = __ushort_as_half(bits);
    uint8_t* dst = q + i * PAY;  // row n, block b: (n * nblk + b) * PAY
#pragma unroll
    for (int k = 0; k < PAY; ++k) dst[k] = src[2 + k];
  }
}

// Integer weights become FP16 halves without an int->float conversion (the
// magic-number method; for 4-bit nibbles the LOP3 form of Kim et al., "Who Says
// Elephants Can't Run?", 2022): a value u < 1024 placed in the mantissa of
// 0x6400 (1024.0) reads as 1024 + u, and one f16x2 subtract (or, for a nibble
// in bits 4-7, one f16x2 fma by 1/16) leaves the signed weight exactly.
__device__ __forceinline__ uint32_t h2_sub(uint32_t a, uint32_t b) {
  __half2 r = __hsub2(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}
__device__ __forceinline__ uint32_t h2_fma(uint32_t a, uint32_t b, uint32_t c) {
  __half2 r = __hfma2(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b),
                      *reinterpret_cast<const __half2*>(&c));
  return *reinterpret_cast<uint32_t*>(&r);
}

// s += q.lo * x.lo; s += q.hi * x.hi -- sm_100 mixed-precision fma: FP16 inputs,
// FP32 accumulator, one rounding (the product of two halves is exact in FP32, so
// this equals fmaf(float(q), float(x), s)).
__device__ __forceinline__ void fma_h2(float& s, uint32_t q2, uint32_t x2) {
  asm("{\n .reg .f16 ql, qh, xl, xh;\n mov.b32 {ql, qh}, %1;\n mov.b32 {xl, xh}, %2;\n"
      " fma.rn.f32.f16 %0, ql, xl, %0;\n fma.rn.f32.f16 %0, qh, xh, %0;\n}"
      : "+f"(s) : "r"(q2), "r"(x2));
}

/// sum_i q_i * x_i over one block; xv = the block's 32 x values (4 x uint4).
template <int QT>
__device__ __forceinline__ float block_dot(const uint4 (&p)[2], const uint4 (&xv)[4]) {
  const uint32_t* xw = reinterpret_cast<const uint32_t*>(&xv[0]);
  const uint32_t* w = reinterpret_cast<const uint32_t*>(&p[0]);
  float s = 0.0f;
  if constexpr (QT == 8) {
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const uint32_t u = w[k] ^ 0x80808080u;
      const uint32_t q01 = h2_sub(__byte_perm(u, 0x64646464u, 0x4140), 0x64806480u);
      const uint32_t q23 = h2_sub(__byte_perm(u, 0x64646464u, 0x4342), 0x64806480u);
      fma_h2(s, q01, xw[2 * k]);
      fma_h2(s, q23, xw[2 * k + 1]);
    }
  } else {
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const uint32_t v0 = w[m];
      const uint32_t v1 = w[m] >> 8;
      const uint32_t a = h2_sub((v0 & 0x000f000fu) | 0x64006400u, 0x64086408u);
      const uint32_t b = h2_fma((v0 & 0x00f000f0u) | 0x64006400u, 0x2c002c00u, 0xd480d480u);
      const uint32_t c = h2_sub((v1 & 0x000f000fu) | 0x64006400u, 0x64086408u);
      const uint32_t e = h2_fma((v1 & 0x00f000f0u) | 0x64006400u, 0x2c002c00u, 0xd480d480u);
      const uint32_t x01 = xw[2 * m], x23 = xw[2 * m + 1];
      const uint32_t y01 = xw[8 + 2 * m], y23 = xw[9 + 2 * m];
      asm("{\n .reg .f16 al, ah, bl, bh, cl, chh, el, eh, x0, x1, x2, x3, y0, y1, y2, y3;\n"
          " mov.b32 {al, ah}, %1;\n mov.b32 {bl, bh}, %2;\n mov.b32 {cl, chh}, %3;\n"
          " mov.b32 {el, eh}, %4;\n mov.b32 {x0, x1}, %5;\n mov.b32 {x2, x3}, %6;\n"
          " mov.b32 {y0, y1}, %7;\n mov.b32 {y2, y3}, %8;\n"
          " fma.rn.f32.f16 %0, al, x0, %0;\n fma.rn.f32.f16 %0, bl, y0, %0;\n"
          " fma.rn.f32.f16 %0, cl, x1, %0;\n fma.rn.f32.f16 %0, el, y1, %0;\n"
          " fma.rn.f32.f16 %0, ah, x2, %0;\n fma.rn.f32.f16 %0, bh, y2, %0;\n"
          " fma.rn.f32.f16 %0, chh, x3, %0;\n fma.rn.f32.f16 %0, eh, y3, %0;\n}"
          : "+f"(s)
          : "r"(a), "r"(b), "r"(c), "r"(e), "r"(x01), "r"(x23), "r"(y01), "r"(y23));
    }
  }
  return s;
}

template <int QT, int RPW, int SK, bool RESID>
__global__ void __launch_bounds__(kQWarps * 32, 2) gemv_q_kernel(
    const uint8_t* __restrict__ q, const __half* __restrict__ d, const __half* __restrict__ x,
    const __half* __restrict__ R, __half* __restrict__ y, int64_t N, int64_t K) {
  constexpr int GROUPS = kQWarps / SK;
  constexpr int PAY = QT == 8 ? 32 : 16;  // payload bytes per block
  __shared__ float red[kQWarps][RPW];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int grp = warp / SK;
  const int sub = warp % SK;
  const int64_t nblk = K / 32;
  const int64_t row0 = (static_cast<int64_t>(blockIdx.x) * GROUPS + grp) * RPW;
  const uint8_t* prow[RPW];
  const __half* drow[RPW];
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    const int64_t n = (row0 + r < N) ? row0 + r : N - 1;  // clamped rows: not stored
    prow[r] = q + n * nblk * PAY;
    drow[r] = d + n * nblk;
  }
  const int64_t b0 = static_cast<int64_t>(sub) * 32 + lane;
  constexpr int64_t kStride = 32 * SK;
  pdl_trigger();
  if (row0 < N && b0 < nblk) {  // warm L2 with this lane's first payload block
#pragma unroll
    for (int r = 0; r < RPW; ++r) prefetch_l2(prow[r] + b0 * PAY);
  }
  pdl_wait();

  float acc[RPW];
#pragma unroll
  for (int r = 0; r < RPW; ++r) acc[r] = 0.0f;
  // Software pipeline: U blocks per lane per buffer, two buffers -- the next U
  // blocks' payload and scales are in flight while the current U are multiplied
  // (U x RPW x 16 bytes per buffer: 128 payload bytes per lane in flight with
  // four rows a warp).  Each x chunk loaded from L1 feeds all RPW rows.
  constexpr int U = QT == 8 ? 1 : 2;
  constexpr int NP = QT == 8 ? 2 : 1;  // 16-byte payload words per block
  uint4 pa[U][RPW][NP], pb[U][RPW][NP];
  float sa[U][RPW], sb[U][RPW];
  auto load = [&](int64_t bb, uint4 (&p)[U][RPW][NP], float (&sc)[U][RPW]) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t b = bb + kStride * u;
      if (b < nblk) {
#pragma unroll
        for (int r = 0; r < RPW; ++r) {
#pragma unroll
          for (int w = 0; w < NP; ++w) p[u][r][w] = ld_stream_v4(prow[r] + b * PAY + 16 * w);
          sc[u][r] = __half2float(drow[r][b]);
        }
      }
    }
  };
  auto compute = [&](int64_t bb, uint4 (&p)[U][RPW][NP], float (&sc)[U][RPW]) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t b = bb + kStride * u;
      if (b < nblk) {
        uint4 xv[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) xv[c] = __ldg(reinterpret_cast<const uint4*>(x + 32 * b) + c);
#pragma unroll
        for (int r = 0; r < RPW; ++r) {
          uint4 pp[2];
          pp[0] = p[u][r][0];
          pp[1] = p[u][r][NP - 1];
          acc[r] = fmaf(sc[u][r], block_dot<QT>(pp, xv), acc[r]);
        }
      }
    }
  };
  if (row0 < N) {
    int64_t b = b0;
    load(b, pa, sa);
    for (; b < nblk; b += 2 * kStride * U) {
      load(b + kStride * U, pb, sb);
      compute(b, pa, sa);
      load(b + 2 * kStride * U, pa, sa);
      compute(b + kStride * U, pb, sb);
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
  for (int o = threadIdx.x; o < GROUPS * RPW; o += blockDim.x) {
    const int g = o / RPW;
    const int r = o % RPW;
    const int64_t row = (static_cast<int64_t>(blockIdx.x) * GROUPS + g) * RPW + r;
    if (row >= N) continue;
    float v = 0.0f;
#pragma unroll
    for (int s = 0; s < SK; ++s) v += red[g * SK + s][r];
    if constexpr (RESID) v += __half2float(R[row]);
    y[row] = __float2half_rn(v);
  }
}

template <int QT, bool RESID, int SK>
int launch_q_split(const uint8_t* q, const __half* d, const __half* x, const __half* R,
                    __half* y, int64_t N, int64_t K, cudaStream_t stream) {
  constexpr int RPW = 4;
  constexpr int64_t rows_per_cta = (kQWarps / SK) * RPW;
  const unsigned grid = static_cast<unsigned>((N + rows_per_cta - 1) / rows_per_cta);
  B200_CUDA(launch_pdl(gemv_q_kernel<QT, RPW, SK, RESID>, dim3(grid), dim3(kQWarps * 32), 0,
                       stream, q, d, x, R, y, N, K));
  return ENGINE_OK;
}

template <int QT, bool RESID>
int launch_gemv_q(const uint8_t* q, const __half* d, const __half* x, const __half* R, __half* y,
                  int64_t N, int64_t K, cudaStream_t stream) {
  // Four rows per warp group (measured on B200 against two: 14336x4096 Q8_0
  // 19.6 -> 15.5 us, Q4_0 17.8 -> 14.3 us; 4096x4096 7.1 -> 5.7 / 6.5 -> 4.9 us;
  // 4096x14336 unchanged).  K is split over two warps up to 1024 blocks a row
  // (32768 weights), so that 4096 rows still give enough warps.
  if (K / 32 <= 1024) return launch_q_split<QT, RESID, 2>(q, d, x, R, y, N, K, stream);
  return launch_q_split<QT, RESID, 1>(q, d, x, R, y, N, K, stream);
}

}  // namespace
}  // namespace b200

using namespace b200;

extern "C" {

int engine_cuda_quant_repack(int qtype, const void* blocks, void* q_out,
                             engine_half_t* scales_out, int64_t N, int64_t K,
                             engine_stream_t stream) {
  B200_ENTRY_BEGIN
  B200_REQUIRE(qtype == ENGINE_Q8_0 || qtype == ENGINE_Q4_0,
               "quant_repack: qtype must be ENGINE_Q8_0 or ENGINE_Q4_0");
  B200_REQUIRE(N >= 0 && K >= 0, "quant_repack: negative dimension");
  B200_REQUIRE(K % 32 == 0, "quant_repack: K must be a multiple of the 32-element block");
  B200_REQUIRE(blocks != nullptr && q_out != nullptr && scales_out != nullptr,
               "quant_repack: null device pointer");
  if (N == 0 || K == 0) return ENGINE_OK;
  const int64_t nblk = K / 32;
  const int64_t total = N * nblk;
  const int64_t g64 = (total + 255) / 256;
  const unsigned grid = static_cast<unsigned>(g64 < 65535 * 8 ? g64 : 65535 * 8);
  const auto* in = static_cast<const uint8_t*>(blocks);
  auto* q = static_cast<uint8_t*>(q_out);
  auto* d = reinterpret_cast<__half*>(scales_out);
  auto st = static_cast<cudaStream_t>(stream);
  if (qtype == ENGINE_Q8_0) {
    B200_CUDA(launch_pdl(quant_repack_kernel<8>, dim3(grid), dim3(256), 0, st, in, q, d, N, nblk));
  } else {
    B200_CUDA(launch_pdl(quant_repack_kernel<4>, dim3(grid), dim3(256), 0, st, in, q, d, N, nblk));
  }
  return check_launch("quant_repack");
  B200_ENTRY_END
}

int engine_cuda_gemv_q_nk(int qtype, const void* q, const engine_half_t* scales,
                          const engine_half_t* x, const engine_half_t* residual, engine_half_t* y,
                          int64_t N, int64_t K, engine_stream_t stream) {
  B200_ENTRY_BEGIN
  B200_REQUIRE(qtype == ENGINE_Q8_0 || qtype == ENGINE_Q4_0,
               "gemv_q_nk: qtype must be ENGINE_Q8_0 or ENGINE_Q4_0");
  B200_REQUIRE(N >= 0 && K >= 0, "gemv_q_nk: dimensions must be non-negative");
  B200_REQUIRE(K % 32 == 0, "gemv_q_nk: K must be a multiple of the 32-element block");
  B200_REQUIRE(q != nullptr && scales != nullptr && x != nullptr && y != nullptr,
               "gemv_q_nk: null device pointer");
  if (N == 0) return ENGINE_OK;
  auto st = static_cast<cudaStream_t>(stream);
  if (K == 0) {  // empty rows: y = residual, or zeros
    if (residual != nullptr) {
      B200_CUDA(cudaMemcpyAsync(y, residual, static_cast<size_t>(N) * 2, cudaMemcpyDeviceToDevice, st));
    } else {
      B200_CUDA(cudaMemsetAsync(y, 0, static_cast<size_t>(N) * 2, st));
    }
    return ENGINE_OK;
  }
  B200_REQUIRE(reinterpret_cast<uintptr_t>(q) % 16 == 0 && reinterpret_cast<uintptr_t>(x) % 16 == 0,
               "gemv_q_nk: payload and x must be 16-byte aligned");
  const auto* qq = static_cast<const uint8_t*>(q);
  const auto* d = reinterpret_cast<const __half*>(scales);
  const auto* xx = reinterpret_cast<const __half*>(x);
  const auto* r = reinterpret_cast<const __half*>(residual);
  auto* yy = reinterpret_cast<__half*>(y);
  int rc;
  if (qtype == ENGINE_Q8_0) {
    rc = r ? launch_gemv_q<8, true>(qq, d, xx, r, yy, N, K, st)
           : launch_gemv_q<8, false>(qq, d, xx, r, yy, N, K, st);
  } else {
    rc = r ? launch_gemv_q<4, true>(qq, d, xx, r, yy, N, K, st)
           : launch_gemv_q<4, false>(qq, d, xx, r, yy, N, K, st);
  }
  if (rc != ENGINE_OK) return rc;
  return check_launch("gemv_q_nk");
  B200_ENTRY_END
}

}  // extern "C"
