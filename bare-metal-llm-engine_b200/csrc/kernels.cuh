// kernels.cuh -- internal launchers shared between the library's translation units.
// All take raw device pointers, validated arguments and a stream; each returns
// ENGINE_OK or an ENGINE_ERR_* code with the message recorded (common.cuh).
#pragma once

#include "common.cuh"

namespace b200 {

/// C[M,N] = A[M,K] * B[K,N] FP32 on CUDA cores; with norm=true, A rows are
/// RMS-normalised (rms_w may be null) on the way in.  gemm_simt.cu.
int sgemm(const float* A, const float* B, float* C, int64_t M, int64_t N, int64_t K,
          const float* rms_w, float eps, bool norm, cudaStream_t stream);

/// out[N] = x[K] * A[K,N] (legacy [K,N] layout), FP32; with norm=true x is
/// RMS-normalised first.  gemv.cu.
int gemv_kn_f32(const float* A, const float* x, float* out, int64_t N, int64_t K,
                const float* rms_w, float eps, bool norm, cudaStream_t stream);

/// out[N] = x[K] * A[K,N] (legacy [K,N] layout), FP16 in/out, FP32 accumulate.  gemv.cu.
int gemv_kn_f16(const __half* A, const __half* x, __half* out, int64_t N, int64_t K,
                cudaStream_t stream);

/// y[r, n] = sum_k X[r, k] W[n, k] for r < M <= 8 rows of X (W is [N,K]), FP32
/// accumulate, optional RMSNorm of X (gamma may be null) and residual.  gemv.cu.
int gemv_nk_f16(const __half* W, const __half* X, const __half* gamma, float eps, bool norm,
                const __half* residual, __half* Y, int64_t M, int64_t N, int64_t K,
                cudaStream_t stream);

/// Row RMSNorm FP16 -> FP16 (gamma may be null): normalised activations for the
/// tensor-core GEMM path of rmsnorm_linear_f16.  gemv.cu.
int rmsnorm_f16(const __half* x, const __half* gamma, __half* out, int64_t rows, int64_t cols,
                float eps, cudaStream_t stream);

/// Tensor-core GEMM (tcgen05): C[M,N] = A[M,K] * op(B) where op(B) is B[K,N]
/// (b_kmajor=false) or W[N,K]^T (b_kmajor=true); FP16/BF16 in and out, FP32
/// accumulate, optional residual added in FP32 before rounding.  gemm_tc.cu.
int gemm_tc(const void* A, const void* B, const void* residual, void* C, int64_t M, int64_t N,
            int64_t K, bool bf16, bool b_kmajor, cudaStream_t stream);

/// As gemm_tc; with hilo=true, A holds 2*half_b activation rows (the FP16
/// roundings of an FP32 activation, then the FP16 roundings of the remainders),
/// B is W[N,K], and the first M rows of C receive the product.  gemm_tc.cu.
int gemm_tc_general(const void* A, const void* B, const void* residual, void* C, int64_t M,
                    int64_t N, int64_t K, bool bf16, bool b_kmajor, bool hilo, int half_b,
                    cudaStream_t stream);

/// Writes the hi/lo normalised activations of x[M,K] into out[2*hb, K] (rows
/// [0,M) = FP16 roundings of (x*scale)*gamma, rows [hb, hb+M) = roundings of the
/// remainders, all other rows zero).  linear.cu.
int rmsnorm_hilo(const __half* x, const __half* gamma, __half* out, int64_t M, int64_t K, int hb,
                 float eps, cudaStream_t stream);

/// Stream-ordered scratch from the library's own per-device memory pool
/// (cudaMallocFromPoolAsync; memory stays cached in the pool between calls).
/// Returns nullptr with the error recorded on failure.  abi.cu.
void* scratch_alloc(size_t bytes, cudaStream_t stream);
void scratch_free(void* p, cudaStream_t stream);

/// Batch-1 RMSNorm -> gate/up projection with the SwiGLU in its epilogue:
/// Y[F] = swiglu(rmsnorm(x) W[0:F]^T, rmsnorm(x) W[F:2F]^T).  Returns
/// ENGINE_ERR_UNSUPPORTED (nothing launched) when the shape / alignment does not
/// fit the fused kernel.  gemv.cu.
int gemv_nk_norm1_swiglu_f16(const __half* W, const __half* X, const __half* gamma, float eps,
                             __half* Y, int64_t F, int64_t K, cudaStream_t stream);

/// Attention prefill on tcgen05 (attention_tc.cu): the attention_prefill
/// contract for head_dim 64 / 128.  Returns ENGINE_ERR_UNSUPPORTED, with nothing
/// launched, when a stride or pointer alignment does not allow its TMA maps.
int attention_prefill_tc(const __half* q, const __half* k, const __half* v, __half* out,
                         int64_t s_q, int64_t s_kv, int64_t n_heads, int64_t n_kv_heads, int64_t d,
                         int64_t kv_head_stride, float scale, int64_t q_pos_offset, bool causal,
                         float* lse, cudaStream_t stream);

/// Attention decode on tcgen05 (attention_tc.cu): one query position, d = 128,
/// up to 16 query heads per KV head.  The keys of each KV head are split, in
/// whole 128-key blocks, so that all heads together give about two CTAs per SM:
/// one split writes the output directly, up to 8 merge inside a thread-block
/// cluster through distributed shared memory, more write (m, l, O) to
/// ws[n_heads][splits][d + 2], which the caller merges with attn_merge_kernel.  attention_decode_tc_splits returns that split count (0:
/// no workspace) and the keys per split.  Returns ENGINE_ERR_UNSUPPORTED, with
/// nothing launched, for shapes or alignments it does not take.
int attention_decode_tc_splits(int64_t s_kv, int64_t n_kv_heads, int64_t* chunk);
int attention_decode_tc(const __half* q, const __half* k, const __half* v, __half* out, float* lse,
                        float* ws, int64_t s_kv, int64_t n_heads, int64_t n_kv_heads, int64_t d,
                        int64_t kv_head_stride, float scale, cudaStream_t stream);

/// Zeroes the stream-K tile counters of every workspace on `dev` (after a
/// device-side time-out may have left a launch half counted).  The device must
/// be idle.  gemm_tc.cu.
void sk_workspace_reset(int dev);

}  // namespace b200
