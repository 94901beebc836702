/*
 * engine_b200.h -- C ABI of the B200 (sm_100a) matrix-multiply hot path.
 *
 * Drop-in boundary for the launch API of Parag63/bare-metal-llm-engine
 * (include/engine/kernels.hpp, namespace engine::cuda).  Each engine_cuda_<name>
 * symbol below replaces the engine::cuda::<name> launcher cited beside it, with
 * the same argument order and meaning: raw DEVICE pointers, int64 dimensions, all
 * 2-D data row-major and contiguous, and the CUDA stream last (0 = legacy default
 * stream).  include/engine/kernels_b200.hpp wraps these symbols back into the
 * engine's C++ signatures and rethrows failures as engine::EngineError.
 *
 * Error convention (the reference's ENGINE_CHECK / CUDA_CHECK, check.hpp:36-107,
 * expressed without C++ exceptions): every entry point returns ENGINE_OK (0) or a
 * nonzero ENGINE_ERR_* code, and engine_last_error() returns the calling thread's
 * message for its most recent failure.  Messages keep the reference's wording so
 * substring checks carry over: "... must be non-negative" / "negative dimension",
 * "... is null" / "null device pointer", "eps must be non-negative".
 *
 * Empty work follows the reference launchers: M == 0 or N == 0 returns ENGINE_OK
 * without launching; K == 0 writes the zero matrix / vector (the empty sum)
 * asynchronously on `stream` (matmul_register_tiled.cu:184-191, gemv_fp16.cu:124-131),
 * except rmsnorm_linear, which like the reference returns without writing when any
 * of M, N, K is zero (rmsnorm_linear.cu:180).
 *
 * All calls are asynchronous and stream-ordered and safe to call from several
 * host threads on different streams.  Split-K partial sums are reduced through
 * distributed shared memory inside a thread-block cluster, so the GEMV paths and
 * the small-batch projections need no scratch.  Device memory the library
 * allocates itself:
 *   - from a library-owned stream-ordered memory pool (cached between calls):
 *     engine_cuda_rmsnorm_linear_f16 with M > 4 (normalised activation rows),
 *     engine_cuda_rmsnorm_linear_swiglu_f16 with M > 1 (the gate/up rows) and
 *     engine_cuda_attention_decode / _prefill with split partials to merge (the
 *     tcgen05 decode with more than 8 splits per KV head, or the CUDA-core
 *     kernels with more than one; up to 8 tcgen05 splits merge inside a
 *     thread-block cluster and need none);
 *   - once per (device, stream), on the first call that needs it, never during
 *     a stream capture: the stream-K workspace of the large 16-bit GEMMs
 *     (engine_cuda_matmul_* / linear_* with M, N >= 256; about 38 MB);
 *   - at engine_tp_comm_create: the communicator's exchange region.
 * engine_cuda_rmsnorm_linear_f16_noalloc is the variant of the fused norm
 * projection that allocates nothing.
 *
 * FP16 / BF16 data crosses the ABI as 16-bit IEEE binary16 / bfloat16 bit
 * patterns (engine::half is __half: the same 2-byte layout, half.hpp:28).
 */
#ifndef ENGINE_B200_H_
#define ENGINE_B200_H_

#include <stdint.h>

#if defined(__GNUC__)
#define ENGINE_B200_API __attribute__((visibility("default")))
#else
#define ENGINE_B200_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* engine_stream_t; /* identical to cudaStream_t */
typedef uint16_t engine_half_t;              /* IEEE binary16 bits (engine::half) */
typedef uint16_t engine_bf16_t;              /* bfloat16 bits */

enum {
  ENGINE_OK = 0,
  ENGINE_ERR_INVALID = 1,     /* bad argument: negative dim, null pointer, eps < 0 */
  ENGINE_ERR_CUDA = 2,        /* a CUDA runtime call or launch failed */
  ENGINE_ERR_UNSUPPORTED = 3, /* shape / alignment outside what the kernels support */
  ENGINE_ERR_DEVICE = 4,      /* a kernel reported a device-side error (wait timeout) */
  ENGINE_ERR_INTERNAL = 5,
  ENGINE_ERR_FORMAT = 6,      /* a model file is malformed or truncated */
  ENGINE_ERR_IO = 7           /* a model file could not be opened or mapped */
};

/* Version of this ABI (bumped on any signature change). */
ENGINE_B200_API int engine_abi_version(void);

/* Message of the calling thread's most recent failed call ("" if none). */
ENGINE_B200_API const char* engine_last_error(void);

/* Reads and clears the device-side error word of `device` (bits: 1 = a bounded
 * wait inside a kernel ran out, 2 = a kernel's own bounds check fired).  Kernels
 * set it instead of hanging; the call synchronises the device first. */
ENGINE_B200_API int engine_device_status(int device, unsigned int* flags);

/* ---------------------------------------------------------------------------
 * Legacy launch API (FP32 and FP16 [K,N] layouts), kept behaviour-compatible.
 * ------------------------------------------------------------------------- */

/* C[M,N] = A[M,K] * B[K,N], FP32.  kernels.hpp:67 (matmul_naive). */
ENGINE_B200_API int engine_cuda_matmul_naive(const float* A, const float* B, float* C, int64_t M, int64_t N,
                             int64_t K, engine_stream_t stream);
/* kernels.hpp:74 (matmul_tiled). */
ENGINE_B200_API int engine_cuda_matmul_tiled(const float* A, const float* B, float* C, int64_t M, int64_t N,
                             int64_t K, engine_stream_t stream);
/* kernels.hpp:80 (matmul_register_tiled). */
ENGINE_B200_API int engine_cuda_matmul_register_tiled(const float* A, const float* B, float* C, int64_t M,
                                      int64_t N, int64_t K, engine_stream_t stream);

/* out[N] = x[K] * A[K,N], FP32.  kernels.hpp:85 (gemv). */
ENGINE_B200_API int engine_cuda_gemv(const float* A, const float* x, float* out, int64_t N, int64_t K,
                     engine_stream_t stream);

/* out[N] = x[K] * A[K,N], FP16 in/out, FP32 accumulate.  kernels.hpp:120 (gemv_fp16). */
ENGINE_B200_API int engine_cuda_gemv_fp16(const engine_half_t* A, const engine_half_t* x, engine_half_t* out,
                          int64_t N, int64_t K, engine_stream_t stream);

/* Row RMSNorm, eps inside the square root; weight may be null.  kernels.hpp:62 (rmsnorm). */
ENGINE_B200_API int engine_cuda_rmsnorm(const float* in, const float* weight, float* out, int64_t rows,
                        int64_t cols, float eps, engine_stream_t stream);

/* Fused residual add + RMSNorm: sum_out = x + residual, norm_out =
 * rmsnorm(sum_out) * weight (weight may be null; x, residual, norm_out and
 * sum_out may not).  kernels.hpp:110 (residual_rmsnorm), launcher
 * kernels/residual_rmsnorm.cu:124-147. */
ENGINE_B200_API int engine_cuda_residual_rmsnorm(const float* x, const float* residual,
                                                 const float* weight, float* norm_out,
                                                 float* sum_out, int64_t rows, int64_t cols,
                                                 float eps, engine_stream_t stream);

/* out[M,N] = rmsnorm(in[M,K], rms_weight, eps) * W[K,N]; rms_weight may be null.
 * kernels.hpp:97 (rmsnorm_linear).  One fused launch for every M. */
ENGINE_B200_API int engine_cuda_rmsnorm_linear(const float* in, const float* rms_weight, const float* W,
                               float* out, int64_t M, int64_t N, int64_t K, float eps,
                               engine_stream_t stream);
/* kernels.hpp:102 (rmsnorm_linear_fused_direct): same fused kernel. */
ENGINE_B200_API int engine_cuda_rmsnorm_linear_fused_direct(const float* in, const float* rms_weight,
                                            const float* W, float* out, int64_t M, int64_t N,
                                            int64_t K, float eps, engine_stream_t stream);

/* out[i] = a[i] + b[i].  kernels.hpp:49 (vector_add): the residual add that the new
 * entry points fold into their epilogues. */
ENGINE_B200_API int engine_cuda_vector_add(const float* a, const float* b, float* out, int64_t n,
                           engine_stream_t stream);

/* ---------------------------------------------------------------------------
 * New entry points for the B200 configurations (tcgen05 / HBM-streaming).
 * No reference counterpart exists for these layouts; each is the FP16/BF16,
 * [N,K]-weight form of the legacy call named beside it.
 * ------------------------------------------------------------------------- */

/* C[M,N] = A[M,K] * B[K,N] (all row-major), FP16 in/out, FP32 accumulate, on
 * tcgen05 tensor cores.  FP16 form of kernels.hpp:80 (matmul_register_tiled). */
ENGINE_B200_API int engine_cuda_matmul_f16(const engine_half_t* A, const engine_half_t* B, engine_half_t* C,
                           int64_t M, int64_t N, int64_t K, engine_stream_t stream);
/* BF16 form of the above. */
ENGINE_B200_API int engine_cuda_matmul_bf16(const engine_bf16_t* A, const engine_bf16_t* B, engine_bf16_t* C,
                            int64_t M, int64_t N, int64_t K, engine_stream_t stream);

/* Y[M,N] = X[M,K] * W[N,K]^T (+ residual[M,N] if non-null), FP16, FP32 accumulate:
 * the activation x weight projection with weights stored [N,K] (K contiguous).
 * M == 1 streams W through the decode GEMV; small M uses a swap-AB tcgen05 tile;
 * larger M the persistent tcgen05 GEMM.  Residual form of matmul_register_tiled +
 * vector_add (tests/test_kernels.cu:2805-2810). */
ENGINE_B200_API int engine_cuda_linear_f16(const engine_half_t* X, const engine_half_t* W,
                           const engine_half_t* residual, engine_half_t* Y, int64_t M,
                           int64_t N, int64_t K, engine_stream_t stream);
/* BF16 form of the above. */
ENGINE_B200_API int engine_cuda_linear_bf16(const engine_bf16_t* X, const engine_bf16_t* W,
                            const engine_bf16_t* residual, engine_bf16_t* Y, int64_t M,
                            int64_t N, int64_t K, engine_stream_t stream);

/* y[N] = W[N,K] * x[K] (+ residual[N]), FP16, FP32 accumulate: the batch-1 decode
 * GEMV over [N,K] weights.  [N,K] form of kernels.hpp:120 (gemv_fp16). */
ENGINE_B200_API int engine_cuda_gemv_f16_nk(const engine_half_t* W, const engine_half_t* x,
                            const engine_half_t* residual, engine_half_t* y, int64_t N,
                            int64_t K, engine_stream_t stream);

/* Y[M,N] = rmsnorm(x[M,K], gamma, eps) * W[N,K]^T (+ residual), FP16 in/out, FP32
 * accumulate, eps inside the square root, gamma may be null.  FP16 [N,K] form of
 * kernels.hpp:97 (rmsnorm_linear). */
ENGINE_B200_API int engine_cuda_rmsnorm_linear_f16(const engine_half_t* x, const engine_half_t* gamma,
                                   const engine_half_t* W, const engine_half_t* residual,
                                   engine_half_t* Y, int64_t M, int64_t N, int64_t K,
                                   float eps, engine_stream_t stream);

/* rmsnorm_linear_f16 for callers that cannot allocate device memory.  No
 * counterpart in the reference.  Same arguments as
 * engine_cuda_rmsnorm_linear_f16, but the normalised activations live in a
 * fixed 2 MiB array inside the library instead of a stream-ordered pool, so the
 * call allocates nothing: for serving loops that reserve all device memory at
 * start-up and may not allocate per request, and for hosts whose device memory
 * is owned by another allocator.  It always takes the tensor-core path with
 * hi/lo activations formed by a pre-pass into that array.  For 5 <= M <= 32
 * engine_cuda_rmsnorm_linear_f16 runs the same pre-pass (into pool memory) and
 * the same GEMM, so the results are identical; for M <= 4 it streams W on CUDA
 * cores instead, and the two agree within rounding (both inside the FP32
 * bound).
 * Limits: 1 <= M <= 32, K <= 16384, K a multiple of 8, W 16-byte aligned;
 * larger sizes return ENGINE_ERR_UNSUPPORTED.  Make one warm-up call per device
 * at start-up: it looks up the array's device address, and with lazy module
 * loading it is also the call that loads the library's device code, which is
 * when the 2 MiB array is reserved.  Make it before any stream capture.  All
 * calls share the one array: calls that overlap on the GPU race. */
ENGINE_B200_API int engine_cuda_rmsnorm_linear_f16_noalloc(
    const engine_half_t* x, const engine_half_t* gamma, const engine_half_t* W,
    const engine_half_t* residual, engine_half_t* Y, int64_t M, int64_t N, int64_t K, float eps,
    engine_stream_t stream);

/* Fused RMSNorm -> gate/up projection -> SwiGLU.  No single reference
 * counterpart: it is kernels.hpp:97 (rmsnorm_linear, FP16 [N,K] form) followed by
 * kernels.hpp:141 (swiglu_fp16), in one call.  W_gu[2F,K] holds the gate rows
 * [0, F) then the up rows [F, 2F) (the tensor-parallel shard layout);
 * Y[M,F] = swiglu(g, u) with g, u the FP16 projections -- bit-identical to
 * engine_cuda_rmsnorm_linear_f16 into [M,2F] followed by engine_cuda_swiglu_f16.
 * Batch 1 is one kernel that never writes g and u; larger batches use a
 * stream-ordered scratch for them. */
ENGINE_B200_API int engine_cuda_rmsnorm_linear_swiglu_f16(const engine_half_t* x,
                                                          const engine_half_t* gamma,
                                                          const engine_half_t* W_gu,
                                                          engine_half_t* Y, int64_t M, int64_t F,
                                                          int64_t K, float eps,
                                                          engine_stream_t stream);

/* out[i] = silu(gate[i]) * up[i], FP16: glue between the gate/up and down
 * projections of the tensor-parallel layer.  kernels.hpp:141 (swiglu_fp16). */
ENGINE_B200_API int engine_cuda_swiglu_f16(const engine_half_t* gate, const engine_half_t* up,
                           engine_half_t* out, int64_t n, engine_stream_t stream);

/* out[t, :] = table[ids[t], :], FP16 rows: token-embedding glue of the layer set.
 * kernels.hpp:128 (embedding_fp16); ids outside [0, vocab) are rejected on device
 * by writing zeros and setting error bit 2. */
ENGINE_B200_API int engine_cuda_embedding_f16(const engine_half_t* table, const int32_t* ids,
                              engine_half_t* out, int64_t num_tokens, int64_t hidden,
                              int64_t vocab, engine_stream_t stream);

/* ---------------------------------------------------------------------------
 * Block-quantised decode GEMV.  The reference declares the formats but has no
 * kernel for them (include/engine/dtype.hpp:95-125: GGUF's 32-element blocks
 * with one FP16 scale):
 *   ENGINE_Q8_0  { half d; int8 q[32]; }     34 bytes/block, w = d * q
 *   ENGINE_Q4_0  { half d; uint8 nib[16]; }  18 bytes/block, w[j] = d * (lo(nib[j]) - 8),
 *                                            w[j+16] = d * (hi(nib[j]) - 8)
 * ------------------------------------------------------------------------- */
#define ENGINE_Q8_0 8
#define ENGINE_Q4_0 4

/* Converts W[N,K] stored as packed GGUF blocks (row-major, K/32 blocks per row)
 * into the layout engine_cuda_gemv_q_nk streams: q_out [N][K] int8 (Q8_0) or
 * [N][K/2] bytes (Q4_0, each block's 16 bytes in GGUF order), and scales_out
 * [N][K/32] FP16.  Run once when the weights are loaded.  K % 32 == 0. */
ENGINE_B200_API int engine_cuda_quant_repack(int qtype, const void* blocks, void* q_out,
                                             engine_half_t* scales_out, int64_t N, int64_t K,
                                             engine_stream_t stream);

/* y[N] = W x (+ residual) for W in the repacked block-quantised layout; FP16 x,
 * y; FP32 accumulation.  The quantised form of gemv_f16_nk (kernels.hpp:120).
 * q and x 16-byte aligned; K % 32 == 0. */
ENGINE_B200_API int engine_cuda_gemv_q_nk(int qtype, const void* q, const engine_half_t* scales,
                                          const engine_half_t* x, const engine_half_t* residual,
                                          engine_half_t* y, int64_t N, int64_t K,
                                          engine_stream_t stream);

/* ---------------------------------------------------------------------------
 * Tensor-parallel communicator over NVLink peer memory.  No counterpart in the
 * reference (it has no multi-GPU code): these replace the NCCL all-reduce (sum,
 * FP16) that follows the row-split O and down projections of the
 * tensor-parallel layer set, and fuse it into the projection for decode.
 *
 * One process per GPU.  Set-up, with the rank's device current:
 *   1. engine_tp_comm_create(rank, world, max_elems, &c)
 *   2. engine_tp_comm_handle(c, h)     -- ENGINE_TP_HANDLE_BYTES bytes; exchange
 *      them between the ranks on the host (all-gather)
 *   3. engine_tp_comm_open(c, all)     -- world x ENGINE_TP_HANDLE_BYTES, rank order
 *   ... calls ...
 *   4. a host barrier across the ranks, then engine_tp_comm_destroy(c).
 * Every rank must make the same sequence of calls, all stream-ordered on one
 * stream per rank.  Each call waits for the peers on the device with a bounded
 * wait (ENGINE_WAIT_TIMEOUT_MS); on expiry the kernel sets bit 1 of the device
 * error word (engine_device_status) and leaves Y unwritten.  Results are
 * bit-identical on every rank: the sum runs in FP32 in rank order, then the
 * residual is added and the value is rounded once to FP16.  Calls may be
 * captured in CUDA graphs; the per-call state lives in device memory.
 * ------------------------------------------------------------------------- */
#define ENGINE_TP_HANDLE_BYTES 64

typedef struct engine_tp_comm engine_tp_comm_t;

/* Allocates this rank's exchange region on the current device:
 * 2 x world x max_elems FP32 slots, flags, call counts.  max_elems bounds the
 * elements (M*N) of one call.  world <= 8. */
ENGINE_B200_API int engine_tp_comm_create(int rank, int world, int64_t max_elems,
                                          engine_tp_comm_t** comm);

/* Copies the region's CUDA IPC handle (ENGINE_TP_HANDLE_BYTES bytes) to `handle`. */
ENGINE_B200_API int engine_tp_comm_handle(const engine_tp_comm_t* comm, void* handle);

/* Maps every peer's region.  `handles` holds world handles in rank order.  A
 * handle equal to this rank's own maps to its own region (single-process
 * loopback). */
ENGINE_B200_API int engine_tp_comm_open(engine_tp_comm_t* comm, const void* handles);

/* Unmaps the peers and frees the region.  Call after a host barrier. */
ENGINE_B200_API int engine_tp_comm_destroy(engine_tp_comm_t* comm);

/* y[i] = sum over ranks of partial[i] (+ residual[i]), on every rank. */
ENGINE_B200_API int engine_tp_allreduce_f16(engine_tp_comm_t* comm, const engine_half_t* partial,
                                            const engine_half_t* residual, engine_half_t* y,
                                            int64_t n, engine_stream_t stream);

/* Row-split projection fused with its all-reduce:
 * Y[M,N] = sum over ranks r of X_r[M,K] * W_r[N,K]^T (+ residual[M,N]) on every rank.
 * For M <= 4 one kernel streams W_r as the decode GEMV does, pushes its FP32
 * partial rows to every rank over NVLink and reduces.  Larger M runs the
 * tensor-core projection, then the one-shot all-reduce. */
ENGINE_B200_API int engine_tp_linear_allreduce_f16(engine_tp_comm_t* comm, const engine_half_t* X,
                                                   const engine_half_t* W,
                                                   const engine_half_t* residual, engine_half_t* Y,
                                                   int64_t M, int64_t N, int64_t K,
                                                   engine_stream_t stream);

/* ---------------------------------------------------------------------------
 * Attention (MHA / GQA), the engine's launchers: q / out [s_q][n_heads][d],
 * k / v [n_kv_heads][kv_head_stride], d = 64 or 128; query row i sees keys
 * j <= q_pos_offset + i when causal.  Same contract and messages as
 * kernels/attention_prefill.cu:329-360 and kernels/attention_decode.cu:637-660.
 * ------------------------------------------------------------------------- */

/* kernels.hpp:153 (attention_prefill).  out_lse [s_q][n_heads] may be null. */
ENGINE_B200_API int engine_cuda_attention_prefill(const engine_half_t* q, const engine_half_t* k,
                                                  const engine_half_t* v, engine_half_t* out,
                                                  int64_t s_q, int64_t s_kv, int64_t n_heads,
                                                  int64_t n_kv_heads, int64_t head_dim,
                                                  int64_t kv_head_stride, float scale,
                                                  int64_t q_pos_offset, int is_causal,
                                                  float* out_lse, engine_stream_t stream);

/* kernels.hpp:191 (attention_decode): one query row per head over kv_len keys,
 * split-KV; split_kv = 0 chooses the split count. */
ENGINE_B200_API int engine_cuda_attention_decode(const engine_half_t* q, const engine_half_t* k,
                                                 const engine_half_t* v, engine_half_t* out,
                                                 int64_t kv_len, int64_t n_heads,
                                                 int64_t n_kv_heads, int64_t head_dim,
                                                 int64_t kv_head_stride, float scale, int split_kv,
                                                 engine_stream_t stream);

/* kernels.hpp:184 (detail::kv_cache_write): token-major K / V [s_new][n_kv_heads]
 * [head_dim] scattered into head-major caches [n_kv_heads][kv_max_seq_len]
 * [head_dim] from position pos_offset.  Same checks and messages as
 * kernels/attention_bridge.cu:89-103.  A copy: bit-exact. */
ENGINE_B200_API int engine_cuda_kv_cache_write(const engine_half_t* k_new, const engine_half_t* v_new,
                                               engine_half_t* k_cache, engine_half_t* v_cache,
                                               int64_t s_new, int64_t n_kv_heads, int64_t head_dim,
                                               int64_t pos_offset, int64_t kv_max_seq_len,
                                               engine_stream_t stream);

/* The same for n_seq sequences of s_new tokens read from strided rows: row
 * b * s_new + t starts at k_new + (b * s_new + t) * row_pitch (elements), so
 * the K and V parts of a fused Q/K/V projection's output go to the caches
 * without a copy.  Sequence b's caches are the heads [b * n_kv_heads, (b + 1) *
 * n_kv_heads) of k_cache / v_cache, so a batch of equal-length sequences is one
 * attention_decode call with n_seq * n_kv_heads KV heads.  No counterpart in the
 * reference (its kv_cache_write is the n_seq = 1, contiguous case above). */
ENGINE_B200_API int engine_cuda_kv_cache_write_rows(const engine_half_t* k_new,
                                                    const engine_half_t* v_new, int64_t row_pitch,
                                                    engine_half_t* k_cache, engine_half_t* v_cache,
                                                    int64_t n_seq, int64_t s_new,
                                                    int64_t n_kv_heads, int64_t head_dim,
                                                    int64_t pos_offset, int64_t kv_max_seq_len,
                                                    engine_stream_t stream);

/* Batch-1 decode: the fused Q/K/V projection of one token and its KV-cache
 * write as one kernel.  Y[N] = rmsnorm(x) W^T (+ residual), exactly as
 * engine_cuda_rmsnorm_linear_f16 with M = 1, and output rows [kv_row0,
 * kv_row0 + n_kv_heads * head_dim) (the token's K row) and the next
 * n_kv_heads * head_dim rows (its V row) are also stored at position pos of
 * head-major caches [n_kv_heads][max_len][head_dim] -- what
 * engine_cuda_kv_cache_write of those rows would store.  No counterpart in the
 * reference: it fuses rmsnorm_linear (kernels.hpp:97) with detail::kv_cache_write
 * (kernels.hpp:184) and saves the write's launch in every layer of a decode
 * step.  Needs K a positive multiple of 8 (at most 40960) and 16-byte aligned
 * W, x and gamma (gamma may be null: unit gains). */
ENGINE_B200_API int engine_cuda_rmsnorm_linear_kv_f16(
    const engine_half_t* x, const engine_half_t* gamma, const engine_half_t* W,
    const engine_half_t* residual, engine_half_t* Y, int64_t N, int64_t K, float eps,
    engine_half_t* k_cache, engine_half_t* v_cache, int64_t kv_row0, int64_t n_kv_heads,
    int64_t head_dim, int64_t max_len, int64_t pos, engine_stream_t stream);

/* ---------------------------------------------------------------------------
 * GGUF model files, memory-mapped, feeding the projections.  The engine plans a
 * GGUF-style mmap'd loader (README.md:247, Module 7; tensor.hpp:19-23: weight
 * tensors aliasing one mapped region) but has none; this is that loader's
 * read side, for the weights the projections above consume.
 *
 * A file is GGUF version 2 or 3: header, typed metadata, tensor table, then the
 * tensor data at general.alignment (default 32).  Every read is bounds-checked:
 * a malformed or truncated file returns ENGINE_ERR_FORMAT, never a fault.
 * Tensor dims are in the file's order: dims[0] is the contiguous extent (K of a
 * [N,K] weight), and block-quantised rows run along dims[0].
 * ------------------------------------------------------------------------- */
typedef struct engine_gguf engine_gguf_t;

/* GGML tensor type codes the loader can place on the device. */
#define ENGINE_GGML_F32 0
#define ENGINE_GGML_F16 1
#define ENGINE_GGML_Q4_0 2
#define ENGINE_GGML_Q8_0 8
#define ENGINE_GGML_BF16 30

/* GGUF metadata value type codes. */
#define ENGINE_GGUF_UINT8 0
#define ENGINE_GGUF_INT8 1
#define ENGINE_GGUF_UINT16 2
#define ENGINE_GGUF_INT16 3
#define ENGINE_GGUF_UINT32 4
#define ENGINE_GGUF_INT32 5
#define ENGINE_GGUF_FLOAT32 6
#define ENGINE_GGUF_BOOL 7
#define ENGINE_GGUF_STRING 8
#define ENGINE_GGUF_ARRAY 9
#define ENGINE_GGUF_UINT64 10
#define ENGINE_GGUF_INT64 11
#define ENGINE_GGUF_FLOAT64 12

typedef struct {
  const char* name;   /* NUL-terminated, owned by the handle */
  int32_t type;       /* GGML type code */
  int32_t n_dims;     /* 1..4 */
  int64_t dims[4];    /* dims[0] innermost; unused entries are 1 */
  uint64_t offset;    /* absolute byte offset of the data in the file */
  uint64_t nbytes;    /* 0 when the type's block size is unknown to the loader */
  const void* data;   /* host pointer into the read-only mapping */
} engine_gguf_tensor_t;

/* Maps `path` read-only and parses it.  On success *out owns the mapping. */
ENGINE_B200_API int engine_gguf_open(const char* path, engine_gguf_t** out);
/* Unmaps and frees; null is a no-op. */
ENGINE_B200_API int engine_gguf_close(engine_gguf_t* g);
ENGINE_B200_API int engine_gguf_version(const engine_gguf_t* g, int32_t* version,
                                        uint64_t* alignment);

ENGINE_B200_API int engine_gguf_tensor_count(const engine_gguf_t* g, int64_t* n);
ENGINE_B200_API int engine_gguf_tensor(const engine_gguf_t* g, int64_t index,
                                       engine_gguf_tensor_t* out);
/* ENGINE_ERR_INVALID when no tensor has that name. */
ENGINE_B200_API int engine_gguf_find_tensor(const engine_gguf_t* g, const char* name,
                                            int64_t* index);

ENGINE_B200_API int engine_gguf_meta_count(const engine_gguf_t* g, int64_t* n);
/* Key and value type of entry `index`; for arrays also the element type and count. */
ENGINE_B200_API int engine_gguf_meta_entry(const engine_gguf_t* g, int64_t index,
                                           const char** key, int32_t* type, int32_t* elem_type,
                                           uint64_t* count);
/* Typed lookups by key: ENGINE_ERR_INVALID when the key is missing or its value
 * has another kind (integer types and bool read as int; float32/64 as float). */
ENGINE_B200_API int engine_gguf_meta_int(const engine_gguf_t* g, const char* key, int64_t* v);
ENGINE_B200_API int engine_gguf_meta_float(const engine_gguf_t* g, const char* key, double* v);
ENGINE_B200_API int engine_gguf_meta_string(const engine_gguf_t* g, const char* key,
                                            const char** s, uint64_t* len);

/* Places tensor `index` on the device in the layout the projections read:
 *  F32 / F16 / BF16: `payload` receives the nbytes of elements, row-major with
 *    dims[0] contiguous (a [N,K] weight for linear_* / gemv_f16_nk);
 *  Q8_0 / Q4_0: the packed blocks are copied to `staging` (device, >= nbytes)
 *    and engine_cuda_quant_repack writes `payload` and `scales` for
 *    engine_cuda_gemv_q_nk, with K = dims[0] and N = the product of the others.
 * The host copy goes through pinned double buffers owned by the handle; the
 * call returns once the copy and the repack are enqueued on `stream`
 * (engine_gguf_close waits for this handle's copies before freeing the
 * buffers).  Other types: ENGINE_ERR_UNSUPPORTED.
 * One handle's pinned buffers serve one load at a time: calls on the same
 * handle from several host threads must be serialised by the caller. */
ENGINE_B200_API int engine_gguf_load_tensor(engine_gguf_t* g, int64_t index, void* payload,
                                            engine_half_t* scales, void* staging,
                                            engine_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* ENGINE_B200_H_ */
