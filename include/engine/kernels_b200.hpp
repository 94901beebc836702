#pragma once
//===----------------------------------------------------------------------===//
// engine/kernels_b200.hpp -- the engine's C++ launch API over the B200 C ABI.
//
// Restores the exact signatures of include/engine/kernels.hpp (namespace
// engine::cuda, raw device pointers, int64 dims, `cudaStream_t stream = 0`) on
// top of include/engine_b200.h, so an engine translation unit switches to the
// B200 kernels by including this header instead of kernels.hpp and linking
// libengine_b200.so in place of kernels/matmul*.cu, gemv*.cu and
// rmsnorm_linear.cu.  A nonzero status is rethrown as engine::EngineError with
// the library's message, like the reference's ENGINE_CHECK (check.hpp:36-65).
//
// When the engine's own <engine/check.hpp> is reachable its EngineError is
// used, so existing catch sites and EXPECT_THROWS_MSG checks keep working;
// otherwise a compatible engine::EngineError is declared here.
//===----------------------------------------------------------------------===//

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <stdexcept>
#include <string>

#include "../engine_b200.h"

#if __has_include(<engine/check.hpp>) && __has_include(<engine/config.hpp>)
#include <engine/check.hpp>
#else
namespace engine {
class EngineError : public std::runtime_error {
 public:
  explicit EngineError(const std::string& what) : std::runtime_error(what) {}
};
}  // namespace engine
#endif

namespace engine::cuda {

namespace b200_detail {
inline void check(int rc) {
  if (rc != ENGINE_OK) throw ::engine::EngineError(std::string("[engine] ") + engine_last_error());
}
inline const engine_half_t* h(const __half* p) { return reinterpret_cast<const engine_half_t*>(p); }
inline engine_half_t* h(__half* p) { return reinterpret_cast<engine_half_t*>(p); }
inline const engine_bf16_t* b(const __nv_bfloat16* p) {
  return reinterpret_cast<const engine_bf16_t*>(p);
}
inline engine_bf16_t* b(__nv_bfloat16* p) { return reinterpret_cast<engine_bf16_t*>(p); }
}  // namespace b200_detail

// -- kernels.hpp:62-104, 120: the legacy hot-path launchers ------------------

inline void rmsnorm(const float* in, const float* weight, float* out, std::int64_t rows,
                    std::int64_t cols, float eps, cudaStream_t stream = 0) {
  b200_detail::check(engine_cuda_rmsnorm(in, weight, out, rows, cols, eps, stream));
}

// kernels.hpp:110
inline void residual_rmsnorm(const float* x, const float* residual, const float* weight,
                             float* norm_out, float* sum_out, std::int64_t rows,
                             std::int64_t cols, float eps, cudaStream_t stream = 0) {
  b200_detail::check(engine_cuda_residual_rmsnorm(x, residual, weight, norm_out, sum_out, rows,
                                                  cols, eps, stream));
}

inline void matmul_naive(const float* A, const float* B, float* C, std::int64_t M,
                         std::int64_t N, std::int64_t K, cudaStream_t stream = 0) {
  b200_detail::check(engine_cuda_matmul_naive(A, B, C, M, N, K, stream));
}

inline void matmul_tiled(const float* A, const float* B, float* C, std::int64_t M,
                         std::int64_t N, std::int64_t K, cudaStream_t stream = 0) {
  b200_detail::check(engine_cuda_matmul_tiled(A, B, C, M, N, K, stream));
}

inline void matmul_register_tiled(const float* A, const float* B, float* C, std::int64_t M,
                                  std::int64_t N, std::int64_t K, cudaStream_t stream = 0) {
  b200_detail::check(engine_cuda_matmul_register_tiled(A, B, C, M, N, K, stream));
}

inline void gemv(const float* A, const float* x, float* out, std::int64_t N, std::int64_t K,
                 cudaStream_t stream = 0) {
  b200_detail::check(engine_cuda_gemv(A, x, out, N, K, stream));
}

inline void rmsnorm_linear(const float* in, const float* rms_weight, const float* W, float* out,
                           std::int64_t M, std::int64_t N, std::int64_t K, float eps,
                           cudaStream_t stream = 0) {
  b200_detail::check(engine_cuda_rmsnorm_linear(in, rms_weight, W, out, M, N, K, eps, stream));
}

inline void rmsnorm_linear_fused_direct(const float* in, const float* rms_weight, const float* W,
                                        float* out, std::int64_t M, std::int64_t N,
                                        std::int64_t K, float eps, cudaStream_t stream = 0) {
  b200_detail::check(
      engine_cuda_rmsnorm_linear_fused_direct(in, rms_weight, W, out, M, N, K, eps, stream));
}

inline void gemv_fp16(const __half* A, const __half* x, __half* out, std::int64_t N,
                      std::int64_t K, cudaStream_t stream = 0) {
  b200_detail::check(engine_cuda_gemv_fp16(b200_detail::h(A), b200_detail::h(x),
                                           b200_detail::h(out), N, K, stream));
}

inline void vector_add(const float* a, const float* b, float* out, std::int64_t n,
                       cudaStream_t stream = 0) {
  b200_detail::check(engine_cuda_vector_add(a, b, out, n, stream));
}

inline void swiglu_fp16(const __half* gate, const __half* up, __half* out, std::int64_t n,
                        cudaStream_t stream = 0) {
  b200_detail::check(engine_cuda_swiglu_f16(b200_detail::h(gate), b200_detail::h(up),
                                            b200_detail::h(out), n, stream));
}

// -- new B200 entry points: FP16/BF16 and [N,K] weights ------------------------

inline void matmul_f16(const __half* A, const __half* B, __half* C, std::int64_t M,
                       std::int64_t N, std::int64_t K, cudaStream_t stream = 0) {
  b200_detail::check(engine_cuda_matmul_f16(b200_detail::h(A), b200_detail::h(B),
                                            b200_detail::h(C), M, N, K, stream));
}

inline void linear_f16(const __half* X, const __half* W, const __half* residual, __half* Y,
                       std::int64_t M, std::int64_t N, std::int64_t K, cudaStream_t stream = 0) {
  b200_detail::check(engine_cuda_linear_f16(b200_detail::h(X), b200_detail::h(W),
                                            b200_detail::h(residual), b200_detail::h(Y), M, N, K,
                                            stream));
}

inline void gemv_f16_nk(const __half* W, const __half* x, const __half* residual, __half* y,
                        std::int64_t N, std::int64_t K, cudaStream_t stream = 0) {
  b200_detail::check(engine_cuda_gemv_f16_nk(b200_detail::h(W), b200_detail::h(x),
                                             b200_detail::h(residual), b200_detail::h(y), N, K,
                                             stream));
}

inline void rmsnorm_linear_f16(const __half* x, const __half* gamma, const __half* W,
                               const __half* residual, __half* Y, std::int64_t M, std::int64_t N,
                               std::int64_t K, float eps, cudaStream_t stream = 0) {
  b200_detail::check(engine_cuda_rmsnorm_linear_f16(
      b200_detail::h(x), b200_detail::h(gamma), b200_detail::h(W), b200_detail::h(residual),
      b200_detail::h(Y), M, N, K, eps, stream));
}

inline void matmul_bf16(const __nv_bfloat16* A, const __nv_bfloat16* B, __nv_bfloat16* C,
                        std::int64_t M, std::int64_t N, std::int64_t K, cudaStream_t stream = 0) {
  b200_detail::check(engine_cuda_matmul_bf16(b200_detail::b(A), b200_detail::b(B),
                                             b200_detail::b(C), M, N, K, stream));
}

inline void linear_bf16(const __nv_bfloat16* X, const __nv_bfloat16* W,
                        const __nv_bfloat16* residual, __nv_bfloat16* Y, std::int64_t M,
                        std::int64_t N, std::int64_t K, cudaStream_t stream = 0) {
  b200_detail::check(engine_cuda_linear_bf16(b200_detail::b(X), b200_detail::b(W),
                                             b200_detail::b(residual), b200_detail::b(Y), M, N,
                                             K, stream));
}

// Fused RMSNorm -> gate/up projection -> SwiGLU: rmsnorm_linear followed by
// swiglu_fp16 in one call (W_gu = gate rows, then up rows).
inline void rmsnorm_linear_swiglu_fp16(const __half* x, const __half* gamma, const __half* W_gu,
                                       __half* Y, std::int64_t M, std::int64_t F, std::int64_t K,
                                       float eps, cudaStream_t stream = 0) {
  b200_detail::check(engine_cuda_rmsnorm_linear_swiglu_f16(
      b200_detail::h(x), b200_detail::h(gamma), b200_detail::h(W_gu), b200_detail::h(Y), M, F, K,
      eps, stream));
}

// kernels.hpp:128 (embedding_fp16)
inline void embedding_fp16(const __half* table, const std::int32_t* ids, __half* out,
                           std::int64_t num_tokens, std::int64_t hidden, std::int64_t vocab,
                           cudaStream_t stream = 0) {
  b200_detail::check(engine_cuda_embedding_f16(b200_detail::h(table), ids, b200_detail::h(out),
                                               num_tokens, hidden, vocab, stream));
}

// Block-quantised weights (DType::Q8_0 / DType::Q4_0, dtype.hpp:95-125): split
// GGUF's packed blocks once at load time, then run the decode GEMV over the
// split layout.  qtype is ENGINE_Q8_0 or ENGINE_Q4_0; K % 32 == 0.
inline void quant_repack(int qtype, const void* blocks, void* payload, __half* scales,
                         std::int64_t N, std::int64_t K, cudaStream_t stream = 0) {
  b200_detail::check(
      engine_cuda_quant_repack(qtype, blocks, payload, b200_detail::h(scales), N, K, stream));
}

inline void gemv_q_nk(int qtype, const void* payload, const __half* scales, const __half* x,
                      const __half* residual, __half* y, std::int64_t N, std::int64_t K,
                      cudaStream_t stream = 0) {
  b200_detail::check(engine_cuda_gemv_q_nk(qtype, payload, b200_detail::h(scales),
                                           b200_detail::h(x), b200_detail::h(residual),
                                           b200_detail::h(y), N, K, stream));
}

// kernels.hpp:153 / :191 -- attention.  An engine build that keeps its own
// kernels/attention_*.cu (for attention_naive and the *_with_mode variants,
// which this library does not provide) defines ENGINE_B200_NO_ATTENTION.
#ifndef ENGINE_B200_NO_ATTENTION
inline void attention_prefill(const __half* q, const __half* k, const __half* v, __half* out,
                              std::int64_t s_q, std::int64_t s_kv, std::int64_t n_heads,
                              std::int64_t n_kv_heads, std::int64_t head_dim,
                              std::int64_t kv_head_stride, float scale,
                              std::int64_t q_pos_offset = 0, bool is_causal = true,
                              float* out_lse = nullptr, cudaStream_t stream = 0) {
  b200_detail::check(engine_cuda_attention_prefill(
      b200_detail::h(q), b200_detail::h(k), b200_detail::h(v), b200_detail::h(out), s_q, s_kv,
      n_heads, n_kv_heads, head_dim, kv_head_stride, scale, q_pos_offset, is_causal ? 1 : 0,
      out_lse, stream));
}

inline void attention_decode(const __half* q, const __half* k, const __half* v, __half* out,
                             std::int64_t kv_len, std::int64_t n_heads, std::int64_t n_kv_heads,
                             std::int64_t head_dim, std::int64_t kv_head_stride, float scale,
                             int split_kv = 0, cudaStream_t stream = 0) {
  b200_detail::check(engine_cuda_attention_decode(
      b200_detail::h(q), b200_detail::h(k), b200_detail::h(v), b200_detail::h(out), kv_len,
      n_heads, n_kv_heads, head_dim, kv_head_stride, scale, split_kv, stream));
}
namespace detail {
// kernels.hpp:184 -- the head-major KV-cache scatter of the attention bridge.
inline void kv_cache_write(const __half* k_new, const __half* v_new, __half* k_cache,
                           __half* v_cache, std::int64_t s_new, std::int64_t n_kv_heads,
                           std::int64_t head_dim, std::int64_t pos_offset,
                           std::int64_t kv_max_seq_len, cudaStream_t stream = 0) {
  b200_detail::check(engine_cuda_kv_cache_write(
      b200_detail::h(k_new), b200_detail::h(v_new), b200_detail::h(k_cache),
      b200_detail::h(v_cache), s_new, n_kv_heads, head_dim, pos_offset, kv_max_seq_len, stream));
}
}  // namespace detail
#endif  // ENGINE_B200_NO_ATTENTION

// -- tensor-parallel communicator (engine_tp_*) --------------------------------
// One per rank, on the rank's current device.  The host exchanges handle()
// between the ranks (all-gather), then calls open() with all of them in rank
// order.  Destroy only after a host barrier across the ranks.
class TpComm {
 public:
  TpComm(int rank, int world, std::int64_t max_elems) {
    b200_detail::check(engine_tp_comm_create(rank, world, max_elems, &comm_));
  }
  ~TpComm() { engine_tp_comm_destroy(comm_); }
  TpComm(const TpComm&) = delete;
  TpComm& operator=(const TpComm&) = delete;

  std::string handle() const {
    std::string h(ENGINE_TP_HANDLE_BYTES, '\0');
    b200_detail::check(engine_tp_comm_handle(comm_, &h[0]));
    return h;
  }
  void open(const std::string& all_handles) {
    b200_detail::check(engine_tp_comm_open(comm_, all_handles.data()));
  }
  // y = sum over ranks of partial (+ residual), on every rank
  void allreduce(const __half* partial, const __half* residual, __half* y, std::int64_t n,
                 cudaStream_t stream = 0) {
    b200_detail::check(engine_tp_allreduce_f16(comm_, b200_detail::h(partial),
                                               b200_detail::h(residual), b200_detail::h(y), n,
                                               stream));
  }
  // Y = sum over ranks of X_r W_r^T (+ residual): the row-split projection fused
  // with its all-reduce
  void linear_allreduce(const __half* X, const __half* W, const __half* residual, __half* Y,
                        std::int64_t M, std::int64_t N, std::int64_t K, cudaStream_t stream = 0) {
    b200_detail::check(engine_tp_linear_allreduce_f16(
        comm_, b200_detail::h(X), b200_detail::h(W), b200_detail::h(residual), b200_detail::h(Y),
        M, N, K, stream));
  }

 private:
  engine_tp_comm_t* comm_ = nullptr;
};

}  // namespace engine::cuda

// Tensor-typed overloads of the launchers above, when the engine's Tensor is on
// the include path.
#if __has_include(<engine/tensor.hpp>) && __has_include(<engine/config.hpp>)
#include "kernels_b200_tensor.hpp"
#endif

