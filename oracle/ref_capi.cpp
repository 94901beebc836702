// ref_capi.cpp -- TEST INFRASTRUCTURE ONLY.
//
// A C-ABI shim over the REFERENCE engine's own scalar CPU oracle, so that Python
// tests and bench.py's reference arm can call it through ctypes.  It is compiled
// together with the unmodified reference sources src/cpu_ref/{matmul,gemv,
// rmsnorm,rmsnorm_linear,swiglu,vector_add}_cpu.cpp (read where they lie; nothing
// is copied) by oracle/Makefile into oracle/_ref/, which is never committed.
//
// Every function forwards to engine::cpu::<name> (include/engine/cpu_ref.hpp:
// matmul :55, gemv :60, rmsnorm :50, rmsnorm_linear :90, gemv_fp16 :99,
// swiglu_fp16 :116, vector_add :27).  The *_rows_mt helpers split the output rows
// into contiguous blocks over std::thread and call the same function once per
// block; per-element arithmetic is unchanged, so results are bit-identical to the
// single-thread call.  FP16 data crosses the ABI as raw binary16 bits.

#include <engine/cpu_ref.hpp>

#include <cstdint>
#include <cstring>
#include <exception>
#include <thread>
#include <vector>

namespace {

template <class F>
void split_rows(std::int64_t M, int nthreads, F&& body) {
  if (nthreads < 1) nthreads = 1;
  if (nthreads > M) nthreads = static_cast<int>(M > 0 ? M : 1);
  const std::int64_t per = (M + nthreads - 1) / nthreads;
  std::vector<std::thread> pool;
  for (int t = 0; t < nthreads; ++t) {
    const std::int64_t r0 = t * per;
    const std::int64_t r1 = std::min<std::int64_t>(M, r0 + per);
    if (r0 >= r1) break;
    if (nthreads == 1) {
      body(r0, r1);
    } else {
      pool.emplace_back([=] { body(r0, r1); });
    }
  }
  for (auto& th : pool) th.join();
}

const engine::half* as_half(const std::uint16_t* p) {
  return reinterpret_cast<const engine::half*>(p);
}
engine::half* as_half(std::uint16_t* p) { return reinterpret_cast<engine::half*>(p); }

}  // namespace

extern "C" {

int ref_abi_half_bytes() { return static_cast<int>(sizeof(engine::half)); }

void ref_matmul(const float* A, const float* B, float* C, std::int64_t M, std::int64_t N,
                std::int64_t K, int nthreads) {
  split_rows(M, nthreads, [&](std::int64_t r0, std::int64_t r1) {
    engine::cpu::matmul(A + r0 * K, B, C + r0 * N, r1 - r0, N, K);
  });
}

void ref_gemv(const float* A, const float* x, float* out, std::int64_t N, std::int64_t K) {
  engine::cpu::gemv(A, x, out, N, K);
}

void ref_gemv_fp16(const std::uint16_t* A, const std::uint16_t* x, std::uint16_t* out,
                   std::int64_t N, std::int64_t K) {
  engine::cpu::gemv_fp16(as_half(A), as_half(x), as_half(out), N, K);
}

void ref_rmsnorm(const float* in, const float* weight, float* out, std::int64_t rows,
                 std::int64_t cols, float eps) {
  engine::cpu::rmsnorm(in, weight, out, rows, cols, eps);
}

void ref_residual_rmsnorm(const float* x, const float* residual, const float* weight,
                          float* norm_out, float* sum_out, std::int64_t rows, std::int64_t cols,
                          float eps) {
  engine::cpu::residual_rmsnorm(x, residual, weight, norm_out, sum_out, rows, cols, eps);
}

void ref_rmsnorm_linear(const float* in, const float* rms_weight, const float* W, float* out,
                        std::int64_t M, std::int64_t N, std::int64_t K, float eps,
                        int nthreads) {
  split_rows(M, nthreads, [&](std::int64_t r0, std::int64_t r1) {
    engine::cpu::rmsnorm_linear(in + r0 * K, rms_weight, W, out + r0 * N, r1 - r0, N, K, eps);
  });
}

void ref_swiglu_fp16(const std::uint16_t* gate, const std::uint16_t* up, std::uint16_t* out,
                     std::int64_t n) {
  engine::cpu::swiglu_fp16(as_half(gate), as_half(up), as_half(out), n);
}

int ref_attention(const std::uint16_t* q, const std::uint16_t* k, const std::uint16_t* v,
                  std::uint16_t* out, std::int64_t s_q, std::int64_t s_kv, std::int64_t n_heads,
                  std::int64_t n_kv_heads, std::int64_t head_dim, std::int64_t kv_head_stride,
                  float scale, std::int64_t q_pos_offset, int is_causal, float* out_lse) {
  try {
    engine::cpu::attention(as_half(q), as_half(k), as_half(v), as_half(out), s_q, s_kv, n_heads,
                           n_kv_heads, head_dim, kv_head_stride, scale, q_pos_offset,
                           is_causal != 0, out_lse);
  } catch (const std::exception&) {
    return 1;  // the reference's contract check (EngineError)
  }
  return 0;
}

int ref_attention_online(const std::uint16_t* q, const std::uint16_t* k, const std::uint16_t* v,
                         std::uint16_t* out, std::int64_t s_q, std::int64_t s_kv,
                         std::int64_t n_heads, std::int64_t n_kv_heads, std::int64_t head_dim,
                         std::int64_t kv_head_stride, float scale, std::int64_t q_pos_offset,
                         int is_causal, float* out_lse) {
  try {
    engine::cpu::attention_online(as_half(q), as_half(k), as_half(v), as_half(out), s_q, s_kv,
                                  n_heads, n_kv_heads, head_dim, kv_head_stride, scale,
                                  q_pos_offset, is_causal != 0, out_lse);
  } catch (const std::exception&) {
    return 1;
  }
  return 0;
}

void ref_vector_add(const float* a, const float* b, float* out, std::int64_t n) {
  engine::cpu::vector_add(a, b, out, n);
}

// FP16 GEMM as the reference would run it on the CPU: widen FP16 (exact) to
// float and call engine::cpu::matmul, row blocks over threads.  Bt != 0 means B
// is given as W[N,K] and is transposed on the host (an exact copy) first.
void ref_matmul_f16_as_f32(const std::uint16_t* A, const std::uint16_t* B, float* C,
                           std::int64_t M, std::int64_t N, std::int64_t K, int Bt,
                           int nthreads) {
  std::vector<float> a(static_cast<std::size_t>(M * K));
  std::vector<float> b(static_cast<std::size_t>(K * N));
  for (std::int64_t i = 0; i < M * K; ++i) a[i] = engine::half_to_float(as_half(A)[i]);
  if (Bt) {
    for (std::int64_t n = 0; n < N; ++n)
      for (std::int64_t k = 0; k < K; ++k)
        b[k * N + n] = engine::half_to_float(as_half(B)[n * K + k]);
  } else {
    for (std::int64_t i = 0; i < K * N; ++i) b[i] = engine::half_to_float(as_half(B)[i]);
  }
  ref_matmul(a.data(), b.data(), C, M, N, K, nthreads);
}

}  // extern "C"
