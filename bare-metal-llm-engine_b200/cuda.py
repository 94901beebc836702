"""Raw-pointer mirror of ``engine::cuda`` (include/engine/kernels.hpp:34-204).

Same names, argument order and meaning as the reference's C++ launchers:
device pointers are ints (``tensor.data_ptr()``), dimensions are int64 and the
stream is last (an int handle, 0 = legacy default stream).  Every function
raises :class:`EngineError` when the library rejects the call.
"""
from __future__ import annotations

from . import _check, lib


def _s(stream) -> int | None:
    return int(stream) if stream else None


def matmul_naive(A, B, C, M, N, K, stream=0):  # kernels.hpp:67
    _check(lib().engine_cuda_matmul_naive(A, B, C, M, N, K, _s(stream)))


def matmul_tiled(A, B, C, M, N, K, stream=0):  # kernels.hpp:74
    _check(lib().engine_cuda_matmul_tiled(A, B, C, M, N, K, _s(stream)))


def matmul_register_tiled(A, B, C, M, N, K, stream=0):  # kernels.hpp:80
    _check(lib().engine_cuda_matmul_register_tiled(A, B, C, M, N, K, _s(stream)))


def gemv(A, x, out, N, K, stream=0):  # kernels.hpp:85
    _check(lib().engine_cuda_gemv(A, x, out, N, K, _s(stream)))


def gemv_fp16(A, x, out, N, K, stream=0):  # kernels.hpp:120
    _check(lib().engine_cuda_gemv_fp16(A, x, out, N, K, _s(stream)))


def rmsnorm(inp, weight, out, rows, cols, eps, stream=0):  # kernels.hpp:62
    _check(lib().engine_cuda_rmsnorm(inp, weight, out, rows, cols, eps, _s(stream)))


def residual_rmsnorm(x, residual, weight, norm_out, sum_out, rows, cols, eps,  # kernels.hpp:110
                     stream=0):
    _check(lib().engine_cuda_residual_rmsnorm(x, residual, weight, norm_out, sum_out, rows, cols,
                                              eps, _s(stream)))


def attention_prefill(q, k, v, out, s_q, s_kv, n_heads, n_kv_heads, head_dim,  # kernels.hpp:153
                      kv_head_stride, scale, q_pos_offset=0, is_causal=True, out_lse=0, stream=0):
    _check(lib().engine_cuda_attention_prefill(q, k, v, out, s_q, s_kv, n_heads, n_kv_heads,
                                               head_dim, kv_head_stride, scale, q_pos_offset,
                                               1 if is_causal else 0, out_lse, _s(stream)))


def attention_decode(q, k, v, out, kv_len, n_heads, n_kv_heads, head_dim,  # kernels.hpp:191
                     kv_head_stride, scale, split_kv=0, stream=0):
    _check(lib().engine_cuda_attention_decode(q, k, v, out, kv_len, n_heads, n_kv_heads, head_dim,
                                              kv_head_stride, scale, split_kv, _s(stream)))


def kv_cache_write(k_new, v_new, k_cache, v_cache, s_new, n_kv_heads, head_dim,  # kernels.hpp:184
                   pos_offset, kv_max_seq_len, stream=0):
    _check(lib().engine_cuda_kv_cache_write(k_new, v_new, k_cache, v_cache, s_new, n_kv_heads,
                                            head_dim, pos_offset, kv_max_seq_len, _s(stream)))


def kv_cache_write_rows(k_new, v_new, row_pitch, k_cache, v_cache, n_seq, s_new, n_kv_heads,
                        head_dim, pos_offset, kv_max_seq_len, stream=0):
    _check(lib().engine_cuda_kv_cache_write_rows(k_new, v_new, row_pitch, k_cache, v_cache, n_seq,
                                                 s_new, n_kv_heads, head_dim, pos_offset,
                                                 kv_max_seq_len, _s(stream)))


def rmsnorm_linear(inp, rms_weight, W, out, M, N, K, eps, stream=0):  # kernels.hpp:97
    _check(lib().engine_cuda_rmsnorm_linear(inp, rms_weight, W, out, M, N, K, eps, _s(stream)))


def rmsnorm_linear_fused_direct(inp, rms_weight, W, out, M, N, K, eps, stream=0):  # kernels.hpp:102
    _check(lib().engine_cuda_rmsnorm_linear_fused_direct(inp, rms_weight, W, out, M, N, K, eps,
                                                         _s(stream)))


def vector_add(a, b, out, n, stream=0):  # kernels.hpp:49
    _check(lib().engine_cuda_vector_add(a, b, out, n, _s(stream)))


def swiglu_fp16(gate, up, out, n, stream=0):  # kernels.hpp:141
    _check(lib().engine_cuda_swiglu_f16(gate, up, out, n, _s(stream)))


def embedding_fp16(table, ids, out, num_tokens, hidden_dim, vocab_size, stream=0):  # kernels.hpp:128
    _check(lib().engine_cuda_embedding_f16(table, ids, out, num_tokens, hidden_dim, vocab_size,
                                           _s(stream)))


# -- new entry points for the B200 configurations ([N,K] weights, FP16/BF16) --

def matmul_f16(A, B, C, M, N, K, stream=0):
    _check(lib().engine_cuda_matmul_f16(A, B, C, M, N, K, _s(stream)))


def matmul_bf16(A, B, C, M, N, K, stream=0):
    _check(lib().engine_cuda_matmul_bf16(A, B, C, M, N, K, _s(stream)))


def linear_f16(X, W, residual, Y, M, N, K, stream=0):
    _check(lib().engine_cuda_linear_f16(X, W, residual, Y, M, N, K, _s(stream)))


def linear_bf16(X, W, residual, Y, M, N, K, stream=0):
    _check(lib().engine_cuda_linear_bf16(X, W, residual, Y, M, N, K, _s(stream)))


def gemv_f16_nk(W, x, residual, y, N, K, stream=0):
    _check(lib().engine_cuda_gemv_f16_nk(W, x, residual, y, N, K, _s(stream)))


def rmsnorm_linear_f16(x, gamma, W, residual, Y, M, N, K, eps, stream=0):
    _check(lib().engine_cuda_rmsnorm_linear_f16(x, gamma, W, residual, Y, M, N, K, eps,
                                                _s(stream)))


def rmsnorm_linear_swiglu_f16(x, gamma, W_gu, Y, M, F, K, eps, stream=0):
    """Y[M,F] = swiglu(rmsnorm(x) W_gu[0:F]^T, rmsnorm(x) W_gu[F:2F]^T) in one call
    (kernels.hpp rmsnorm_linear followed by swiglu_fp16)."""
    _check(lib().engine_cuda_rmsnorm_linear_swiglu_f16(x, gamma, W_gu, Y, M, F, K, eps, _s(stream)))


def rmsnorm_linear_kv_f16(x, gamma, W, residual, Y, N, K, eps, k_cache, v_cache, kv_row0,
                          n_kv_heads, head_dim, max_len, pos, stream=0):
    """Batch-1 rmsnorm_linear_f16 that also stores output rows [kv_row0, +n_kv_heads*head_dim)
    (K) and the next n_kv_heads*head_dim (V) at position pos of the head-major caches."""
    _check(lib().engine_cuda_rmsnorm_linear_kv_f16(x, gamma, W, residual, Y, N, K, eps, k_cache,
                                                   v_cache, kv_row0, n_kv_heads, head_dim,
                                                   max_len, pos, _s(stream)))


def rmsnorm_linear_f16_noalloc(x, gamma, W, residual, Y, M, N, K, eps, stream=0):
    """rmsnorm_linear_f16 without any device allocation (fixed in-library scratch;
    M <= 32, K <= 16384).  Concurrent calls on unordered streams race."""
    _check(lib().engine_cuda_rmsnorm_linear_f16_noalloc(x, gamma, W, residual, Y, M, N, K, eps,
                                                        _s(stream)))


# ------------------------------------------------- block-quantised weights
# engine_cuda_quant_repack / engine_cuda_gemv_q_nk: GGUF Q8_0 / Q4_0 blocks, the
# formats the engine declares (include/engine/dtype.hpp:95-125).

Q8_0, Q4_0 = 8, 4


def quant_repack(qtype, blocks, q_out, scales_out, N, K, stream=0):
    _check(lib().engine_cuda_quant_repack(qtype, blocks, q_out, scales_out, N, K, _s(stream)))


def gemv_q_nk(qtype, q, scales, x, residual, y, N, K, stream=0):
    _check(lib().engine_cuda_gemv_q_nk(qtype, q, scales, x, residual, y, N, K, _s(stream)))


# ------------------------------------------------- tensor-parallel communicator
# engine_tp_* (include/engine_b200.h): no counterpart in the reference.

TP_HANDLE_BYTES = 64


def tp_comm_create(rank, world, max_elems) -> int:
    """Allocates this rank's exchange region on the current device; returns the
    communicator handle (an int)."""
    import ctypes

    out = ctypes.c_void_p(0)
    _check(lib().engine_tp_comm_create(rank, world, max_elems, ctypes.byref(out)))
    return int(out.value)


def tp_comm_handle(comm) -> bytes:
    import ctypes

    buf = ctypes.create_string_buffer(TP_HANDLE_BYTES)
    _check(lib().engine_tp_comm_handle(comm, buf))
    return buf.raw


def tp_comm_open(comm, handles: bytes):
    """handles: world x TP_HANDLE_BYTES bytes in rank order."""
    import ctypes

    buf = ctypes.create_string_buffer(handles, len(handles))
    _check(lib().engine_tp_comm_open(comm, buf))


def tp_comm_destroy(comm):
    _check(lib().engine_tp_comm_destroy(comm))


def tp_allreduce_f16(comm, partial, residual, y, n, stream=0):
    _check(lib().engine_tp_allreduce_f16(comm, partial, residual, y, n, _s(stream)))


def tp_linear_allreduce_f16(comm, X, W, residual, Y, M, N, K, stream=0):
    _check(lib().engine_tp_linear_allreduce_f16(comm, X, W, residual, Y, M, N, K, _s(stream)))

