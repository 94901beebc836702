"""Torch-tensor front end of the hot path.

Tensors supply device memory and the current CUDA stream; every computation is
a call into libengine_b200.so.  Inputs must be contiguous CUDA tensors of the
stated dtype (checked here, loudly); outputs are allocated when not given.
"""
from __future__ import annotations

import torch

from . import cuda as _c


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _req(t: torch.Tensor, dtype: torch.dtype, name: str) -> torch.Tensor:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (the library has no CPU path)")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous (row-major)")
    return t


def _ptr(t):
    return 0 if t is None else t.data_ptr()


def matmul_f32(A, B, out=None, variant: str = "register_tiled"):
    """C = A @ B, FP32 [M,K] x [K,N] (engine::cuda::matmul_<variant>)."""
    _req(A, torch.float32, "A")
    _req(B, torch.float32, "B")
    M, K = A.shape
    N = B.shape[1]
    C = out if out is not None else torch.empty(M, N, device=A.device, dtype=torch.float32)
    fn = {"naive": _c.matmul_naive, "tiled": _c.matmul_tiled,
          "register_tiled": _c.matmul_register_tiled}[variant]
    fn(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K, _stream())
    return C


def matmul(A, B, out=None):
    """C = A @ B with FP16 or BF16 A[M,K], B[K,N] on tcgen05 tensor cores."""
    bf16 = A.dtype == torch.bfloat16
    dt = torch.bfloat16 if bf16 else torch.float16
    _req(A, dt, "A")
    _req(B, dt, "B")
    M, K = A.shape
    N = B.shape[1]
    C = out if out is not None else torch.empty(M, N, device=A.device, dtype=dt)
    (_c.matmul_bf16 if bf16 else _c.matmul_f16)(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K,
                                                _stream())
    return C


def linear(X, W, residual=None, out=None):
    """Y = X @ W^T (+ residual) with W stored [N,K]; FP16 or BF16."""
    bf16 = X.dtype == torch.bfloat16
    dt = torch.bfloat16 if bf16 else torch.float16
    _req(X, dt, "X")
    _req(W, dt, "W")
    if residual is not None:
        _req(residual, dt, "residual")
    M, K = X.shape
    N = W.shape[0]
    Y = out if out is not None else torch.empty(M, N, device=X.device, dtype=dt)
    (_c.linear_bf16 if bf16 else _c.linear_f16)(X.data_ptr(), W.data_ptr(), _ptr(residual),
                                                Y.data_ptr(), M, N, K, _stream())
    return Y


def gemv(W, x, residual=None, out=None):
    """y = W[N,K] @ x[K] (+ residual), FP16 decode GEMV."""
    _req(W, torch.float16, "W")
    _req(x, torch.float16, "x")
    N, K = W.shape
    y = out if out is not None else torch.empty(N, device=W.device, dtype=torch.float16)
    _c.gemv_f16_nk(W.data_ptr(), x.data_ptr(), _ptr(residual), y.data_ptr(), N, K, _stream())
    return y


def rmsnorm_linear(x, gamma, W, eps: float = 1e-5, residual=None, out=None):
    """Y = rmsnorm(x; gamma, eps) @ W^T (+ residual), FP16, W stored [N,K]."""
    _req(x, torch.float16, "x")
    _req(W, torch.float16, "W")
    if gamma is not None:
        _req(gamma, torch.float16, "gamma")
    if residual is not None:
        _req(residual, torch.float16, "residual")
    M, K = x.shape
    N = W.shape[0]
    Y = out if out is not None else torch.empty(M, N, device=x.device, dtype=torch.float16)
    _c.rmsnorm_linear_f16(x.data_ptr(), _ptr(gamma), W.data_ptr(), _ptr(residual), Y.data_ptr(),
                          M, N, K, eps, _stream())
    return Y


def rmsnorm_linear_kv(x, gamma, W, eps, k_cache, v_cache, kv_row0: int, pos: int, out=None):
    """Batch-1 rmsnorm_linear (x [1, K]) whose output rows [kv_row0, kv_row0 + H_kv*d)
    and the next H_kv*d rows (the token's K and V) are also stored at position pos
    of the head-major caches [H_kv, max_len, d], in the same kernel."""
    _req(x, torch.float16, "x")
    _req(W, torch.float16, "W")
    if gamma is not None:
        _req(gamma, torch.float16, "gamma")
    for t, n in ((k_cache, "k_cache"), (v_cache, "v_cache")):
        if t.dtype != torch.float16 or not t.is_cuda or not t.is_contiguous():
            raise TypeError(f"{n} must be a contiguous CUDA float16 tensor [H_kv, max_len, d]")
    M, K = x.shape
    if M != 1:
        raise ValueError("rmsnorm_linear_kv: one token (x [1, K])")
    N = W.shape[0]
    hk, max_len, d = k_cache.shape
    Y = out if out is not None else torch.empty(1, N, device=x.device, dtype=torch.float16)
    _c.rmsnorm_linear_kv_f16(x.data_ptr(), _ptr(gamma), W.data_ptr(), 0, Y.data_ptr(), N, K, eps,
                             k_cache.data_ptr(), v_cache.data_ptr(), kv_row0, hk, d, max_len, pos,
                             _stream())
    return Y


def rmsnorm_linear_swiglu(x, gamma, W_gu, eps: float = 1e-5, out=None):
    """swiglu(g, u) with [g | u] = rmsnorm(x; gamma, eps) @ W_gu^T, W_gu [2F,K] = gate
    rows then up rows; FP16.  Same result as rmsnorm_linear followed by swiglu."""
    _req(x, torch.float16, "x")
    _req(W_gu, torch.float16, "W_gu")
    if gamma is not None:
        _req(gamma, torch.float16, "gamma")
    M, K = x.shape
    F = W_gu.shape[0] // 2
    Y = out if out is not None else torch.empty(M, F, device=x.device, dtype=torch.float16)
    _c.rmsnorm_linear_swiglu_f16(x.data_ptr(), _ptr(gamma), W_gu.data_ptr(), Y.data_ptr(), M, F,
                                 K, eps, _stream())
    return Y


def quant_repack(qtype, blocks, N, K):
    """Packed GGUF blocks (uint8 CUDA tensor) -> (payload, scales) in the layout
    gemv_q streams: payload [N, K] int8 (Q8_0) or [N, K/2] uint8 (Q4_0, each
    block's 16 nibble bytes in GGUF order), scales [N, K/32] FP16."""
    _req(blocks, torch.uint8, "blocks")
    pay = K if qtype == _c.Q8_0 else K // 2
    q = torch.empty(N, pay, device=blocks.device, dtype=torch.uint8)
    d = torch.empty(N, K // 32, device=blocks.device, dtype=torch.float16)
    _c.quant_repack(qtype, blocks.data_ptr(), q.data_ptr(), d.data_ptr(), N, K, _stream())
    return q, d


def gemv_q(qtype, q, scales, x, residual=None, out=None):
    """y = W x (+ residual) for W given by quant_repack's (payload, scales)."""
    _req(q, torch.uint8, "q")
    _req(scales, torch.float16, "scales")
    _req(x, torch.float16, "x")
    N, K = scales.shape[0], x.numel()
    y = out if out is not None else torch.empty(N, device=x.device, dtype=torch.float16)
    _c.gemv_q_nk(qtype, q.data_ptr(), scales.data_ptr(), x.data_ptr(), _ptr(residual),
                 y.data_ptr(), N, K, _stream())
    return y


def residual_rmsnorm(x, residual, weight=None, eps: float = 1e-5):
    """(norm_out, sum_out): sum_out = x + residual, norm_out = rmsnorm(sum_out) *
    weight, FP32 [rows, cols] (engine::cuda::residual_rmsnorm)."""
    _req(x, torch.float32, "x")
    _req(residual, torch.float32, "residual")
    if weight is not None:
        _req(weight, torch.float32, "weight")
    rows, cols = x.shape
    norm = torch.empty_like(x)
    sm = torch.empty_like(x)
    _c.residual_rmsnorm(x.data_ptr(), residual.data_ptr(), _ptr(weight), norm.data_ptr(),
                        sm.data_ptr(), rows, cols, eps, _stream())
    return norm, sm


def attention(q, k, v, scale=None, q_pos_offset: int = 0, is_causal: bool = True,
              want_lse: bool = False):
    """out [s_q, H, d] (FP16) of q [s_q, H, d] over k / v [H_kv, s_kv, d]
    (engine::cuda::attention_prefill); with want_lse also lse [s_q, H] (FP32)."""
    for t, n in ((q, "q"), (k, "k"), (v, "v")):
        _req(t, torch.float16, n)
    s_q, H, d = q.shape
    H_kv, s_kv, _ = k.shape
    scale = d ** -0.5 if scale is None else scale
    out = torch.empty_like(q)
    lse = torch.empty(s_q, H, device=q.device, dtype=torch.float32) if want_lse else None
    _c.attention_prefill(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), s_q, s_kv, H,
                         H_kv, d, s_kv * d, scale, q_pos_offset, is_causal, _ptr(lse), _stream())
    return (out, lse) if want_lse else out


def attention_decode(q, k, v, scale=None, split_kv: int = 0):
    """out [H, d] of one query row q [H, d] over all kv_len keys of k / v
    [H_kv, kv_len, d] (engine::cuda::attention_decode, split-KV)."""
    for t, n in ((q, "q"), (k, "k"), (v, "v")):
        _req(t, torch.float16, n)
    H, d = q.shape
    H_kv, kv_len, _ = k.shape
    scale = d ** -0.5 if scale is None else scale
    out = torch.empty_like(q)
    _c.attention_decode(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), kv_len, H, H_kv,
                        d, kv_len * d, scale, split_kv, _stream())
    return out


def kv_cache_write(k_rows, v_rows, k_cache, v_cache, pos: int, n_seq: int = 1):
    """Scatters K / V rows into head-major caches [n_seq * H_kv, max_len, d] at
    positions pos.. (engine::cuda::detail::kv_cache_write, batched over n_seq
    sequences).  k_rows / v_rows are [n_seq * s_new, H_kv * d] views whose rows
    may be strided (e.g. the K and V columns of a fused Q/K/V projection)."""
    for t, n in ((k_rows, "k_rows"), (v_rows, "v_rows"), (k_cache, "k_cache"), (v_cache, "v_cache")):
        if t.dtype != torch.float16 or not t.is_cuda:
            raise TypeError(f"{n} must be a CUDA float16 tensor")
    if k_rows.stride(1) != 1 or v_rows.stride(1) != 1 or k_rows.stride(0) != v_rows.stride(0):
        raise ValueError("k_rows / v_rows: rows must be contiguous and share one pitch")
    if not (k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise ValueError("caches must be contiguous [n_seq * H_kv, max_len, d]")
    hk, max_len, d = k_cache.shape
    H_kv = hk // n_seq
    s_new = k_rows.shape[0] // n_seq
    if k_rows.shape[1] != H_kv * d:
        raise ValueError("k_rows: width != H_kv * d")
    _c.kv_cache_write_rows(k_rows.data_ptr(), v_rows.data_ptr(), k_rows.stride(0), k_cache.data_ptr(),
                           v_cache.data_ptr(), n_seq, s_new, H_kv, d, pos, max_len, _stream())


def attention_cached(q, k_cache, v_cache, kv_len: int, q_pos_offset: int, is_causal: bool = True,
                     scale=None, out=None):
    """attention_prefill of q [s_q, H, d] over the first kv_len positions of the
    caches [H_kv, max_len, d] (kv_head_stride = max_len * d)."""
    _req(q, torch.float16, "q")
    s_q, H, d = q.shape
    H_kv, max_len, _ = k_cache.shape
    scale = d ** -0.5 if scale is None else scale
    o = out if out is not None else torch.empty_like(q)
    _c.attention_prefill(q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), o.data_ptr(), s_q,
                         kv_len, H, H_kv, d, max_len * d, scale, q_pos_offset, is_causal, 0,
                         _stream())
    return o


def attention_decode_cached(q, k_cache, v_cache, kv_len: int, scale=None, out=None):
    """attention_decode of one query row per head, q [H, d], over the first
    kv_len positions of the caches [H_kv, max_len, d]; a batch of equal-length
    sequences is q [B * H, d] over caches [B * H_kv, max_len, d]."""
    _req(q, torch.float16, "q")
    H, d = q.shape
    H_kv, max_len, _ = k_cache.shape
    scale = d ** -0.5 if scale is None else scale
    o = out if out is not None else torch.empty_like(q)
    _c.attention_decode(q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), o.data_ptr(), kv_len,
                        H, H_kv, d, max_len * d, scale, 0, _stream())
    return o


def swiglu(gate, up, out=None):
    _req(gate, torch.float16, "gate")
    _req(up, torch.float16, "up")
    o = out if out is not None else torch.empty_like(gate)
    _c.swiglu_fp16(gate.data_ptr(), up.data_ptr(), o.data_ptr(), gate.numel(), _stream())
    return o


def embedding(table, ids, out=None):
    _req(table, torch.float16, "table")
    _req(ids, torch.int32, "ids")
    V, D = table.shape
    T = ids.numel()
    o = out if out is not None else torch.empty(T, D, device=table.device, dtype=torch.float16)
    _c.embedding_fp16(table.data_ptr(), ids.data_ptr(), o.data_ptr(), T, D, V, _stream())
    return o
