"""oracle -- TEST INFRASTRUCTURE ONLY: the CPU checkers for the B200 hot path.

Two checkers live here, both loaded through ctypes and both operating on numpy
arrays:

* ``liboracle.so`` -- ``cpu_oracle.c``, a plain-C restatement of the reference
  engine's scalar oracle (Parag63/bare-metal-llm-engine ``src/cpu_ref/``): FP64
  accumulation, eps inside the square root, round-to-nearest-even FP16 output.
* ``_ref/libref_cpu.so`` -- the reference's OWN ``src/cpu_ref`` sources compiled
  in place by ``oracle/Makefile`` (present only where the reference tree was
  available when ``build()`` ran; it travels to the GPU box as a built file).
* ``_ref/libref_cuda.so`` -- the reference's own CUDA launchers compiled for
  sm_100a: bench.py's same-GPU "old kernel" baseline leg.

The reference tree is found by ``reference_dir()``: the ENGINE_REF_DIR
environment variable, else a checkout named ``reference`` beside this
repository.

Only ``tests/``, ``__graft_entry__`` and ``bench.py``'s baseline legs (the CPU
baseline, the old-kernel baseline and the reference arm) may import this
package.  The CUDA library never does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
_LIB = HERE / "liboracle.so"
_REF = HERE / "_ref" / "libref_cpu.so"
_REF_CUDA = HERE / "_ref" / "libref_cuda.so"


def reference_dir():
    """The reference engine's source tree, or None: ENGINE_REF_DIR when set,
    else a checkout named ``reference`` beside this repository (it must hold
    src/cpu_ref).  Only build steps and fixture generators read it; nothing that
    runs on a GPU box does."""
    env = os.environ.get("ENGINE_REF_DIR")
    cand = Path(env) if env else HERE.parent.parent / "reference"
    return cand if (cand / "src" / "cpu_ref").is_dir() else None

_i64 = ctypes.c_int64
_p = ctypes.c_void_p
_f = ctypes.c_float
_i = ctypes.c_int


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _load_oracle():
    if not _LIB.exists() or _LIB.stat().st_mtime < (HERE / "cpu_oracle.c").stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(HERE), "all"], check=True)
    lib = ctypes.CDLL(str(_LIB))
    sig = {
        "orc_f32_to_f16": (ctypes.c_uint16, [_f]),
        "orc_f16_to_f32": (_f, [ctypes.c_uint16]),
        "orc_f32_to_bf16": (ctypes.c_uint16, [_f]),
        "orc_f32_to_f16_array": (None, [_p, _p, _i64]),
        "orc_f16_to_f32_array": (None, [_p, _p, _i64]),
        "orc_matmul": (None, [_p, _p, _p, _i64, _i64, _i64]),
        "orc_matmul_mt": (None, [_p, _p, _p, _i64, _i64, _i64, _i]),
        "orc_gemv": (None, [_p, _p, _p, _i64, _i64]),
        "orc_gemv_fp16": (None, [_p, _p, _p, _i64, _i64]),
        "orc_rmsnorm": (None, [_p, _p, _p, _i64, _i64, _f]),
        "orc_residual_rmsnorm": (None, [_p, _p, _p, _p, _p, _i64, _i64, _f]),
        "orc_attention": (_i, [_p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _f, _i64, _i, _p]),
        "orc_attention_online": (_i, [_p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _f, _i64, _i, _p]),
        "orc_rmsnorm_linear": (None, [_p, _p, _p, _p, _i64, _i64, _i64, _f]),
        "orc_rmsnorm_linear_mt": (None, [_p, _p, _p, _p, _i64, _i64, _i64, _f, _i]),
        "orc_vector_add": (None, [_p, _p, _p, _i64]),
        "orc_linear_f16": (None, [_p, _p, _p, _p, _i64, _i64, _i64, _i, _p]),
        "orc_linear_f16_mt": (None, [_p, _p, _p, _p, _i64, _i64, _i64, _i, _p, _i]),
        "orc_matmul_f16": (None, [_p, _p, _p, _p, _i64, _i64, _i64, _i]),
        "orc_matmul_f16_mt": (None, [_p, _p, _p, _p, _i64, _i64, _i64, _i, _i]),
        "orc_rmsnorm_linear_f16": (None, [_p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _f]),
        "orc_rmsnorm_linear_f16_mt": (None, [_p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _f, _i]),
        "orc_swiglu_f16": (None, [_p, _p, _p, _i64]),
        "orc_dequant_q": (None, [_i, _p, _p, _i64, _i64]),
        "orc_gemv_q": (None, [_i, _p, _p, _p, _p, _p, _i64, _i64]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


_lib = None


def lib():
    global _lib
    if _lib is None:
        _lib = _load_oracle()
    return _lib


def ref_available() -> bool:
    return _REF.exists()


_ref = None


def ref_lib():
    """The reference's own compiled cpu_ref (raises if it was never built)."""
    global _ref
    if _ref is None:
        if not _REF.exists():
            raise FileNotFoundError(f"{_REF} not built (make -C oracle ref)")
        r = ctypes.CDLL(str(_REF))
        sig = {
            "ref_abi_half_bytes": (_i, []),
            "ref_matmul": (None, [_p, _p, _p, _i64, _i64, _i64, _i]),
            "ref_gemv": (None, [_p, _p, _p, _i64, _i64]),
            "ref_gemv_fp16": (None, [_p, _p, _p, _i64, _i64]),
            "ref_rmsnorm": (None, [_p, _p, _p, _i64, _i64, _f]),
            "ref_residual_rmsnorm": (None, [_p, _p, _p, _p, _p, _i64, _i64, _f]),
            "ref_attention": (_i, [_p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _f, _i64, _i, _p]),
            "ref_attention_online": (_i, [_p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _f, _i64, _i, _p]),
            "ref_rmsnorm_linear": (None, [_p, _p, _p, _p, _i64, _i64, _i64, _f, _i]),
            "ref_swiglu_fp16": (None, [_p, _p, _p, _i64]),
            "ref_vector_add": (None, [_p, _p, _p, _i64]),
            "ref_matmul_f16_as_f32": (None, [_p, _p, _p, _i64, _i64, _i64, _i, _i]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(r, name)
            fn.restype = res
            fn.argtypes = args
        _ref = r
    return _ref


_refcuda = None


def ref_cuda_available() -> bool:
    return _REF_CUDA.exists()


def ref_cuda_lib():
    """The reference's own CUDA launchers built for sm_100a (raises if never built)."""
    global _refcuda
    if _refcuda is None:
        if not _REF_CUDA.exists():
            raise FileNotFoundError(f"{_REF_CUDA} not built (make -C oracle refcuda)")
        r = ctypes.CDLL(str(_REF_CUDA))
        sig = {
            "refcuda_matmul_register_tiled": [_p, _p, _p, _i64, _i64, _i64, _p],
            "refcuda_matmul_tiled": [_p, _p, _p, _i64, _i64, _i64, _p],
            "refcuda_gemv": [_p, _p, _p, _i64, _i64, _p],
            "refcuda_gemv_fp16": [_p, _p, _p, _i64, _i64, _p],
            "refcuda_rmsnorm_linear": [_p, _p, _p, _p, _i64, _i64, _i64, _f, _p],
        }
        for name, args in sig.items():
            fn = getattr(r, name)
            fn.restype = _i
            fn.argtypes = args
        _refcuda = r
    return _refcuda


def ncores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


# ----------------------------------------------------------------- conversions

def f16_bits(a: np.ndarray) -> np.ndarray:
    """numpy float16 array -> uint16 bit view (no copy when already contiguous)."""
    return np.ascontiguousarray(a, dtype=np.float16).view(np.uint16)


def to_f16(a: np.ndarray) -> np.ndarray:
    """float32 -> float16 through the oracle's own round-to-nearest-even."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    out = np.empty(a.shape, dtype=np.uint16)
    lib().orc_f32_to_f16_array(_ptr(a), _ptr(out), a.size)
    return out.view(np.float16)


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


# ------------------------------------------------------------------ FP32 forms

def matmul(A, B, nthreads: int = 1):
    A, B = _c(A, np.float32), _c(B, np.float32)
    M, K = A.shape
    N = B.shape[1]
    C = np.empty((M, N), np.float32)
    lib().orc_matmul_mt(_ptr(A), _ptr(B), _ptr(C), M, N, K, nthreads)
    return C


def gemv(A, x):
    A, x = _c(A, np.float32), _c(x, np.float32)
    K, N = A.shape
    out = np.empty(N, np.float32)
    lib().orc_gemv(_ptr(A), _ptr(x), _ptr(out), N, K)
    return out


def rmsnorm(x, w, eps):
    x = _c(x, np.float32)
    w = None if w is None else _c(w, np.float32)
    out = np.empty_like(x)
    rows, cols = x.shape
    lib().orc_rmsnorm(_ptr(x), _ptr(w), _ptr(out), rows, cols, eps)
    return out


def residual_rmsnorm(x, residual, w, eps):
    """(norm_out, sum_out) of src/cpu_ref/residual_rmsnorm_cpu.cpp:19-51."""
    x = _c(x, np.float32)
    residual = None if residual is None else _c(residual, np.float32)
    w = None if w is None else _c(w, np.float32)
    norm = np.empty_like(x)
    sm = np.empty_like(x)
    rows, cols = x.shape
    lib().orc_residual_rmsnorm(_ptr(x), _ptr(residual), _ptr(w), _ptr(norm), _ptr(sm), rows, cols, eps)
    return norm, sm


def rmsnorm_linear(x, w, W, eps, nthreads: int = 1):
    x, W = _c(x, np.float32), _c(W, np.float32)
    w = None if w is None else _c(w, np.float32)
    M, K = x.shape
    N = W.shape[1]
    out = np.empty((M, N), np.float32)
    lib().orc_rmsnorm_linear_mt(_ptr(x), _ptr(w), _ptr(W), _ptr(out), M, N, K, eps, nthreads)
    return out


def vector_add(a, b):
    a, b = _c(a, np.float32), _c(b, np.float32)
    out = np.empty_like(a)
    lib().orc_vector_add(_ptr(a), _ptr(b), _ptr(out), a.size)
    return out


# ------------------------------------------------------------- FP16/BF16 forms
# Arrays of dtype float16 are passed as binary16; BF16 data is passed as uint16
# bit patterns with bf16=True.

def _bits(a):
    if a is None:
        return None
    if a.dtype == np.float16:
        return np.ascontiguousarray(a).view(np.uint16)
    return _c(a, np.uint16)


def gemv_fp16(A, x):
    """out[N] = x[K] * A[K,N]; A, x float16 -> float16."""
    A, x = _bits(A), _bits(x)
    K, N = A.shape
    out = np.empty(N, np.uint16)
    lib().orc_gemv_fp16(_ptr(A), _ptr(x), _ptr(out), N, K)
    return out.view(np.float16)


def linear_f16(X, W, residual=None, bf16=False, nthreads: int = 1, want_f32=False):
    """Y[M,N] = X[M,K] * W[N,K]^T (+ residual) in the 16-bit type; FP64 accumulate."""
    X, W, R = _bits(X), _bits(W), _bits(residual)
    M, K = X.shape
    N = W.shape[0]
    Y = np.empty((M, N), np.uint16)
    Y32 = np.empty((M, N), np.float32) if want_f32 else None
    lib().orc_linear_f16_mt(_ptr(X), _ptr(W), _ptr(R), _ptr(Y), M, N, K, int(bf16), _ptr(Y32), nthreads)
    Y = Y if bf16 else Y.view(np.float16)
    return (Y, Y32) if want_f32 else Y


def matmul_f16(A, B, bf16=False, nthreads: int = 1, want_f32=False):
    """C[M,N] = A[M,K] * B[K,N] in the 16-bit type; FP64 accumulate."""
    A, B = _bits(A), _bits(B)
    M, K = A.shape
    N = B.shape[1]
    C = np.empty((M, N), np.uint16)
    C32 = np.empty((M, N), np.float32) if want_f32 else None
    lib().orc_matmul_f16_mt(_ptr(A), _ptr(B), _ptr(C), _ptr(C32), M, N, K, int(bf16), nthreads)
    C = C if bf16 else C.view(np.float16)
    return (C, C32) if want_f32 else C


def rmsnorm_linear_f16(x, gamma, W, eps, residual=None, nthreads: int = 1, want_f32=False):
    """Y[M,N] = rmsnorm(x)[M,K] * W[N,K]^T (+ residual); FP16 in/out."""
    x, g, W, R = _bits(x), _bits(gamma), _bits(W), _bits(residual)
    M, K = x.shape
    N = W.shape[0]
    Y = np.empty((M, N), np.uint16)
    Y32 = np.empty((M, N), np.float32) if want_f32 else None
    lib().orc_rmsnorm_linear_f16_mt(_ptr(x), _ptr(g), _ptr(W), _ptr(R), _ptr(Y), _ptr(Y32), M, N, K, eps, nthreads)
    return (Y.view(np.float16), Y32) if want_f32 else Y.view(np.float16)


def attention(q, k, v, scale, q_pos_offset=0, is_causal=True, ref=False, online=False):
    """(out, lse) of src/cpu_ref/attention_cpu.cpp:87-155 (online=True: the
    tiled online-softmax form, :159-244): q [s_q, n_heads, d], k / v
    [n_kv_heads, s_kv, d] FP16 -> out FP16 [s_q, n_heads, d], lse FP32
    [s_q, n_heads].  ref=True runs the reference's own compiled code instead."""
    q = _c(q, np.float16)
    k = _c(k, np.float16)
    v = _c(v, np.float16)
    s_q, n_heads, d = q.shape
    n_kv, s_kv, _ = k.shape
    out = np.empty_like(q)
    lse = np.empty((s_q, n_heads), np.float32)
    if online:
        fn = ref_lib().ref_attention_online if ref else lib().orc_attention_online
    else:
        fn = ref_lib().ref_attention if ref else lib().orc_attention
    rc = fn(_ptr(q), _ptr(k), _ptr(v), _ptr(out), s_q, s_kv, n_heads, n_kv, d, s_kv * d,
            float(scale), q_pos_offset, int(bool(is_causal)), _ptr(lse))
    if rc != 0:
        raise ValueError("attention: arguments break the contract")
    return out, lse


def swiglu_f16(gate, up):
    g, u = _bits(gate), _bits(up)
    out = np.empty(g.shape, np.uint16)
    lib().orc_swiglu_f16(_ptr(g), _ptr(u), _ptr(out), g.size)
    return out.view(np.float16)


# ---------------------------------------------------------- block-quantised

Q8_0, Q4_0 = 8, 4


def q_block_bytes(qtype: int) -> int:
    """Bytes of one 32-element block, FP16 scale included (34 for Q8_0, 18 for Q4_0)."""
    return 2 + (32 if qtype == Q8_0 else 16)


def dequant_q(qtype, blocks, N, K):
    """float32 W[N,K] from packed GGUF blocks (uint8 array of N*K/32 blocks)."""
    b = np.ascontiguousarray(blocks, dtype=np.uint8)
    w = np.empty((N, K), np.float32)
    lib().orc_dequant_q(int(qtype), _ptr(b), _ptr(w), N, K)
    return w


def gemv_q(qtype, blocks, x, residual=None, want_f32=False):
    """y[N] = W x (+ residual) for W as packed blocks; FP64 accumulation, FP16 out."""
    b = np.ascontiguousarray(blocks, dtype=np.uint8)
    x = _bits(x)
    R = _bits(residual)
    K = x.size
    N = b.size // (K // 32 * q_block_bytes(qtype))
    y = np.empty(N, np.uint16)
    y32 = np.empty(N, np.float32) if want_f32 else None
    lib().orc_gemv_q(int(qtype), _ptr(b), _ptr(x), _ptr(R), _ptr(y), _ptr(y32), N, K)
    y = y.view(np.float16)
    return (y, y32) if want_f32 else y


# ---------------------------------------------------------- derived bounds

def abs_dot_bound(A, B):
    """sum_k |a_ik| |b_kj| as float64 (the factor the derived tolerance scales)."""
    return np.abs(np.asarray(A, np.float64)) @ np.abs(np.asarray(B, np.float64))
