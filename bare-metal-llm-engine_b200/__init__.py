"""B200-native matrix-multiply hot path for Parag63/bare-metal-llm-engine.

Python mirror of the engine's launch API (include/engine/kernels.hpp,
namespace engine::cuda) over the in-tree CUDA library ``libengine_b200.so``
(C ABI declared in ``include/engine_b200.h``):

* ``cuda`` -- one function per launcher with the reference's name, argument
  order and meaning: raw DEVICE pointers (ints), int64 dimensions and a trailing
  ``stream`` (0 = legacy default stream).  Failures raise :class:`EngineError`
  carrying the library's message, whose wording matches the reference's
  ENGINE_CHECK messages ("non-negative", "null", "eps").
* ``ops`` -- the same calls on torch CUDA tensors (device memory and streams
  come from torch; the arithmetic is the library's).
* ``tp`` -- the tensor-parallel layer set (one process per GPU) and the
  library's NVLink communicator.
* ``gguf`` -- the memory-mapped GGUF reader that places weights on the device
  for these kernels.

There is no CPU or library fallback: if the CUDA library is missing or fails
to load, importing this package raises.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libengine_b200.so"

__all__ = ["EngineError", "lib", "cuda", "ops", "gguf", "LIB_PATH", "EXPORTS", "build"]


class EngineError(RuntimeError):
    """Raised when a library call returns a nonzero status (engine::EngineError)."""

    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


class GgufTensorInfo(ctypes.Structure):
    """engine_gguf_tensor_t (include/engine_b200.h)."""
    _fields_ = [("name", ctypes.c_char_p), ("type", ctypes.c_int32), ("n_dims", ctypes.c_int32),
                ("dims", ctypes.c_int64 * 4), ("offset", ctypes.c_uint64),
                ("nbytes", ctypes.c_uint64), ("data", ctypes.c_void_p)]


# name -> (argtypes) ; every entry returns int status
_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_f = ctypes.c_float
_P = ctypes.POINTER
EXPORTS: dict[str, list] = {
    "engine_cuda_matmul_naive": [_p, _p, _p, _i64, _i64, _i64, _p],
    "engine_cuda_matmul_tiled": [_p, _p, _p, _i64, _i64, _i64, _p],
    "engine_cuda_matmul_register_tiled": [_p, _p, _p, _i64, _i64, _i64, _p],
    "engine_cuda_gemv": [_p, _p, _p, _i64, _i64, _p],
    "engine_cuda_gemv_fp16": [_p, _p, _p, _i64, _i64, _p],
    "engine_cuda_rmsnorm": [_p, _p, _p, _i64, _i64, _f, _p],
    "engine_cuda_residual_rmsnorm": [_p, _p, _p, _p, _p, _i64, _i64, _f, _p],
    "engine_cuda_rmsnorm_linear": [_p, _p, _p, _p, _i64, _i64, _i64, _f, _p],
    "engine_cuda_rmsnorm_linear_fused_direct": [_p, _p, _p, _p, _i64, _i64, _i64, _f, _p],
    "engine_cuda_vector_add": [_p, _p, _p, _i64, _p],
    "engine_cuda_matmul_f16": [_p, _p, _p, _i64, _i64, _i64, _p],
    "engine_cuda_matmul_bf16": [_p, _p, _p, _i64, _i64, _i64, _p],
    "engine_cuda_linear_f16": [_p, _p, _p, _p, _i64, _i64, _i64, _p],
    "engine_cuda_linear_bf16": [_p, _p, _p, _p, _i64, _i64, _i64, _p],
    "engine_cuda_gemv_f16_nk": [_p, _p, _p, _p, _i64, _i64, _p],
    "engine_cuda_rmsnorm_linear_f16": [_p, _p, _p, _p, _p, _i64, _i64, _i64, _f, _p],
    "engine_cuda_rmsnorm_linear_f16_noalloc": [_p, _p, _p, _p, _p, _i64, _i64, _i64, _f, _p],
    "engine_cuda_swiglu_f16": [_p, _p, _p, _i64, _p],
    "engine_cuda_rmsnorm_linear_swiglu_f16": [_p, _p, _p, _p, _i64, _i64, _i64, _f, _p],
    "engine_cuda_embedding_f16": [_p, _p, _p, _i64, _i64, _i64, _p],
    "engine_cuda_quant_repack": [ctypes.c_int, _p, _p, _p, _i64, _i64, _p],
    "engine_cuda_gemv_q_nk": [ctypes.c_int, _p, _p, _p, _p, _p, _i64, _i64, _p],
    "engine_tp_comm_create": [ctypes.c_int, ctypes.c_int, _i64, ctypes.POINTER(ctypes.c_void_p)],
    "engine_cuda_attention_prefill": [_p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _f, _i64,
                                      ctypes.c_int, _p, _p],
    "engine_cuda_attention_decode": [_p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _f, ctypes.c_int,
                                     _p],
    "engine_cuda_kv_cache_write": [_p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _p],
    "engine_cuda_kv_cache_write_rows": [_p, _p, _i64, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64,
                                        _p],
    "engine_cuda_rmsnorm_linear_kv_f16": [_p, _p, _p, _p, _p, _i64, _i64, _f, _p, _p, _i64, _i64,
                                          _i64, _i64, _i64, _p],
    "engine_gguf_open": [ctypes.c_char_p, _P(ctypes.c_void_p)],
    "engine_gguf_close": [_p],
    "engine_gguf_version": [_p, _P(ctypes.c_int32), _P(ctypes.c_uint64)],
    "engine_gguf_tensor_count": [_p, _P(ctypes.c_int64)],
    "engine_gguf_tensor": [_p, _i64, _P(GgufTensorInfo)],
    "engine_gguf_find_tensor": [_p, ctypes.c_char_p, _P(ctypes.c_int64)],
    "engine_gguf_meta_count": [_p, _P(ctypes.c_int64)],
    "engine_gguf_meta_entry": [_p, _i64, _P(ctypes.c_char_p), _P(ctypes.c_int32),
                               _P(ctypes.c_int32), _P(ctypes.c_uint64)],
    "engine_gguf_meta_int": [_p, ctypes.c_char_p, _P(ctypes.c_int64)],
    "engine_gguf_meta_float": [_p, ctypes.c_char_p, _P(ctypes.c_double)],
    "engine_gguf_meta_string": [_p, ctypes.c_char_p, _P(ctypes.c_void_p), _P(ctypes.c_uint64)],
    "engine_gguf_load_tensor": [_p, _i64, _p, _p, _p, _p],
    "engine_tp_comm_handle": [_p, _p],
    "engine_tp_comm_open": [_p, _p],
    "engine_tp_comm_destroy": [_p],
    "engine_tp_allreduce_f16": [_p, _p, _p, _p, _i64, _p],
    "engine_tp_linear_allreduce_f16": [_p, _p, _p, _p, _p, _i64, _i64, _i64, _p],
}

_lib = None


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile libengine_b200.so in-tree (nvcc, sm_100a)."""
    import importlib.util

    spec = importlib.util.spec_from_file_location("_bmle_b200_build", HERE / "build.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.build(force=force, verbose=verbose)


def lib() -> ctypes.CDLL:
    """The loaded CUDA library (built on first use if absent)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists() and os.environ.get("ENGINE_B200_NO_AUTOBUILD") != "1":
        build()
    if not LIB_PATH.exists():
        raise ImportError(f"{LIB_PATH} is missing: run bare-metal-llm-engine_b200/build.py")
    h = ctypes.CDLL(str(LIB_PATH))
    h.engine_last_error.restype = ctypes.c_char_p
    h.engine_last_error.argtypes = []
    h.engine_abi_version.restype = ctypes.c_int
    h.engine_device_status.restype = ctypes.c_int
    h.engine_device_status.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_uint)]
    for name, args in EXPORTS.items():
        fn = getattr(h, name)
        fn.restype = ctypes.c_int
        fn.argtypes = args
    _lib = h
    return h


def _check(rc: int) -> None:
    if rc != 0:
        msg = lib().engine_last_error().decode("utf-8", "replace")
        raise EngineError(rc, msg)


def device_status(device: int = 0) -> int:
    """Reads and clears the device error word (1 = a kernel's bounded wait ran out)."""
    flags = ctypes.c_uint(0)
    _check(lib().engine_device_status(device, ctypes.byref(flags)))
    return int(flags.value)


from . import cuda, gguf, ops, tp  # noqa: E402  (after lib/_check are defined)
