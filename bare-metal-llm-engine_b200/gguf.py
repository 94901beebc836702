"""GGUF model files through the library's memory-mapped reader (engine_gguf_*).

``GGUFFile(path)`` maps a GGUF v2/v3 file read-only and parses it in C++
(csrc/gguf.cpp): metadata, the tensor table, and every tensor's place in the
mapping, with every read bounds-checked (a malformed file raises EngineError
with code ENGINE_ERR_FORMAT).  ``data(name)`` is a zero-copy NumPy view of a
tensor's bytes; ``load(name)`` places a weight on the GPU in the layout the
projections read -- an [N, K] FP16/BF16/F32 tensor for linear / gemv, or the
(payload, scales) pair of ops.quant_repack for the Q8_0 / Q4_0 decode GEMV.
"""
from __future__ import annotations

import ctypes
from typing import NamedTuple

import numpy as np

from . import GgufTensorInfo, _check, lib

# GGML tensor types the device layouts cover (engine_b200.h ENGINE_GGML_*).
F32, F16, Q4_0, Q8_0, BF16 = 0, 1, 2, 8, 30
# GGUF metadata value types.
(UINT8, INT8, UINT16, INT16, UINT32, INT32, FLOAT32, BOOL, STRING, ARRAY, UINT64, INT64,
 FLOAT64) = range(13)

ERR_FORMAT, ERR_IO = 6, 7  # ENGINE_ERR_FORMAT / ENGINE_ERR_IO


def gemv_qtype(ggml_type: int) -> int:
    """The qtype ops.gemv_q / engine_cuda_gemv_q_nk take for a GGML block type
    (ENGINE_Q8_0 = 8, ENGINE_Q4_0 = 4)."""
    return {Q8_0: 8, Q4_0: 4}[ggml_type]


class Tensor(NamedTuple):
    index: int
    name: str
    type: int
    dims: tuple      # file order: dims[0] is the contiguous extent
    offset: int      # absolute byte offset in the file
    nbytes: int      # 0 for a GGML type the reader does not size

    @property
    def shape(self) -> tuple:
        """Row-major shape, outermost first (a [N, K] weight has dims (K, N))."""
        return tuple(reversed(self.dims))


class GGUFFile:
    def __init__(self, path):
        h = ctypes.c_void_p()
        _check(lib().engine_gguf_open(str(path).encode(), ctypes.byref(h)))
        self._h = h
        v, al = ctypes.c_int32(), ctypes.c_uint64()
        _check(lib().engine_gguf_version(h, ctypes.byref(v), ctypes.byref(al)))
        self.version, self.alignment = v.value, al.value
        n = ctypes.c_int64()
        _check(lib().engine_gguf_tensor_count(h, ctypes.byref(n)))
        self.tensors: list[Tensor] = []
        info = GgufTensorInfo()
        for i in range(n.value):
            _check(lib().engine_gguf_tensor(h, i, ctypes.byref(info)))
            self.tensors.append(Tensor(i, info.name.decode("utf-8", "replace"), info.type,
                                       tuple(info.dims[: info.n_dims]), info.offset, info.nbytes))
        self._by_name = {t.name: t for t in self.tensors}

    # ------------------------------------------------------------ lifetime
    def close(self) -> None:
        if self._h is not None:
            _check(lib().engine_gguf_close(self._h))
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ------------------------------------------------------------ metadata
    def metadata(self) -> dict:
        """key -> int | float | str, or ("array", element_type, count)."""
        n = ctypes.c_int64()
        _check(lib().engine_gguf_meta_count(self._h, ctypes.byref(n)))
        out = {}
        key, ty, et, cnt = ctypes.c_char_p(), ctypes.c_int32(), ctypes.c_int32(), ctypes.c_uint64()
        for i in range(n.value):
            _check(lib().engine_gguf_meta_entry(self._h, i, ctypes.byref(key), ctypes.byref(ty),
                                                ctypes.byref(et), ctypes.byref(cnt)))
            kb = key.value  # look up by the raw key bytes
            out[kb.decode("utf-8", "replace")] = (
                ("array", et.value, cnt.value) if ty.value == ARRAY else self.meta(kb))
        return out

    def meta(self, key):
        """One metadata value: int (integer types and bool), float or str."""
        kb = key if isinstance(key, bytes) else key.encode()
        iv, fv = ctypes.c_int64(), ctypes.c_double()
        if lib().engine_gguf_meta_int(self._h, kb, ctypes.byref(iv)) == 0:
            return iv.value
        if lib().engine_gguf_meta_float(self._h, kb, ctypes.byref(fv)) == 0:
            return fv.value
        sp, ln = ctypes.c_void_p(), ctypes.c_uint64()
        _check(lib().engine_gguf_meta_string(self._h, kb, ctypes.byref(sp), ctypes.byref(ln)))
        return ctypes.string_at(sp.value, ln.value).decode("utf-8", "replace") if ln.value else ""

    # ------------------------------------------------------------ tensors
    def tensor(self, name: str) -> Tensor:
        t = self._by_name.get(name)
        if t is None:  # let the library produce the error message
            idx = ctypes.c_int64()
            _check(lib().engine_gguf_find_tensor(self._h, name.encode(), ctypes.byref(idx)))
        return t

    def data(self, name: str) -> np.ndarray:
        """The tensor's bytes as a read-only uint8 view of the mapping (valid
        until close())."""
        t = self.tensor(name)
        info = GgufTensorInfo()
        _check(lib().engine_gguf_tensor(self._h, t.index, ctypes.byref(info)))
        if t.nbytes == 0:
            return np.empty(0, np.uint8)
        buf = (ctypes.c_uint8 * t.nbytes).from_address(info.data)
        a = np.frombuffer(buf, dtype=np.uint8)
        a.flags.writeable = False
        return a

    def load(self, name: str, device=None):
        """Places a weight on the GPU: an [N, K] (row-major, outermost first)
        torch tensor for F32/F16/BF16, or (payload, scales) for Q8_0/Q4_0."""
        import torch

        t = self.tensor(name)
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else device
        stream = torch.cuda.current_stream(dev).cuda_stream
        K = t.dims[0]
        rows = int(np.prod(t.dims[1:])) if len(t.dims) > 1 else 1
        if t.type in (F32, F16, BF16):
            dt = {F32: torch.float32, F16: torch.float16, BF16: torch.bfloat16}[t.type]
            out = torch.empty(t.shape, device=dev, dtype=dt)
            _check(lib().engine_gguf_load_tensor(self._h, t.index, out.data_ptr(), None, None,
                                                 stream))
            return out
        if t.type in (Q8_0, Q4_0):
            staging = torch.empty(t.nbytes, device=dev, dtype=torch.uint8)
            pay = torch.empty(rows, K if t.type == Q8_0 else K // 2, device=dev, dtype=torch.uint8)
            sc = torch.empty(rows, K // 32, device=dev, dtype=torch.float16)
            _check(lib().engine_gguf_load_tensor(self._h, t.index, pay.data_ptr(), sc.data_ptr(),
                                                 staging.data_ptr(), stream))
            torch.cuda.current_stream(dev).synchronize()  # staging is freed on return
            return pay, sc
        rc = lib().engine_gguf_load_tensor(self._h, t.index, None, None, None, stream)
        _check(rc)  # ENGINE_ERR_UNSUPPORTED with the type in the message
