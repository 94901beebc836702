"""Writes GGUF files for the loader's tests: a restatement of the published
GGUF layout (version 3, little-endian).

  header   u32 magic "GGUF", u32 version, u64 tensor_count, u64 kv_count
  metadata { string key, u32 value_type, value } per entry; a string is
           { u64 length, bytes }, an array { u32 elem_type, u64 count, elements }
  tensors  { string name, u32 n_dims, u64 dims[n_dims] (innermost first),
           u32 ggml_type, u64 offset } per tensor
  data     padded to the alignment (general.alignment, default 32); each
           tensor at its offset, a multiple of the alignment

`raw` lets a test corrupt any part of the file after it is laid out.
"""
from __future__ import annotations

import struct

import numpy as np

UINT8, INT8, UINT16, INT16, UINT32, INT32, FLOAT32, BOOL, STRING, ARRAY, UINT64, INT64, FLOAT64 = range(13)
_SCALAR = {UINT8: "<B", INT8: "<b", UINT16: "<H", INT16: "<h", UINT32: "<I", INT32: "<i",
           FLOAT32: "<f", BOOL: "<?", UINT64: "<Q", INT64: "<q", FLOAT64: "<d"}
F32, F16, Q4_0, Q8_0, BF16 = 0, 1, 2, 8, 30


def _string(s) -> bytes:
    b = s.encode() if isinstance(s, str) else bytes(s)
    return struct.pack("<Q", len(b)) + b


def _value(vt: int, v) -> bytes:
    if vt in _SCALAR:
        return struct.pack(_SCALAR[vt], v)
    if vt == STRING:
        return _string(v)
    if vt == ARRAY:
        et, items = v
        out = struct.pack("<IQ", et, len(items))
        return out + b"".join(_value(et, x) for x in items)
    raise ValueError(vt)


def build(meta, tensors, alignment: int = 32, version: int = 3, magic: bytes = b"GGUF"):
    """meta: [(key, value_type, value)]; tensors: [(name, ggml_type, dims, bytes)]
    with dims innermost first.  Returns (file bytes, {name: data offset})."""
    head = magic + struct.pack("<IQQ", version, len(tensors), len(meta))
    kv = b"".join(_string(k) + struct.pack("<I", vt) + _value(vt, v) for k, vt, v in meta)
    rel, infos, blobs = 0, [], []
    offsets = {}
    for name, ty, dims, data in tensors:
        infos.append(_string(name) + struct.pack("<I", len(dims)) +
                     b"".join(struct.pack("<Q", d) for d in dims) + struct.pack("<IQ", ty, rel))
        offsets[name] = rel
        pad = (-len(data)) % alignment
        blobs.append(bytes(data) + b"\0" * pad)
        rel += len(data) + pad
    body = head + kv + b"".join(infos)
    start = (len(body) + alignment - 1) // alignment * alignment
    out = body + b"\0" * (start - len(body)) + b"".join(blobs)
    return out, {k: start + v for k, v in offsets.items()}


def f16_tensor(a: np.ndarray) -> bytes:
    return np.ascontiguousarray(a, dtype=np.float16).tobytes()
