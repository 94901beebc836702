"""TEST HELPER: numpy restatement of GGUF's Q8_0 / Q4_0 block formats (the ones
the engine declares in include/engine/dtype.hpp:95-125), independent of the C
oracle: quantise float weights into packed blocks, dequantise, and split packed
blocks into the (payload, scales) layout the CUDA GEMV streams."""
from __future__ import annotations

import numpy as np

Q8_0, Q4_0 = 8, 4


def block_bytes(qtype):
    return 2 + (32 if qtype == Q8_0 else 16)


def quantize(qtype, W):
    """W [N,K] float -> packed blocks, uint8 [N * K/32 * block_bytes].  Q8_0:
    d = max|w| / 127, q = rint(w / d).  Q4_0: d = (signed value of largest
    magnitude) / -8, q = clip(rint(w / d) + 8, 0, 15)."""
    N, K = W.shape
    blk = W.reshape(N, K // 32, 32).astype(np.float32)
    if qtype == Q8_0:
        d = (np.abs(blk).max(axis=2) / 127.0).astype(np.float16)
        df = d.astype(np.float32)[..., None]
        q = np.where(df > 0, np.rint(blk / np.where(df > 0, df, 1)), 0).clip(-127, 127).astype(np.int8)
        pay = q.view(np.uint8)
    else:
        idx = np.abs(blk).argmax(axis=2)
        mx = np.take_along_axis(blk, idx[..., None], axis=2)[..., 0]
        d = (mx / -8.0).astype(np.float16)
        df = d.astype(np.float32)[..., None]
        q = np.where(df != 0, np.rint(blk / np.where(df != 0, df, 1)) + 8, 8).clip(0, 15).astype(np.uint8)
        pay = (q[..., :16] | (q[..., 16:] << 4)).astype(np.uint8)
    out = np.empty((N, K // 32, block_bytes(qtype)), np.uint8)
    out[..., 0:2] = d.view(np.uint8).reshape(N, K // 32, 2)
    out[..., 2:] = pay
    return out.reshape(-1)


def split(qtype, blocks, N, K):
    """Packed blocks -> (payload [N, K or K/2] uint8, scales [N, K/32] float16)."""
    b = blocks.reshape(N, K // 32, block_bytes(qtype))
    d = np.ascontiguousarray(b[..., 0:2]).view(np.float16).reshape(N, K // 32)
    pay = np.ascontiguousarray(b[..., 2:]).reshape(N, -1)
    return pay, d


def dequantize(qtype, blocks, N, K):
    pay, d = split(qtype, blocks, N, K)
    df = d.astype(np.float32)
    if qtype == Q8_0:
        q = pay.view(np.int8).reshape(N, K // 32, 32).astype(np.float32)
    else:
        p = pay.reshape(N, K // 32, 16)
        q = np.concatenate([(p & 15).astype(np.float32) - 8, (p >> 4).astype(np.float32) - 8],
                           axis=2)
    return (q * df[..., None]).reshape(N, K).astype(np.float32)
