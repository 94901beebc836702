"""CPU: the oracle's block-quantised weights (GGUF Q8_0 / Q4_0).

The engine declares these formats (include/engine/dtype.hpp:95-125) but has no
kernel, CPU path or golden data for them, so parity with the reference is
unpinned for this row.  Instead, the C oracle is checked against an independent
numpy restatement of the published format (tests/quant_np.py): the
dequantised weights bit for bit, and the GEMV against a float64 dot product.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from tests import quant_np as qn


@pytest.mark.parametrize("qtype", [qn.Q8_0, qn.Q4_0])
def test_block_sizes_match_the_declared_format(qtype):
    # dtype.hpp / tests/test_dtype.cpp:142-144: Q4_0 = 16 + 2 bytes, Q8_0 = 32 + 2.
    assert oracle.q_block_bytes(qtype) == qn.block_bytes(qtype) == (34 if qtype == 8 else 18)


@pytest.mark.parametrize("qtype", [qn.Q8_0, qn.Q4_0])
@pytest.mark.parametrize("N,K", [(3, 32), (17, 128), (64, 4096)])
def test_oracle_dequant_matches_numpy(qtype, N, K):
    rng = np.random.default_rng(N * K + qtype)
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    W[0, :32] = 0.0  # an all-zero block (scale 0)
    blocks = qn.quantize(qtype, W)
    assert blocks.size == N * K // 32 * qn.block_bytes(qtype)
    got = oracle.dequant_q(qtype, blocks, N, K)
    want = qn.dequantize(qtype, blocks, N, K)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    assert np.all(want[0, :32] == 0.0)


@pytest.mark.parametrize("qtype", [qn.Q8_0, qn.Q4_0])
def test_oracle_gemv_matches_float64_dot(qtype):
    N, K = 96, 1024
    rng = np.random.default_rng(7 + qtype)
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    x = rng.standard_normal(K).astype(np.float16)
    R = rng.standard_normal(N).astype(np.float16)
    blocks = qn.quantize(qtype, W)
    y, y32 = oracle.gemv_q(qtype, blocks, x, residual=R, want_f32=True)
    w = qn.dequantize(qtype, blocks, N, K).astype(np.float64)
    exact = w @ x.astype(np.float64) + R.astype(np.float64)
    np.testing.assert_allclose(y32, exact.astype(np.float32), rtol=1e-6, atol=1e-6)
    assert np.array_equal(y, y32.astype(np.float16))


# ------------------------------------------------ property: arbitrary blocks
from hypothesis import given, settings  # noqa: E402
from hypothesis import strategies as st  # noqa: E402


@settings(max_examples=80, deadline=None)
@given(qtype=st.sampled_from([qn.Q8_0, qn.Q4_0]), N=st.integers(1, 6), nblk=st.integers(1, 6),
       seed=st.integers(0, 2 ** 31), scale_kind=st.sampled_from(["normal", "tiny", "huge", "zero"]))
def test_property_arbitrary_blocks_dequantise_identically(qtype, N, nblk, seed, scale_kind):
    """Any payload bytes and any finite FP16 scale -- subnormal, the FP16
    maximum, zero -- dequantise bit for bit alike in the C oracle and the numpy
    restatement, and the FP64 GEMV equals a float64 dot product of them."""
    K = 32 * nblk
    rng = np.random.default_rng(seed)
    blocks = rng.integers(0, 256, N * nblk * qn.block_bytes(qtype), dtype=np.uint8)
    b = blocks.reshape(N, nblk, qn.block_bytes(qtype))
    d = {"normal": rng.standard_normal((N, nblk)) * 1e-2,
         "tiny": rng.uniform(-1, 1, (N, nblk)) * 6e-8,      # FP16 subnormals
         "huge": np.where(rng.random((N, nblk)) < 0.5, -65504.0, 65504.0),
         "zero": np.zeros((N, nblk))}[scale_kind].astype(np.float16)
    b[..., 0:2] = d.view(np.uint8).reshape(N, nblk, 2)
    got = oracle.dequant_q(qtype, blocks, N, K)
    want = qn.dequantize(qtype, blocks, N, K)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    x = rng.standard_normal(K).astype(np.float16)
    _, y32 = oracle.gemv_q(qtype, blocks, x, want_f32=True)
    exact = want.astype(np.float64) @ x.astype(np.float64)
    bound = 1e-12 * (np.abs(want.astype(np.float64)) @ np.abs(x.astype(np.float64))) + 1e-30
    assert np.all(np.abs(y32.astype(np.float64) - exact.astype(np.float32).astype(np.float64))
                  <= np.abs(exact) * 2 ** -23 + bound), (y32, exact)
