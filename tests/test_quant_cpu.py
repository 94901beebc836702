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
