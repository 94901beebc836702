"""GPU: block-quantised decode GEMV (GGUF Q8_0 / Q4_0) through the C ABI.

engine_cuda_quant_repack must split packed blocks into (payload, scales) in
the streamed layout exactly as the numpy restatement (quant_np.split) does.
engine_cuda_gemv_q_nk must match the oracle's FP64 GEMV on the same blocks
within the derived bound for FP32 accumulation and one FP16 output rounding
(tests/bounds.py gemv16_bound, with sum |w||x| over the dequantised weights).
The shapes cover the K-split and whole-row warp paths (K <= 8192 and > 8192:
K = 32, 64, 4096, 8192 + 96, 14336, 65536 + 256), ragged N, several rows per
warp group past N, with and without a residual, an all-zero block, the
4096x14336 decode shape, and K = 0.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from tests import bounds
from tests import quant_np as qn

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _dev(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


@pytest.mark.parametrize("qtype", [qn.Q8_0, qn.Q4_0])
@pytest.mark.parametrize("N,K,resid", [(4096, 4096, False), (1000, 4096, True), (300, 14336, True),
                                       (64, 32, False), (5, 64, True), (4096, 14336, False),
                                       (33, 8192 + 96, True), (14336, 4096, True),
                                       (64, 65536 + 256, False)])
def test_gemv_q_matches_oracle(pkg, dev, qtype, N, K, resid):
    rng = np.random.default_rng(N + K + qtype)
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    W[N // 2, :32] = 0.0  # an all-zero block: scale 0
    x = rng.standard_normal(K).astype(np.float16)
    R = rng.standard_normal(N).astype(np.float16) if resid else None
    blocks = qn.quantize(qtype, W)
    q, d = pkg.ops.quant_repack(qtype, _dev(blocks, dev), N, K)
    pay, sc = qn.split(qtype, blocks, N, K)
    torch.cuda.synchronize()
    assert np.array_equal(q.cpu().numpy(), pay)
    assert np.array_equal(d.cpu().numpy().view(np.uint16), sc.view(np.uint16))
    y = pkg.ops.gemv_q(qtype, q, d, _dev(x, dev), residual=_dev(R, dev) if resid else None)
    _, exact = oracle.gemv_q(qtype, blocks, x, residual=R, want_f32=True)
    w = qn.dequantize(qtype, blocks, N, K).astype(np.float64)
    absdot = np.abs(w) @ np.abs(x.astype(np.float64))
    bound = bounds.gemv16_bound(K, absdot, exact)
    if resid:
        bound = bound + bounds.U16 * np.abs(exact)
    bounds.check(y.cpu().numpy().astype(np.float64), exact.astype(np.float64), bound,
                 f"gemv_q{qtype} {N}x{K}")


def test_gemv_q_deterministic_and_empty_k(pkg, dev):
    N, K = 2048, 4096
    rng = np.random.default_rng(11)
    blocks = qn.quantize(qn.Q8_0, (rng.standard_normal((N, K)) * 0.02).astype(np.float32))
    q, d = pkg.ops.quant_repack(qn.Q8_0, _dev(blocks, dev), N, K)
    x = _dev(rng.standard_normal(K).astype(np.float16), dev)
    y1 = pkg.ops.gemv_q(qn.Q8_0, q, d, x)
    y2 = pkg.ops.gemv_q(qn.Q8_0, q, d, x)
    assert torch.equal(y1, y2)
    # K = 0: y = residual (no blocks to read)
    R = _dev(rng.standard_normal(N).astype(np.float16), dev)
    y0 = torch.empty(N, device=dev, dtype=torch.float16)
    pkg.cuda.gemv_q_nk(qn.Q8_0, q.data_ptr(), d.data_ptr(), x.data_ptr(), R.data_ptr(),
                       y0.data_ptr(), N, 0)
    torch.cuda.synchronize()
    assert torch.equal(y0, R)
