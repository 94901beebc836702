"""GPU parity of the legacy launch API (FP32 matmul / gemv / rmsnorm_linear,
FP16 [K,N] gemv) through the C ABI, mirroring the reference's hot-path tests
(tests/test_kernels.cu:735-1431) on the reference's own golden vectors, plus
the derived per-element bound against the oracle.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from tests import bounds
from tests.golden import golden

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

K_MATMUL_RTOL, K_MATMUL_ATOL = 1e-4, 5e-5  # test_kernels.cu:171-172
EPS = 1e-5


# Device copies made by dev_t stay alive until the test ends: the library is
# handed raw pointers, so a temporary tensor must not be freed (and its memory
# reused) before the call has run.
_KEEP: list = []


@pytest.fixture(autouse=True)
def _keep_device_tensors_alive():
    yield
    _KEEP.clear()


def dev_t(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    t = t.cuda()
    _KEEP.append(t)
    return t


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def close(got, exp, rtol, atol, what):
    np.testing.assert_allclose(np.asarray(got, np.float64), np.asarray(exp, np.float64), rtol=rtol,
                               atol=atol, err_msg=what)


MATMULS = ["matmul_naive", "matmul_tiled", "matmul_register_tiled"]


@pytest.mark.parametrize("fn", MATMULS)
@pytest.mark.parametrize("stem", golden.stems("matmul__"))
def test_matmul_matches_reference(pkg, dev, fn, stem):
    g = golden.load(stem)
    M, K = g["A"].shape
    N = g["B"].shape[1]
    A, B = dev_t(g["A"]), dev_t(g["B"])
    C = torch.zeros(M, N, device=dev)
    getattr(pkg.cuda, fn)(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K)
    out = host(C)
    close(out, g["expected"], K_MATMUL_RTOL, K_MATMUL_ATOL, stem)
    exact = oracle.matmul(g["A"], g["B"])
    bounds.check(out, exact, bounds.fp32_dot_bound(K, oracle.abs_dot_bound(g["A"], g["B"]), exact),
                 stem)


@pytest.mark.parametrize("stem", golden.stems("matmul__"))
def test_matmul_variants_agree(pkg, dev, stem):
    """tiled / register_tiled vs naive near-exactly (test_kernels.cu:792, :853)."""
    g = golden.load(stem)
    M, K = g["A"].shape
    N = g["B"].shape[1]
    A, B = dev_t(g["A"]), dev_t(g["B"])
    outs = []
    for fn in MATMULS:
        C = torch.zeros(M, N, device=dev)
        getattr(pkg.cuda, fn)(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K)
        outs.append(host(C))
    for o in outs[1:]:
        close(o, outs[0], 1e-6, 1e-6, stem)


@pytest.mark.parametrize("M,N,K", [(3, 7, 11), (65, 137, 73), (129, 257, 65), (1, 65, 127),
                                   (71, 97, 113), (512, 512, 512), (1000, 40, 3000),
                                   (2, 2, 100000)])
def test_matmul_non_tile_multiples(pkg, dev, M, N, K):
    """test_kernels.cu:879-930 (same sin/cos inputs), plus split-K-heavy shapes."""
    sA = np.float32(1.0 / np.sqrt(np.float32(K)))
    hA = (np.sin((np.arange(M * K, dtype=np.float32) + 1) * np.float32(0.1)) * sA).reshape(M, K)
    hB = (np.cos((np.arange(K * N, dtype=np.float32) + 1) * np.float32(0.1)) * sA).reshape(K, N)
    hA, hB = hA.astype(np.float32), hB.astype(np.float32)
    exact = oracle.matmul(hA, hB, nthreads=8)
    C = torch.zeros(M, N, device=dev)
    pkg.cuda.matmul_register_tiled(dev_t(hA).data_ptr(), dev_t(hB).data_ptr(), C.data_ptr(), M, N, K)
    out = host(C)
    close(out, exact, K_MATMUL_RTOL, K_MATMUL_ATOL, f"{M}x{N}x{K}")
    bounds.check(out, exact, bounds.fp32_dot_bound(K, oracle.abs_dot_bound(hA, hB), exact))


def test_matmul_unaligned_pointers_use_scalar_path(pkg, dev):
    M, N, K = 33, 41, 57
    rng = np.random.default_rng(2)
    hA = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    hB = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    bufA = torch.zeros(M * K + 1, device=dev)
    bufB = torch.zeros(K * N + 1, device=dev)
    bufA[1:] = dev_t(hA).flatten()
    bufB[1:] = dev_t(hB).flatten()
    C = torch.zeros(M, N, device=dev)
    pkg.cuda.matmul_tiled(bufA.data_ptr() + 4, bufB.data_ptr() + 4, C.data_ptr(), M, N, K)
    exact = oracle.matmul(hA, hB)
    bounds.check(host(C), exact, bounds.fp32_dot_bound(K, oracle.abs_dot_bound(hA, hB), exact))


def test_matmul_with_k_zero_is_the_zero_matrix(pkg, dev):
    """test_kernels.cu:932: the output is zeroed over a poisoned buffer."""
    M, N = 4, 3
    d = torch.zeros(1, device=dev)
    for fn in MATMULS:
        C = torch.full((M, N), 7.0, device=dev)
        getattr(pkg.cuda, fn)(d.data_ptr(), d.data_ptr(), C.data_ptr(), M, N, 0)
        assert (host(C) == 0).all()


@pytest.mark.parametrize("stem", golden.stems("rmsnorm_linear__"))
@pytest.mark.parametrize("fn", ["rmsnorm_linear", "rmsnorm_linear_fused_direct"])
def test_rmsnorm_linear_matches_reference(pkg, dev, stem, fn):
    g = golden.load(stem)
    M, K = g["input"].shape
    N = g["W"].shape[1]
    w = g.get("weight")
    d_w = dev_t(w) if w is not None else None
    out = torch.zeros(M, N, device=dev)
    getattr(pkg.cuda, fn)(dev_t(g["input"]).data_ptr(), 0 if d_w is None else d_w.data_ptr(),
                          dev_t(g["W"]).data_ptr(), out.data_ptr(), M, N, K, EPS)
    got = host(out)
    close(got, g["expected"], K_MATMUL_RTOL, K_MATMUL_ATOL, stem)
    exact = oracle.rmsnorm_linear(g["input"], w, g["W"], EPS)
    t = oracle.rmsnorm(g["input"], w, EPS)
    # temp is bit-identical in the fused kernel, so only the dot product and the
    # 1-ulp float scale of the double-summed norm separate it from the oracle.
    absdot = oracle.abs_dot_bound(t, g["W"])
    bounds.check(got, exact, bounds.fp32_dot_bound(K, absdot, exact) + 2 * bounds.U32 * absdot, stem)


def test_rmsnorm_linear_null_weight_equals_unit_weight(pkg, dev):
    g = golden.load("rmsnorm_linear__32x256x512_now")
    M, N, K = 32, 256, 512
    x, W = dev_t(g["input"]), dev_t(g["W"])
    ones = torch.ones(K, device=dev)
    a = torch.zeros(M, N, device=dev)
    b = torch.zeros(M, N, device=dev)
    pkg.cuda.rmsnorm_linear(x.data_ptr(), 0, W.data_ptr(), a.data_ptr(), M, N, K, EPS)
    pkg.cuda.rmsnorm_linear(x.data_ptr(), ones.data_ptr(), W.data_ptr(), b.data_ptr(), M, N, K, EPS)
    close(host(a), host(b), 1e-6, 1e-6, "null vs ones")


@pytest.mark.parametrize("stem", golden.stems("rmsnorm_linear__"))
def test_rmsnorm_linear_agrees_with_separate_rmsnorm_and_matmul(pkg, dev, stem):
    g = golden.load(stem)
    M, K = g["input"].shape
    N = g["W"].shape[1]
    w = g.get("weight")
    d_w = dev_t(w) if w is not None else None
    x, W = dev_t(g["input"]), dev_t(g["W"])
    fused = torch.zeros(M, N, device=dev)
    temp = torch.zeros(M, K, device=dev)
    sep = torch.zeros(M, N, device=dev)
    wp = 0 if d_w is None else d_w.data_ptr()
    pkg.cuda.rmsnorm_linear(x.data_ptr(), wp, W.data_ptr(), fused.data_ptr(), M, N, K, EPS)
    pkg.cuda.rmsnorm(x.data_ptr(), wp, temp.data_ptr(), M, K, EPS)
    pkg.cuda.matmul_tiled(temp.data_ptr(), W.data_ptr(), sep.data_ptr(), M, N, K)
    close(host(fused), host(sep), 1e-4, 5e-5, stem)


@pytest.mark.parametrize("stem", golden.stems("rmsnorm__"))
def test_rmsnorm_matches_reference(pkg, dev, stem):
    g = golden.load(stem)
    rows, cols = g["input"].shape
    w = g.get("weight")
    d_w = dev_t(w) if w is not None else None
    out = torch.zeros(rows, cols, device=dev)
    pkg.cuda.rmsnorm(dev_t(g["input"]).data_ptr(), 0 if d_w is None else d_w.data_ptr(),
                     out.data_ptr(), rows, cols, EPS)
    got = host(out)
    close(got, g["expected"], 1e-5, 1e-6, stem)  # kRmsRtol / kRmsAtol
    assert not np.isnan(got).any()
    # The scale is formed exactly as the oracle forms it: bit-identical output.
    assert np.array_equal(got, oracle.rmsnorm(g["input"], w, EPS))


@pytest.mark.parametrize("stem", [s for s in golden.stems("residual_rmsnorm__") if not s.endswith("zeros")])
def test_residual_rmsnorm_matches_reference(pkg, dev, stem):
    """test_kernels.cu:972-1010: norm and sum against the reference's golden data,
    kRmsRtol / kRmsAtol; plus bit-identity with the oracle (same arithmetic)."""
    g = golden.load(stem)
    rows, cols = g["x"].shape
    w = g.get("weight")
    d_w = dev_t(w) if w is not None else None
    norm = torch.zeros(rows, cols, device=dev)
    sm = torch.zeros(rows, cols, device=dev)
    pkg.cuda.residual_rmsnorm(dev_t(g["x"]).data_ptr(), dev_t(g["residual"]).data_ptr(),
                              0 if d_w is None else d_w.data_ptr(), norm.data_ptr(),
                              sm.data_ptr(), rows, cols, EPS)
    got_norm, got_sum = host(norm), host(sm)
    close(got_norm, g["expected"], 1e-5, 1e-6, stem + " (norm)")
    close(got_sum, g["sum_out"], 1e-5, 1e-6, stem + " (sum)")
    o_norm, o_sum = oracle.residual_rmsnorm(g["x"], g["residual"], w, EPS)
    assert np.array_equal(got_sum, o_sum)
    assert np.array_equal(got_norm, o_norm)


def test_residual_rmsnorm_of_zeros_is_zeros_not_nan(pkg, dev):
    """test_kernels.cu:1012-1050: outputs pre-filled with NaN must become exact zeros."""
    g = golden.load("residual_rmsnorm__zeros")
    rows, cols = 2, 256
    norm = torch.full((rows, cols), float("nan"), device=dev)
    sm = torch.full((rows, cols), float("nan"), device=dev)
    pkg.cuda.residual_rmsnorm(dev_t(g["x"]).data_ptr(), dev_t(g["residual"]).data_ptr(), 0,
                              norm.data_ptr(), sm.data_ptr(), rows, cols, EPS)
    assert np.array_equal(host(norm), np.zeros((rows, cols), np.float32))
    assert np.array_equal(host(sm), np.zeros((rows, cols), np.float32))


def test_residual_rmsnorm_null_weight_equals_unit_weight(pkg, dev):
    """test_kernels.cu:1052-1085 (kAddRtol = kAddAtol = 0: bit-identical)."""
    g = golden.load("residual_rmsnorm__32x4096_now")
    rows, cols = 32, 4096
    x, r = dev_t(g["x"]), dev_t(g["residual"])
    ones = dev_t(np.ones(cols, np.float32))
    outs = []
    for wp in (0, ones.data_ptr()):
        norm = torch.empty(rows, cols, device=dev)
        sm = torch.empty(rows, cols, device=dev)
        pkg.cuda.residual_rmsnorm(x.data_ptr(), r.data_ptr(), wp, norm.data_ptr(), sm.data_ptr(),
                                  rows, cols, EPS)
        outs.append((host(norm), host(sm)))
    assert np.array_equal(outs[0][0], outs[1][0])
    assert np.array_equal(outs[0][1], outs[1][1])


def test_rmsnorm_linear_multi_stream(pkg, dev):
    """test_kernels.cu:1197: M=32 and M=1 calls interleaved on two streams."""
    K = N = 512
    s_a, s_b = torch.cuda.Stream(), torch.cuda.Stream()
    runs = []
    for i in range(6):
        M = 32 if i % 2 == 0 else 1
        seed = np.float32((i + 1) * 1.37)
        x = np.sin(seed + np.arange(M * K, dtype=np.float32) * np.float32(0.013)).reshape(M, K)
        w = (np.float32(0.75) + np.float32(0.25) * np.cos(seed + np.arange(K, dtype=np.float32) * np.float32(0.031)))
        W = (np.float32(0.05) * np.cos(seed * np.float32(1.7) + np.arange(K * N, dtype=np.float32) * np.float32(0.007))).reshape(K, N)
        x, w, W = x.astype(np.float32), w.astype(np.float32), W.astype(np.float32)
        exp = oracle.rmsnorm_linear(x, w, W, EPS)
        runs.append((M, dev_t(x), dev_t(w), dev_t(W), torch.zeros(M, N, device=dev), exp))
    torch.cuda.synchronize()
    for i, (M, x, w, W, out, _) in enumerate(runs):
        s = s_a if i % 2 == 0 else s_b
        pkg.cuda.rmsnorm_linear(x.data_ptr(), w.data_ptr(), W.data_ptr(), out.data_ptr(), M, N, K,
                                EPS, s.cuda_stream)
    s_a.synchronize()
    s_b.synchronize()
    for i, (M, x, w, W, out, exp) in enumerate(runs):
        close(host(out), exp, K_MATMUL_RTOL, K_MATMUL_ATOL, f"multi-stream #{i}")


@pytest.mark.parametrize("stem", golden.stems("gemv__"))
def test_gemv_matches_reference(pkg, dev, stem):
    g = golden.load(stem)
    K, N = g["A"].shape
    out = torch.zeros(N, device=dev)
    pkg.cuda.gemv(dev_t(g["A"]).data_ptr(), dev_t(g["x"]).data_ptr(), out.data_ptr(), N, K)
    got = host(out)
    close(got, g["expected"], K_MATMUL_RTOL, K_MATMUL_ATOL, stem)
    exact = oracle.gemv(g["A"], g["x"])
    bounds.check(got, exact, bounds.fp32_dot_bound(K, oracle.abs_dot_bound(g["x"][None], g["A"])[0], exact))


@pytest.mark.parametrize("stem", golden.stems("gemv__"))
def test_gemv_agrees_with_matmul_at_m1(pkg, dev, stem):
    g = golden.load(stem)
    K, N = g["A"].shape
    A, x = dev_t(g["A"]), dev_t(g["x"])
    a = torch.zeros(N, device=dev)
    b = torch.zeros(N, device=dev)
    pkg.cuda.gemv(A.data_ptr(), x.data_ptr(), a.data_ptr(), N, K)
    pkg.cuda.matmul_naive(x.data_ptr(), A.data_ptr(), b.data_ptr(), 1, N, K)
    close(host(a), host(b), K_MATMUL_RTOL, K_MATMUL_ATOL, stem)


def test_gemv_of_zero_input(pkg, dev):
    N, K = 64, 128
    out = torch.full((N,), 3.0, device=dev)
    pkg.cuda.gemv(torch.ones(K, N, device=dev).data_ptr(), torch.zeros(K, device=dev).data_ptr(),
                  out.data_ptr(), N, K)
    assert (host(out) == 0).all()


def test_gemv_and_gemv_fp16_with_k_zero_zero_output(pkg, dev):
    N = 13
    d = torch.zeros(1, device=dev)
    out = torch.full((N,), 7.0, device=dev)
    pkg.cuda.gemv(d.data_ptr(), d.data_ptr(), out.data_ptr(), N, 0)
    assert (host(out) == 0).all()
    dh = torch.zeros(1, device=dev, dtype=torch.float16)
    outh = torch.full((N,), 7.0, device=dev, dtype=torch.float16)
    pkg.cuda.gemv_fp16(dh.data_ptr(), dh.data_ptr(), outh.data_ptr(), N, 0)
    assert (host(outh) == 0).all()


@pytest.mark.parametrize("stem", golden.stems("gemv_fp16__"))
def test_gemv_fp16_matches_reference(pkg, dev, stem):
    g = golden.load(stem)
    K, N = g["A"].shape
    A16 = g["A"].astype(np.float16)
    x16 = g["x"].astype(np.float16)
    out = torch.zeros(N, device=dev, dtype=torch.float16)
    pkg.cuda.gemv_fp16(dev_t(A16).data_ptr(), dev_t(x16).data_ptr(), out.data_ptr(), N, K)
    got = host(out).astype(np.float32)
    close(got, g["expected"], 2e-3, 2e-3, stem)  # test_kernels.cu:1429
    _, exact = oracle.linear_f16(x16[None], np.ascontiguousarray(A16.T), want_f32=True)
    absdot = oracle.abs_dot_bound(x16.astype(np.float32)[None], A16.astype(np.float32))
    bounds.check(got[None], exact, bounds.gemv16_bound(K, absdot, exact), stem)


@pytest.mark.parametrize("N,K", [(4096, 4096), (14336, 4096), (4096, 14336), (1000, 3000), (8, 24)])
def test_gemv_fp16_legacy_layout_full_sizes(pkg, dev, N, K):
    rng = np.random.default_rng(N + K)
    A16 = (rng.standard_normal((K, N)) * 0.02).astype(np.float16)
    x16 = rng.standard_normal(K).astype(np.float16)
    out = torch.zeros(N, device=dev, dtype=torch.float16)
    pkg.cuda.gemv_fp16(dev_t(A16).data_ptr(), dev_t(x16).data_ptr(), out.data_ptr(), N, K)
    got = host(out).astype(np.float32)
    _, exact = oracle.linear_f16(x16[None], np.ascontiguousarray(A16.T), want_f32=True, nthreads=8)
    absdot = oracle.abs_dot_bound(x16.astype(np.float32)[None], A16.astype(np.float32))
    bounds.check(got[None], exact, bounds.gemv16_bound(K, absdot, exact), f"{N}x{K}")


def test_vector_add_is_bit_exact(pkg, dev):
    rng = np.random.default_rng(4)
    for n in [1, 31, 32, 33, 255, 256, 257, 4096, 1 << 20]:
        a = rng.standard_normal(n).astype(np.float32)
        b = rng.standard_normal(n).astype(np.float32)
        out = torch.zeros(n, device=dev)
        pkg.cuda.vector_add(dev_t(a).data_ptr(), dev_t(b).data_ptr(), out.data_ptr(), n)
        assert np.array_equal(host(out), oracle.vector_add(a, b))
