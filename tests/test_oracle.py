"""CPU: pin the oracle (oracle/cpu_oracle.c) to the reference.

1. Against every hot-path golden vector the reference's own generator produces
   (tools/gen_reference.py, replayed and hash-checked by tests/golden/golden.py),
   with the reference's oracle-vs-golden tolerances (tests/test_cpu_ref.cpp:83-90:
   rtol 1e-5, atol 1e-6; gemv_fp16 2e-3 as test_kernels.cu:1429).
2. Bit-for-bit against the reference's own compiled cpu_ref (oracle/_ref, built
   from the reference sources by oracle/Makefile) on seeded random inputs,
   including the [N,K] forms against the reference fed the exact transpose.
3. The FP16 / BF16 conversions against numpy's IEEE round-to-nearest-even.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from tests.golden import golden

RTOL, ATOL = 1e-5, 1e-6
EPS = 1e-5


def _close(got, exp, rtol=RTOL, atol=ATOL):
    np.testing.assert_allclose(np.asarray(got, np.float64), np.asarray(exp, np.float64),
                               rtol=rtol, atol=atol)


@pytest.mark.parametrize("stem", golden.stems("matmul__"))
def test_oracle_matmul_matches_golden(stem):
    g = golden.load(stem)
    _close(oracle.matmul(g["A"], g["B"]), g["expected"])


@pytest.mark.parametrize("stem", golden.stems("gemv__"))
def test_oracle_gemv_matches_golden(stem):
    g = golden.load(stem)
    _close(oracle.gemv(g["A"], g["x"]), g["expected"])


@pytest.mark.parametrize("stem", golden.stems("gemv_fp16__"))
def test_oracle_gemv_fp16_matches_golden(stem):
    g = golden.load(stem)
    out = oracle.gemv_fp16(g["A"].astype(np.float16), g["x"].astype(np.float16))
    _close(out.astype(np.float32), g["expected"], 2e-3, 2e-3)


@pytest.mark.parametrize("stem", golden.stems("rmsnorm_linear__"))
def test_oracle_rmsnorm_linear_matches_golden(stem):
    g = golden.load(stem)
    out = oracle.rmsnorm_linear(g["input"], g.get("weight"), g["W"], EPS)
    _close(out, g["expected"], 1e-4, 5e-5)


@pytest.mark.parametrize("stem", golden.stems("rmsnorm__"))
def test_oracle_rmsnorm_matches_golden(stem):
    g = golden.load(stem)
    _close(oracle.rmsnorm(g["input"], g.get("weight"), EPS), g["expected"], 1e-5, 1e-6)


@pytest.mark.parametrize("stem", golden.stems("residual_rmsnorm__"))
def test_oracle_residual_rmsnorm_matches_golden(stem):
    g = golden.load(stem)
    norm, sm = oracle.residual_rmsnorm(g["x"], g["residual"], g.get("weight"), EPS)
    _close(norm, g["expected"], 1e-5, 1e-6)  # kRmsRtol / kRmsAtol, test_kernels.cu:141-142
    assert np.array_equal(sm, g["sum_out"])  # one float addition, exactly the reference's


def _attention_tol(s_kv):
    """test_kernels.cu:288-299 / test_cpu_ref.cpp:165-175: 2*eps16 relative and
    1.5*eps16 + 4*s_kv*u32 absolute on the output; 2e-5 (+ 4*s_kv*u32) on lse."""
    e16, u32 = 2.0 ** -10, 2.0 ** -23
    return (2 * e16, 1.5 * e16 + 4 * s_kv * u32), (2e-5, 2e-5 + 4 * s_kv * u32)


@pytest.mark.parametrize("stem", golden.stems("attention__"))
def test_oracle_attention_matches_golden(stem):
    g = golden.load(stem)
    s_kv, d = g["k"].shape[1], g["q"].shape[2]
    p = next(c for c in golden._meta()["cases"] if c["stem"] == stem)["params"]
    (rt, at), (lrt, lat) = _attention_tol(s_kv)
    for online in (False, True):
        out, lse = oracle.attention(g["q"], g["k"], g["v"],
                                    1.0 / np.float32(np.sqrt(np.float32(d))), p["q_pos_offset"],
                                    p["is_causal"], online=online)
        _close(out.astype(np.float32), g["expected"], rt, at)
        _close(lse, g["lse"], lrt, lat)


def test_golden_case_inventory():
    """Every hot-path case of the reference's generator is present."""
    assert len(golden.stems("matmul__")) == 5
    assert len(golden.stems("gemv__")) == 4
    assert len(golden.stems("gemv_fp16__")) == 4
    assert len(golden.stems("rmsnorm_linear__")) == 5
    assert len(golden.stems("rmsnorm__")) == 5
    assert len(golden.stems("residual_rmsnorm__")) == 5
    assert len(golden.stems("attention__")) == 10


# ------------------------------------------------------- vs the reference's own code

needs_ref = pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built")


def _p(a):
    return None if a is None else a.ctypes.data_as(__import__("ctypes").c_void_p)


@needs_ref
@pytest.mark.parametrize("M,N,K", [(1, 1, 1), (17, 23, 31), (64, 48, 200), (3, 129, 65)])
def test_oracle_matmul_bit_exact_vs_reference(M, N, K):
    rng = np.random.default_rng(M * 1000 + N * 10 + K)
    A = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    B = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    ref = np.empty((M, N), np.float32)
    oracle.ref_lib().ref_matmul(_p(A), _p(B), _p(ref), M, N, K, 2)
    assert np.array_equal(oracle.matmul(A, B, nthreads=3), ref)


@needs_ref
@pytest.mark.parametrize("with_w", [True, False])
def test_oracle_rmsnorm_linear_bit_exact_vs_reference(with_w):
    rng = np.random.default_rng(7)
    M, N, K = 5, 33, 70
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = (rng.standard_normal(K) * 0.1 + 1).astype(np.float32) if with_w else None
    W = rng.standard_normal((K, N)).astype(np.float32)
    ref = np.empty((M, N), np.float32)
    oracle.ref_lib().ref_rmsnorm_linear(_p(x), _p(w), _p(W), _p(ref), M, N, K, EPS, 2)
    assert np.array_equal(oracle.rmsnorm_linear(x, w, W, EPS), ref)
    out = np.empty((M, K), np.float32)
    oracle.ref_lib().ref_rmsnorm(_p(x), _p(w), _p(out), M, K, EPS)
    assert np.array_equal(oracle.rmsnorm(x, w, EPS), out)


@needs_ref
@pytest.mark.parametrize("with_w,with_res,with_sum", [(True, True, True), (False, True, True),
                                                      (True, False, True), (True, True, False)])
def test_oracle_residual_rmsnorm_bit_exact_vs_reference(with_w, with_res, with_sum):
    """residual, weight and sum_out may each be null in the CPU reference."""
    import ctypes
    rows, cols = 9, 333
    rng = np.random.default_rng(cols)
    x = rng.standard_normal((rows, cols)).astype(np.float32)
    res = rng.standard_normal((rows, cols)).astype(np.float32) if with_res else None
    w = (rng.standard_normal(cols) * 0.1 + 1).astype(np.float32) if with_w else None
    outs = []
    for fn in (oracle.lib().orc_residual_rmsnorm, oracle.ref_lib().ref_residual_rmsnorm):
        norm = np.full((rows, cols), np.nan, np.float32)
        sm = np.full((rows, cols), np.nan, np.float32) if with_sum else None
        fn(_p(x), _p(res), _p(w), _p(norm), _p(sm), ctypes.c_int64(rows), ctypes.c_int64(cols),
           ctypes.c_float(EPS))
        outs.append((norm, sm))
    assert np.array_equal(outs[0][0], outs[1][0])
    if with_sum:
        assert np.array_equal(outs[0][1], outs[1][1])


@needs_ref
@pytest.mark.parametrize("s_q,s_kv,h,h_kv,d,off,causal,amp", [
    (1, 1, 1, 1, 64, 0, True, 1.0), (17, 17, 8, 2, 64, 0, True, 1.0),
    (33, 65, 8, 2, 128, 32, True, 1.0), (1, 257, 32, 4, 64, 256, False, 1.0),
    (16, 32, 4, 4, 64, 0, True, 4.0), (7, 300, 4, 1, 128, 100, True, 8.0),
    (4, 0, 2, 1, 64, 0, True, 1.0)])
def test_oracle_attention_bit_exact_vs_reference(s_q, s_kv, h, h_kv, d, off, causal, amp):
    """src/cpu_ref/attention_cpu.cpp compiled in place: outputs and lse bit for
    bit, GQA, causal offsets, decode shapes and s_kv = 0 included."""
    rng = np.random.default_rng(s_q * 1000 + s_kv)
    q = (rng.standard_normal((s_q, h, d)) * amp).astype(np.float16)
    k = (rng.standard_normal((h_kv, s_kv, d)) * amp).astype(np.float16)
    v = rng.standard_normal((h_kv, s_kv, d)).astype(np.float16)
    scale = 1.0 / np.sqrt(d)
    for online in (False, True):  # :87-155 and the tiled online form :159-244
        a = oracle.attention(q, k, v, scale, off, causal, online=online)
        b = oracle.attention(q, k, v, scale, off, causal, ref=True, online=online)
        assert np.array_equal(a[0].view(np.uint16), b[0].view(np.uint16))
        assert np.array_equal(a[1], b[1])


@needs_ref
def test_oracle_attention_contract_matches_reference():
    q = np.zeros((2, 4, 96), np.float16)  # head_dim 96 is outside the contract
    k = np.zeros((2, 3, 96), np.float16)
    for ref in (False, True):
        with pytest.raises(ValueError):
            oracle.attention(q, k, k, 0.1, 0, True, ref=ref)
        with pytest.raises(ValueError):  # 3 heads over 2 KV heads
            oracle.attention(np.zeros((2, 3, 64), np.float16), np.zeros((2, 3, 64), np.float16),
                             np.zeros((2, 3, 64), np.float16), 0.1, 0, True, ref=ref)


@needs_ref
@pytest.mark.parametrize("N,K", [(64, 64), (73, 125), (256, 4096)])
def test_oracle_gemv_fp16_bit_exact_vs_reference(N, K):
    rng = np.random.default_rng(N + K)
    A = (rng.standard_normal((K, N)) / np.sqrt(K)).astype(np.float16)
    x = rng.standard_normal(K).astype(np.float16)
    ref = np.empty(N, np.uint16)
    oracle.ref_lib().ref_gemv_fp16(_p(A.view(np.uint16)), _p(x.view(np.uint16)), _p(ref), N, K)
    assert np.array_equal(oracle.gemv_fp16(A, x).view(np.uint16), ref)
    Af = np.ascontiguousarray(A.astype(np.float32))
    xf = np.ascontiguousarray(x.astype(np.float32))
    reff = np.empty(N, np.float32)
    oracle.ref_lib().ref_gemv(_p(Af), _p(xf), _p(reff), N, K)
    assert np.array_equal(oracle.gemv(Af, xf), reff)


@needs_ref
def test_oracle_nk_forms_equal_reference_on_transpose():
    """linear_f16 / matmul_f16 (FP32 pre-narrowing value) == cpu::matmul on W^T."""
    rng = np.random.default_rng(11)
    M, N, K = 7, 40, 96
    X = rng.standard_normal((M, K)).astype(np.float16)
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float16)
    ref = np.empty((M, N), np.float32)
    oracle.ref_lib().ref_matmul_f16_as_f32(_p(X.view(np.uint16)), _p(W.view(np.uint16)), _p(ref),
                                           M, N, K, 1, 2)
    _, y32 = oracle.linear_f16(X, W, want_f32=True)
    assert np.array_equal(y32, ref)
    B = np.ascontiguousarray(W.T)
    _, c32 = oracle.matmul_f16(X, B, want_f32=True)
    assert np.array_equal(c32, ref)


@needs_ref
def test_oracle_rmsnorm_linear_f16_equals_reference_on_widened_inputs():
    rng = np.random.default_rng(5)
    M, N, K = 3, 24, 80
    x = rng.standard_normal((M, K)).astype(np.float16)
    g = (1 + 0.1 * rng.standard_normal(K)).astype(np.float16)
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float16)
    xf = x.astype(np.float32)
    gf = g.astype(np.float32)
    Wt = np.ascontiguousarray(W.astype(np.float32).T)
    ref = np.empty((M, N), np.float32)
    oracle.ref_lib().ref_rmsnorm_linear(_p(xf), _p(gf), _p(Wt), _p(ref), M, N, K, EPS, 1)
    _, y32 = oracle.rmsnorm_linear_f16(x, g, W, EPS, want_f32=True)
    assert np.array_equal(y32, ref)


@needs_ref
def test_oracle_swiglu_f16_bit_exact_vs_reference():
    rng = np.random.default_rng(3)
    g = (3 * rng.standard_normal(4099)).astype(np.float16)
    u = rng.standard_normal(4099).astype(np.float16)
    ref = np.empty(4099, np.uint16)
    oracle.ref_lib().ref_swiglu_fp16(_p(g.view(np.uint16)), _p(u.view(np.uint16)), _p(ref), 4099)
    assert np.array_equal(oracle.swiglu_f16(g, u).view(np.uint16), ref)


# ------------------------------------------------------------------ conversions

def test_f16_conversion_matches_numpy_rne():
    rng = np.random.default_rng(0)
    vals = np.concatenate([
        rng.standard_normal(200000).astype(np.float32) * np.float32(3.0),
        (rng.standard_normal(50000) * 1e-5).astype(np.float32),   # subnormal halves
        (rng.standard_normal(50000) * 3e4).astype(np.float32),    # near overflow
        np.array([0.0, -0.0, 65504, 65519.99, 65520, -65520, 6.1e-5, 5.96e-8, 2.98e-8,
                  2.99e-8, np.inf, -np.inf, 1e-9], np.float32),
    ])
    ours = oracle.to_f16(vals).view(np.uint16)
    ref = vals.astype(np.float16).view(np.uint16)
    assert np.array_equal(ours, ref)
    back = np.empty(ours.size, np.float32)
    import ctypes
    oracle.lib().orc_f16_to_f32_array(ours.ctypes.data_as(ctypes.c_void_p),
                                      back.ctypes.data_as(ctypes.c_void_p), ours.size)
    assert np.array_equal(back, ref.view(np.float16).astype(np.float32))


def test_bf16_conversion_rne():
    rng = np.random.default_rng(1)
    vals = rng.standard_normal(100000).astype(np.float32)
    bits = vals.view(np.uint32)
    exp = ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16).astype(np.uint16)
    ours = np.array([oracle.lib().orc_f32_to_bf16(float(v)) for v in vals[:2000]], np.uint16)
    assert np.array_equal(ours, exp[:2000])


def test_multithreaded_oracle_is_bit_identical():
    rng = np.random.default_rng(9)
    A = rng.uniform(-1, 1, (37, 53)).astype(np.float32)
    B = rng.uniform(-1, 1, (53, 29)).astype(np.float32)
    assert np.array_equal(oracle.matmul(A, B, 1), oracle.matmul(A, B, 5))
    X = rng.standard_normal((9, 64)).astype(np.float16)
    W = rng.standard_normal((31, 64)).astype(np.float16)
    assert np.array_equal(oracle.linear_f16(X, W, nthreads=1), oracle.linear_f16(X, W, nthreads=4))


# ------------------------------------------- property-based pin, random shapes
from hypothesis import given, settings  # noqa: E402
from hypothesis import strategies as st  # noqa: E402

_dims = st.integers(1, 40)


def _arr(seed, shape, dtype=np.float32, scale=1.0):
    return (np.random.default_rng(seed).standard_normal(shape) * scale).astype(dtype)


@needs_ref
@settings(max_examples=60, deadline=None)
@given(M=_dims, N=_dims, K=st.integers(0, 40), seed=st.integers(0, 2 ** 31))
def test_property_matmul_and_gemv_fp16_bit_exact(M, N, K, seed):
    A, B = _arr(seed, (M, K)), _arr(seed + 1, (K, N))
    ref = np.empty((M, N), np.float32)
    oracle.ref_lib().ref_matmul(_p(A), _p(B), _p(ref), M, N, K, 1)
    assert np.array_equal(oracle.matmul(A, B), ref)
    if K > 0:
        Ah, xh = _arr(seed, (K, N), np.float16), _arr(seed + 2, K, np.float16)
        refh = np.empty(N, np.float16)
        oracle.ref_lib().ref_gemv_fp16(_p(Ah.view(np.uint16)), _p(xh.view(np.uint16)),
                                       _p(refh.view(np.uint16)), N, K)
        assert np.array_equal(oracle.gemv_fp16(Ah, xh).view(np.uint16), refh.view(np.uint16))


@needs_ref
@settings(max_examples=60, deadline=None)
@given(M=_dims, N=_dims, K=_dims, with_w=st.booleans(), seed=st.integers(0, 2 ** 31))
def test_property_rmsnorm_linear_and_residual_rmsnorm_bit_exact(M, N, K, with_w, seed):
    import ctypes

    x, W = _arr(seed, (M, K)), _arr(seed + 1, (K, N))
    w = (_arr(seed + 2, K) * 0.1 + 1).astype(np.float32) if with_w else None
    ref = np.empty((M, N), np.float32)
    oracle.ref_lib().ref_rmsnorm_linear(_p(x), _p(w), _p(W), _p(ref), M, N, K, EPS, 1)
    assert np.array_equal(oracle.rmsnorm_linear(x, w, W, EPS), ref)
    r = _arr(seed + 3, (M, K))
    norm, sm = oracle.residual_rmsnorm(x, r, w, EPS)
    rn, rs = np.empty_like(x), np.empty_like(x)
    oracle.ref_lib().ref_residual_rmsnorm(_p(x), _p(r), _p(w), _p(rn), _p(rs), ctypes.c_int64(M),
                                          ctypes.c_int64(K), ctypes.c_float(EPS))
    assert np.array_equal(norm, rn) and np.array_equal(sm, rs)


@needs_ref
@settings(max_examples=40, deadline=None)
@given(s_q=st.integers(0, 9), s_kv=st.integers(0, 40), h_kv=st.sampled_from([1, 2]),
       grp=st.sampled_from([1, 2, 4]), d=st.sampled_from([64, 128]), off=st.integers(0, 8),
       causal=st.booleans(), amp=st.sampled_from([0.5, 1.0, 6.0]), online=st.booleans(),
       seed=st.integers(0, 2 ** 31))
def test_property_attention_bit_exact(s_q, s_kv, h_kv, grp, d, off, causal, amp, online, seed):
    h = h_kv * grp
    q = _arr(seed, (s_q, h, d), np.float16, amp)
    k = _arr(seed + 1, (h_kv, s_kv, d), np.float16, amp)
    v = _arr(seed + 2, (h_kv, s_kv, d), np.float16)
    a = oracle.attention(q, k, v, d ** -0.5, off, causal, online=online)
    b = oracle.attention(q, k, v, d ** -0.5, off, causal, ref=True, online=online)
    assert np.array_equal(a[0].view(np.uint16), b[0].view(np.uint16))
    assert np.array_equal(a[1], b[1])
