"""GPU parity of the FP16/BF16 entry points (tcgen05 GEMM, swap-AB + split-K
skinny tiles, decode GEMV, fused RMSNorm->linear) through the C ABI.

Each output is compared element by element with the oracle (FP64 accumulation
of the widened 16-bit inputs, i.e. the reference's cpu::matmul /
cpu::rmsnorm_linear fed W^T) under the derived bounds of tests/bounds.py.  At
the BASELINE sizes (4096^3, 4096 x 14336, ...) a seeded sample of output rows is
checked exactly against the oracle run on those rows alone: the row-sampled
oracle is exact for every sampled element, and the sample covers every tile row
position and every column.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from tests import bounds

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
EPS = 1e-5


# Device copies made by dev_t stay alive until the test ends: the library is
# handed raw pointers, so a temporary tensor must not be freed (and its memory
# reused) before the call has run.
_KEEP: list = []


@pytest.fixture(autouse=True)
def _keep_device_tensors_alive():
    yield
    _KEEP.clear()


def dev_t(a):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:  # bfloat16 bit patterns: move as int16
        a = a.view(np.int16)
    t = torch.from_numpy(a).cuda()
    _KEEP.append(t)
    return t


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def f16(rng, shape, scale=1.0):
    return (rng.standard_normal(shape) * scale).astype(np.float16)


def bf16_bits(rng, shape, scale=1.0):
    x = (rng.standard_normal(shape) * scale).astype(np.float32)
    b = x.view(np.uint32)
    return ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)


def bf16_to_f32(bits):
    return (bits.astype(np.uint32) << 16).view(np.float32)


def sample_rows(M, n, seed=0):
    if M <= n:
        return np.arange(M)
    rng = np.random.default_rng(seed)
    rows = set(rng.choice(M, n - 4, replace=False).tolist()) | {0, 1, M - 2, M - 1}
    return np.array(sorted(rows))


def check_linear(got16, X, W, R, rows, bf16=False, what=""):
    """got16: device output [M,N] (16-bit); X [M,K], W [N,K] host 16-bit arrays."""
    Xs = X[rows]
    Rs = None if R is None else R[rows]
    _, exact = oracle.linear_f16(Xs, W, residual=Rs, bf16=bf16, want_f32=True, nthreads=8)
    g = host(got16)[rows]
    if bf16:
        g = bf16_to_f32(g.view(np.uint16))
        Xf, Wf = bf16_to_f32(Xs), bf16_to_f32(W)
    else:
        g = g.astype(np.float32)
        Xf, Wf = Xs.astype(np.float32), W.astype(np.float32)
    absdot = np.abs(Xf.astype(np.float64)) @ np.abs(Wf.astype(np.float64)).T
    K = X.shape[1]
    ou = bounds.UBF if bf16 else bounds.U16
    bound = bounds.tc_bound(K, absdot, exact, ou)
    if R is not None:
        bound = bound + ou * np.abs(exact)
    return bounds.check(g, exact, bound, what)


# ------------------------------------------------------------------ matmul (B[K,N])

@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 128), (200, 136, 72), (1, 8, 8),
                                   (300, 320, 1000), (129, 64, 4104), (17, 23, 31), (5, 7, 9)])
@pytest.mark.parametrize("dt", ["f16", "bf16"])
def test_matmul_16bit_matches_oracle(pkg, dev, M, N, K, dt):
    rng = np.random.default_rng(M * 7 + N * 3 + K)
    bf = dt == "bf16"
    A = bf16_bits(rng, (M, K)) if bf else f16(rng, (M, K))
    B = bf16_bits(rng, (K, N)) if bf else f16(rng, (K, N))
    C = torch.empty(M, N, device=dev, dtype=torch.bfloat16 if bf else torch.float16)
    fn = pkg.cuda.matmul_bf16 if bf else pkg.cuda.matmul_f16
    fn(dev_t(A).data_ptr(), dev_t(B).data_ptr(), C.data_ptr(), M, N, K)
    out = C.view(torch.int16) if bf else C
    W = np.ascontiguousarray(B.T)
    check_linear(out, A, W, None, np.arange(M), bf16=bf, what=f"{dt} {M}x{N}x{K}")


def test_matmul_f16_4096_cubed_sampled_rows(pkg, dev):
    """BASELINE config 4a: 4096^3 FP16 A, B ~ N(0,1)."""
    M = N = K = 4096
    g = torch.Generator(device="cuda").manual_seed(20260826)
    A = torch.randn(M, K, device=dev, generator=g).half()
    B = torch.randn(K, N, device=dev, generator=g).half()
    C = torch.empty(M, N, device=dev, dtype=torch.float16)
    pkg.cuda.matmul_f16(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K)
    rows = sample_rows(M, 48)
    check_linear(C, host(A), np.ascontiguousarray(host(B).T), None, rows, what="4096^3")


# Shapes whose 256 x 256 tile count leaves a partial last wave on 74 CTA pairs, so
# the 2-SM kernel splits the last tiles along K (stream-K) and the second pair
# to finish a shared tile adds the other's parked partial.  N % 8 != 0 turns
# the TMA-store epilogue off, so both epilogue paths do the fix-up.
@pytest.mark.parametrize("M,N,K,resid", [(2304, 2304, 512, False), (2300, 2310, 520, False),
                                         (2304, 2304, 1000, True)])
def test_linear_f16_stream_k_tiles(pkg, dev, M, N, K, resid):
    rng = np.random.default_rng(M + N + K)
    X = f16(rng, (M, K))
    W = f16(rng, (N, K), 0.05)
    R = f16(rng, (M, N)) if resid else None
    Y = torch.empty(M, N, device=dev, dtype=torch.float16)
    pkg.cuda.linear_f16(dev_t(X).data_ptr(), dev_t(W).data_ptr(),
                        dev_t(R).data_ptr() if resid else 0, Y.data_ptr(), M, N, K)
    check_linear(Y, X, W, R, np.arange(M), what=f"stream-K {M}x{N}x{K}")


def test_matmul_bf16_stream_k_tiles(pkg, dev):
    M, N, K = 2304, 2560, 640
    rng = np.random.default_rng(5)
    A = bf16_bits(rng, (M, K))
    B = bf16_bits(rng, (K, N))
    C = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
    pkg.cuda.matmul_bf16(dev_t(A).data_ptr(), dev_t(B).data_ptr(), C.data_ptr(), M, N, K)
    check_linear(C.view(torch.int16), A, np.ascontiguousarray(B.T), None, np.arange(M),
                 bf16=True, what="bf16 stream-K")


def test_matmul_f16_stream_k_deterministic_and_graph_replay(pkg, dev):
    """4096^3 runs stream-K on a full B200; repeated eager calls and CUDA graph
    replays of a captured call (the tile counters reset themselves) agree bit
    for bit."""
    M = N = K = 4096
    g = torch.Generator(device="cuda").manual_seed(3)
    A = torch.randn(M, K, device=dev, generator=g).half()
    B = torch.randn(K, N, device=dev, generator=g).half()
    C1 = torch.empty(M, N, device=dev, dtype=torch.float16)
    C2 = torch.empty_like(C1)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        pkg.cuda.matmul_f16(A.data_ptr(), B.data_ptr(), C1.data_ptr(), M, N, K, s.cuda_stream)
        pkg.cuda.matmul_f16(A.data_ptr(), B.data_ptr(), C2.data_ptr(), M, N, K, s.cuda_stream)
    torch.cuda.synchronize()
    assert torch.equal(C1, C2)
    C3 = torch.zeros_like(C1)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        pkg.cuda.matmul_f16(A.data_ptr(), B.data_ptr(), C3.data_ptr(), M, N, K, s.cuda_stream)
    for _ in range(3):
        C3.zero_()
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(C1, C3)
    del graph
    rows = sample_rows(M, 24, seed=3)
    check_linear(C1, host(A), np.ascontiguousarray(host(B).T), None, rows, what="4096^3 sk")


def test_matmul_f16_deterministic(pkg, dev):
    M = N = K = 1024
    g = torch.Generator(device="cuda").manual_seed(1)
    A = torch.randn(M, K, device=dev, generator=g).half()
    B = torch.randn(K, N, device=dev, generator=g).half()
    C1 = torch.empty(M, N, device=dev, dtype=torch.float16)
    C2 = torch.empty_like(C1)
    pkg.cuda.matmul_f16(A.data_ptr(), B.data_ptr(), C1.data_ptr(), M, N, K)
    pkg.cuda.matmul_f16(A.data_ptr(), B.data_ptr(), C2.data_ptr(), M, N, K)
    assert torch.equal(C1, C2)


# ------------------------------------------------------------------ linear (W[N,K])

@pytest.mark.parametrize("M", [1, 2, 3, 4, 5, 8, 16, 31, 32, 33, 64, 65, 128, 200])
@pytest.mark.parametrize("resid", [False, True])
def test_linear_f16_all_paths(pkg, dev, M, resid):
    N, K = 384, 512
    rng = np.random.default_rng(M + 100 * resid)
    X = f16(rng, (M, K))
    W = f16(rng, (N, K), 0.02)
    R = f16(rng, (M, N)) if resid else None
    Y = torch.empty(M, N, device=dev, dtype=torch.float16)
    pkg.cuda.linear_f16(dev_t(X).data_ptr(), dev_t(W).data_ptr(),
                        dev_t(R).data_ptr() if resid else 0, Y.data_ptr(), M, N, K)
    check_linear(Y, X, W, R, np.arange(M), what=f"linear M={M} resid={resid}")


@pytest.mark.parametrize("M", [1, 16, 100])
def test_linear_bf16(pkg, dev, M):
    N, K = 256, 384
    rng = np.random.default_rng(M)
    X = bf16_bits(rng, (M, K))
    W = bf16_bits(rng, (N, K), 0.02)
    R = bf16_bits(rng, (M, N))
    Y = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
    pkg.cuda.linear_bf16(dev_t(X).data_ptr(), dev_t(W).data_ptr(), dev_t(R).data_ptr(),
                         Y.data_ptr(), M, N, K)
    check_linear(Y.view(torch.int16), X, W, R, np.arange(M), bf16=True, what=f"bf16 M={M}")


@pytest.mark.parametrize("S", [512, 2048, 4096])
def test_linear_f16_prefill_config_sampled_rows(pkg, dev, S):
    """BASELINE config 4b: X[S,4096] ~ N(0,1) times W[14336,4096]^T ~ N(0,0.02)."""
    N, K = 14336, 4096
    g = torch.Generator(device="cuda").manual_seed(S)
    X = torch.randn(S, K, device=dev, generator=g).half()
    W = (torch.randn(N, K, device=dev, generator=g) * 0.02).half()
    Y = torch.empty(S, N, device=dev, dtype=torch.float16)
    pkg.cuda.linear_f16(X.data_ptr(), W.data_ptr(), 0, Y.data_ptr(), S, N, K)
    check_linear(Y, host(X), host(W), None, sample_rows(S, 24, S), what=f"S={S}")


def test_linear_unaligned_k_falls_back(pkg, dev):
    M, N, K = 37, 50, 131
    rng = np.random.default_rng(3)
    X, W = f16(rng, (M, K)), f16(rng, (N, K), 0.05)
    Y = torch.empty(M, N, device=dev, dtype=torch.float16)
    pkg.cuda.linear_f16(dev_t(X).data_ptr(), dev_t(W).data_ptr(), 0, Y.data_ptr(), M, N, K)
    check_linear(Y, X, W, None, np.arange(M), what="unaligned K")


# ------------------------------------------------------------------ decode GEMV (W[N,K])

@pytest.mark.parametrize("N,K", [(4096, 4096), (14336, 4096), (4096, 14336), (6144, 4096),
                                 (100, 8), (77, 4100), (1, 64)])
@pytest.mark.parametrize("resid", [False, True])
def test_gemv_f16_nk(pkg, dev, N, K, resid):
    """W ~ N(0,0.02), x ~ N(0,1)."""
    rng = np.random.default_rng(N * 3 + K + resid)
    W = f16(rng, (N, K), 0.02)
    x = f16(rng, (1, K))
    R = f16(rng, (1, N)) if resid else None
    y = torch.empty(N, device=dev, dtype=torch.float16)
    pkg.cuda.gemv_f16_nk(dev_t(W).data_ptr(), dev_t(x).data_ptr(),
                         dev_t(R).data_ptr() if resid else 0, y.data_ptr(), N, K)
    _, exact = oracle.linear_f16(x, W, residual=R, want_f32=True, nthreads=8)
    absdot = np.abs(x.astype(np.float64)) @ np.abs(W.astype(np.float64)).T
    bound = bounds.gemv16_bound(K, absdot, exact) + (bounds.U16 * np.abs(exact) if resid else 0)
    bounds.check(host(y).astype(np.float32)[None], exact, bound, f"gemv {N}x{K}")


# ------------------------------------------------------------------ fused RMSNorm -> linear

def rms_bound(M, K, absdot, exact):
    if M <= 4:       # CUDA cores: FP32 dot, scale from an FP32 sum of squares
        c = K + K / 64 + 16
    elif M <= 32:    # tcgen05 with hi/lo activations (~2^-22 relative)
        c = 2 * K + 8
    else:            # tcgen05 with the activation rounded once to FP16
        c = 2 * K + 8 + 2 ** 13
    return c * bounds.U32 * absdot + (bounds.U32 + bounds.U16) * np.abs(exact) + 2.0 ** -25


@pytest.mark.parametrize("M", [1, 2, 4, 5, 8, 16, 32, 33, 100])
@pytest.mark.parametrize("gamma", [True, False])
def test_rmsnorm_linear_f16(pkg, dev, M, gamma):
    """BASELINE config 3 (W[6144,4096], B in {1, 16}) and every dispatch path."""
    N, K = 6144, 4096
    rng = np.random.default_rng(M * 2 + gamma)
    x = f16(rng, (M, K))
    g = (1 + 0.1 * rng.standard_normal(K)).astype(np.float16) if gamma else None
    W = f16(rng, (N, K), 0.02)
    Y = torch.empty(M, N, device=dev, dtype=torch.float16)
    pkg.cuda.rmsnorm_linear_f16(dev_t(x).data_ptr(), dev_t(g).data_ptr() if gamma else 0,
                                dev_t(W).data_ptr(), 0, Y.data_ptr(), M, N, K, EPS)
    _, exact = oracle.rmsnorm_linear_f16(x, g, W, EPS, want_f32=True, nthreads=8)
    t = oracle.rmsnorm(x.astype(np.float32), None if g is None else g.astype(np.float32), EPS)
    absdot = np.abs(t.astype(np.float64)) @ np.abs(W.astype(np.float64)).T
    bounds.check(host(Y).astype(np.float32), exact, rms_bound(M, K, absdot, exact), f"M={M}")


@pytest.mark.parametrize("M", [1, 16, 48])
def test_rmsnorm_linear_f16_residual(pkg, dev, M):
    N, K = 512, 1024
    rng = np.random.default_rng(M)
    x = f16(rng, (M, K))
    g = (1 + 0.1 * rng.standard_normal(K)).astype(np.float16)
    W = f16(rng, (N, K), 0.02)
    R = f16(rng, (M, N))
    Y = torch.empty(M, N, device=dev, dtype=torch.float16)
    pkg.cuda.rmsnorm_linear_f16(dev_t(x).data_ptr(), dev_t(g).data_ptr(), dev_t(W).data_ptr(),
                                dev_t(R).data_ptr(), Y.data_ptr(), M, N, K, EPS)
    _, exact = oracle.rmsnorm_linear_f16(x, g, W, EPS, residual=R, want_f32=True)
    t = oracle.rmsnorm(x.astype(np.float32), g.astype(np.float32), EPS)
    absdot = np.abs(t.astype(np.float64)) @ np.abs(W.astype(np.float64)).T
    bound = rms_bound(M, K, absdot, exact) + bounds.U16 * np.abs(exact)
    bounds.check(host(Y).astype(np.float32), exact, bound, f"resid M={M}")


@pytest.mark.parametrize("M,N,K,gamma,resid", [
    (7, 300, 1000, True, False),     # partial weight tile, last k-block partial (K % 64 = 40)
    (32, 640, 4104, True, True),     # 32 rows (64 hi/lo activation rows), residual
    (5, 128, 64, False, False),      # one k-block, no gamma
    (16, 6144, 14336, True, False),  # long K: split-K cluster partials and row sums
])
def test_rmsnorm_linear_f16_hilo_edges(pkg, dev, M, N, K, gamma, resid):
    """5 <= M <= 32 (hi/lo activations, swap-AB tcgen05, split-K clusters) at the
    edges of its tiling: a partial weight tile, a partial last k-block, a single
    k-block, 32 rows, a long K; run twice for determinism."""
    rng = np.random.default_rng(M + N + K)
    x = f16(rng, (M, K))
    g = (1 + 0.1 * rng.standard_normal(K)).astype(np.float16) if gamma else None
    W = f16(rng, (N, K), 0.02)
    R = f16(rng, (M, N)) if resid else None
    Y = torch.empty(M, N, device=dev, dtype=torch.float16)
    pkg.cuda.rmsnorm_linear_f16(dev_t(x).data_ptr(), dev_t(g).data_ptr() if gamma else 0,
                                dev_t(W).data_ptr(), dev_t(R).data_ptr() if resid else 0,
                                Y.data_ptr(), M, N, K, EPS)
    _, exact = oracle.rmsnorm_linear_f16(x, g, W, EPS, residual=R, want_f32=True, nthreads=8)
    t = oracle.rmsnorm(x.astype(np.float32), None if g is None else g.astype(np.float32), EPS)
    absdot = np.abs(t.astype(np.float64)) @ np.abs(W.astype(np.float64)).T
    bound = rms_bound(M, K, absdot, exact) + (bounds.U16 * np.abs(exact) if resid else 0)
    bounds.check(host(Y).astype(np.float32), exact, bound, f"hilo M={M} N={N} K={K}")
    Y2 = torch.empty_like(Y)
    pkg.cuda.rmsnorm_linear_f16(dev_t(x).data_ptr(), dev_t(g).data_ptr() if gamma else 0,
                                dev_t(W).data_ptr(), dev_t(R).data_ptr() if resid else 0,
                                Y2.data_ptr(), M, N, K, EPS)
    assert torch.equal(Y, Y2)  # fixed-order cluster reduction: deterministic


@pytest.mark.parametrize("M,F,gamma", [(1, 1792, True), (1, 14336, True), (1, 3584, False),
                                       (3, 1792, True), (16, 3584, True)])
def test_rmsnorm_linear_swiglu_fused(pkg, dev, M, F, gamma):
    """The fused gate/up projection + SwiGLU equals rmsnorm_linear_f16 into
    [M, 2F] followed by swiglu_f16, bit for bit (batch 1: one kernel; larger
    batches: scratch + the same two steps), and the oracle composition of the
    reference's ops within a derived bound."""
    K = 4096
    rng = np.random.default_rng(M * 1000 + F)
    x = f16(rng, (M, K))
    g = (1 + 0.1 * rng.standard_normal(K)).astype(np.float16)
    W = f16(rng, (2 * F, K), 0.02)
    tx, tg, tw = dev_t(x), dev_t(g), dev_t(W)
    gp = tg if gamma else None
    fused = pkg.ops.rmsnorm_linear_swiglu(tx, gp, tw, EPS)
    gu = pkg.ops.rmsnorm_linear(tx, gp, tw, EPS)
    ref = pkg.ops.swiglu(gu[:, :F].contiguous(), gu[:, F:].contiguous())
    torch.cuda.synchronize()
    assert torch.equal(fused, ref)
    # Oracle composition: gate/up rounded to FP16, then silu(g) * u.  The GPU's and
    # the oracle's g (and u) are each within the derived GEMV bound of the exact
    # projection, so |dg| <= 2 * gemv16_bound; with |silu'| <= 1.1,
    # |d(silu(g) u)| <= 1.1 |dg| |u| + |silu(g)| |du| + 1.1 |dg| |du|, plus the
    # final FP16 rounding of each side.
    gm = g if gamma else None
    go, exact = oracle.rmsnorm_linear_f16(x, gm, W, EPS, want_f32=True, nthreads=8)
    want = oracle.swiglu_f16(np.ascontiguousarray(go[:, :F]), np.ascontiguousarray(go[:, F:]))
    tn = oracle.rmsnorm(x.astype(np.float32), g.astype(np.float32) if gamma else None, EPS)
    absdot = np.abs(tn.astype(np.float64)) @ np.abs(W.astype(np.float64)).T
    d = 2 * bounds.gemv16_bound(K, absdot, exact)
    dg, du = d[:, :F], d[:, F:]
    gv = go[:, :F].astype(np.float64)
    uv = np.abs(go[:, F:].astype(np.float64))
    silu = np.abs(gv / (1 + np.exp(-gv)))
    w64 = want.astype(np.float64)
    bound = 1.1 * dg * uv + silu * du + 1.1 * dg * du + 2 * bounds.U16 * np.abs(w64) + 2.0 ** -24
    bounds.check(host(fused).astype(np.float64), w64, bound,
                 f"fused swiglu M={M} F={F}")


def test_swiglu_and_embedding_glue(pkg, dev):
    rng = np.random.default_rng(0)
    n = 14336 * 2 + 3
    gte = (3 * rng.standard_normal(n)).astype(np.float16)
    up = rng.standard_normal(n).astype(np.float16)
    out = torch.empty(n, device=dev, dtype=torch.float16)
    pkg.cuda.swiglu_fp16(dev_t(gte).data_ptr(), dev_t(up).data_ptr(), out.data_ptr(), n)
    exp = oracle.swiglu_f16(gte, up).astype(np.float32)
    got = host(out).astype(np.float32)
    # float silu (expf) vs double: a few float ulps before the single FP16 rounding.
    np.testing.assert_allclose(got, exp, rtol=2 * bounds.U16 + 1e-6, atol=2.0 ** -24)
    V, D = 1000, 256
    table = f16(rng, (V, D))
    ids = np.array([0, V - 1, 5, 17], np.int32)
    o = torch.empty(4, D, device=dev, dtype=torch.float16)
    pkg.cuda.embedding_fp16(dev_t(table).data_ptr(), dev_t(ids).data_ptr(), o.data_ptr(), 4, D, V)
    assert np.array_equal(host(o), table[ids])


def test_device_status_clean_after_suite(pkg, dev):
    torch.cuda.synchronize()
    assert pkg.device_status(0) == 0
