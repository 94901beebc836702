"""GPU: engine_cuda_rmsnorm_linear_f16_noalloc, the allocation-free variant.

It serves callers that may not allocate device memory (serving loops that
reserve every buffer at start-up, hosts whose device memory belongs to another
allocator); its normalised activations live in a fixed array inside the
library.  Called through the C ABI and compared with the existing
engine_cuda_rmsnorm_linear_f16 on the same inputs, within the derived bounds
the other parity tests use, on two calls in a row (the second with different
inputs and a smaller batch, so stale rows from the first call would show).

The file name sorts last so that a run stopping at the first failure has
already run every other test.
"""
from __future__ import annotations

import subprocess
import sys
import textwrap
from pathlib import Path

import numpy as np
import pytest

import oracle
from tests import bounds

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
EPS = 1e-5


def _bound(M, K, absdot, exact):
    """Derived bound of rmsnorm_linear_f16 on each of its dispatch paths
    (CUDA-core GEMV for M <= 4, tcgen05 with hi/lo activations for M <= 32)."""
    c = (K + K / 64 + 16) if M <= 4 else (2 * K + 8)
    return c * bounds.U32 * absdot + (bounds.U32 + bounds.U16) * np.abs(exact) + 2.0 ** -25


def _case(rng, M, N, K, dev):
    x = (rng.standard_normal((M, K))).astype(np.float16)
    g = (1 + 0.1 * rng.standard_normal(K)).astype(np.float16)
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float16)
    R = rng.standard_normal((M, N)).astype(np.float16)
    t = {k: torch.from_numpy(v).to(dev) for k, v in dict(x=x, g=g, W=W, R=R).items()}
    return (x, g, W, R), t


def _run(pkg, fn, t, M, N, K, dev):
    Y = torch.empty(M, N, device=dev, dtype=torch.float16)
    fn(t["x"].data_ptr(), t["g"].data_ptr(), t["W"].data_ptr(), t["R"].data_ptr(), Y.data_ptr(),
       M, N, K, EPS)
    torch.cuda.synchronize()
    return Y.cpu().numpy().astype(np.float32)


def test_noalloc_matches_existing_entry_point_on_two_calls(pkg, dev):
    N, K = 6144, 4096
    rng = np.random.default_rng(20260826)
    for M in (16, 5):  # second call: new inputs, fewer rows than the first
        (x, g, W, R), t = _case(rng, M, N, K, dev)
        got = _run(pkg, pkg.cuda.rmsnorm_linear_f16_noalloc, t, M, N, K, dev)
        ref = _run(pkg, pkg.cuda.rmsnorm_linear_f16, t, M, N, K, dev)
        _, exact = oracle.rmsnorm_linear_f16(x, g, W, EPS, residual=R, want_f32=True, nthreads=8)
        tn = oracle.rmsnorm(x.astype(np.float32), g.astype(np.float32), EPS)
        absdot = np.abs(tn.astype(np.float64)) @ np.abs(W.astype(np.float64)).T
        b = _bound(M, K, absdot, exact) + bounds.U16 * np.abs(exact)  # + residual rounding
        bounds.check(got, ref, 2 * b, f"noalloc vs existing, M={M}")
        bounds.check(got, exact, b, f"noalloc vs oracle, M={M}")


def test_noalloc_batch_one_against_gemv_path(pkg, dev):
    """M = 1: the existing entry point streams W on CUDA cores; the variant
    uses the tensor-core path with the fixed scratch.  Same answer within bound."""
    N, K = 4096, 4096
    rng = np.random.default_rng(1)
    (x, g, W, R), t = _case(rng, 1, N, K, dev)
    got = _run(pkg, pkg.cuda.rmsnorm_linear_f16_noalloc, t, 1, N, K, dev)
    ref = _run(pkg, pkg.cuda.rmsnorm_linear_f16, t, 1, N, K, dev)
    _, exact = oracle.rmsnorm_linear_f16(x, g, W, EPS, residual=R, want_f32=True)
    tn = oracle.rmsnorm(x.astype(np.float32), g.astype(np.float32), EPS)
    absdot = np.abs(tn.astype(np.float64)) @ np.abs(W.astype(np.float64)).T
    b_gemv = _bound(1, K, absdot, exact) + bounds.U16 * np.abs(exact)
    b_tc = _bound(32, K, absdot, exact) + bounds.U16 * np.abs(exact)
    bounds.check(got, ref, b_gemv + b_tc, "noalloc vs existing, M=1")


def test_noalloc_rejects_sizes_beyond_its_scratch(pkg, dev):
    (_, _, _, _), t = _case(np.random.default_rng(2), 33, 64, 64, dev)
    Y = torch.empty(33, 64, device=dev, dtype=torch.float16)
    with pytest.raises(pkg.EngineError) as e:
        pkg.cuda.rmsnorm_linear_f16_noalloc(t["x"].data_ptr(), t["g"].data_ptr(), t["W"].data_ptr(),
                                            0, Y.data_ptr(), 33, 64, 64, EPS)
    assert "exceeds the fixed scratch" in str(e.value)
    with pytest.raises(pkg.EngineError):
        pkg.cuda.rmsnorm_linear_f16_noalloc(t["x"].data_ptr(), t["g"].data_ptr(), t["W"].data_ptr(),
                                            0, Y.data_ptr(), 1, 64, 16392, EPS)


def test_noalloc_reserves_no_device_memory_per_call(pkg, dev):
    """The property the entry point exists for.  In a fresh process (so no pool
    of the library holds cached blocks from earlier calls): one warm-up call,
    then calls at the largest and smaller sizes; the device's free memory
    (cudaMemGetInfo) must not move.  A variant that drew on the library's
    stream-ordered pool would reserve at least its 2 MiB of activation rows."""
    root = Path(__file__).resolve().parent.parent
    code = textwrap.dedent(f"""
        import sys
        sys.path.insert(0, {str(root)!r})
        import torch
        from tests.conftest import load_package
        pkg = load_package()
        dev = torch.device("cuda", 0)
        torch.cuda.set_device(dev)
        K, N = 16384, 256
        x = torch.randn(32, K, device=dev).half()
        g = torch.ones(K, device=dev).half()
        W = (torch.randn(N, K, device=dev) * 0.02).half()
        Y = torch.empty(32, N, device=dev, dtype=torch.float16)
        f = pkg.cuda.rmsnorm_linear_f16_noalloc
        f(x.data_ptr(), g.data_ptr(), W.data_ptr(), 0, Y.data_ptr(), 32, N, K, 1e-5)
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info()[0]
        for M in (32, 7, 1, 32, 16):
            f(x.data_ptr(), g.data_ptr(), W.data_ptr(), 0, Y.data_ptr(), M, N, K, 1e-5)
        torch.cuda.synchronize()
        free1 = torch.cuda.mem_get_info()[0]
        print("FREE", free0, free1)
    """)
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    line = [ln for ln in r.stdout.splitlines() if ln.startswith("FREE")][0]
    free0, free1 = map(int, line.split()[1:])
    assert free1 == free0, f"free device memory moved by {free0 - free1} bytes"
