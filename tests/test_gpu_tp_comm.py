"""GPU (one B200): the tensor-parallel communicator (engine_tp_*) on one rank.

* world = 1: the fused projection + all-reduce (M <= 4) and its tensor-core
  fallback (M > 4) stay inside the derived bounds of the oracle; the plain
  all-reduce of one rank is exactly partial + residual, rounded once;
* a captured CUDA graph replays the communicator (its call counts live in
  device memory);
* bounded wait: a world = 2 loopback communicator whose second rank never
  pushes.  Nothing sets the flag it waits for, so the kernel gives up after
  ENGINE_WAIT_TIMEOUT_MS, sets bit 1 of the device error word and returns.
  The context stays usable.  The check runs in a child process so that the
  short limit applies there only.

Multi-GPU runs of the same calls are in tests/test_tp_gpu.py.
"""
from __future__ import annotations

import os
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
ROOT = Path(__file__).resolve().parent.parent


@pytest.fixture(scope="module")
def comm1(pkg, dev):
    c = pkg.tp.NvlinkComm(0, 1, 64 * 4096)
    yield c
    c.close()


@pytest.mark.parametrize("M", [1, 2, 3, 4])
@pytest.mark.parametrize("K", [512, 1792, 14336])
def test_fused_world1_matches_oracle(pkg, dev, comm1, M, K):
    """One rank: Y = X W^T + R by the fused kernel (FP32 CUDA-core dot products,
    one FP16 rounding) within the derived GEMV bound of the oracle."""
    N = 4096
    rng = np.random.default_rng(M * 100 + K)
    X = rng.standard_normal((M, K)).astype(np.float16)
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float16)
    R = rng.standard_normal((M, N)).astype(np.float16)
    t = lambda a: torch.from_numpy(a).to(dev)  # noqa: E731
    got = comm1.linear_allreduce(t(X), t(W), residual=t(R)).float().cpu().numpy()
    _, exact = oracle.linear_f16(X, W, residual=R, want_f32=True, nthreads=8)
    absdot = np.abs(X.astype(np.float64)) @ np.abs(W.astype(np.float64)).T
    bounds.check(got, exact, bounds.gemv16_bound(K, absdot, exact), f"fused M={M} K={K}")
    got0 = comm1.linear_allreduce(t(X), t(W)).float().cpu().numpy()
    _, exact0 = oracle.linear_f16(X, W, want_f32=True, nthreads=8)
    bounds.check(got0, exact0, bounds.gemv16_bound(K, absdot, exact0), f"fused M={M} K={K} no R")


@pytest.mark.parametrize("M", [8, 32])
def test_fallback_world1_within_bound(pkg, dev, comm1, M):
    N, K = 4096, 1792
    rng = np.random.default_rng(M)
    X = rng.standard_normal((M, K)).astype(np.float16)
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float16)
    R = rng.standard_normal((M, N)).astype(np.float16)
    t = lambda a: torch.from_numpy(a).to(dev)  # noqa: E731
    got = comm1.linear_allreduce(t(X), t(W), residual=t(R)).float().cpu().numpy()
    _, exact = oracle.linear_f16(X, W, residual=R, want_f32=True, nthreads=8)
    absdot = np.abs(X.astype(np.float64)) @ np.abs(W.astype(np.float64)).T
    # projection rounded to FP16 once (the partial), then the residual sum rounded once more
    part = np.abs(exact - R.astype(np.float64))
    bound = bounds.tc_bound(K, absdot, exact, bounds.U16) + bounds.U16 * part
    bounds.check(got, exact, bound, f"fallback M={M}")


def test_allreduce_world1_is_partial_plus_residual(pkg, dev, comm1):
    n = 3 * 4096 + 8
    g = torch.Generator(device=dev).manual_seed(5)
    P = torch.randn(n, device=dev, generator=g).half()
    R = torch.randn(n, device=dev, generator=g).half()
    got = comm1.allreduce(P, residual=R)
    want = (P.float() + R.float()).half()  # one FP32 add, one rounding
    assert torch.equal(got, want)
    odd = comm1.allreduce(P[1:], residual=R[1:])  # unaligned, scalar path
    assert torch.equal(odd, (P[1:].float() + R[1:].float()).half())


def test_graph_replay_of_fused_call(pkg, dev, comm1):
    N, K = 4096, 1792
    g = torch.Generator(device=dev).manual_seed(9)
    X = torch.randn(1, K, device=dev, generator=g).half()
    W = (torch.randn(N, K, device=dev, generator=g) * 0.02).half()
    R = torch.randn(1, N, device=dev, generator=g).half()
    Y = torch.empty(1, N, device=dev, dtype=torch.float16)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        comm1.linear_allreduce(X, W, residual=R, out=Y)
    torch.cuda.synchronize()
    ref = Y.clone()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        comm1.linear_allreduce(X, W, residual=R, out=Y)
    for _ in range(3):
        Y.zero_()
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(Y, ref)
    del graph
    assert pkg.device_status(dev.index or 0) == 0


_TIMEOUT_CHILD = textwrap.dedent("""
    import sys
    sys.path.insert(0, {root!r})
    import torch
    from tests.conftest import load_package
    pkg = load_package()
    c = pkg.cuda
    dev = torch.device("cuda", 0)
    assert pkg.device_status(0) == 0
    comm = c.tp_comm_create(0, 2, 4096)
    h = c.tp_comm_handle(comm)
    c.tp_comm_open(comm, h + h)          # rank 1 maps to this rank's own region
    P = torch.ones(4096, device=dev, dtype=torch.float16)
    Y = torch.zeros_like(P)
    c.tp_allreduce_f16(comm, P.data_ptr(), 0, Y.data_ptr(), 4096)
    torch.cuda.synchronize()
    flags = pkg.device_status(0)
    assert flags & 1, flags               # the bounded wait ran out and said so
    assert int((Y != 0).sum()) == 0       # no reduction after a time-out
    W = torch.ones(8, 64, device=dev, dtype=torch.float16)
    x = torch.ones(1, 64, device=dev, dtype=torch.float16)
    y = pkg.ops.linear(x, W)              # the context is still usable
    torch.cuda.synchronize()
    assert float(y[0, 0]) == 64.0
    assert pkg.device_status(0) == 0
    c.tp_comm_destroy(comm)
    print("TIMEOUT-OK")
""")


def test_bounded_wait_times_out_and_reports(pkg, dev):
    env = dict(os.environ, ENGINE_WAIT_TIMEOUT_MS="200")
    r = subprocess.run([sys.executable, "-c", _TIMEOUT_CHILD.format(root=str(ROOT))], env=env,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "TIMEOUT-OK" in r.stdout, r.stdout + r.stderr
