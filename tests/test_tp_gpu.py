"""GPU: the tensor-parallel layer set (Llama-3-8B shapes, two layers) on B200s.

* t = 1 on one GPU: each layer, fed the GPU's own input, against the oracle
  composition of the reference's ops (rmsnorm_linear -> linear + residual ->
  rmsnorm_linear -> swiglu -> linear + residual, tests/test_kernels.cu:2813-2938)
  with FP16 rounding at the same op boundaries;
* t = 1 with the library's attention over KV caches (prefill and a decode
  step) against the oracle composition with the reference's attention;
* t = 2, 4, 8 (one process per GPU; skipped when the box has fewer GPUs):
  every rank's hidden state and its logits shard against t = 1 on the same full
  weights (the tokens as one causal sequence through the real attention), sharded by the product's own shard_layer / shard_head -- once with
  NCCL all-reduces and once with the library's NVLink communicator (the O /
  down projections fused with their all-reduce);
* the communicator's fused call alone on t ranks: Y = sum_r X_r W_r^T + R
  within the derived bound of the oracle sum, and bit-identical on every rank.

Tolerances.  Each op of the chain is pinned to the oracle by its own parity test.
Here the chains themselves differ in rounding: the GPU accumulates in FP32 and
the oracle in FP64, and at t > 1 every rank rounds its partial projection to
FP16 before the all-reduce, where t = 1 rounds the full sum once.  One FP16 ulp
at the hidden state's magnitude (|x| < 8) is <= 2^-8; the headroom below
(atol 2e-2 + rtol 2e-2) allows a few ulps per op over the chain, the same kind of
documented headroom the reference uses for stacked layers
(tests/test_kernels.cu:3387-3390).
"""
from __future__ import annotations

import dataclasses
import os
import socket

import numpy as np
import pytest

import oracle
from tests.conftest import load_package

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

N_LAYERS = 2
TOKENS = [0, 5, 128255, 4242]
ATOL = 2e-2
RTOL = 2e-2


def full_weights(cfg, dev, seed=11):
    """Unsharded FP16 weights drawn on `dev`; identical on every GPU for a seed."""
    g = torch.Generator(device=dev).manual_seed(seed)

    def rn(*shape, scale=0.02):
        return (torch.randn(*shape, device=dev, generator=g) * scale).half()

    layers = []
    for _ in range(cfg.n_layers):
        layers.append({
            "attn_norm": (1 + rn(cfg.d_model, scale=0.1).float()).half(),
            "ffn_norm": (1 + rn(cfg.d_model, scale=0.1).float()).half(),
            "qkv": rn(cfg.qkv_rows, cfg.d_model),
            "o": rn(cfg.d_model, cfg.n_heads * cfg.head_dim),
            "gate": rn(cfg.ffn, cfg.d_model),
            "up": rn(cfg.ffn, cfg.d_model),
            "down": rn(cfg.d_model, cfg.ffn),
        })
    lm = rn(cfg.vocab, cfg.d_model)
    embed = rn(cfg.vocab, cfg.d_model, scale=1.0)
    fnorm = (1 + rn(cfg.d_model, scale=0.1).float()).half()
    return layers, lm, embed, fnorm


def build(tp, cfg, t, r, weights, group=None):
    layers, lm, embed, fnorm = weights
    shards = [tp.shard_layer(L, cfg, t, r) for L in layers]
    return tp.TPLayerSet(cfg, r, t, shards, tp.shard_head(lm, cfg, t, r), embed, fnorm,
                         group=group)


def small_cfg(tp):
    return dataclasses.replace(tp.LLAMA3_8B, n_layers=N_LAYERS)


def oracle_layer(x, L, cfg):
    """One layer of the reference composition on the host, FP16 at op boundaries."""
    f = cfg.ffn
    h = lambda t: t.detach().cpu().numpy()  # noqa: E731
    Wgu = np.concatenate([h(L["gate"]), h(L["up"])])
    qkv = oracle.rmsnorm_linear_f16(x, h(L["attn_norm"]), h(L["qkv"]), cfg.eps, nthreads=8)
    attn = np.ascontiguousarray(qkv[:, : cfg.n_heads * cfg.head_dim])
    x1 = oracle.linear_f16(attn, h(L["o"]), residual=x, nthreads=8)
    gu = oracle.rmsnorm_linear_f16(x1, h(L["ffn_norm"]), Wgu, cfg.eps, nthreads=8)
    sw = oracle.swiglu_f16(np.ascontiguousarray(gu[:, :f]), np.ascontiguousarray(gu[:, f:]))
    return oracle.linear_f16(sw, h(L["down"]), residual=x1, nthreads=8)


def test_tp_layer_set_t1_matches_oracle_composition(pkg, dev):
    tp = pkg.tp
    cfg = small_cfg(tp)
    weights = full_weights(cfg, dev)
    layers, lm, embed, fnorm = weights
    ids = torch.tensor(TOKENS, dtype=torch.int32, device=dev)
    x = pkg.ops.embedding(embed, ids)
    assert torch.equal(x, embed[ids.long()])
    for li, L in enumerate(layers):
        one = tp.TPLayerSet(dataclasses.replace(cfg, n_layers=1), 0, 1,
                            [tp.shard_layer(L, cfg, 1, 0)], lm, embed, fnorm)
        x_in = x.detach().cpu().numpy()
        x = one.hidden(x)
        torch.cuda.synchronize()
        want = oracle_layer(x_in, L, cfg).astype(np.float32)
        got = x.float().cpu().numpy()
        assert np.isfinite(got).all()
        np.testing.assert_allclose(got, want, rtol=RTOL, atol=ATOL,
                                   err_msg=f"layer {li} against the oracle composition")
    # Greedy next token over the full vocabulary equals the host argmax of the
    # GPU's own logits (lowest index on ties).
    m = build(tp, cfg, 1, 0, weights)
    logits = m.logits_shard(x)
    nxt = m.greedy(logits)
    lg = logits.float().cpu().numpy()
    assert (nxt.cpu().numpy() == lg.argmax(axis=1)).all()


def oracle_layer_attn(x, L, cfg, k_prev=None, v_prev=None):
    """oracle_layer with the real attention: the rows of x are the new tokens of
    one sequence at positions P.. (P = cached positions, whose K / V rows are
    k_prev / v_prev [H_kv, P, d]); causal attention over all positions, FP16 at
    the op boundaries.  Returns (x_out, k_all, v_all)."""
    f = cfg.ffn
    d, H, Hk = cfg.head_dim, cfg.n_heads, cfg.n_kv_heads
    h = lambda t: t.detach().cpu().numpy()  # noqa: E731
    Wgu = np.concatenate([h(L["gate"]), h(L["up"])])
    S = x.shape[0]
    qkv = oracle.rmsnorm_linear_f16(x, h(L["attn_norm"]), h(L["qkv"]), cfg.eps, nthreads=8)
    q = np.ascontiguousarray(qkv[:, :H * d].reshape(S, H, d))
    k = qkv[:, H * d:(H + Hk) * d].reshape(S, Hk, d).transpose(1, 0, 2)
    v = qkv[:, (H + Hk) * d:].reshape(S, Hk, d).transpose(1, 0, 2)
    P = 0 if k_prev is None else k_prev.shape[1]
    if P:
        k = np.concatenate([k_prev, k], axis=1)
        v = np.concatenate([v_prev, v], axis=1)
    k, v = np.ascontiguousarray(k), np.ascontiguousarray(v)
    att, _ = oracle.attention(q, k, v, d ** -0.5, P, True)
    attn = np.ascontiguousarray(att.astype(np.float16).reshape(S, H * d))
    x1 = oracle.linear_f16(attn, h(L["o"]), residual=x, nthreads=8)
    gu = oracle.rmsnorm_linear_f16(x1, h(L["ffn_norm"]), Wgu, cfg.eps, nthreads=8)
    sw = oracle.swiglu_f16(np.ascontiguousarray(gu[:, :f]), np.ascontiguousarray(gu[:, f:]))
    return oracle.linear_f16(sw, h(L["down"]), residual=x1, nthreads=8), k, v


def test_tp_layer_set_t1_attention_matches_oracle_composition(pkg, dev):
    """The layer set with the library's attention over KV caches at t = 1: a
    32-token causal prefill (the tcgen05 FlashAttention kernel) and then one
    decode step attending to all 33 positions (the tcgen05 decode kernel),
    each layer fed the GPU's own input and its own cache, against the oracle
    composition with the reference's two-pass attention at the same FP16
    boundaries."""
    tp = pkg.tp
    cfg = small_cfg(tp)
    layers, lm, embed, fnorm = full_weights(cfg, dev, seed=23)
    S = 32
    ids = torch.randint(0, cfg.vocab, (S + 1,), device=dev,
                        generator=torch.Generator(device=dev).manual_seed(5), dtype=torch.int32)
    one_cfg = dataclasses.replace(cfg, n_layers=1)
    ones = []
    x = pkg.ops.embedding(embed, ids[:S])
    for li, L in enumerate(layers):
        one = tp.TPLayerSet(one_cfg, 0, 1, [tp.shard_layer(L, cfg, 1, 0)], lm, embed, fnorm)
        one.enable_attention(S + 1)
        x_in = x.detach().cpu().numpy()
        x = one.hidden(x)
        torch.cuda.synchronize()
        want, _, _ = oracle_layer_attn(x_in, L, cfg)
        np.testing.assert_allclose(x.float().cpu().numpy(), want.astype(np.float32), rtol=RTOL,
                                   atol=ATOL, err_msg=f"prefill layer {li}")
        ones.append(one)
    xd = pkg.ops.embedding(embed, ids[S:])
    for li, (L, one) in enumerate(zip(layers, ones)):
        one.pos = S
        kc, vc = one.kv[0]
        k_prev = kc[:, :S].cpu().numpy()
        v_prev = vc[:, :S].cpu().numpy()
        x_in = xd.detach().cpu().numpy()
        xd = one.hidden(xd)
        torch.cuda.synchronize()
        want, k_all, v_all = oracle_layer_attn(x_in, L, cfg, k_prev, v_prev)
        np.testing.assert_allclose(xd.float().cpu().numpy(), want.astype(np.float32), rtol=RTOL,
                                   atol=ATOL, err_msg=f"decode layer {li}")
        # the new token's K / V landed at position S (the GPU's projection against
        # the oracle's: within the projection's rounding)
        for got_c, want_c in ((kc, k_all), (vc, v_all)):
            np.testing.assert_allclose(got_c[:, S].float().cpu().numpy(),
                                       want_c[:, S].astype(np.float32), rtol=RTOL, atol=ATOL)


# ------------------------------------------------------------------ t > 1

def _worker(rank, world, port, q, use_comm):
    import datetime

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist

    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=dev)
        pkg = load_package()
        tp = pkg.tp
        cfg = small_cfg(tp)
        weights = full_weights(cfg, dev)
        ids = torch.tensor(TOKENS, dtype=torch.int32, device=dev)
        comm = tp.NvlinkComm(rank, world, len(TOKENS) * cfg.d_model) if use_comm else None
        m = build(tp, cfg, world, rank, weights)
        m.comm = comm
        m.enable_attention(len(TOKENS))  # the tokens as one causal sequence
        x = m.hidden(pkg.ops.embedding(weights[2], ids))
        logits = m.logits_shard(x)
        nxt = m.greedy(logits)
        res = {"x": x.float().cpu().numpy(), "logits": logits.float().cpu().numpy(),
               "next": nxt.cpu().numpy(), "allreduces": m.allreduce_count}
        if comm is not None:
            comm.close()
        if rank == 0:
            m1 = build(tp, cfg, 1, 0, weights)
            m1.enable_attention(len(TOKENS))
            x1 = m1.hidden(pkg.ops.embedding(weights[2], ids))
            res["x1"] = x1.float().cpu().numpy()
            res["logits1"] = m1.logits_shard(x1).float().cpu().numpy()
        torch.cuda.synchronize()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, res))
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _run_ranks(target, world, *args):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q) + args) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=600) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r, res in results.items():
        assert not isinstance(res, str), f"rank {r} failed: {res}"
    return results


@pytest.mark.parametrize("collective", ["nccl", "nvlink"])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_layer_set_matches_t1(pkg, world, collective):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    cfg = small_cfg(pkg.tp)
    results = _run_ranks(_worker, world, collective == "nvlink")
    x1, l1 = results[0]["x1"], results[0]["logits1"]
    v = cfg.vocab // world
    for r, res in results.items():
        assert res["allreduces"] == 2 * cfg.n_layers
        np.testing.assert_allclose(res["x"], x1, rtol=RTOL, atol=ATOL, err_msg=f"rank {r} hidden")
        np.testing.assert_allclose(res["logits"], l1[:, r * v:(r + 1) * v], rtol=RTOL, atol=ATOL,
                                   err_msg=f"rank {r} logits")
        assert (res["next"] == results[0]["next"]).all()


# ------------------------------------------------------------------ communicator alone

def _comm_worker(rank, world, port, q, M, N, K):
    import datetime

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist

    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=dev)
        pkg = load_package()
        rng = np.random.default_rng(1000 + rank)
        X = rng.standard_normal((M, K)).astype(np.float16)
        W = (rng.standard_normal((N, K)) * 0.02).astype(np.float16)
        R = np.random.default_rng(7).standard_normal((M, N)).astype(np.float16)
        comm = pkg.tp.NvlinkComm(rank, world, M * N)
        t = lambda a: torch.from_numpy(a).to(dev)  # noqa: E731
        Y = comm.linear_allreduce(t(X), t(W), residual=t(R))
        Y2 = comm.linear_allreduce(t(X), t(W), residual=t(R))  # second call: other parity
        torch.cuda.synchronize()
        res = {"Y": Y.cpu().numpy(), "Y2": Y2.cpu().numpy(), "X": X, "W": W, "R": R,
               "status": pkg.device_status(rank)}
        comm.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, res))
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e)))


@pytest.mark.parametrize("M,K", [(1, 512), (4, 1792), (32, 1792)])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_fused_linear_allreduce_matches_oracle_sum(pkg, world, M, K):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    N = 4096
    results = _run_ranks(_comm_worker, world, M, N, K)
    Y0 = results[0]["Y"]
    for r, res in results.items():
        assert res["status"] == 0
        assert np.array_equal(res["Y"].view(np.uint16), Y0.view(np.uint16)), f"rank {r} differs"
        assert np.array_equal(res["Y2"].view(np.uint16), Y0.view(np.uint16))
    exact = results[0]["R"].astype(np.float64)
    absdot = np.zeros((M, N))
    for r in range(world):
        _, e = oracle.linear_f16(results[r]["X"], results[r]["W"], want_f32=True, nthreads=8)
        exact = exact + e
        absdot += np.abs(results[r]["X"].astype(np.float64)) @ np.abs(
            results[r]["W"].astype(np.float64)).T
    from tests import bounds

    # per-rank FP32 dot products (c = 2 covers the tensor-core fallback at M = 32),
    # the FP32 sum over ranks, one FP16 rounding (plus the FP16 partial at M = 32)
    bound = (bounds.tc_bound(K, absdot, exact, bounds.U16) + world * bounds.U32 * absdot
             + (bounds.U16 * absdot if M > 4 else 0))
    bounds.check(Y0.astype(np.float64), exact, bound, f"fused all-reduce t={world} M={M}")
