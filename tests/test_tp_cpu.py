"""CPU: tensor-parallel sharding and collectives of the layer set on gloo ranks.

World size 2 and 4 processes (spawned), a small Llama-shaped config, full
weights drawn once from a seed and sharded with the product's own shard_layer /
qkv_rows_for_rank / shard_head; projections by the float64 CPU test double.
Every rank's TP result must equal the unsharded (t = 1) result, and the
collective count must be exactly two all-reduces per layer.
"""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from tests.conftest import load_package

CFG_KW = dict(d_model=64, n_heads=8, n_kv_heads=4, head_dim=8, ffn=96, n_layers=3, vocab=200,
              eps=1e-5)


def full_weights(cfg, seed=3):
    g = torch.Generator().manual_seed(seed)
    layers = []
    for _ in range(cfg.n_layers):
        layers.append({
            "attn_norm": 1 + 0.1 * torch.randn(cfg.d_model, generator=g, dtype=torch.float64),
            "ffn_norm": 1 + 0.1 * torch.randn(cfg.d_model, generator=g, dtype=torch.float64),
            "qkv": 0.1 * torch.randn(cfg.qkv_rows, cfg.d_model, generator=g, dtype=torch.float64),
            "o": 0.1 * torch.randn(cfg.d_model, cfg.n_heads * cfg.head_dim, generator=g, dtype=torch.float64),
            "gate": 0.1 * torch.randn(cfg.ffn, cfg.d_model, generator=g, dtype=torch.float64),
            "up": 0.1 * torch.randn(cfg.ffn, cfg.d_model, generator=g, dtype=torch.float64),
            "down": 0.1 * torch.randn(cfg.d_model, cfg.ffn, generator=g, dtype=torch.float64),
        })
    lm = 0.1 * torch.randn(cfg.vocab, cfg.d_model, generator=g, dtype=torch.float64)
    embed = torch.randn(cfg.vocab, cfg.d_model, generator=g, dtype=torch.float64)
    fnorm = 1 + 0.1 * torch.randn(cfg.d_model, generator=g, dtype=torch.float64)
    return layers, lm, embed, fnorm


def run_model(tp, cfg, world, rank, ops, group=None):
    layers, lm, embed, fnorm = full_weights(cfg)
    shards = [tp.shard_layer(L, cfg, world, rank) for L in layers]
    m = tp.TPLayerSet(cfg, rank, world, shards, tp.shard_head(lm, cfg, world, rank), embed, fnorm,
                      ops=ops, group=group)
    ids = torch.tensor([0, 5, 199, 42], dtype=torch.int32)
    x = m.hidden(ops.embedding(embed, ids))
    nxt = m.greedy(m.logits_shard(x))
    return x, nxt, m.allreduce_count


def run_model_attention(tp, cfg, world, rank, ops, group=None):
    """Prefill of four tokens (one causal sequence) and one decode step over the
    caches, with the real per-rank attention heads."""
    layers, lm, embed, fnorm = full_weights(cfg)
    shards = [tp.shard_layer(L, cfg, world, rank) for L in layers]
    m = tp.TPLayerSet(cfg, rank, world, shards, tp.shard_head(lm, cfg, world, rank), embed, fnorm,
                      ops=ops, group=group)
    ids = torch.tensor([0, 5, 199, 42], dtype=torch.int32)
    m.enable_attention(5, dtype=torch.float64)
    x = m.hidden(ops.embedding(embed, ids))
    m.pos = 4
    xd = m.hidden(ops.embedding(embed, torch.tensor([7], dtype=torch.int32)))
    return torch.cat([x, xd]), m.greedy(m.logits_shard(xd)), m.allreduce_count


def _worker(rank, world, port, q, cfg_kw=None, attention=False):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist

    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        pkg = load_package()
        from tests.tp_cpu_ops import CpuOps

        tp = pkg.tp
        cfg = tp.TPConfig(**(cfg_kw or CFG_KW))
        run = run_model_attention if attention else run_model
        x, nxt, n_ar = run(tp, cfg, world, rank, CpuOps())
        q.put((rank, x.numpy(), nxt.numpy(), n_ar))
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e), None, None))
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


# d_model need not equal n_heads * head_dim: O's input is the query heads
GEMMA_LIKE_KW = dict(CFG_KW, d_model=48)


@pytest.mark.parametrize("world,cfg_kw", [(2, CFG_KW), (4, CFG_KW), (2, GEMMA_LIKE_KW)])
def test_tp_layer_set_matches_unsharded_on_gloo(world, cfg_kw):
    pkg = load_package()
    from tests.tp_cpu_ops import CpuOps

    tp = pkg.tp
    cfg = tp.TPConfig(**cfg_kw)
    x1, n1, ar1 = run_model(tp, cfg, 1, 0, CpuOps())
    assert ar1 == 0
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, cfg_kw)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, x, nxt, n_ar in results:
        assert not isinstance(x, str), f"rank {rank} failed: {x}"
        torch.testing.assert_close(torch.from_numpy(x), x1, rtol=1e-12, atol=1e-12)
        assert (nxt == n1.numpy()).all()
        assert n_ar == 2 * cfg.n_layers


# 16 query heads on 8 KV heads: t = 8 leaves one KV head (and two query heads) per rank
WIDE_KW = dict(CFG_KW, n_heads=16, n_kv_heads=8, d_model=128)


@pytest.mark.parametrize("world,cfg_kw", [(2, CFG_KW), (4, CFG_KW), (8, WIDE_KW)])
def test_tp_layer_set_with_attention_matches_unsharded_on_gloo(world, cfg_kw):
    """The per-rank attention heads and KV caches: a causal prefill and a decode
    step at t = 2, 4, 8 equal the unsharded run (each rank attends with its own
    query heads over its own KV heads; two all-reduces per layer per step)."""
    pkg = load_package()
    from tests.tp_cpu_ops import CpuOps

    tp = pkg.tp
    cfg = tp.TPConfig(**cfg_kw)
    x1, n1, _ = run_model_attention(tp, cfg, 1, 0, CpuOps())
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, cfg_kw, True))
             for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=180) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, x, nxt, n_ar in results:
        assert not isinstance(x, str), f"rank {rank} failed: {x}"
        torch.testing.assert_close(torch.from_numpy(x), x1, rtol=1e-12, atol=1e-12)
        assert (nxt == n1.numpy()).all()
        assert n_ar == 4 * cfg.n_layers


def test_qkv_shards_are_head_aligned_and_partition_the_rows():
    tp = load_package().tp
    cfg = tp.LLAMA3_8B
    for t in (1, 2, 4, 8):
        rows = torch.cat([tp.qkv_rows_for_rank(cfg, t, r) for r in range(t)])
        assert rows.numel() == cfg.qkv_rows
        assert torch.equal(rows.sort().values, torch.arange(cfg.qkv_rows))
        r0 = tp.qkv_rows_for_rank(cfg, t, 0)
        assert r0.numel() == cfg.qkv_rows // t
        # q block of rank 0 is whole heads
        assert (r0[: cfg.n_heads // t * cfg.head_dim] < cfg.n_heads * cfg.head_dim).all()


def test_tp_rejects_indivisible_degree():
    tp = load_package().tp
    with pytest.raises(ValueError):
        tp.LLAMA3_8B.check(3)


def test_weight_and_flop_accounting():
    tp = load_package().tp
    cfg = tp.LLAMA3_8B
    assert abs(tp.weight_bytes_per_rank(cfg, 1) - 15.01e9) / 15.01e9 < 0.01
    assert tp.weight_bytes_per_rank(cfg, 8) * 8 == pytest.approx(tp.weight_bytes_per_rank(cfg, 1))


# ------------------------------------------------------------ failure paths
# A rank fails on the host, never on a GPU: it never joins, exits right after
# joining, or raises before its first collective.  Rank 0 runs the TP layer
# set; its rendezvous or its next all-reduce must end with an error within the
# process group's short timeout, never hang.

PG_TIMEOUT_S = 5


def _fail_worker(rank, world, port, q, mode):
    import datetime
    import time

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist

    t0 = time.monotonic()
    if mode == "never_joins" and rank == 1:
        q.put((rank, "absent", 0.0))
        return
    joined = False
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=PG_TIMEOUT_S))
        joined = True
        if rank == 1 and mode == "exits_early":
            q.put((rank, "exited", time.monotonic() - t0))
            q.close()
            q.join_thread()  # the message is flushed before the process vanishes
            os._exit(0)  # leaves without a goodbye: its sockets close under rank 0
        if rank == 1 and mode == "raises":
            raise RuntimeError("failure injected on rank 1")
        pkg = load_package()
        from tests.tp_cpu_ops import CpuOps

        tp = pkg.tp
        run_model(tp, tp.TPConfig(**CFG_KW), world, rank, CpuOps())
        q.put((rank, "ok", time.monotonic() - t0))
    except Exception as e:  # the error is the expected outcome on rank 0
        q.put((rank, "error: " + repr(e)[:300], time.monotonic() - t0))
    finally:
        if joined:
            try:
                dist.destroy_process_group()
            except Exception:
                pass


@pytest.mark.parametrize("mode", ["never_joins", "exits_early", "raises"])
def test_tp_peer_failure_is_an_error_not_a_hang(mode):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_fail_worker, args=(r, world, port, q, mode)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        res = dict((r, (s, t)) for r, s, t in (q.get(timeout=120) for _ in range(world)))
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():  # never expected; do not leave a process behind
                p.kill()
                p.join()
    status0, t0 = res[0]
    assert status0.startswith("error"), f"rank 0 did not report the failed peer: {status0}"
    # within the process-group timeout plus start-up (spawn, imports, the store)
    assert t0 < PG_TIMEOUT_S + 60, f"rank 0 took {t0:.0f} s to notice"
    assert res[1][0] in ({"never_joins": "absent", "exits_early": "exited"}.get(mode) or
                         "error: RuntimeError('failure injected on rank 1')",)


# ------------------------------------------------ sharding properties
from hypothesis import given, settings  # noqa: E402
from hypothesis import strategies as st  # noqa: E402


@st.composite
def _cfg_and_degree(draw):
    t = draw(st.sampled_from([1, 2, 4, 8]))
    kv = t * draw(st.integers(1, 2))
    h = kv * draw(st.integers(1, 3))
    hd = draw(st.sampled_from([2, 4, 6]))
    # d_model need not equal n_heads * head_dim (Gemma-style shapes)
    d = t * draw(st.integers(1, 4))
    return dict(d_model=d, n_heads=h, n_kv_heads=kv, head_dim=hd, ffn=t * draw(st.integers(1, 4)),
                n_layers=1, vocab=t * draw(st.integers(1, 5)), eps=1e-5), t


@settings(max_examples=80, deadline=None)
@given(ct=_cfg_and_degree())
def test_shards_partition_every_weight(ct):
    """Over the ranks, the shards of every weight reassemble it exactly: QKV rows
    (head-aligned), O columns (the rank's query heads), gate and up rows, down
    columns and the vocab rows of the LM head."""
    kw, t = ct
    tp = load_package().tp
    cfg = tp.TPConfig(**kw)
    cfg.check(t)
    hd_all = cfg.n_heads * cfg.head_dim
    g = torch.Generator().manual_seed(1)
    full = {"attn_norm": torch.randn(cfg.d_model, generator=g),
            "ffn_norm": torch.randn(cfg.d_model, generator=g),
            "qkv": torch.randn(cfg.qkv_rows, cfg.d_model, generator=g),
            "o": torch.randn(cfg.d_model, hd_all, generator=g),
            "gate": torch.randn(cfg.ffn, cfg.d_model, generator=g),
            "up": torch.randn(cfg.ffn, cfg.d_model, generator=g),
            "down": torch.randn(cfg.d_model, cfg.ffn, generator=g)}
    lm = torch.randn(cfg.vocab, cfg.d_model, generator=g)
    shards = [tp.shard_layer(full, cfg, t, r) for r in range(t)]
    rows = torch.cat([tp.qkv_rows_for_rank(cfg, t, r) for r in range(t)])
    assert torch.equal(rows.sort().values, torch.arange(cfg.qkv_rows))
    assert torch.equal(torch.cat([s["qkv"] for s in shards]), full["qkv"][rows])
    assert torch.equal(torch.cat([s["o"] for s in shards], dim=1), full["o"])
    f = cfg.ffn // t
    assert torch.equal(torch.cat([s["gate_up"][:f] for s in shards]), full["gate"])
    assert torch.equal(torch.cat([s["gate_up"][f:] for s in shards]), full["up"])
    assert torch.equal(torch.cat([s["down"] for s in shards], dim=1), full["down"])
    assert torch.equal(torch.cat([tp.shard_head(lm, cfg, t, r) for r in range(t)]), lm)
    for s in shards:  # each rank's q rows are whole heads, and its O input matches them
        assert s["o"].shape[1] == cfg.n_heads // t * cfg.head_dim
