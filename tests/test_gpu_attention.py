"""GPU: attention_prefill / attention_decode through the C ABI.

Against the reference's golden attention cases (outputs and LSE) with its own
derived tolerances (test_kernels.cu:288-299: 2*eps16 relative, 1.5*eps16 +
4*s_kv*u32 absolute; LSE 2e-5 + 4*s_kv*u32), and against the oracle
(orc_attention, pinned bit-exact to the reference's attention_cpu.cpp) at
Llama-3-8B shapes: 32 query heads over 8 KV heads, d = 128, causal prefill
with an offset, decode over 4096 keys for several split counts.  Edge cases:
no keys (zeros, lse = -inf), a KV stride that is not a multiple of 8 (the
scalar-load path), determinism.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from tests.golden import golden

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

E16, U32 = 2.0 ** -10, 2.0 ** -23


def _tol(s_kv):
    return (2 * E16, 1.5 * E16 + 4 * s_kv * U32), (2e-5, 2e-5 + 4 * s_kv * U32)


def _close(got, want, rtol, atol, what):
    np.testing.assert_allclose(np.asarray(got, np.float64), np.asarray(want, np.float64),
                               rtol=rtol, atol=atol, err_msg=what)


def _scale(d):
    return float(np.float32(1.0) / np.sqrt(np.float32(d)))


@pytest.mark.parametrize("stem", golden.stems("attention__"))
def test_prefill_matches_golden(pkg, dev, stem):
    g = golden.load(stem)
    p = next(c for c in golden._meta()["cases"] if c["stem"] == stem)["params"]
    q, k, v = (torch.from_numpy(g[n]).to(dev) for n in ("q", "k", "v"))
    out, lse = pkg.ops.attention(q, k, v, _scale(p["head_dim"]), p["q_pos_offset"],
                                 p["is_causal"], want_lse=True)
    (rt, at), (lrt, lat) = _tol(p["s_kv"])
    _close(out.cpu().numpy().astype(np.float32), g["expected"], rt, at, stem)
    _close(lse.cpu().numpy(), g["lse"], lrt, lat, stem + " lse")


@pytest.mark.parametrize("stem", [s for s in golden.stems("attention__")
                                  if "_decode" in s or "nocausal" in s])
def test_decode_matches_golden(pkg, dev, stem):
    """The non-causal one-row cases are decode: every key visible."""
    g = golden.load(stem)
    q = torch.from_numpy(g["q"][0]).to(dev)
    k, v = (torch.from_numpy(g[n]).to(dev) for n in ("k", "v"))
    out = pkg.ops.attention_decode(q, k, v, _scale(q.shape[1]))
    (rt, at), _ = _tol(k.shape[1])
    _close(out.cpu().numpy().astype(np.float32), g["expected"][0], rt, at, stem)


def _rand(rng, s_q, h, h_kv, s_kv, d, amp=1.0):
    q = (rng.standard_normal((s_q, h, d)) * amp).astype(np.float16)
    k = (rng.standard_normal((h_kv, s_kv, d)) * amp).astype(np.float16)
    v = rng.standard_normal((h_kv, s_kv, d)).astype(np.float16)
    return q, k, v


@pytest.mark.parametrize("s_q,s_kv,off", [(256, 256, 0), (64, 320, 256)])
def test_prefill_llama_shape_matches_oracle(pkg, dev, s_q, s_kv, off):
    rng = np.random.default_rng(s_q + s_kv)
    q, k, v = _rand(rng, s_q, 32, 8, s_kv, 128)
    want, want_lse = oracle.attention(q, k, v, _scale(128), off, True)
    out, lse = pkg.ops.attention(*(torch.from_numpy(a).to(dev) for a in (q, k, v)), _scale(128),
                                 off, True, want_lse=True)
    (rt, at), (lrt, lat) = _tol(s_kv)
    _close(out.cpu().numpy().astype(np.float32), want.astype(np.float32), rt, at, "prefill")
    _close(lse.cpu().numpy(), want_lse, lrt, lat, "prefill lse")


@pytest.mark.parametrize("split_kv", [0, 1, 3, 7, 64])
def test_decode_llama_shape_matches_oracle(pkg, dev, split_kv):
    rng = np.random.default_rng(7)
    kv_len = 4096
    q, k, v = _rand(rng, 1, 32, 8, kv_len, 128)
    want, _ = oracle.attention(q, k, v, _scale(128), 0, False)
    qd, kd, vd = (torch.from_numpy(a).to(dev) for a in (q[0], k, v))
    out = pkg.ops.attention_decode(qd, kd, vd, _scale(128), split_kv)
    (rt, at), _ = _tol(kv_len)
    _close(out.cpu().numpy().astype(np.float32), want[0].astype(np.float32), rt, at,
           f"decode split_kv={split_kv}")
    again = pkg.ops.attention_decode(qd, kd, vd, _scale(128), split_kv)
    assert torch.equal(out, again)  # fixed-order merges: deterministic


def test_empty_kv_and_unaligned_stride(pkg, dev):
    c = pkg.cuda
    q = torch.randn(3, 4, 64, device=dev).half()
    out = torch.full_like(q, float("nan"))
    lse = torch.zeros(3, 4, device=dev)
    c.attention_prefill(q.data_ptr(), q.data_ptr(), q.data_ptr(), out.data_ptr(), 3, 0, 4, 2, 64,
                        0, 0.125, 0, True, lse.data_ptr())
    torch.cuda.synchronize()
    assert torch.equal(out, torch.zeros_like(out)) and bool(torch.isneginf(lse).all())
    # KV heads 4 elements apart beyond s_kv * d: the stride is not a multiple of 8
    rng = np.random.default_rng(3)
    s_kv, d, h_kv = 40, 64, 2
    stride = s_kv * d + 4
    q, k, v = _rand(rng, 5, 4, h_kv, s_kv, d)
    kp = np.zeros(h_kv * stride, np.float16)
    vp = np.zeros(h_kv * stride, np.float16)
    for hh in range(h_kv):
        kp[hh * stride: hh * stride + s_kv * d] = k[hh].ravel()
        vp[hh * stride: hh * stride + s_kv * d] = v[hh].ravel()
    want, _ = oracle.attention(q, k, v, 0.125, 2, True)
    qd, kd, vd = (torch.from_numpy(a).to(dev) for a in (q, kp, vp))
    od = torch.empty_like(qd)
    c.attention_prefill(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), od.data_ptr(), 5, s_kv, 4,
                        h_kv, d, stride, 0.125, 2, True, 0)
    (rt, at), _ = _tol(s_kv)
    _close(od.cpu().numpy().astype(np.float32), want.astype(np.float32), rt, at, "strided")


def test_decode_throughput_llama8b(pkg, dev):
    """Prints the decode kernel's HBM rate at Llama-3-8B, 4096 keys (not asserted)."""
    H, H_kv, d, kv_len = 32, 8, 128, 4096
    sets = [(torch.randn(H, d, device=dev).half(),
             torch.randn(H_kv, kv_len, d, device=dev).half(),
             torch.randn(H_kv, kv_len, d, device=dev).half()) for _ in range(8)]  # 134 MB
    out = torch.empty(H, d, device=dev, dtype=torch.float16)
    for s in sets[:3]:
        pkg.ops.attention_decode(s[0], s[1], s[2])
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n = 80
    e0.record()
    for it in range(n):
        s = sets[it % len(sets)]
        pkg.cuda.attention_decode(s[0].data_ptr(), s[1].data_ptr(), s[2].data_ptr(), out.data_ptr(),
                                  kv_len, H, H_kv, d, kv_len * d, d ** -0.5, 0,
                                  torch.cuda.current_stream().cuda_stream)
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) / n * 1e3
    byt = 2 * H_kv * kv_len * d * 2 + 2 * 2 * H * d
    print(f"attention_decode Llama-3-8B kv_len=4096: {us:.1f} us, {byt / us / 1e3:.0f} GB/s")


# ------------------------------------------------------------------ tcgen05 prefill / bulk decode

@pytest.mark.parametrize("s_q,s_kv,off,causal,h,h_kv,d", [
    (130, 129, 0, True, 4, 2, 128),     # partial query block and partial key tile
    (200, 300, 100, True, 8, 8, 64),    # d = 64, MHA, causal with an offset
    (200, 300, 0, False, 8, 2, 128),    # non-causal, s_q != s_kv
    (1024, 1024, 0, True, 8, 2, 128),   # eight key tiles, rescales across tiles
    (16, 700, 684, True, 4, 1, 64),     # the smallest s_q the tensor-core path takes
])
def test_prefill_tensor_core_path_matches_oracle(pkg, dev, s_q, s_kv, off, causal, h, h_kv, d):
    rng = np.random.default_rng(s_q * 7 + s_kv)
    q, k, v = _rand(rng, s_q, h, h_kv, s_kv, d)
    want, want_lse = oracle.attention(q, k, v, _scale(d), off, causal)
    args = [torch.from_numpy(a).to(dev) for a in (q, k, v)]
    out, lse = pkg.ops.attention(*args, _scale(d), off, causal, want_lse=True)
    (rt, at), (lrt, lat) = _tol(s_kv)
    _close(out.cpu().numpy().astype(np.float32), want.astype(np.float32), rt, at, "prefill tc")
    _close(lse.cpu().numpy(), want_lse, lrt, lat, "prefill tc lse")
    again, lse2 = pkg.ops.attention(*args, _scale(d), off, causal, want_lse=True)
    assert torch.equal(out, again) and torch.equal(lse, lse2)  # deterministic


def test_prefill_large_scores_and_peaked_rows(pkg, dev):
    """Scores of magnitude ~50: every row's max moves across tiles and the
    probabilities underflow for most keys; the online rescaling must agree with
    the two-pass oracle."""
    rng = np.random.default_rng(11)
    q, k, v = _rand(rng, 384, 4, 2, 512, 128, amp=2.5)
    want, want_lse = oracle.attention(q, k, v, _scale(128), 128, True)
    out, lse = pkg.ops.attention(*(torch.from_numpy(a).to(dev) for a in (q, k, v)), _scale(128),
                                 128, True, want_lse=True)
    (rt, at), (lrt, lat) = _tol(512)
    _close(out.cpu().numpy().astype(np.float32), want.astype(np.float32), rt, at, "peaked")
    _close(lse.cpu().numpy(), want_lse, lrt, lat, "peaked lse")


@pytest.mark.parametrize("kv_len,h,h_kv,d,split", [
    (1000, 32, 8, 128, 0), (1000, 8, 8, 64, 0), (777, 16, 8, 128, 5), (64, 4, 2, 64, 0),
    (1, 4, 4, 128, 0), (8191, 32, 8, 128, 0)])
def test_decode_bulk_path_matches_oracle(pkg, dev, kv_len, h, h_kv, d, split):
    rng = np.random.default_rng(kv_len + h)
    q, k, v = _rand(rng, 1, h, h_kv, kv_len, d)
    want, _ = oracle.attention(q, k, v, _scale(d), 0, False)
    qd, kd, vd = (torch.from_numpy(a).to(dev) for a in (q[0], k, v))
    out = pkg.ops.attention_decode(qd, kd, vd, _scale(d), split)
    (rt, at), _ = _tol(kv_len)
    _close(out.cpu().numpy().astype(np.float32), want[0].astype(np.float32), rt, at,
           f"decode kv_len={kv_len}")
    assert torch.equal(out, pkg.ops.attention_decode(qd, kd, vd, _scale(d), split))


@pytest.mark.parametrize("kv_len,h,h_kv", [
    (129, 16, 8),    # 2 query heads per KV head, 2 key blocks (cluster of 2, partial block)
    (640, 64, 8),    # 8 per KV head, cluster of 5
    (1024, 8, 8),    # 1 per KV head, cluster of 8
    (1025, 32, 8),   # 9 key blocks: cluster of 5 with two blocks each (two-stage ring),
                     # the last CTA one partial block
    (2048, 32, 8),   # 16 key blocks: cluster of 8 with two blocks each
    (2200, 32, 8),   # 18 key blocks: one-block splits through the workspace
    (3000, 16, 1),   # 16 query heads on one KV head (the widest group the MMA takes)
    (300, 32, 1)])   # 32 per KV head: beyond the tcgen05 decode, the bulk kernel
def test_decode_tcgen05_groups_and_splits(pkg, dev, kv_len, h, h_kv):
    """attention_decode at head_dim 128 with automatic splits runs on tcgen05:
    GQA groups of 1-16 heads, split merges inside a cluster and through the
    workspace; compared with the oracle (pinned to the reference's
    attention_cpu) under the reference's tolerances, and the LSE through the
    one-row non-causal prefill entry."""
    rng = np.random.default_rng(kv_len * 7 + h)
    q, k, v = _rand(rng, 1, h, h_kv, kv_len, 128)
    want, want_lse = oracle.attention(q, k, v, _scale(128), 0, False)
    qd, kd, vd = (torch.from_numpy(a).to(dev) for a in (q[0], k, v))
    out = pkg.ops.attention_decode(qd, kd, vd, _scale(128))
    (rt, at), (lrt, lat) = _tol(kv_len)
    _close(out.cpu().numpy().astype(np.float32), want[0].astype(np.float32), rt, at,
           f"tc decode kv_len={kv_len} h={h} h_kv={h_kv}")
    assert torch.equal(out, pkg.ops.attention_decode(qd, kd, vd, _scale(128)))
    out2, lse = pkg.ops.attention(qd[None], kd, vd, _scale(128), 0, False, want_lse=True)
    _close(out2[0].cpu().numpy().astype(np.float32), want[0].astype(np.float32), rt, at,
           "one-row prefill")
    _close(lse.cpu().numpy(), want_lse, lrt, lat, "one-row prefill lse")


@pytest.mark.parametrize("n_seq,s_new,h_kv,d,pitch_extra,pos", [
    (1, 5, 8, 128, 0, 3),      # the engine's contiguous form (16-byte copies)
    (3, 1, 2, 128, 4608, 7),   # three sequences, rows strided like a Q/K/V projection
    (2, 4, 3, 6, 2, 0)])       # head_dim 6: the element-wise path
def test_kv_cache_write_scatter_is_exact(pkg, dev, n_seq, s_new, h_kv, d, pitch_extra, pos):
    """kv_cache_write (kernels.hpp:184) and its strided batched form against the
    layout rule of kernels/attention_bridge.cu:45-56: token-major rows to
    head-major caches from pos, every other position untouched, bit for bit."""
    rng = np.random.default_rng(n_seq * 100 + s_new)
    max_len = pos + s_new + 2
    pitch = h_kv * d + pitch_extra
    rows = n_seq * s_new
    src = rng.standard_normal((rows, 2 * pitch)).astype(np.float16)
    k_rows, v_rows = src[:, :h_kv * d], src[:, pitch:pitch + h_kv * d]
    kc0 = rng.standard_normal((n_seq * h_kv, max_len, d)).astype(np.float16)
    vc0 = rng.standard_normal((n_seq * h_kv, max_len, d)).astype(np.float16)
    kc, vc = torch.from_numpy(kc0).to(dev), torch.from_numpy(vc0).to(dev)
    ts = torch.from_numpy(src).to(dev)
    if n_seq == 1 and pitch_extra == 0:
        kn = torch.from_numpy(np.ascontiguousarray(k_rows)).to(dev)
        vn = torch.from_numpy(np.ascontiguousarray(v_rows)).to(dev)
        pkg.cuda.kv_cache_write(kn.data_ptr(), vn.data_ptr(), kc.data_ptr(), vc.data_ptr(), s_new,
                                h_kv, d, pos, max_len)
    else:
        pkg.ops.kv_cache_write(ts[:, :h_kv * d], ts[:, pitch:pitch + h_kv * d], kc, vc, pos, n_seq)
    torch.cuda.synchronize()
    want_k, want_v = kc0.copy(), vc0.copy()
    for b in range(n_seq):
        for t in range(s_new):
            r = b * s_new + t
            want_k[b * h_kv:(b + 1) * h_kv, pos + t] = k_rows[r].reshape(h_kv, d)
            want_v[b * h_kv:(b + 1) * h_kv, pos + t] = v_rows[r].reshape(h_kv, d)
    assert np.array_equal(kc.cpu().numpy().view(np.uint16), want_k.view(np.uint16))
    assert np.array_equal(vc.cpu().numpy().view(np.uint16), want_v.view(np.uint16))


@pytest.mark.parametrize("N,K,kv_row0,h_kv,d,max_len,pos,gamma,resid", [
    (6144, 4096, 4096, 8, 128, 40, 17, True, False),   # Llama-3-8B Q/K/V, t = 1
    (768, 4096, 512, 1, 128, 16, 0, True, True),       # the t = 8 shard, residual
    (1536, 4096, 1024, 2, 128, 9, 8, False, False),    # t = 4 shard, unit gains, last slot
    (100, 64, 20, 5, 8, 3, 2, True, False)])           # small heads, the V rows end at row N
def test_rmsnorm_linear_kv_equals_projection_then_cache_write(pkg, dev, N, K, kv_row0, h_kv, d,
                                                              max_len, pos, gamma, resid):
    """engine_cuda_rmsnorm_linear_kv_f16 (the batch-1 Q/K/V projection that stores
    the token's K / V rows itself) against rmsnorm_linear_f16 at M = 1 followed
    by kv_cache_write of those rows: Y and both caches bit for bit, every other
    cache position untouched."""
    rng = np.random.default_rng(N + K + pos)
    x = torch.from_numpy(rng.standard_normal((1, K)).astype(np.float16)).to(dev)
    g = torch.from_numpy((1 + 0.1 * rng.standard_normal(K)).astype(np.float16)).to(dev) if gamma else None
    W = torch.from_numpy((rng.standard_normal((N, K)) * 0.02).astype(np.float16)).to(dev)
    R = torch.from_numpy(rng.standard_normal((1, N)).astype(np.float16)).to(dev) if resid else None
    kc0 = torch.from_numpy(rng.standard_normal((h_kv, max_len, d)).astype(np.float16)).to(dev)
    vc0 = torch.from_numpy(rng.standard_normal((h_kv, max_len, d)).astype(np.float16)).to(dev)
    kc, vc = kc0.clone(), vc0.clone()
    Y = torch.empty(1, N, device=dev, dtype=torch.float16)
    gp = g.data_ptr() if g is not None else 0
    rp = R.data_ptr() if R is not None else 0
    pkg.cuda.rmsnorm_linear_kv_f16(x.data_ptr(), gp, W.data_ptr(), rp, Y.data_ptr(), N, K, 1e-5,
                                   kc.data_ptr(), vc.data_ptr(), kv_row0, h_kv, d, max_len, pos)
    Y2 = torch.empty(1, N, device=dev, dtype=torch.float16)
    pkg.cuda.rmsnorm_linear_f16(x.data_ptr(), gp, W.data_ptr(), rp, Y2.data_ptr(), 1, N, K, 1e-5)
    kc2, vc2 = kc0.clone(), vc0.clone()
    n = h_kv * d
    pkg.ops.kv_cache_write(Y2[:, kv_row0:kv_row0 + n], Y2[:, kv_row0 + n:kv_row0 + 2 * n], kc2, vc2,
                           pos, 1)
    torch.cuda.synchronize()
    assert torch.equal(Y.view(torch.int16), Y2.view(torch.int16))
    assert torch.equal(kc.view(torch.int16), kc2.view(torch.int16))
    assert torch.equal(vc.view(torch.int16), vc2.view(torch.int16))
    assert not torch.equal(kc[:, pos], kc0[:, pos])  # the slot was written


@pytest.mark.parametrize("B,H,Hk,kv,max_len,check", [
    (3, 8, 2, 700, 800, (0, 1, 2)),       # 6 KV heads: each split one block, merged in a cluster
    (40, 32, 8, 1000, 1024, (0, 39))])    # 320 KV heads: one CTA per head streams 8 blocks
def test_batched_decode_matches_oracle(pkg, dev, B, H, Hk, kv, max_len, check):
    """A batch of equal-length sequences as one attention_decode call (the
    sequences folded into the KV-head dimension, as the layer set does) against
    the oracle per sequence; with few heads also bit for bit against one call
    per sequence (the same split plan per head)."""
    rng = np.random.default_rng(41 + B)
    d = 128
    q = rng.standard_normal((B * H, d)).astype(np.float16)
    kc = rng.standard_normal((B * Hk, max_len, d)).astype(np.float16)
    vc = rng.standard_normal((B * Hk, max_len, d)).astype(np.float16)
    tq, tk, tv = (torch.from_numpy(a).to(dev) for a in (q, kc, vc))
    batched = pkg.ops.attention_decode_cached(tq, tk, tv, kv)
    (rt, at), _ = _tol(kv)
    for b in check:
        got = batched[b * H:(b + 1) * H]
        if B * Hk < 64:
            one = pkg.ops.attention_decode_cached(tq[b * H:(b + 1) * H].contiguous(),
                                                  tk[b * Hk:(b + 1) * Hk].contiguous(),
                                                  tv[b * Hk:(b + 1) * Hk].contiguous(), kv)
            assert torch.equal(got, one), f"sequence {b}"
        want, _ = oracle.attention(q[None, b * H:(b + 1) * H], np.ascontiguousarray(kc[b * Hk:(b + 1) * Hk, :kv]),
                                   np.ascontiguousarray(vc[b * Hk:(b + 1) * Hk, :kv]), _scale(d), 0, False)
        _close(got.cpu().numpy().astype(np.float32), want[0].astype(np.float32), rt, at,
               f"decode sequence {b}")


def test_prefill_throughput_llama8b(pkg, dev):
    """Prints the tcgen05 prefill's rate at Llama-3-8B, S = 2048 causal (not asserted)."""
    H, H_kv, d, S = 32, 8, 128, 2048
    q = torch.randn(S, H, d, device=dev).half()
    k = torch.randn(H_kv, S, d, device=dev).half()
    v = torch.randn(H_kv, S, d, device=dev).half()
    out = torch.empty_like(q)
    st = torch.cuda.current_stream().cuda_stream
    fn = lambda: pkg.cuda.attention_prefill(q.data_ptr(), k.data_ptr(), v.data_ptr(),  # noqa: E731
                                            out.data_ptr(), S, S, H, H_kv, d, S * d, d ** -0.5,
                                            0, True, 0, st)
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(20):
        fn()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / 20
    print(f"attention_prefill Llama-3-8B S=2048 causal: {ms * 1e3:.1f} us, "
          f"{4.0 * S * S * d * H / 2 / (ms * 1e-3) / 1e12:.0f} TFLOP/s")
