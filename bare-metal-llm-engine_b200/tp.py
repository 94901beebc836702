"""Tensor-parallel projection layer set (Llama-3-8B shapes) over the hot path.

One process per GPU.  Weights are FP16 [N,K] (K contiguous), sharded Megatron
style over t ranks:

* QKV  [6144, 4096]   column split, HEAD-ALIGNED: rank r holds q heads
  [r*32/t, (r+1)*32/t), k heads and v heads [r*8/t, (r+1)*8/t) -- its rows of the
  full matrix are gathered, not a contiguous slice;
* O    [4096, 4096]   row split on its input dim: rank r holds columns
  [r*4096/t, (r+1)*4096/t) (the local attention heads);
* gate/up [2*14336, 4096] column split, kept interleaved per rank (rows
  [0, 14336/t) = gate, [14336/t, 2*14336/t) = up) so SwiGLU stays local;
* down [4096, 14336]  row split on its input dim (14336/t columns per rank);
* LM head [128256, 4096] vocab split; greedy sampling = local argmax, then a
  tiny all-gather of (value, index) pairs.

Per layer: x -> rmsnorm_linear(QKV) -> attention -> linear(O) -> all-reduce ->
rmsnorm_linear_swiglu(gate/up, SwiGLU fused) -> linear(down) -> all-reduce.
The residual add is folded into rank 0's O / down epilogue, so the all-reduced
sum is already x + sum_r proj_r.

Attention is local to a rank (its query heads and their KV heads).  With
``enable_attention`` the layer set keeps per-layer head-major K / V caches and
runs the library's attention: the Q/K/V projection's K and V columns are
scattered into the caches (engine_cuda_kv_cache_write_rows), a prefill of one
sequence runs the tcgen05 FlashAttention kernel (attention_prefill, causal,
from the cached position), and decode -- one new token for each of n_seq
equal-length sequences -- is ONE attention_decode call with the sequences
folded into the KV-head dimension.  No RoPE is applied (positional encoding is
outside this hot path).  Without it, the stand-in passes each rank's q-head
slice straight to O, which keeps every token row independent (a row-sampled
oracle stays exact; the CPU tests use this form).

The ``ops`` object performs the projections.  ``CudaOps`` is the product path
(the CUDA library); tests inject a CPU double to check the sharding and the
collective sequence on gloo ranks without a GPU.

The all-reduces run through one of two collectives:
- ``NvlinkComm`` (engine_tp_*), when given and the message fits its capacity
  (decode).  The O / down projection and its all-reduce are then ONE kernel:
  every rank pushes its FP32 partial rows to every peer over NVLink and adds
  the world partials plus the residual in rank order.
- torch.distributed ``all_reduce`` otherwise (NCCL on GPUs, gloo in the CPU
  tests).  Prefill messages (16 MiB) take this path, where a ring beats a
  one-shot push.
"""
from __future__ import annotations

import json
import os
import statistics
import time
from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass(frozen=True)
class TPConfig:
    d_model: int = 4096
    n_heads: int = 32
    n_kv_heads: int = 8
    head_dim: int = 128
    ffn: int = 14336
    n_layers: int = 32
    vocab: int = 128256
    eps: float = 1e-5

    @property
    def qkv_rows(self) -> int:
        return (self.n_heads + 2 * self.n_kv_heads) * self.head_dim

    def check(self, t: int) -> None:
        for name, v in [("n_heads", self.n_heads), ("n_kv_heads", self.n_kv_heads),
                        ("ffn", self.ffn), ("vocab", self.vocab), ("d_model", self.d_model)]:
            if v % t:
                raise ValueError(f"{name}={v} is not divisible by the TP degree {t}")


LLAMA3_8B = TPConfig()


# ------------------------------------------------------------------ sharding

def qkv_rows_for_rank(cfg: TPConfig, t: int, r: int) -> torch.Tensor:
    """Row indices of W_qkv (q rows, then k rows, then v rows) owned by rank r."""
    hd = cfg.head_dim
    qh = cfg.n_heads // t
    kh = cfg.n_kv_heads // t
    q0 = r * qh * hd
    k0 = cfg.n_heads * hd + r * kh * hd
    v0 = (cfg.n_heads + cfg.n_kv_heads) * hd + r * kh * hd
    return torch.cat([torch.arange(q0, q0 + qh * hd), torch.arange(k0, k0 + kh * hd),
                      torch.arange(v0, v0 + kh * hd)])


def shard_layer(full: dict, cfg: TPConfig, t: int, r: int) -> dict:
    """Slices one layer's full weights ({qkv, o, gate, up, down, attn_norm,
    ffn_norm}) into rank r's shard."""
    f = cfg.ffn // t
    a = cfg.n_heads // t * cfg.head_dim  # O's input columns of this rank's query heads
    return {
        "attn_norm": full["attn_norm"],
        "ffn_norm": full["ffn_norm"],
        "qkv": full["qkv"][qkv_rows_for_rank(cfg, t, r)].contiguous(),
        "o": full["o"][:, r * a:(r + 1) * a].contiguous(),
        "gate_up": torch.cat([full["gate"][r * f:(r + 1) * f], full["up"][r * f:(r + 1) * f]]).contiguous(),
        "down": full["down"][:, r * f:(r + 1) * f].contiguous(),
    }


def shard_head(full_lm: torch.Tensor, cfg: TPConfig, t: int, r: int) -> torch.Tensor:
    v = cfg.vocab // t
    return full_lm[r * v:(r + 1) * v].contiguous()


# ------------------------------------------------------------------ ops

class CudaOps:
    """The product path: every projection is a call into libengine_b200.so."""

    def __init__(self):
        from . import ops

        self._o = ops

    def rmsnorm_linear(self, x, gamma, W, eps, residual=None, out=None):
        return self._o.rmsnorm_linear(x, gamma, W, eps, residual=residual, out=out)

    def linear(self, x, W, residual=None, out=None):
        return self._o.linear(x, W, residual=residual, out=out)

    def swiglu(self, g, u, out=None):
        return self._o.swiglu(g, u, out=out)

    def rmsnorm_linear_swiglu(self, x, gamma, W_gu, eps, out=None):
        return self._o.rmsnorm_linear_swiglu(x, gamma, W_gu, eps, out=out)

    def kv_cache_write(self, k_rows, v_rows, k_cache, v_cache, pos, n_seq=1):
        self._o.kv_cache_write(k_rows, v_rows, k_cache, v_cache, pos, n_seq)

    def rmsnorm_linear_kv(self, x, gamma, W, eps, k_cache, v_cache, kv_row0, pos, out=None):
        return self._o.rmsnorm_linear_kv(x, gamma, W, eps, k_cache, v_cache, kv_row0, pos, out=out)

    def attention_prefill(self, q, k_cache, v_cache, kv_len, q_pos_offset):
        return self._o.attention_cached(q, k_cache, v_cache, kv_len, q_pos_offset, True)

    def attention_decode(self, q, k_cache, v_cache, kv_len):
        return self._o.attention_decode_cached(q, k_cache, v_cache, kv_len)

    def embedding(self, table, ids, out=None):
        return self._o.embedding(table, ids, out=out)


# ------------------------------------------------------------------ collective

class NvlinkComm:
    """The library's tensor-parallel communicator on this rank's current GPU.

    The exchange regions' CUDA IPC handles are all-gathered through
    torch.distributed (``group``); ``max_elems`` bounds the elements of one
    call (B x d_model for decode).  Every rank must make the same calls in the
    same order on one stream.
    """

    def __init__(self, rank: int, world: int, max_elems: int, group=None):
        from . import cuda as _c
        from . import ops as _ops

        self._c = _c
        self._ops = _ops
        self.rank, self.world, self.max_elems, self.group = rank, world, int(max_elems), group
        self.handle = _c.tp_comm_create(rank, world, self.max_elems)
        mine = _c.tp_comm_handle(self.handle)
        if world > 1:
            parts = [None] * world
            dist.all_gather_object(parts, mine, group=group)
            handles = b"".join(parts)
        else:
            handles = mine
        _c.tp_comm_open(self.handle, handles)

    def fits(self, rows: int, cols: int) -> bool:
        return rows * cols <= self.max_elems

    def linear_allreduce(self, x, W, residual=None, out=None):
        """sum over ranks of x_r @ W_r^T (+ residual), on every rank."""
        o = self._ops
        o._req(x, torch.float16, "x")
        o._req(W, torch.float16, "W")
        if residual is not None:
            o._req(residual, torch.float16, "residual")
        M, K = x.shape
        N = W.shape[0]
        Y = out if out is not None else torch.empty(M, N, device=x.device, dtype=torch.float16)
        self._c.tp_linear_allreduce_f16(self.handle, x.data_ptr(), W.data_ptr(),
                                        o._ptr(residual), Y.data_ptr(), M, N, K, o._stream())
        return Y

    def allreduce(self, partial, residual=None, out=None):
        """sum over ranks of partial (+ residual), on every rank."""
        o = self._ops
        o._req(partial, torch.float16, "partial")
        if residual is not None:
            o._req(residual, torch.float16, "residual")
        Y = out if out is not None else torch.empty_like(partial)
        self._c.tp_allreduce_f16(self.handle, partial.data_ptr(), o._ptr(residual), Y.data_ptr(),
                                 partial.numel(), o._stream())
        return Y

    def close(self):
        """Host barrier over the group, then frees the region (every rank)."""
        if self.handle:
            torch.cuda.synchronize()
            if self.world > 1:
                dist.barrier(group=self.group)
            self._c.tp_comm_destroy(self.handle)
            self.handle = 0


# ------------------------------------------------------------------ model

class TPLayerSet:
    """Rank-local state of the tensor-parallel layer set.

    ``layers`` is a list of shard dicts (see shard_layer), ``lm_head`` the vocab
    shard, ``embed`` the replicated token-embedding table, ``final_norm`` the
    final RMSNorm gain.
    """

    def __init__(self, cfg: TPConfig, rank: int, world: int, layers: list, lm_head, embed,
                 final_norm, ops=None, group=None, comm=None):
        cfg.check(world)
        self.comm = comm
        self.cfg = cfg
        self.rank = rank
        self.world = world
        self.layers = layers
        self.lm_head = lm_head
        self.embed = embed
        self.final_norm = final_norm
        self.ops = ops if ops is not None else CudaOps()
        self.group = group
        self.allreduce_count = 0
        self.kv = None  # per-layer (k_cache, v_cache) once enable_attention ran
        self.pos = 0  # cached positions before this step (every sequence alike)
        self.n_seq = 1
        self.max_len = 0

    def enable_attention(self, max_len: int, n_seq: int = 1, pos: int = 0,
                         dtype=torch.float16):
        """Replaces the stand-in by attention over per-layer K / V caches
        [n_seq * n_kv_heads / t, max_len, head_dim] (zero-filled; FP16 for the
        library, float64 for the CPU test double).  ``pos`` = positions already
        cached; a step attends to positions [0, pos + new) and does not advance
        ``pos`` (set it between steps)."""
        cfg = self.cfg
        hk = cfg.n_kv_heads // self.world
        dev = self.embed.device
        self.kv = [(torch.zeros(n_seq * hk, max_len, cfg.head_dim, device=dev, dtype=dtype),
                    torch.zeros(n_seq * hk, max_len, cfg.head_dim, device=dev, dtype=dtype))
                   for _ in self.layers]
        self.n_seq, self.max_len, self.pos = n_seq, max_len, pos

    def _attention(self, qkv, li: int, cached: bool = False):
        """Rank-local attention of one layer: qkv [rows, (hq + 2 hk) * d] -> [rows, hq * d].
        cached: the projection has already stored this token's K / V rows."""
        cfg, ops = self.cfg, self.ops
        d = cfg.head_dim
        hq = cfg.n_heads // self.world
        hk = cfg.n_kv_heads // self.world
        qd, kd = hq * d, hk * d
        rows = qkv.shape[0]
        kc, vc = self.kv[li]
        q = qkv[:, :qd].contiguous()
        k_rows, v_rows = qkv[:, qd:qd + kd], qkv[:, qd + kd:qd + 2 * kd]
        if self.n_seq > 1 or rows == 1:  # decode: one new token per sequence
            if rows != self.n_seq:
                raise ValueError(f"decode step of {rows} tokens for {self.n_seq} sequences")
            if self.pos + 1 > self.max_len:
                raise ValueError("KV cache full")
            if not cached:
                ops.kv_cache_write(k_rows, v_rows, kc, vc, self.pos, n_seq=rows)
            out = ops.attention_decode(q.view(rows * hq, d), kc, vc, self.pos + 1)
        else:  # prefill of one sequence: `rows` tokens from position pos
            if self.pos + rows > self.max_len:
                raise ValueError("KV cache full")
            ops.kv_cache_write(k_rows, v_rows, kc, vc, self.pos, n_seq=1)
            out = ops.attention_prefill(q.view(rows, hq, d), kc, vc, self.pos + rows, self.pos)
        return out.view(rows, qd)

    def _all_reduce(self, t):
        if self.world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)
            self.allreduce_count += 1
        return t

    def hidden(self, x):
        """Runs every layer on the replicated residual stream x [B, d_model]."""
        cfg, ops = self.cfg, self.ops
        qd = cfg.n_heads * cfg.head_dim // self.world
        lead = self.rank == 0
        fused = (self.comm is not None and self.world > 1
                 and self.comm.fits(x.shape[0], cfg.d_model))
        # Decode of one sequence: the Q/K/V projection stores the token's K / V
        # rows into the caches itself (one kernel instead of two per layer).
        fuse_kv = (self.kv is not None and x.shape[0] == 1 and self.n_seq == 1
                   and hasattr(ops, "rmsnorm_linear_kv") and self.pos + 1 <= self.max_len)
        for li, L in enumerate(self.layers):
            if fuse_kv:
                kc, vc = self.kv[li]
                qkv = ops.rmsnorm_linear_kv(x, L["attn_norm"], L["qkv"], cfg.eps, kc, vc, qd,
                                            self.pos)
            else:
                qkv = ops.rmsnorm_linear(x, L["attn_norm"], L["qkv"], cfg.eps)
            if self.kv is not None:
                attn = self._attention(qkv, li, cached=fuse_kv)
            else:
                attn = qkv[:, :qd].contiguous()  # stand-in: the q-head slice
            x = self._row_split(attn, L["o"], x, lead, fused)
            # gate/up projection with the SwiGLU fused (one kernel at batch 1)
            h = ops.rmsnorm_linear_swiglu(x, L["ffn_norm"], L["gate_up"], cfg.eps)
            x = self._row_split(h, L["down"], x, lead, fused)
        return x

    def _row_split(self, a, W, x, lead, fused):
        """x + sum over ranks of a_r @ W_r^T (the O / down projection)."""
        if fused:
            self.allreduce_count += 1
            return self.comm.linear_allreduce(a, W, residual=x)
        y = self.ops.linear(a, W, residual=x if lead else None)
        return self._all_reduce(y)

    def logits_shard(self, x):
        return self.ops.rmsnorm_linear(x, self.final_norm, self.lm_head, self.cfg.eps)

    def greedy(self, logits):
        """Global argmax over the vocab shards (lowest index wins ties)."""
        val, idx = logits.float().max(dim=-1)
        idx = idx + self.rank * (self.cfg.vocab // self.world)
        if self.world == 1:
            return idx.to(torch.int32)
        vals = [torch.empty_like(val) for _ in range(self.world)]
        idxs = [torch.empty_like(idx) for _ in range(self.world)]
        dist.all_gather(vals, val, group=self.group)
        dist.all_gather(idxs, idx, group=self.group)
        V = torch.stack(vals)  # [world, B]
        I = torch.stack(idxs)
        best = V.max(dim=0, keepdim=True).values
        cand = torch.where(V == best, I, torch.full_like(I, torch.iinfo(I.dtype).max))
        return cand.min(dim=0).values.to(torch.int32)

    def step(self, ids):
        """One decode / prefill pass: token ids [B] -> next token ids [B]."""
        x = self.ops.embedding(self.embed, ids)
        x = self.hidden(x)
        return self.greedy(self.logits_shard(x))


# ------------------------------------------------------------------ weights

def random_shards(cfg: TPConfig, rank: int, world: int, device, seed: int = 20260826,
                  dtype=torch.float16):
    """Rank-local random shards (~N(0,0.02) weights, ~1+N(0,0.1) gains) drawn
    directly on the device; the same (seed, layer, rank) gives the same shard."""
    g = torch.Generator(device=device)
    f = cfg.ffn // world
    a = cfg.n_heads // world * cfg.head_dim  # O's input columns: this rank's query heads
    qkv = cfg.qkv_rows // world

    def rn(shape, salt, scale=0.02, replicated=False):
        g.manual_seed(seed * 1000003 + salt * 131 + (0 if replicated else 7919 * (rank + 1)))
        return (torch.randn(shape, device=device, generator=g) * scale).to(dtype)

    def gain(salt):  # identical on every rank: the residual stream is replicated
        return (1 + rn((cfg.d_model,), salt, 0.1, replicated=True).float()).to(dtype)

    layers = []
    for l in range(cfg.n_layers):
        layers.append({
            "attn_norm": gain(10 * l + 0),
            "ffn_norm": gain(10 * l + 1),
            "qkv": rn((qkv, cfg.d_model), 10 * l + 2),
            "o": rn((cfg.d_model, a), 10 * l + 3),
            "gate_up": rn((2 * f, cfg.d_model), 10 * l + 4),
            "down": rn((cfg.d_model, f), 10 * l + 5),
        })
    lm = rn((cfg.vocab // world, cfg.d_model), 999_001)
    g.manual_seed(seed)  # replicated on every rank
    embed = (torch.randn(cfg.vocab, cfg.d_model, device=device, generator=g) * 0.02).to(dtype)
    g.manual_seed(seed + 1)
    final_norm = (1 + 0.1 * torch.randn(cfg.d_model, device=device, generator=g)).to(dtype)
    return layers, lm, embed, final_norm


def _layer_weights(cfg: TPConfig) -> int:
    """Elements of one layer's projections: QKV, O (d_model x the query heads'
    width), gate and up, down."""
    return (cfg.qkv_rows * cfg.d_model + cfg.d_model * cfg.n_heads * cfg.head_dim +
            2 * cfg.ffn * cfg.d_model + cfg.d_model * cfg.ffn)


def weight_bytes_per_rank(cfg: TPConfig, world: int) -> float:
    per_layer = _layer_weights(cfg) / world
    return 2.0 * (cfg.n_layers * per_layer + cfg.vocab * cfg.d_model / world)


def flops_per_token(cfg: TPConfig) -> float:
    per_layer = _layer_weights(cfg)
    return 2.0 * (cfg.n_layers * per_layer + cfg.vocab * cfg.d_model)


# Decode steps attend to this many cached positions (the new token included).
DECODE_CONTEXT = 1024


def attention_prefill_flops(cfg: TPConfig, S: int) -> float:
    """Causal attention of an S-token prefill from position 0, all layers:
    Q K^T and P V over the S (S + 1) / 2 visible (row, key) pairs."""
    return 4.0 * cfg.head_dim * cfg.n_heads * S * (S + 1) / 2 * cfg.n_layers


def kv_bytes_per_rank(cfg: TPConfig, world: int, n_seq: int, kv_len: int) -> float:
    """K and V bytes a decode step reads from the caches on one rank."""
    return 2.0 * 2 * cfg.n_layers * n_seq * (cfg.n_kv_heads // world) * kv_len * cfg.head_dim


# ------------------------------------------------------------------ benchmark

def bench_main(args, metric: str) -> int:
    """bench.py --workload tp-decode|tp-prefill: the layer set on every rank."""
    import datetime

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    cfg = LLAMA3_8B
    layers, lm, embed, fnorm = random_shards(cfg, rank, world, dev)
    prefill = args.workload == "tp-prefill"
    B = 2048 if prefill else args.batch
    comm = None
    collective = "none" if world == 1 else "nccl all_reduce"
    if world > 1 and not prefill and os.environ.get("ENGINE_TP_COMM", "nvlink") != "nccl":
        comm = NvlinkComm(rank, world, B * cfg.d_model)
        collective = "nvlink one-shot all-reduce fused into the O / down projection"
    model = TPLayerSet(cfg, rank, world, layers, lm, embed, fnorm, comm=comm)
    if prefill:
        model.enable_attention(B)
    else:
        model.enable_attention(DECODE_CONTEXT, n_seq=B, pos=DECODE_CONTEXT - 1)
    gen = torch.Generator(device=dev).manual_seed(7)
    ids = torch.randint(0, cfg.vocab, (B,), device=dev, generator=gen, dtype=torch.int32)
    if world > 1:
        dist.broadcast(ids, 0)
    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        out = model.step(ids)
    torch.cuda.synchronize()
    graph = None
    if not prefill:
        # Capture the whole decode step (kernels + NCCL all-reduces) in one graph.
        graph = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(stream)
        with torch.cuda.stream(s):
            model.step(ids)
        stream.wait_stream(s)
        torch.cuda.synchronize()
        with torch.cuda.graph(graph):
            out = model.step(ids)
        torch.cuda.synchronize()
        for _ in range(3):
            graph.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        if graph is not None:
            graph.replay()
        else:
            out = model.step(ids)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item()) / args.steps
    tokens_s = B / (ms * 1e-3)
    wbytes = weight_bytes_per_rank(cfg, world)
    kvb = 0.0 if prefill else kv_bytes_per_rank(cfg, world, B, DECODE_CONTEXT)
    flops = flops_per_token(cfg) * B + (attention_prefill_flops(cfg, B) if prefill else 0.0)
    line = {
        "metric": f"Llama-3-8B-shaped TP layer set {'prefill' if prefill else 'decode'} tokens/s",
        "value": tokens_s, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f16", "data": "synthetic: random N(0,0.02) FP16 weights",
        "config": {"workload": "tp-prefill" if prefill else "tp-decode", "model": "llama3-8b-shaped",
                   "layers": cfg.n_layers, "batch": B, "parallelism": f"tp{world}",
                   "attention": ("tcgen05, causal from position 0" if prefill else
                                 f"tcgen05 decode over {DECODE_CONTEXT} cached positions"),
                   "cuda_graph": graph is not None,
                   "collective": collective},
        "per_gpu_weight_bytes": wbytes,
        "per_gpu_kv_bytes": kvb,
        "hbm_gbs_per_gpu": ((wbytes + kvb) / (ms * 1e-3) / 1e9) if not prefill else None,
        "tflops_per_gpu": flops / world / (ms * 1e-3) / 1e12,
        "allreduces_per_step": 2 * cfg.n_layers if world > 1 else 0,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    del graph
    if comm is not None:
        comm.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def full_random_weights(cfg: TPConfig, device, seed: int = 11, dtype=torch.float16):
    """Unsharded random weights drawn on `device` from a seeded device generator:
    every GPU draws the same values for the same seed, so each rank can shard
    them itself (the parity check of the sharded layer set against t = 1)."""
    g = torch.Generator(device=device).manual_seed(seed)

    def rn(*shape, scale=0.02):
        return (torch.randn(*shape, device=device, generator=g) * scale).to(dtype)

    layers = []
    for _ in range(cfg.n_layers):
        layers.append({
            "attn_norm": (1 + rn(cfg.d_model, scale=0.1).float()).to(dtype),
            "ffn_norm": (1 + rn(cfg.d_model, scale=0.1).float()).to(dtype),
            "qkv": rn(cfg.qkv_rows, cfg.d_model),
            "o": rn(cfg.d_model, cfg.n_heads * cfg.head_dim),
            "gate": rn(cfg.ffn, cfg.d_model),
            "up": rn(cfg.ffn, cfg.d_model),
            "down": rn(cfg.d_model, cfg.ffn),
        })
    lm = rn(cfg.vocab, cfg.d_model)
    embed = rn(cfg.vocab, cfg.d_model, scale=1.0)
    fnorm = (1 + rn(cfg.d_model, scale=0.1).float()).to(dtype)
    return layers, lm, embed, fnorm


# Parity headroom of the t = N layer set against t = 1: each op is pinned to the
# oracle by its own test; the chains differ only in rounding (every rank rounds
# its partial projection to FP16 before the sum at t > 1, t = 1 rounds once).
# One FP16 ulp at the hidden state's magnitude (|x| < 8) is <= 2^-8; a few ulps
# per op over a two-layer chain stay inside 2e-2 absolute + 2e-2 relative, the
# same kind of documented headroom the reference uses for stacked layers
# (tests/test_kernels.cu:3387-3390).
TP_PARITY_ATOL = 2e-2
TP_PARITY_RTOL = 2e-2
TP_PARITY_TOKENS = (0, 5, 128255, 4242)


def _max_over_ranks(x: float, world: int, dev) -> float:
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def tp_parity(cfg: TPConfig, world: int, rank: int, dev, comm=None) -> dict:
    """The t = N layer set (two layers, the product's own sharding) against t = 1
    on the same weights: every rank's hidden state and logits shard, once with
    NCCL all-reduces and once with the NVLink communicator when given.  Rank 0
    computes t = 1 and broadcasts it.  Returns {"ok", "max_abs_err", ...}, the
    same on every rank."""
    import dataclasses

    pcfg = dataclasses.replace(cfg, n_layers=2)
    layers, lm, embed, fnorm = full_random_weights(pcfg, dev)
    ids = torch.tensor(TP_PARITY_TOKENS, dtype=torch.int32, device=dev)
    shards = [shard_layer(L, pcfg, world, rank) for L in layers]
    m = TPLayerSet(pcfg, rank, world, shards, shard_head(lm, pcfg, world, rank), embed, fnorm)
    ops = m.ops
    B = len(TP_PARITY_TOKENS)
    m.enable_attention(B)  # the tokens as one causal sequence: the real attention
    ref_x = torch.empty(B, pcfg.d_model, device=dev, dtype=torch.float16)
    ref_l = torch.empty(B, pcfg.vocab, device=dev, dtype=torch.float16)
    if rank == 0:
        m1 = TPLayerSet(pcfg, 0, 1, [shard_layer(L, pcfg, 1, 0) for L in layers], lm, embed, fnorm)
        m1.enable_attention(B)
        x1 = m1.hidden(ops.embedding(embed, ids))
        ref_x.copy_(x1)
        ref_l.copy_(m1.logits_shard(x1))
        del m1
    if world > 1:
        dist.broadcast(ref_x, 0)
        dist.broadcast(ref_l, 0)
    v = pcfg.vocab // world
    want_l = ref_l[:, rank * v:(rank + 1) * v].float()
    res = {"ok": True, "max_abs_err": 0.0, "layers": pcfg.n_layers, "tokens": B,
           "atol": TP_PARITY_ATOL, "rtol": TP_PARITY_RTOL, "collectives": []}
    for name, c in (("nccl", None), ("nvlink", comm)):
        if name == "nvlink" and (c is None or world == 1):
            continue
        m.comm = c
        m.allreduce_count = 0
        x = m.hidden(ops.embedding(embed, ids))
        lg = m.logits_shard(x)
        err_x = (x.float() - ref_x.float()).abs()
        err_l = (lg.float() - want_l).abs()
        ok = bool((err_x <= TP_PARITY_ATOL + TP_PARITY_RTOL * ref_x.float().abs()).all() and
                  (err_l <= TP_PARITY_ATOL + TP_PARITY_RTOL * want_l.abs()).all() and
                  m.allreduce_count == (2 * pcfg.n_layers if world > 1 else 0))
        bad = _max_over_ranks(0.0 if ok else 1.0, world, dev)
        err = _max_over_ranks(max(err_x.max().item(), err_l.max().item()), world, dev)
        res["ok"] = res["ok"] and bad == 0.0
        res["max_abs_err"] = max(res["max_abs_err"], err)
        res["collectives"].append(name)
    m.comm = None
    return res


def _time_tp_step(model, ids, steps: int, warmup: int, graph: bool, world: int, dev) -> float:
    """ms per step of model.step(ids), max over ranks; the whole step in one CUDA
    graph when `graph` (released before returning)."""
    stream = torch.cuda.current_stream()
    for _ in range(warmup):
        model.step(ids)
    torch.cuda.synchronize()
    g = None
    if graph:
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(stream)
        with torch.cuda.stream(s):
            model.step(ids)
        stream.wait_stream(s)
        torch.cuda.synchronize()
        with torch.cuda.graph(g):
            model.step(ids)
        torch.cuda.synchronize()
        for _ in range(2):
            g.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        if g is not None:
            g.replay()
        else:
            model.step(ids)
    e1.record(stream)
    torch.cuda.synchronize()
    del g
    return _max_over_ranks(e0.elapsed_time(e1) / steps, world, dev)


def _time_calls(fn, calls: int, world: int, dev, graph: bool = True) -> float:
    """us per call of fn() (CUDA graph of `calls` calls when `graph`), max over ranks."""
    stream = torch.cuda.current_stream()
    s = torch.cuda.Stream()
    s.wait_stream(stream)
    with torch.cuda.stream(s):
        for _ in range(3):
            fn()
    torch.cuda.synchronize()
    g = None
    if graph:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for _ in range(calls):
                fn()
        g.replay()
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    if g is not None:
        g.replay()
    else:
        for _ in range(calls):
            fn()
    e1.record(stream)
    torch.cuda.synchronize()
    del g
    return _max_over_ranks(e0.elapsed_time(e1) * 1e3 / calls, world, dev)


def bench_tp_block(steps: int, warmup: int, hbm_peak: float, tensor_peak: float,
                   peak_kind: str) -> dict:
    """The Llama-3-8B-shaped tensor-parallel layer set at t = the process group's
    size (1 without one), for bench.py's JSON line: decode B = 1 and B = 32 (one
    CUDA graph per step; the library's NVLink communicator fused into O / down
    at t > 1), prefill S = 2048 (NCCL all-reduces), the all-reduces alone, and
    the t = N vs t = 1 parity check.  Every rank takes the same steps; the
    figures are max over ranks."""
    world = dist.get_world_size() if dist.is_initialized() else 1
    rank = dist.get_rank() if dist.is_initialized() else 0
    dev = torch.device("cuda", torch.cuda.current_device())
    cfg = LLAMA3_8B
    comm = NvlinkComm(rank, world, 32 * cfg.d_model) if world > 1 else None
    out = {"t": world, "model": "llama3-8b-shaped", "layers": cfg.n_layers,
           "attention": (f"the library's tcgen05 attention over per-layer KV caches: decode attends "
                         f"to {DECODE_CONTEXT} cached positions (batch = sequences), prefill is "
                         f"causal from position 0; no RoPE"),
           "nccl_ranks": dist.get_world_size() if dist.is_initialized() else 0,
           "collective_decode": ("nvlink one-shot all-reduce fused into the O / down projection"
                                 if comm is not None else "none (t = 1)"),
           "collective_prefill": "nccl all_reduce" if world > 1 else "none (t = 1)",
           "peak_kind": peak_kind}
    if world > 1:
        out["parity"] = tp_parity(cfg, world, rank, dev, comm)
        out["parity_ok"] = out["parity"]["ok"]
    else:
        out["parity_ok"] = None
        out["parity"] = "t = 1 is the reference of the t = N check"
    torch.cuda.empty_cache()
    layers, lm, embed, fnorm = random_shards(cfg, rank, world, dev)
    wbytes = weight_bytes_per_rank(cfg, world)
    gen = torch.Generator(device=dev).manual_seed(7)
    for B in (1, 32):
        model = TPLayerSet(cfg, rank, world, layers, lm, embed, fnorm, comm=comm)
        model.enable_attention(DECODE_CONTEXT, n_seq=B, pos=DECODE_CONTEXT - 1)
        ids = torch.randint(0, cfg.vocab, (B,), device=dev, generator=gen, dtype=torch.int32)
        if world > 1:
            dist.broadcast(ids, 0)
        ms = _time_tp_step(model, ids, max(steps, 10), warmup, True, world, dev)
        kvb = kv_bytes_per_rank(cfg, world, B, DECODE_CONTEXT)
        gbs = (wbytes + kvb) / (ms * 1e-3) / 1e9
        out[f"decode_b{B}"] = {"ms_per_step": ms, "tokens_s": B / (ms * 1e-3),
                               "kv_bytes_per_gpu": kvb,
                               "hbm_gbs_per_gpu": gbs, "hbm_frac_per_gpu": gbs / hbm_peak}
        del model
        torch.cuda.empty_cache()
    # prefill S = 2048, eager (16 MiB all-reduces over NCCL)
    S = 2048
    model = TPLayerSet(cfg, rank, world, layers, lm, embed, fnorm, comm=None)
    model.enable_attention(S)
    ids = torch.randint(0, cfg.vocab, (S,), device=dev, generator=gen, dtype=torch.int32)
    if world > 1:
        dist.broadcast(ids, 0)
    ms = _time_tp_step(model, ids, max(3, min(steps, 8)), min(warmup, 3), False, world, dev)
    tf = (flops_per_token(cfg) * S + attention_prefill_flops(cfg, S)) / world / (ms * 1e-3) / 1e12
    out["prefill_s2048"] = {"ms_per_step": ms, "tokens_s": S / (ms * 1e-3),
                            "tflops_per_gpu": tf, "tensor_frac_per_gpu": tf / tensor_peak}
    # The all-reduces alone at the step's message sizes (64 per step), for the share.
    if world > 1:
        calls = 2 * cfg.n_layers
        for B in (1, 32):
            P = torch.randn(B * cfg.d_model, device=dev, generator=gen).half()
            Y = torch.empty_like(P)
            us = _time_calls(lambda: comm.allreduce(P, out=Y), calls, world, dev)
            out[f"decode_b{B}"]["allreduce_us"] = us
            out[f"decode_b{B}"]["allreduce_share_est"] = calls * us * 1e-3 / out[f"decode_b{B}"]["ms_per_step"]
        P = torch.randn(S * cfg.d_model, device=dev, generator=gen).half()
        us = _time_calls(lambda: dist.all_reduce(P), 8, world, dev, graph=False)
        out["prefill_s2048"]["allreduce_us"] = us
        out["prefill_s2048"]["allreduce_share_est"] = calls * us * 1e-3 / out["prefill_s2048"]["ms_per_step"]
        del P, Y
    del model, layers, lm, embed, fnorm
    if comm is not None:
        comm.close()
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return out


def bench_collectives(args) -> int:
    """bench.py --workload tp-comm (one process per GPU, world >= 2): device time
    per call of the row-split projection + all-reduce at the decode shapes,
    NVLink fused vs GEMV/GEMM + NVLink all-reduce vs GEMV/GEMM + NCCL, and the
    all-reduces alone.  Each figure is one CUDA graph of 64 back-to-back calls,
    replayed 5 times, max over ranks."""
    import datetime

    from . import ops

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world < 2:
        if rank == 0:
            print(json.dumps({"workload": "tp-comm", "unavailable": "needs >= 2 GPUs (torchrun)"}))
        return 0
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    cfg = LLAMA3_8B
    comm = NvlinkComm(rank, world, 32 * cfg.d_model)
    calls = 64

    def timed(fn):
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(max(args.warmup, 3)):
                fn()
        torch.cuda.synchronize()
        dist.barrier()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for _ in range(calls):
                fn()
        g.replay()
        torch.cuda.synchronize()
        dist.barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(5):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) * 1e3 / (5 * calls)], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        del g
        return float(t.item())

    gen = torch.Generator(device=dev).manual_seed(1234 + rank)
    out = {}
    for name, M, K in (("o_b1", 1, cfg.d_model // world), ("down_b1", 1, cfg.ffn // world),
                       ("down_b32", 32, cfg.ffn // world)):
        N = cfg.d_model
        X = torch.randn(M, K, device=dev, generator=gen).half()
        W = (torch.randn(N, K, device=dev, generator=gen) * 0.02).half()
        R = torch.randn(M, N, device=dev, generator=gen).half()
        Y = torch.empty(M, N, device=dev, dtype=torch.float16)
        P = torch.empty(M, N, device=dev, dtype=torch.float16)

        def nccl_path():
            ops.linear(X, W, residual=R if rank == 0 else None, out=Y)
            dist.all_reduce(Y)

        def nv_unfused():
            ops.linear(X, W, out=P)
            comm.allreduce(P, residual=R, out=Y)

        out[name] = {
            "projection_alone_us": timed(lambda: ops.linear(X, W, residual=R, out=Y)),
            "nvlink_fused_us": timed(lambda: comm.linear_allreduce(X, W, residual=R, out=Y)),
            "projection_then_nvlink_allreduce_us": timed(nv_unfused),
            "projection_then_nccl_allreduce_us": timed(nccl_path),
        }
    for n in (cfg.d_model, 32 * cfg.d_model):
        P = torch.randn(n, device=dev, generator=gen).half()
        Y = torch.empty_like(P)
        out[f"allreduce_{n * 2 // 1024}KiB"] = {
            "nvlink_us": timed(lambda: comm.allreduce(P, out=Y)),
            "nccl_us": timed(lambda: dist.all_reduce(P)),
        }
    line = {"metric": "TP row-split projection + all-reduce, device us per call (decode shapes)",
            "unit": "us", "higher_is_better": False, "n_gpus": world,
            "config": {"workload": "tp-comm", "model": "llama3-8b-shaped", "parallelism": f"tp{world}",
                       "timing": f"CUDA graph of {calls} calls x 5 replays, max over ranks"},
            "results": out}
    if rank == 0:
        print(json.dumps(line), flush=True)
    comm.close()
    dist.barrier()
    dist.destroy_process_group()
    return 0

