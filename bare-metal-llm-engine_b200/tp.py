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

Per layer: x -> rmsnorm_linear(QKV) -> [attention stand-in] -> linear(O) ->
all-reduce -> rmsnorm_linear(gate/up) -> swiglu -> linear(down) -> all-reduce.
The residual add is folded into rank 0's O / down epilogue, so the all-reduced
sum is already x + sum_r proj_r.  Attention itself is out of scope for this
hot path: the stand-in passes each rank's q-head slice straight to O, which
keeps every token row independent (a row-sampled oracle stays exact).

The ``ops`` object performs the projections.  ``CudaOps`` is the product path
(the CUDA library); tests inject a CPU double to check the sharding and the
collective sequence on gloo ranks without a GPU.
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
    d = cfg.d_model // t
    return {
        "attn_norm": full["attn_norm"],
        "ffn_norm": full["ffn_norm"],
        "qkv": full["qkv"][qkv_rows_for_rank(cfg, t, r)].contiguous(),
        "o": full["o"][:, r * d:(r + 1) * d].contiguous(),
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

    def embedding(self, table, ids, out=None):
        return self._o.embedding(table, ids, out=out)


# ------------------------------------------------------------------ model

class TPLayerSet:
    """Rank-local state of the tensor-parallel layer set.

    ``layers`` is a list of shard dicts (see shard_layer), ``lm_head`` the vocab
    shard, ``embed`` the replicated token-embedding table, ``final_norm`` the
    final RMSNorm gain.
    """

    def __init__(self, cfg: TPConfig, rank: int, world: int, layers: list, lm_head, embed,
                 final_norm, ops=None, group=None):
        cfg.check(world)
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

    def _all_reduce(self, t):
        if self.world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)
            self.allreduce_count += 1
        return t

    def hidden(self, x):
        """Runs every layer on the replicated residual stream x [B, d_model]."""
        cfg, ops = self.cfg, self.ops
        qd = cfg.n_heads * cfg.head_dim // self.world
        f = cfg.ffn // self.world
        lead = self.rank == 0
        for L in self.layers:
            qkv = ops.rmsnorm_linear(x, L["attn_norm"], L["qkv"], cfg.eps)
            attn = qkv[:, :qd].contiguous()  # attention stand-in (out of scope)
            x = ops.linear(attn, L["o"], residual=x if lead else None)
            x = self._all_reduce(x)
            gu = ops.rmsnorm_linear(x, L["ffn_norm"], L["gate_up"], cfg.eps)
            h = ops.swiglu(gu[:, :f].contiguous(), gu[:, f:].contiguous())
            x = ops.linear(h, L["down"], residual=x if lead else None)
            x = self._all_reduce(x)
        return x

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
    d = cfg.d_model // world
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
            "o": rn((cfg.d_model, d), 10 * l + 3),
            "gate_up": rn((2 * f, cfg.d_model), 10 * l + 4),
            "down": rn((cfg.d_model, f), 10 * l + 5),
        })
    lm = rn((cfg.vocab // world, cfg.d_model), 999_001)
    g.manual_seed(seed)  # replicated on every rank
    embed = (torch.randn(cfg.vocab, cfg.d_model, device=device, generator=g) * 0.02).to(dtype)
    g.manual_seed(seed + 1)
    final_norm = (1 + 0.1 * torch.randn(cfg.d_model, device=device, generator=g)).to(dtype)
    return layers, lm, embed, final_norm


def weight_bytes_per_rank(cfg: TPConfig, world: int) -> float:
    per_layer = (cfg.qkv_rows * cfg.d_model + cfg.d_model * cfg.d_model +
                 2 * cfg.ffn * cfg.d_model + cfg.d_model * cfg.ffn) / world
    return 2.0 * (cfg.n_layers * per_layer + cfg.vocab * cfg.d_model / world)


def flops_per_token(cfg: TPConfig) -> float:
    per_layer = (cfg.qkv_rows * cfg.d_model + cfg.d_model * cfg.d_model +
                 2 * cfg.ffn * cfg.d_model + cfg.d_model * cfg.ffn)
    return 2.0 * (cfg.n_layers * per_layer + cfg.vocab * cfg.d_model)


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
    model = TPLayerSet(cfg, rank, world, layers, lm, embed, fnorm)
    prefill = args.workload == "tp-prefill"
    B = 2048 if prefill else args.batch
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
    line = {
        "metric": f"Llama-3-8B-shaped TP layer set {'prefill' if prefill else 'decode'} tokens/s",
        "value": tokens_s, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f16", "data": "synthetic: random N(0,0.02) FP16 weights",
        "config": {"workload": "tp-prefill" if prefill else "tp-decode", "model": "llama3-8b-shaped",
                   "layers": cfg.n_layers, "batch": B, "parallelism": f"tp{world}",
                   "attention": "stand-in (out of scope)", "cuda_graph": graph is not None},
        "per_gpu_weight_bytes": wbytes,
        "hbm_gbs_per_gpu": (wbytes / (ms * 1e-3) / 1e9) if not prefill else None,
        "tflops_per_gpu": (flops_per_token(cfg) * B / world / (ms * 1e-3) / 1e12),
        "allreduces_per_step": 2 * cfg.n_layers if world > 1 else 0,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    del graph
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0
