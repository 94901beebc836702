"""TEST DOUBLE: CPU float64 stand-ins for the CUDA projections of the TP layer.

Used only by the gloo tests to exercise the tensor-parallel sharding and the
collective sequence on CPU ranks, including the per-rank attention heads and
their KV caches (float64 softmax attention, the reference's two-pass form).  The arithmetic is the reference's composition
(rmsnorm -> matmul -> swiglu -> vector_add, tests/test_kernels.cu:2813-2938) in
float64 with the result kept in float64, so sharded and unsharded runs can be
compared tightly.
"""
from __future__ import annotations

import torch


class CpuOps:
    def __init__(self):
        self.calls = []

    def rmsnorm_linear(self, x, gamma, W, eps, residual=None, out=None):
        self.calls.append("rmsnorm_linear")
        x64 = x.double()
        t = x64 * torch.rsqrt((x64 * x64).mean(-1, keepdim=True) + eps)
        if gamma is not None:
            t = t * gamma.double()
        y = t @ W.double().T
        return y if residual is None else y + residual.double()

    def linear(self, x, W, residual=None, out=None):
        self.calls.append("linear")
        y = x.double() @ W.double().T
        return y if residual is None else y + residual.double()

    def swiglu(self, g, u, out=None):
        self.calls.append("swiglu")
        g = g.double()
        return g / (1 + torch.exp(-g)) * u.double()

    def rmsnorm_linear_swiglu(self, x, gamma, W_gu, eps, out=None):
        self.calls.append("rmsnorm_linear_swiglu")
        gu = self.rmsnorm_linear(x, gamma, W_gu, eps)
        f = W_gu.shape[0] // 2
        return self.swiglu(gu[:, :f], gu[:, f:])

    def embedding(self, table, ids, out=None):
        self.calls.append("embedding")
        return table[ids.long()].double()

    def rmsnorm_linear_kv(self, x, gamma, W, eps, k_cache, v_cache, kv_row0, pos, out=None):
        """The batch-1 projection that also stores the token's K / V rows at pos."""
        y = self.rmsnorm_linear(x, gamma, W, eps)
        self.calls[-1] = "rmsnorm_linear_kv"
        hk, _, d = k_cache.shape
        n = hk * d
        k_cache[:, pos] = y[0, kv_row0:kv_row0 + n].reshape(hk, d)
        v_cache[:, pos] = y[0, kv_row0 + n:kv_row0 + 2 * n].reshape(hk, d)
        return y

    # -- attention over head-major caches [n_seq * H_kv, max_len, d]

    def kv_cache_write(self, k_rows, v_rows, k_cache, v_cache, pos, n_seq=1):
        self.calls.append("kv_cache_write")
        rows = k_rows.shape[0]
        s_new = rows // n_seq
        hk = k_cache.shape[0] // n_seq
        d = k_cache.shape[2]
        for b in range(n_seq):
            blk = slice(b * s_new, (b + 1) * s_new)
            k_cache[b * hk:(b + 1) * hk, pos:pos + s_new] = k_rows[blk].reshape(s_new, hk, d).transpose(0, 1)
            v_cache[b * hk:(b + 1) * hk, pos:pos + s_new] = v_rows[blk].reshape(s_new, hk, d).transpose(0, 1)

    @staticmethod
    def _attend(q, k, v, q_pos_offset, causal):
        """q [S, H, d] over k / v [H_kv, L, d]; query i sees keys j <= offset + i."""
        S, H, d = q.shape
        g = H // k.shape[0]
        out = torch.empty(S, H, d, dtype=torch.float64)
        for h in range(H):
            sc = (q[:, h].double() @ k[h // g].double().T) * d ** -0.5
            if causal:
                j = torch.arange(k.shape[1])[None, :]
                i = torch.arange(S)[:, None]
                sc = sc.masked_fill(j > q_pos_offset + i, float("-inf"))
            out[:, h] = torch.softmax(sc, dim=-1) @ v[h // g].double()
        return out

    def attention_prefill(self, q, k_cache, v_cache, kv_len, q_pos_offset):
        self.calls.append("attention_prefill")
        return self._attend(q, k_cache[:, :kv_len], v_cache[:, :kv_len], q_pos_offset, True)

    def attention_decode(self, q, k_cache, v_cache, kv_len):
        self.calls.append("attention_decode")
        return self._attend(q[None], k_cache[:, :kv_len], v_cache[:, :kv_len], 0, False)[0]
