"""TEST DOUBLE: CPU float64 stand-ins for the CUDA projections of the TP layer.

Used only by the gloo tests to exercise the tensor-parallel sharding and the
collective sequence on CPU ranks.  The arithmetic is the reference's composition
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
