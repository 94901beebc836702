"""Derived error bounds for the GPU-vs-oracle parity tests.

Notation: u32 = 2^-24 (FP32 unit roundoff), u16 = 2^-11 (binary16), ubf = 2^-8
(bfloat16).  ``absdot`` is sum_k |a_k||b_k| for each output element (computed in
float64), ``exact`` the oracle's FP64-accumulated result rounded once to float.

* FP32 CUDA-core dot products of length K in any summation order (sequential,
  split-K, tree) satisfy |err| <= gamma_K * absdot with gamma_K ~= K*u32
  (the reference's derivation, tests/test_kernels.cu:144-172); the oracle's own
  rounding to float adds u32*|exact|.
* tcgen05 FP32 accumulation is not IEEE round-per-add (products of a K=16 step
  are summed internally and the accumulator update may truncate), so its
  constant is c = 2: |err| <= 2*K*u32*absdot.
* A 16-bit output adds one rounding: u16*|exact| (ubf for BF16), plus half the
  smallest subnormal spacing as an absolute floor.

Every constant here is derived, never tuned; a kernel that misses one is wrong.
"""
from __future__ import annotations

import numpy as np

U32 = 2.0 ** -24
U16 = 2.0 ** -11
UBF = 2.0 ** -8


def check(got, exact, bound, what=""):
    got = np.asarray(got, np.float64)
    exact = np.asarray(exact, np.float64)
    bound = np.broadcast_to(np.asarray(bound, np.float64), exact.shape)
    err = np.abs(got - exact)
    bad = ~(err <= bound)  # NaN counts as bad
    if bad.any():
        idx = np.argwhere(bad)[:5]
        details = ", ".join(
            f"{tuple(i)}: got {got[tuple(i)]:.8g} exact {exact[tuple(i)]:.8g} "
            f"err {err[tuple(i)]:.3g} > bound {bound[tuple(i)]:.3g}" for i in idx)
        worst = float(np.nanmax(err / np.maximum(bound, 1e-300)))
        raise AssertionError(f"{what}: {int(bad.sum())} of {bad.size} elements outside the "
                             f"derived bound (worst err/bound {worst:.3g}); {details}")
    return float(np.max(err / np.maximum(bound, 1e-300))) if err.size else 0.0


def fp32_dot_bound(K, absdot, exact):
    return K * U32 * absdot + U32 * np.abs(exact) + 1e-30


def tc_bound(K, absdot, exact, out_u):
    """tcgen05 FP32 accumulate (c = 2) plus one rounding to the 16-bit output."""
    return 2 * K * U32 * absdot + U32 * np.abs(exact) + out_u * np.abs(exact) + 2.0 ** -25


def gemv16_bound(K, absdot, exact):
    """CUDA-core FP32 accumulate plus one FP16 output rounding."""
    return K * U32 * absdot + (U32 + U16) * np.abs(exact) + 2.0 ** -25
