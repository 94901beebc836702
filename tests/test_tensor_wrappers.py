"""The Tensor-typed overloads of include/engine/kernels_b200.hpp against the
engine's own Tensor class.

oracle/Makefile's `tensor` target compiles the reference's src/tensor.cpp (with
dtype.cpp and allocator.cpp) unmodified into oracle/_ref/libref_tensor.so and
links tests/tensor_wrappers_test.cpp against it and libengine_b200.so.  On CPU
the program checks every argument error (dtype, contiguity, shape, device,
undefined tensors); on a B200 it checks that each overload's output is
bit-identical to the pointer launcher's on the same inputs.
"""
from __future__ import annotations

import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
BIN = ROOT / "oracle" / "_ref" / "tensor_wrappers_test"


def _binary(rebuild: bool) -> Path:
    import oracle

    ref = oracle.reference_dir()
    if rebuild and ref is not None:  # the CPU test rebuilds when sources changed
        subprocess.run(["make", "-s", "-C", str(ROOT / "oracle"), f"REF={ref}", "tensor"],
                       check=True)
    if not BIN.exists():
        pytest.skip("oracle/_ref/tensor_wrappers_test not built (needs the reference tree)")
    return BIN


def _run(mode: str):
    r = subprocess.run([str(_binary(mode == "cpu")), mode], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert " 0 failures" in r.stdout, r.stdout


def test_argument_checks_on_cpu(pkg):
    pkg.lib()  # the library the program links is built
    _run("cpu")


@pytest.mark.gpu
def test_overloads_forward_bit_exactly(pkg, dev):
    _run("gpu")
