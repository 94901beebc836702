#!/usr/bin/env python3
"""Regenerate the hot-path golden fixtures from the reference's own generator.

The reference engine writes its golden data with ``tools/gen_reference.py``
(float64 NumPy results cast to float32, inputs from ``np.random.default_rng(
20260826)`` drawn in one sequence across all cases, ``gen_reference.py:58``).
This script imports that generator read-only, runs it with its NumPy backend
and, for every case on the matrix-multiply hot path (``matmul__*``,
``gemv__*``, ``gemv_fp16__*``, ``rmsnorm_linear__*``, the ``rmsnorm__*``
dependency, the ``residual_rmsnorm__*`` epilogue and the ``attention__*``
cases of the next row), records:

* the generator state immediately BEFORE the case's draws, so the inputs can be
  regenerated bit-for-bit anywhere NumPy is present (``golden.py`` replays the
  case's draws from that state);
* the SHA-256 of every input tensor exactly as the reference writes it, so a
  replay that drifts from the reference's inputs fails loudly;
* the reference's ``expected`` tensor (float32), verbatim.

Outputs: ``hotpath_cases.json`` and ``hotpath_expected.npz`` beside this file.
Run it only where the reference tree exists (it is not needed on the GPU box):

    python tests/golden/make_golden.py [--reference <reference source tree>]
"""
from __future__ import annotations

import argparse
import hashlib
import importlib.util
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
PREFIXES = ("matmul__", "gemv__", "gemv_fp16__", "rmsnorm_linear__", "rmsnorm__",
            "residual_rmsnorm__", "attention__")
# Outputs stored verbatim (the rest of a case's tensors are inputs, replayed).
OUTPUTS = ("expected", "lse")


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a, dtype=np.float32).tobytes()).hexdigest()


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None,
                    help="the reference source tree (default: ENGINE_REF_DIR, else a "
                         "`reference` checkout beside this repository)")
    args = ap.parse_args()
    if args.reference is None:
        sys.path.insert(0, str(HERE.parent.parent))
        import oracle

        ref = oracle.reference_dir()
        if ref is None:
            raise SystemExit("reference tree not found: pass --reference or set ENGINE_REF_DIR")
        args.reference = str(ref)

    gen_path = Path(args.reference) / "tools" / "gen_reference.py"
    spec = importlib.util.spec_from_file_location("ref_gen_reference", gen_path)
    gen = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(gen)

    rng = np.random.default_rng(gen.SEED)
    backend = gen.NumpyBackend()
    state_before = rng.bit_generator.state
    cases = []
    expected = {}
    attention = {c[0]: c[1:] for c in gen.ATTENTION_CASES}
    for stem, tensors in gen.build_cases(rng, backend):
        if stem.startswith(PREFIXES):
            inputs = {k: sha(v) for k, v in tensors.items() if k not in OUTPUTS}
            shapes = {k: list(np.asarray(v).shape) for k, v in tensors.items()}
            case = {
                "stem": stem,
                "state": state_before,
                "input_sha256": inputs,
                "shapes": shapes,
            }
            if stem.startswith("attention__"):  # the draws need the case's parameters
                s_q, s_kv, h, h_kv, d, off, causal, amp = attention[stem[len("attention__"):]]
                case["params"] = {"s_q": s_q, "s_kv": s_kv, "n_heads": h, "n_kv_heads": h_kv,
                                  "head_dim": d, "q_pos_offset": off, "is_causal": bool(causal),
                                  "qk_amp": float(amp)}
            cases.append(case)
            expected[stem] = np.asarray(tensors["expected"]).astype(np.float32)
            if "lse" in tensors:
                expected[stem + "::lse"] = np.asarray(tensors["lse"]).astype(np.float32)
        state_before = rng.bit_generator.state

    meta = {
        "generator": "tools/gen_reference.py (NumPy backend)",
        "seed": int(gen.SEED),
        "numpy": np.__version__,
        "cases": cases,
    }
    (HERE / "hotpath_cases.json").write_text(json.dumps(meta, indent=1) + "\n")
    np.savez_compressed(HERE / "hotpath_expected.npz", **expected)
    print(f"wrote {len(cases)} hot-path cases to {HERE}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
