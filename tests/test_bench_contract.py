"""CPU: bench.py's reference arm keeps the JSON-line contract.

`bench.py --impl reference` times the reference's own CPU implementation of the
path (the compiled engine::cpu::matmul in oracle/_ref, else the oracle port) and
needs no GPU, so its line can be checked here: the required keys, the
"reference" impl tag, a cpu_baseline describing the run, and an e2e block with
zero host<->device bytes.
"""
from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent

REQUIRED = ["metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
            "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config"]


def test_reference_arm_prints_one_contract_line():
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference",
                        "--steps", "1", "--warmup", "3"],
                       capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip().startswith("{")]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    for k in REQUIRED:
        assert k in d, k
    assert d["impl"] == "reference"
    assert d["value"] > 0 and d["higher_is_better"] is True
    assert d["steps"] == 1 and d["warmup"] == 3 and d["n_gpus"] == 1
    assert d["config"]["workload"]
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["sample"]
    assert cb["value"] == d["value"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    env = d["environment"]  # provenance: host, and the library build when it exists
    assert env["host_cores"] >= 1 and "python" in env


def test_warmup_is_at_least_three():
    """The bench raises a smaller --warmup to the contract's minimum of 3."""
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference",
                        "--steps", "1", "--warmup", "1"],
                       capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    d = json.loads([ln for ln in r.stdout.splitlines() if ln.strip().startswith("{")][0])
    assert d["warmup"] == 3


def test_secondary_lines_carry_their_roofline_fraction():
    """Every other_configs line gets frac: HBM lines against the measured copy
    bandwidth, tensor lines against the bf16 burst peak, FP32 CUDA-core lines
    against the nominal SIMT peak; one "peaks" entry names the three peaks."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    b = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(b)
    pk, kind = b.peaks()
    out = b.with_fractions({"gemv_4096x4096": {"us": 7.0, "gbs": 4800.0},
                            "prefill_s2048": {"us": 180.0, "tflops": 1320.0},
                            "matmul_f32_512": {"us": 14.6, "tflops": 18.3}})
    assert out["gemv_4096x4096"]["frac"] == 4800.0 / pk["hbm_gbs"]
    assert out["prefill_s2048"]["frac"] == 1320.0 / pk["bf16_tflops"]
    assert abs(out["matmul_f32_512"]["frac"] - 18.3 / 74.4) < 1e-3
    assert set(out["peaks"]) == {"gbs", "tflops", "matmul_f32"}
    assert all("frac" in d for k, d in out.items() if k != "peaks")


def test_compact_rounds_floats_and_keeps_structure():
    import importlib.util
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    b = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(b)
    d = b.compact({"a": {"us": 11.623680591583252, "n": 3, "ok": True, "s": "x"},
                   "l": [0.1234567, None]})
    assert d == {"a": {"us": 11.62, "n": 3, "ok": True, "s": "x"}, "l": [0.1235, None]}
    assert b.compact(None) is None


def test_reference_arm_config_equals_ours():
    """Both arms quote the same config dict, so the driver compares like with like."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    b = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(b)
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference",
                        "--steps", "1", "--warmup", "3"],
                       capture_output=True, text=True, timeout=600, cwd=ROOT)
    d = json.loads([ln for ln in r.stdout.splitlines() if ln.strip().startswith("{")][0])
    assert d["config"] == b.headline_config(1)
