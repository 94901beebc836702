"""CPU: the C-ABI library loads, exports every symbol include/engine_b200.h
declares, and enforces the reference's argument contract.

The contract tests mirror the reference's launchers_reject_negative_dimensions,
launchers_reject_null_pointers and empty_work_is_a_no_op_not_an_error
(tests/test_kernels.cu:1664-1838): argument validation happens before any
device work, so they run without a GPU (the pointers are never dereferenced).
"""
from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "engine_b200.h"
P = 4096  # a non-null pointer value; never dereferenced by a rejected call


def header_symbols() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"ENGINE_B200_API\s+(?:int|const char\*)\s+(engine_\w+)\(", text)))


def test_header_declares_the_boundary():
    syms = header_symbols()
    for legacy in ["matmul_naive", "matmul_tiled", "matmul_register_tiled", "gemv", "gemv_fp16",
                   "rmsnorm", "rmsnorm_linear", "rmsnorm_linear_fused_direct"]:
        assert f"engine_cuda_{legacy}" in syms
    assert len(syms) >= 20


def test_library_exports_every_declared_symbol(pkg):
    lib = pkg.lib()
    out = subprocess.run(["nm", "-D", "--defined-only", str(pkg.LIB_PATH)], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r" T (engine_\w+)", out))
    for s in header_symbols():
        assert s in exported, f"{s} declared in engine_b200.h but not exported"
        assert hasattr(lib, s)
    assert set(pkg.EXPORTS) <= exported
    assert lib.engine_abi_version() == 1


def test_library_has_no_cuda_shared_object_dependency(pkg):
    out = subprocess.run(["ldd", str(pkg.LIB_PATH)], capture_output=True, text=True).stdout
    assert "libcudart" not in out and "libcuda.so" not in out


def _throws(pkg, fn, *args, substr):
    with pytest.raises(pkg.EngineError) as e:
        fn(*args)
    assert substr in str(e.value), str(e.value)
    assert e.value.code == 1


def test_launchers_reject_negative_dimensions(pkg):
    c = pkg.cuda
    _throws(pkg, c.rmsnorm, P, P, P, -1, 4, 1e-5, substr="negative")
    _throws(pkg, c.matmul_naive, P, P, P, -1, 4, 4, substr="negative")
    _throws(pkg, c.matmul_tiled, P, P, P, 4, 4, -1, substr="negative")
    _throws(pkg, c.rmsnorm_linear, P, P, P, P, -1, 4, 4, 1e-5, substr="negative")
    _throws(pkg, c.rmsnorm_linear, P, P, P, P, 4, -1, 4, 1e-5, substr="negative")
    _throws(pkg, c.rmsnorm_linear, P, P, P, P, 4, 4, -1, 1e-5, substr="negative")
    _throws(pkg, c.gemv, P, P, P, -1, 4, substr="non-negative")
    _throws(pkg, c.gemv, P, P, P, 4, -1, substr="non-negative")
    _throws(pkg, c.gemv_fp16, P, P, P, -1, 4, substr="non-negative")
    _throws(pkg, c.gemv_fp16, P, P, P, 4, -1, substr="non-negative")
    _throws(pkg, c.matmul_register_tiled, P, P, P, -1, 4, 4, substr="non-negative")
    _throws(pkg, c.matmul_register_tiled, P, P, P, 4, -1, 4, substr="non-negative")
    _throws(pkg, c.matmul_register_tiled, P, P, P, 4, 4, -1, substr="non-negative")
    _throws(pkg, c.vector_add, P, P, P, -1, substr="non-negative")
    _throws(pkg, c.swiglu_fp16, P, P, P, -1, substr="non-negative")
    _throws(pkg, c.matmul_f16, P, P, P, 4, 4, -1, substr="non-negative")
    _throws(pkg, c.linear_f16, P, P, 0, P, -1, 4, 4, substr="non-negative")
    _throws(pkg, c.gemv_f16_nk, P, P, 0, P, -1, 4, substr="non-negative")
    _throws(pkg, c.rmsnorm_linear_f16, P, P, P, 0, P, 4, -1, 4, 1e-5, substr="negative")
    _throws(pkg, c.residual_rmsnorm, P, P, P, P, P, -1, 4, 1e-5, substr="negative")
    _throws(pkg, c.residual_rmsnorm, P, P, P, P, P, 4, -1, 1e-5, substr="negative")
    # attention: the reference launchers' contracts (attention_prefill.cu:331-347,
    # attention_decode.cu:637-652)
    ap, ad = c.attention_prefill, c.attention_decode
    _throws(pkg, ap, P, P, P, P, -1, 4, 2, 2, 64, 256, 0.1, substr="s_q must be non-negative")
    _throws(pkg, ap, P, P, P, P, 4, 4, 3, 2, 64, 256, 0.1, substr="divisible")
    _throws(pkg, ap, P, P, P, P, 4, 4, 2, 2, 96, 384, 0.1, substr="head_dim must be 64 or 128")
    _throws(pkg, ap, P, P, P, P, 4, 4, 2, 2, 64, 100, 0.1, substr="kv_head_stride")
    _throws(pkg, ap, P, P, P, P, 4, 4, 2, 2, 64, 256, float("inf"), substr="scale must be finite")
    _throws(pkg, ap, P, P, P, P, 4, 4, 2, 2, 64, 256, 0.1, -1, substr="q_pos_offset")
    _throws(pkg, ad, P, P, P, P, 4, 2, 2, 64, 256, 0.1, -1, substr="split_kv")
    _throws(pkg, ad, P, P, P, P, -1, 2, 2, 64, 256, 0.1, substr="kv_len must be non-negative")
    _throws(pkg, ad, 0, P, P, P, 4, 2, 2, 64, 256, 0.1, substr="q is null")
    _throws(pkg, ap, P, P, P, 0, 4, 4, 2, 2, 64, 256, 0.1, substr="out is null")
    c.attention_prefill(P, P, P, P, 0, 4, 2, 2, 64, 256, 0.1)  # s_q = 0: a no-op
    # tcgen05 tile coordinates are 32-bit: larger dimensions are rejected, not wrapped
    _throws(pkg, c.matmul_f16, P, P, P, 2 ** 31, 8, 8, substr="too large")
    _throws(pkg, c.matmul_f16, P, P, P, 8, 2 ** 31, 8, substr="too large")
    # eps < 0 would put a negative number under the square root.
    _throws(pkg, c.rmsnorm, P, P, P, 4, 4, -1.0, substr="eps")
    _throws(pkg, c.residual_rmsnorm, P, P, P, P, P, 4, 4, -1.0, substr="eps")
    _throws(pkg, c.rmsnorm_linear, P, P, P, P, 4, 4, 4, -1.0, substr="eps")
    _throws(pkg, c.rmsnorm_linear_f16, P, P, P, 0, P, 4, 4, 4, -1.0, substr="eps")


def test_launchers_reject_null_pointers(pkg):
    c = pkg.cuda
    _throws(pkg, c.rmsnorm, 0, P, P, 2, 2, 1e-5, substr="null")
    _throws(pkg, c.rmsnorm, P, P, 0, 2, 2, 1e-5, substr="null")
    _throws(pkg, c.matmul_naive, 0, P, P, 2, 2, 2, substr="null")
    _throws(pkg, c.matmul_tiled, P, P, 0, 2, 2, 2, substr="null")
    _throws(pkg, c.rmsnorm_linear, 0, P, P, P, 2, 2, 2, 1e-5, substr="null")
    _throws(pkg, c.rmsnorm_linear, P, P, 0, P, 2, 2, 2, 1e-5, substr="null")
    _throws(pkg, c.rmsnorm_linear, P, P, P, 0, 2, 2, 2, 1e-5, substr="null")
    _throws(pkg, c.gemv, 0, P, P, 4, 4, substr="null")
    _throws(pkg, c.gemv, P, 0, P, 4, 4, substr="null")
    _throws(pkg, c.gemv, P, P, 0, 4, 4, substr="null")
    _throws(pkg, c.gemv_fp16, 0, P, P, 4, 4, substr="null")
    _throws(pkg, c.gemv_fp16, P, 0, P, 4, 4, substr="null")
    _throws(pkg, c.gemv_fp16, P, P, 0, 4, 4, substr="null")
    _throws(pkg, c.matmul_register_tiled, 0, P, P, 2, 2, 2, substr="null")
    _throws(pkg, c.matmul_register_tiled, P, 0, P, 2, 2, 2, substr="null")
    _throws(pkg, c.matmul_register_tiled, P, P, 0, 2, 2, 2, substr="null")
    _throws(pkg, c.matmul_f16, P, 0, P, 2, 2, 2, substr="null")
    _throws(pkg, c.linear_bf16, P, 0, 0, P, 2, 2, 2, substr="null")
    _throws(pkg, c.rmsnorm_linear_f16, P, P, 0, 0, P, 2, 2, 2, 1e-5, substr="null")
    _throws(pkg, c.swiglu_fp16, P, 0, P, 4, substr="null")
    _throws(pkg, c.vector_add, P, P, 0, 4, substr="null")
    # residual_rmsnorm: every pointer but the weight (test_kernels.cu:1752-1758)
    _throws(pkg, c.residual_rmsnorm, 0, P, P, P, P, 2, 2, 1e-5, substr="null")
    _throws(pkg, c.residual_rmsnorm, P, 0, P, P, P, 2, 2, 1e-5, substr="null")
    _throws(pkg, c.residual_rmsnorm, P, P, P, 0, P, 2, 2, 1e-5, substr="null")
    _throws(pkg, c.residual_rmsnorm, P, P, P, P, 0, 2, 2, 1e-5, substr="null")
    # rms weight / gamma may be null: "no learned gain" is a valid configuration.
    c.residual_rmsnorm(P, P, 0, P, P, 0, 0, 1e-5)
    c.rmsnorm(P, 0, P, 0, 0, 1e-5)
    c.rmsnorm_linear(P, 0, P, P, 0, 0, 0, 1e-5)
    c.rmsnorm_linear_f16(P, 0, P, 0, P, 0, 0, 0, 1e-5)


def test_empty_work_is_a_no_op_not_an_error(pkg):
    c = pkg.cuda
    c.residual_rmsnorm(P, P, P, P, P, 0, 8, 1e-5)
    c.residual_rmsnorm(P, P, P, P, P, 8, 0, 1e-5)
    c.rmsnorm(P, P, P, 0, 8, 1e-5)
    c.rmsnorm(P, P, P, 8, 0, 1e-5)
    c.matmul_naive(P, P, P, 0, 8, 8)
    c.matmul_naive(P, P, P, 8, 0, 8)
    c.matmul_tiled(P, P, P, 0, 8, 8)
    c.matmul_tiled(P, P, P, 8, 0, 8)
    c.matmul_register_tiled(P, P, P, 0, 8, 8)
    c.matmul_register_tiled(P, P, P, 8, 0, 8)
    c.rmsnorm_linear(P, P, P, P, 0, 8, 8, 1e-5)
    c.rmsnorm_linear(P, P, P, P, 8, 0, 8, 1e-5)
    c.rmsnorm_linear(P, P, P, P, 8, 8, 0, 1e-5)
    c.gemv(P, P, P, 0, 8)
    c.gemv_fp16(P, P, P, 0, 8)
    c.swiglu_fp16(P, P, P, 0)
    c.matmul_f16(P, P, P, 0, 8, 8)
    c.linear_f16(P, P, 0, P, 8, 0, 8)
    c.rmsnorm_linear_f16(P, P, P, 0, P, 8, 8, 0, 1e-5)


def test_last_error_is_per_thread(pkg):
    import threading

    c = pkg.cuda
    msgs = {}

    def worker(name, args):
        try:
            c.gemv(*args)
        except pkg.EngineError as e:
            msgs[name] = str(e)

    t1 = threading.Thread(target=worker, args=("a", (0, P, P, 4, 4)))
    t2 = threading.Thread(target=worker, args=("b", (P, P, P, -1, 4)))
    t1.start(); t2.start(); t1.join(); t2.join()
    assert "null" in msgs["a"] and "non-negative" in msgs["b"]


def test_cpp_adapter_header_compiles():
    """include/engine/kernels_b200.hpp compiles as C++17 against the C ABI, with
    and without its attention launchers (ENGINE_B200_NO_ATTENTION leaves them to
    an engine that keeps its own attention sources)."""
    for defs, uses_attention in (([], True), (["-DENGINE_B200_NO_ATTENTION"], False)):
        body = ("engine::cuda::attention_decode(nullptr, nullptr, nullptr, nullptr, 0, 1, 1, "
                "64, 0, 0.125f);" if uses_attention else "")
        src = ('#include <engine/kernels_b200.hpp>\n'
               f'int main(){{ {body} return 0; }}\n')
        r = subprocess.run(["g++", "-std=c++17", "-fsyntax-only", *defs, f"-I{ROOT / 'include'}",
                            "-I/usr/local/cuda/include", "-x", "c++", "-"], input=src,
                           capture_output=True, text=True)
        assert r.returncode == 0, r.stderr
    # with the macro the launchers are absent: a call no longer compiles
    src = ('#include <engine/kernels_b200.hpp>\nint main(){ engine::cuda::attention_decode('
           'nullptr, nullptr, nullptr, nullptr, 0, 1, 1, 64, 0, 0.125f); return 0; }\n')
    r = subprocess.run(["g++", "-std=c++17", "-fsyntax-only", "-DENGINE_B200_NO_ATTENTION",
                        f"-I{ROOT / 'include'}", "-I/usr/local/cuda/include", "-x", "c++", "-"],
                       input=src, capture_output=True, text=True)
    assert r.returncode != 0


def test_tp_comm_rejects_bad_arguments(pkg):
    """engine_tp_*: validation happens before any device work."""
    c = pkg.cuda
    _throws(pkg, c.tp_comm_create, 0, 0, 16, substr="world")
    _throws(pkg, c.tp_comm_create, 0, 9, 16, substr="world")
    _throws(pkg, c.tp_comm_create, 2, 2, 16, substr="rank")
    _throws(pkg, c.tp_comm_create, -1, 2, 16, substr="rank")
    _throws(pkg, c.tp_comm_create, 0, 2, 0, substr="max_elems")
    _throws(pkg, c.tp_comm_create, 0, 2, 2 ** 40, substr="max_elems")
    _throws(pkg, c.tp_allreduce_f16, 0, P, 0, P, 8, substr="null")
    _throws(pkg, c.tp_linear_allreduce_f16, 0, P, P, 0, P, 1, 8, 8, substr="null")
    with pytest.raises(pkg.EngineError):
        c.tp_comm_handle(0)
    c.tp_comm_destroy(0)  # destroying nothing is a no-op


def test_fused_swiglu_entry_rejects_bad_arguments(pkg):
    """engine_cuda_rmsnorm_linear_swiglu_f16 follows the rmsnorm_linear contract."""
    c = pkg.cuda
    _throws(pkg, c.rmsnorm_linear_swiglu_f16, P, P, P, P, -1, 4, 4, 1e-5, substr="negative")
    _throws(pkg, c.rmsnorm_linear_swiglu_f16, P, P, P, P, 1, -4, 4, 1e-5, substr="negative")
    _throws(pkg, c.rmsnorm_linear_swiglu_f16, P, P, P, P, 1, 4, -4, 1e-5, substr="negative")
    _throws(pkg, c.rmsnorm_linear_swiglu_f16, 0, P, P, P, 1, 4, 4, 1e-5, substr="null")
    _throws(pkg, c.rmsnorm_linear_swiglu_f16, P, P, 0, P, 1, 4, 4, 1e-5, substr="null")
    _throws(pkg, c.rmsnorm_linear_swiglu_f16, P, P, P, 0, 1, 4, 4, 1e-5, substr="null")
    _throws(pkg, c.rmsnorm_linear_swiglu_f16, P, P, P, P, 1, 4, 4, -1e-5, substr="eps")
    # empty work is a no-op (nothing is launched), gamma may be null
    c.rmsnorm_linear_swiglu_f16(P, 0, P, P, 0, 4, 4, 1e-5)
    c.rmsnorm_linear_swiglu_f16(P, 0, P, P, 2, 0, 4, 1e-5)


def test_quant_entries_reject_bad_arguments(pkg):
    c = pkg.cuda
    _throws(pkg, c.quant_repack, 5, P, P, P, 4, 32, substr="qtype")
    _throws(pkg, c.quant_repack, 8, P, P, P, -1, 32, substr="negative")
    _throws(pkg, c.quant_repack, 8, P, P, P, 4, 48, substr="multiple")
    _throws(pkg, c.quant_repack, 4, 0, P, P, 4, 32, substr="null")
    _throws(pkg, c.gemv_q_nk, 5, P, P, P, 0, P, 4, 32, substr="qtype")
    _throws(pkg, c.gemv_q_nk, 8, P, P, P, 0, P, -4, 32, substr="non-negative")
    _throws(pkg, c.gemv_q_nk, 8, P, P, P, 0, P, 4, 40, substr="multiple")
    _throws(pkg, c.gemv_q_nk, 4, P, 0, P, 0, P, 4, 32, substr="null")
    c.gemv_q_nk(8, P, P, P, 0, P, 0, 32)   # N == 0: no-op
    c.quant_repack(4, P, P, P, 0, 32)      # no rows: no-op


def test_kv_cache_write_entries_reject_bad_arguments(pkg):
    """engine_cuda_kv_cache_write keeps the engine's checks and messages
    (kernels/attention_bridge.cu:89-103); the strided batched form adds its own."""
    c = pkg.cuda
    _throws(pkg, c.kv_cache_write, P, P, P, P, -1, 8, 128, 0, 16, substr="s_new must be non-negative")
    _throws(pkg, c.kv_cache_write, P, P, P, P, 4, 0, 128, 0, 16, substr="n_kv_heads must be positive")
    _throws(pkg, c.kv_cache_write, P, P, P, P, 4, 8, 0, 0, 16, substr="head_dim must be positive")
    _throws(pkg, c.kv_cache_write, P, P, P, P, 4, 8, 128, -1, 16, substr="pos_offset")
    _throws(pkg, c.kv_cache_write, P, P, P, P, 4, 8, 128, 14, 16, substr="kv_max_seq_len <")
    _throws(pkg, c.kv_cache_write, 0, P, P, P, 4, 8, 128, 0, 16, substr="k_new/v_new is null")
    _throws(pkg, c.kv_cache_write, P, P, P, 0, 4, 8, 128, 0, 16, substr="k_cache/v_cache is null")
    c.kv_cache_write(0, 0, 0, 0, 0, 8, 128, 3, 3)  # s_new == 0: no-op, null pointers allowed
    _throws(pkg, c.kv_cache_write_rows, P, P, 100, P, P, 1, 1, 1, 128, 0, 4, substr="row_pitch")
    _throws(pkg, c.kv_cache_write_rows, P, P, 128, P, P, -1, 1, 1, 128, 0, 4, substr="n_seq")
    _throws(pkg, c.kv_cache_write_rows, P, P, 128, P, P, 2, 3, 1, 128, 2, 4, substr="kv_max_seq_len <")
    c.kv_cache_write_rows(0, 0, 128, 0, 0, 0, 3, 1, 128, 0, 4)  # no sequences: no-op


def test_rmsnorm_linear_kv_rejects_bad_arguments(pkg):
    """The fused batch-1 projection + KV-cache store checks its arguments before
    any launch: dimensions, null pointers, the K / V rows inside the N outputs,
    the position inside the cache, K and the 16-byte alignment the kernel needs."""
    c = pkg.cuda
    f = c.rmsnorm_linear_kv_f16
    # x, gamma, W, residual, Y, N, K, eps, k_cache, v_cache, kv_row0, n_kv_heads, head_dim, max_len, pos
    _throws(pkg, f, P, P, P, 0, P, -1, 4096, 1e-5, P, P, 4096, 8, 128, 16, 0, substr="negative dimension")
    _throws(pkg, f, 0, P, P, 0, P, 6144, 4096, 1e-5, P, P, 4096, 8, 128, 16, 0, substr="null device pointer")
    _throws(pkg, f, P, P, P, 0, P, 6144, 4096, 1e-5, 0, P, 4096, 8, 128, 16, 0, substr="cache is null")
    _throws(pkg, f, P, P, P, 0, P, 6144, 4096, -1.0, P, P, 4096, 8, 128, 16, 0, substr="eps")
    _throws(pkg, f, P, P, P, 0, P, 6144, 4096, 1e-5, P, P, 4096, 0, 128, 16, 0, substr="positive")
    _throws(pkg, f, P, P, P, 0, P, 6144, 4096, 1e-5, P, P, 4100, 8, 128, 16, 0, substr="inside the N")
    _throws(pkg, f, P, P, P, 0, P, 6144, 4096, 1e-5, P, P, 4096, 8, 128, 16, 16, substr="pos must")
    _throws(pkg, f, P, P, P, 0, P, 6144, 4100, 1e-5, P, P, 4096, 8, 128, 16, 0, substr="multiple of 8")
    _throws(pkg, f, P + 2, P, P, 0, P, 6144, 4096, 1e-5, P, P, 4096, 8, 128, 16, 0, substr="aligned")


def test_c_abi_links_and_runs_from_plain_c(pkg, tmp_path):
    """include/engine_b200.h is C99 (pedantic, warnings as errors), and a plain C
    program links libengine_b200.so and makes calls that need no GPU: the ABI
    version, a rejected argument with its message, and a GGUF file that is not
    one."""
    pkg.lib()
    src = tmp_path / "abi.c"
    src.write_text(r'''
#include <stdio.h>
#include <string.h>
#include "engine_b200.h"
int main(void) {
  if (engine_abi_version() < 1) return 1;
  engine_half_t* p = (engine_half_t*)16; /* never dereferenced: the call is rejected first */
  if (engine_cuda_matmul_f16(p, p, p, -1, 4, 4, 0) != ENGINE_ERR_INVALID) return 2;
  if (strstr(engine_last_error(), "non-negative") == NULL) return 3;
  FILE* f = fopen("not.gguf", "wb");
  fputs("this is not a gguf file, but it is long enough", f);
  fclose(f);
  engine_gguf_t* g = NULL;
  if (engine_gguf_open("not.gguf", &g) != ENGINE_ERR_FORMAT || g != NULL) return 4;
  puts("ok");
  return 0;
}
''')
    exe = tmp_path / "abi"
    lib_dir = str(pkg.LIB_PATH.parent)
    r = subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-pedantic", "-Werror",
                        f"-I{ROOT / 'include'}", str(src), "-o", str(exe), f"-L{lib_dir}",
                        "-lengine_b200", f"-Wl,-rpath,{lib_dir}"], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([str(exe)], capture_output=True, text=True, cwd=tmp_path, timeout=60)
    assert r.returncode == 0 and r.stdout.strip() == "ok", (r.returncode, r.stdout, r.stderr)


# ------------------------------------------------ property: validation first
from hypothesis import given, settings  # noqa: E402
from hypothesis import strategies as st  # noqa: E402

# entry point -> (pointer argument required?, number of dims); optional pointers
# (residual, gamma, weight, lse) may be null.  Every call below is invalid by
# construction (a negative dimension or a null required pointer), so none can
# reach a kernel launch, on any machine.
_CALLS = {
    "matmul_f16": ([True, True, True], 3),
    "linear_f16": ([True, True, False, True], 3),
    "gemv_f16_nk": ([True, True, False, True], 2),
    "rmsnorm_linear_f16": ([True, False, True, False, True], 3),
    "matmul_register_tiled": ([True, True, True], 3),
    "gemv": ([True, True, True], 2),
    "gemv_fp16": ([True, True, True], 2),
}


@settings(max_examples=150, deadline=None)
@given(name=st.sampled_from(sorted(_CALLS)), data=st.data())
def test_property_invalid_arguments_are_rejected_before_any_device_work(pkg, name, data):
    req, ndims = _CALLS[name]
    ptrs = [data.draw(st.sampled_from([0, P])) for _ in req]
    dims = [data.draw(st.integers(-3, 6)) for _ in range(ndims)]
    if all(p for p, r in zip(ptrs, req) if r) and min(dims) >= 0:
        dims[data.draw(st.integers(0, ndims - 1))] = -1  # make it invalid
    fn = getattr(pkg.cuda, name)
    args = ptrs + dims + ([1e-5] if name == "rmsnorm_linear_f16" else [])
    with pytest.raises(pkg.EngineError) as ei:
        fn(*args)
    assert ei.value.code == 1 and str(ei.value)
