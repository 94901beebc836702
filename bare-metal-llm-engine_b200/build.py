"""Builds the in-tree CUDA library ``libengine_b200.so`` for sm_100a.

Every ``csrc/*.cu`` file is compiled with nvcc
(``-gencode arch=compute_100a,code=sm_100a -lineinfo -O3``) into an object under
``_build/`` and linked into one shared library beside this file, with the CUDA
runtime linked statically, so the library loads without any CUDA shared object
on the search path (the driver is reached at run time).  Objects are rebuilt
only when their source or a header is newer; builds run in parallel.

    python bare-metal-llm-engine_b200/build.py [--force] [-v]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import json
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
OUT = HERE / "libengine_b200.so"
OBJ = HERE / "_build"
INCLUDE = HERE.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found (CUDA toolkit required to build the CUDA library)")
    return cand


def _newest_header() -> float:
    hdrs = list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    return max(p.stat().st_mtime for p in hdrs)


def _compile(src: Path, verbose: bool, extra: list[str]) -> Path:
    obj = OBJ / (src.stem + ".o")
    cmd = [nvcc(), *ARCH, *FLAGS, *extra, f"-I{INCLUDE}", "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    if verbose and (r.stdout.strip() or r.stderr.strip()):
        print(r.stdout, r.stderr, flush=True)
    return obj


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> Path:
    extra = list(extra or [])
    OBJ.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cpp"))  # .cpp: host-only code
    hdr_t = _newest_header()
    todo = []
    for s in srcs:
        o = OBJ / (s.stem + ".o")
        if force or not o.exists() or o.stat().st_mtime < max(s.stat().st_mtime, hdr_t):
            todo.append(s)
    if todo:
        with cf.ThreadPoolExecutor(max_workers=min(len(todo), os.cpu_count() or 4)) as ex:
            list(ex.map(lambda s: _compile(s, verbose, extra), todo))
    objs = [OBJ / (s.stem + ".o") for s in srcs]
    if force or todo or not OUT.exists() or OUT.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        tmp = OUT.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs),
               "-lpthread", "-ldl", "-lrt"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, OUT)
        write_build_info()
    return OUT


def write_build_info() -> None:
    """Records what the library was built from beside it (build_info.json): the
    git commit of the working tree, whether it had local changes, the nvcc
    version and the compile flags.  The GPU box receives a snapshot without
    .git, so the bench reads this file for its provenance block."""
    def run(*cmd):
        try:
            return subprocess.run(cmd, capture_output=True, text=True, cwd=HERE, timeout=30).stdout.strip()
        except Exception:
            return ""
    info = {
        "git_commit": run("git", "rev-parse", "HEAD") or "unknown",
        "git_dirty": bool(run("git", "status", "--porcelain", "--untracked-files=no")),
        "nvcc": (run(nvcc(), "--version").splitlines() or ["unknown"])[-1],
        "arch": ARCH[-1],
        "flags": " ".join(FLAGS),
        "built_utc": __import__("datetime").datetime.now(__import__("datetime").timezone.utc)
        .strftime("%Y-%m-%dT%H:%M:%SZ"),
    }
    (HERE / "build_info.json").write_text(json.dumps(info, indent=1) + "\n")


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true", help="print register / smem usage")
    a = ap.parse_args()
    extra = ["-Xptxas", "-v"] if a.ptxas_verbose else []
    out = build(force=a.force or a.ptxas_verbose, verbose=a.verbose or a.ptxas_verbose, extra=extra)
    print(out)
    return 0


if __name__ == "__main__":
    sys.exit(main())
