"""Build the engine library in-tree: cwen_b200/libcwen_cuda.so.

CUDA sources (csrc/*.cu) compile with nvcc for sm_100a only; the host C
sources (host/*.c) with gcc; everything links into one shared library that
exports the C ABI of include/cwen_cuda.h.  Objects go to cwen_b200/_build/
and are rebuilt only when a source or header is newer.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
BUILD = PKG / "_build"
LIB = PKG / "libcwen_cuda.so"
CLI = PKG / "cwen"
NVCC = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVFLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xptxas", "-v",
           "--expt-relaxed-constexpr", "-I" + str(ROOT / "include")]
CFLAGS = ["-O2", "-std=gnu11", "-fPIC", "-Wall", "-Wextra", "-I" + str(PKG / "host"),
          "-I" + str(ROOT / "include")]


def _headers() -> list[Path]:
    return list((PKG / "csrc").glob("*.cuh")) + list((PKG / "host").glob("*.h")) + [ROOT / "include" / "cwen_cuda.h"]


def _stale(obj: Path, src: Path, deps: list[Path]) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(p.stat().st_mtime > t for p in [src, *deps] if p.exists())


def _run(cmd: list[str], log: Path) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    log.write_text(r.stdout + r.stderr)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("build failed: " + " ".join(cmd[:4]) + " ...")


def build(verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    deps = _headers()
    jobs = []
    objs = []
    for src in sorted((PKG / "csrc").glob("*.cu")):
        obj = BUILD / (src.stem + ".o")
        objs.append(obj)
        if _stale(obj, src, deps):
            jobs.append(([NVCC, *ARCH, *NVFLAGS, "-c", str(src), "-o", str(obj)], BUILD / (src.stem + ".log")))
    for src in sorted((PKG / "host").glob("*.c")):
        if src.stem.endswith("_main"):
            continue
        obj = BUILD / (src.stem + ".o")
        objs.append(obj)
        if _stale(obj, src, deps):
            jobs.append((["gcc", *CFLAGS, "-c", str(src), "-o", str(obj)], BUILD / (src.stem + ".log")))
    with cf.ThreadPoolExecutor(max_workers=max(1, os.cpu_count() or 1)) as ex:
        list(ex.map(lambda j: _run(*j), jobs))
    if jobs or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        _run([NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lpthread", "-lm"], BUILD / "link.log")
    main_src = PKG / "host" / "cwen_main.c"
    if main_src.exists() and (not CLI.exists() or CLI.stat().st_mtime < max(LIB.stat().st_mtime,
                                                                             main_src.stat().st_mtime)):
        _run(["gcc", *CFLAGS, "-o", str(CLI), str(main_src), "-L" + str(PKG), "-lcwen_cuda",
              "-Wl,-rpath,$ORIGIN"], BUILD / "cli.log")
    if verbose:
        for lg in sorted(BUILD.glob("*.log")):
            sys.stdout.write(lg.read_text())
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
