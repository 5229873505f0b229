"""Builds inference_c_b200/lib/libpkv_b200.so in-tree.

C11 host sources (allocator, pool, step transaction) are compiled with gcc,
CUDA sources with nvcc for sm_100a only, and everything is linked into one
shared library with a static CUDA runtime.  Objects go to
inference_c_b200/_build/; a source is recompiled when it or any header in
csrc/ or include/ is newer than its object.
"""
from __future__ import annotations

import os
import pathlib
import shutil
import subprocess
from concurrent.futures import ThreadPoolExecutor

HERE = pathlib.Path(__file__).resolve().parent
CSRC = HERE / "csrc"
INCLUDE = HERE.parent / "include"
OBJDIR = HERE / "_build"
LIBDIR = HERE / "lib"
LIBRARY = LIBDIR / "libpkv_b200.so"

C_SOURCES = ["paged_kv_cache.c", "pkv_pool.c", "pkv_comm.c"]
CU_SOURCES = ["pkv_copy.cu", "pkv_decode.cu", "pkv_prefill.cu", "pkv_sequence.cu", "pkv_dense.cu",
              "pkv_peer.cu"]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def cuda_home() -> pathlib.Path:
    env = os.environ.get("CUDA_HOME") or os.environ.get("CUDA_PATH")
    if env:
        return pathlib.Path(env)
    nvcc = shutil.which("nvcc")
    if nvcc:
        return pathlib.Path(nvcc).resolve().parent.parent
    return pathlib.Path("/usr/local/cuda")


def _headers() -> list[pathlib.Path]:
    return sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _stale(src: pathlib.Path, obj: pathlib.Path) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return src.stat().st_mtime > t or any(h.stat().st_mtime > t for h in _headers())


def _run(cmd: list[str]) -> None:
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"build step failed ({proc.returncode}):\n{' '.join(cmd)}\n"
                           f"{proc.stdout}\n{proc.stderr}")


def build(force: bool = False, verbose_ptxas: bool = False) -> pathlib.Path:
    """Compiles stale objects and relinks the library; returns its path."""
    home = cuda_home()
    nvcc = str(home / "bin" / "nvcc")
    inc = ["-I", str(INCLUDE), "-I", str(CSRC), "-I", str(home / "include")]
    OBJDIR.mkdir(exist_ok=True)
    LIBDIR.mkdir(exist_ok=True)
    jobs = []
    for name in C_SOURCES:
        src, obj = CSRC / name, OBJDIR / (name + ".o")
        if force or _stale(src, obj):
            jobs.append(["gcc", "-std=c11", "-D_POSIX_C_SOURCE=200809L", "-O2", "-fPIC",
                         "-Wall", "-Wextra", "-Wno-unused-parameter", *inc, "-c", str(src),
                         "-o", str(obj)])
    for name in CU_SOURCES:
        src, obj = CSRC / name, OBJDIR / (name + ".o")
        if force or _stale(src, obj):
            cmd = [nvcc, *ARCH, "-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC",
                   "--expt-relaxed-constexpr", *inc, "-c", str(src), "-o", str(obj)]
            if verbose_ptxas:
                cmd.insert(1, "-Xptxas=-v")
            jobs.append(cmd)
    if jobs:
        with ThreadPoolExecutor(max_workers=min(8, len(jobs))) as pool:
            list(pool.map(_run, jobs))
    objs = [str(OBJDIR / (n + ".o")) for n in C_SOURCES + CU_SOURCES]
    newest = max(pathlib.Path(o).stat().st_mtime for o in objs)
    if force or jobs or not LIBRARY.exists() or LIBRARY.stat().st_mtime < newest:
        tmp = LIBRARY.with_suffix(".so.tmp")
        _run([nvcc, *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *objs,
              "-lpthread", "-lrt", "-ldl"])
        os.replace(tmp, LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    import sys
    print(build(force="--force" in sys.argv, verbose_ptxas="--ptxas-v" in sys.argv))
