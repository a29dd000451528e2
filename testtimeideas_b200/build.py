"""Build libttt_attn.so (the sm_100a kernels + C ABI) in-tree with nvcc, and
libttt_torch.so (the ttt::fwd / ttt::bwd / ttt::bwd2 PyTorch operators over
that C ABI) with g++ against the installed torch.

The libraries are written to ``testtimeideas_b200/_lib/`` and object files to
``testtimeideas_b200/_build/``; both are git-ignored build products. Usage::

    python -m testtimeideas_b200.build            # incremental
    python -m testtimeideas_b200.build --force    # rebuild everything
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
BUILD = PKG / "_build"
LIBDIR = PKG / "_lib"
LIB = LIBDIR / "libttt_attn.so"
TORCH_SRC = CSRC / "torch_ops.cpp"
TORCH_LIB = LIBDIR / "libttt_torch.so"

SOURCES = ["capi.cu", "attn_fwd.cu", "attn_bwd_qm.cu", "attn_bwd_km.cu", "misc.cu", "noalloc.cu", "attn_from_p.cu",
           "attn_pwrite.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-Xptxas", "-warn-spills"]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libttt_attn.so")
    return cand


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))


def _stale(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(p.stat().st_mtime > t for p in [src, *_headers()])


def _compile(src: Path, obj: Path, extra: list[str]) -> tuple[Path, str]:
    cmd = [nvcc(), *ARCH, *FLAGS, *extra, "-I", str(CSRC), "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> Path:
    """Compile every CUDA source for sm_100a and link the shared library."""
    extra = list(extra or [])
    BUILD.mkdir(parents=True, exist_ok=True)
    LIBDIR.mkdir(parents=True, exist_ok=True)
    jobs = []
    for name in SOURCES:
        src = CSRC / name
        obj = BUILD / (name + ".o")
        if force or _stale(obj, src):
            jobs.append((src, obj))
    if jobs:
        workers = min(len(jobs), max(1, os.cpu_count() or 1))
        with cf.ThreadPoolExecutor(workers) as ex:
            for obj, log in ex.map(lambda j: _compile(j[0], j[1], extra), jobs):
                if verbose and log.strip():
                    print(f"[{obj.name}]\n{log}", file=sys.stderr)
    objs = [BUILD / (n + ".o") for n in SOURCES]
    if force or jobs or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


def cuda_home() -> Path:
    return Path(nvcc()).resolve().parent.parent


def build_torch_ops(force: bool = False, verbose: bool = False) -> Path:
    """Compile torch_ops.cpp into libttt_torch.so, linked against libttt_attn.so
    (found next to it through an $ORIGIN run path) and torch's libraries."""
    import torch

    deps = [TORCH_SRC, LIB, *sorted(INCLUDE.glob("*.h"))]
    if not force and TORCH_LIB.exists() and all(d.stat().st_mtime <= TORCH_LIB.stat().st_mtime for d in deps):
        return TORCH_LIB
    torch_dir = Path(torch.__file__).resolve().parent
    incs = [torch_dir / "include", torch_dir / "include" / "torch" / "csrc" / "api" / "include",
            cuda_home() / "include", INCLUDE]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    tmp = TORCH_LIB.with_suffix(".so.tmp")
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           *[f"-I{p}" for p in incs], str(TORCH_SRC), "-o", str(tmp),
           f"-L{torch_dir / 'lib'}", "-lc10", "-lc10_cuda", "-ltorch_cpu", "-ltorch_cuda", "-ltorch",
           f"-L{LIBDIR}", "-lttt_attn", "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{torch_dir / 'lib'}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"g++ failed for {TORCH_SRC.name}:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    if verbose and r.stderr.strip():
        print(r.stderr, file=sys.stderr)
    os.replace(tmp, TORCH_LIB)
    return TORCH_LIB


def build_all(force: bool = False, verbose: bool = False) -> Path:
    """The kernel library, then the operator library that links it."""
    lib = build(force=force, verbose=verbose)
    build_torch_ops(force=force, verbose=verbose)
    return lib


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    args = ap.parse_args()
    print(build_all(force=args.force, verbose=args.verbose))
    print(TORCH_LIB)


if __name__ == "__main__":
    main()
