"""Builds the backend in-tree:

* ``vllm_nt/_lib/libntb200.so`` -- every CUDA kernel and the C ABI of include/ntb200.h,
  compiled by nvcc for sm_100a only (``-gencode arch=compute_100a,code=sm_100a``), CUDA
  runtime linked statically;
* ``vllm_nt/_lib/_ntb200_C.so`` -- the torch.ops.ntb200 binding (csrc/torch_bind.cpp),
  linked against libntb200.so with an $ORIGIN rpath.

Objects go to ``vllm-nt_b200/_build``; a source is recompiled only when it, a shared
header, or this file is newer than its object.  Usage: ``python vllm-nt_b200/csrc/build.py
[-v] [--force]``.
"""

from __future__ import annotations

import argparse
import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

CSRC = Path(__file__).resolve().parent
PKG_ROOT = CSRC.parent
REPO = PKG_ROOT.parent
INCLUDE = REPO / "include"
LIB_DIR = PKG_ROOT / "vllm_nt" / "_lib"
OBJ_DIR = PKG_ROOT / "_build"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))

KERNEL_SOURCES = (
    "common.cu",
    "rms_norm.cu",
    "silu_and_mul.cu",
    "rope.cu",
    "rope_cache.cu",
    "kv_cache.cu",
    "embedding.cu",
    "paged_decode.cu",
    "paged_decode_noalloc.cu",
    "gemm.cu",
    "paged_prefill.cu",
    "allreduce.cu",
    "sampler.cu",
)
SHARED_HEADERS = (CSRC / "common.cuh", CSRC / "tcgen05.cuh", CSRC / "rope_math.cuh", INCLUDE / "ntb200.h", Path(__file__).resolve())

NVCC_FLAGS = [
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
    "--expt-relaxed-constexpr",
    f"-I{INCLUDE}",
    f"-I{CSRC}",
]

LIB_NAME = "libntb200.so"
BIND_NAME = "_ntb200_C.so"


def _nvcc() -> str:
    cand = CUDA_HOME / "bin" / "nvcc"
    if cand.exists():
        return str(cand)
    found = shutil.which("nvcc")
    if found is None:
        raise RuntimeError("nvcc not found (set CUDA_HOME)")
    return found


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"command failed ({proc.returncode}): {' '.join(cmd)}\n{proc.stdout}\n{proc.stderr}")
    if verbose and (proc.stdout or proc.stderr):
        print(proc.stdout + proc.stderr, flush=True)


def build_kernels(force: bool = False, verbose: bool = False) -> Path:
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    nvcc = _nvcc()
    jobs = []
    objects = []
    for src in KERNEL_SOURCES:
        s = CSRC / src
        o = OBJ_DIR / (s.stem + ".o")
        objects.append(o)
        if force or _stale(o, [s, *SHARED_HEADERS]):
            jobs.append([nvcc, *NVCC_FLAGS, "-c", str(s), "-o", str(o)])
    workers = max(1, min(len(jobs), os.cpu_count() or 4))
    if jobs:
        with concurrent.futures.ThreadPoolExecutor(max_workers=workers) as pool:
            for fut in [pool.submit(_run, j, verbose) for j in jobs]:
                fut.result()
    lib = LIB_DIR / LIB_NAME
    if force or jobs or _stale(lib, objects):
        _run([nvcc, "-shared", "-o", str(lib), *map(str, objects), f"-Xlinker=-soname={LIB_NAME}"], verbose)
    return lib


def build_binding(force: bool = False, verbose: bool = False) -> Path:
    import torch  # noqa: F401  (only for its include/library paths)
    from torch.utils import cpp_extension

    src = CSRC / "torch_bind.cpp"
    out = LIB_DIR / BIND_NAME
    lib = LIB_DIR / LIB_NAME
    if not (force or _stale(out, [src, lib, *SHARED_HEADERS])):
        return out
    includes = [*cpp_extension.include_paths(device_type="cuda"), str(CUDA_HOME / "include"), str(INCLUDE)]
    libdirs = [*cpp_extension.library_paths(device_type="cuda"), str(LIB_DIR)]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = [
        os.environ.get("CXX", "g++"),
        "-O2",
        "-std=c++17",
        "-fPIC",
        "-shared",
        str(src),
        "-o",
        str(out),
        f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
        "-DTORCH_EXTENSION_NAME=_ntb200_C",
        *[f"-I{p}" for p in includes],
        *[f"-L{p}" for p in libdirs],
        "-lc10",
        "-lc10_cuda",
        "-ltorch",
        "-ltorch_cpu",
        "-lntb200",
        "-Wl,-rpath,$ORIGIN",
    ]
    _run(cmd, verbose)
    return out


def build(force: bool = False, verbose: bool = False) -> tuple[Path, Path]:
    lib = build_kernels(force=force, verbose=verbose)
    bind = build_binding(force=force, verbose=verbose)
    return lib, bind


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args(argv)
    lib, bind = build(force=args.force, verbose=args.verbose)
    print(f"built {lib}\nbuilt {bind}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
