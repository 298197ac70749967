"""Build the sm_100a kernels in-tree.

Produces, next to the Python package (dip_b200/_lib/):
  libdip_core.so     the C ABI of include/dip_b200.h (CUDA runtime only, no torch)
  dip_torch_ops.so   the torch operator registrations over that ABI

nvcc cross-compiles for sm_100a without a GPU, so this runs on any machine with
CUDA 12.9 and torch headers.  Rebuilds only what is older than its sources.

    python dynamic-input-pruning_b200/build.py [--force]
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
import sysconfig
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent
REPO = PKG_ROOT.parent
CSRC = PKG_ROOT / "csrc"
LIBDIR = PKG_ROOT / "dip_b200" / "_lib"
INCLUDE = REPO / "include"

CORE_SOURCES = ["capi.cu", "gemv_int4.cu", "topk.cu", "gather_down.cu", "quant.cu",
                "stack_ops.cu", "layer_fused.cu", "gemv_batch.cu", "gemm_tc.cu", "p2p.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    p = Path(home) / "bin" / "nvcc"
    return str(p) if p.exists() else (shutil.which("nvcc") or "nvcc")


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str]) -> None:
    print("+", " ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def build_core(force: bool = False) -> Path:
    LIBDIR.mkdir(parents=True, exist_ok=True)
    out = LIBDIR / "libdip_core.so"
    srcs = [CSRC / s for s in CORE_SOURCES]
    deps = srcs + [CSRC / "dip_common.cuh", CSRC / "dip_block.cuh", INCLUDE / "dip_b200.h"]
    if not force and not _stale(out, deps):
        return out
    objdir = PKG_ROOT / "_build"
    objdir.mkdir(exist_ok=True)
    objs = [str(objdir / (s.stem + ".o")) for s in srcs]
    cmds = [[_nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
             "-Xcompiler", "-fvisibility=hidden", "-I", str(INCLUDE), "-c", str(s), "-o", o]
            for s, o in zip(srcs, objs)]
    # the translation units are independent: compile them concurrently
    with ThreadPoolExecutor(max_workers=min(len(cmds), os.cpu_count() or 1)) as ex:
        list(ex.map(_run, cmds))
    _run([_nvcc(), *ARCH, "-shared", "-o", str(out), *objs, "-lcudart"])
    return out


def build_torch_ops(force: bool = False) -> Path:
    import torch
    from torch.utils import cpp_extension as ce

    core = build_core(force)
    out = LIBDIR / "dip_torch_ops.so"
    src = CSRC / "torch_ops.cpp"
    if not force and not _stale(out, [src, core, INCLUDE / "dip_b200.h"]):
        return out
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    inc = [f"-I{p}" for p in ce.include_paths()] + [f"-I{cuda_home}/include",
                                                    f"-I{sysconfig.get_paths()['include']}"]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    libs = ce.library_paths()
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           *inc, str(src), "-o", str(out), f"-L{LIBDIR}", "-ldip_core",
           *[f"-L{p}" for p in libs], "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu",
           f"-L{cuda_home}/lib64", "-lcudart", "-Wl,-rpath,$ORIGIN"]
    _run(cmd)
    return out


def build_all(force: bool = False) -> None:
    build_core(force)
    build_torch_ops(force)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv)
