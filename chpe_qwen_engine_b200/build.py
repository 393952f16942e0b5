"""Build the native libraries in-tree.

* libchpe.so        -- the product: C ABI + CUDA kernels for sm_100a (nvcc)
* libchpe_synth.so  -- deterministic synthetic archive generator (gcc)
* chpe_fwd          -- the command-line front end over libchpe.so (the
                       reference's chpe_fwd contract)

Usage: python -m chpe_qwen_engine_b200.build [--force]
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG, "csrc")
ROOT = os.path.dirname(PKG)
LIBCHPE = os.path.join(PKG, "libchpe.so")
LIBSYNTH = os.path.join(PKG, "libchpe_synth.so")
CHPE_FWD = os.path.join(PKG, "chpe_fwd")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
    "--expt-relaxed-constexpr",
    "-I", CSRC, "-I", os.path.join(ROOT, "include"),
]

ENGINE_SRCS = ["engine.cu", "engine_verify.cu", "attention_noalloc.cu", "deltanet.cu", "chpe_convert.cu", "tc_probe.cu",
               "chpe_c_api.cpp", "chpe_maps.c"]
ENGINE_DEPS = ENGINE_SRCS + ["engine.h", "engine_types.h", "gemv.cuh", "attention.cuh",
                             "aux_kernels.cuh", "gemv_tma.cuh", "gemv_flat_tma.cuh", "gemv_rowblk.cuh", "device_common.cuh", "chpe_maps.h",
                             "tc_common.cuh", "bgemm_tc.cuh",
                             "qwen3b_cell_map.inc", "../../include/chpe.h"]
SYNTH_SRCS = ["chpe_synth.c", "chpe_maps.c"]
SYNTH_DEPS = SYNTH_SRCS + ["chpe_synth.h", "chpe_maps.h", "qwen3b_cell_map.inc"]


def _nvcc() -> str:
    for c in ("nvcc", "/usr/local/cuda/bin/nvcc"):
        p = shutil.which(c) or (c if os.path.exists(c) else None)
        if p:
            return p
    raise RuntimeError("nvcc not found")


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(os.path.join(CSRC, d)) > t for d in deps)


def build_synth(force: bool = False) -> str:
    if force or _stale(LIBSYNTH, SYNTH_DEPS):
        cmd = ["gcc", "-O2", "-fPIC", "-shared", "-pthread", "-Wall", "-Wextra", "-o", LIBSYNTH]
        cmd += [os.path.join(CSRC, s) for s in SYNTH_SRCS]
        subprocess.run(cmd, check=True)
    return LIBSYNTH


def build_engine(force: bool = False) -> str:
    if force or _stale(LIBCHPE, ENGINE_DEPS):
        objdir = os.path.join(PKG, "_build")
        os.makedirs(objdir, exist_ok=True)
        nvcc = _nvcc()
        objs = []
        for s in ENGINE_SRCS:
            o = os.path.join(objdir, os.path.splitext(s)[0] + ".o")
            src = os.path.join(CSRC, s)
            if s.endswith(".c"):
                cmd = ["gcc", "-O2", "-fPIC", "-c", src, "-o", o, "-I", CSRC]
            else:
                cmd = [nvcc] + NVCC_FLAGS + ["-c", src, "-o", o]
            subprocess.run(cmd, check=True)
            objs.append(o)
        cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", LIBCHPE] + objs
        subprocess.run(cmd, check=True)
    return LIBCHPE


def build_cli(force: bool = False) -> str:
    """chpe_fwd, linked against the in-tree libchpe.so (found through $ORIGIN)."""
    if force or _stale(CHPE_FWD, ["chpe_fwd.cpp", "../../include/chpe.h"]) or (
            os.path.exists(CHPE_FWD) and os.path.getmtime(LIBCHPE) > os.path.getmtime(CHPE_FWD)):
        cmd = [_nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-O2", "-std=c++17", "-o", CHPE_FWD, os.path.join(CSRC, "chpe_fwd.cpp"),
               "-I", os.path.join(ROOT, "include"), "-L", PKG, "-lchpe", "-Xlinker", "-rpath=$ORIGIN"]
        subprocess.run(cmd, check=True)
    return CHPE_FWD


def build_all(force: bool = False) -> None:
    build_synth(force)
    build_engine(force)
    build_cli(force)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv)
    print("built", LIBCHPE, LIBSYNTH)
