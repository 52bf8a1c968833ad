"""Build recipe for the native parts of ggemm_asm_b200 (sm_100a only).

Outputs, all inside the package directory so they travel with the source tree:
  libggemm_vark.so          the C-ABI library (include/ggemm_vark.h); cudart linked statically,
                            so the library loads on hosts without a GPU driver
  _build/ggemm_vark_launcher the standalone CUDA-event timing launcher (csrc/launcher.cu)

Run ``python -m ggemm_asm_b200.build`` (or ``__graft_entry__.build()``). Rebuilds only when a
source file is newer than its output.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIB_PATH = PKG / "libggemm_vark.so"
LAUNCHER_PATH = PKG / "_build" / "ggemm_vark_launcher"

LIB_SOURCES = ["vark_tc.cu", "vark_tc2.cu", "vark_simt.cu", "vark_capi.cu", "vark_noalloc.cu",
               "vark_quant.cu", "vark_fwd.cu"]
HEADERS = ["vark_ptx.cuh", "vark_internal.h"]

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr",
                "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall", "-Xcompiler", "-fvisibility=hidden"]


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build ggemm_asm_b200")
    return cand


def _stale(out: Path, inputs: list[Path]) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(p.stat().st_mtime > t for p in inputs)


def _inputs(extra: list[str]) -> list[Path]:
    files = [CSRC / s for s in LIB_SOURCES + HEADERS + extra]
    files.append(INCLUDE / "ggemm_vark.h")
    files.append(Path(__file__))
    return files


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"build failed ({res.returncode}):\n{' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout.strip() or res.stderr.strip()):
        print(res.stdout + res.stderr, flush=True)


def build_library(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    if not force and not _stale(LIB_PATH, _inputs([])):
        return LIB_PATH
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc_path(), *ARCH_FLAGS, *COMMON_FLAGS, "-shared", "-cudart", "static",
           "-I", str(INCLUDE), "-o", str(tmp), *[str(CSRC / s) for s in LIB_SOURCES]]
    if ptxas_verbose:
        cmd.insert(1, "-Xptxas=-v")
    _run(cmd, verbose or ptxas_verbose)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def build_launcher(force: bool = False, verbose: bool = False) -> Path:
    if not force and not _stale(LAUNCHER_PATH, _inputs(["launcher.cu"])):
        return LAUNCHER_PATH
    LAUNCHER_PATH.parent.mkdir(parents=True, exist_ok=True)
    cmd = [nvcc_path(), *ARCH_FLAGS, *COMMON_FLAGS, "-cudart", "static", "-I", str(INCLUDE),
           "-o", str(LAUNCHER_PATH), str(CSRC / "launcher.cu"),
           *[str(CSRC / s) for s in LIB_SOURCES]]
    _run(cmd, verbose)
    return LAUNCHER_PATH


def build_all(force: bool = False, verbose: bool = False) -> None:
    build_library(force=force, verbose=verbose)
    build_launcher(force=force, verbose=verbose)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv, verbose=True)
    if "-v" in sys.argv:
        build_library(force=True, ptxas_verbose=True)
    print(f"built {LIB_PATH} and {LAUNCHER_PATH}")
