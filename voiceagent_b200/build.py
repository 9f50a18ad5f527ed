"""Build ``libb200asr.so`` (sm_100a only) in-tree with nvcc.

    python -m voiceagent_b200.build            # incremental
    python -m voiceagent_b200.build --force    # rebuild everything

Each ``csrc/*.cu`` compiles to an object under ``voiceagent_b200/_build`` and the
objects link into ``voiceagent_b200/libb200asr.so`` (static CUDA runtime, no torch
dependency). No JIT cache is involved, so the built library travels with the tree.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libb200asr.so"
INCLUDE = PKG.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--use_fast_math", "-Xcompiler", "-fPIC",
         "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr"]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(path):
        raise RuntimeError("nvcc not found; the b200asr kernels need the CUDA toolkit")
    return path


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    newest_header = max((p.stat().st_mtime for p in _headers()), default=0.0)
    objects = []
    for src in _sources():
        obj = BUILD / (src.stem + ".o")
        objects.append(obj)
        stale = (force or not obj.exists() or obj.stat().st_mtime < src.stat().st_mtime
                 or obj.stat().st_mtime < newest_header)
        if not stale:
            continue
        cmd = [nvcc(), *ARCH, *FLAGS, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
        if ptxas_info:
            cmd.insert(1, "-Xptxas=-v")
        if verbose:
            print(" ".join(cmd), flush=True)
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            sys.stderr.write(proc.stdout + proc.stderr)
            raise RuntimeError(f"nvcc failed on {src.name}")
        if ptxas_info:
            sys.stderr.write(proc.stderr)
    lib_stale = force or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objects)
    if lib_stale:
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-Xcompiler", "-fPIC", *map(str, objects), "-o", str(tmp)]
        if verbose:
            print(" ".join(cmd), flush=True)
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            sys.stderr.write(proc.stdout + proc.stderr)
            raise RuntimeError("linking libb200asr.so failed")
        os.replace(tmp, LIB)
    return LIB


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true")
    parser.add_argument("--ptxas-info", action="store_true", help="print registers/spills per kernel")
    args = parser.parse_args()
    print(build(force=args.force, verbose=args.verbose, ptxas_info=args.ptxas_info))


if __name__ == "__main__":
    main()
