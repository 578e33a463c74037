"""Builds libpackr_b200.so (all CUDA kernels + the C ABI) in-tree for sm_100a.

    python -m packr_b200.build          # incremental
    python -m packr_b200.build --force  # rebuild
    python -m packr_b200.build -D PACKR_STREAM_K=0 --output /tmp/lib.so
                                        # a variant with compile-time switches,
                                        # loaded through PACKR_B200_LIB=/tmp/lib.so

nvcc cross-compiles for sm_100a without a GPU, so the library can be built
anywhere the CUDA 12.9 toolkit is installed.
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
INCLUDE = PKG.parent / "include"
LIB = PKG / "libpackr_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found: the CUDA 12.9 toolkit is required to build libpackr_b200.so")
    return cand


def _sources() -> list[Path]:
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h")))


def needs_build() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(s.stat().st_mtime > t for s in _sources())


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False, defines=(),
          output: Path | None = None) -> Path:
    """Builds the library; `defines` ("NAME=VALUE" compile-time switches) and
    `output` make a variant elsewhere (always rebuilt), leaving the in-tree
    library alone."""
    out = Path(output) if output is not None else LIB
    if output is None and not defines and not force and not needs_build():
        return LIB
    if output is None and defines:
        raise ValueError("a build with compile-time switches needs its own output path")
    tmp = out.with_suffix(".so.tmp")
    cmd = [
        nvcc_path(), *ARCH, "-O3", "-lineinfo", "-std=c++17",
        "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC,-O3", "-shared",
        *(f"-D{d}" for d in defines),
        "-I", str(INCLUDE), "-I", str(CSRC),
        str(CSRC / "libpackr_b200.cu"), "-o", str(tmp),
    ]
    if ptxas_verbose:
        cmd.insert(1, "-Xptxas=-v")
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, out)
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true")
    ap.add_argument("-D", "--define", action="append", default=[], metavar="NAME=VALUE",
                    help="compile-time switch of a variant build (needs --output)")
    ap.add_argument("--output", type=Path, default=None, help="build a variant library at this path")
    a = ap.parse_args()
    print(build(force=a.force, verbose=True, ptxas_verbose=a.ptxas_verbose, defines=a.define, output=a.output))


if __name__ == "__main__":
    main()
