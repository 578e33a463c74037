"""Builds the CPU oracle (test infrastructure) and, when the reference sources
are present, the reference's own code for this path into oracle/_ref/.

    python -m oracle.build [--force] [--reference-root DIR]

The reference tree's location comes from --reference-root or the
PACKR_REFERENCE_ROOT environment variable; without either only the oracle's
own C library is built.

Outputs (all git-ignored, all travel with the working tree):
  oracle/liboracle.so            C restatement of the 8-bit AdamW step.
  oracle/_ref/ref_adam8_cuda.so  packr/cuda_adam_kernel.cu compiled UNMODIFIED
                                 from the reference tree for sm_100a (no fast
                                 math, the reference's own flag set plus the
                                 arch), loaded as a torch extension on a GPU.
  oracle/_ref/ref_cpu_adam8.so   the reference's single-threaded C++ CPU 8-bit
                                 AdamW (packr/offload.py:33-130, compiled from
                                 the source string in that file), the CPU
                                 timing baseline of the optimizer step.
The reference tree is only read here; nothing at run time reads it.
"""
from __future__ import annotations

import argparse
import os
import re
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REF_OUT = HERE / "_ref"
ORACLE_LIB = HERE / "liboracle.so"


def build_oracle(force: bool = False) -> Path:
    src = HERE / "adam8_oracle.c"
    if not force and ORACLE_LIB.exists() and ORACLE_LIB.stat().st_mtime > src.stat().st_mtime:
        return ORACLE_LIB
    cc = shutil.which("gcc") or "cc"
    tmp = ORACLE_LIB.with_suffix(".so.tmp")
    subprocess.run([cc, "-O2", "-std=c11", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared",
                    str(src), "-o", str(tmp), "-lm"], check=True)
    os.replace(tmp, ORACLE_LIB)
    return ORACLE_LIB


def _torch_ext(name: str, sources: list[str], cuda: bool) -> None:
    from torch.utils import cpp_extension
    bdir = REF_OUT / f"build_{name}"
    bdir.mkdir(parents=True, exist_ok=True)
    kw = dict(name=name, sources=sources, build_directory=str(bdir), verbose=False, is_python_module=True)
    if cuda:
        # The reference's flags (setup.py:27-31) plus the B200 arch; a -gencode
        # in the flags makes torch skip its own arch list.
        kw["extra_cuda_cflags"] = ["--expt-relaxed-constexpr", "-gencode", "arch=compute_100a,code=sm_100a"]
    else:
        kw["extra_cflags"] = ["-O3"]
    os.environ.setdefault("MAX_JOBS", "4")
    cpp_extension.load(**kw)
    built = bdir / f"{name}.so"
    shutil.copy2(built, REF_OUT / f"{name}.so")


def reference_root(root: str | os.PathLike | None = None) -> Path | None:
    """The reference tree: `root`, else $PACKR_REFERENCE_ROOT, else None."""
    r = root if root is not None else os.environ.get("PACKR_REFERENCE_ROOT")
    return Path(r) if r else None


def build_reference(force: bool = False, root: str | os.PathLike | None = None) -> list[Path]:
    """Compiles the reference's Adam kernels from the tree at `root` (or
    $PACKR_REFERENCE_ROOT); returns the .so files made (none without a tree)."""
    out: list[Path] = []
    ref = reference_root(root)
    if ref is None:
        return out
    cu = ref / "packr" / "cuda_adam_kernel.cu"
    off = ref / "packr" / "offload.py"
    if not cu.exists():
        return out
    REF_OUT.mkdir(exist_ok=True)
    tgt = REF_OUT / "ref_adam8_cuda.so"
    if force or not tgt.exists():
        _torch_ext("ref_adam8_cuda", [str(cu)], cuda=True)
    out.append(tgt)
    if off.exists():
        tgt = REF_OUT / "ref_cpu_adam8.so"
        if force or not tgt.exists():
            text = off.read_text()
            m = re.search(r'_cpu_adam_source\s*=\s*r"""(.*?)"""', text, re.S)
            if m is None:
                raise RuntimeError("CPU Adam source string not found in packr/offload.py")
            src = REF_OUT / "ref_cpu_adam8.cpp"
            body = m.group(1)
            src.write_text(body + "\n#include <torch/extension.h>\n"
                           "PYBIND11_MODULE(TORCH_EXTENSION_NAME, mod) {\n"
                           "  mod.def(\"cpu_fused_adam_8bit_kernel\", &cpu_fused_adam_8bit_kernel);\n}\n")
            _torch_ext("ref_cpu_adam8", [str(src)], cuda=False)
        out.append(tgt)
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--no-ref", action="store_true")
    ap.add_argument("--reference-root", default=None, help="the reference tree (default: $PACKR_REFERENCE_ROOT)")
    a = ap.parse_args()
    print(build_oracle(a.force))
    if not a.no_ref:
        for p in build_reference(a.force, a.reference_root):
            print(p)


if __name__ == "__main__":
    sys.exit(main())
