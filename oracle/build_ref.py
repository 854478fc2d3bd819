"""Build the reference's own CPU op library into oracle/_ref/ (checker and
timed CPU baseline only — never part of the product).

Compiles patches/littlebit_cpu_optimized.cpp straight from the read-only
reference checkout (LITTLESPEC_REF, default REF below) as a torch
extension.  -mavx2 -mfma instead of -march=native so the .so built here also
runs on the GPU box's host CPU; libgomp is linked from gcc's own directory
because the bare -lgomp of the reference's recipe does not resolve with this
image's toolchain.  Output: oracle/_ref/littlebit_cpu_ops.so, which registers
torch.ops.littlebit_cpu_ops.* when loaded with torch.ops.load_library.

    python oracle/build_ref.py
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
SO = OUT / "littlebit_cpu_ops.so"
REF = Path(os.environ.get("LITTLESPEC_REF", "/root/reference"))
SRC = REF / "patches" / "littlebit_cpu_optimized.cpp"


def gomp_dir() -> str:
    try:
        p = subprocess.run(["g++", "-print-file-name=libgomp.so"], capture_output=True, text=True).stdout.strip()
        if p and os.path.exists(p):
            return os.path.dirname(p)
    except OSError:
        pass
    cands = glob.glob("/usr/lib/gcc/x86_64-linux-gnu/*/libgomp.so")
    return os.path.dirname(sorted(cands)[-1]) if cands else ""


def build(force: bool = False) -> Path | None:
    if SO.exists() and not force:
        return SO
    if not SRC.exists():
        return None
    import torch.utils.cpp_extension as ce

    OUT.mkdir(exist_ok=True)
    bdir = OUT / "build"
    bdir.mkdir(exist_ok=True)
    ldf = ["-lgomp"]
    gd = gomp_dir()
    if gd:
        ldf = [f"-L{gd}", "-lgomp"]
    ce.load(name="littlebit_cpu_ops", sources=[str(SRC)], build_directory=str(bdir),
            extra_cflags=["-O3", "-mavx2", "-mfma", "-fopenmp"], extra_ldflags=ldf,
            with_cuda=False, is_python_module=False, verbose=False)
    built = bdir / "littlebit_cpu_ops.so"
    shutil.copy2(built, SO)
    return SO


def load() -> bool:
    """Load the built reference ops into torch.ops.littlebit_cpu_ops (no build)."""
    import torch

    if hasattr(torch.ops, "littlebit_cpu_ops") and hasattr(torch.ops.littlebit_cpu_ops, "littlebit_linear"):
        return True
    if not SO.exists():
        return False
    torch.ops.load_library(str(SO))
    return True


if __name__ == "__main__":
    p = build(force="--force" in sys.argv)
    print(p if p else "reference source not found; nothing built")
