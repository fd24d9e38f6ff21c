"""Build libflour_attn.so (sm_100a) in-tree with nvcc.

    python -m flour_b200.build [--verbose]

The library is a single translation unit (csrc/flour_attn.cu includes the kernel headers), so
the per-device status word has one definition. cudart is linked statically: the library only
needs the NVIDIA driver at run time, and callers hand it their own stream handles.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
HOST = PKG / "host"
LIB = PKG / "libflour_attn.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def sources() -> list[Path]:
    return (sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted(HOST.glob("*.cpp")) +
            sorted(HOST.glob("*.h")) + [ROOT / "include" / "flour_attn.h"])


def needs_build() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(s.stat().st_mtime > t for s in sources())


def build(verbose: bool = False, force: bool = False, out: Path | None = None) -> Path:
    """Compile the library to `out` (default: the in-tree libflour_attn.so); the in-tree build
    is skipped when the library is newer than every source."""
    target = Path(out) if out is not None else LIB
    if out is None and not force and not needs_build():
        return LIB
    cmd = [
        nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
        "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr",
        "-I", str(ROOT / "include"), "-I", str(CSRC), "-I", str(HOST),
        "-cudart", "static",
        "-o", str(target), str(CSRC / "flour_attn.cu"), str(HOST / "flour_host.cpp"),
    ]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("nvcc failed building libflour_attn.so")
    if verbose:
        sys.stderr.write(r.stderr)
    return target


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true", help="print ptxas register/smem usage")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(verbose=a.verbose, force=a.force or a.verbose))
