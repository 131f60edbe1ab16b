"""Build libb200scan.so (the C-ABI library) in-tree with nvcc for sm_100a.

    python -m armhackathon_b200.build        # or: python armhackathon_b200/build.py

The library is written next to this file so that it travels with the source
tree; the loader (``_ffi.py``) finds it there.
"""

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB = PKG / "libb200scan.so"
SOURCES = ["abi.cu", "m1_scan.cu", "m1_tile.cu", "m1_lane.cu", "m1_decode.cu", "m3_scan.cu", "m3_chunk.cu", "m3_angles.cu", "m3_tc.cu", "m3_mixer.cu", "m3_noncausal.cu", "m1_conv.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2",
         "--expt-relaxed-constexpr", "-diag-suppress", "128"]


def nvcc():
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(home) / "bin" / "nvcc"
    return str(cand) if cand.exists() else "nvcc"


def stale():
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h"))
    deps.append(PKG.parent / "include" / "b200scan.h")
    return any(p.stat().st_mtime > t for p in deps)


def build(force=False, verbose=False):
    if not force and not stale():
        return LIB
    objs = []
    build_dir = PKG / "_build"
    build_dir.mkdir(exist_ok=True)
    for src in SOURCES:
        obj = build_dir / (Path(src).stem + ".o")
        cmd = [nvcc(), *ARCH, *FLAGS, "-c", str(CSRC / src), "-o", str(obj)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
        objs.append(str(obj))
    tmp = LIB.with_suffix(".so.tmp")
    subprocess.run([nvcc(), *ARCH, "-shared", "-o", str(tmp), *objs, "-lcudart"], check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
