"""Build libmoe_b200.so in-tree with nvcc for sm_100a.

The shared library is the product's native half: every CUDA kernel and the C
ABI declared in include/moe_b200.h.  It is built next to this file
(lightreason_b200/_native/) so that it travels with the source tree.
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
OUT_DIR = PKG / "_native"
LIB = OUT_DIR / "libmoe_b200.so"
SOURCES = ["host.cu", "router.cu", "permute.cu", "experts.cu", "layer.cu", "gather.cu", "grouped.cu",
           "expert_rows_noalloc.cu", "expert_parallel.cu", "router_tc.cu", "primary.cu", "ep_p2p.cu",
           "codec.cu", "decode.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libmoe_b200.so")
    return cand


def _stale() -> bool:
    if not LIB.exists():
        return True
    built = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES] + list(CSRC.glob("*.cuh")) + [ROOT / "include" / "moe_b200.h"]
    return any(p.stat().st_mtime > built for p in deps if p.exists())


def build(force: bool = False, verbose: bool = False, jobs: int = 0) -> Path:
    """Compile every .cu in csrc/ for sm_100a and link libmoe_b200.so."""
    if not force and not _stale():
        return LIB
    OUT_DIR.mkdir(exist_ok=True)
    obj_dir = OUT_DIR / "obj"
    obj_dir.mkdir(exist_ok=True)
    flags = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-I", str(ROOT / "include"),
                    "-I", str(CSRC), "--expt-relaxed-constexpr"]
    if verbose:
        flags += ["-Xptxas", "-v"]
    objs, procs = [], []
    for src in SOURCES:
        obj = obj_dir / (Path(src).stem + ".o")
        objs.append(obj)
        cmd = [nvcc(), *flags, "-c", str(CSRC / src), "-o", str(obj)]
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
    failed = []
    for src, proc in procs:
        out, _ = proc.communicate()
        if verbose or proc.returncode:
            sys.stderr.write(out)
        if proc.returncode:
            failed.append(src)
    if failed:
        raise RuntimeError(f"nvcc failed for {failed}")
    tmp = LIB.with_suffix(".so.tmp")
    subprocess.run([nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs),], check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
