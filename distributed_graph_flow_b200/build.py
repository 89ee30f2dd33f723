"""Builds libdgfx.so (the sm_100a kernels behind the C ABI in include/dgfx.h).

Run ``python -m distributed_graph_flow_b200.build`` (or ``__graft_entry__.build()``).
The shared library is written next to this file so that it ships with the
source tree; it links the CUDA runtime statically and nothing from torch.
"""

from __future__ import annotations

import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
LIB = PKG / "libdgfx.so"
BUILD_DIR = PKG / "_build"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    f"-I{INCLUDE}",
]
SOURCES = ["capi.cu", "primitives.cu", "csr_build.cu", "sampler.cu", "aggregate.cu", "halo.cu", "peer.cu", "synth.cu",
           "transform.cu", "dense.cu", "subgraph.cu", "negatives.cu", "idmap.cu", "timeseries.cu", "sparse_ops.cu"]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(path).exists():
        raise RuntimeError("nvcc not found: the dgfx CUDA library cannot be built")
    return path


def _deps(src: Path) -> list[Path]:
    return [src] + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _compile(src: Path, obj: Path, extra: list[str]) -> None:
    if obj.exists() and all(obj.stat().st_mtime >= d.stat().st_mtime for d in _deps(src)):
        return
    cmd = [nvcc(), *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")


def build(verbose: bool = False, ptxas_info: bool = False) -> Path:
    BUILD_DIR.mkdir(exist_ok=True)
    extra = ["-Xptxas", "-v"] if ptxas_info else []
    objs = [BUILD_DIR / (Path(s).stem + ".o") for s in SOURCES]
    with concurrent.futures.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
        futs = [ex.submit(_compile, CSRC / s, o, extra) for s, o in zip(SOURCES, objs)]
        for f in futs:
            f.result()
    if not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB)
    if verbose:
        print(f"built {LIB}")
    return LIB


if __name__ == "__main__":
    build(verbose=True, ptxas_info="--ptxas" in sys.argv)
