"""Build ``libq3s_sampler.so`` in-tree with nvcc for sm_100a.

The library holds the CUDA kernels and the C ABI declared in
``include/q3s_sampler.h``; it links the CUDA runtime statically and has no
torch dependency, so any FFI (ctypes here) can load it.
"""
from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
ROOT = PKG_DIR.parent
REPO = ROOT.parent
CSRC = ROOT / "csrc"
INCLUDE = REPO / "include"
LIB_PATH = PKG_DIR / "libq3s_sampler.so"
SOURCES = [CSRC / "q3s_sampler.cu", CSRC / "q3s_warp.cu"]
DEPS = SOURCES + [CSRC / "q3s_args.cuh", CSRC / "q3s_device.cuh", CSRC / "q3s_warp.cuh", CSRC / "q3s_philox.cuh", CSRC / "q3s_step.cuh",
                  INCLUDE / "q3s_sampler.h"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC",
    "-Xptxas", "-warn-spills",
]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: the q3s CUDA library cannot be built")
    return cand


def up_to_date() -> bool:
    if not LIB_PATH.exists():
        return False
    t = LIB_PATH.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in DEPS)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the library unless it is newer than every source.  The
    translation units compile in parallel, then link into one shared object
    (CUDA runtime linked statically)."""
    if not force and up_to_date():
        return LIB_PATH
    objdir = PKG_DIR / "_obj"
    objdir.mkdir(exist_ok=True)
    objs, procs = [], []
    for src in SOURCES:
        obj = objdir / (src.stem + ".o")
        cmd = [nvcc(), *NVCC_FLAGS, f"-I{INCLUDE}", "-c", "-o", str(obj), str(src)]
        procs.append((cmd, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
        objs.append(obj)
    failed = []
    for cmd, pr in procs:
        out, _ = pr.communicate()
        if verbose or pr.returncode != 0:
            print(" ".join(cmd))
            print(out)
        if pr.returncode != 0:
            failed.append(cmd[-1])
    if failed:
        raise RuntimeError(f"nvcc failed building {', '.join(failed)}")
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", str(tmp), *map(str, objs)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or res.returncode != 0:
        print(" ".join(cmd))
        print(res.stdout + res.stderr)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc link failed ({res.returncode}) for {LIB_PATH.name}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force=True, verbose=True))
