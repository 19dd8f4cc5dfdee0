"""Build ``libq3s_sampler.so`` in-tree with nvcc for sm_100a, and the
``torch.ops.q3s`` operator library over it.

``libq3s_sampler.so`` holds the CUDA kernels and the C ABI declared in
``include/q3s_sampler.h``; it links the CUDA runtime statically and has no
torch dependency, so any FFI (ctypes here) can load it.
``libq3s_torch_ops.so`` registers the PyTorch operators (schemas, CUDA and
Meta kernels) that call that C ABI; it links libq3s_sampler.so through an
``$ORIGIN`` run path, so the pair can move together.
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
TORCH_OPS_PATH = PKG_DIR / "libq3s_torch_ops.so"
TORCH_OPS_SRC = CSRC / "q3s_torch_ops.cpp"
SOURCES = [CSRC / "q3s_sampler.cu", CSRC / "q3s_warp.cu", CSRC / "q3s_head.cu", CSRC / "q3s_lean.cu"]
DEPS = SOURCES + [CSRC / "q3s_args.cuh", CSRC / "q3s_device.cuh", CSRC / "q3s_warp.cuh", CSRC / "q3s_philox.cuh", CSRC / "q3s_step.cuh", CSRC / "q3s_head.cuh", CSRC / "q3s_lean.cuh", CSRC / "q3s_cp.cuh", CSRC / "q3s_core.cuh",
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


def torch_ops_up_to_date() -> bool:
    if not TORCH_OPS_PATH.exists():
        return False
    t = TORCH_OPS_PATH.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in (TORCH_OPS_SRC, INCLUDE / "q3s_sampler.h", LIB_PATH))


def build_torch_ops(force: bool = False, verbose: bool = False) -> Path:
    """Compile the torch.ops.q3s operator library (g++ against torch's
    headers; no GPU needed)."""
    if not force and torch_ops_up_to_date():
        return TORCH_OPS_PATH
    import torch
    from torch.utils import cpp_extension as ce

    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    incs = [f"-I{p}" for p in ce.include_paths(device_type="cuda")] + [f"-I{INCLUDE}"]
    libdirs = [f"-L{p}" for p in ce.library_paths(device_type="cuda")]
    tmp = TORCH_OPS_PATH.with_suffix(".so.tmp")
    cmd = [system_cxx(), "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           *incs, str(TORCH_OPS_SRC), "-o", str(tmp), *libdirs, f"-L{PKG_DIR}", "-lq3s_sampler",
           "-lc10", "-lc10_cuda", "-ltorch_cpu", "-ltorch", "-Wl,-rpath,$ORIGIN"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or res.returncode != 0:
        print(" ".join(cmd))
        print(res.stdout + res.stderr)
    if res.returncode != 0:
        raise RuntimeError(f"g++ failed ({res.returncode}) building {TORCH_OPS_PATH.name}")
    bad = defined_libstdcxx_internals(tmp)
    if bad:
        tmp.unlink()
        raise RuntimeError(f"{TORCH_OPS_PATH.name} would carry its own copy of libstdc++ internals ({bad[0]}): "
                           "build it with the system g++ that torch was built against")
    os.replace(tmp, TORCH_OPS_PATH)
    return TORCH_OPS_PATH


def system_cxx() -> str:
    """The system C++ compiler, whose libstdc++ is the one torch and the
    Python process use.  $CXX is not consulted: a different toolchain can
    link parts of its own libstdc++ (locale facet ids and the like) into the
    library, and a stream formatting an error message then crashes."""
    for cand in ("/usr/bin/g++", shutil.which("g++")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("no g++ found to build the torch operator library")


def defined_libstdcxx_internals(path: Path) -> list[str]:
    """Dynamic symbols of libstdc++'s locale / stream machinery that `path`
    defines itself (it should define none); [] when nm is unavailable."""
    nm = shutil.which("nm")
    if not nm:
        return []
    res = subprocess.run([nm, "-DC", "--defined-only", str(path)], capture_output=True, text=True)
    keys = ("std::locale", "num_put<", "codecvt", "std::ios_base")
    return [ln for ln in res.stdout.splitlines() if any(k in ln for k in keys)]


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
    print(build_torch_ops(force=True, verbose=True))
