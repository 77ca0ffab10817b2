"""Build step for the CUDA bridge: nvcc -> rustane_b200/libcudabridge.so (in tree).

The library is compiled for sm_100a only (B200). nvcc cross-compiles without a
GPU, so this runs on any machine with CUDA 12.9.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libcudabridge.so"
SOURCES = [CSRC / "bridge.cu"]
HEADERS = sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [ROOT / "include" / "cuda_bridge.h"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "--expt-relaxed-constexpr",
]


def nccl_dirs():
    """(include dir, library file) of the NCCL that ships with torch, if present."""
    try:
        import nvidia.nccl  # namespace package from the nvidia-nccl wheel
        base = Path(list(nvidia.nccl.__path__)[0])
    except Exception:
        return None, None
    inc, lib = base / "include", base / "lib" / "libnccl.so.2"
    return (inc if (inc / "nccl.h").exists() else None), (lib if lib.exists() else None)


def nvcc_path() -> str:
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    p = Path(cuda) / "bin" / "nvcc"
    return str(p) if p.exists() else "nvcc"


def needs_build() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(p.stat().st_mtime > t for p in SOURCES + HEADERS if p.exists())


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not needs_build():
        return LIB
    inc, nccl_lib = nccl_dirs()
    if inc is None:
        raise RuntimeError("nccl.h not found (the nvidia-nccl wheel provides it)")
    extra = [f"-I{inc}"]
    if nccl_lib is not None:
        extra.append(f'-DCB_NCCL_DEFAULT_PATH="{nccl_lib}"')
    cmd = [nvcc_path(), *NVCC_FLAGS, f"-I{ROOT / 'include'}", f"-I{CSRC}", *extra,
           "-o", str(LIB), *map(str, SOURCES), "-ldl", "-lpthread"]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed ({r.returncode}):\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
