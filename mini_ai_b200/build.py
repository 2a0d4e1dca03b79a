"""Build the sm_100a engine library in-tree: mini_ai_b200/libmq_b200.so.

nvcc cross-compiles for B200 (compute_100a / sm_100a) without a GPU.
Usage: python -m mini_ai_b200.build [--force]
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libmq_b200.so"
SOURCES = [CSRC / "mq_abi.cu", CSRC / "mq_noalloc.cu", CSRC / "mq_comm.cu"]
DEPS = sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [ROOT / "include" / "mq_b200.h"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC,-O2",
         "-Xptxas", "-v", "-I", str(ROOT / "include"), "-I", str(CSRC)]


def nccl_include() -> str:
    """nccl.h of the NCCL that torch loads at run time (the wheel's), else the system one.
    Only the header is used: mq_comm.cu loads libnccl.so.2 with dlopen."""
    try:
        import nvidia.nccl  # noqa: F401

        inc = Path(list(nvidia.nccl.__path__)[0]) / "include"
        if (inc / "nccl.h").exists():
            return str(inc)
    except Exception:
        pass
    return "/usr/include"


def stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(p.stat().st_mtime > t for p in DEPS)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not stale():
        return LIB
    cmd = [NVCC, *ARCH, *FLAGS, "-I", nccl_include(), "-shared", "-o", str(LIB), *map(str, SOURCES), "-lpthread",
           "-ldl"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    log = PKG / "build.log"
    log.write_text(res.stdout + res.stderr)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError(f"nvcc failed ({res.returncode}); see {log}")
    if verbose:
        print(res.stderr)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
