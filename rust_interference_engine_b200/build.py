"""Builds librie_cuda.so in-tree (sm_100a only) with nvcc.

Run `python -m rust_interference_engine_b200.build` or call build(). The library is a
plain C-ABI shared object; nothing here depends on torch.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "librie_cuda.so")
ROOT = os.path.dirname(HERE)

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-warn-spills",
]


def nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h"))
    deps += glob.glob(os.path.join(ROOT, "include", "*.h"))
    return any(os.path.getmtime(d) > t for d in deps)


def nccl_link() -> list:
    """Link NCCL by soname (libnccl.so.2): the process uses whichever copy it loads first
    (the one PyTorch brings, when present)."""
    for d in ("/usr/lib/x86_64-linux-gnu", "/usr/local/cuda/lib64"):
        if os.path.exists(os.path.join(d, "libnccl.so.2")):
            return ["-L" + d, "-l:libnccl.so.2"]
    try:
        import nvidia.nccl  # pip wheel layout
        d = os.path.join(os.path.dirname(nvidia.nccl.__file__), "lib")
        return ["-L" + d, "-l:libnccl.so.2", "-Xlinker", "-rpath=" + d]
    except Exception:
        return ["-l:libnccl.so.2"]


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not _stale():
        return LIB
    bdir = os.path.join(HERE, "_build")
    os.makedirs(bdir, exist_ok=True)
    objs = []
    procs = []
    for src in sources():
        obj = os.path.join(bdir, os.path.basename(src) + ".o")
        cmd = [nvcc(), *NVCC_FLAGS, "-I", os.path.join(ROOT, "include"), "-dc" if False else "-c", src, "-o", obj]
        procs.append((cmd, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
        objs.append(obj)
    failed = False
    for cmd, p in procs:
        out, _ = p.communicate()
        if verbose or p.returncode != 0:
            sys.stderr.write(" ".join(cmd) + "\n" + (out or ""))
        failed |= p.returncode != 0
    if failed:
        raise RuntimeError("nvcc failed")
    tmp = LIB + ".tmp"
    cmd = [nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", tmp, *objs, "-lcuda", *nccl_link()]
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
