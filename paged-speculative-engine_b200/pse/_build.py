"""Build libpse.so in-tree with nvcc for sm_100a (no JIT cache, no torch
headers: the library is plain CUDA C++ behind the C ABI of include/pse.h)."""
from __future__ import annotations

import os
import subprocess

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)                 # paged-speculative-engine_b200/
REPO = os.path.dirname(ROOT)
CSRC = os.path.join(ROOT, "csrc")
INCLUDE = os.path.join(REPO, "include")
LIB = os.path.join(PKG, "lib", "libpse.so")

SOURCES = ["kv_cache.cu", "attention.cu", "attention_tc.cu", "attention_prefill.cu", "gemm_tc.cu", "sampling.cu", "model_ops.cu", "sched.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (os.path.sep not in cand or os.path.exists(cand)):
            return cand
    return "nvcc"


def needs_build() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in os.listdir(CSRC)] + [os.path.join(INCLUDE, "pse.h")]
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile libpse.so if a source is newer than it (or ``force``).  Several
    processes may call this at once (one per GPU under torchrun): the build
    runs under an exclusive file lock, the staleness test is repeated once the
    lock is held, and each build writes its own temporary file before the
    atomic rename."""
    if not force and not needs_build():
        return LIB
    import fcntl
    os.makedirs(os.path.dirname(LIB), exist_ok=True)
    with open(LIB + ".lock", "w") as lock:
        fcntl.flock(lock, fcntl.LOCK_EX)
        try:
            if not force and not needs_build():
                return LIB  # another process built it while this one waited
            tmp = f"{LIB}.tmp{os.getpid()}"
            cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
                   f"-I{INCLUDE}", "-o", tmp] + [os.path.join(CSRC, s) for s in SOURCES]
            if verbose:
                print(" ".join(cmd))
            subprocess.run(cmd, check=True)
            os.replace(tmp, LIB)
        finally:
            fcntl.flock(lock, fcntl.LOCK_UN)
    return LIB


if __name__ == "__main__":
    print(build(force=True, verbose=True))
