"""Build the engine's shared library (vault_b200/libvault_b200.so) for sm_100a with nvcc.

The library is a plain C-ABI .so (include/vault_b200.h) built in-tree so it ships with the repository snapshot;
`python -m vault_b200.build` rebuilds it when any source is newer than the library.
"""

from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libvault_b200.so")
SOURCES = ["v3g_weights.cu", "v3g_step.cu", "v3g_attn.cu", "v3g_api.cu", "v3g_noalloc.cu", "v3g_gemm.cu", "v3g_prefill.cu", "v3g_sample.cu",
           "v3g_tokenizer.cu"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-O3", "-std=c++17",
    "-shared", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills",
]


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in os.listdir(CSRC)] + [os.path.join(REPO, "include", "vault_b200.h")]
    return any(os.path.getmtime(p) > t for p in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not _stale():
        return LIB
    cmd = [NVCC, *FLAGS, "-I", os.path.join(REPO, "include"), *[os.path.join(CSRC, s) for s in SOURCES], "-o", LIB + ".tmp"]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
