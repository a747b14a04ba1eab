"""Build libg4b200.so (sm_100a) in-tree: moa-workspace_b200/g4b200/libg4b200.so.

    python moa-workspace_b200/build.py

nvcc cross-compiles without a GPU. The library links only the CUDA runtime.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
SOURCES = ["csrc/g4_proj.cu", "csrc/g4_batch.cu", "csrc/g4_batch_attn.cu", "csrc/g4_attention.cu", "csrc/g4_vocab.cu", "csrc/g4_logits_batch.cu", "csrc/g4_decoder.cu", "csrc/g4_abi.cu"]
HEADERS = ["csrc/g4_common.cuh", "csrc/g4_tc.cuh", "csrc/g4_gemv.cuh", "csrc/g4_ops.cuh", "csrc/g4_ctx.cuh", "csrc/g4_batch.cuh",
           "../include/g4b200.h"]
OUTPUT = HERE / "g4b200" / "libg4b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-shared"]


def nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(cuda_home) / "bin" / "nvcc"
    return str(cand) if cand.exists() else (shutil.which("nvcc") or "nvcc")


def up_to_date() -> bool:
    if not OUTPUT.exists():
        return False
    built = OUTPUT.stat().st_mtime
    return all((HERE / f).stat().st_mtime <= built for f in SOURCES + HEADERS + ["build.py"])


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return OUTPUT
    OUTPUT.parent.mkdir(parents=True, exist_ok=True)
    tmp = OUTPUT.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, *FLAGS, *[str(HERE / s) for s in SOURCES], "-o", str(tmp)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError(f"nvcc failed ({res.returncode}) building {OUTPUT.name}")
    if verbose:
        sys.stderr.write(res.stderr)
    os.replace(tmp, OUTPUT)
    return OUTPUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
