"""Build recipe of libps_b200.so (nvcc, sm_100a only, in-tree output).

    python -c "import build_lib; build_lib.build()"   (from this directory)

Produces ``lib/libps_b200.so`` next to this file.  The CUDA runtime is
linked statically; kernels use the driver's cuTensorMapEncodeTiled through
cudaGetDriverEntryPoint, so no -lcuda is needed.
"""
from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
SOURCES = ["csrc/attention.cu", "csrc/prepass.cu", "csrc/proj.cu", "csrc/capi.cu", "csrc/static_block.cu",
           "csrc/selftest.cu"]
HEADERS = ["csrc/ptx.cuh", "csrc/internal.h"]
OUTPUT = HERE / "lib" / "libps_b200.so"
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-shared", f"-I{ROOT / 'include'}"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def up_to_date() -> bool:
    if not OUTPUT.exists():
        return False
    built = OUTPUT.stat().st_mtime
    deps = [HERE / s for s in SOURCES + HEADERS] + [ROOT / "include" / "ps_b200.h"]
    return all(d.stat().st_mtime <= built for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    if up_to_date() and not force:
        return OUTPUT
    OUTPUT.parent.mkdir(parents=True, exist_ok=True)
    tmp = OUTPUT.with_suffix(f".so.tmp{os.getpid()}")
    cmd = [nvcc(), *ARCH_FLAGS, *FLAGS, "-o", str(tmp), *[str(HERE / s) for s in SOURCES]]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stderr[-4000:]}")
    if verbose:
        print(res.stderr)
    tmp.replace(OUTPUT)
    return OUTPUT


if __name__ == "__main__":
    print(build(force=True, verbose=True))
