"""Builds oracle/_ref/libnes_ref.so: the reference's own batched NES emulator
(nes_emulator_gpu/src/cuda/host/nes_batch_gpu.cu and
src/cuda/kernels/nes_batch_kernel.cu, compiled from where they lie in the
reference checkout, for sm_100a) with the extern "C" shim oracle/nes_ref_shim.cu.
Test infrastructure only; the library is not committed (oracle/_ref/ is
git-ignored) but travels with the repository copy to the GPU box.

    python oracle/build_ref.py [REFERENCE_ROOT]   (default /root/reference)
"""
from __future__ import annotations

import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref" / "libnes_ref.so"


def build(ref_root: str = "/root/reference") -> Path | None:
    cuda = Path(ref_root) / "nes_emulator_gpu" / "src" / "cuda"
    srcs = [cuda / "host" / "nes_batch_gpu.cu", cuda / "kernels" / "nes_batch_kernel.cu"]
    if not all(p.exists() for p in srcs):
        return None
    OUT.parent.mkdir(exist_ok=True)
    cmd = ["nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-shared",
           "-Xcompiler", "-fPIC", f"-I{cuda}", f"-I{cuda / 'host'}", str(HERE / "nes_ref_shim.cu"),
           *map(str, srcs), "-o", str(OUT)]
    subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    print(build(*sys.argv[1:]))
