"""Compile the reference's own fused decode kernels into oracle/_ref/ (test oracle only).

    LATENT_ATTN_REF=<reference checkout> python oracle/build_ref.py [--force]

The sources are compiled where they lie (src/fused_mla.cu, src/fused_mla_batched.cu
of anishesg/latent-attn) with the reference's own flags (setup.py:26-32: -O3
--use_fast_math -DTILE_SEQ=32), retargeted to sm_100a, plus -rdc=true because the
batched kernel calls device functions defined in fused_mla.cu
(src/fused_mla_batched.cu:2,72-73). oracle/ref_shim.cu adds C entry points. The
output oracle/_ref/libref_mla.so is git-ignored and travels to the GPU box with
the working tree. Nothing is copied out of the reference tree.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_ref")
OUT = os.path.join(OUT_DIR, "libref_mla.so")


def build(ref: str | None = None, force: bool = False) -> str | None:
    """Build from the reference checkout `ref` (or $LATENT_ATTN_REF). Without a checkout the
    previously built library is returned if there is one (the GPU box only uses that), else None."""
    ref = ref or os.environ.get("LATENT_ATTN_REF")
    if not ref:
        return OUT if os.path.exists(OUT) else None
    src = os.path.join(ref, "src")
    files = [os.path.join(src, "fused_mla.cu"), os.path.join(src, "fused_mla_batched.cu")]
    if not all(os.path.exists(f) for f in files):
        return OUT if os.path.exists(OUT) else None
    os.makedirs(OUT_DIR, exist_ok=True)
    shim = os.path.join(HERE, "ref_shim.cu")
    newest = max(os.path.getmtime(f) for f in files + [shim, __file__])
    if not force and os.path.exists(OUT) and os.path.getmtime(OUT) >= newest:
        return OUT
    nvcc = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    cmd = [nvcc, "-O3", "--use_fast_math", "-DTILE_SEQ=32", "-std=c++17", "-rdc=true",
           "-gencode", "arch=compute_100a,code=sm_100a", "-Xcompiler", "-fPIC", "-shared",
           "-I", src, *files, shim, "-o", OUT]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("reference kernel build failed:\n" + r.stdout + r.stderr)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
