"""Load the golden fixtures (tests/golden/*.npz) and regenerate their inputs.

Each fixture stores the input recipe and SHA-256 digests of the inputs; the
inputs are regenerated with latent_attn.synthetic and checked against the
digests before use, so a drift of the generator is caught instead of producing
a false parity failure.
"""

from __future__ import annotations

import glob
import hashlib
import json
import os

import numpy as np
import torch

from latent_attn import synthetic

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def case_names():
    return sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN_DIR, "*.npz")))


def digest(t: torch.Tensor) -> str:
    t = t.detach().contiguous().cpu()
    if t.dtype in (torch.bfloat16, torch.float16):
        b = t.view(torch.int16).numpy().tobytes()
    else:
        b = t.numpy().tobytes()
    return hashlib.sha256(b).hexdigest()


def load_case(name: str):
    z = np.load(os.path.join(GOLDEN_DIR, name + ".npz"))
    meta = json.loads(bytes(z["meta"]).decode())
    out = z["out"]
    kw = dict(meta["kwargs"])
    dtype = getattr(torch, kw.pop("dtype"))
    if meta["recipe"] == "baseline":
        inp = synthetic.baseline_inputs(dtype=dtype, **kw)
    else:
        inp = synthetic.reference_test_inputs(dtype=dtype, **kw)
    for key, want in meta["digests"].items():
        got = digest(getattr(inp, key))
        assert got == want, f"{name}: regenerated {key} differs from the fixture (generator drift)"
    return meta, inp, out
