"""Generate the golden MLA decode fixtures from the reference's own oracle.

Run in a container that has the reference checkout (read-only), named by
``$LATENT_ATTN_REF``:

    LATENT_ATTN_REF=<reference checkout> python tests/golden/make_golden.py

For every case it draws seeded inputs with ``latent_attn/synthetic.py`` (loaded
by file path, so the reference's own ``latent_attn`` package is the one on
``sys.path``), runs the reference's ``torch_mla_reference``
(tests/test_python.py:26-63) with the reference's ``build_rope_tables``
(tests/test_python.py:17-23) and ``MLAConfig`` (latent_attn/__init__.py:13-28),
and stores

* the recipe (seed, shapes, dtype, lengths) so the inputs can be regenerated,
* SHA-256 digests of every regenerated input tensor (regeneration is checked),
* the reference output, fp32, shape (B, H, dv).

Batched cases over one shared cache (the reference's ``batched_fused_mla``
semantics, src/fused_mla_batched.cuh:5-11) are the per-token loop of the same
oracle; variable-length cases loop over sequences, each attending to its own
rows at RoPE positions 0..L-1.
"""

from __future__ import annotations

import hashlib
import importlib.util
import json
import os
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
REF = os.environ.get("LATENT_ATTN_REF")  # the reference checkout; required (see main())


def _load_synthetic():
    path = os.path.join(REPO, "latent-attn_b200", "latent_attn", "synthetic.py")
    spec = importlib.util.spec_from_file_location("mla_synthetic_for_golden", path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod
    spec.loader.exec_module(mod)
    return mod


def digest(t: torch.Tensor) -> str:
    t = t.detach().contiguous().cpu()
    if t.dtype in (torch.bfloat16, torch.float16):
        b = t.view(torch.int16).numpy().tobytes()
    else:
        b = t.numpy().tobytes()
    return hashlib.sha256(b).hexdigest()


# (name, recipe, kwargs)
CASES = [
    # the CPU-baseline configuration (H=16, L=1024), bf16-rounded inputs
    ("cfg0_h16_l1024", "baseline", dict(num_heads=16, seq_lens=[1024], dtype="bfloat16", seed=0)),
    # the reference pytest sweep (tests/test_python.py:72-138), fp16, H=128
    ("reftest_h128_s512", "reference_test", dict(num_heads=128, seq_len=512, dtype="float16", seed=42)),
    ("reftest_h128_s2048", "reference_test", dict(num_heads=128, seq_len=2048, dtype="float16", seed=42)),
    ("reftest_h128_s8192", "reference_test", dict(num_heads=128, seq_len=8192, dtype="float16", seed=42)),
    # the C++ test's smaller head counts (tests/test_correctness.cu:246-257)
    ("reftest_h16_s512", "reference_test", dict(num_heads=16, seq_len=512, dtype="float16", seed=7)),
    ("reftest_h64_s2048", "reference_test", dict(num_heads=64, seq_len=2048, dtype="float16", seed=8)),
    # batched over a shared cache (tests/test_batched.py:33-88 recipe shape, B=4, S=1024)
    ("batched_h128_s1024_b4", "reference_test", dict(num_heads=128, seq_len=1024, batch=4, dtype="float16", seed=4)),
    # DeepSeek-V2 shape, bf16, tile-boundary lengths
    ("v2_bf16_l1", "baseline", dict(num_heads=128, seq_lens=[1], dtype="bfloat16", seed=11)),
    ("v2_bf16_l63", "baseline", dict(num_heads=128, seq_lens=[63], dtype="bfloat16", seed=12)),
    ("v2_bf16_l65", "baseline", dict(num_heads=128, seq_lens=[65], dtype="bfloat16", seed=13)),
    ("v2_bf16_l1000", "baseline", dict(num_heads=128, seq_lens=[1000], dtype="bfloat16", seed=14)),
    # variable-length batch, bf16
    ("varlen_bf16_b5", "baseline", dict(num_heads=128, seq_lens=[1, 64, 129, 700, 2049], dtype="bfloat16", seed=21)),
    # non-DeepSeek dims (generic path): d_c=256, d_R=32, dn=dv=64, H=8
    ("small_dims_h8", "baseline", dict(num_heads=8, seq_lens=[300, 17], kv_lora_rank=256, qk_rope_head_dim=32,
                                       qk_nope_head_dim=64, v_head_dim=64, dtype="float16", seed=31)),
]


def run_case(syn, ref_tests, RefCfg, name, recipe, kw):
    kw = dict(kw)
    dtype = getattr(torch, kw.pop("dtype"))
    if recipe == "baseline":
        inp = syn.baseline_inputs(dtype=dtype, **kw)
    else:
        inp = syn.reference_test_inputs(dtype=dtype, **kw)
    H = inp.q_nope.shape[1]
    dn = inp.q_nope.shape[2]
    dR = inp.q_rope.shape[2]
    dc = inp.W_UK.shape[1]
    dv = inp.W_UV.shape[0] // H
    cfg = RefCfg(d_model=0, kv_lora_rank=dc, qk_nope_head_dim=dn, qk_rope_head_dim=dR,
                 num_heads=H, v_head_dim=dv)
    outs = []
    for b in range(inp.batch):
        L, off = inp.seq_lens[b], inp.kv_offsets[b]
        cos, sin = ref_tests.build_rope_tables(L, dR, "cpu")
        kv = inp.kv_cache[off:off + L]
        out = ref_tests.torch_mla_reference(kv, inp.W_UK.float(), inp.W_UV.float(),
                                            inp.q_nope[b].float(), inp.q_rope[b].float(),
                                            cos, sin, cfg)
        outs.append(out.float())
    out = torch.stack(outs)
    meta = {
        "name": name, "recipe": recipe, "kwargs": {**kw, "dtype": str(dtype).replace("torch.", "")},
        "num_heads": H, "kv_lora_rank": dc, "qk_rope_head_dim": dR, "qk_nope_head_dim": dn,
        "v_head_dim": dv, "seq_lens": inp.seq_lens, "kv_offsets": inp.kv_offsets,
        "shared_cache": bool(inp.meta.get("shared_cache", False)),
        "digests": {
            "kv_cache": digest(inp.kv_cache), "q_nope": digest(inp.q_nope),
            "q_rope": digest(inp.q_rope), "W_UK": digest(inp.W_UK), "W_UV": digest(inp.W_UV),
        },
        "generator": "torch_mla_reference (reference tests/test_python.py:26-63), torch %s" % torch.__version__,
    }
    return meta, out.numpy().astype(np.float32)


def main():
    if not REF or not os.path.isdir(REF):
        raise SystemExit("set LATENT_ATTN_REF to the reference checkout")
    sys.path.insert(0, os.path.join(REF, "tests"))
    sys.path.insert(0, REF)
    import latent_attn as ref_pkg  # the reference's package (torch only; _C is imported lazily)
    assert os.path.realpath(os.path.dirname(ref_pkg.__file__)).startswith(os.path.realpath(REF)), ref_pkg.__file__
    import test_python as ref_tests  # noqa: E402  (reference tests/test_python.py)
    syn = _load_synthetic()
    torch.set_num_threads(os.cpu_count() or 1)
    only = set(sys.argv[1:])
    for name, recipe, kw in CASES:
        if only and name not in only:
            continue
        t0 = time.time()
        meta, out = run_case(syn, ref_tests, ref_pkg.MLAConfig, name, recipe, kw)
        np.savez_compressed(os.path.join(HERE, name + ".npz"), out=out,
                            meta=np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8))
        print(f"{name}: out {out.shape} absmax {np.abs(out).max():.4f} ({time.time() - t0:.1f}s)")


if __name__ == "__main__":
    main()
