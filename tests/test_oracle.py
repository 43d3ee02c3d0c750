"""The CPU oracle against the golden vectors produced by the reference's own
torch_mla_reference (tests/test_python.py:26-63 of anishesg/latent-attn)."""

import math

import numpy as np
import pytest
import torch

from golden_cases import case_names, load_case
from oracle import mla_oracle as O
from latent_attn import synthetic


@pytest.mark.parametrize("name", case_names())
def test_oracle_matches_reference_golden(name):
    meta, inp, want = load_case(name)
    H, dc, dR = meta["num_heads"], meta["kv_lora_rank"], meta["qk_rope_head_dim"]
    dn, dv = meta["qk_nope_head_dim"], meta["v_head_dim"]
    kv = inp.kv_cache.float().numpy()
    q_abs = O.absorb_query(inp.q_nope.float().numpy(), inp.W_UK.float().numpy(), H, dc)
    for b in range(inp.batch):
        L, off = inp.seq_lens[b], inp.kv_offsets[b]
        cos, sin = O.rope_tables(L, dR)
        got = O.absorbed_decode(kv[off:off + L], q_abs[b], inp.q_rope[b].float().numpy(),
                                inp.W_UV.float().numpy(), cos, sin, H, dc, dn, dR, dv)
        c = O.compare(got, want[b])
        # fp64 restatement vs the reference's fp32 torch computation
        assert c["max_rel"] < 2e-5, (name, b, c)
        if L <= 2048 and H <= 128:
            got32 = O.naive_decode(kv[off:off + L], inp.W_UK.float().numpy(), inp.W_UV.float().numpy(),
                                   inp.q_nope[b].float().numpy(), inp.q_rope[b].float().numpy(), cos, sin,
                                   H, dc, dn, dR, dv)
            c32 = O.compare(got32, want[b])
            assert c32["max_rel"] < 2e-5, (name, b, c32)


def test_rope_tables_match_torch_builder():
    """numpy's float32 pow and torch's differ by one ulp for a few frequencies, so
    the angle (pos * freq) drifts by up to ~pos * 2^-24 rad; parity tests therefore
    always hand the same tables to the kernel and to the oracle."""
    for L, dR in ((1, 64), (1000, 64), (77, 32)):
        c_np, s_np = O.rope_tables(L, dR)
        c_t, s_t = synthetic.build_rope_tables(L, dR)
        tol = 4 * L * 2.0 ** -24 + 1e-6
        assert np.abs(c_np - c_t.numpy()).max() < tol
        assert np.abs(s_np - s_t.numpy()).max() < tol


@pytest.mark.parametrize("bounds", [[0, 100], [0, 1, 100], [0, 33, 33, 64, 100], [0, 50, 99, 100]])
def test_split_combine_identity(bounds):
    """Log-sum-exp merge of split partials equals the unsplit softmax (any split, empty ranges included)."""
    rng = np.random.default_rng(0)
    H, dc, dR, L = 8, 64, 16, 100
    kv = rng.standard_normal((L, dc + dR)).astype(np.float32)
    q = rng.standard_normal((H, dc)) * 0.5
    qr = rng.standard_normal((H, dR))
    cos, sin = O.rope_tables(L, dR)
    scale = 1 / math.sqrt(96)
    m, l, o = O.split_partials(kv, q, qr, cos, sin, dc, scale, bounds)
    got = O.combine_partials(m, l, o)
    want = O.absorbed_latent(kv, q, qr, cos, sin, dc, scale)
    assert np.abs(got - want).max() < 1e-12


def test_naive_equals_absorbed_small():
    rng = np.random.default_rng(1)
    H, dc, dR, dn, dv, L = 4, 32, 8, 16, 16, 40
    kv = rng.standard_normal((L, dc + dR)).astype(np.float32)
    WK = (rng.standard_normal((H * dn, dc)) * 0.1).astype(np.float32)
    WV = (rng.standard_normal((H * dv, dc)) * 0.1).astype(np.float32)
    qn = rng.standard_normal((H, dn)).astype(np.float32)
    qr = rng.standard_normal((H, dR)).astype(np.float32)
    cos, sin = O.rope_tables(L, dR)
    a = O.naive_decode(kv, WK, WV, qn, qr, cos, sin, H, dc, dn, dR, dv)
    b = O.absorbed_decode(kv, O.absorb_query(qn, WK, H, dc), qr, WV, cos, sin, H, dc, dn, dR, dv)
    assert np.abs(a - b).max() < 1e-5
