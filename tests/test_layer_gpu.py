"""The layer-level caller (the reference's LatentAttentionLayer, latent_attn/__init__.py:41-198) on
this library's kernels: the projection GEMM (_C.linear, mla_linear) against float64 matmuls, and
the layer's forward / batched decode_step against the float64 oracle of the corrected
reference_forward (oracle.layer_forward), at d_model 5120 and 7168 with B = 1 and 256.

Tolerance: the decode parity bound (max-abs <= 1e-2, max|d| / max|ref| <= 2e-2, cosine > 0.998),
with the oracle given the same 16-bit weights and activations the kernels read.
"""

import numpy as np
import pytest
import torch

from oracle import mla_oracle as O
from latent_attn import LatentAttentionLayer, MLAConfig, _C

pytestmark = pytest.mark.gpu

MAX_ABS, MAX_REL, MIN_COS = 1e-2, 2e-2, 0.998


def _close(got, ref, what):
    c = O.compare(np.asarray(got, np.float64), np.asarray(ref, np.float64))
    assert c["finite"] and c["max_abs"] <= MAX_ABS and c["max_rel"] <= MAX_REL and c["cosine"] > MIN_COS, (what, c)


@pytest.mark.parametrize("M,N,K", [(1, 128, 64), (17, 1000, 520), (256, 8192, 512), (1, 7168, 16384),
                                   (4, 65536, 7168)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_linear_matches_float64(M, N, K, dtype):
    """Row tiles with a ragged last tile (N = 1000), token counts from 1 to 256, and the split-K
    path (N = 7168 with K = 16384: 56 row tiles, K split over CTAs)."""
    g = torch.Generator().manual_seed(M * 7 + N + K)
    x = torch.randn(M, K, generator=g).to(dtype)
    W = (torch.randn(N, K, generator=g) / K ** 0.5).to(dtype)
    got = _C.linear(x.cuda(), W.cuda())
    want = x.double() @ W.double().T
    c = O.compare(got.cpu().numpy(), want.numpy())
    assert c["finite"] and c["max_rel"] < 1e-3 and c["cosine"] > 0.99999, c


def _layer(d_model, max_seq_len, seed):
    torch.manual_seed(seed)
    cfg = MLAConfig(d_model, 512, 128, 64, 128, 128)
    return LatentAttentionLayer(cfg, max_seq_len).cuda(), cfg


def _oracle(layer, cfg, x_row, kv_rows, dt):
    """Oracle of one token with the layer's weights rounded to the kernels' 16-bit type."""
    w = {n: getattr(layer, n).detach().to(dt).float().cpu().numpy() for n in ("W_Q_absorbed", "W_Q_rope", "W_UV", "W_O")}
    S = kv_rows.shape[0]
    cos = layer.rope_cos[:S].cpu().numpy()
    sin = layer.rope_sin[:S].cpu().numpy()
    return O.layer_forward(x_row.to(dt).float().cpu().numpy(), w["W_Q_absorbed"], w["W_Q_rope"], w["W_UV"], w["W_O"],
                           kv_rows.float().cpu().numpy(), cos, sin, cfg.num_heads, 512, 128, 64, 128)


@pytest.mark.parametrize("d_model", [5120, 7168])
def test_layer_forward_single_token(d_model):
    """forward(x, kv_cache) with the reference's contract: (d_model,) fp32 for one token."""
    layer, cfg = _layer(d_model, 4096, 1)
    g = torch.Generator().manual_seed(2)
    S = 3000
    kv = torch.randn(S, 576, generator=g).to(torch.bfloat16).cuda()
    x = torch.randn(d_model, generator=g).cuda()
    y = layer(x, kv)
    assert y.shape == (d_model,) and y.dtype == torch.float32
    want = _oracle(layer, cfg, x, kv, torch.bfloat16)
    _close(y.cpu().numpy(), want, f"forward d_model={d_model}")
    # the corrected reference_forward (fp32 torch, unrounded weights) agrees too
    ref = layer.reference_forward(x, kv).detach().double().cpu().numpy()
    _close(y.cpu().numpy(), ref, f"forward vs reference_forward d_model={d_model}")


@pytest.mark.parametrize("d_model", [5120, 7168])
def test_layer_decode_step_batch256(d_model):
    """B = 256 tokens, each over its own sequence of a variable-length batch (the projection GEMMs
    at M = 256); six tokens against the oracle."""
    layer, cfg = _layer(d_model, 512, 3)
    g = torch.Generator().manual_seed(4)
    B = 256
    lens = [1 + (97 * b) % 400 for b in range(B)]
    offs = np.concatenate([[0], np.cumsum(lens)[:-1]]).tolist()
    kv = torch.randn(sum(lens), 576, generator=g).to(torch.bfloat16).cuda()
    x = torch.randn(B, d_model, generator=g).cuda()
    y = layer.decode_step(x, kv, seq_lens=torch.tensor(lens, dtype=torch.int32, device="cuda"),
                          kv_offsets=torch.tensor(offs, dtype=torch.int64, device="cuda"), max_seq_len=max(lens),
                          seq_lens_host=lens)
    assert y.shape == (B, d_model)
    for b in (0, 1, 77, 128, 200, 255):
        want = _oracle(layer, cfg, x[b], kv[offs[b]:offs[b] + lens[b]], torch.bfloat16)
        _close(y[b].cpu().numpy(), want, f"decode_step b={b} L={lens[b]} d_model={d_model}")


def test_layer_decode_step_rotated_query_and_otf_rope():
    """decode_step with the query's RoPE part rotated to the token position and the cache's RoPE
    computed on the fly: the oracle rotates q_rope the same way and uses the on-the-fly angles."""
    layer, cfg = _layer(5120, 1024, 5)
    g = torch.Generator().manual_seed(6)
    S = 700
    kv = torch.randn(S, 576, generator=g).to(torch.bfloat16).cuda()
    x = torch.randn(1, 5120, generator=g).cuda()
    y = layer.decode_step(x, kv, positions=torch.tensor([S]), rope_tables=False)[0]
    dt = torch.bfloat16
    w = {n: getattr(layer, n).detach().to(dt).float().cpu().numpy() for n in ("W_Q_absorbed", "W_Q_rope", "W_UV", "W_O")}
    xd = x[0].to(dt).float().cpu().numpy().astype(np.float64)
    q_abs = (w["W_Q_absorbed"].astype(np.float64) @ xd).reshape(128, 512)
    q_r = (w["W_Q_rope"].astype(np.float64) @ xd).reshape(128, 64)
    qc, qs = O.rope_tables(1, 64, pos_offset=S)
    q_r = np.concatenate([q_r[:, :32] * qc - q_r[:, 32:] * qs, q_r[:, :32] * qs + q_r[:, 32:] * qc], axis=1)
    cos, sin = O.rope_tables_otf(S, 64)
    out = O.absorbed_decode(kv.float().cpu().numpy(), q_abs, q_r, w["W_UV"], cos, sin, 128, 512, 128, 64, 128)
    _close(y.cpu().numpy(), w["W_O"].astype(np.float64) @ out.reshape(-1), "rotated query, on-the-fly RoPE")
