"""CPU oracle for MLA decode -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference arm may import this module. It is the checker, never the product:
the library's decode path runs exclusively through the CUDA kernels in
``latent-attn_b200/csrc`` and fails loudly when they are unavailable.

Parity pin: the functions here are checked against golden vectors that were
produced by importing the reference's own ``torch_mla_reference``
(tests/test_python.py:26-63 of anishesg/latent-attn) -- see
``tests/golden/make_golden.py`` and ``tests/test_oracle.py``.

Everything is plain numpy.

* ``rope_tables`` restates ``_build_rope_tables`` (latent_attn/__init__.py:31-38);
  ``rope_tables_otf`` gives the rotation of the library's on-the-fly mode (fp32
  frequencies from a double-precision power, exact angles).
* ``naive_decode`` restates ``torch_mla_reference`` (tests/test_python.py:26-63):
  decompress ``K_nope = c @ W_UK^T`` and ``V = c @ W_UV^T``, rotate ``k_rope``,
  score with ``scale = 1/sqrt(dn + dR)`` and take a softmax, then ``out = P @ V``.
* ``absorbed_decode`` restates the fused kernel's math (src/fused_mla.cu:216-268):
  ``score = (q_abs . c_t + q_rope . RoPE(k_rope, pos)) * scale``, two-pass
  softmax, ``o_lat = sum_p w_p c_p / l``, then ``out[h, j] = o_lat . W_UV[h*dv + j]``
  (src/fused_mla.cu:258-267). It runs in float64 so it can check large shapes.
* ``layer_forward`` restates the layer-level caller (latent_attn/__init__.py:110-145) around
  ``absorbed_decode``, with the reference_forward's shape error corrected.
* ``split_partials`` / ``combine_partials`` restate the split-KV log-sum-exp
  merge that the build adds (no reference counterpart; the merge identity is
  the standard flash-decoding one).
"""

from __future__ import annotations

import math
from typing import List, Optional, Sequence, Tuple

import numpy as np


def rope_tables(seq_len: int, d_R: int, theta: float = 10000.0, pos_offset: int = 0
                ) -> Tuple[np.ndarray, np.ndarray]:
    """(cos, sin), each (seq_len, d_R/2) float32 (latent_attn/__init__.py:31-38)."""
    half = d_R // 2
    pos = np.arange(pos_offset, pos_offset + seq_len, dtype=np.float32)
    dims = np.arange(half, dtype=np.float32)
    freqs = (np.float32(1.0) / (np.float32(theta) ** (np.float32(2.0) * dims / np.float32(d_R)))).astype(np.float32)
    ang = (pos[:, None] * freqs[None, :]).astype(np.float32)
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def rope_tables_otf(seq_len: int, d_R: int, theta: float = 10000.0, pos_offset: int = 0
                    ) -> Tuple[np.ndarray, np.ndarray]:
    """(cos, sin) of the library's on-the-fly RoPE mode (no tables passed): the reference
    builder's rotation (latent_attn/__init__.py:31-38) with ``freq_i = theta^(-2i/d_R)`` taken
    as the double-precision power rounded once to fp32 and the angle ``pos * freq_i`` taken
    exactly (in float64, not rounded to fp32 as the table builder rounds it); cos / sin
    evaluated in float64, then rounded to fp32."""
    half = d_R // 2
    freqs = np.array([np.float32(theta ** (-2.0 * i / d_R)) for i in range(half)], dtype=np.float64)
    pos = np.arange(pos_offset, pos_offset + seq_len, dtype=np.float64)
    ang = pos[:, None] * freqs[None, :]
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def _rotate(k_rope: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """Rotate-half RoPE of (S, dR) rows (tests/test_python.py:41-44)."""
    half = k_rope.shape[1] // 2
    k0, k1 = k_rope[:, :half], k_rope[:, half:]
    return np.concatenate([k0 * cos - k1 * sin, k0 * sin + k1 * cos], axis=1)


def _softmax_rows(s: np.ndarray) -> np.ndarray:
    m = s.max(axis=-1, keepdims=True)
    e = np.exp(s - m)
    return e / e.sum(axis=-1, keepdims=True)


def naive_decode(kv_cache: np.ndarray, W_UK: np.ndarray, W_UV: np.ndarray,
                 q_nope: np.ndarray, q_rope: np.ndarray, cos: np.ndarray, sin: np.ndarray,
                 num_heads: int, kv_lora_rank: int, qk_nope_head_dim: int,
                 qk_rope_head_dim: int, v_head_dim: int) -> np.ndarray:
    """Decompress-then-attend for one query token, float32 (tests/test_python.py:26-63).

    kv_cache (S, dc+dR); W_UK (H*dn, dc); W_UV (H*dv, dc); q_nope (H, dn);
    q_rope (H, dR); cos/sin (S, dR/2). Returns (H, dv) float32.
    """
    S = kv_cache.shape[0]
    dc, dR, H, dn, dv = kv_lora_rank, qk_rope_head_dim, num_heads, qk_nope_head_dim, v_head_dim
    f = np.float32
    c = kv_cache[:, :dc].astype(f)
    kr = kv_cache[:, dc:dc + dR].astype(f)
    K_nope = (c @ W_UK.astype(f).T).reshape(S, H, dn)
    V = (c @ W_UV.astype(f).T).reshape(S, H, dv)
    K_rope = _rotate(kr, cos.astype(f), sin.astype(f))
    scale = f(1.0 / math.sqrt(dn + dR))
    s = np.einsum("hd,shd->hs", q_nope.astype(f), K_nope) * scale
    s = s + (q_rope.astype(f) @ K_rope.T) * scale
    p = _softmax_rows(s.astype(f)).astype(f)
    return np.einsum("hs,shv->hv", p, V).astype(f)


def absorb_query(q_nope: np.ndarray, W_UK: np.ndarray, num_heads: int, kv_lora_rank: int
                 ) -> np.ndarray:
    """q_abs[..., h, c] = sum_i q_nope[..., h, i] * W_UK[h*dn + i, c] (float64).
    Restates tests/test_python.py:98-99 / tests/test_correctness.cu:29-46."""
    dn = q_nope.shape[-1]
    W = W_UK.astype(np.float64).reshape(num_heads, dn, kv_lora_rank)
    return np.einsum("...hd,hdc->...hc", q_nope.astype(np.float64), W)


def _scores64(kv: np.ndarray, q_abs: np.ndarray, q_rope: np.ndarray, cos: np.ndarray,
              sin: np.ndarray, dc: int, scale: float) -> np.ndarray:
    c = kv[:, :dc].astype(np.float64)
    kr = _rotate(kv[:, dc:].astype(np.float64), cos.astype(np.float64), sin.astype(np.float64))
    return (q_abs.astype(np.float64) @ c.T + q_rope.astype(np.float64) @ kr.T) * scale


def absorbed_latent(kv_cache: np.ndarray, q_abs: np.ndarray, q_rope: np.ndarray,
                    cos: np.ndarray, sin: np.ndarray, kv_lora_rank: int, scale: float
                    ) -> np.ndarray:
    """Normalised latent output o_lat (H, dc), float64 (src/fused_mla.cu:226-256)."""
    s = _scores64(kv_cache, q_abs, q_rope, cos, sin, kv_lora_rank, scale)
    m = s.max(axis=1, keepdims=True)
    w = np.exp(s - m)
    l = w.sum(axis=1, keepdims=True)
    return (w @ kv_cache[:, :kv_lora_rank].astype(np.float64)) / l


def project_wuv(o_lat: np.ndarray, W_UV: np.ndarray, num_heads: int, v_head_dim: int
                ) -> np.ndarray:
    """out[..., h, j] = sum_i o_lat[..., h, i] * W_UV[h*dv + j, i] (src/fused_mla.cu:258-267)."""
    dc = W_UV.shape[1]
    W = W_UV.astype(np.float64).reshape(num_heads, v_head_dim, dc)
    return np.einsum("...hc,hjc->...hj", o_lat.astype(np.float64), W)


def absorbed_decode(kv_cache: np.ndarray, q_abs: np.ndarray, q_rope: np.ndarray,
                    W_UV: np.ndarray, cos: np.ndarray, sin: np.ndarray, num_heads: int,
                    kv_lora_rank: int, qk_nope_head_dim: int, qk_rope_head_dim: int,
                    v_head_dim: int) -> np.ndarray:
    """Fused absorbed decode for one token over one cache: (H, dv) float64."""
    scale = 1.0 / math.sqrt(qk_nope_head_dim + qk_rope_head_dim)
    o = absorbed_latent(kv_cache, q_abs, q_rope, cos, sin, kv_lora_rank, scale)
    return project_wuv(o, W_UV, num_heads, v_head_dim)


def layer_forward(x: np.ndarray, W_Q_absorbed: np.ndarray, W_Q_rope: np.ndarray, W_UV: np.ndarray,
                  W_O: np.ndarray, kv_cache: np.ndarray, cos: np.ndarray, sin: np.ndarray, num_heads: int,
                  kv_lora_rank: int, qk_nope_head_dim: int, qk_rope_head_dim: int, v_head_dim: int) -> np.ndarray:
    """One token through the reference's LatentAttentionLayer (latent_attn/__init__.py:110-198), float64:
    ``q_abs = x @ W_Q_absorbed^T``, ``q_rope = x @ W_Q_rope^T`` (unrotated, as the reference), the
    absorbed decode, then ``@ W_O^T``. Its ``reference_forward`` multiplies shapes that cannot be
    multiplied (``(H, d_c) @ (H * dn, d_c)`` at :183); the nope score is taken in the latent space
    (``q_abs . c_t``), the identity the fused path computes. x (d_model,) -> (d_model,)."""
    H, dc, dR = num_heads, kv_lora_rank, qk_rope_head_dim
    xd = x.astype(np.float64)
    q_abs = (W_Q_absorbed.astype(np.float64) @ xd).reshape(H, dc)
    q_r = (W_Q_rope.astype(np.float64) @ xd).reshape(H, dR)
    out = absorbed_decode(kv_cache, q_abs, q_r, W_UV, cos, sin, H, dc, qk_nope_head_dim, dR, v_head_dim)
    return W_O.astype(np.float64) @ out.reshape(-1)


def varlen_decode(kv_cache: np.ndarray, seq_lens: Sequence[int], kv_offsets: Sequence[int],
                  q_abs: np.ndarray, q_rope: np.ndarray, W_UV: np.ndarray, num_heads: int,
                  kv_lora_rank: int, qk_nope_head_dim: int, qk_rope_head_dim: int,
                  v_head_dim: int, theta: float = 10000.0) -> np.ndarray:
    """Batched variable-length decode as a loop of single-sequence oracles:
    sequence b attends over rows kv_offsets[b] .. +seq_lens[b] at RoPE positions
    0 .. seq_lens[b]-1. q_abs (B, H, dc), q_rope (B, H, dR). Returns (B, H, dv)."""
    dR = qk_rope_head_dim
    out = []
    for b, (L, off) in enumerate(zip(seq_lens, kv_offsets)):
        cos, sin = rope_tables(L, dR, theta)
        out.append(absorbed_decode(kv_cache[off:off + L], q_abs[b], q_rope[b], W_UV, cos, sin,
                                   num_heads, kv_lora_rank, qk_nope_head_dim, dR, v_head_dim))
    return np.stack(out)


def split_partials(kv_cache: np.ndarray, q_abs: np.ndarray, q_rope: np.ndarray,
                   cos: np.ndarray, sin: np.ndarray, kv_lora_rank: int, scale: float,
                   bounds: Sequence[int]):
    """Per-range partials (m, l, o) for ranges [bounds[i], bounds[i+1]) in float64,
    with m in natural-log units and o the UNnormalised sum_p e^(s_p - m) c_p.
    Empty ranges give m = -inf, l = 0, o = 0."""
    s = _scores64(kv_cache, q_abs, q_rope, cos, sin, kv_lora_rank, scale)
    c = kv_cache[:, :kv_lora_rank].astype(np.float64)
    H = q_abs.shape[0]
    ms, ls, os_ = [], [], []
    for a, b in zip(bounds[:-1], bounds[1:]):
        if b <= a:
            ms.append(np.full(H, -np.inf)); ls.append(np.zeros(H)); os_.append(np.zeros((H, kv_lora_rank)))
            continue
        m = s[:, a:b].max(axis=1)
        w = np.exp(s[:, a:b] - m[:, None])
        ms.append(m); ls.append(w.sum(axis=1)); os_.append(w @ c[a:b])
    return np.stack(ms), np.stack(ls), np.stack(os_)


def combine_partials(m: np.ndarray, l: np.ndarray, o: np.ndarray) -> np.ndarray:
    """Log-sum-exp merge over axis 0: m (R, H), l (R, H), o (R, H, dc) ->
    normalised o_lat (H, dc)."""
    M = m.max(axis=0)
    a = np.where(np.isfinite(m), np.exp(m - M[None, :]), 0.0)
    L = (a * l).sum(axis=0)
    return (a[:, :, None] * o).sum(axis=0) / L[:, None]


def compare(out: np.ndarray, ref: np.ndarray) -> dict:
    """max-abs, norm-relative max error (max|d| / max|ref|) and cosine."""
    a = np.asarray(out, dtype=np.float64).ravel()
    b = np.asarray(ref, dtype=np.float64).ravel()
    d = np.abs(a - b)
    denom = max(np.abs(b).max(), 1e-30)
    cos = float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-300))
    return {"max_abs": float(d.max()) if d.size else 0.0,
            "max_rel": float(d.max() / denom) if d.size else 0.0,
            "cosine": cos,
            "finite": bool(np.isfinite(a).all())}
