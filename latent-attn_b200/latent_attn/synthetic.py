"""Seeded synthetic MLA decode inputs.

Two recipes are provided:

* ``baseline_inputs`` -- the workload recipe of the benchmark configurations:
  latent cache rows ``[c_t (d_c) | k_rope (d_R)]`` ~ N(0, 1), ``q_nope`` and
  ``q_rope`` ~ N(0, 1), ``W_UK`` and ``W_UV`` ~ N(0, sigma = 1/sqrt(d_c)), drawn
  in fp32 from ``torch.Generator().manual_seed(seed)`` and then cast.
* ``reference_test_inputs`` -- the recipe of the reference's own pytest
  (tests/test_python.py:89-93 in anishesg/latent-attn): cache ~ N(0, 1),
  weights ~ 0.02 * N(0, 1), queries ~ 0.1 * N(0, 1).

The RoPE table builder restates latent_attn/__init__.py:31-38 of the reference
(``freq_i = 1 / 10000^(2i/d_R)``, ``angle = pos * freq_i`` in fp32, rotate-half
pairing ``(i, i + d_R/2)``).

This module only depends on torch; it is loaded by file path from the golden
fixture generator, so it must not import anything else from this package.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import List, Optional, Sequence

import torch


def build_rope_tables(seq_len: int, d_R: int, theta: float = 10000.0,
                      pos_offset: int = 0, device="cpu"):
    """Return ``(cos, sin)``, each ``(seq_len, d_R // 2)`` fp32, for positions
    ``pos_offset .. pos_offset + seq_len - 1``."""
    half = d_R // 2
    positions = torch.arange(pos_offset, pos_offset + seq_len, dtype=torch.float32, device=device)
    dims = torch.arange(half, dtype=torch.float32, device=device)
    freqs = 1.0 / (theta ** (2.0 * dims / d_R))
    angles = positions[:, None] * freqs[None, :]
    return angles.cos(), angles.sin()


def rotate_query_rope(q_rope: torch.Tensor, position: int, theta: float = 10000.0) -> torch.Tensor:
    """Rotate ``q_rope[..., d_R]`` (fp32) to ``position`` with the same rotate-half
    convention as the cache tables. The reference never rotates the query; the
    benchmark recipe places the decode query at position ``seq_len``."""
    d_R = q_rope.shape[-1]
    cos, sin = build_rope_tables(1, d_R, theta, pos_offset=position, device=q_rope.device)
    cos, sin = cos[0], sin[0]
    half = d_R // 2
    q0, q1 = q_rope[..., :half], q_rope[..., half:]
    return torch.cat([q0 * cos - q1 * sin, q0 * sin + q1 * cos], dim=-1)


@dataclass
class MLAInputs:
    """One decode step's inputs (CPU tensors).

    ``kv_cache`` is the concatenation of every sequence's packed rows;
    sequence ``b`` occupies rows ``kv_offsets[b] .. kv_offsets[b] + seq_lens[b]``.
    Queries are ``(B, H, .)`` fp32, weights ``(H * 128, d_c)`` in ``dtype``.
    """
    kv_cache: torch.Tensor
    seq_lens: List[int]
    kv_offsets: List[int]
    q_nope: torch.Tensor
    q_rope: torch.Tensor
    W_UK: torch.Tensor
    W_UV: torch.Tensor
    dtype: torch.dtype
    meta: dict = field(default_factory=dict)

    @property
    def batch(self) -> int:
        return len(self.seq_lens)

    def q_absorbed(self) -> torch.Tensor:
        """``q_abs[b, h, c] = sum_i q_nope[b, h, i] * W_UK[h * dn + i, c]`` in fp32
        (tests/test_python.py:98-99 of the reference)."""
        B, H, dn = self.q_nope.shape
        W = self.W_UK.float().view(H, dn, -1)
        return torch.einsum("bhd,hdc->bhc", self.q_nope.float(), W).contiguous()


def _uniform_lengths(batch: int, seq_len: int) -> List[int]:
    return [int(seq_len)] * batch


def varlen_lengths(batch: int, lo: int, hi: int, seed: int = 0) -> List[int]:
    """Per-sequence lengths ~ U[lo, hi] drawn with ``torch.randint(lo, hi + 1)``."""
    g = torch.Generator().manual_seed(seed)
    return [int(x) for x in torch.randint(lo, hi + 1, (batch,), generator=g)]


def baseline_inputs(num_heads: int = 128, seq_lens: Sequence[int] = (8192,),
                    kv_lora_rank: int = 512, qk_rope_head_dim: int = 64,
                    qk_nope_head_dim: int = 128, v_head_dim: int = 128,
                    dtype: torch.dtype = torch.bfloat16, seed: int = 0,
                    rotate_query: bool = True) -> MLAInputs:
    """Benchmark-configuration recipe (one generator, fixed draw order:
    cache, q_nope, q_rope, W_UK, W_UV). With ``rotate_query`` the query's RoPE
    part is rotated to position ``seq_len`` of its sequence."""
    g = torch.Generator().manual_seed(seed)
    seq_lens = [int(s) for s in seq_lens]
    B, H = len(seq_lens), num_heads
    dc, dR, dn, dv = kv_lora_rank, qk_rope_head_dim, qk_nope_head_dim, v_head_dim
    total = sum(seq_lens)
    kv = torch.randn(total, dc + dR, generator=g)
    q_nope = torch.randn(B, H, dn, generator=g)
    q_rope = torch.randn(B, H, dR, generator=g)
    sigma = 1.0 / math.sqrt(dc)
    W_UK = torch.randn(H * dn, dc, generator=g) * sigma
    W_UV = torch.randn(H * dv, dc, generator=g) * sigma
    if rotate_query:
        q_rope = torch.stack([rotate_query_rope(q_rope[b], seq_lens[b]) for b in range(B)])
    offsets, acc = [], 0
    for s in seq_lens:
        offsets.append(acc)
        acc += s
    return MLAInputs(kv_cache=kv.to(dtype), seq_lens=seq_lens, kv_offsets=offsets,
                     q_nope=q_nope, q_rope=q_rope, W_UK=W_UK.to(dtype), W_UV=W_UV.to(dtype),
                     dtype=dtype, meta={"recipe": "baseline", "seed": seed})


def reference_test_inputs(num_heads: int, seq_len: int, batch: int = 1,
                          kv_lora_rank: int = 512, qk_rope_head_dim: int = 64,
                          qk_nope_head_dim: int = 128, v_head_dim: int = 128,
                          dtype: torch.dtype = torch.float16, seed: int = 42) -> MLAInputs:
    """The reference pytest's recipe (tests/test_python.py:89-93), drawn on a CPU
    generator: one shared cache of ``seq_len`` rows for all ``batch`` tokens."""
    g = torch.Generator().manual_seed(seed)
    H, dc, dR, dn, dv = num_heads, kv_lora_rank, qk_rope_head_dim, qk_nope_head_dim, v_head_dim
    kv = torch.randn(seq_len, dc + dR, generator=g)
    W_UK = torch.randn(H * dn, dc, generator=g) * 0.02
    W_UV = torch.randn(H * dv, dc, generator=g) * 0.02
    q_nope = torch.randn(batch, H, dn, generator=g) * 0.1
    q_rope = torch.randn(batch, H, dR, generator=g) * 0.1
    return MLAInputs(kv_cache=kv.to(dtype), seq_lens=[seq_len] * batch, kv_offsets=[0] * batch,
                     q_nope=q_nope, q_rope=q_rope, W_UK=W_UK.to(dtype), W_UV=W_UV.to(dtype),
                     dtype=dtype, meta={"recipe": "reference_test", "seed": seed, "shared_cache": True})
