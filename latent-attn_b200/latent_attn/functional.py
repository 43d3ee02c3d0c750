"""Stateless functional API, same signatures as the reference's
latent_attn/functional.py (anishesg/latent-attn, :24, :55, :88), plus the general
``mla_decode`` entry point of this library."""

from __future__ import annotations

from typing import TYPE_CHECKING, Optional, Sequence

import torch

if TYPE_CHECKING:
    from latent_attn import MLAConfig


_EXT = None


def _load_ext():
    global _EXT
    if _EXT is not None:
        return _EXT
    try:
        from latent_attn import _C, _lib
        _lib.load()
        _EXT = _C
        return _C
    except ImportError as e:
        raise ImportError(
            "latent_attn B200 library not found. "
            "Run `python latent-attn_b200/build.py` from the repo root to build it."
        ) from e


def _dims(cfg):
    return (cfg.d_model, cfg.kv_lora_rank, cfg.qk_nope_head_dim, cfg.qk_rope_head_dim,
            cfg.num_heads, cfg.v_head_dim)


def fused_mla(kv_cache: torch.Tensor, q_absorbed: torch.Tensor, q_rope: torch.Tensor,
              W_UV: torch.Tensor, rope_cos: torch.Tensor, rope_sin: torch.Tensor,
              cfg: "MLAConfig") -> torch.Tensor:
    """Single-token fused absorbed MLA decode.

    kv_cache (S, d_c + d_R) fp16/bf16; q_absorbed (H, d_c) fp32; q_rope (H, d_R) fp32;
    W_UV (H * dv, d_c) same dtype as kv_cache; rope_cos / rope_sin (S, d_R / 2) fp32.
    Returns (H, dv) fp32.
    """
    return _load_ext().fused_mla_forward(kv_cache, q_absorbed, q_rope, W_UV, rope_cos, rope_sin,
                                         *_dims(cfg))


def naive_mla(kv_cache: torch.Tensor, W_UK: torch.Tensor, W_UV: torch.Tensor, q_nope: torch.Tensor,
              q_rope: torch.Tensor, rope_cos: torch.Tensor, rope_sin: torch.Tensor,
              cfg: "MLAConfig") -> torch.Tensor:
    """Decompress-then-attend baseline for one token. Returns (H, dv) fp32."""
    return _load_ext().naive_mla_forward(kv_cache, W_UK, W_UV, q_nope, q_rope, rope_cos, rope_sin,
                                         *_dims(cfg))


def batched_fused_mla(kv_cache: torch.Tensor, q_absorbed: torch.Tensor, q_rope: torch.Tensor,
                      W_UV: torch.Tensor, rope_cos: torch.Tensor, rope_sin: torch.Tensor,
                      cfg: "MLAConfig") -> torch.Tensor:
    """B query tokens over one shared cache. q_absorbed (B, H, d_c), q_rope (B, H, d_R).
    Returns (B, H, dv) fp32."""
    return _load_ext().batched_fused_mla_forward(kv_cache, q_absorbed, q_rope, W_UV, rope_cos, rope_sin,
                                                 *_dims(cfg))


def mla_decode(kv_cache: torch.Tensor, q_rope: torch.Tensor, W_UV: torch.Tensor,
               rope_cos: Optional[torch.Tensor], rope_sin: Optional[torch.Tensor], cfg: "MLAConfig", *,
               q_absorbed: Optional[torch.Tensor] = None, q_nope: Optional[torch.Tensor] = None,
               W_UK: Optional[torch.Tensor] = None, seq_lens: Optional[torch.Tensor] = None,
               kv_offsets: Optional[torch.Tensor] = None, max_seq_len: Optional[int] = None,
               seq_lens_host: Optional[Sequence[int]] = None, shared_cache: bool = False,
               kv_pos_offset: int = 0, softmax_scale: float = 0.0, kv_row_stride: int = 0,
               kernel: int = 0, out: Optional[torch.Tensor] = None,
               workspace: Optional[torch.Tensor] = None, timer=None,
               page_table: Optional[torch.Tensor] = None, page_rows: int = 0,
               rope_theta: float = 0.0) -> torch.Tensor:
    """General decode over a (variable-length, optionally paged) batch; see ``_C.mla_decode``.
    ``rope_cos`` / ``rope_sin`` may both be ``None``: the kernels then compute the RoPE rotation
    from ``rope_theta`` (0: 10000). Returns (B, H, dv) fp32."""
    return _load_ext().mla_decode(kv_cache, q_rope, W_UV, rope_cos, rope_sin, *_dims(cfg),
                                  q_absorbed=q_absorbed, q_nope=q_nope, W_UK=W_UK, seq_lens=seq_lens,
                                  kv_offsets=kv_offsets, max_seq_len=max_seq_len,
                                  seq_lens_host=seq_lens_host, shared_cache=shared_cache,
                                  kv_pos_offset=kv_pos_offset, softmax_scale=softmax_scale,
                                  kv_row_stride=kv_row_stride, kernel=kernel, out=out, workspace=workspace,
                                  timer=timer, page_table=page_table, page_rows=page_rows,
                                  rope_theta=rope_theta)
