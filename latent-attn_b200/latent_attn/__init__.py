"""B200 (sm_100a) multi-head latent attention decode.

Drop-in for the reference package ``latent_attn`` (anishesg/latent-attn): the
same ``MLAConfig`` (latent_attn/__init__.py:13-28 there), the same functional API
(``latent_attn.functional``) and the same ``_C`` op names, backed by the CUDA
library ``libmla_b200.so`` built from ``csrc/``.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .synthetic import build_rope_tables


@dataclass
class MLAConfig:
    d_model: int
    kv_lora_rank: int        # d_c: compressed KV latent dimension
    qk_nope_head_dim: int    # per-head non-RoPE dim
    qk_rope_head_dim: int    # per-head RoPE dim (d_R)
    num_heads: int
    v_head_dim: int

    @staticmethod
    def deepseek_v2() -> "MLAConfig":
        return MLAConfig(5120, 512, 128, 64, 128, 128)

    @staticmethod
    def deepseek_v3() -> "MLAConfig":
        return MLAConfig(7168, 512, 128, 64, 128, 128)


def _build_rope_tables(seq_len: int, d_R: int, device: torch.device):
    """(cos, sin), each (seq_len, d_R // 2) fp32 (reference latent_attn/__init__.py:31-38)."""
    return build_rope_tables(seq_len, d_R, device=device)


from .layer import LatentAttentionLayer  # noqa: E402  (needs MLAConfig above)

__all__ = ["MLAConfig", "LatentAttentionLayer", "build_rope_tables", "_build_rope_tables"]
