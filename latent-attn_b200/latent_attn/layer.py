"""``LatentAttentionLayer``: the reference's model layer (latent_attn/__init__.py:41-198 of
anishesg/latent-attn) on this library's kernels.

Same parameters (names, shapes, initialisation), same ``forward(x, kv_cache)`` contract and
result: ``q_absorbed = x @ W_Q_absorbed^T`` and ``q_rope = x @ W_Q_rope^T`` (not rotated, as in
the reference), the fused absorbed decode with W_UV in the cache's dtype, then ``@ W_O^T``
(latent_attn/__init__.py:110-145). The three projections run on the tcgen05 projection GEMM
(``_C.linear``) with weights and activations in the cache's 16-bit type; the decode runs through
``mla_decode``.

``decode_step`` is the batched form for a serving loop: B tokens (B <= 256), each attending to
its own sequence (variable lengths, contiguous or paged cache), optionally with the query's RoPE
part rotated to the token's position.

``reference_forward`` is the reference's pure-torch check with its shape error corrected: the
reference multiplies ``(H, d_c) @ (H * dn, d_c)`` (latent_attn/__init__.py:183), which cannot
run. Since ``q_absorbed`` already lives in the latent space, the nope score is
``q_absorbed . c_t`` (the absorbed identity the fused path computes), and the rope score and
softmax are the reference's.
"""

from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn as nn

from . import MLAConfig, _C
from .synthetic import build_rope_tables


def _rotate_half(q: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    half = q.shape[-1] // 2
    q0, q1 = q[..., :half], q[..., half:]
    return torch.cat([q0 * cos - q1 * sin, q0 * sin + q1 * cos], dim=-1)


class LatentAttentionLayer(nn.Module):
    """Multi-head latent attention with the absorbed query projection (drop-in for the reference's
    ``latent_attn.LatentAttentionLayer``)."""

    def __init__(self, cfg: MLAConfig, max_seq_len: int = 8192) -> None:
        super().__init__()
        self.cfg = cfg
        self.max_seq_len = max_seq_len
        H, dc, dR, dn, dv, dm = (cfg.num_heads, cfg.kv_lora_rank, cfg.qk_rope_head_dim, cfg.qk_nope_head_dim,
                                 cfg.v_head_dim, cfg.d_model)
        self.W_Q_absorbed = nn.Parameter(torch.empty(H * dc, dm))
        self.W_Q_rope = nn.Parameter(torch.empty(H * dR, dm))
        self.W_UK = nn.Parameter(torch.empty(H * dn, dc))
        self.W_UV = nn.Parameter(torch.empty(H * dv, dc))
        self.W_O = nn.Parameter(torch.empty(dm, H * dv))
        self._init_weights()
        cos, sin = build_rope_tables(max_seq_len, dR)
        self.register_buffer("rope_cos", cos)
        self.register_buffer("rope_sin", sin)
        self._lowp = {}

    def _init_weights(self) -> None:
        std = 0.02
        nn.init.normal_(self.W_Q_absorbed, std=std)
        nn.init.normal_(self.W_Q_rope, std=std)
        nn.init.normal_(self.W_UK, std=std)
        nn.init.normal_(self.W_UV, std=std)
        nn.init.normal_(self.W_O, std=std / math.sqrt(2.0))

    @staticmethod
    def from_config(cfg: MLAConfig, max_seq_len: int = 8192) -> "LatentAttentionLayer":
        return LatentAttentionLayer(cfg, max_seq_len)

    def _weight(self, name: str, dtype: torch.dtype) -> torch.Tensor:
        """16-bit copy of a parameter, refreshed when the parameter changes."""
        p = getattr(self, name)
        key = (name, dtype)
        hit = self._lowp.get(key)
        stamp = (p.data_ptr(), p._version, p.device)
        if hit is None or hit[0] != stamp:
            hit = (stamp, p.detach().to(dtype).contiguous())
            self._lowp[key] = hit
        return hit[1]

    def _w_uv_fp16(self) -> torch.Tensor:
        return self._weight("W_UV", torch.float16)

    def _w_uk_fp16(self) -> torch.Tensor:
        return self._weight("W_UK", torch.float16)

    def forward(self, x: torch.Tensor, kv_cache: torch.Tensor) -> torch.Tensor:
        """One decode token: ``x`` (d_model,) or (1, d_model), ``kv_cache`` (seq_len, d_c + d_R)
        fp16/bf16 on CUDA. Returns (d_model,) fp32."""
        if x.dim() == 2:
            x = x.squeeze(0)
        assert x.dim() == 1 and x.size(0) == self.cfg.d_model
        return self.decode_step(x.unsqueeze(0), kv_cache)[0]

    def decode_step(self, x: torch.Tensor, kv_cache: torch.Tensor, *, seq_lens: Optional[torch.Tensor] = None,
                    kv_offsets: Optional[torch.Tensor] = None, max_seq_len: Optional[int] = None,
                    seq_lens_host=None, page_table: Optional[torch.Tensor] = None, page_rows: int = 0,
                    positions: Optional[torch.Tensor] = None, rope_tables: bool = True,
                    workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
        """B decode tokens: ``x`` (B, d_model) -> (B, d_model) fp32.

        Token b attends to its sequence of ``kv_cache`` (``seq_lens`` / ``kv_offsets`` /
        ``page_table`` as in ``mla_decode``; without them the B sequences are ``kv_cache.size(0) //
        B`` rows each). ``positions`` (B,) int: rotate the query's RoPE part to these positions
        (the reference leaves it unrotated). ``rope_tables=False`` lets the kernels compute the
        cache's RoPE on the fly instead of reading the layer's tables."""
        from .functional import mla_decode
        cfg = self.cfg
        H, dc, dR, dv = cfg.num_heads, cfg.kv_lora_rank, cfg.qk_rope_head_dim, cfg.v_head_dim
        dt = kv_cache.dtype
        B = x.size(0)
        xh = x.to(dt).contiguous()
        q_abs = _C.linear(xh, self._weight("W_Q_absorbed", dt)).view(B, H, dc)
        q_r = _C.linear(xh, self._weight("W_Q_rope", dt)).view(B, H, dR)
        if positions is not None:
            # the table builder's angles (latent_attn/__init__.py:31-38) at each token's position
            dims = torch.arange(dR // 2, dtype=torch.float32, device=x.device)
            freqs = 1.0 / (10000.0 ** (2.0 * dims / dR))
            ang = positions.to(device=x.device, dtype=torch.float32)[:, None] * freqs[None, :]
            q_r = _rotate_half(q_r, ang.cos()[:, None, :], ang.sin()[:, None, :]).contiguous()
        if max_seq_len is None:
            max_seq_len = kv_cache.size(0) // B if seq_lens is None else int(self.max_seq_len)
        if rope_tables:
            need = max_seq_len
            if need > self.rope_cos.size(0):
                cos, sin = build_rope_tables(need, dR, device=kv_cache.device)
            else:
                cos = self.rope_cos[:need].to(kv_cache.device).contiguous()
                sin = self.rope_sin[:need].to(kv_cache.device).contiguous()
        else:
            cos = sin = None
        o = mla_decode(kv_cache, q_r, self._weight("W_UV", dt), cos, sin, cfg, q_absorbed=q_abs.contiguous(),
                       seq_lens=seq_lens, kv_offsets=kv_offsets, max_seq_len=max_seq_len,
                       seq_lens_host=seq_lens_host, page_table=page_table, page_rows=page_rows, workspace=workspace)
        return _C.linear(o.view(B, H * dv).to(dt), self._weight("W_O", dt))

    def reference_forward(self, x: torch.Tensor, kv_cache: torch.Tensor) -> torch.Tensor:
        """Pure-torch fp32 decode of one token (the reference's check, shape error corrected)."""
        if x.dim() == 2:
            x = x.squeeze(0)
        cfg = self.cfg
        S = kv_cache.size(0)
        c_t = kv_cache[:, :cfg.kv_lora_rank].float()
        k_rope = kv_cache[:, cfg.kv_lora_rank:].float()
        cos = self.rope_cos[:S].float().to(kv_cache.device)
        sin = self.rope_sin[:S].float().to(kv_cache.device)
        K_rope = _rotate_half(k_rope, cos, sin)
        xf = x.float()
        q_abs = (xf @ self.W_Q_absorbed.float().T).view(cfg.num_heads, cfg.kv_lora_rank)
        q_r = (xf @ self.W_Q_rope.float().T).view(cfg.num_heads, cfg.qk_rope_head_dim)
        scale = 1.0 / math.sqrt(cfg.qk_nope_head_dim + cfg.qk_rope_head_dim)
        scores = (q_abs @ c_t.T + q_r @ K_rope.T) * scale
        attn = torch.softmax(scores, dim=-1)
        o_lat = attn @ c_t                                                        # (H, d_c)
        W_UV = self.W_UV.float().view(cfg.num_heads, cfg.v_head_dim, cfg.kv_lora_rank)
        out = torch.einsum("hc,hjc->hj", o_lat, W_UV)                             # (H, dv)
        return out.reshape(-1) @ self.W_O.float().T
