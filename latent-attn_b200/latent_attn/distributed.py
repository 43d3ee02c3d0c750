"""Multi-GPU MLA decode: one process per GPU, ``torch.distributed`` (NCCL) for the plumbing.

The reference decodes on one GPU only. Two ways of spreading the same decode over
the GPUs of one node are provided here:

* **Batch sharding** (many sequences). Every rank decodes a subset of the
  sequences against its own copy of their caches; no data crosses GPUs.
  ``lpt_shard`` assigns sequences longest-first to the least-loaded rank, so
  the per-rank sums of cache rows (the work) are balanced.
* **KV-range sharding** (one sequence too long for one GPU's share of the step).
  Rank ``r`` holds rows ``kv_range(L, world, r)`` of the cache, decodes them
  with ``mla_decode_partial`` (positions offset by the range start, so RoPE
  angles match a single-GPU decode), and the per-head partials -- max ``m``,
  sum of exponentials ``l`` and the unnormalised latent sum ``o`` (512 floats
  per head) -- are exchanged with one all-gather. Every rank then merges all
  ranks' partials with ``mla_combine_partials`` (log-sum-exp merge + W_UV), so
  every rank ends with the full output.

The all-gather moves ``world * B * H * (2 + d_c) * 4`` bytes (1 MiB for one
DeepSeek-V2 token on 4 GPUs), small next to the cache each rank streams.
"""

from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist


def lpt_shard(lens: Sequence[int], world: int) -> List[List[int]]:
    """Indices of the sequences each of ``world`` ranks decodes.

    Longest-processing-time order: sequences sorted by length (longest first,
    ties by index) go to the rank with the smallest total so far (lowest rank
    on ties). Every index appears exactly once; each rank's list is ascending.
    The largest per-rank total is at most 4/3 of the optimum (Graham's bound).
    """
    if world < 1:
        raise ValueError("world must be >= 1")
    order = sorted(range(len(lens)), key=lambda i: (-int(lens[i]), i))
    loads = [0] * world
    parts: List[List[int]] = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda k: (loads[k], k))
        parts[r].append(i)
        loads[r] += int(lens[i])
    return [sorted(p) for p in parts]


def kv_range(total_len: int, world: int, rank: int) -> Tuple[int, int]:
    """Rows ``[lo, hi)`` of a ``total_len``-row cache held by ``rank``.

    Contiguous ranges, sizes differing by at most one row, in rank order, so
    rank ``r``'s first row is at RoPE position ``lo``. Every rank needs at least
    one row (``total_len >= world``).
    """
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} out of range for world {world}")
    if total_len < world:
        raise ValueError(f"KV-range sharding needs at least one row per rank ({total_len} rows, {world} ranks)")
    return total_len * rank // world, total_len * (rank + 1) // world


def gather_partials(ml: torch.Tensor, o: torch.Tensor, group=None,
                    out_ml: Optional[torch.Tensor] = None, out_o: Optional[torch.Tensor] = None
                    ) -> Tuple[torch.Tensor, torch.Tensor]:
    """All-gather every rank's partials, stacked in rank order.

    ``ml`` (B, H, 2) and ``o`` (B, H, d_c) fp32 -> (world, B, H, 2) and
    (world, B, H, d_c). Pass ``out_ml`` / ``out_o`` to reuse buffers across steps.
    Every rank must call this in the same order (it is a collective).
    """
    world = dist.get_world_size(group)
    if out_ml is None:
        out_ml = torch.empty((world,) + tuple(ml.shape), dtype=ml.dtype, device=ml.device)
    if out_o is None:
        out_o = torch.empty((world,) + tuple(o.shape), dtype=o.dtype, device=o.device)
    if out_ml.shape[0] != world or out_o.shape[0] != world:
        raise ValueError("gather buffers must have world_size as their leading dimension")
    dist.all_gather_into_tensor(out_ml, ml.contiguous().unsqueeze(0), group=group)
    dist.all_gather_into_tensor(out_o, o.contiguous().unsqueeze(0), group=group)
    return out_ml, out_o


class KVRangeDecoder:
    """Decode one token per sequence over a cache whose rows are split across ranks.

    ``kv_local`` holds this rank's rows ``[pos_offset, pos_offset + n)`` of every
    sequence (B sequences of ``n`` rows each, packed). ``rope_cos`` / ``rope_sin``
    are the full tables (they are indexed by absolute position). The gather
    buffers are allocated on the first call and reused.
    """

    def __init__(self, cfg, group=None):
        self.cfg = cfg
        self.group = group
        self._ml = None
        self._o = None

    def __call__(self, kv_local: torch.Tensor, q_rope: torch.Tensor, W_UV: torch.Tensor,
                 rope_cos: torch.Tensor, rope_sin: torch.Tensor, *, pos_offset: int,
                 q_absorbed: Optional[torch.Tensor] = None, q_nope: Optional[torch.Tensor] = None,
                 W_UK: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
                 workspace: Optional[torch.Tensor] = None, timer=None) -> torch.Tensor:
        from latent_attn import _C
        c = self.cfg
        dims = (c.d_model, c.kv_lora_rank, c.qk_nope_head_dim, c.qk_rope_head_dim, c.num_heads, c.v_head_dim)
        ml, o = _C.mla_decode_partial(kv_local, q_rope, W_UV, rope_cos, rope_sin, *dims,
                                      q_absorbed=q_absorbed, q_nope=q_nope, W_UK=W_UK,
                                      kv_pos_offset=pos_offset, workspace=workspace, timer=timer)
        world = dist.get_world_size(self.group)
        if self._ml is None or self._ml.shape[1:] != ml.shape or self._ml.device != ml.device:
            self._ml = torch.empty((world,) + tuple(ml.shape), dtype=ml.dtype, device=ml.device)
            self._o = torch.empty((world,) + tuple(o.shape), dtype=o.dtype, device=o.device)
        gml, go = gather_partials(ml, o, self.group, self._ml, self._o)
        return _C.mla_combine_partials(gml, go, W_UV, *dims, out=out)


__all__ = ["lpt_shard", "kv_range", "gather_partials", "KVRangeDecoder"]
