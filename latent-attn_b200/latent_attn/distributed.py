"""Multi-GPU MLA decode: one process per GPU, ``torch.distributed`` (NCCL) for the plumbing.

The reference decodes on one GPU only. Two ways of spreading the same decode over
the GPUs of one node are provided here:

* **Batch sharding** (many sequences). Every rank decodes a subset of the
  sequences against its own copy of their caches; no data crosses GPUs.
  ``lpt_shard`` assigns sequences longest-first to the least-loaded rank, so
  the per-rank sums of cache rows (the work) are balanced.
* **KV-range sharding** (one sequence too long for one GPU's share of the step).
  Rank ``r`` holds rows ``kv_range(L, world, r)`` of the cache and decodes them
  with positions offset by the range start (so RoPE angles match a single-GPU
  decode) into per-head partials: max ``m``, sum of exponentials ``l`` and the
  unnormalised latent sum ``o`` (512 floats per head). The heads are then split
  over the ranks: ``mla_decode_partial_packed`` writes the partials as packed
  rows grouped by head slice, one all-to-all (``exchange_head_slices``) brings
  every rank the partials of its own ``H / world`` heads from all ranks, the rank
  merges them and projects through its slice of W_UV
  (``mla_combine_partials_packed``), and an all-gather of the 128-wide outputs
  (``gather_head_slices``) gives every rank the full output.

The all-to-all moves ``B * H * (d_c + 4) * 4 * (world - 1) / world`` bytes per
rank (about 0.25 MiB for one DeepSeek-V2 token), the output all-gather
``B * H * dv * 4`` bytes, and each rank merges and projects only its slice of
the heads. With a head count the ranks do not divide, the partials are
all-gathered instead and every rank merges all of them (``gather_partials``).
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


def packed_row(b: int, h: int, batch: int, heads: int, slices: int) -> int:
    """Row of (token b, head h) in the packed partial layout of ``mla_decode_partial_packed``:
    rows ordered (head slice, token, head within the slice), ``heads / slices`` heads a slice."""
    hs = heads // slices
    return ((h // hs) * batch + b) * hs + h % hs


def exchange_head_slices(packed: torch.Tensor, group=None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """All-to-all of packed partials: ``packed`` is (world, B, H / world, R) with block q holding the
    heads of rank q; the result is (world, B, H / world, R) with block p holding rank p's partials
    of this rank's heads. A collective: every rank calls it in the same order."""
    world = dist.get_world_size(group)
    if packed.shape[0] != world:
        raise ValueError("packed partials must have world_size head slices as their leading dimension")
    if out is None:
        out = torch.empty_like(packed)
    dist.all_to_all_single(out, packed, group=group)
    return out


def gather_head_slices(o_slice: torch.Tensor, group=None, out: Optional[torch.Tensor] = None,
                       staging: Optional[torch.Tensor] = None) -> torch.Tensor:
    """All-gather every rank's output slice (B, H / world, dv), in rank (= head) order, into the full
    (B, H, dv) output. With one token the slices land in place; otherwise through ``staging``
    (world, B, H / world, dv) and one reordering copy."""
    world = dist.get_world_size(group)
    B, hs, dv = o_slice.shape
    if out is None:
        out = torch.empty(B, world * hs, dv, dtype=o_slice.dtype, device=o_slice.device)
    if B == 1:
        dist.all_gather_into_tensor(out.view(world * hs, dv), o_slice.view(hs, dv), group=group)
        return out
    if staging is None:
        staging = torch.empty((world,) + tuple(o_slice.shape), dtype=o_slice.dtype, device=o_slice.device)
    dist.all_gather_into_tensor(staging.view(world * B, hs, dv), o_slice.contiguous(), group=group)
    out.copy_(staging.permute(1, 0, 2, 3).reshape(B, world * hs, dv))
    return out


class KVRangeDecoder:
    """Decode one token per sequence over a cache whose rows are split across ranks.

    ``kv_local`` holds this rank's rows ``[pos_offset, pos_offset + n)`` of every
    sequence (B sequences of ``n`` rows each, packed). ``rope_cos`` / ``rope_sin``
    are the full tables (they are indexed by absolute position), or both None for
    on-the-fly RoPE. Exchange buffers are allocated on the first call and reused.
    When the ranks divide the heads, each rank merges and projects its slice of the
    heads (one all-to-all, one output all-gather); otherwise every rank merges all
    partials after an all-gather.
    """

    def __init__(self, cfg, group=None):
        self.cfg = cfg
        self.group = group
        self._buf = {}

    def _get(self, name, shape, like):
        t = self._buf.get(name)
        if t is None or tuple(t.shape) != tuple(shape) or t.device != like.device:
            t = torch.empty(shape, dtype=torch.float32, device=like.device)
            self._buf[name] = t
        return t

    def __call__(self, kv_local: torch.Tensor, q_rope: torch.Tensor, W_UV: torch.Tensor,
                 rope_cos: Optional[torch.Tensor], rope_sin: Optional[torch.Tensor], *, pos_offset: int,
                 q_absorbed: Optional[torch.Tensor] = None, q_nope: Optional[torch.Tensor] = None,
                 W_UK: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
                 workspace: Optional[torch.Tensor] = None, timer=None) -> torch.Tensor:
        from latent_attn import _C
        c = self.cfg
        dims = (c.d_model, c.kv_lora_rank, c.qk_nope_head_dim, c.qk_rope_head_dim, c.num_heads, c.v_head_dim)
        world = dist.get_world_size(self.group)
        rank = dist.get_rank(self.group)
        B, H, dc, dv = q_rope.size(0), c.num_heads, c.kv_lora_rank, c.v_head_dim
        if H % world == 0:
            hs = H // world
            send = self._get("send", (world, B, hs, dc + 4), q_rope)
            _C.mla_decode_partial_packed(kv_local, q_rope, W_UV, rope_cos, rope_sin, *dims, num_slices=world,
                                         q_absorbed=q_absorbed, q_nope=q_nope, W_UK=W_UK,
                                         kv_pos_offset=pos_offset, workspace=workspace, timer=timer, out=send)
            recv = exchange_head_slices(send, self.group, out=self._get("recv", send.shape, q_rope))
            o_slice = _C.mla_combine_partials_packed(recv, W_UV[rank * hs * dv:(rank + 1) * hs * dv], *dims,
                                                     out=self._get("slice", (B, hs, dv), q_rope))
            staging = self._get("stage", (world, B, hs, dv), q_rope) if B > 1 else None
            return gather_head_slices(o_slice, self.group, out=out, staging=staging)
        ml, o = _C.mla_decode_partial(kv_local, q_rope, W_UV, rope_cos, rope_sin, *dims,
                                      q_absorbed=q_absorbed, q_nope=q_nope, W_UK=W_UK,
                                      kv_pos_offset=pos_offset, workspace=workspace, timer=timer)
        gml, go = gather_partials(ml, o, self.group, self._get("gml", (world,) + tuple(ml.shape), ml),
                                  self._get("go", (world,) + tuple(o.shape), o))
        return _C.mla_combine_partials(gml, go, W_UV, *dims, out=out)


__all__ = ["lpt_shard", "kv_range", "gather_partials", "packed_row", "exchange_head_slices", "gather_head_slices",
           "KVRangeDecoder"]
