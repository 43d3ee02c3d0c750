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

The exchanges run either through NCCL (``exchange="nccl"``) or inside the
library's own kernels (``exchange="p2p"``, the default): every rank maps the
others' buffers (CUDA IPC, ``PeerExchange``) and the kernels store into them
over NVLink, flag their receivers, and a bounded wait kernel orders the next
kernel after the flags. Flags carry a device-resident step counter, so the
exchange can be captured in a CUDA graph and replayed.

* Batches up to ``GATHER_MAX_BATCH`` (the long-sequence case) take one exchange
  inside one kernel (``mla_decode_kv_range``): block h merges this rank's
  records of head h, stores the partial into every rank's receive area as
  16-byte units that carry the step number beside each value, reads the other
  ranks' partials of head h from its own area (a bounded spin on the data
  itself: no flag, no fence), merges them and projects. Every rank merges all
  heads: one block per head costs the same for 64 or 128 heads, so the output
  all-gather is saved. The receive area is double-buffered by step parity.
  (``mla_decode_partial_gather`` + ``mla_peer_wait`` +
  ``mla_combine_partials_gathered`` are the same exchange as three kernels.)
* Larger batches keep the head-sliced pair: ``mla_decode_partial_put`` stores
  each head slice into its owner's receive area, and ``mla_combine_partials_put``
  stores the merged rows into every rank's output area.
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


# Largest batch the gathered exchange takes (the GEMV merge kernels' limit).
GATHER_MAX_BATCH = 4


def _blocks_for(nbytes: int) -> int:
    """Thread blocks a put kernel gives one destination: one per 16 KiB, 1 to 32."""
    return max(1, min(32, -(-nbytes // 16384)))


class PeerExchange:
    """Peer-memory buffers of the KV-range exchange on the ranks of one node.

    Every rank allocates one IPC buffer holding the flag words of the two exchanges (one word per
    sender for each), the receive area of the partials (``halves`` copies of world blocks of
    ``slice_bytes``; two halves double-buffer it by the step's flag value) and the output area
    (``out_bytes``); the handles are all-gathered once and every rank maps every peer's buffer.
    ``sig_partials`` / ``sig_outputs`` describe how this rank's kernels signal the receivers of
    each exchange (flag word ``rank`` or ``world + rank``); the matching waits are
    ``wait_partials`` and ``wait_outputs``, and the step's last wait advances the step counter.
    ``close()`` is a collective (unmap everywhere, barrier, free)."""

    def __init__(self, slice_bytes: int, out_bytes: int, device: torch.device, group=None, halves: int = 1):
        from latent_attn import _C
        self.group, self.device = group, device
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.slice_bytes, self.out_bytes = slice_bytes, out_bytes
        self.parity_bytes = -(-self.world * slice_bytes // 256) * 256   # one half of the receive area
        self.halves = halves
        self.flag_bytes = -(-2 * self.world * 4 // 256) * 256
        self.recv_off = self.flag_bytes
        self.out_off = self.recv_off + halves * self.parity_bytes
        total = self.out_off + -(-out_bytes // 256) * 256
        self.buf = _C.IpcBuffer(total, device)
        handles = [None] * self.world
        dist.all_gather_object(handles, self.buf.handle, group=group)
        self.mapped = []
        ptrs = []
        try:
            for q in range(self.world):
                if q == self.rank:
                    ptrs.append(self.buf.ptr)
                else:
                    ptrs.append(_C.ipc_open(handles[q], device))
                    self.mapped.append(ptrs[-1])
        except Exception:
            for p in self.mapped:
                _C.ipc_close(p, device)
            self.buf.free()
            raise
        base = torch.tensor(ptrs, dtype=torch.int64, device=device)
        self.flag_ptrs = base
        self.recv_ptrs = base + self.recv_off
        self.out_ptrs = base + self.out_off
        self.flags = self.buf.view(torch.int32, 2 * self.world)
        self.epoch = torch.zeros(1, dtype=torch.int32, device=device)
        self.status = torch.zeros(1, dtype=torch.int32, device=device)
        self.counters = torch.zeros(2 * self.world, dtype=torch.int32, device=device)
        self.done = torch.zeros(1, dtype=torch.int32, device=device)   # block counter of the one-kernel exchange
        self.sig_partials = _C.PeerSignal(self.flag_ptrs, self.rank, self.epoch, self.counters[:self.world])
        self.sig_outputs = _C.PeerSignal(self.flag_ptrs, self.world + self.rank, self.epoch,
                                         self.counters[self.world:])

    def recv(self, dtype=torch.float32) -> torch.Tensor:
        """The receive area: every half (``halves * parity_bytes`` bytes) as one flat tensor."""
        return self.buf.view(dtype, self.halves * self.parity_bytes // 4, self.recv_off)

    def out(self, dtype=torch.float32) -> torch.Tensor:
        return self.buf.view(dtype, self.out_bytes // 4, self.out_off)

    def wait_partials(self, advance: bool = False) -> None:
        """Orders the stream after every rank's partials for this rank have landed; with
        ``advance`` it ends the step (the gathered exchange has no second half)."""
        from latent_attn import _C
        _C.peer_wait(self.flags[:self.world], self.epoch, advance, self.status)

    def wait_outputs(self) -> None:
        """Orders the stream after every rank's outputs have landed; ends the exchange step."""
        from latent_attn import _C
        _C.peer_wait(self.flags[self.world:], self.epoch, True, self.status)

    def all_to_all(self, send: torch.Tensor) -> None:
        """Put kernel: slice q of ``send`` (world slices of ``slice_bytes``) to rank q's receive
        block ``rank``; then ``wait_partials``."""
        from latent_attn import _C
        sb = self.slice_bytes
        _C.peer_put(send, 1, sb, 0, sb, self.recv_ptrs, 0, self.rank * sb, _blocks_for(sb), self.sig_partials)
        self.wait_partials()

    def all_gather_rows(self, src: torch.Tensor, rows: int, row_bytes: int, dst_pitch: int) -> None:
        """Put kernel: ``src`` (rows x row_bytes) to every rank's output area at column offset
        ``rank * row_bytes`` (rows ``dst_pitch`` apart); then ``wait_outputs``."""
        from latent_attn import _C
        _C.peer_put(src, rows, row_bytes, row_bytes, 0, self.out_ptrs, dst_pitch, self.rank * row_bytes,
                    _blocks_for(rows * row_bytes), self.sig_outputs)
        self.wait_outputs()

    def check(self) -> None:
        """Raises if a wait of this rank gave up (a peer did not deliver within 2 s)."""
        if int(self.status.item()):
            raise RuntimeError("peer exchange: a wait for a peer's data timed out")

    def close(self) -> None:
        from latent_attn import _C
        if self.buf is None:
            return
        torch.cuda.synchronize(self.device)
        for p in self.mapped:
            _C.ipc_close(p, self.device)
        self.mapped = []
        dist.barrier(group=self.group)
        self.buf.free()
        self.buf = None


class KVRangeDecoder:
    """Decode one token per sequence over a cache whose rows are split across ranks.

    ``kv_local`` holds this rank's rows ``[pos_offset, pos_offset + n)`` of every
    sequence (B sequences of ``n`` rows each, packed). ``rope_cos`` / ``rope_sin``
    are the full tables (they are indexed by absolute position), or both None for
    on-the-fly RoPE. Exchange buffers are allocated on the first call and reused.
    When the ranks divide the heads, each rank merges and projects its slice of the
    heads (one all-to-all, one output all-gather): through peer memory with
    ``exchange="p2p"`` (the default; ranks of one node) or NCCL with
    ``exchange="nccl"``. Otherwise every rank merges all partials after an NCCL
    all-gather.

    With the peer-memory exchange and no ``out``, the returned tensor is the
    exchange's output area: it is overwritten by the next call. ``close()``
    releases the peer buffers (a collective).
    """

    def __init__(self, cfg, group=None, exchange: str = "p2p"):
        if exchange not in ("p2p", "nccl"):
            raise ValueError("exchange must be 'p2p' or 'nccl'")
        self.cfg = cfg
        self.group = group
        self.exchange = exchange
        self._buf = {}
        self._peer = None
        self._peer_key = None

    def _get(self, name, shape, like):
        t = self._buf.get(name)
        if t is None or tuple(t.shape) != tuple(shape) or t.device != like.device:
            t = torch.empty(shape, dtype=torch.float32, device=like.device)
            self._buf[name] = t
        return t

    def _peers(self, B, hs, world, device, gather) -> PeerExchange:
        c = self.cfg
        key = (B, hs, world, device, gather)
        if self._peer_key != key:
            if self._peer is not None:
                self._peer.close()
            R = c.kv_lora_rank + 4
            if gather:   # every rank's (B, H) rows as 16-byte {value, step, value, step} units, double-buffered
                self._peer = PeerExchange(B * c.num_heads * R * 8, 0, device, self.group, halves=2)
            else:
                self._peer = PeerExchange(B * hs * R * 4, B * world * hs * c.v_head_dim * 4, device, self.group)
            self._peer_key = key
        return self._peer

    def check(self) -> None:
        if self._peer is not None:
            self._peer.check()

    def close(self) -> None:
        if self._peer is not None:
            self._peer.close()
            self._peer, self._peer_key = None, None

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
        if self.exchange == "p2p" and B <= GATHER_MAX_BATCH:
            # one exchange inside one kernel: block h stores this rank's partial of head h into every
            # rank's receive area (NVLink stores carrying the step number), reads the others' partials
            # of head h from its own area, merges them and projects all heads
            px = self._peers(B, H, world, q_rope.device, True)
            if out is None:
                out = self._get("full", (B, H, dv), q_rope)
            return _C.mla_decode_kv_range(kv_local, q_rope, W_UV, rope_cos, rope_sin, *dims, world=world, rank=rank,
                                          recv_ptrs=px.recv_ptrs, half_bytes=px.parity_bytes, epoch=px.epoch,
                                          counter=px.done, status=px.status, out=out, q_absorbed=q_absorbed,
                                          q_nope=q_nope, W_UK=W_UK, kv_pos_offset=pos_offset, workspace=workspace,
                                          timer=timer)
        if H % world == 0:
            hs = H // world
            W_slice = W_UV[rank * hs * dv:(rank + 1) * hs * dv]
            if self.exchange == "p2p":
                # the export kernel stores each head slice into its owner's receive area, the merge
                # kernel stores the merged rows into every rank's output area (NVLink stores)
                px = self._peers(B, hs, world, q_rope.device, False)
                _C.mla_decode_partial_put(kv_local, q_rope, W_UV, rope_cos, rope_sin, *dims, dst_ptrs=px.recv_ptrs,
                                          dst_offset=rank * px.slice_bytes, signal=px.sig_partials,
                                          q_absorbed=q_absorbed, q_nope=q_nope, W_UK=W_UK, kv_pos_offset=pos_offset,
                                          workspace=workspace, timer=timer)
                px.wait_partials()
                recv = px.recv()[:world * B * hs * (dc + 4)].view(world, B, hs, dc + 4)
                _C.mla_combine_partials_put(recv, W_slice, *dims, dst_ptrs=px.out_ptrs, dst_offset=rank * hs * dv * 4,
                                            dst_pitch=H * dv * 4, signal=px.sig_outputs,
                                            scratch=self._get("slice", (B, hs, dv), q_rope))
                px.wait_outputs()
                full = px.out().view(B, H, dv)
                if out is None:
                    return full
                return out.copy_(full)
            send = self._get("send", (world, B, hs, dc + 4), q_rope)
            _C.mla_decode_partial_packed(kv_local, q_rope, W_UV, rope_cos, rope_sin, *dims, num_slices=world,
                                         q_absorbed=q_absorbed, q_nope=q_nope, W_UK=W_UK,
                                         kv_pos_offset=pos_offset, workspace=workspace, timer=timer, out=send)
            recv = exchange_head_slices(send, self.group, out=self._get("recv", send.shape, q_rope))
            o_slice = _C.mla_combine_partials_packed(recv, W_slice, *dims, out=self._get("slice", (B, hs, dv), q_rope))
            staging = self._get("stage", (world, B, hs, dv), q_rope) if B > 1 else None
            return gather_head_slices(o_slice, self.group, out=out, staging=staging)
        ml, o = _C.mla_decode_partial(kv_local, q_rope, W_UV, rope_cos, rope_sin, *dims,
                                      q_absorbed=q_absorbed, q_nope=q_nope, W_UK=W_UK,
                                      kv_pos_offset=pos_offset, workspace=workspace, timer=timer)
        gml, go = gather_partials(ml, o, self.group, self._get("gml", (world,) + tuple(ml.shape), ml),
                                  self._get("go", (world,) + tuple(o.shape), o))
        return _C.mla_combine_partials(gml, go, W_UV, *dims, out=out)


__all__ = ["lpt_shard", "kv_range", "gather_partials", "packed_row", "exchange_head_slices", "gather_head_slices",
           "GATHER_MAX_BATCH", "PeerExchange", "KVRangeDecoder"]
