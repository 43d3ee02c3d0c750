"""Host logic of the multi-GPU decode (latent_attn.distributed) on CPU ranks.

The ranks are ``gloo`` processes; each one stands in for a GPU. The per-rank
decode is the oracle's (the CUDA kernels need a GPU), so these tests check what
the host side decides: which rows and positions each rank owns, that the
all-gather stacks the partials in rank order, and that merging them gives the
single-device result. The CUDA path of the same steps is in test_parity_gpu.py.
"""

import math
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import mla_oracle as O
from latent_attn import distributed as D
from latent_attn import synthetic

H, DC, DR, DN, DV = 16, 512, 64, 128, 128
SCALE = 1.0 / math.sqrt(DN + DR)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _spawn(fn, world, *args):
    port = _free_port()
    mp.spawn(fn, args=(world, port) + args, nprocs=world, join=True)


def _init(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))


def _kv_problem(L, seed):
    inp = synthetic.baseline_inputs(num_heads=H, seq_lens=[L], seed=seed)
    kv = inp.kv_cache.float().numpy()
    q_abs = O.absorb_query(inp.q_nope.float().numpy(), inp.W_UK.float().numpy(), H, DC)[0]
    return kv, q_abs, inp.q_rope[0].float().numpy()


# --------------------------------------------------------------------------- pure host logic

def test_lpt_shard_covers_every_sequence_once_and_balances():
    lens = synthetic.varlen_lengths(64, 1024, 16384, seed=0)
    for world in (1, 2, 3, 4, 8):
        parts = D.lpt_shard(lens, world)
        assert len(parts) == world
        flat = sorted(i for p in parts for i in p)
        assert flat == list(range(len(lens)))
        assert all(p == sorted(p) for p in parts)
        loads = [sum(lens[i] for i in p) for p in parts]
        lower = max(sum(lens) / world, max(lens))
        assert max(loads) <= 4.0 / 3.0 * lower + 1e-9, (world, loads)
    assert D.lpt_shard(lens, 8) == D.lpt_shard(list(lens), 8)       # deterministic
    assert D.lpt_shard([], 4) == [[], [], [], []]
    assert D.lpt_shard([5, 5, 5], 4) == [[0], [1], [2], []]          # more ranks than sequences
    with pytest.raises(ValueError):
        D.lpt_shard([1], 0)


@pytest.mark.parametrize("L,world", [(131072, 8), (8192, 3), (301, 4), (4, 4)])
def test_kv_range_is_a_contiguous_balanced_cover(L, world):
    rs = [D.kv_range(L, world, r) for r in range(world)]
    assert rs[0][0] == 0 and rs[-1][1] == L
    assert all(a[1] == b[0] for a, b in zip(rs, rs[1:]))
    sizes = [hi - lo for lo, hi in rs]
    assert min(sizes) >= 1 and max(sizes) - min(sizes) <= 1


def test_kv_range_rejects_bad_arguments():
    with pytest.raises(ValueError):
        D.kv_range(3, 4, 0)
    with pytest.raises(ValueError):
        D.kv_range(100, 4, 4)


# --------------------------------------------------------------------------- gloo ranks

def _kv_range_worker(rank, world, port, L, seed):
    _init(rank, world, port)
    try:
        kv, q_abs, q_rope = _kv_problem(L, seed)
        cos, sin = O.rope_tables(L, DR)
        lo, hi = D.kv_range(L, world, rank)
        # this rank's decode over its rows only; the RoPE tables are indexed by absolute position
        m, l, o = O.split_partials(kv[lo:hi], q_abs, q_rope, cos[lo:hi], sin[lo:hi], DC, SCALE, [0, hi - lo])
        ml = torch.from_numpy(np.stack([m[0], l[0]], axis=-1)).unsqueeze(0)      # (B=1, H, 2)
        ot = torch.from_numpy(o[0]).unsqueeze(0)                                  # (B=1, H, dc)
        gml, go = D.gather_partials(ml, ot)
        assert gml.shape == (world, 1, H, 2) and go.shape == (world, 1, H, DC)
        # rank order: slot r holds rank r's range
        for r in range(world):
            a, b = D.kv_range(L, world, r)
            mr, lr, orr = O.split_partials(kv[a:b], q_abs, q_rope, cos[a:b], sin[a:b], DC, SCALE, [0, b - a])
            np.testing.assert_array_equal(gml[r, 0, :, 0].numpy(), mr[0])
            np.testing.assert_array_equal(go[r, 0].numpy(), orr[0])
        merged = O.combine_partials(gml[:, 0, :, 0].numpy(), gml[:, 0, :, 1].numpy(), go[:, 0].numpy())
        want = O.absorbed_latent(kv, q_abs, q_rope, cos, sin, DC, SCALE)
        np.testing.assert_allclose(merged, want, rtol=1e-10, atol=1e-12)
        # reuse of caller buffers: same result
        gml2, go2 = D.gather_partials(ml, ot, out_ml=torch.empty_like(gml), out_o=torch.empty_like(go))
        assert torch.equal(gml2, gml) and torch.equal(go2, go)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,L", [(2, 1000), (3, 301)])
def test_kv_range_shards_merge_to_the_single_device_decode(world, L):
    _spawn(_kv_range_worker, world, L, 7)


def _batch_worker(rank, world, port, lens, seed):
    _init(rank, world, port)
    try:
        inp = synthetic.baseline_inputs(num_heads=H, seq_lens=lens, seed=seed)
        kv = inp.kv_cache.float().numpy()
        q_abs = O.absorb_query(inp.q_nope.float().numpy(), inp.W_UK.float().numpy(), H, DC)
        q_rope = inp.q_rope.float().numpy()
        W_UV = inp.W_UV.float().numpy()
        mine = D.lpt_shard(lens, world)[rank]
        # this rank's sequences only, each over its own rows (no collective on the data path)
        out = O.varlen_decode(kv, [lens[i] for i in mine], [inp.kv_offsets[i] for i in mine],
                              q_abs[mine], q_rope[mine], W_UV, H, DC, DN, DR, DV) if mine else None
        got = [None] * world
        dist.all_gather_object(got, (mine, out))                 # test-side reassembly only
        full = np.empty((len(lens), H, DV))
        seen = []
        for idx, o in got:
            if idx:
                full[idx] = o
                seen += idx
        assert sorted(seen) == list(range(len(lens)))
        want = O.varlen_decode(kv, lens, inp.kv_offsets, q_abs, q_rope, W_UV, H, DC, DN, DR, DV)
        np.testing.assert_array_equal(full, want)
    finally:
        dist.destroy_process_group()


def test_batch_shards_reassemble_to_the_single_device_decode():
    _spawn(_batch_worker, 2, [300, 17, 129, 64, 1, 250], 11)


def _kv_range_sliced_worker(rank, world, port, L, B, seed):
    """Head-sliced exchange: packed partials (mla_decode_partial_packed's layout), one all-to-all,
    a per-rank merge + W_UV of its heads (the oracle stands in for mla_combine_partials_packed),
    and the output all-gather give the single-device decode on every rank."""
    _init(rank, world, port)
    try:
        inp = synthetic.baseline_inputs(num_heads=H, seq_lens=[L] * B, seed=seed)
        kv = inp.kv_cache.float().numpy()
        q_abs = O.absorb_query(inp.q_nope.float().numpy(), inp.W_UK.float().numpy(), H, DC)
        q_rope = inp.q_rope.float().numpy()
        W_UV = inp.W_UV.float().numpy()
        cos, sin = O.rope_tables(L, DR)
        lo, hi = D.kv_range(L, world, rank)
        hs = H // world
        R = DC + 4
        send = np.zeros((world * B * hs, R), dtype=np.float32)
        for b in range(B):
            rows = kv[b * L + lo:b * L + hi]
            m, l, o = O.split_partials(rows, q_abs[b], q_rope[b], cos[lo:hi], sin[lo:hi], DC, SCALE, [0, hi - lo])
            for h in range(H):
                r = D.packed_row(b, h, B, H, world)
                send[r, 0], send[r, 1] = m[0, h], l[0, h]
                send[r, 4:] = o[0, h]
        recv = D.exchange_head_slices(torch.from_numpy(send).view(world, B, hs, R))
        assert recv.shape == (world, B, hs, R)
        # this rank's heads: merge the partials every rank sent, project through its W_UV slice
        o_slice = np.zeros((B, hs, DV), dtype=np.float32)
        for b in range(B):
            p = recv[:, b].double().numpy()                                     # (world, hs, R)
            olat = O.combine_partials(p[:, :, 0], p[:, :, 1], p[:, :, 4:])      # (hs, dc)
            Ws = W_UV[rank * hs * DV:(rank + 1) * hs * DV]
            o_slice[b] = O.project_wuv(olat, Ws, hs, DV)
        out = D.gather_head_slices(torch.from_numpy(o_slice))
        assert out.shape == (B, H, DV)
        for b in range(B):
            want = O.absorbed_decode(kv[b * L:(b + 1) * L], q_abs[b], q_rope[b], W_UV, cos, sin, H, DC, DN, DR, DV)
            np.testing.assert_allclose(out[b].numpy(), want, rtol=2e-5, atol=2e-6)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,B", [(2, 1), (4, 2)])
def test_kv_range_head_sliced_exchange_matches_single_device(world, B):
    _spawn(_kv_range_sliced_worker, world, 257, B, 13)


def test_packed_row_layout():
    B, Hh, S = 3, 16, 4
    rows = sorted(D.packed_row(b, h, B, Hh, S) for b in range(B) for h in range(Hh))
    assert rows == list(range(B * Hh))
    # slice q is one contiguous block of B * H / S rows
    for q in range(S):
        block = [D.packed_row(b, h, B, Hh, S) for b in range(B) for h in range(q * Hh // S, (q + 1) * Hh // S)]
        assert min(block) == q * B * Hh // S and max(block) == (q + 1) * B * Hh // S - 1
