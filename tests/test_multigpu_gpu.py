"""KV-range decode through latent_attn.distributed on CUDA: the NCCL exchange and the library's
peer-memory exchange (put / wait kernels over CUDA IPC mappings).

The put / wait kernels are checked on one GPU (every "rank" a local buffer, the puts stream-
ordered before the waits, so nothing waits on a kernel that runs beside it), including a wait that
runs out because nothing sets its flag. A one-rank process group checks the decode glue on any GPU
box; the two-rank cases run when the box has two GPUs, one process per GPU, and compare every
rank's output with the fp64 oracle of the whole sequence and the two exchanges with each other,
eagerly and replayed from a CUDA graph: bit-identical for the head-sliced form (the same export and
merge kernels), within 1e-6 for the one-kernel exchange of batches up to 4 (its own merge); every
rank's output, and every call's, bit-identical.

The one-kernel exchange (mla_decode_kv_range) waits on peers inside the kernel, so it runs only with
one rank per GPU (or a single rank), never with emulated ranks on one GPU.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import mla_oracle as O
from latent_attn import MLAConfig, synthetic
from latent_attn.distributed import GATHER_MAX_BATCH, KVRangeDecoder, kv_range

pytestmark = pytest.mark.gpu

MAX_ABS, MAX_REL, MIN_COS = 1e-2, 2e-2, 0.998


def _close(got, ref, what):
    c = O.compare(got, ref)
    assert c["finite"] and c["max_abs"] <= MAX_ABS and c["max_rel"] <= MAX_REL and c["cosine"] > MIN_COS, (what, c)


def _oracle(inp, L):
    cos, sin = O.rope_tables(L, 64)
    q_abs = O.absorb_query(inp.q_nope[0].float().numpy(), inp.W_UK.float().numpy(), 128, 512)
    return O.absorbed_decode(inp.kv_cache.float().numpy(), q_abs, inp.q_rope[0].float().numpy(),
                             inp.W_UV.float().numpy(), cos, sin, 128, 512, 128, 64, 128)


def _oracle_batch(inp, L, B):
    cos, sin = O.rope_tables(L, 64)
    outs = []
    for b in range(B):
        q_abs = O.absorb_query(inp.q_nope[b].float().numpy(), inp.W_UK.float().numpy(), 128, 512)
        kv = inp.kv_cache[b * L:(b + 1) * L].float().numpy()
        outs.append(O.absorbed_decode(kv, q_abs, inp.q_rope[b].float().numpy(), inp.W_UV.float().numpy(), cos, sin,
                                      128, 512, 128, 64, 128))
    return np.stack(outs)


def _decode_rank(rank, world, L, seed, exchange="nccl", B=1, graph=False):
    """Two eager calls (the second reuses the exchange buffers) and, with ``graph``, two replays
    of a captured call; returns the inputs and every call's (B, H, dv) output."""
    dev = torch.device("cuda", rank)
    inp = synthetic.baseline_inputs(num_heads=128, seq_lens=[L] * B, seed=seed)
    lo, hi = kv_range(L, world, rank)
    cos, sin = synthetic.build_rope_tables(L, 64, device=dev)
    dec = KVRangeDecoder(MLAConfig.deepseek_v2(), exchange=exchange)
    kv = torch.cat([inp.kv_cache[b * L + lo:b * L + hi] for b in range(B)]).contiguous().to(dev)
    args = (kv, inp.q_rope.float().to(dev), inp.W_UV.to(dev), cos, sin)
    kw = dict(pos_offset=lo, q_nope=inp.q_nope.float().to(dev), W_UK=inp.W_UK.to(dev))
    outs = []
    for _ in range(2):
        outs.append(dec(*args, **kw).cpu().numpy())
    if graph:
        g = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(dev)
        with torch.cuda.graph(g, stream=side):
            o = dec(*args, **kw)
        for _ in range(2):
            g.replay()
            torch.cuda.synchronize(dev)
            outs.append(o.cpu().numpy())
        g.reset()
        del g
    dec.check()
    dec.close()
    return inp, outs


@pytest.mark.parametrize("exchange", ["nccl", "p2p"])
def test_kv_range_decoder_single_rank(exchange):
    L = 5000
    dist.init_process_group("nccl", rank=0, world_size=1, store=dist.HashStore(),
                            device_id=torch.device("cuda", 0))
    try:
        inp, outs = _decode_rank(0, 1, L, 3, exchange, graph=exchange == "p2p")
    finally:
        dist.destroy_process_group()
    ref = _oracle(inp, L)
    for o in outs:
        _close(o[0], ref, "one rank")
        np.testing.assert_array_equal(outs[0], o)


def _ptrs(values):
    return torch.tensor(values, dtype=torch.int64, device="cuda")


def _signals(flag_ptrs, world, r, epoch, counters):
    from latent_attn import _C
    return (_C.PeerSignal(flag_ptrs, r, epoch, counters[:world]),
            _C.PeerSignal(flag_ptrs, world + r, epoch, counters[world:]))


def test_peer_put_all_to_all_and_row_gather_on_one_gpu():
    """Two emulated ranks on one GPU: an all-to-all of 4144-byte slices (rows = 1, three blocks
    each) and a row-wise all-gather (rows = 5, destination pitch of the full row); every byte
    checked, the flags at the step count, the block counters back at zero, and the step counter
    advanced once per step by the ending wait."""
    from latent_attn import _C
    world, nblk = 2, 3
    slice_bytes, rows, row_bytes = 4096 + 48, 5, 192
    full_pitch = world * row_bytes
    bufs = [_C.IpcBuffer(1 << 16, torch.device("cuda", 0)) for _ in range(world)]
    try:
        flags = [b.view(torch.int32, 2 * world) for b in bufs]
        recv_off, out_off = 1024, 1024 + world * slice_bytes
        flag_ptrs = _ptrs([b.ptr for b in bufs])
        recv_ptrs, out_ptrs = flag_ptrs + recv_off, flag_ptrs + out_off
        epochs = [torch.zeros(1, dtype=torch.int32, device="cuda") for _ in range(world)]
        counters = [torch.zeros(2 * world, dtype=torch.int32, device="cuda") for _ in range(world)]
        sigs = [_signals(flag_ptrs, world, r, epochs[r], counters[r]) for r in range(world)]
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        g = torch.Generator().manual_seed(9)
        send = [torch.randint(0, 256, (world * slice_bytes,), generator=g, dtype=torch.uint8).cuda()
                for _ in range(world)]
        rowsrc = [torch.randint(0, 256, (rows * row_bytes,), generator=g, dtype=torch.uint8).cuda()
                  for _ in range(world)]
        for step in range(2):
            for r in range(world):
                _C.peer_put(send[r], 1, slice_bytes, 0, slice_bytes, recv_ptrs, 0, r * slice_bytes, nblk, sigs[r][0])
            for r in range(world):
                _C.peer_wait(flags[r][:world], epochs[r], False, status)
            for r in range(world):
                _C.peer_put(rowsrc[r], rows, row_bytes, row_bytes, 0, out_ptrs, full_pitch, r * row_bytes, nblk,
                            sigs[r][1])
            for r in range(world):
                _C.peer_wait(flags[r][world:], epochs[r], True, status)
            torch.cuda.synchronize()
            assert int(status.item()) == 0
            for r in range(world):
                assert int(epochs[r].item()) == step + 1
                assert torch.all(flags[r] == step + 1)
                assert torch.all(counters[r] == 0)
                recv = bufs[r].view(torch.uint8, world * slice_bytes, recv_off).view(world, slice_bytes)
                for p in range(world):   # block p of rank r's receive area = rank p's slice r
                    assert torch.equal(recv[p], send[p].view(world, slice_bytes)[r])
                out = bufs[r].view(torch.uint8, rows * full_pitch, out_off).view(rows, world, row_bytes)
                for p in range(world):
                    assert torch.equal(out[:, p], rowsrc[p].view(rows, row_bytes))
            send = [s.roll(1) for s in send]
    finally:
        for b in bufs:
            b.free()


@pytest.mark.parametrize("B", [1, 5])
def test_fused_exchange_kernels_two_emulated_ranks_on_one_gpu(B):
    """The kernels that store into other ranks' memory, with two emulated ranks on one GPU (every
    call stream-ordered): the partial export (mla_decode_partial_put; B = 1 the GEMV merge, B = 5
    the CUDA-core combine) must fill receiver q's block p with exactly what
    mla_decode_partial_packed gives rank p for slice q, and the merge + projection
    (mla_combine_partials_put; B = 1 stored by the GEMV kernel, B = 5 staged and put) must give
    every receiver the same full output, bit-identical to mla_combine_partials_packed and within
    the decode tolerance of the oracle."""
    from latent_attn import _C
    world, L, H, dc, dv = 2, 3001, 128, 512, 128
    hs = H // world
    cfg = MLAConfig.deepseek_v2()
    dims = (cfg.d_model, 512, 128, 64, 128, 128)
    dev = torch.device("cuda", 0)
    inp = synthetic.baseline_inputs(num_heads=H, seq_lens=[L] * B, seed=11)
    cos, sin = synthetic.build_rope_tables(L, 64, device=dev)
    W_UV = inp.W_UV.to(dev)
    qn, qr, WK = inp.q_nope.float().to(dev), inp.q_rope.float().to(dev), inp.W_UK.to(dev)
    shards = []
    for r in range(world):
        lo, hi = kv_range(L, world, r)
        shards.append((lo, torch.cat([inp.kv_cache[b * L + lo:b * L + hi] for b in range(B)]).contiguous().to(dev)))
    sends = [_C.mla_decode_partial_packed(kv, qr, W_UV, cos, sin, *dims, num_slices=world, q_nope=qn, W_UK=WK,
                                          kv_pos_offset=lo) for lo, kv in shards]
    slice_bytes = B * hs * (dc + 4) * 4
    out_bytes = B * H * dv * 4
    recv_off = 256
    out_off = recv_off + world * slice_bytes
    bufs = [_C.IpcBuffer(out_off + out_bytes, dev) for _ in range(world)]
    try:
        flag_ptrs = _ptrs([b.ptr for b in bufs])
        epochs = [torch.zeros(1, dtype=torch.int32, device=dev) for _ in range(world)]
        counters = [torch.zeros(2 * world, dtype=torch.int32, device=dev) for _ in range(world)]
        sigs = [_signals(flag_ptrs, world, r, epochs[r], counters[r]) for r in range(world)]
        flags = [b.view(torch.int32, 2 * world) for b in bufs]
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        for r, (lo, kv) in enumerate(shards):
            _C.mla_decode_partial_put(kv, qr, W_UV, cos, sin, *dims, dst_ptrs=flag_ptrs + recv_off,
                                      dst_offset=r * slice_bytes, signal=sigs[r][0], q_nope=qn, W_UK=WK,
                                      kv_pos_offset=lo)
        for q in range(world):
            _C.peer_wait(flags[q][:world], epochs[q], False, status)
        recvs = [bufs[q].view(torch.float32, world * slice_bytes // 4, recv_off).view(world, B, hs, dc + 4)
                 for q in range(world)]
        for q in range(world):
            for p in range(world):
                assert torch.equal(recvs[q][p], sends[p][q]), (q, p)
        scratch = torch.empty(B, hs, dv, device=dev)
        want = []
        for r in range(world):
            W_slice = W_UV[r * hs * dv:(r + 1) * hs * dv]
            want.append(_C.mla_combine_partials_packed(recvs[r].clone(), W_slice, *dims))
            _C.mla_combine_partials_put(recvs[r], W_slice, *dims, dst_ptrs=flag_ptrs + out_off,
                                        dst_offset=r * hs * dv * 4, dst_pitch=H * dv * 4, signal=sigs[r][1],
                                        scratch=scratch)
        for q in range(world):
            _C.peer_wait(flags[q][world:], epochs[q], True, status)
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        full = torch.cat(want, dim=1)
        for q in range(world):
            assert int(epochs[q].item()) == 1 and torch.all(flags[q] == 1) and torch.all(counters[q] == 0)
            got = bufs[q].view(torch.float32, out_bytes // 4, out_off).view(B, H, dv)
            assert torch.equal(got, full), q
        ref = _oracle_batch(inp, L, B)
        _close(full.cpu().numpy(), ref, f"fused exchange B={B}")
    finally:
        for b in bufs:
            b.free()


@pytest.mark.parametrize("world,B", [(2, 1), (2, 3), (8, 1)])
def test_gathered_exchange_emulated_ranks_on_one_gpu(world, B):
    """The gathered exchange (batch <= 4) with 2 or 8 emulated ranks on one GPU, three steps: the export
    (mla_decode_partial_gather) must put exactly the rows mla_decode_partial_packed gives (one
    slice) into block r of every receiver, in the half of the receive area the step's flag value
    selects (the other half, zeroed before the step, stays zero); the merge of all heads
    (mla_combine_partials_gathered) reads that half and must be bit-identical on both receivers and
    to mla_combine_partials_packed over the same sets, and within the decode tolerance of the
    oracle."""
    from latent_attn import _C
    L, H, dc, dv = 2501, 128, 512, 128
    cfg = MLAConfig.deepseek_v2()
    dims = (cfg.d_model, 512, 128, 64, 128, 128)
    dev = torch.device("cuda", 0)
    inp = synthetic.baseline_inputs(num_heads=H, seq_lens=[L] * B, seed=13)
    W_UV = inp.W_UV.to(dev)
    qn, qr, WK = inp.q_nope.float().to(dev), inp.q_rope.float().to(dev), inp.W_UK.to(dev)
    shards = []
    for r in range(world):
        lo, hi = kv_range(L, world, r)
        shards.append((lo, torch.cat([inp.kv_cache[b * L + lo:b * L + hi] for b in range(B)]).contiguous().to(dev)))
    # on-the-fly RoPE (no tables), as the benchmark runs it
    sets = torch.cat([_C.mla_decode_partial_packed(kv, qr, W_UV, None, None, *dims, num_slices=1, q_nope=qn, W_UK=WK,
                                                   kv_pos_offset=lo) for lo, kv in shards])   # (world, B, H, dc + 4)
    want = _C.mla_combine_partials_packed(sets, W_UV, *dims)
    set_bytes = B * H * (dc + 4) * 4
    parity = world * set_bytes
    recv_off = 256
    bufs = [_C.IpcBuffer(recv_off + 2 * parity, dev) for _ in range(world)]
    try:
        flag_ptrs = _ptrs([b.ptr for b in bufs])
        epochs = [torch.zeros(1, dtype=torch.int32, device=dev) for _ in range(world)]
        counters = [torch.zeros(2 * world, dtype=torch.int32, device=dev) for _ in range(world)]
        sigs = [_signals(flag_ptrs, world, r, epochs[r], counters[r]) for r in range(world)]
        flags = [b.view(torch.int32, 2 * world) for b in bufs]
        recvs = [b.view(torch.float32, 2 * parity // 4, recv_off) for b in bufs]
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        for step in range(3):
            for q in range(world):
                recvs[q].zero_()
            for r, (lo, kv) in enumerate(shards):
                _C.mla_decode_partial_gather(kv, qr, W_UV, None, None, *dims, dst_ptrs=flag_ptrs + recv_off,
                                             dst_offset=r * set_bytes, parity_bytes=parity, signal=sigs[r][0],
                                             q_nope=qn, W_UK=WK, kv_pos_offset=lo)
            for q in range(world):
                _C.peer_wait(flags[q][:world], epochs[q], True, status)
            outs = [_C.mla_combine_partials_gathered(recvs[q], parity, epochs[q], W_UV, *dims, parts=world, batch=B)
                    for q in range(world)]
            torch.cuda.synchronize()
            assert int(status.item()) == 0
            half = (step + 1) & 1
            for q in range(world):
                assert int(epochs[q].item()) == step + 1 and torch.all(flags[q][:world] == step + 1)
                assert torch.all(counters[q] == 0)
                halves = recvs[q].view(2, world, B, H, dc + 4)
                assert torch.equal(halves[half], sets), (step, q)
                assert not torch.any(halves[1 - half] != 0), (step, q)
                assert torch.equal(outs[q], want), (step, q)
        cos, sin = O.rope_tables_otf(L, 64)
        ref = []
        for b in range(B):
            q_abs = O.absorb_query(inp.q_nope[b].float().numpy(), inp.W_UK.float().numpy(), 128, 512)
            ref.append(O.absorbed_decode(inp.kv_cache[b * L:(b + 1) * L].float().numpy(), q_abs,
                                         inp.q_rope[b].float().numpy(), inp.W_UV.float().numpy(), cos, sin,
                                         128, 512, 128, 64, 128))
        _close(want.cpu().numpy(), np.stack(ref), f"gathered exchange B={B}")
    finally:
        for b in bufs:
            b.free()


def test_peer_wait_gives_up_and_reports():
    """A flag that nothing sets: the wait ends after its bound (2 s), stores 1 to the status word,
    does not advance the counter, and the context stays usable."""
    from latent_attn import _C
    buf = _C.IpcBuffer(4096, torch.device("cuda", 0))
    try:
        flags = buf.view(torch.int32, 4)
        epoch = torch.zeros(1, dtype=torch.int32, device="cuda")
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        _C.peer_wait(flags, epoch, False, status)
        torch.cuda.synchronize()
        assert int(status.item()) == 1 and int(epoch.item()) == 0
        x = torch.arange(10, device="cuda")
        assert int(x.sum().item()) == 45
    finally:
        buf.free()


def _rank_worker(rank, world, port, L, seed, B, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    from datetime import timedelta
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        _, ref = _decode_rank(rank, world, L, seed, "nccl", B)
        _, outs = _decode_rank(rank, world, L, seed, "p2p", B, graph=True)
        for o in outs:
            if B > GATHER_MAX_BATCH:   # head-sliced: the same export and merge kernels as the NCCL path
                np.testing.assert_array_equal(o, ref[-1])
            else:                      # the one-kernel exchange: its own merge, equal to the last bits
                np.testing.assert_allclose(o, ref[-1], rtol=1e-5, atol=1e-6)
            np.testing.assert_array_equal(o, outs[0])   # eager calls and graph replays agree bit for bit
        q.put((rank, outs[-1]))
    finally:
        dist.destroy_process_group()


def _run_ranks(world, L, B, seed=4):
    """``world`` processes, one per GPU; returns every rank's output of the p2p decoder (each rank has
    checked it against the NCCL exchange)."""
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = mp.start_processes(_rank_worker, args=(world, port, L, seed, B, q), nprocs=world, join=False,
                               start_method="spawn")
    got = {}
    try:
        for _ in range(world):                   # read before joining: a full pipe would block the writers
            r, o = q.get(timeout=300)
            got[r] = o
    finally:
        import time
        deadline = time.monotonic() + 300
        while not procs.join(timeout=10):        # re-raises a rank's exception
            if time.monotonic() > deadline:
                for p in procs.processes:
                    p.kill()
                pytest.fail("ranks did not finish")
    return got


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("L,B", [(20011, 1), (3001, 3), (1501, 5)])
def test_kv_range_decoder_two_ranks(L, B):
    got = _run_ranks(2, L, B)                   # odd lengths: the ranks' row counts differ by one
    inp = synthetic.baseline_inputs(num_heads=128, seq_lens=[L] * B, seed=4)
    ref = _oracle_batch(inp, L, B)
    for r in range(2):
        _close(got[r], ref, f"rank {r}")
    np.testing.assert_array_equal(got[0], got[1])


@pytest.mark.skipif(torch.cuda.device_count() < 3, reason="needs three or more GPUs")
@pytest.mark.parametrize("L,B", [(40003, 1), (2003, 5)])
def test_kv_range_decoder_all_gpus(L, B):
    """Every GPU of the box a rank (the gathered exchange at B = 1, head-sliced at B = 5 when the
    ranks divide the heads, else the NCCL all-gather of whole partial sets)."""
    world = torch.cuda.device_count()
    got = _run_ranks(world, L, B)
    inp = synthetic.baseline_inputs(num_heads=128, seq_lens=[L] * B, seed=4)
    ref = _oracle_batch(inp, L, B)
    for r in range(world):
        _close(got[r], ref, f"rank {r} of {world}")
        np.testing.assert_array_equal(got[0], got[r])
