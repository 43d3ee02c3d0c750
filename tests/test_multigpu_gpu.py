"""KV-range decode through latent_attn.distributed on CUDA with NCCL.

A one-rank process group checks the glue (partial -> all-gather -> merge) on any
GPU box; the two-rank case runs when the box has two GPUs, one process per GPU,
and compares every rank's output with the fp64 oracle of the whole sequence.
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
from latent_attn.distributed import KVRangeDecoder, kv_range

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


def _decode_rank(rank, world, L, seed):
    dev = torch.device("cuda", rank)
    inp = synthetic.baseline_inputs(num_heads=128, seq_lens=[L], seed=seed)
    lo, hi = kv_range(L, world, rank)
    cos, sin = synthetic.build_rope_tables(L, 64, device=dev)
    dec = KVRangeDecoder(MLAConfig.deepseek_v2())
    outs = []
    for _ in range(2):                        # the second call reuses the gather buffers
        out = dec(inp.kv_cache[lo:hi].contiguous().to(dev), inp.q_rope.float().to(dev), inp.W_UV.to(dev), cos,
                  sin, pos_offset=lo, q_nope=inp.q_nope.float().to(dev), W_UK=inp.W_UK.to(dev))
        outs.append(out.cpu().numpy()[0])
    return inp, outs


def test_kv_range_decoder_single_rank():
    L = 5000
    dist.init_process_group("nccl", rank=0, world_size=1, store=dist.HashStore(),
                            device_id=torch.device("cuda", 0))
    try:
        inp, outs = _decode_rank(0, 1, L, 3)
    finally:
        dist.destroy_process_group()
    ref = _oracle(inp, L)
    for o in outs:
        _close(o, ref, "one rank")
    np.testing.assert_array_equal(outs[0], outs[1])


def _two_rank_worker(rank, world, port, L, seed, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    from datetime import timedelta
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        _, outs = _decode_rank(rank, world, L, seed)
        q.put((rank, outs[-1]))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_kv_range_decoder_two_ranks():
    L, seed = 20011, 4                          # odd length: ranks hold 10005 and 10006 rows
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = mp.start_processes(_two_rank_worker, args=(2, port, L, seed, q), nprocs=2, join=False,
                               start_method="spawn")
    got = {}
    try:
        for _ in range(2):                       # read before joining: a full pipe would block the writers
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
    inp = synthetic.baseline_inputs(num_heads=128, seq_lens=[L], seed=seed)
    ref = _oracle(inp, L)
    for r in range(2):
        _close(got[r], ref, f"rank {r}")
    np.testing.assert_array_equal(got[0], got[1])
