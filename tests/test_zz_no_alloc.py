"""mla_launch_fused_noalloc: the allocation-free variant of mla_launch_fused.

It exists for callers that may not allocate device memory (hosts that own every
allocation, latency-critical loops that must not touch an allocator); it keeps
its scratch in a fixed device array inside the library. These tests call it
through the C ABI on raw device pointers and compare it with mla_launch_fused,
which takes its scratch from the stream-ordered memory pool, on two calls in a
row (the shared array keeps the previous call's contents), against a golden
output of the reference directly, at a problem size just inside the array
(one split-KV worker), and check that a problem too large for the array is
rejected on the host.

This file is named to be collected last, so a stop-at-first-failure run has
already run every other test when it gets here.
"""

import ctypes as C

import numpy as np
import pytest
import torch

from oracle import mla_oracle as O
from latent_attn import _lib, synthetic

pytestmark = pytest.mark.gpu

# the tolerance used by the other GPU parity tests
MAX_ABS, MAX_REL, MIN_COS = 1e-2, 2e-2, 0.998


def _close(a, b, what):
    c = O.compare(a, b)
    assert c["finite"] and c["max_abs"] <= MAX_ABS and c["max_rel"] <= MAX_REL and c["cosine"] > MIN_COS, (what, c)


def _launch(fn, cfg, kv, S, qa, qr, wuv, cos, sin, out):
    p = _lib.MlaFusedParams(kv.data_ptr(), S, qa.data_ptr(), qr.data_ptr(), wuv.data_ptr(), cos.data_ptr(),
                            sin.data_ptr(), out.data_ptr(), C.pointer(cfg))
    return fn(C.byref(p), _lib.DTYPE_BF16, C.c_void_p(torch.cuda.current_stream().cuda_stream))


def _inputs(S, seed):
    dev = torch.device("cuda")
    inp = synthetic.baseline_inputs(num_heads=128, seq_lens=[S], seed=seed)
    cos, sin = synthetic.build_rope_tables(S, 64, device=dev)
    return (inp.kv_cache.to(dev), inp.q_absorbed()[0].to(dev).contiguous(),
            inp.q_rope[0].float().to(dev).contiguous(), inp.W_UV.to(dev), cos, sin)


def test_noalloc_matches_pool_launcher_on_consecutive_calls():
    lib = _lib.load()
    cfg = _lib.MlaConfig(5120, 512, 128, 64, 128, 128)
    # two calls in a row with different inputs and lengths: the second must not see the first's scratch
    for S, seed in ((8192, 1), (3001, 2)):
        kv, qa, qr, wuv, cos, sin = _inputs(S, seed)
        want = torch.full((128, 128), float("nan"), device="cuda")
        got = torch.full((128, 128), float("nan"), device="cuda")
        assert _launch(lib.mla_launch_fused, cfg, kv, S, qa, qr, wuv, cos, sin, want) == _lib.MLA_OK, \
            lib.mla_last_error()
        st = _launch(lib.mla_launch_fused_noalloc, cfg, kv, S, qa, qr, wuv, cos, sin, got)
        assert st == _lib.MLA_OK, lib.mla_last_error()
        torch.cuda.synchronize()
        _close(got.cpu().numpy(), want.cpu().numpy(), f"noalloc vs pool launcher, S={S}")


def test_noalloc_matches_golden_directly():
    """The allocation-free call against the reference's own output for one golden case
    (fp16 inputs of the reference pytest recipe, H=128, S=2048), not only against the pool
    launcher."""
    from golden_cases import load_case
    lib = _lib.load()
    meta, inp, want = load_case("reftest_h128_s2048")
    dev = torch.device("cuda")
    S = inp.seq_lens[0]
    kv, wuv = inp.kv_cache.to(dev), inp.W_UV.to(dev)
    cos, sin = synthetic.build_rope_tables(S, 64, device=dev)
    qa = inp.q_absorbed()[0].to(dev).contiguous()
    qr = inp.q_rope[0].float().to(dev).contiguous()
    cfg = _lib.MlaConfig(5120, 512, 128, 64, 128, 128)
    out = torch.full((128, 128), float("nan"), device=dev)
    p = _lib.MlaFusedParams(kv.data_ptr(), S, qa.data_ptr(), qr.data_ptr(), wuv.data_ptr(), cos.data_ptr(),
                            sin.data_ptr(), out.data_ptr(), C.pointer(cfg))
    st = lib.mla_launch_fused_noalloc(C.byref(p), _lib.DTYPE_F16, C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == _lib.MLA_OK, lib.mla_last_error()
    torch.cuda.synchronize()
    _close(out.cpu().numpy(), want[0], "noalloc vs golden reftest_h128_s2048")


def test_noalloc_near_its_scratch_limit():
    """3840 heads (30 query groups) fit the static array only with a single split-KV worker
    (query pack 4,423,680 bytes + 30 records of 132,096 bytes + status and prefix, 8,387,072 of
    8,388,608 bytes): the call runs with the reduced worker count and matches the pool launcher,
    which splits the same problem over many workers."""
    lib = _lib.load()
    H, S = 3840, 300
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(17)
    kv = torch.randn(S, 576, generator=g).to(torch.bfloat16).to(dev)
    qa = torch.randn(H, 512, generator=g).to(dev)
    qr = torch.randn(H, 64, generator=g).to(dev)
    wuv = (torch.randn(H * 128, 512, generator=g) / 512 ** 0.5).to(torch.bfloat16).to(dev)
    cos, sin = synthetic.build_rope_tables(S, 64, device=dev)
    cfg = _lib.MlaConfig(0, 512, 128, 64, H, 128)
    want = torch.full((H, 128), float("nan"), device=dev)
    got = torch.full((H, 128), float("nan"), device=dev)
    assert _launch(lib.mla_launch_fused, cfg, kv, S, qa, qr, wuv, cos, sin, want) == _lib.MLA_OK, \
        lib.mla_last_error()
    st = _launch(lib.mla_launch_fused_noalloc, cfg, kv, S, qa, qr, wuv, cos, sin, got)
    assert st == _lib.MLA_OK, lib.mla_last_error()
    torch.cuda.synchronize()
    _close(got.cpu().numpy(), want.cpu().numpy(), "noalloc vs pool launcher, H=3840")


def test_noalloc_rejects_problems_beyond_its_scratch():
    """3968 heads need 31 query groups, one more than the largest accepted problem (3840 heads,
    test_noalloc_near_its_scratch_limit): with one split-KV worker the plan needs 8,666,624 bytes of the
    8,388,608. The call is refused on the host before any launch. Every buffer still has the size the
    problem needs, so that a launch, were the call ever accepted, would stay inside them."""
    lib = _lib.load()
    H, S = 3968, 16
    dev = torch.device("cuda")
    cfg = _lib.MlaConfig(0, 512, 128, 64, H, 128)
    kv = torch.zeros(S, 576, dtype=torch.bfloat16, device=dev)
    qa = torch.zeros(H, 512, dtype=torch.float32, device=dev)
    qr = torch.zeros(H, 64, dtype=torch.float32, device=dev)
    wuv = torch.zeros(H * 128, 512, dtype=torch.bfloat16, device=dev)
    cos, sin = synthetic.build_rope_tables(S, 64, device=dev)
    out = torch.zeros(H, 128, dtype=torch.float32, device=dev)
    p = _lib.MlaFusedParams(kv.data_ptr(), S, qa.data_ptr(), qr.data_ptr(), wuv.data_ptr(), cos.data_ptr(),
                            sin.data_ptr(), out.data_ptr(), C.pointer(cfg))
    st = lib.mla_launch_fused_noalloc(C.byref(p), _lib.DTYPE_BF16, C.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert st == _lib.MLA_ERR_UNSUPPORTED
    msg = lib.mla_last_error().decode()
    assert "scratch" in msg and str(_lib.NOALLOC_SCRATCH_BYTES) in msg, msg
