"""The library against the reference's OWN fused CUDA kernels (src/fused_mla.cu,
src/fused_mla_batched.cu of anishesg/latent-attn), compiled from source for
sm_100a into oracle/_ref/ by oracle/build_ref.py, on identical fp16 inputs
(the reference is fp16-only). Skipped when that library was not built."""

import ctypes as C
import os

import numpy as np
import pytest
import torch

from golden_cases import load_case
from oracle import mla_oracle as O
from latent_attn import MLAConfig, synthetic
from latent_attn.functional import batched_fused_mla, fused_mla

pytestmark = pytest.mark.gpu

REF_LIB = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref",
                       "libref_mla.so")


def ref_lib():
    if not os.path.exists(REF_LIB):
        pytest.skip("oracle/_ref/libref_mla.so not built (needs the reference sources at build time)")
    lib = C.CDLL(REF_LIB)
    for name in ("ref_fused_mla", "ref_batched_fused_mla"):
        getattr(lib, name).restype = C.c_int
    return lib


def _close(a, b, what):
    c = O.compare(a, b)
    assert c["finite"] and c["max_abs"] <= 1e-2 and c["max_rel"] <= 2e-2 and c["cosine"] > 0.998, (what, c)
    return c


@pytest.mark.parametrize("name", ["reftest_h128_s512", "reftest_h128_s2048", "reftest_h16_s512",
                                  "reftest_h64_s2048"])
def test_fused_matches_reference_kernel(name):
    lib = ref_lib()
    meta, inp, golden = load_case(name)
    cfg = MLAConfig(5120, 512, 128, 64, meta["num_heads"], 128)
    dev = torch.device("cuda")
    S = inp.seq_lens[0]
    kv = inp.kv_cache.to(dev)
    W_UV = inp.W_UV.to(dev)
    cos, sin = synthetic.build_rope_tables(S, 64, device=dev)
    qa = inp.q_absorbed()[0].to(dev).contiguous()
    qr = inp.q_rope[0].float().to(dev).contiguous()
    ref_out = torch.full((cfg.num_heads, 128), float("nan"), device=dev)
    st = lib.ref_fused_mla(C.c_void_p(kv.data_ptr()), S, C.c_void_p(qa.data_ptr()), C.c_void_p(qr.data_ptr()),
                           C.c_void_p(W_UV.data_ptr()), C.c_void_p(cos.data_ptr()), C.c_void_p(sin.data_ptr()),
                           C.c_void_p(ref_out.data_ptr()), 5120, 512, 128, 64, cfg.num_heads, 128,
                           C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0
    ours = fused_mla(kv, qa, qr, W_UV, cos, sin, cfg)
    torch.cuda.synchronize()
    r, o = ref_out.cpu().numpy(), ours.cpu().numpy()
    _close(r, golden[0], name + ": reference kernel vs golden")  # the reference kernel itself is right
    _close(o, r, name + ": library vs reference kernel")


def test_batched_matches_reference_batched_kernel():
    lib = ref_lib()
    meta, inp, golden = load_case("batched_h128_s1024_b4")
    cfg = MLAConfig.deepseek_v2()
    dev = torch.device("cuda")
    S, B = inp.seq_lens[0], inp.batch
    kv = inp.kv_cache.to(dev)
    W_UV = inp.W_UV.to(dev)
    cos, sin = synthetic.build_rope_tables(S, 64, device=dev)
    qa = inp.q_absorbed().to(dev).contiguous()
    qr = inp.q_rope.float().to(dev).contiguous()
    ref_out = torch.full((B, 128, 128), float("nan"), device=dev)
    st = lib.ref_batched_fused_mla(C.c_void_p(kv.data_ptr()), S, B, C.c_void_p(qa.data_ptr()),
                                   C.c_void_p(qr.data_ptr()), C.c_void_p(W_UV.data_ptr()),
                                   C.c_void_p(cos.data_ptr()), C.c_void_p(sin.data_ptr()),
                                   C.c_void_p(ref_out.data_ptr()), 5120, 512, 128, 64, 128, 128,
                                   C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0
    ours = batched_fused_mla(kv, qa, qr, W_UV, cos, sin, cfg)
    torch.cuda.synchronize()
    _close(ref_out.cpu().numpy(), golden, "reference batched kernel vs golden")
    _close(ours.cpu().numpy(), ref_out.cpu().numpy(), "library vs reference batched kernel")
