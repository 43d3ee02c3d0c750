"""GPU parity: the CUDA path against the reference's golden outputs and the CPU oracle.

Tolerance (bf16/fp16 I/O, fp32 accumulation; the bound stated for this path):
max-abs <= 1e-2, norm-relative max error (max|d| / max|ref|) <= 2e-2, and the
reference's own criterion cosine > 0.998 (tests/test_python.py:136-138).
"""

import math

import numpy as np
import pytest
import torch

from golden_cases import case_names, load_case
from oracle import mla_oracle as O
from latent_attn import MLAConfig, synthetic, _C, _lib
from latent_attn.functional import batched_fused_mla, fused_mla, mla_decode, naive_mla

pytestmark = pytest.mark.gpu

MAX_ABS = 1e-2
MAX_REL = 2e-2
MIN_COS = 0.998

TC = _lib.KERNEL_TENSOR_CORE
CC = _lib.KERNEL_CUDA_CORE


def assert_close(got, ref, what=""):
    c = O.compare(np.asarray(got, dtype=np.float64), np.asarray(ref, dtype=np.float64))
    assert c["finite"], (what, c)
    assert c["max_abs"] <= MAX_ABS and c["max_rel"] <= MAX_REL and c["cosine"] > MIN_COS, (what, c)
    return c


def cfg_of(meta):
    return MLAConfig(0, meta["kv_lora_rank"], meta["qk_nope_head_dim"], meta["qk_rope_head_dim"],
                     meta["num_heads"], meta["v_head_dim"])


def tc_available(cfg):
    return cfg.kv_lora_rank == 512 and cfg.qk_rope_head_dim == 64 and \
        torch.cuda.get_device_capability()[0] == 10


def kernels_for(cfg):
    return [CC, TC] if tc_available(cfg) else [CC]


@pytest.mark.parametrize("name", case_names())
def test_golden_through_ops(name):
    """Every golden case through the public torch-facing API, on every kernel that covers it."""
    meta, inp, want = load_case(name)
    cfg = cfg_of(meta)
    dev = torch.device("cuda")
    kv = inp.kv_cache.to(dev)
    W_UV = inp.W_UV.to(dev)
    W_UK = inp.W_UK.to(dev)
    q_rope = inp.q_rope.float().to(dev)
    q_nope = inp.q_nope.float().to(dev)
    Lmax = max(inp.seq_lens)
    cos, sin = synthetic.build_rope_tables(Lmax, cfg.qk_rope_head_dim, device=dev)
    for kern in kernels_for(cfg):
        if meta["shared_cache"]:
            q_abs = inp.q_absorbed().to(dev)
            got = _C.mla_decode(kv, q_rope, W_UV, cos, sin, cfg.d_model, cfg.kv_lora_rank,
                                cfg.qk_nope_head_dim, cfg.qk_rope_head_dim, cfg.num_heads, cfg.v_head_dim,
                                q_absorbed=q_abs, shared_cache=True, max_seq_len=Lmax, kernel=kern)
        else:
            lens = torch.tensor(inp.seq_lens, dtype=torch.int32, device=dev)
            offs = torch.tensor(inp.kv_offsets, dtype=torch.int64, device=dev)
            got = mla_decode(kv, q_rope, W_UV, cos, sin, cfg, q_nope=q_nope, W_UK=W_UK, seq_lens=lens,
                             kv_offsets=offs, max_seq_len=Lmax, kernel=kern)
        torch.cuda.synchronize()
        assert_close(got.cpu().numpy(), want, f"{name} kernel={kern}")


@pytest.mark.parametrize("name", ["reftest_h128_s512", "reftest_h128_s2048", "reftest_h16_s512",
                                  "reftest_h64_s2048", "batched_h128_s1024_b4"])
def test_reference_ops_drop_in(name):
    """fused_mla / batched_fused_mla / naive_mla with the reference's fp16 inputs
    (tests/test_python.py:72-138, tests/test_batched.py:33-88)."""
    meta, inp, want = load_case(name)
    cfg = cfg_of(meta)
    dev = torch.device("cuda")
    kv = inp.kv_cache.to(dev)
    W_UV = inp.W_UV.to(dev)
    S = inp.seq_lens[0]
    cos, sin = synthetic.build_rope_tables(S, cfg.qk_rope_head_dim, device=dev)
    q_abs = inp.q_absorbed().to(dev)
    q_rope = inp.q_rope.float().to(dev)
    if inp.batch == 1:
        out = fused_mla(kv, q_abs[0].contiguous(), q_rope[0].contiguous(), W_UV, cos, sin, cfg)
        assert out.shape == (cfg.num_heads, cfg.v_head_dim) and out.dtype == torch.float32
        assert_close(out.cpu().numpy(), want[0], name)
        nv = naive_mla(kv, inp.W_UK.to(dev), W_UV, inp.q_nope[0].float().to(dev).contiguous(),
                       q_rope[0].contiguous(), cos, sin, cfg)
        assert_close(nv.cpu().numpy(), want[0], name + " naive")
    else:
        out = batched_fused_mla(kv, q_abs, q_rope, W_UV, cos, sin, cfg)
        assert out.shape == (inp.batch, cfg.num_heads, cfg.v_head_dim)
        assert_close(out.cpu().numpy(), want, name)
        loop = torch.stack([fused_mla(kv, q_abs[i].contiguous(), q_rope[i].contiguous(), W_UV, cos, sin, cfg)
                            for i in range(inp.batch)])
        for i in range(inp.batch):  # tests/test_batched.py:82-86 criterion
            a, b = out[i].flatten().double(), loop[i].flatten().double()
            assert float(a @ b / (a.norm() * b.norm())) > 0.998


def test_c_abi_launch_fused_matches_golden():
    """The reference-shaped C entry point (launch_fused_mla's replacement) called with raw pointers."""
    import ctypes as C
    meta, inp, want = load_case("reftest_h128_s2048")
    cfg = cfg_of(meta)
    dev = torch.device("cuda")
    kv = inp.kv_cache.to(dev)
    W_UV = inp.W_UV.to(dev)
    S = inp.seq_lens[0]
    cos, sin = synthetic.build_rope_tables(S, 64, device=dev)
    q_abs = inp.q_absorbed()[0].to(dev).contiguous()
    q_rope = inp.q_rope[0].float().to(dev).contiguous()
    out = torch.full((128, 128), float("nan"), device=dev)
    lib = _lib.load()
    c = _lib.MlaConfig(5120, 512, 128, 64, 128, 128)
    p = _lib.MlaFusedParams(kv.data_ptr(), S, q_abs.data_ptr(), q_rope.data_ptr(), W_UV.data_ptr(),
                            cos.data_ptr(), sin.data_ptr(), out.data_ptr(), C.pointer(c))
    st = lib.mla_launch_fused(C.byref(p), _lib.DTYPE_F16, C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0, lib.mla_last_error()
    torch.cuda.synchronize()
    assert_close(out.cpu().numpy(), want[0], "mla_launch_fused")
    # batched entry point, B=2 tokens sharing the cache
    q2 = torch.stack([q_abs, q_abs * 0.5]).contiguous()
    r2 = torch.stack([q_rope, q_rope]).contiguous()
    out2 = torch.full((2, 128, 128), float("nan"), device=dev)
    pb = _lib.MlaBatchedFusedParams(kv.data_ptr(), S, 2, q2.data_ptr(), r2.data_ptr(), W_UV.data_ptr(),
                                    cos.data_ptr(), sin.data_ptr(), out2.data_ptr(), C.pointer(c))
    st = lib.mla_launch_batched_fused(C.byref(pb), _lib.DTYPE_F16,
                                      C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0, lib.mla_last_error()
    torch.cuda.synchronize()
    assert_close(out2[0].cpu().numpy(), want[0], "batched token 0")


def _oracle_single(inp, b, cos_np, sin_np, H=128, dc=512, dn=128, dR=64, dv=128):
    L, off = inp.seq_lens[b], inp.kv_offsets[b]
    kv = inp.kv_cache[off:off + L].float().numpy()
    q_abs = O.absorb_query(inp.q_nope[b].float().numpy(), inp.W_UK.float().numpy(), H, dc)
    return O.absorbed_decode(kv, q_abs, inp.q_rope[b].float().numpy(), inp.W_UV.float().numpy(),
                             cos_np[:L], sin_np[:L], H, dc, dn, dR, dv)


@pytest.mark.parametrize("L", [8192, 131072])
def test_full_size_single_sequence_vs_oracle(L):
    """BASELINE configs 1 and 3 (B=1, H=128, L=8192 / 131072, bf16) against the fp64 oracle."""
    inp = synthetic.baseline_inputs(num_heads=128, seq_lens=[L], seed=0)
    cfg = MLAConfig.deepseek_v2()
    dev = torch.device("cuda")
    cos, sin = synthetic.build_rope_tables(L, 64, device=dev)
    got = {}
    for kern in kernels_for(cfg):
        out = mla_decode(inp.kv_cache.to(dev), inp.q_rope.float().to(dev), inp.W_UV.to(dev), cos, sin, cfg,
                         q_nope=inp.q_nope.float().to(dev), W_UK=inp.W_UK.to(dev), kernel=kern)
        got[kern] = out.cpu().numpy()[0]
    ref = _oracle_single(inp, 0, cos.cpu().numpy(), sin.cpu().numpy())
    for kern, g in got.items():
        assert_close(g, ref, f"L={L} kernel={kern}")


def test_varlen_batch_config2_sample():
    """BASELINE config 2 shape (B=64, L_b ~ U[1024, 16384]): 6 sequences checked against the oracle,
    and the whole batch against per-sequence single decodes (batching must not change results)."""
    lens = synthetic.varlen_lengths(64, 1024, 16384, seed=0)
    inp = synthetic.baseline_inputs(num_heads=128, seq_lens=lens, seed=0)
    cfg = MLAConfig.deepseek_v2()
    dev = torch.device("cuda")
    Lmax = max(lens)
    cos, sin = synthetic.build_rope_tables(Lmax, 64, device=dev)
    kv = inp.kv_cache.to(dev)
    W_UV, W_UK = inp.W_UV.to(dev), inp.W_UK.to(dev)
    q_nope, q_rope = inp.q_nope.float().to(dev), inp.q_rope.float().to(dev)
    seq = torch.tensor(lens, dtype=torch.int32, device=dev)
    offs = torch.tensor(inp.kv_offsets, dtype=torch.int64, device=dev)
    out = mla_decode(kv, q_rope, W_UV, cos, sin, cfg, q_nope=q_nope, W_UK=W_UK, seq_lens=seq,
                     kv_offsets=offs, max_seq_len=Lmax).cpu().numpy()
    out_h = mla_decode(kv, q_rope, W_UV, cos, sin, cfg, q_nope=q_nope, W_UK=W_UK, seq_lens=seq,
                       kv_offsets=offs, max_seq_len=Lmax, seq_lens_host=lens).cpu().numpy()
    np.testing.assert_array_equal(out, out_h)  # host-planned == device-planned (same split)
    cos_np, sin_np = cos.cpu().numpy(), sin.cpu().numpy()
    for b in (0, 1, 17, 31, 50, 63):
        assert_close(out[b], _oracle_single(inp, b, cos_np, sin_np), f"seq {b} (L={lens[b]})")
    for b in (3, 40):
        L, off = lens[b], inp.kv_offsets[b]
        single = mla_decode(kv[off:off + L], q_rope[b:b + 1].contiguous(), W_UV, cos, sin, cfg,
                            q_nope=q_nope[b:b + 1].contiguous(), W_UK=W_UK).cpu().numpy()[0]
        assert_close(out[b], single, f"batched vs single seq {b}")


def test_edge_cases_zero_length_strided_offset():
    dev = torch.device("cuda")
    cfg = MLAConfig.deepseek_v2()
    lens = [0, 5, 64, 0, 130]
    inp = synthetic.baseline_inputs(num_heads=128, seq_lens=lens, seed=5)
    Lmax = max(lens)
    cos, sin = synthetic.build_rope_tables(Lmax + 100, 64, device=dev)
    cos_np, sin_np = cos.cpu().numpy(), sin.cpu().numpy()
    # strided cache: rows padded to 640 elements
    kv = torch.zeros(inp.kv_cache.size(0), 640, dtype=inp.kv_cache.dtype)
    kv[:, :576] = inp.kv_cache
    kv = kv.to(dev)
    for kern in kernels_for(cfg):
        out = mla_decode(kv, inp.q_rope.float().to(dev), inp.W_UV.to(dev), cos, sin, cfg,
                         q_nope=inp.q_nope.float().to(dev), W_UK=inp.W_UK.to(dev),
                         seq_lens=torch.tensor(lens, dtype=torch.int32, device=dev),
                         kv_offsets=torch.tensor(inp.kv_offsets, dtype=torch.int64, device=dev),
                         max_seq_len=Lmax, kv_row_stride=640, kernel=kern).cpu().numpy()
        for b, L in enumerate(lens):
            if L == 0:
                assert np.all(out[b] == 0), "empty sequence must give zeros"
            else:
                assert_close(out[b], _oracle_single(inp, b, cos_np, sin_np), f"b={b} L={L} kernel={kern}")
        # kv_pos_offset: the tables are read from row kv_pos_offset on
        off = 37
        b = 4
        L = lens[b]
        kvb = inp.kv_cache[inp.kv_offsets[b]:inp.kv_offsets[b] + L].contiguous().to(dev)
        out2 = mla_decode(kvb, inp.q_rope[b:b + 1].float().to(dev), inp.W_UV.to(dev), cos, sin, cfg,
                          q_nope=inp.q_nope[b:b + 1].float().to(dev), W_UK=inp.W_UK.to(dev),
                          kv_pos_offset=off, kernel=kern).cpu().numpy()[0]
        q_abs = O.absorb_query(inp.q_nope[b].float().numpy(), inp.W_UK.float().numpy(), 128, 512)
        ref = O.absorbed_decode(kvb.cpu().float().numpy(), q_abs, inp.q_rope[b].float().numpy(),
                                inp.W_UV.float().numpy(), cos_np[off:off + L], sin_np[off:off + L],
                                128, 512, 128, 64, 128)
        assert_close(out2, ref, f"kv_pos_offset kernel={kern}")


def test_kv_range_shards_combine():
    """Single long sequence cut into 4 KV-range shards: partials + mla_combine_partials == one decode."""
    dev = torch.device("cuda")
    cfg = MLAConfig.deepseek_v2()
    L, G = 4096, 4
    inp = synthetic.baseline_inputs(num_heads=128, seq_lens=[L], seed=9)
    cos, sin = synthetic.build_rope_tables(L, 64, device=dev)
    kv = inp.kv_cache.to(dev)
    W_UV, W_UK = inp.W_UV.to(dev), inp.W_UK.to(dev)
    qn, qr = inp.q_nope.float().to(dev), inp.q_rope.float().to(dev)
    full = mla_decode(kv, qr, W_UV, cos, sin, cfg, q_nope=qn, W_UK=W_UK).cpu().numpy()
    step = L // G
    mls, os_ = [], []
    for g in range(G):
        ml, o = _C.mla_decode_partial(kv[g * step:(g + 1) * step].contiguous(), qr, W_UV, cos, sin,
                                      *[cfg.d_model, 512, 128, 64, 128, 128], q_nope=qn, W_UK=W_UK,
                                      kv_pos_offset=g * step)
        mls.append(ml)
        os_.append(o)
    out = _C.mla_combine_partials(torch.stack(mls), torch.stack(os_), W_UV, cfg.d_model, 512, 128, 64, 128,
                                  128).cpu().numpy()
    assert_close(out, full, "sharded vs whole")
    ref = _oracle_single(inp, 0, cos.cpu().numpy(), sin.cpu().numpy())
    assert_close(out[0], ref, "sharded vs oracle")


@pytest.mark.parametrize("parts,B", [(1, 3), (40, 5), (128, 70)])
def test_combine_partials_many_parts_with_empty(parts, B):
    """mla_combine_partials on synthetic partial sets: natural-log maxima spread over a wide
    range, every third part empty (l = 0, o = 0), more than one block of tokens; checked
    against the log-sum-exp merge and the W_UV projection in numpy."""
    dev = torch.device("cuda")
    H, dc, dv = 16, 512, 128
    g = torch.Generator().manual_seed(parts * 131 + B)
    m = torch.randn(parts, B, H, generator=g) * 4.0
    l = torch.rand(parts, B, H, generator=g) * 50.0 + 0.5
    o = torch.randn(parts, B, H, dc, generator=g) * l[..., None]   # unnormalised sums
    if parts > 1:
        l[::3] = 0.0
        o[::3] = 0.0
        m[::3] = -1e30
    W_UV = (torch.randn(H * dv, dc, generator=g) * 0.05).to(torch.bfloat16)
    ml = torch.stack([m, l], dim=-1).contiguous()
    out = _C.mla_combine_partials(ml.to(dev), o.contiguous().to(dev), W_UV.to(dev), 0, dc, 128, 64, H,
                                  dv).cpu().numpy()
    mm = np.where(l.numpy() > 0, m.numpy(), -np.inf).astype(np.float64)
    ll, oo = l.numpy().astype(np.float64), o.numpy().astype(np.float64)
    W = W_UV.float().numpy().astype(np.float64).reshape(H, dv, dc)
    for b in range(B):
        olat = O.combine_partials(mm[:, b], ll[:, b], oo[:, b])             # (H, dc)
        ref = np.einsum("hc,hjc->hj", olat, W)
        assert_close(out[b], ref, f"parts={parts} b={b}")


def test_errors_raise_runtime_error():
    dev = torch.device("cuda")
    cfg = MLAConfig.deepseek_v2()
    kv = torch.zeros(16, 576, dtype=torch.float16, device=dev)
    W_UV = torch.zeros(128 * 128, 512, dtype=torch.float16, device=dev)
    q = torch.zeros(128, 512, device=dev)
    qr = torch.zeros(128, 64, device=dev)
    cos, sin = synthetic.build_rope_tables(16, 64, device=dev)
    with pytest.raises(RuntimeError, match="float16 or bfloat16"):
        fused_mla(kv.float(), q, qr, W_UV, cos, sin, cfg)
    with pytest.raises(RuntimeError, match="q_absorbed shape mismatch"):
        fused_mla(kv, q[:5], qr, W_UV, cos, sin, cfg)
    with pytest.raises(RuntimeError, match="contiguous"):
        fused_mla(kv, q.t(), qr, W_UV, cos, sin, cfg)
    with pytest.raises(ValueError, match="positive"):
        fused_mla(kv, q, qr, W_UV, cos, sin, MLAConfig(0, 512, 128, 64, 0, 128))


def test_deterministic():
    dev = torch.device("cuda")
    cfg = MLAConfig.deepseek_v2()
    inp = synthetic.baseline_inputs(num_heads=128, seq_lens=[3000], seed=3)
    cos, sin = synthetic.build_rope_tables(3000, 64, device=dev)
    args = (inp.kv_cache.to(dev), inp.q_rope.float().to(dev), inp.W_UV.to(dev), cos, sin, cfg)
    kw = dict(q_nope=inp.q_nope.float().to(dev), W_UK=inp.W_UK.to(dev))
    a = mla_decode(*args, **kw)
    b = mla_decode(*args, **kw)
    assert torch.equal(a, b)


def test_decode_timer_eager_and_graph():
    """The decode-kernel timer (mla_timer_t) works on a plain stream and inside a captured CUDA
    graph, and a graph replay computes the same output as a direct call."""
    dev = torch.device("cuda:0")
    cfg = MLAConfig.deepseek_v2()
    inp = synthetic.baseline_inputs(num_heads=128, seq_lens=[4096], seed=11)
    kv = inp.kv_cache.to(dev)
    W_UK, W_UV = inp.W_UK.to(dev), inp.W_UV.to(dev)
    qn, qr = inp.q_nope.float().to(dev), inp.q_rope.float().to(dev)
    cos, sin = synthetic.build_rope_tables(4096, 64, device=dev)
    ws = torch.empty(1 << 26, dtype=torch.uint8, device=dev)

    def call(out, timer=None):
        return mla_decode(kv, qr, W_UV, cos, sin, cfg, q_nope=qn, W_UK=W_UK, max_seq_len=4096, out=out,
                          workspace=ws, timer=timer)

    ref = call(torch.empty(1, 128, 128, dtype=torch.float32, device=dev)).clone()
    t_eager = _lib.DecodeTimer()
    out_eager = call(torch.empty_like(ref), t_eager)
    torch.cuda.synchronize()
    assert t_eager.decode_ms() > 0
    assert torch.equal(out_eager, ref)

    out_graph = torch.zeros_like(ref)
    t_graph = _lib.DecodeTimer()
    side = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side):
        call(out_graph, t_graph)
    g.replay()
    torch.cuda.synchronize()
    assert t_graph.decode_ms() > 0
    assert torch.equal(out_graph, ref)
    del g
    t_eager.close()
    t_graph.close()


def _oracle_single_otf(inp, b, H=128, dc=512, dn=128, dR=64, dv=128, pos_offset=0):
    """Oracle of sequence b with the on-the-fly RoPE mode's cos / sin."""
    L, off = inp.seq_lens[b], inp.kv_offsets[b]
    cos, sin = O.rope_tables_otf(L, dR, pos_offset=pos_offset)
    kv = inp.kv_cache[off:off + L].float().numpy()
    q_abs = O.absorb_query(inp.q_nope[b].float().numpy(), inp.W_UK.float().numpy(), H, dc)
    return O.absorbed_decode(kv, q_abs, inp.q_rope[b].float().numpy(), inp.W_UV.float().numpy(), cos, sin,
                             H, dc, dn, dR, dv)


@pytest.mark.parametrize("L", [8192, 131072])
def test_on_the_fly_rope_vs_oracle_and_tables(L):
    """No RoPE tables (rope_cos = rope_sin = None): the kernels compute cos / sin themselves.
    BASELINE configs 1 and 3 on both decode kernels, against the fp64 oracle with the same
    angles, and against the table path (the reference's tables) within the same bound."""
    inp = synthetic.baseline_inputs(num_heads=128, seq_lens=[L], seed=0)
    cfg = MLAConfig.deepseek_v2()
    dev = torch.device("cuda")
    kv, W_UV, W_UK = inp.kv_cache.to(dev), inp.W_UV.to(dev), inp.W_UK.to(dev)
    qn, qr = inp.q_nope.float().to(dev), inp.q_rope.float().to(dev)
    cos, sin = synthetic.build_rope_tables(L, 64, device=dev)
    ref = _oracle_single_otf(inp, 0)
    for kern in kernels_for(cfg):
        otf = mla_decode(kv, qr, W_UV, None, None, cfg, q_nope=qn, W_UK=W_UK, kernel=kern).cpu().numpy()[0]
        tab = mla_decode(kv, qr, W_UV, cos, sin, cfg, q_nope=qn, W_UK=W_UK, kernel=kern).cpu().numpy()[0]
        assert_close(otf, ref, f"on-the-fly L={L} kernel={kern}")
        assert_close(otf, tab, f"on-the-fly vs tables L={L} kernel={kern}")


def test_on_the_fly_rope_offset_theta_and_varlen():
    """On-the-fly RoPE with a KV-range position offset, a non-default theta, a variable-length
    batch with a partial last tile, and the reference-shaped op given no tables."""
    dev = torch.device("cuda")
    cfg = MLAConfig.deepseek_v2()
    lens = [77, 640, 1]
    inp = synthetic.baseline_inputs(num_heads=128, seq_lens=lens, seed=21)
    kv = inp.kv_cache.to(dev)
    qn, qr, W_UK, W_UV = inp.q_nope.float().to(dev), inp.q_rope.float().to(dev), inp.W_UK.to(dev), inp.W_UV.to(dev)
    for kern in kernels_for(cfg):
        out = mla_decode(kv, qr, W_UV, None, None, cfg, q_nope=qn, W_UK=W_UK,
                         seq_lens=torch.tensor(lens, dtype=torch.int32, device=dev),
                         kv_offsets=torch.tensor(inp.kv_offsets, dtype=torch.int64, device=dev),
                         max_seq_len=max(lens), kernel=kern).cpu().numpy()
        for b in range(len(lens)):
            assert_close(out[b], _oracle_single_otf(inp, b), f"varlen b={b} kernel={kern}")
        # one sequence's rows at absolute positions 1000.., theta 50000
        b, off, theta = 1, 1000, 50000.0
        L, r0 = lens[b], inp.kv_offsets[b]
        kvb = kv[r0:r0 + L].contiguous()
        got = mla_decode(kvb, qr[b:b + 1].contiguous(), W_UV, None, None, cfg, q_nope=qn[b:b + 1].contiguous(),
                         W_UK=W_UK, kv_pos_offset=off, rope_theta=theta, kernel=kern).cpu().numpy()[0]
        cos, sin = O.rope_tables_otf(L, 64, theta=theta, pos_offset=off)
        q_abs = O.absorb_query(inp.q_nope[b].float().numpy(), inp.W_UK.float().numpy(), 128, 512)
        ref = O.absorbed_decode(kvb.cpu().float().numpy(), q_abs, inp.q_rope[b].float().numpy(),
                                inp.W_UV.float().numpy(), cos, sin, 128, 512, 128, 64, 128)
        assert_close(got, ref, f"offset + theta kernel={kern}")
    with pytest.raises(RuntimeError, match="both rope_cos and rope_sin"):
        mla_decode(kv, qr, W_UV, synthetic.build_rope_tables(640, 64, device=dev)[0], None, cfg, q_nope=qn,
                   W_UK=W_UK, seq_lens=torch.tensor(lens, dtype=torch.int32, device=dev),
                   kv_offsets=torch.tensor(inp.kv_offsets, dtype=torch.int64, device=dev), max_seq_len=640)


def _per_token_cosine(a, b):
    """The reference's batched-vs-loop criterion (tests/test_batched.py:82-86)."""
    a = np.asarray(a, dtype=np.float64).ravel()
    b = np.asarray(b, dtype=np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))


def test_config4_batch256_vs_oracle():
    """BASELINE config 4 (B=256, L=4096, H=128, bf16, in-op absorption): two full 128-token
    blocks of the absorption GEMM and the projection's four 64-token blocks. Six sequences
    against the fp64 oracle and two against single-sequence decodes, on both decode kernels."""
    L, B = 4096, 256
    inp = synthetic.baseline_inputs(num_heads=128, seq_lens=[L] * B, seed=4)
    cfg = MLAConfig.deepseek_v3()
    dev = torch.device("cuda")
    kv, W_UV, W_UK = inp.kv_cache.to(dev), inp.W_UV.to(dev), inp.W_UK.to(dev)
    qn, qr = inp.q_nope.float().to(dev), inp.q_rope.float().to(dev)
    cos, sin = synthetic.build_rope_tables(L, 64, device=dev)
    cos_np, sin_np = cos.cpu().numpy(), sin.cpu().numpy()
    refs = {b: _oracle_single(inp, b, cos_np, sin_np) for b in (0, 1, 63, 64, 200, 255)}
    for kern in kernels_for(cfg):
        out = mla_decode(kv, qr, W_UV, cos, sin, cfg, q_nope=qn, W_UK=W_UK, max_seq_len=L,
                         kernel=kern).cpu().numpy()
        assert np.isfinite(out).all()
        for b, ref in refs.items():
            assert_close(out[b], ref, f"cfg4 seq {b} kernel={kern}")
        for b in (7, 130):
            single = mla_decode(kv[b * L:(b + 1) * L], qr[b:b + 1].contiguous(), W_UV, cos, sin, cfg,
                                q_nope=qn[b:b + 1].contiguous(), W_UK=W_UK, kernel=kern).cpu().numpy()[0]
            assert_close(out[b], single, f"cfg4 batched vs single seq {b} kernel={kern}")
            assert _per_token_cosine(out[b], single) > 0.998


@pytest.mark.parametrize("B", [65, 257, 300])
def test_batches_crossing_gemm_blocks(B):
    """Batches that cross the absorption GEMM's 128-token blocks (257, 300: a one-token and a
    44-token tail block) and the projection's 64-token blocks (65: a one-token tail block), with
    short variable lengths
    (partial tiles, single-position sequences), every sequence against the oracle, on both
    decode kernels."""
    lens = [1 + (37 * b) % 200 for b in range(B)]
    inp = synthetic.baseline_inputs(num_heads=128, seq_lens=lens, seed=B)
    cfg = MLAConfig.deepseek_v2()
    dev = torch.device("cuda")
    Lmax = max(lens)
    cos, sin = synthetic.build_rope_tables(Lmax, 64, device=dev)
    cos_np, sin_np = cos.cpu().numpy(), sin.cpu().numpy()
    kv, W_UV, W_UK = inp.kv_cache.to(dev), inp.W_UV.to(dev), inp.W_UK.to(dev)
    qn, qr = inp.q_nope.float().to(dev), inp.q_rope.float().to(dev)
    seq = torch.tensor(lens, dtype=torch.int32, device=dev)
    offs = torch.tensor(inp.kv_offsets, dtype=torch.int64, device=dev)
    refs = [_oracle_single(inp, b, cos_np, sin_np) for b in range(B)]
    for kern in kernels_for(cfg):
        out = mla_decode(kv, qr, W_UV, cos, sin, cfg, q_nope=qn, W_UK=W_UK, seq_lens=seq, kv_offsets=offs,
                         max_seq_len=Lmax, kernel=kern).cpu().numpy()
        for b in range(B):
            assert_close(out[b], refs[b], f"B={B} seq {b} (L={lens[b]}) kernel={kern}")


@pytest.mark.parametrize("B", [1, 2])
def test_kv_range_packed_head_slices(B):
    """The head-sliced KV-range path on one GPU: 4 KV-range shards each export packed partials
    (mla_decode_partial_packed, 4 head slices); slice q's merge takes every shard's block q
    (what the all-to-all delivers) and projects through W_UV's rows of those heads
    (mla_combine_partials_packed); the slices side by side equal one whole decode and the oracle."""
    dev = torch.device("cuda")
    cfg = MLAConfig.deepseek_v2()
    L, G = 3000, 4
    inp = synthetic.baseline_inputs(num_heads=128, seq_lens=[L] * B, seed=19)
    kv = inp.kv_cache.to(dev)
    W_UV, W_UK = inp.W_UV.to(dev), inp.W_UK.to(dev)
    qn, qr = inp.q_nope.float().to(dev), inp.q_rope.float().to(dev)
    dims = (cfg.d_model, 512, 128, 64, 128, 128)
    full = mla_decode(kv, qr, W_UV, None, None, cfg, q_nope=qn, W_UK=W_UK, max_seq_len=L).cpu().numpy()
    bounds = [L * g // G for g in range(G + 1)]
    packed = []
    for g in range(G):
        lo, hi = bounds[g], bounds[g + 1]
        shard = torch.cat([kv[b * L + lo:b * L + hi] for b in range(B)]).contiguous()
        packed.append(_C.mla_decode_partial_packed(shard, qr, W_UV, None, None, *dims, num_slices=G, q_nope=qn,
                                                   W_UK=W_UK, kv_pos_offset=lo))
    hs = 128 // G
    slices = []
    for q in range(G):
        recv = torch.stack([packed[g][q] for g in range(G)]).contiguous()     # (G, B, hs, 516)
        slices.append(_C.mla_combine_partials_packed(recv, W_UV[q * hs * 128:(q + 1) * hs * 128], *dims))
    out = torch.cat(slices, dim=1).cpu().numpy()                               # (B, 128, 128)
    for b in range(B):
        assert_close(out[b], full[b], f"packed slices vs whole, b={b}")
        cos, sin = O.rope_tables_otf(L, 64)
        q_abs = O.absorb_query(inp.q_nope[b].float().numpy(), inp.W_UK.float().numpy(), 128, 512)
        ref = O.absorbed_decode(inp.kv_cache[b * L:(b + 1) * L].float().numpy(), q_abs, inp.q_rope[b].float().numpy(),
                                inp.W_UV.float().numpy(), cos, sin, 128, 512, 128, 64, 128)
        assert_close(out[b], ref, f"packed slices vs oracle, b={b}")
    # the layout: row (q * B + b) * hs + h % hs of slice q; m, l, then two zero floats, then o
    p0 = packed[0].view(-1, 516).cpu()
    assert torch.all(p0[:, 2:4] == 0) and torch.all(p0[:, 1] > 0)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("B", [1, 2, 3, 4, 5])
def test_small_batches_gemv_and_tensor_core_gemms(B, dtype):
    """Batches of 1-4 tokens take the fp32 CUDA-core absorption and merge/projection kernels, 5
    tokens the tensor-core ones. Lengths from one position (a single record, no merge) to 20000
    (records of every split-KV worker), every sequence against the oracle, on both decode kernels."""
    lens = [1, 20000, 5, 777, 64][:B]
    inp = synthetic.baseline_inputs(num_heads=128, seq_lens=lens, seed=31 + B, dtype=dtype)
    cfg = MLAConfig.deepseek_v2()
    dev = torch.device("cuda")
    Lmax = max(lens)
    cos, sin = synthetic.build_rope_tables(Lmax, 64, device=dev)
    cos_np, sin_np = cos.cpu().numpy(), sin.cpu().numpy()
    kv, W_UV, W_UK = inp.kv_cache.to(dev), inp.W_UV.to(dev), inp.W_UK.to(dev)
    qn, qr = inp.q_nope.float().to(dev), inp.q_rope.float().to(dev)
    seq = torch.tensor(lens, dtype=torch.int32, device=dev)
    offs = torch.tensor(inp.kv_offsets, dtype=torch.int64, device=dev)
    refs = [_oracle_single(inp, b, cos_np, sin_np) for b in range(B)]
    for kern in kernels_for(cfg):
        out = mla_decode(kv, qr, W_UV, cos, sin, cfg, q_nope=qn, W_UK=W_UK, seq_lens=seq, kv_offsets=offs,
                         max_seq_len=Lmax, kernel=kern).cpu().numpy()
        for b in range(B):
            assert_close(out[b], refs[b], f"B={B} {dtype} seq {b} (L={lens[b]}) kernel={kern}")


@pytest.mark.parametrize("B", [1, 3])
def test_pinned_host_queries_and_output(B):
    """mla_decode given pinned host q_nope / q_rope and a pinned host output (the kernels read and
    write them over the host link) returns exactly what it returns for device tensors."""
    cfg = MLAConfig.deepseek_v2()
    inp = synthetic.baseline_inputs(num_heads=128, seq_lens=[3000] * B, seed=21)
    dev = torch.device("cuda", 0)
    kv, W_UK, W_UV = inp.kv_cache.to(dev), inp.W_UK.to(dev), inp.W_UV.to(dev)
    qn_d, qr_d = inp.q_nope.float().to(dev), inp.q_rope.float().to(dev)
    want = mla_decode(kv, qr_d, W_UV, None, None, cfg, q_nope=qn_d, W_UK=W_UK)
    qn_h, qr_h = inp.q_nope.float().pin_memory(), inp.q_rope.float().pin_memory()
    out_h = torch.full((B, 128, 128), float("nan")).pin_memory()
    got = mla_decode(kv, qr_h, W_UV, None, None, cfg, q_nope=qn_h, W_UK=W_UK, out=out_h)
    torch.cuda.synchronize()
    assert got is out_h
    assert torch.equal(out_h, want.cpu())
