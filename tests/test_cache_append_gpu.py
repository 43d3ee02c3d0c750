"""Device-side cache append (mla_cache_append), the device counterpart of the reference's
LatentKVCache::append_host (src/mla_config.cuh:58-72): the new rows land bit-exact at each
sequence's current length, the lengths advance on the device, a full sequence is left alone and
flagged, and a decode over appended rows equals a decode over the same cache written directly."""

import pytest
import torch

from latent_attn import MLAConfig, synthetic, _C
from latent_attn.functional import mla_decode

pytestmark = pytest.mark.gpu

DIMS = (0, 512, 128, 64, 128, 128)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_append_rows_lengths_and_full_sequence(dtype):
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(7)
    B, cap = 5, 40
    offs = torch.tensor([0, 40, 100, 140, 200], dtype=torch.int64)     # gaps between the sequences
    kv = torch.randn(240, 576, generator=g).to(dtype).to(dev)
    lens = torch.tensor([0, 17, 39, 40, 5], dtype=torch.int32)           # sequence 3 starts full
    expect, cur = kv.clone(), lens.clone()
    lens_d, offs_d = lens.to(dev), offs.to(dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    for _ in range(2):                                                   # sequence 2 fills up on the first call
        c_t = torch.randn(B, 512, generator=g).to(dtype)
        k_r = torch.randn(B, 64, generator=g).to(dtype)
        _C.mla_cache_append(kv, c_t.to(dev), k_r.to(dev), lens_d, cap, *DIMS, kv_offsets=offs_d, status=status)
        for b in range(B):
            if cur[b] < cap:
                r = int(offs[b]) + int(cur[b])
                expect[r, :512] = c_t[b].to(dev)
                expect[r, 512:] = k_r[b].to(dev)
                cur[b] += 1
    torch.cuda.synchronize()
    assert torch.equal(kv, expect)
    assert torch.equal(lens_d.cpu(), cur)
    assert int(status.item()) == 1


def test_append_strided_rows_and_odd_dims():
    """Rows with a padded stride (16-byte path) and dimensions that are not multiples of 8
    (element path); without kv_offsets sequence b starts at row b * max_seq_len."""
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(11)
    B, cap = 3, 8
    full = torch.zeros(B * cap, 640, dtype=torch.bfloat16, device=dev)
    kv = full[:, :576]                                                   # row stride 640 elements
    lens_d = torch.tensor([0, 3, 7], dtype=torch.int32, device=dev)
    c_t = torch.randn(B, 512, generator=g).to(torch.bfloat16).to(dev)
    k_r = torch.randn(B, 64, generator=g).to(torch.bfloat16).to(dev)
    _C.mla_cache_append(kv, c_t, k_r, lens_d, cap, *DIMS)
    torch.cuda.synchronize()
    for b, p in enumerate((0, 3, 7)):
        assert torch.equal(kv[b * cap + p], torch.cat([c_t[b], k_r[b]]))
    assert int(full[:, 576:].abs().sum().item()) == 0                    # padding untouched
    assert lens_d.cpu().tolist() == [1, 4, 8]

    odd = (0, 20, 8, 4, 2, 8)                                            # d_c = 20, d_R = 4
    kv2 = torch.zeros(B * cap, 24, dtype=torch.float16, device=dev)
    lens2 = torch.tensor([1, 0, 5], dtype=torch.int32, device=dev)
    c2 = torch.randn(B, 20, generator=g).to(torch.float16).to(dev)
    r2 = torch.randn(B, 4, generator=g).to(torch.float16).to(dev)
    _C.mla_cache_append(kv2, c2, r2, lens2, cap, *odd)
    torch.cuda.synchronize()
    for b, p in enumerate((1, 0, 5)):
        assert torch.equal(kv2[b * cap + p], torch.cat([c2[b], r2[b]]))
    assert lens2.cpu().tolist() == [2, 1, 6]


def test_decode_after_device_appends_equals_direct_cache():
    """Prefill two sequences, append three decode steps on the device, then decode with the
    device lengths: the output equals a decode over the same rows written directly."""
    dev = torch.device("cuda")
    cfg = MLAConfig.deepseek_v2()
    cap, pre, steps = 256, [100, 37], 3
    inp = synthetic.baseline_inputs(num_heads=128, seq_lens=[cap, cap], seed=21)
    rows = inp.kv_cache.to(dev)                                          # (2 * cap, 576): every row the test needs
    offs = torch.tensor([0, cap], dtype=torch.int64, device=dev)
    kv = torch.zeros_like(rows)
    for b, n in enumerate(pre):
        kv[b * cap:b * cap + n] = rows[b * cap:b * cap + n]
    lens = torch.tensor(pre, dtype=torch.int32, device=dev)
    for s in range(steps):
        new = torch.stack([rows[b * cap + pre[b] + s] for b in range(2)])
        _C.mla_cache_append(kv, new[:, :512].contiguous(), new[:, 512:].contiguous(), lens, cap,
                            cfg.d_model, 512, 128, 64, 128, 128, kv_offsets=offs)
    final = [n + steps for n in pre]
    assert lens.cpu().tolist() == final
    direct = torch.zeros_like(rows)
    for b, n in enumerate(final):
        direct[b * cap:b * cap + n] = rows[b * cap:b * cap + n]
    assert torch.equal(kv, direct)
    cos, sin = synthetic.build_rope_tables(cap, 64, device=dev)
    args = dict(q_nope=inp.q_nope.float().to(dev), W_UK=inp.W_UK.to(dev), kv_offsets=offs, max_seq_len=cap)
    qr, W_UV = inp.q_rope.float().to(dev), inp.W_UV.to(dev)
    out_a = mla_decode(kv, qr, W_UV, cos, sin, cfg, seq_lens=lens, **args)
    out_b = mla_decode(direct, qr, W_UV, cos, sin, cfg,
                       seq_lens=torch.tensor(final, dtype=torch.int32, device=dev), **args)
    assert torch.equal(out_a, out_b)


def _paged_copy(kv, offs, lens, page_rows, max_pages, n_pool_pages, seed):
    """Scatter each sequence's rows into shuffled pages of a pool pre-filled with noise; unused
    page-table entries are -1 (never read for positions below the sequence length)."""
    g = torch.Generator().manual_seed(seed)
    pool = torch.randn(n_pool_pages * page_rows, kv.size(1), generator=g).to(kv.dtype).to(kv.device)
    perm = torch.randperm(n_pool_pages, generator=g).tolist()
    table = torch.full((len(lens), max_pages), -1, dtype=torch.int32)
    nxt = 0
    for b, n in enumerate(lens):
        for k in range((n + page_rows - 1) // page_rows):
            pid = perm[nxt]
            nxt += 1
            table[b, k] = pid
            m = min(page_rows, n - k * page_rows)
            pool[pid * page_rows:pid * page_rows + m] = kv[offs[b] + k * page_rows:offs[b] + k * page_rows + m]
    return pool, table.to(kv.device)


@pytest.mark.parametrize("page_rows", [64, 128])
@pytest.mark.parametrize("kernel", [1, 2])          # tensor-core, CUDA-core decode
def test_paged_decode_equals_contiguous(page_rows, kernel):
    dev = torch.device("cuda")
    cfg = MLAConfig.deepseek_v2()
    lens, cap = [300, 1000, 327], 1024
    inp = synthetic.baseline_inputs(num_heads=128, seq_lens=lens, seed=31)
    kv = inp.kv_cache.to(dev)
    max_pages = cap // page_rows
    need = sum((n + page_rows - 1) // page_rows for n in lens)
    pool, table = _paged_copy(kv, inp.kv_offsets, lens, page_rows, max_pages, need + 5, seed=page_rows)
    cos, sin = synthetic.build_rope_tables(cap, 64, device=dev)
    lens_d = torch.tensor(lens, dtype=torch.int32, device=dev)
    common = dict(q_nope=inp.q_nope.float().to(dev), W_UK=inp.W_UK.to(dev), seq_lens=lens_d, max_seq_len=cap,
                  kernel=kernel)
    qr, W_UV = inp.q_rope.float().to(dev), inp.W_UV.to(dev)
    contig = mla_decode(kv, qr, W_UV, cos, sin, cfg,
                        kv_offsets=torch.tensor(inp.kv_offsets, dtype=torch.int64, device=dev), **common)
    paged = mla_decode(pool, qr, W_UV, cos, sin, cfg, page_table=table, page_rows=page_rows, **common)
    assert torch.isfinite(paged).all()
    assert torch.equal(paged, contig)

    # a page id outside the pool reads nothing and makes the output NaN
    bad = table.clone()
    bad[1, 3] = 1 << 20
    broken = mla_decode(pool, qr, W_UV, cos, sin, cfg, page_table=bad, page_rows=page_rows, **common)
    assert torch.isnan(broken).any()


def test_paged_append_then_decode():
    """Device appends through a page table cross a page boundary and land in the mapped pages;
    the decode over the pool then equals the contiguous decode of the same rows."""
    dev = torch.device("cuda")
    cfg = MLAConfig.deepseek_v2()
    page_rows, cap, pre, steps = 64, 256, [70, 62], 4
    inp = synthetic.baseline_inputs(num_heads=128, seq_lens=[cap, cap], seed=41)
    rows = inp.kv_cache.to(dev)                                       # (2 * cap, 576)
    offs = [0, cap]
    pool, table = _paged_copy(rows, offs, pre, page_rows, cap // page_rows, 12, seed=5)
    for b in range(2):                                                # pages for the rows still to come
        used = set(table[b].tolist()) | set(table[1 - b].tolist())
        free = [p for p in range(12) if p not in used]
        for k in range(cap // page_rows):
            if int(table[b, k]) < 0:
                table[b, k] = free.pop(0)
                used.add(int(table[b, k]))
    lens = torch.tensor(pre, dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    for s in range(steps):
        new = torch.stack([rows[offs[b] + pre[b] + s] for b in range(2)])
        _C.mla_cache_append(pool, new[:, :512].contiguous(), new[:, 512:].contiguous(), lens, cap,
                            cfg.d_model, 512, 128, 64, 128, 128, page_table=table, page_rows=page_rows,
                            status=status)
    final = [n + steps for n in pre]
    torch.cuda.synchronize()
    assert lens.cpu().tolist() == final and int(status.item()) == 0
    for b in range(2):
        for p in range(pre[b], final[b]):
            r = int(table[b, p // page_rows]) * page_rows + p % page_rows
            assert torch.equal(pool[r], rows[offs[b] + p])
    cos, sin = synthetic.build_rope_tables(cap, 64, device=dev)
    common = dict(q_nope=inp.q_nope.float().to(dev), W_UK=inp.W_UK.to(dev), seq_lens=lens, max_seq_len=cap)
    qr, W_UV = inp.q_rope.float().to(dev), inp.W_UV.to(dev)
    paged = mla_decode(pool, qr, W_UV, cos, sin, cfg, page_table=table, page_rows=page_rows, **common)
    contig = mla_decode(rows, qr, W_UV, cos, sin, cfg,
                        kv_offsets=torch.tensor(offs, dtype=torch.int64, device=dev), **common)
    assert torch.equal(paged, contig)


def test_append_rejects_rows_outside_the_cache():
    """A page id near INT_MAX (whose page end would overflow 32-bit arithmetic) and an offset
    past the cache's rows are not written: the cache stays untouched, the length does not
    advance, and bit 1 of the status word is set."""
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(13)
    kv = torch.randn(256, 576, generator=g).to(torch.bfloat16).to(dev)
    before = kv.clone()
    c_t = torch.randn(1, 512, generator=g).to(torch.bfloat16).to(dev)
    k_r = torch.randn(1, 64, generator=g).to(torch.bfloat16).to(dev)
    # paged: the sequence's only page id is INT_MAX
    table = torch.full((1, 2), 2 ** 31 - 1, dtype=torch.int32, device=dev)
    lens = torch.tensor([3], dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    _C.mla_cache_append(kv, c_t, k_r, lens, 128, *DIMS, page_table=table, page_rows=64, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 2 and int(lens.item()) == 3
    assert torch.equal(kv, before)
    # contiguous: an offset whose row lies past the cache's 256 rows
    offs = torch.tensor([250], dtype=torch.int64, device=dev)
    lens = torch.tensor([10], dtype=torch.int32, device=dev)
    status.zero_()
    _C.mla_cache_append(kv, c_t, k_r, lens, 64, *DIMS, kv_offsets=offs, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 2 and int(lens.item()) == 10
    assert torch.equal(kv, before)
