"""Torch-facing operators, mirroring the reference's ``latent_attn._C`` module
(csrc/bindings.cpp:1-256 of anishesg/latent-attn): same op names, same argument
order and meaning, output allocated by the op on the current CUDA stream, and
``RuntimeError`` on a wrong dtype, layout, device or shape.

Differences from the reference, all additive:
* the cache / weight tensors may be float16 (the reference's only type) or
  bfloat16;
* the computation runs through the C ABI (``libmla_b200.so``): query packing,
  the tensor-core split-KV decode (or the CUDA-core kernel for shapes it does not
  cover) and the log-sum-exp combine with the W_UV projection;
* ``mla_decode`` / ``mla_decode_partial`` / ``mla_combine_partials`` expose the
  general decode (in-op absorption, variable-length batches, KV-range shards).

PyTorch is used only for tensors, streams and workspace memory.
"""

from __future__ import annotations

import ctypes as C
import math
from typing import Optional, Sequence

import torch

from . import _lib

_DT = {torch.float16: _lib.DTYPE_F16, torch.bfloat16: _lib.DTYPE_BF16}


def _check_half(t: torch.Tensor, name: str) -> None:
    if t.dtype not in _DT:
        raise RuntimeError(f"{name} must be float16 or bfloat16, got {t.dtype}")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be on CUDA")


def _check_f32(t: torch.Tensor, name: str) -> None:
    if t.dtype != torch.float32:
        raise RuntimeError(f"{name} must be float32, got {t.dtype}")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be on CUDA")


def _check_f32_io(t: torch.Tensor, name: str) -> None:
    """A float32 query or output tensor: on the GPU, or in pinned host memory, which the kernels
    read or write directly (CUDA maps pinned allocations into the device address space)."""
    if t.dtype != torch.float32:
        raise RuntimeError(f"{name} must be float32, got {t.dtype}")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")
    if not (t.is_cuda or t.is_pinned()):
        raise RuntimeError(f"{name} must be on CUDA or in pinned host memory")


def _cfg(d_model, kv_lora_rank, qk_nope_head_dim, qk_rope_head_dim, num_heads, v_head_dim):
    key = (int(d_model), int(kv_lora_rank), int(qk_nope_head_dim), int(qk_rope_head_dim), int(num_heads),
           int(v_head_dim))
    c = _CFG_CACHE.get(key)
    if c is None:
        # MLAConfig::validate (src/mla_config.cuh:35-40) raises std::invalid_argument -> ValueError
        if kv_lora_rank <= 0 or qk_nope_head_dim <= 0 or qk_rope_head_dim <= 0:
            raise ValueError("MLA dims must be positive")
        if num_heads <= 0 or v_head_dim <= 0:
            raise ValueError("num_heads and v_head_dim must be positive")
        # the C side only reads the struct: one instance per configuration serves every call
        c = _lib.MlaConfig(*key)
        _CFG_CACHE[key] = c
    return c


_CFG_CACHE: dict = {}
# the raw current-stream query skips building a torch.cuda.Stream object on every call
_RAW_STREAM = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream(device: torch.device) -> int:
    if _RAW_STREAM is not None:
        return _RAW_STREAM(device.index if device.index is not None else torch.cuda.current_device())
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _decode_args(dtype, batch, shared, kv_cache, max_seq_len, q_rope, W_UV, rope_cos, rope_sin, out,
                 q_absorbed=None, q_nope=None, W_UK=None, seq_lens=None, kv_offsets=None,
                 seq_lens_host=None, kv_pos_offset=0, softmax_scale=0.0, kv_row_stride=0, kernel=0,
                 timer=None, page_table=None, page_rows=0, rope_theta=0.0):
    a = _lib.MlaDecodeArgs()
    a.dtype = _DT[dtype]
    a.batch = int(batch)
    a.shared_cache = 1 if shared else 0
    a.kv_cache = kv_cache.data_ptr()
    a.kv_row_stride = int(kv_row_stride)
    a.kv_total_rows = int(kv_cache.size(0))
    a.kv_offsets = _ptr(kv_offsets)
    a.seq_lens = _ptr(seq_lens)
    a.seq_lens_host = C.cast(seq_lens_host, C.c_void_p) if seq_lens_host is not None else None
    a.max_seq_len = int(max_seq_len)
    a.kv_pos_offset = int(kv_pos_offset)
    a.q_absorbed = _ptr(q_absorbed)
    a.q_nope = _ptr(q_nope)
    a.W_UK = _ptr(W_UK)
    a.q_rope = q_rope.data_ptr()
    a.W_UV = W_UV.data_ptr()
    # no tables: the kernels compute cos / sin from rope_theta (on-the-fly RoPE)
    a.rope_cos = _ptr(rope_cos)
    a.rope_sin = _ptr(rope_sin)
    a.rope_theta = float(rope_theta)
    a.softmax_scale = float(softmax_scale)
    a.output = _ptr(out)
    a.kernel = int(kernel)
    a.timer = timer.handle if timer is not None else None
    if page_table is not None:
        a.page_table = page_table.data_ptr()
        a.page_rows = int(page_rows)
        a.max_pages = int(page_table.size(-1))
    return a


def _workspace(cfg, args, device, workspace: Optional[torch.Tensor]) -> torch.Tensor:
    lib = _lib.load()
    n = C.c_size_t(0)
    _lib.check(lib.mla_decode_workspace_size(C.byref(cfg), C.byref(args), C.byref(n)))
    if workspace is not None and workspace.numel() * workspace.element_size() >= n.value \
            and workspace.data_ptr() % 256 == 0:
        return workspace
    return torch.empty(max(int(n.value), 1), dtype=torch.uint8, device=device)


def workspace_size(cfg, args) -> int:
    n = C.c_size_t(0)
    _lib.check(_lib.load().mla_decode_workspace_size(C.byref(cfg), C.byref(args), C.byref(n)))
    return int(n.value)


# ---------------------------------------------------------------------------
# reference ops
# ---------------------------------------------------------------------------

def fused_mla_forward(kv_cache, q_absorbed, q_rope, W_UV, rope_cos, rope_sin,
                      d_model, kv_lora_rank, qk_nope_head_dim, qk_rope_head_dim, num_heads, v_head_dim):
    """Single-token fused absorbed decode (csrc/bindings.cpp:126-176). Returns (H, dv) fp32."""
    _check_half(kv_cache, "kv_cache")
    _check_f32(q_absorbed, "q_absorbed")
    _check_f32(q_rope, "q_rope")
    _check_half(W_UV, "W_UV")
    _check_f32(rope_cos, "rope_cos")
    _check_f32(rope_sin, "rope_sin")
    cfg = _cfg(d_model, kv_lora_rank, qk_nope_head_dim, qk_rope_head_dim, num_heads, v_head_dim)
    seq_len = kv_cache.size(0)
    if kv_cache.dim() != 2 or kv_cache.size(1) != kv_lora_rank + qk_rope_head_dim:
        raise RuntimeError("kv_cache dim1 mismatch")
    if q_absorbed.dim() != 2 or q_absorbed.size(0) != num_heads or q_absorbed.size(1) != kv_lora_rank:
        raise RuntimeError("q_absorbed shape mismatch")
    if q_rope.dim() != 2 or q_rope.size(0) != num_heads or q_rope.size(1) != qk_rope_head_dim:
        raise RuntimeError("q_rope shape mismatch")
    _check_common(kv_cache, W_UV, rope_cos, rope_sin, seq_len, num_heads, v_head_dim, kv_lora_rank,
                  qk_rope_head_dim)
    out = torch.empty(num_heads, v_head_dim, dtype=torch.float32, device=kv_cache.device)
    if seq_len == 0:
        return out.zero_()
    _run_decode(cfg, kv_cache.dtype, 1, False, kv_cache, seq_len, q_rope, W_UV, rope_cos, rope_sin, out,
                q_absorbed=q_absorbed)
    return out


def batched_fused_mla_forward(kv_cache, q_absorbed, q_rope, W_UV, rope_cos, rope_sin,
                              d_model, kv_lora_rank, qk_nope_head_dim, qk_rope_head_dim, num_heads,
                              v_head_dim):
    """B query tokens over one shared cache (csrc/bindings.cpp:188-244). Returns (B, H, dv) fp32."""
    _check_half(kv_cache, "kv_cache")
    _check_f32(q_absorbed, "q_absorbed")
    _check_f32(q_rope, "q_rope")
    _check_half(W_UV, "W_UV")
    _check_f32(rope_cos, "rope_cos")
    _check_f32(rope_sin, "rope_sin")
    cfg = _cfg(d_model, kv_lora_rank, qk_nope_head_dim, qk_rope_head_dim, num_heads, v_head_dim)
    if q_absorbed.dim() != 3:
        raise RuntimeError("q_absorbed must be 3D (batch, num_heads, kv_lora_rank)")
    if q_rope.dim() != 3:
        raise RuntimeError("q_rope must be 3D (batch, num_heads, qk_rope_head_dim)")
    batch = q_absorbed.size(0)
    seq_len = kv_cache.size(0)
    if batch <= 0:
        raise RuntimeError(f"batch_size must be positive, got {batch}")
    if q_rope.size(0) != batch:
        raise RuntimeError(f"q_rope batch dim must match q_absorbed batch dim: {q_rope.size(0)} vs {batch}")
    if q_absorbed.size(1) != num_heads or q_absorbed.size(2) != kv_lora_rank:
        raise RuntimeError(
            f"q_absorbed shape mismatch: expected ({batch}, {num_heads}, {kv_lora_rank}) got "
            f"({q_absorbed.size(0)}, {q_absorbed.size(1)}, {q_absorbed.size(2)})")
    if q_rope.size(1) != num_heads or q_rope.size(2) != qk_rope_head_dim:
        raise RuntimeError("q_rope shape mismatch")
    if kv_cache.dim() != 2 or kv_cache.size(1) != kv_lora_rank + qk_rope_head_dim:
        raise RuntimeError("kv_cache dim1 mismatch")
    _check_common(kv_cache, W_UV, rope_cos, rope_sin, seq_len, num_heads, v_head_dim, kv_lora_rank,
                  qk_rope_head_dim)
    out = torch.empty(batch, num_heads, v_head_dim, dtype=torch.float32, device=kv_cache.device)
    if seq_len == 0:
        return out.zero_()
    _run_decode(cfg, kv_cache.dtype, batch, True, kv_cache, seq_len, q_rope, W_UV, rope_cos, rope_sin,
                out, q_absorbed=q_absorbed)
    return out


def naive_mla_forward(kv_cache, W_UK, W_UV, q_nope, q_rope, rope_cos, rope_sin,
                      d_model, kv_lora_rank, qk_nope_head_dim, qk_rope_head_dim, num_heads, v_head_dim):
    """Decompress-then-attend baseline (csrc/bindings.cpp:53-114, src/naive_mla.cu:58-246).

    This is the comparison baseline the fused path exists to beat, not part of the
    accelerated path: it materialises K_nope = c @ W_UK^T and V = c @ W_UV^T with
    plain library GEMMs and attends with fp32 torch ops, with the reference's
    output-layout error (its cuBLAS outputs are read transposed) corrected.
    Returns (H, dv) fp32.
    """
    _check_half(kv_cache, "kv_cache")
    _check_half(W_UK, "W_UK")
    _check_half(W_UV, "W_UV")
    _check_f32(q_nope, "q_nope")
    _check_f32(q_rope, "q_rope")
    _check_f32(rope_cos, "rope_cos")
    _check_f32(rope_sin, "rope_sin")
    _cfg(d_model, kv_lora_rank, qk_nope_head_dim, qk_rope_head_dim, num_heads, v_head_dim)
    S = kv_cache.size(0)
    dc, dR, H, dn, dv = kv_lora_rank, qk_rope_head_dim, num_heads, qk_nope_head_dim, v_head_dim
    if kv_cache.size(1) != dc + dR:
        raise RuntimeError(f"kv_cache dim1 must be {dc + dR}")
    if q_nope.size(0) != H or q_nope.size(1) != dn:
        raise RuntimeError("q_nope shape mismatch")
    if q_rope.size(0) != H or q_rope.size(1) != dR:
        raise RuntimeError("q_rope shape mismatch")
    c = kv_cache[:, :dc]
    K_nope = torch.matmul(c, W_UK.t()).float().view(S, H, dn)
    V = torch.matmul(c, W_UV.t()).float().view(S, H, dv)
    kr = kv_cache[:, dc:].float()
    half = dR // 2
    k0, k1 = kr[:, :half], kr[:, half:]
    K_rope = torch.cat([k0 * rope_cos[:S] - k1 * rope_sin[:S], k0 * rope_sin[:S] + k1 * rope_cos[:S]], dim=-1)
    scale = 1.0 / math.sqrt(dn + dR)
    s = torch.einsum("hd,shd->hs", q_nope, K_nope) * scale + (q_rope @ K_rope.t()) * scale
    p = torch.softmax(s, dim=-1)
    return torch.einsum("hs,shv->hv", p, V).contiguous()


def _check_tables(rope_cos, rope_sin):
    """Both RoPE tables (fp32, contiguous, CUDA), or neither (on-the-fly RoPE)."""
    if (rope_cos is None) != (rope_sin is None):
        raise RuntimeError("give both rope_cos and rope_sin, or neither (on-the-fly RoPE)")
    if rope_cos is not None:
        _check_f32(rope_cos, "rope_cos")
        _check_f32(rope_sin, "rope_sin")


def _check_common(kv_cache, W_UV, rope_cos, rope_sin, seq_len, H, dv, dc, dR):
    if W_UV.dtype != kv_cache.dtype:
        raise RuntimeError(f"W_UV dtype {W_UV.dtype} must match kv_cache dtype {kv_cache.dtype}")
    if W_UV.dim() != 2 or W_UV.size(0) != H * dv or W_UV.size(1) != dc:
        raise RuntimeError("W_UV shape mismatch")
    for t, n in ((rope_cos, "rope_cos"), (rope_sin, "rope_sin")):
        if t.dim() != 2 or t.size(1) != dR // 2 or t.size(0) < seq_len:
            raise RuntimeError(f"{n} shape mismatch: expected (>= {seq_len}, {dR // 2})")
    if kv_cache.data_ptr() % 16 != 0:
        raise RuntimeError("kv_cache must be 16-byte aligned")


def _run_decode(cfg, dtype, batch, shared, kv_cache, max_seq_len, q_rope, W_UV, rope_cos, rope_sin, out,
                workspace=None, **kw):
    args = _decode_args(dtype, batch, shared, kv_cache, max_seq_len, q_rope, W_UV, rope_cos, rope_sin, out,
                        **kw)
    lib = _lib.load()
    stream = C.c_void_p(_stream(kv_cache.device))
    if workspace is not None and workspace.data_ptr() % 256 == 0:
        # a caller's workspace is tried as it is: the call itself checks its size, and only a
        # too-small one costs the size query and an allocation
        st = lib.mla_decode(C.byref(cfg), C.byref(args), C.c_void_p(workspace.data_ptr()),
                            C.c_size_t(workspace.numel() * workspace.element_size()), stream)
        if st != _lib.MLA_ERR_WORKSPACE:
            _lib.check(st)
            return workspace
    ws = _workspace(cfg, args, kv_cache.device, workspace)
    _lib.check(lib.mla_decode(C.byref(cfg), C.byref(args), C.c_void_p(ws.data_ptr()),
                              C.c_size_t(ws.numel() * ws.element_size()), stream))
    return ws


# ---------------------------------------------------------------------------
# general decode (no reference counterpart)
# ---------------------------------------------------------------------------

def mla_decode(kv_cache: torch.Tensor, q_rope: torch.Tensor, W_UV: torch.Tensor,
               rope_cos: Optional[torch.Tensor], rope_sin: Optional[torch.Tensor], d_model: int,
               kv_lora_rank: int, qk_nope_head_dim: int,
               qk_rope_head_dim: int, num_heads: int, v_head_dim: int, *,
               q_absorbed: Optional[torch.Tensor] = None, q_nope: Optional[torch.Tensor] = None,
               W_UK: Optional[torch.Tensor] = None, seq_lens: Optional[torch.Tensor] = None,
               kv_offsets: Optional[torch.Tensor] = None, max_seq_len: Optional[int] = None,
               seq_lens_host: Optional[Sequence[int]] = None, shared_cache: bool = False,
               kv_pos_offset: int = 0, softmax_scale: float = 0.0, kv_row_stride: int = 0,
               kernel: int = 0, out: Optional[torch.Tensor] = None,
               workspace: Optional[torch.Tensor] = None, timer=None,
               page_table: Optional[torch.Tensor] = None, page_rows: int = 0,
               rope_theta: float = 0.0) -> torch.Tensor:
    """General decode: (B, H, dv) fp32 for B sequences (or B tokens over one shared cache).

    Give ``q_absorbed`` (B, H, d_c) fp32, or ``q_nope`` (B, H, dn) fp32 with ``W_UK``
    (H*dn, d_c) for in-op absorption. The queries and ``out`` may be pinned host tensors: the
    kernels then read the queries and store the output over the host link themselves, with no
    copy launches (for small batches, where a copy's fixed latency exceeds the transfer). ``seq_lens`` (B,) int32 and ``kv_offsets`` (B,)
    int64 (device) describe a variable-length batch packed in ``kv_cache``; without
    them every sequence has ``max_seq_len`` rows at ``b * max_seq_len``. With ``page_table``
    (B, max_pages) int32 (device) the cache is paged: position p of sequence b is row
    ``page_table[b, p // page_rows] * page_rows + p % page_rows`` (``page_rows`` a multiple of 64).
    With ``rope_cos`` and ``rope_sin`` both ``None`` the kernels compute the RoPE rotation
    themselves from ``rope_theta`` (0: 10000), as the reference's table builder defines it,
    and read no table.
    """
    if kv_row_stride:
        if kv_cache.dtype not in _DT or not kv_cache.is_cuda or kv_cache.stride(-1) != 1:
            raise RuntimeError("kv_cache must be a CUDA fp16/bf16 tensor with unit inner stride")
    else:
        _check_half(kv_cache, "kv_cache")
    _check_half(W_UV, "W_UV")
    _check_f32_io(q_rope, "q_rope")
    _check_tables(rope_cos, rope_sin)
    cfg = _cfg(d_model, kv_lora_rank, qk_nope_head_dim, qk_rope_head_dim, num_heads, v_head_dim)
    if q_absorbed is not None:
        _check_f32_io(q_absorbed, "q_absorbed")
        q_nope = None
        W_UK = None
    else:
        if q_nope is None or W_UK is None:
            raise RuntimeError("give q_absorbed, or q_nope together with W_UK")
        _check_f32_io(q_nope, "q_nope")
        _check_half(W_UK, "W_UK")
        if W_UK.dtype != kv_cache.dtype:
            raise RuntimeError("W_UK dtype must match kv_cache dtype")
    if q_rope.dim() != 3:
        raise RuntimeError("q_rope must be 3D (batch, num_heads, qk_rope_head_dim)")
    B = q_rope.size(0)
    if max_seq_len is None:
        if seq_lens_host is not None:
            max_seq_len = max(int(x) for x in seq_lens_host)
        elif seq_lens is None:
            max_seq_len = kv_cache.size(0) if shared_cache else kv_cache.size(0) // B
        else:
            raise RuntimeError("max_seq_len is required with device seq_lens")
    if seq_lens is not None:
        if seq_lens.dtype != torch.int32 or not seq_lens.is_cuda or seq_lens.numel() != B:
            raise RuntimeError("seq_lens must be a CUDA int32 tensor of shape (batch,)")
    if kv_offsets is not None:
        if kv_offsets.dtype != torch.int64 or not kv_offsets.is_cuda or kv_offsets.numel() != B:
            raise RuntimeError("kv_offsets must be a CUDA int64 tensor of shape (batch,)")
    if page_table is not None:
        if page_table.dtype != torch.int32 or not page_table.is_cuda or page_table.dim() != 2 \
                or page_table.size(0) != B or not page_table.is_contiguous():
            raise RuntimeError("page_table must be a contiguous CUDA int32 tensor of shape (batch, max_pages)")
    host_arr = None
    if seq_lens_host is not None:
        host_arr = (C.c_int * B)(*[int(x) for x in seq_lens_host])
    if out is None:
        out = torch.empty(B, num_heads, v_head_dim, dtype=torch.float32, device=kv_cache.device)
    else:
        _check_f32_io(out, "out")
        if out.numel() != B * num_heads * v_head_dim:
            raise RuntimeError(f"out must hold ({B}, {num_heads}, {v_head_dim}) floats")
    _run_decode(cfg, kv_cache.dtype, B, shared_cache, kv_cache, max_seq_len, q_rope, W_UV, rope_cos,
                rope_sin, out, workspace=workspace, q_absorbed=q_absorbed, q_nope=q_nope, W_UK=W_UK,
                seq_lens=seq_lens, kv_offsets=kv_offsets, seq_lens_host=host_arr,
                kv_pos_offset=kv_pos_offset, softmax_scale=softmax_scale, kv_row_stride=kv_row_stride,
                kernel=kernel, timer=timer, page_table=page_table, page_rows=page_rows, rope_theta=rope_theta)
    return out


def mla_decode_partial(kv_cache, q_rope, W_UV, rope_cos, rope_sin, d_model, kv_lora_rank,
                       qk_nope_head_dim, qk_rope_head_dim, num_heads, v_head_dim, *,
                       q_absorbed=None, q_nope=None, W_UK=None, kv_pos_offset: int = 0,
                       softmax_scale: float = 0.0, workspace=None, kernel: int = 0, timer=None,
                       rope_theta: float = 0.0):
    """One KV-range shard of a single-token-per-sequence decode over all rows of
    ``kv_cache`` (B sequences of ``kv_cache.size(0) // B`` rows). Returns
    (ml (B, H, 2), o (B, H, d_c)): natural-log max, sum of exponentials, and the
    unnormalised latent sum, ready for ``mla_combine_partials``. ``rope_cos`` / ``rope_sin``
    ``None``: on-the-fly RoPE from ``rope_theta``."""
    _check_half(kv_cache, "kv_cache")
    _check_tables(rope_cos, rope_sin)
    cfg = _cfg(d_model, kv_lora_rank, qk_nope_head_dim, qk_rope_head_dim, num_heads, v_head_dim)
    B = q_rope.size(0)
    L = kv_cache.size(0) // B
    ml = torch.empty(B, num_heads, 2, dtype=torch.float32, device=kv_cache.device)
    o = torch.empty(B, num_heads, kv_lora_rank, dtype=torch.float32, device=kv_cache.device)
    args = _decode_args(kv_cache.dtype, B, False, kv_cache, L, q_rope, W_UV, rope_cos, rope_sin, None,
                        q_absorbed=q_absorbed, q_nope=None if q_absorbed is not None else q_nope,
                        W_UK=None if q_absorbed is not None else W_UK, kv_pos_offset=kv_pos_offset,
                        softmax_scale=softmax_scale, kernel=kernel, timer=timer, rope_theta=rope_theta)
    ws = _workspace(cfg, args, kv_cache.device, workspace)
    lib = _lib.load()
    _lib.check(lib.mla_decode_partial(C.byref(cfg), C.byref(args), C.c_void_p(ml.data_ptr()),
                                      C.c_void_p(o.data_ptr()), C.c_void_p(ws.data_ptr()),
                                      C.c_size_t(ws.numel()), C.c_void_p(_stream(kv_cache.device))))
    return ml, o


def mla_decode_partial_packed(kv_cache, q_rope, W_UV, rope_cos, rope_sin, d_model, kv_lora_rank,
                              qk_nope_head_dim, qk_rope_head_dim, num_heads, v_head_dim, *, num_slices: int,
                              q_absorbed=None, q_nope=None, W_UK=None, kv_pos_offset: int = 0,
                              softmax_scale: float = 0.0, workspace=None, kernel: int = 0, timer=None,
                              rope_theta: float = 0.0, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``mla_decode_partial`` with the partials packed for a head-sliced exchange: returns
    (num_slices, B, H / num_slices, d_c + 4) fp32 rows [m, l, 0, 0, o] (m in natural-log
    units), slice q holding heads [q H / num_slices, (q + 1) H / num_slices)."""
    _check_half(kv_cache, "kv_cache")
    _check_tables(rope_cos, rope_sin)
    cfg = _cfg(d_model, kv_lora_rank, qk_nope_head_dim, qk_rope_head_dim, num_heads, v_head_dim)
    B = q_rope.size(0)
    L = kv_cache.size(0) // B
    if num_slices <= 0 or num_heads % num_slices:
        raise RuntimeError(f"num_slices ({num_slices}) must divide num_heads ({num_heads})")
    shape = (num_slices, B, num_heads // num_slices, kv_lora_rank + 4)
    if out is None:
        out = torch.empty(shape, dtype=torch.float32, device=kv_cache.device)
    elif tuple(out.shape) != shape or out.dtype != torch.float32 or not out.is_contiguous():
        raise RuntimeError(f"out must be a contiguous float32 tensor of shape {shape}")
    args = _decode_args(kv_cache.dtype, B, False, kv_cache, L, q_rope, W_UV, rope_cos, rope_sin, None,
                        q_absorbed=q_absorbed, q_nope=None if q_absorbed is not None else q_nope,
                        W_UK=None if q_absorbed is not None else W_UK, kv_pos_offset=kv_pos_offset,
                        softmax_scale=softmax_scale, kernel=kernel, timer=timer, rope_theta=rope_theta)
    ws = _workspace(cfg, args, kv_cache.device, workspace)
    _lib.check(_lib.load().mla_decode_partial_packed(C.byref(cfg), C.byref(args), int(num_slices),
                                                     C.c_void_p(out.data_ptr()), C.c_void_p(ws.data_ptr()),
                                                     C.c_size_t(ws.numel()), C.c_void_p(_stream(kv_cache.device))))
    return out


def mla_combine_partials_packed(packed: torch.Tensor, W_UV_slice: torch.Tensor, d_model, kv_lora_rank,
                                qk_nope_head_dim, qk_rope_head_dim, num_heads, v_head_dim,
                                out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Merge packed partial sets (P, B, heads, d_c + 4) of one head slice and project with that
    slice's W_UV rows (heads * dv, d_c) -> (B, heads, dv) fp32."""
    _check_f32(packed, "packed")
    _check_half(W_UV_slice, "W_UV_slice")
    cfg = _cfg(d_model, kv_lora_rank, qk_nope_head_dim, qk_rope_head_dim, num_heads, v_head_dim)
    if packed.dim() != 4 or packed.size(3) != kv_lora_rank + 4:
        raise RuntimeError("packed must be (parts, batch, heads, kv_lora_rank + 4)")
    P, B, heads = packed.size(0), packed.size(1), packed.size(2)
    if W_UV_slice.dim() != 2 or W_UV_slice.size(0) != heads * v_head_dim or W_UV_slice.size(1) != kv_lora_rank:
        raise RuntimeError("W_UV_slice must be (heads * v_head_dim, kv_lora_rank)")
    if out is None:
        out = torch.empty(B, heads, v_head_dim, dtype=torch.float32, device=packed.device)
    _lib.check(_lib.load().mla_combine_partials_packed(C.byref(cfg), _DT[W_UV_slice.dtype], B, P, heads,
                                                       C.c_void_p(packed.data_ptr()), C.c_void_p(W_UV_slice.data_ptr()),
                                                       C.c_void_p(out.data_ptr()), C.c_void_p(_stream(packed.device))))
    return out


def mla_decode_partial_put(kv_cache, q_rope, W_UV, rope_cos, rope_sin, d_model, kv_lora_rank, qk_nope_head_dim,
                           qk_rope_head_dim, num_heads, v_head_dim, *, dst_ptrs: torch.Tensor, dst_offset: int,
                           signal: "PeerSignal", q_absorbed=None, q_nope=None, W_UK=None, kv_pos_offset: int = 0,
                           softmax_scale: float = 0.0, workspace=None, kernel: int = 0, timer=None,
                           rope_theta: float = 0.0) -> None:
    """``mla_decode_partial_packed`` whose slice q lands in rank q's buffer
    (``dst_ptrs[q] + dst_offset``), written by the export kernel itself, and rank q is signalled
    (``signal``). world = ``dst_ptrs.numel()`` divides the heads."""
    _check_half(kv_cache, "kv_cache")
    _check_tables(rope_cos, rope_sin)
    if dst_ptrs.dtype != torch.int64 or not dst_ptrs.is_cuda or dst_ptrs.dim() != 1:
        raise RuntimeError("dst_ptrs must be a CUDA int64 vector of pointers")
    world = int(dst_ptrs.numel())
    if world != signal.world:
        raise RuntimeError("dst_ptrs and the signal's flag pointers must have one entry per rank")
    cfg = _cfg(d_model, kv_lora_rank, qk_nope_head_dim, qk_rope_head_dim, num_heads, v_head_dim)
    B = q_rope.size(0)
    L = kv_cache.size(0) // B
    args = _decode_args(kv_cache.dtype, B, False, kv_cache, L, q_rope, W_UV, rope_cos, rope_sin, None,
                        q_absorbed=q_absorbed, q_nope=None if q_absorbed is not None else q_nope,
                        W_UK=None if q_absorbed is not None else W_UK, kv_pos_offset=kv_pos_offset,
                        softmax_scale=softmax_scale, kernel=kernel, timer=timer, rope_theta=rope_theta)
    ws = _workspace(cfg, args, kv_cache.device, workspace)
    _lib.check(_lib.load().mla_decode_partial_put(C.byref(cfg), C.byref(args), world, C.c_void_p(dst_ptrs.data_ptr()),
                                                  C.c_size_t(dst_offset), C.byref(signal.struct),
                                                  C.c_void_p(ws.data_ptr()), C.c_size_t(ws.numel()),
                                                  C.c_void_p(_stream(kv_cache.device))))


def mla_combine_partials_put(packed: torch.Tensor, W_UV_slice: torch.Tensor, d_model, kv_lora_rank,
                             qk_nope_head_dim, qk_rope_head_dim, num_heads, v_head_dim, *, dst_ptrs: torch.Tensor,
                             dst_offset: int, dst_pitch: int, signal: "PeerSignal", scratch: torch.Tensor) -> None:
    """``mla_combine_partials_packed`` whose (B, heads, dv) output lands in every rank's buffer:
    token b's rows at ``dst_ptrs[q] + dst_offset + b * dst_pitch``; every rank is signalled.
    ``scratch``: (B, heads, dv) fp32 of this rank (staging for batches the GEMV kernel does not
    take)."""
    _check_f32(packed, "packed")
    _check_half(W_UV_slice, "W_UV_slice")
    _check_f32(scratch, "scratch")
    cfg = _cfg(d_model, kv_lora_rank, qk_nope_head_dim, qk_rope_head_dim, num_heads, v_head_dim)
    if packed.dim() != 4 or packed.size(3) != kv_lora_rank + 4:
        raise RuntimeError("packed must be (parts, batch, heads, kv_lora_rank + 4)")
    P, B, heads = packed.size(0), packed.size(1), packed.size(2)
    if W_UV_slice.dim() != 2 or W_UV_slice.size(0) != heads * v_head_dim or W_UV_slice.size(1) != kv_lora_rank:
        raise RuntimeError("W_UV_slice must be (heads * v_head_dim, kv_lora_rank)")
    if scratch.numel() < B * heads * v_head_dim:
        raise RuntimeError("scratch must hold batch * heads * v_head_dim floats")
    if dst_ptrs.dtype != torch.int64 or not dst_ptrs.is_cuda or dst_ptrs.dim() != 1:
        raise RuntimeError("dst_ptrs must be a CUDA int64 vector of pointers")
    if dst_ptrs.numel() != signal.world:
        raise RuntimeError("dst_ptrs and the signal's flag pointers must have one entry per rank")
    _lib.check(_lib.load().mla_combine_partials_put(
        C.byref(cfg), _DT[W_UV_slice.dtype], B, P, heads, C.c_void_p(packed.data_ptr()),
        C.c_void_p(W_UV_slice.data_ptr()), int(dst_ptrs.numel()), C.c_void_p(dst_ptrs.data_ptr()),
        C.c_size_t(dst_offset), C.c_size_t(dst_pitch), C.byref(signal.struct), C.c_void_p(scratch.data_ptr()),
        C.c_void_p(_stream(packed.device))))


def mla_decode_kv_range(kv_cache, q_rope, W_UV, rope_cos, rope_sin, d_model, kv_lora_rank, qk_nope_head_dim,
                        qk_rope_head_dim, num_heads, v_head_dim, *, world: int, rank: int, recv_ptrs: torch.Tensor,
                        half_bytes: int, epoch: torch.Tensor, counter: torch.Tensor, status: torch.Tensor,
                        out: torch.Tensor, q_absorbed=None, q_nope=None, W_UK=None, kv_pos_offset: int = 0,
                        softmax_scale: float = 0.0, workspace=None, kernel: int = 0, timer=None,
                        rope_theta: float = 0.0) -> torch.Tensor:
    """``mla_decode_kv_range``: this rank's KV-range step for batch 1 .. 4 with the exchange of per-head
    partials inside one kernel (stores into every rank's receive area ``recv_ptrs[q]``, two halves of
    ``half_bytes``), every rank merging and projecting all heads into ``out`` (B, H, dv)."""
    _check_half(kv_cache, "kv_cache")
    _check_tables(rope_cos, rope_sin)
    _check_f32(out, "out")
    if recv_ptrs.dtype != torch.int64 or not recv_ptrs.is_cuda or recv_ptrs.numel() != world:
        raise RuntimeError("recv_ptrs must be a CUDA int64 vector of world pointers")
    for t, name in ((epoch, "epoch"), (counter, "counter"), (status, "status")):
        if t.dtype != torch.int32 or not t.is_cuda:
            raise RuntimeError(f"{name} must be a CUDA int32 tensor")
    cfg = _cfg(d_model, kv_lora_rank, qk_nope_head_dim, qk_rope_head_dim, num_heads, v_head_dim)
    B = q_rope.size(0)
    L = kv_cache.size(0) // B
    args = _decode_args(kv_cache.dtype, B, False, kv_cache, L, q_rope, W_UV, rope_cos, rope_sin, out,
                        q_absorbed=q_absorbed, q_nope=None if q_absorbed is not None else q_nope,
                        W_UK=None if q_absorbed is not None else W_UK, kv_pos_offset=kv_pos_offset,
                        softmax_scale=softmax_scale, kernel=kernel, timer=timer, rope_theta=rope_theta)
    ws = _workspace(cfg, args, kv_cache.device, workspace)
    _lib.check(_lib.load().mla_decode_kv_range(
        C.byref(cfg), C.byref(args), int(world), int(rank), C.c_void_p(recv_ptrs.data_ptr()), C.c_size_t(half_bytes),
        C.c_void_p(epoch.data_ptr()), C.c_void_p(counter.data_ptr()), C.c_void_p(status.data_ptr()),
        C.c_void_p(ws.data_ptr()), C.c_size_t(ws.numel()), C.c_void_p(_stream(kv_cache.device))))
    return out


def mla_decode_partial_gather(kv_cache, q_rope, W_UV, rope_cos, rope_sin, d_model, kv_lora_rank, qk_nope_head_dim,
                              qk_rope_head_dim, num_heads, v_head_dim, *, dst_ptrs: torch.Tensor, dst_offset: int,
                              parity_bytes: int, signal: "PeerSignal", q_absorbed=None, q_nope=None, W_UK=None,
                              kv_pos_offset: int = 0, softmax_scale: float = 0.0, workspace=None, kernel: int = 0,
                              timer=None, rope_theta: float = 0.0) -> None:
    """The gathered export (batch 1 .. 4): this rank's (B, H) packed partial rows land in every
    rank's buffer at ``dst_ptrs[q] + dst_offset + ((epoch + 1) & 1) * parity_bytes``, written by
    the export kernel itself; every rank is signalled."""
    _check_half(kv_cache, "kv_cache")
    _check_tables(rope_cos, rope_sin)
    if dst_ptrs.dtype != torch.int64 or not dst_ptrs.is_cuda or dst_ptrs.dim() != 1:
        raise RuntimeError("dst_ptrs must be a CUDA int64 vector of pointers")
    if dst_ptrs.numel() != signal.world:
        raise RuntimeError("dst_ptrs and the signal's flag pointers must have one entry per rank")
    cfg = _cfg(d_model, kv_lora_rank, qk_nope_head_dim, qk_rope_head_dim, num_heads, v_head_dim)
    B = q_rope.size(0)
    L = kv_cache.size(0) // B
    args = _decode_args(kv_cache.dtype, B, False, kv_cache, L, q_rope, W_UV, rope_cos, rope_sin, None,
                        q_absorbed=q_absorbed, q_nope=None if q_absorbed is not None else q_nope,
                        W_UK=None if q_absorbed is not None else W_UK, kv_pos_offset=kv_pos_offset,
                        softmax_scale=softmax_scale, kernel=kernel, timer=timer, rope_theta=rope_theta)
    ws = _workspace(cfg, args, kv_cache.device, workspace)
    _lib.check(_lib.load().mla_decode_partial_gather(
        C.byref(cfg), C.byref(args), int(dst_ptrs.numel()), C.c_void_p(dst_ptrs.data_ptr()), C.c_size_t(dst_offset),
        C.c_size_t(parity_bytes), C.byref(signal.struct), C.c_void_p(ws.data_ptr()), C.c_size_t(ws.numel()),
        C.c_void_p(_stream(kv_cache.device))))


def mla_combine_partials_gathered(packed: torch.Tensor, parity_bytes: int, epoch: torch.Tensor, W_UV: torch.Tensor,
                                  d_model, kv_lora_rank, qk_nope_head_dim, qk_rope_head_dim, num_heads, v_head_dim,
                                  *, parts: int, batch: int, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Merge the gathered sets (parts, batch, H, d_c + 4) at ``packed`` + ``(epoch & 1) *
    parity_bytes`` and project with W_UV -> (batch, H, dv) fp32."""
    _check_f32(packed, "packed")
    _check_half(W_UV, "W_UV")
    if epoch.dtype != torch.int32 or not epoch.is_cuda:
        raise RuntimeError("epoch must be a CUDA int32 tensor")
    need = (parity_bytes + parts * batch * num_heads * (kv_lora_rank + 4) * 4) // 4
    if packed.numel() < need:
        raise RuntimeError("packed is smaller than two halves of the gathered sets")
    cfg = _cfg(d_model, kv_lora_rank, qk_nope_head_dim, qk_rope_head_dim, num_heads, v_head_dim)
    if out is None:
        out = torch.empty(batch, num_heads, v_head_dim, dtype=torch.float32, device=packed.device)
    elif tuple(out.shape) != (batch, num_heads, v_head_dim) or out.dtype != torch.float32 or not out.is_contiguous():
        raise RuntimeError(f"out must be a contiguous float32 tensor of shape ({batch}, {num_heads}, {v_head_dim})")
    _lib.check(_lib.load().mla_combine_partials_gathered(
        C.byref(cfg), _DT[W_UV.dtype], int(batch), int(parts), C.c_void_p(packed.data_ptr()), C.c_size_t(parity_bytes),
        C.c_void_p(epoch.data_ptr()), C.c_void_p(W_UV.data_ptr()), C.c_void_p(out.data_ptr()),
        C.c_void_p(_stream(packed.device))))
    return out


def mla_combine_partials(part_ml: torch.Tensor, part_o: torch.Tensor, W_UV: torch.Tensor, d_model,
                         kv_lora_rank, qk_nope_head_dim, qk_rope_head_dim, num_heads, v_head_dim,
                         out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Merge ``P`` shards' partials (P, B, H, 2) / (P, B, H, d_c) and project with W_UV -> (B, H, dv)."""
    _check_f32(part_ml, "part_ml")
    _check_f32(part_o, "part_o")
    _check_half(W_UV, "W_UV")
    cfg = _cfg(d_model, kv_lora_rank, qk_nope_head_dim, qk_rope_head_dim, num_heads, v_head_dim)
    P, B = part_ml.size(0), part_ml.size(1)
    if out is None:
        out = torch.empty(B, num_heads, v_head_dim, dtype=torch.float32, device=part_ml.device)
    lib = _lib.load()
    _lib.check(lib.mla_combine_partials(C.byref(cfg), _DT[W_UV.dtype], B, P, C.c_void_p(part_ml.data_ptr()),
                                        C.c_void_p(part_o.data_ptr()), C.c_void_p(W_UV.data_ptr()),
                                        C.c_void_p(out.data_ptr()), C.c_void_p(_stream(part_ml.device))))
    return out


def linear(x: torch.Tensor, W: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``x (M, K) @ W (N, K)^T`` -> (M, N) fp32 on the tcgen05 projection kernel (``mla_linear``):
    x and W fp16 or bf16 of the same dtype, contiguous, 1 <= M <= 256."""
    _check_half(x, "x")
    _check_half(W, "W")
    if x.dtype != W.dtype:
        raise RuntimeError("x and W must have the same dtype")
    if x.dim() != 2 or W.dim() != 2 or x.size(1) != W.size(1):
        raise RuntimeError(f"shape mismatch: x {tuple(x.shape)}, W {tuple(W.shape)}")
    M, K = x.shape
    N = W.size(0)
    if out is None:
        out = torch.empty(M, N, dtype=torch.float32, device=x.device)
    elif tuple(out.shape) != (M, N) or out.dtype != torch.float32 or not out.is_contiguous():
        raise RuntimeError(f"out must be a contiguous float32 tensor of shape ({M}, {N})")
    _lib.check(_lib.load().mla_linear(_DT[x.dtype], M, N, K, C.c_void_p(x.data_ptr()), C.c_void_p(W.data_ptr()),
                                      C.c_void_p(out.data_ptr()), C.c_void_p(_stream(x.device))))
    return out


def mla_cache_append(kv_cache: torch.Tensor, c_t: torch.Tensor, k_rope: torch.Tensor, seq_lens: torch.Tensor,
                     max_seq_len: int, d_model, kv_lora_rank, qk_nope_head_dim, qk_rope_head_dim, num_heads,
                     v_head_dim, *, kv_offsets: Optional[torch.Tensor] = None,
                     page_table: Optional[torch.Tensor] = None, page_rows: int = 0,
                     status: Optional[torch.Tensor] = None) -> None:
    """Append one row per sequence on the device: the row of position ``seq_lens[b]`` (at
    ``kv_offsets[b]`` or ``b * max_seq_len`` plus the position, or through ``page_table`` (B,
    max_pages) int32 with ``page_rows`` rows a page) receives ``[c_t[b] | k_rope[b]]`` (k_rope
    unrotated) and ``seq_lens[b]`` advances by one; nothing waits for the device. ``c_t`` (B, d_c)
    and ``k_rope`` (B, d_R) have the cache's dtype. A full sequence (``max_seq_len`` rows) is left
    unchanged and sets bit 0 of ``status`` (a CUDA int32 tensor), if given; a page outside the
    cache sets bit 1."""
    if kv_cache.dtype not in _DT or not kv_cache.is_cuda or kv_cache.stride(-1) != 1:
        raise RuntimeError("kv_cache must be a CUDA fp16/bf16 tensor with unit inner stride")
    for t, name in ((c_t, "c_t"), (k_rope, "k_rope")):
        _check_half(t, name)
        if t.dtype != kv_cache.dtype:
            raise RuntimeError(f"{name} dtype must match kv_cache dtype")
    B = c_t.size(0)
    if tuple(c_t.shape) != (B, kv_lora_rank) or tuple(k_rope.shape) != (B, qk_rope_head_dim):
        raise RuntimeError("c_t must be (batch, kv_lora_rank) and k_rope (batch, qk_rope_head_dim)")
    if seq_lens.dtype != torch.int32 or not seq_lens.is_cuda or seq_lens.numel() != B:
        raise RuntimeError("seq_lens must be a CUDA int32 tensor of shape (batch,)")
    if kv_offsets is not None and (kv_offsets.dtype != torch.int64 or not kv_offsets.is_cuda or kv_offsets.numel() != B):
        raise RuntimeError("kv_offsets must be a CUDA int64 tensor of shape (batch,)")
    if status is not None and (status.dtype != torch.int32 or not status.is_cuda):
        raise RuntimeError("status must be a CUDA int32 tensor")
    if page_table is not None and (page_table.dtype != torch.int32 or not page_table.is_cuda
                                   or page_table.dim() != 2 or page_table.size(0) != B
                                   or not page_table.is_contiguous()):
        raise RuntimeError("page_table must be a contiguous CUDA int32 tensor of shape (batch, max_pages)")
    cfg = _cfg(d_model, kv_lora_rank, qk_nope_head_dim, qk_rope_head_dim, num_heads, v_head_dim)
    stride = kv_cache.stride(0) if kv_cache.dim() == 2 else 0
    lib = _lib.load()
    max_pages = int(page_table.size(1)) if page_table is not None else 0
    _lib.check(lib.mla_cache_append(C.byref(cfg), _DT[kv_cache.dtype], C.c_void_p(kv_cache.data_ptr()),
                                    C.c_int64(stride), C.c_int64(kv_cache.size(0)), B, C.c_void_p(c_t.data_ptr()),
                                    C.c_void_p(k_rope.data_ptr()), C.c_void_p(_ptr(kv_offsets)),
                                    C.c_void_p(_ptr(page_table)), int(page_rows), max_pages,
                                    C.c_void_p(seq_lens.data_ptr()), int(max_seq_len),
                                    C.c_void_p(_ptr(status)), C.c_void_p(_stream(kv_cache.device))))


# ---- peer memory for the multi-GPU exchange (mla_ipc_* / mla_peer_*)

class IpcBuffer:
    """A device allocation other processes of the node can map (``mla_ipc_alloc``), zero-filled.

    ``handle`` (bytes) goes to the peers, which map it with ``ipc_open``; ``view(dtype, count,
    offset)`` is a tensor over part of it. The tensors do not own the memory: keep this object
    alive while they are used, and ``free()`` it only after every peer has closed its mapping."""

    def __init__(self, nbytes: int, device: torch.device):
        self.nbytes, self.device = int(nbytes), device
        p = C.c_void_p()
        h = (C.c_char * _lib.IPC_HANDLE_BYTES)()
        with torch.cuda.device(device):
            _lib.check(_lib.load().mla_ipc_alloc(C.c_size_t(self.nbytes), C.byref(p), h))
        self.ptr, self.handle = int(p.value), bytes(h)

    def view(self, dtype: torch.dtype, count: int, offset: int = 0) -> torch.Tensor:
        item = torch.empty((), dtype=dtype).element_size()
        if offset % item or offset < 0 or offset + count * item > self.nbytes:
            raise ValueError("view outside the allocation")
        return _device_view(self.ptr + offset, dtype, count, self.device)

    def free(self) -> None:
        if self.ptr:
            with torch.cuda.device(self.device):
                _lib.check(_lib.load().mla_ipc_free(C.c_void_p(self.ptr)))
            self.ptr = 0


_TYPESTR = {torch.float32: "<f4", torch.int32: "<i4", torch.int64: "<i8", torch.uint8: "|u1"}


def _device_view(ptr: int, dtype: torch.dtype, count: int, device: torch.device) -> torch.Tensor:
    class _Iface:   # __cuda_array_interface__ v2 over a raw device pointer
        __cuda_array_interface__ = {"shape": (int(count),), "typestr": _TYPESTR[dtype], "data": (int(ptr), False),
                                    "version": 2, "strides": None}
    return torch.as_tensor(_Iface(), device=device)


def ipc_open(handle: bytes, device: torch.device) -> int:
    """Maps a peer's ``IpcBuffer`` (by its handle) into this process; returns the device pointer."""
    if len(handle) != _lib.IPC_HANDLE_BYTES:
        raise ValueError("bad IPC handle length")
    p = C.c_void_p()
    with torch.cuda.device(device):
        _lib.check(_lib.load().mla_ipc_open(C.c_char_p(handle), C.byref(p)))
    return int(p.value)


def ipc_close(ptr: int, device: torch.device) -> None:
    with torch.cuda.device(device):
        _lib.check(_lib.load().mla_ipc_close(C.c_void_p(ptr)))


class PeerSignal:
    """``mla_peer_signal_t``: how a kernel storing into other ranks' buffers flags them. Receiver
    q's word ``flag_index`` (of the int32 words ``flag_ptrs[q]`` points to) is set to ``epoch + 1``
    once the kernel's stores bound for q are done; ``counters`` are this rank's ``world`` zeroed
    int32 words the kernel's blocks count themselves in. All tensors on this rank's GPU."""

    def __init__(self, flag_ptrs: torch.Tensor, flag_index: int, epoch: torch.Tensor, counters: torch.Tensor):
        if flag_ptrs.dtype != torch.int64 or not flag_ptrs.is_cuda or flag_ptrs.dim() != 1:
            raise RuntimeError("flag_ptrs must be a CUDA int64 vector of pointers")
        if epoch.dtype != torch.int32 or not epoch.is_cuda:
            raise RuntimeError("epoch must be a CUDA int32 tensor")
        if counters.dtype != torch.int32 or not counters.is_cuda or counters.numel() < flag_ptrs.numel():
            raise RuntimeError("counters must be a CUDA int32 tensor with one word per rank")
        self.world = int(flag_ptrs.numel())
        self._keep = (flag_ptrs, epoch, counters)
        self.struct = _lib.MlaPeerSignal(flag_ptrs.data_ptr(), int(flag_index), epoch.data_ptr(), counters.data_ptr())


def peer_put(src: torch.Tensor, rows: int, row_bytes: int, src_pitch: int, src_stride: int, dst_ptrs: torch.Tensor,
             dst_pitch: int, dst_offset: int, blocks: int, signal: PeerSignal) -> None:
    """``mla_peer_put`` on the current stream: slice q of ``src`` (rows x row_bytes, rows
    ``src_pitch`` apart, slices ``src_stride`` apart) to ``dst_ptrs[q] + dst_offset`` (rows
    ``dst_pitch`` apart), ``blocks`` blocks a slice, then receiver q is signalled.
    ``dst_ptrs``: CUDA int64 tensor of world pointers."""
    if not src.is_cuda or not src.is_contiguous():
        raise RuntimeError("src must be a contiguous CUDA tensor")
    if dst_ptrs.dtype != torch.int64 or not dst_ptrs.is_cuda or dst_ptrs.dim() != 1:
        raise RuntimeError("dst_ptrs must be a CUDA int64 vector of pointers")
    if dst_ptrs.numel() != signal.world:
        raise RuntimeError("dst_ptrs and the signal's flag pointers must have one entry per rank")
    _lib.check(_lib.load().mla_peer_put(
        C.c_void_p(src.data_ptr()), C.c_size_t(rows), C.c_size_t(row_bytes), C.c_size_t(src_pitch),
        C.c_size_t(src_stride), C.c_void_p(dst_ptrs.data_ptr()), C.c_size_t(dst_pitch), C.c_size_t(dst_offset),
        int(dst_ptrs.numel()), int(blocks), C.byref(signal.struct), C.c_void_p(_stream(src.device))))


def peer_wait(flags: torch.Tensor, epoch: torch.Tensor, advance: bool, status: Optional[torch.Tensor]) -> None:
    """``mla_peer_wait`` on the current stream: waits (bounded, 2 s) until every word of the int32
    vector ``flags`` reaches ``epoch + 1``; ``advance`` then increments ``epoch``. A wait that
    gives up stores 1 to ``status``."""
    if flags.dtype != torch.int32 or not flags.is_cuda or not flags.is_contiguous():
        raise RuntimeError("flags must be a contiguous CUDA int32 tensor")
    if epoch.dtype != torch.int32 or not epoch.is_cuda:
        raise RuntimeError("epoch must be a CUDA int32 tensor")
    _lib.check(_lib.load().mla_peer_wait(C.c_void_p(flags.data_ptr()), int(flags.numel()),
                                         C.c_void_p(epoch.data_ptr()), 1 if advance else 0,
                                         C.c_void_p(_ptr(status)), C.c_void_p(_stream(flags.device))))
