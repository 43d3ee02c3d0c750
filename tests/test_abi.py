"""The C ABI surface, checked without a GPU: every declared entry point is
exported, the ctypes mirrors have the header's layout, argument validation
returns status codes (never aborts), and the C++ drop-in headers compile."""

import ctypes as C
import os
import re
import subprocess
import tempfile

import pytest

from latent_attn import _lib

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INC = os.path.join(REPO, "include")
HEADER = os.path.join(INC, "latent_attn_b200", "mla.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"MLA_API\s+[\w\s\*]+?\b(mla_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_symbols()
    assert len(names) >= 9, names
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (mla_\w+)", out))
    for n in names:
        assert n in exported, f"{n} declared in mla.h but not exported"
        assert hasattr(lib, n)
    assert set(_lib.SIGNATURES) == set(names), "ctypes signatures out of sync with mla.h"


def test_struct_layouts_match_header():
    src = r'''
#include <stdio.h>
#include <stddef.h>
#include "latent_attn_b200/mla.h"
#define P(T, f) printf(#T "." #f " %zu\n", offsetof(T, f));
int main(void) {
  printf("mla_config_t %zu\n", sizeof(mla_config_t));
  printf("mla_fused_params_t %zu\n", sizeof(mla_fused_params_t));
  printf("mla_batched_fused_params_t %zu\n", sizeof(mla_batched_fused_params_t));
  printf("mla_decode_args_t %zu\n", sizeof(mla_decode_args_t));
  P(mla_decode_args_t, kv_total_rows) P(mla_decode_args_t, seq_lens_host) P(mla_decode_args_t, softmax_scale)
  P(mla_decode_args_t, output) P(mla_decode_args_t, kernel) P(mla_fused_params_t, cfg)
  P(mla_batched_fused_params_t, output) P(mla_decode_args_t, page_table) P(mla_decode_args_t, max_pages)
  printf("mla_peer_signal_t %zu\n", sizeof(mla_peer_signal_t));
  P(mla_peer_signal_t, flag_index) P(mla_peer_signal_t, epoch) P(mla_peer_signal_t, counters)
  return 0;
}
'''
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "layout.c")
        exe = os.path.join(d, "layout")
        open(c, "w").write(src)
        subprocess.run(["gcc", "-std=c99", "-I", INC, c, "-o", exe], check=True)
        out = subprocess.run([exe], capture_output=True, text=True, check=True).stdout
    got = dict(line.rsplit(" ", 1) for line in out.strip().splitlines())
    want = {
        "mla_config_t": C.sizeof(_lib.MlaConfig),
        "mla_fused_params_t": C.sizeof(_lib.MlaFusedParams),
        "mla_batched_fused_params_t": C.sizeof(_lib.MlaBatchedFusedParams),
        "mla_decode_args_t": C.sizeof(_lib.MlaDecodeArgs),
        "mla_decode_args_t.kv_total_rows": _lib.MlaDecodeArgs.kv_total_rows.offset,
        "mla_decode_args_t.seq_lens_host": _lib.MlaDecodeArgs.seq_lens_host.offset,
        "mla_decode_args_t.softmax_scale": _lib.MlaDecodeArgs.softmax_scale.offset,
        "mla_decode_args_t.output": _lib.MlaDecodeArgs.output.offset,
        "mla_decode_args_t.kernel": _lib.MlaDecodeArgs.kernel.offset,
        "mla_fused_params_t.cfg": _lib.MlaFusedParams.cfg.offset,
        "mla_batched_fused_params_t.output": _lib.MlaBatchedFusedParams.output.offset,
        "mla_decode_args_t.page_table": _lib.MlaDecodeArgs.page_table.offset,
        "mla_decode_args_t.max_pages": _lib.MlaDecodeArgs.max_pages.offset,
        "mla_peer_signal_t": C.sizeof(_lib.MlaPeerSignal),
        "mla_peer_signal_t.flag_index": _lib.MlaPeerSignal.flag_index.offset,
        "mla_peer_signal_t.epoch": _lib.MlaPeerSignal.epoch.offset,
        "mla_peer_signal_t.counters": _lib.MlaPeerSignal.counters.offset,
    }
    for k, v in want.items():
        assert int(got[k]) == v, (k, got[k], v)


def test_validation_without_gpu():
    lib = _lib.load()
    ok = _lib.MlaConfig(5120, 512, 128, 64, 128, 128)
    assert lib.mla_config_validate(C.byref(ok)) == _lib.MLA_OK
    for bad in (_lib.MlaConfig(0, 0, 128, 64, 128, 128), _lib.MlaConfig(0, 512, 128, 64, 0, 128),
                _lib.MlaConfig(0, 512, 128, 64, 128, -1)):
        assert lib.mla_config_validate(C.byref(bad)) == _lib.MLA_ERR_INVALID_ARGUMENT
        assert b"positive" in lib.mla_last_error()
    assert lib.mla_config_validate(None) == _lib.MLA_ERR_INVALID_ARGUMENT
    # argument errors are reported before any device work
    a = _lib.MlaDecodeArgs()
    a.dtype, a.batch, a.max_seq_len = _lib.DTYPE_BF16, 1, 16
    n = C.c_size_t(0)
    st = lib.mla_decode_workspace_size(C.byref(ok), C.byref(a), C.byref(n))
    assert st == _lib.MLA_ERR_INVALID_ARGUMENT and b"null" in lib.mla_last_error()
    a.dtype = _lib.DTYPE_F32
    assert lib.mla_decode_workspace_size(C.byref(ok), C.byref(a), C.byref(n)) == _lib.MLA_ERR_UNSUPPORTED
    assert lib.mla_decode(C.byref(ok), None, None, 0, None) == _lib.MLA_ERR_INVALID_ARGUMENT
    p = _lib.MlaFusedParams()
    p.cfg = C.pointer(ok)
    assert lib.mla_launch_fused(C.byref(p), _lib.DTYPE_F16, None) == _lib.MLA_ERR_INVALID_ARGUMENT
    # cache append: null pointers, a bad batch and a bad dtype are rejected before any launch
    fake = C.c_void_p(256)
    def append(dtype=_lib.DTYPE_BF16, kv=fake, total=0, batch=1, pages=None, page_rows=0, max_pages=0):
        return lib.mla_cache_append(C.byref(ok), dtype, kv, 0, total, batch, fake, fake, None, pages, page_rows,
                                    max_pages, fake, 8, None, None)
    assert append(kv=None) == _lib.MLA_ERR_INVALID_ARGUMENT
    assert append(batch=0) == _lib.MLA_ERR_INVALID_ARGUMENT
    assert append(dtype=_lib.DTYPE_F32) == _lib.MLA_ERR_UNSUPPORTED
    assert append(pages=fake, page_rows=64, max_pages=1) == _lib.MLA_ERR_INVALID_ARGUMENT    # no kv_total_rows
    assert append(pages=fake, page_rows=4, max_pages=1, total=64) == _lib.MLA_ERR_INVALID_ARGUMENT  # 4 < 8 rows
    assert lib.mla_version().startswith(b"latent-attn-b200")


def test_peer_exchange_validation_without_gpu():
    """The peer-memory entry points reject bad arguments before any device work."""
    lib = _lib.load()
    ok = _lib.MlaConfig(5120, 512, 128, 64, 128, 128)
    fake = C.c_void_p(256)
    sig = _lib.MlaPeerSignal(256, 0, 256, 256)
    no_counters = _lib.MlaPeerSignal(256, 0, 256, None)
    bad_index = _lib.MlaPeerSignal(256, -1, 256, 256)
    put = lambda s, world=2, blocks=1, row=64, off=0: lib.mla_peer_put(fake, 1, row, row, row, fake, row, off, world,
                                                                       blocks, C.byref(s) if s else None, None)
    assert put(None) == _lib.MLA_ERR_INVALID_ARGUMENT and b"signal" in lib.mla_last_error()
    assert put(no_counters) == _lib.MLA_ERR_INVALID_ARGUMENT
    assert put(bad_index) == _lib.MLA_ERR_INVALID_ARGUMENT
    assert put(sig, world=0) == _lib.MLA_ERR_INVALID_ARGUMENT
    assert put(sig, blocks=0) == _lib.MLA_ERR_INVALID_ARGUMENT
    assert put(sig, row=24) == _lib.MLA_ERR_INVALID_ARGUMENT and b"16 bytes" in lib.mla_last_error()
    assert put(sig, off=8) == _lib.MLA_ERR_INVALID_ARGUMENT
    assert lib.mla_peer_wait(None, 1, fake, 0, None, None) == _lib.MLA_ERR_INVALID_ARGUMENT
    assert lib.mla_peer_wait(fake, 0, fake, 0, None, None) == _lib.MLA_ERR_INVALID_ARGUMENT
    a = _lib.MlaDecodeArgs()
    a.dtype, a.batch, a.max_seq_len = _lib.DTYPE_BF16, 5, 16
    gather = lambda args, world=2, off=0, parity=1024, s=sig: lib.mla_decode_partial_gather(
        C.byref(ok), C.byref(args), world, fake, off, parity, C.byref(s), fake, 1 << 20, None)
    assert gather(a) == _lib.MLA_ERR_UNSUPPORTED and b"batch" in lib.mla_last_error()   # batch 5 > 4
    a.batch = 1
    assert gather(a, world=0) == _lib.MLA_ERR_INVALID_ARGUMENT
    assert gather(a, parity=1000) == _lib.MLA_ERR_INVALID_ARGUMENT
    assert gather(a, s=no_counters) == _lib.MLA_ERR_INVALID_ARGUMENT
    assert lib.mla_decode_partial_put(C.byref(ok), C.byref(a), 3, fake, 0, C.byref(sig), fake, 1 << 20,
                                      None) == _lib.MLA_ERR_INVALID_ARGUMENT              # 3 does not divide 128
    assert lib.mla_combine_partials_gathered(C.byref(ok), _lib.DTYPE_BF16, 1, 2, fake, 1000, fake, fake, fake,
                                             None) == _lib.MLA_ERR_INVALID_ARGUMENT        # parity not 16-aligned
    assert lib.mla_combine_partials_gathered(C.byref(ok), _lib.DTYPE_BF16, 1, 2, fake, 1024, None, fake, fake,
                                             None) == _lib.MLA_ERR_INVALID_ARGUMENT        # no step counter
    assert lib.mla_combine_partials_put(C.byref(ok), _lib.DTYPE_BF16, 1, 2, 64, fake, fake, 2, fake, 0, 64,
                                        C.byref(sig), fake, None) == _lib.MLA_ERR_INVALID_ARGUMENT  # pitch < row
    # the one-kernel KV-range step
    a.output = 256
    need = 2 * 1 * 128 * (512 + 4) * 8
    kvr = lambda args, world=2, rank=0, half=need, recv=fake: lib.mla_decode_kv_range(
        C.byref(ok), C.byref(args), world, rank, recv, half, fake, fake, fake, fake, 1 << 20, None)
    assert kvr(a, world=0) == _lib.MLA_ERR_INVALID_ARGUMENT
    assert kvr(a, world=65) == _lib.MLA_ERR_INVALID_ARGUMENT
    assert kvr(a, rank=2) == _lib.MLA_ERR_INVALID_ARGUMENT
    assert kvr(a, recv=None) == _lib.MLA_ERR_INVALID_ARGUMENT
    assert kvr(a, half=need - 16) == _lib.MLA_ERR_INVALID_ARGUMENT and b"half_bytes" in lib.mla_last_error()
    assert kvr(a, half=need + 8) == _lib.MLA_ERR_INVALID_ARGUMENT              # not a multiple of 16
    a.batch = 5
    assert kvr(a) == _lib.MLA_ERR_UNSUPPORTED and b"batch" in lib.mla_last_error()
    a.batch, a.output = 1, None
    assert kvr(a) == _lib.MLA_ERR_INVALID_ARGUMENT


def test_cpp_drop_in_headers_compile():
    """A caller written against the reference's C++ API (tests/test_correctness.cu:186-198 style)
    compiles unchanged against include/latent_attn_b200/*.cuh."""
    src = r'''
#include "latent_attn_b200/fused_mla_batched.cuh"
cudaError_t call(const __half* kv, int S, const float* qa, const float* qr, const __half* wuv,
                 const float* c, const float* s, float* out, cudaStream_t st) {
    MLAConfig cfg = MLAConfig::deepseek_v2();
    cfg.validate();
    FusedMLAParams p;
    p.kv_cache = kv; p.seq_len = S; p.q_absorbed = qa; p.q_rope = qr; p.W_UV = wuv;
    p.rope_cos = c; p.rope_sin = s; p.output = out; p.cfg = &cfg;
    cudaError_t e = launch_fused_mla(p, st);
    BatchedFusedMLAParams b;
    b.kv_cache = kv; b.seq_len = S; b.batch_size = 2; b.q_absorbed = qa; b.q_rope = qr; b.W_UV = wuv;
    b.rope_cos = c; b.rope_sin = s; b.output = out; b.cfg = &cfg;
    return e != cudaSuccess ? e : launch_batched_fused_mla(b, st);
}
'''
    with tempfile.TemporaryDirectory() as d:
        f = os.path.join(d, "caller.cu")
        open(f, "w").write(src)
        r = subprocess.run(["nvcc", "-std=c++17", "-I", INC, "-I", os.path.join(INC, "latent_attn_b200"),
                            "-c", f, "-o", os.path.join(d, "caller.o")], capture_output=True, text=True)
        assert r.returncode == 0, r.stderr


def test_binding_config_cache_validates_and_reuses():
    """The binding builds one read-only config struct per configuration and still rejects
    invalid dimensions the way MLAConfig::validate does (ValueError)."""
    from latent_attn import _C
    a = _C._cfg(0, 512, 128, 64, 128, 128)
    b = _C._cfg(0, 512, 128, 64, 128, 128)
    assert a is b
    assert (a.kv_lora_rank, a.qk_nope_head_dim, a.qk_rope_head_dim, a.num_heads, a.v_head_dim) == (512, 128, 64, 128, 128)
    assert _C._cfg(0, 512, 128, 64, 16, 128) is not a
    with pytest.raises(ValueError):
        _C._cfg(0, 0, 128, 64, 128, 128)
    with pytest.raises(ValueError):
        _C._cfg(0, 512, 128, 64, 0, 128)
