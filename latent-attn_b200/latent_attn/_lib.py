"""ctypes binding of the C ABI declared in include/latent_attn_b200/mla.h.

The shared library ``libmla_b200.so`` is built in-tree by ``build.py`` (next to
this file). Loading fails loudly when it is missing: there is no fallback.
"""

from __future__ import annotations

import ctypes as C
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("LATENT_ATTN_B200_LIB", os.path.join(_HERE, "libmla_b200.so"))

MLA_OK = 0
MLA_ERR_INVALID_ARGUMENT = 1
MLA_ERR_UNSUPPORTED = 2
MLA_ERR_WORKSPACE = 3
MLA_ERR_CUDA = 4
MLA_ERR_NO_DEVICE_CODE = 5
MLA_ERR_TIMEOUT = 6

STATUS_NAMES = {
    0: "MLA_OK", 1: "MLA_ERR_INVALID_ARGUMENT", 2: "MLA_ERR_UNSUPPORTED", 3: "MLA_ERR_WORKSPACE",
    4: "MLA_ERR_CUDA", 5: "MLA_ERR_NO_DEVICE_CODE", 6: "MLA_ERR_TIMEOUT",
}

NOALLOC_SCRATCH_BYTES = 8 << 20

DTYPE_F16 = 0
DTYPE_BF16 = 1
DTYPE_F32 = 2


class MlaConfig(C.Structure):
    _fields_ = [("d_model", C.c_int), ("kv_lora_rank", C.c_int), ("qk_nope_head_dim", C.c_int),
                ("qk_rope_head_dim", C.c_int), ("num_heads", C.c_int), ("v_head_dim", C.c_int)]


class MlaFusedParams(C.Structure):
    _fields_ = [("kv_cache", C.c_void_p), ("seq_len", C.c_int), ("q_absorbed", C.c_void_p),
                ("q_rope", C.c_void_p), ("W_UV", C.c_void_p), ("rope_cos", C.c_void_p),
                ("rope_sin", C.c_void_p), ("output", C.c_void_p), ("cfg", C.POINTER(MlaConfig))]


class MlaBatchedFusedParams(C.Structure):
    _fields_ = [("kv_cache", C.c_void_p), ("seq_len", C.c_int), ("batch_size", C.c_int),
                ("q_absorbed", C.c_void_p), ("q_rope", C.c_void_p), ("W_UV", C.c_void_p),
                ("rope_cos", C.c_void_p), ("rope_sin", C.c_void_p), ("output", C.c_void_p),
                ("cfg", C.POINTER(MlaConfig))]


class MlaDecodeArgs(C.Structure):
    _fields_ = [("dtype", C.c_int), ("batch", C.c_int), ("shared_cache", C.c_int),
                ("kv_cache", C.c_void_p), ("kv_row_stride", C.c_int64), ("kv_total_rows", C.c_int64),
                ("kv_offsets", C.c_void_p),
                ("seq_lens", C.c_void_p), ("seq_lens_host", C.c_void_p), ("max_seq_len", C.c_int),
                ("kv_pos_offset", C.c_int), ("q_absorbed", C.c_void_p), ("q_nope", C.c_void_p),
                ("W_UK", C.c_void_p), ("q_rope", C.c_void_p), ("W_UV", C.c_void_p),
                ("rope_cos", C.c_void_p), ("rope_sin", C.c_void_p), ("softmax_scale", C.c_float),
                ("output", C.c_void_p), ("kernel", C.c_int), ("timer", C.c_void_p),
                ("page_table", C.c_void_p), ("page_rows", C.c_int), ("max_pages", C.c_int),
                ("rope_theta", C.c_float)]

class MlaPeerSignal(C.Structure):
    _fields_ = [("flags", C.c_void_p), ("flag_index", C.c_int), ("epoch", C.c_void_p), ("counters", C.c_void_p)]


KERNEL_AUTO = 0
KERNEL_TENSOR_CORE = 1
KERNEL_CUDA_CORE = 2


# Every symbol the header declares, with (restype, argtypes).
IPC_HANDLE_BYTES = 64   # MLA_IPC_HANDLE_BYTES

SIGNATURES = {
    "mla_config_validate": (C.c_int, [C.POINTER(MlaConfig)]),
    "mla_launch_fused": (C.c_int, [C.POINTER(MlaFusedParams), C.c_int, C.c_void_p]),
    "mla_launch_batched_fused": (C.c_int, [C.POINTER(MlaBatchedFusedParams), C.c_int, C.c_void_p]),
    "mla_launch_fused_noalloc": (C.c_int, [C.POINTER(MlaFusedParams), C.c_int, C.c_void_p]),
    "mla_decode_workspace_size": (C.c_int, [C.POINTER(MlaConfig), C.POINTER(MlaDecodeArgs),
                                            C.POINTER(C.c_size_t)]),
    "mla_decode": (C.c_int, [C.POINTER(MlaConfig), C.POINTER(MlaDecodeArgs), C.c_void_p, C.c_size_t,
                             C.c_void_p]),
    "mla_decode_partial": (C.c_int, [C.POINTER(MlaConfig), C.POINTER(MlaDecodeArgs), C.c_void_p,
                                     C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]),
    "mla_combine_partials": (C.c_int, [C.POINTER(MlaConfig), C.c_int, C.c_int, C.c_int, C.c_void_p,
                                       C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "mla_decode_partial_packed": (C.c_int, [C.POINTER(MlaConfig), C.POINTER(MlaDecodeArgs), C.c_int, C.c_void_p,
                                            C.c_void_p, C.c_size_t, C.c_void_p]),
    "mla_combine_partials_packed": (C.c_int, [C.POINTER(MlaConfig), C.c_int, C.c_int, C.c_int, C.c_int,
                                              C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "mla_cache_append": (C.c_int, [C.POINTER(MlaConfig), C.c_int, C.c_void_p, C.c_int64, C.c_int64, C.c_int,
                                   C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int,
                                   C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]),
    "mla_linear": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "mla_ipc_alloc": (C.c_int, [C.c_size_t, C.POINTER(C.c_void_p), C.c_void_p]),
    "mla_ipc_free": (C.c_int, [C.c_void_p]),
    "mla_ipc_open": (C.c_int, [C.c_void_p, C.POINTER(C.c_void_p)]),
    "mla_ipc_close": (C.c_int, [C.c_void_p]),
    "mla_peer_put": (C.c_int, [C.c_void_p, C.c_size_t, C.c_size_t, C.c_size_t, C.c_size_t, C.c_void_p, C.c_size_t,
                               C.c_size_t, C.c_int, C.c_int, C.POINTER(MlaPeerSignal), C.c_void_p]),
    "mla_decode_partial_put": (C.c_int, [C.POINTER(MlaConfig), C.POINTER(MlaDecodeArgs), C.c_int, C.c_void_p,
                                         C.c_size_t, C.POINTER(MlaPeerSignal), C.c_void_p, C.c_size_t, C.c_void_p]),
    "mla_combine_partials_put": (C.c_int, [C.POINTER(MlaConfig), C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p,
                                           C.c_void_p, C.c_int, C.c_void_p, C.c_size_t, C.c_size_t,
                                           C.POINTER(MlaPeerSignal), C.c_void_p, C.c_void_p]),
    "mla_decode_partial_gather": (C.c_int, [C.POINTER(MlaConfig), C.POINTER(MlaDecodeArgs), C.c_int, C.c_void_p,
                                            C.c_size_t, C.c_size_t, C.POINTER(MlaPeerSignal), C.c_void_p, C.c_size_t,
                                            C.c_void_p]),
    "mla_combine_partials_gathered": (C.c_int, [C.POINTER(MlaConfig), C.c_int, C.c_int, C.c_int, C.c_void_p,
                                                C.c_size_t, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "mla_decode_kv_range": (C.c_int, [C.POINTER(MlaConfig), C.POINTER(MlaDecodeArgs), C.c_int, C.c_int, C.c_void_p,
                                      C.c_size_t, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t,
                                      C.c_void_p]),
    "mla_peer_wait": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]),
    "mla_timer_create": (C.c_int, [C.POINTER(C.c_void_p)]),
    "mla_timer_destroy": (C.c_int, [C.c_void_p]),
    "mla_timer_decode_ms": (C.c_int, [C.c_void_p, C.POINTER(C.c_float)]),
    "mla_kernel_launch_count": (C.c_uint64, []),
    "mla_last_error": (C.c_char_p, []),
    "mla_version": (C.c_char_p, []),
}

_lib = None
_lock = threading.Lock()


class MlaError(RuntimeError):
    """A non-OK status from the C ABI (RuntimeError, like the reference's TORCH_CHECK)."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


def load() -> C.CDLL:
    """Load libmla_b200.so once; raises ImportError if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(
                    f"latent_attn B200 library not found at {LIB_PATH}. "
                    "Build it with `python latent-attn_b200/build.py` (or __graft_entry__.build()).")
            lib = C.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def check(status: int) -> None:
    if status != MLA_OK:
        msg = load().mla_last_error()
        raise MlaError(status, msg.decode() if msg else "")


class DecodeTimer:
    """Owns an mla_timer_t; pass ``.handle`` as ``timer=`` to a decode call, then
    read ``decode_ms()`` (waits for the decode kernel of that call)."""

    def __init__(self):
        lib = load()
        h = C.c_void_p()
        check(lib.mla_timer_create(C.byref(h)))
        self.handle = h.value

    def decode_ms(self) -> float:
        ms = C.c_float(0.0)
        check(load().mla_timer_decode_ms(C.c_void_p(self.handle), C.byref(ms)))
        return float(ms.value)

    def close(self):
        if self.handle:
            load().mla_timer_destroy(C.c_void_p(self.handle))
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def kernel_launch_count() -> int:
    return int(load().mla_kernel_launch_count())
