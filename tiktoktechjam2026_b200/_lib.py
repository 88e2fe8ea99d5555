"""ctypes binding of libtt_b200.so (the C ABI in include/tt_b200.h).

There is no fallback: if the library is missing or fails to load, every entry
point raises.  Build it with ``python -m tiktoktechjam2026_b200.build``.
"""

from __future__ import annotations

import ctypes
import os
import threading
from ctypes import POINTER, c_char_p, c_float, c_int, c_int64, c_size_t, c_uint, c_ulonglong, c_void_p

# TT_B200_LIB selects another build of the same library (e.g. one compiled with different tile constants).
LIB_PATH = os.environ.get("TT_B200_LIB") or os.path.join(os.path.dirname(os.path.abspath(__file__)), "libtt_b200.so")

TT_OK = 0
TT_ERR_SHAPE = 1
TT_ERR_ALIGN = 2
TT_ERR_UNSUPPORTED = 3
TT_ERR_LAUNCH = 4
TT_ERR_TIMEOUT = 5
TT_ERR_ARG = 6
TT_ERR_WORKSPACE = 7

TT_PEER_HANDLE_BYTES = 64

KERNEL_KINDS = ["ln0", "mask", "qkv", "attn", "out_ln", "ffn_in", "ffn_out_ln", "ffn_fused"]


class TTError(RuntimeError):
    """A libtt_b200 entry point returned a nonzero status."""

    def __init__(self, code: int, message: str):
        super().__init__(f"libtt_b200 error {code}: {message}")
        self.code = code


class LayerWeights(ctypes.Structure):
    _fields_ = [
        ("w_qkv", c_void_p),
        ("b_qkv", c_void_p),
        ("w_out", c_void_p),
        ("b_out", c_void_p),
        ("ln_attn_w", c_void_p),
        ("ln_attn_b", c_void_p),
        ("w_ffn_in", c_void_p),
        ("b_ffn_in", c_void_p),
        ("w_ffn_out", c_void_p),
        ("b_ffn_out", c_void_p),
        ("ln_next_w", c_void_p),
        ("ln_next_b", c_void_p),
    ]


class ModelDesc(ctypes.Structure):
    _fields_ = [
        ("d_model", c_int),
        ("heads", c_int),
        ("ffn_dim", c_int),
        ("num_layers", c_int),
        ("causal", c_int),
        ("eps", c_float),
        ("ln0_w", c_void_p),
        ("ln0_b", c_void_p),
        ("layers", POINTER(LayerWeights)),
    ]


# name -> (restype, argtypes)
SIGNATURES = {
    "tt_abi_version": (c_int, []),
    "tt_last_error": (c_char_p, []),
    "tt_device_error": (c_int, [POINTER(c_uint), c_int]),
    "tt_set_wait_timeout_ns": (None, [c_ulonglong]),
    "tt_launch_count": (c_ulonglong, []),
    "tt_watchdog_selftest": (c_int, [c_ulonglong, c_void_p]),
    "tt_selftest_exp2_fma": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_void_p]),
    "tt_layernorm_rows": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_float, c_int, c_void_p]),
    "tt_mask_kv_end": (c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p]),
    "tt_qkv_projection": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p],
    ),
    "tt_causal_attention": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_float,
         c_int, c_void_p],
    ),
    "tt_causal_attention_masked_noalloc": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_float, c_int,
         c_void_p],
    ),
    "tt_linear_residual_layernorm": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int,
         c_float, c_int, c_void_p, c_void_p],
    ),
    "tt_ffn_residual_layernorm": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
         c_int64, c_int, c_int, c_float, c_int, c_void_p, c_void_p],
    ),
    "tt_linear_gelu": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int, c_void_p]),
    "tt_route_describe": (c_int, [c_int, c_int, c_int, c_int, c_char_p, c_int]),
    "tt_model_create": (c_int, [POINTER(ModelDesc), POINTER(c_void_p)]),
    "tt_model_destroy": (None, [c_void_p]),
    "tt_workspace_alloc": (c_int, [c_size_t, POINTER(c_void_p)]),
    "tt_workspace_free": (c_int, [c_void_p]),
    "tt_model_workspace_bytes": (c_int, [c_void_p, c_int, c_int, POINTER(c_size_t)]),
    "tt_model_forward": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p, c_size_t, c_void_p],
    ),
    "tt_model_host_workspace_bytes": (c_int, [c_void_p, c_int, c_int, POINTER(c_size_t)]),
    "tt_model_forward_host": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_size_t, c_void_p],
    ),
    "tt_model_forward_host_chunks": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, POINTER(c_int), c_int, c_void_p, c_size_t,
         c_void_p],
    ),
    "tt_model_graph_create": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p, c_size_t, POINTER(c_void_p)],
    ),
    "tt_peer_export": (c_int, [c_void_p, c_void_p, POINTER(c_size_t)]),
    "tt_peer_open": (c_int, [c_void_p, c_size_t, POINTER(c_void_p)]),
    "tt_peer_close": (c_int, [c_void_p, c_size_t]),
    "tt_model_forward_gather": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p, c_size_t, c_void_p],
    ),
    "tt_model_gather_wait": (c_int, [c_void_p, c_void_p]),
    "tt_graph_launch": (c_int, [c_void_p, c_void_p]),
    "tt_graph_destroy": (None, [c_void_p]),
    "tt_model_set_profiling": (c_int, [c_void_p, c_int]),
    "tt_model_profile_collect": (c_int, [c_void_p, POINTER(c_float), POINTER(c_int), c_int]),
}

_lib = None
_lock = threading.Lock()


def lib() -> ctypes.CDLL:
    """Loads libtt_b200.so once; raises if it is missing (there is no fallback path)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m tiktoktechjam2026_b200.build` "
                "(this package has no CPU or PyTorch fallback)"
            )
        handle = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
        return _lib


def last_error() -> str:
    msg = lib().tt_last_error()
    return msg.decode() if msg else ""


def check(rc: int) -> None:
    if rc != TT_OK:
        raise TTError(rc, last_error())


def route_describe(d_model: int, heads: int, seq: int, ffn: int) -> str:
    buf = ctypes.create_string_buffer(512)
    check(lib().tt_route_describe(d_model, heads, seq, ffn, buf, 512))
    return buf.value.decode()
