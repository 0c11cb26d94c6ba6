"""ctypes binding of the C-ABI library ``libqw_b200.so`` (include/qw_b200.h).

There is no fallback: if the library is missing or CUDA is unavailable, every call
raises.  Status codes map to exceptions the way the reference's operators fail:
QW_ERR_ARG -> ValueError (reference/fused_ops.py validation errors),
QW_ERR_UNSUPPORTED -> NotImplementedError, QW_ERR_CUDA -> RuntimeError,
QW_ERR_TIMEOUT -> TimeoutError.
"""
from __future__ import annotations

import ctypes
import os
import threading

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libqw_b200.so")

QW_OK, QW_ERR_ARG, QW_ERR_UNSUPPORTED, QW_ERR_CUDA, QW_ERR_TIMEOUT = range(5)
QW_F32, QW_F16, QW_BF16 = 0, 1, 2
QW_OUT_BF16, QW_OUT_F32, QW_OUT_RESID_BF16 = 0, 1, 2
QW_MAX_BLOCK = 16
QW_MAX_SEQ = 256   # tokens per sequence in one forward (prefill chunks)
QW_ATTN_NOALLOC_SCRATCH_BYTES = 16 * 1024 * 1024  # static scratch of qw_attention_noalloc

_c = ctypes
P, I32, I64, F32 = _c.c_void_p, _c.c_int32, _c.c_int64, _c.c_float


class GdnLayer(_c.Structure):
    _fields_ = [("proj", P), ("ab", P), ("conv_hist", P), ("conv_w", P), ("A_log", P),
                ("dt_bias", P), ("norm_w", P), ("state", P), ("out", P)]


class GdnDims(_c.Structure):
    _fields_ = [("batch", I32), ("seq", I32), ("k_heads", I32), ("v_heads", I32), ("dk", I32),
                ("dv", I32), ("channels", I32), ("conv_k", I32), ("ldp", I32), ("eps", F32),
                ("slots", P), ("accepted", P)]


# name -> (restype, argtypes)
SIGNATURES = {
    "qw_abi_version": (_c.c_int, []),
    "qw_last_error": (_c.c_char_p, []),
    "qw_rms_norm": (_c.c_int, [P, _c.c_int, P, _c.c_int, P, _c.c_int, I64, I64, F32, P]),
    "qw_conv_state_update": (_c.c_int, [P, P, P, P, _c.c_int, I64, I64, I64, I64, P]),
    "qw_causal_conv1d": (_c.c_int, [P, P, P, _c.c_int, I64, I64, I64, I64, P]),
    "qw_gated_delta_rule": (_c.c_int, [P, P, P, P, P, _c.c_int, P, _c.c_int, P, P, P,
                                       I64, I64, I64, I64, I64, _c.c_int, P]),
    "qw_cache_update": (_c.c_int, [P, P, P, P, P, P, _c.c_int, I64, I64, I64, I64, I64, P]),
    "qw_attention": (_c.c_int, [P, P, P, P, _c.c_int, I64, I64, I64, I64, I64, I64, I64, F32, P, P]),
    "qw_attn_workspace_bytes": (I64, [I64, I64, I64, I64, I64, I64]),
    "qw_attention_noalloc": (_c.c_int, [P, P, P, P, _c.c_int, I64, I64, I64, I64, I64, I64, I64, F32, P]),
    "qw_attn_prep": (_c.c_int, [P, I64, P, P, F32, F32, I32, P, P, I32, I32, P, P, P, I64, I64, I64,
                                I64, I64, P]),
    "qw_attn_paged": (_c.c_int, [P, P, P, P, I32, I32, P, I64, P, I64, P, I64, I64, I64, I64, I64,
                                 F32, P, P]),
    "qw_moe": (_c.c_int, [P, P, P, P, P, _c.c_int, I64, I64, I64, I64, I64, P, P, P]),
    "qw_moe_workspace_bytes": (I64, [I64, I64, I64, I64, I64]),
    "qw_moe_dense_threshold": (I32, [I32]),
    "qw_moe_route": (_c.c_int, [P, _c.c_int, I64, I64, I64, I64, I64, _c.c_int, P, P]),
    "qw_moe_experts_w4_range": (_c.c_int, [P, P, P, P, P, I64, I64, I64, I64, I64, I32, I64, I64, P, P]),
    "qw_moe_ep_recv_workspace_bytes": (I64, [I64, I64, I64, I64, I64]),
    "qw_ep_window_bytes": (I64, [I64, I64, I64]),
    "qw_ep_window_alloc": (_c.c_int, [I64, _c.POINTER(P), _c.c_char_p]),
    "qw_ep_window_open": (_c.c_int, [_c.c_char_p, _c.POINTER(P)]),
    "qw_ep_window_close": (_c.c_int, [P]),
    "qw_ep_window_free": (_c.c_int, [P]),
    "qw_moe_ep_dispatch": (_c.c_int, [P, P, I64, I64, I64, I64, I64, I64, I64, _c.c_int, P, P, P]),
    "qw_moe_ep_recv_route": (_c.c_int, [P, I64, I64, I64, I64, P, P]),
    "qw_moe_ep_experts": (_c.c_int, [P, P, P, I64, I64, I64, I64, I64, I64, _c.c_int32, P, P, P]),
    "qw_moe_ep_combine_norm": (_c.c_int, [P, P, I64, I64, P, I64, I64, I64, I64, I64, _c.c_int, P, P, F32, P, I64,
                                          _c.c_int, P]),
    "qw_moe_ep_scatter": (_c.c_int, [P, P, I64, I64, I64, I64, I64, I64, I64, _c.c_int, P]),
    "qw_moe_route_x": (_c.c_int, [P, _c.c_int, I64, I64, I64, I64, I64, _c.c_int, P, I64, I32, P, P, I32]),
    "qw_moe_route_lists": (_c.c_int, [P, I64, I64, I64, P]),
    "qw_moe_experts_w4": (_c.c_int, [P, P, P, P, P, I64, I64, I64, I64, I64, I32, P, P]),
    "qw_moe_up_w4": (_c.c_int, [P, P, P, P, P, I64, I64, I64, I64, I64, I32, P, P]),
    "qw_moe_down_w4": (_c.c_int, [P, P, P, P, P, I64, I64, I64, I64, I64, I32, P, P]),
    "qw_moe_active_experts": (I32, [P, I64, I64, I64]),
    "qw_moe_combine": (_c.c_int, [P, P, _c.c_int, I64, I64, I64, I64, I64, _c.c_int, P]),
    "qw_moe_combine_norm": (_c.c_int, [P, P, I64, I64, I64, I64, I64, _c.c_int, P, P, F32, P, I64, _c.c_int, P]),
    "qw_moe_partials": (_c.c_int, [P, I64, I64, I64, I64, I64, _c.POINTER(P), _c.POINTER(P),
                                   _c.POINTER(P), _c.POINTER(P)]),
    "qw_w4_stream_bytes": (I64, [I64, I64, I32]),
    "qw_b16_stream_bytes": (I64, [I64, I64]),
    "qw_w4_linear": (_c.c_int, [P, P, P, _c.c_int, I64, I64, I64, I64, I32, P]),
    "qw_b16_linear": (_c.c_int, [P, P, P, _c.c_int, I64, I64, I64, I64, P]),
    "qw_gdn_verify": (_c.c_int, [_c.POINTER(GdnDims), P, _c.c_int, P]),
    "qw_gdn_commit": (_c.c_int, [_c.POINTER(GdnDims), P, _c.c_int, P]),
    "qw_residual_norm": (_c.c_int, [P, P, P, P, P, P, I64, _c.c_int, I64, I64, F32, P]),
    "qw_lmhead_blocks": (I64, [I64]),
    "qw_lmhead_argmax": (_c.c_int, [P, P, P, P, I64, I64, I64, P]),
    "qw_accept": (_c.c_int, [P, I64, P, P, P, P, P, P, I64, I64, _c.c_int, P]),
    "qw_apply_commit": (_c.c_int, [P, P, P, P, I64, I64, P]),
    "qw_attn_paged_masked": (_c.c_int, [P, P, P, P, I32, I32, P, I64, P, I64, I64, I64, I64, I64, F32, _c.c_int,
                                        I32, P, P]),
    "qw_draft_prep": (_c.c_int, [P, I64, _c.c_int, P, P, F32, F32, P, P, P, P, I32, I32, P, P, P, I64, I64, I64,
                                 I64, I64, P]),
    "qw_swiglu": (_c.c_int, [P, P, I64, I64, P]),
    "qw_draft_block_embed": (_c.c_int, [P, P, I32, P, I64, I64, I64, P]),
    "qw_draft_propose": (_c.c_int, [P, I64, P, P, I64, I64, P]),
    "qw_wait_status": (_c.c_int, [P, _c.c_int, P]),
    "qw_check_wait_status": (_c.c_int, [_c.c_int, P]),
    "qw_debug_inject_wait_timeout": (_c.c_int, [I64, I64]),
}

_lock = threading.Lock()
_lib = None


def load(force: bool = False):
    """Load (once) and return the CDLL with typed entry points."""
    global _lib
    with _lock:
        if _lib is not None and not force:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: run __graft_entry__.build() (no CPU fallback)")
        lib = _c.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name, None)
            if fn is None:
                continue
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def exported_symbols() -> list[str]:
    lib = load()
    return [n for n in SIGNATURES if hasattr(lib, n)]


def check(status: int, what: str = "") -> None:
    if status == QW_OK:
        return
    msg = load().qw_last_error().decode(errors="replace")
    text = f"{what}: {msg}" if what else msg
    if status == QW_ERR_ARG:
        raise ValueError(text)
    if status == QW_ERR_UNSUPPORTED:
        raise NotImplementedError(text)
    if status == QW_ERR_TIMEOUT:
        raise TimeoutError(text)
    raise RuntimeError(text)


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args), name)


# --------------------------------------------------------------------------- torch glue
def ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def dtype_code(dtype) -> int:
    import torch
    codes = {torch.float32: QW_F32, torch.float16: QW_F16, torch.bfloat16: QW_BF16}
    if dtype not in codes:
        raise ValueError(f"unsupported dtype {dtype}")
    return codes[dtype]


def stream_ptr(device=None) -> int:
    import torch
    return torch.cuda.current_stream(device).cuda_stream
