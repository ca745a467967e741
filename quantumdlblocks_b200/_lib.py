"""ctypes binding of libflashborn_b200.so (the C ABI declared in include/flashborn_b200.h).

The library is built in-tree by ``python -m quantumdlblocks_b200.build`` (or
``__graft_entry__.build()``).  Loading it needs no GPU; running its entry points does.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libflashborn_b200.so")

FB_OK = 0
FB_ERR_SHAPE = 1
FB_ERR_DTYPE = 2
FB_ERR_ALIGN = 3
FB_ERR_ARG = 4
FB_ERR_LAUNCH = 5
FB_ERR_TIMEOUT = 6
FB_ERR_WORKSPACE = 7
FB_ERR_NO_DEVICE = 8
FB_ERR_UNSUPPORTED = 9
FB_ERR_SCRATCH_LIMIT = 10
FB_STATIC_SCRATCH_BYTES = 16 * 1024 * 1024

FB_F32, FB_F16, FB_BF16 = 0, 1, 2
FB_PATH_AUTO, FB_PATH_TCGEN05, FB_PATH_GENERAL = 0, 1, 2

_I64x4 = ctypes.c_int64 * 4
_I64x2 = ctypes.c_int64 * 2


class FbAttnArgs(ctypes.Structure):
    """Mirror of ``fb_attn_args`` (field order and types must match the header)."""

    _fields_ = [
        ("batch", ctypes.c_int32), ("heads", ctypes.c_int32), ("seq_len", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("dtype", ctypes.c_int32), ("out_dtype", ctypes.c_int32),
        ("is_causal", ctypes.c_int32), ("window_size", ctypes.c_int32),
        ("eps", ctypes.c_float), ("eps_base", ctypes.c_float),
        ("path", ctypes.c_int32), ("deterministic", ctypes.c_int32),
        ("q", ctypes.c_void_p), ("q_stride", _I64x4),
        ("k", ctypes.c_void_p), ("k_stride", _I64x4),
        ("v", ctypes.c_void_p), ("v_stride", _I64x4),
        ("out", ctypes.c_void_p), ("out_stride", _I64x4),
        ("z", ctypes.c_void_p),
        ("scale", ctypes.c_void_p), ("scale_numel", ctypes.c_int32),
        ("tau", ctypes.c_void_p), ("tau_numel", ctypes.c_int32),
        ("doc_ids", ctypes.c_void_p), ("doc_stride", _I64x2),
        ("dout", ctypes.c_void_p), ("dout_stride", _I64x4),
        ("dq", ctypes.c_void_p), ("dq_stride", _I64x4),
        ("dk", ctypes.c_void_p), ("dk_stride", _I64x4),
        ("dv", ctypes.c_void_p), ("dv_stride", _I64x4),
        ("dscale", ctypes.c_void_p), ("dtau", ctypes.c_void_p),
        ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t),
    ]


class FbQkvArgs(ctypes.Structure):
    """Mirror of ``fb_qkv_args`` (the attention layer's Q / K / V prologue)."""
    _fields_ = [
        ("batch", ctypes.c_int32), ("seq_len", ctypes.c_int32), ("heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32), ("dtype", ctypes.c_int32), ("eps", ctypes.c_float),
        ("qkv", ctypes.c_void_p), ("cos", ctypes.c_void_p), ("sin", ctypes.c_void_p),
        ("q", ctypes.c_void_p), ("k", ctypes.c_void_p), ("v", ctypes.c_void_p), ("dqkv", ctypes.c_void_p),
    ]


class FbRowsArgs(ctypes.Structure):
    """Mirror of ``fb_rows_args`` (row L2 normalisation)."""
    _fields_ = [
        ("rows", ctypes.c_int64), ("cols", ctypes.c_int32), ("dtype", ctypes.c_int32), ("eps", ctypes.c_float),
        ("x", ctypes.c_void_p), ("y", ctypes.c_void_p), ("dy", ctypes.c_void_p), ("dx", ctypes.c_void_p),
    ]


class FbXentArgs(ctypes.Structure):
    """Mirror of ``fb_xent_args`` (the GPT training loss)."""
    _fields_ = [
        ("rows", ctypes.c_int64), ("vocab", ctypes.c_int32), ("ld", ctypes.c_int64),
        ("logits", ctypes.c_void_p), ("targets", ctypes.c_void_p), ("lse", ctypes.c_void_p),
        ("loss", ctypes.c_void_p), ("grad", ctypes.c_void_p), ("gscale", ctypes.c_void_p),
    ]


class FbRotArgs(ctypes.Structure):
    """Mirror of ``fb_rot_args``."""
    _fields_ = [("rows", ctypes.c_int64), ("head_dim", ctypes.c_int32), ("dtype", ctypes.c_int32),
                ("adjoint", ctypes.c_int32), ("a", ctypes.c_void_p), ("b", ctypes.c_void_p), ("dst", ctypes.c_void_p)]


class FbCombineArgs(ctypes.Structure):
    """Mirror of ``fb_combine_args``."""
    _fields_ = [
        ("batch", ctypes.c_int32), ("heads", ctypes.c_int32), ("seq_len", ctypes.c_int32),
        ("head_dim", ctypes.c_int32), ("n_terms", ctypes.c_int32), ("out_dtype", ctypes.c_int32),
        ("o", ctypes.c_void_p * 4), ("z", ctypes.c_void_p * 4),
        ("out", ctypes.c_void_p), ("out_stride", _I64x4), ("z_out", ctypes.c_void_p), ("z_stride", ctypes.c_int64 * 3),
    ]


class FbDeltaArgs(ctypes.Structure):
    """Mirror of ``fb_delta_args``."""
    _fields_ = [
        ("batch", ctypes.c_int32), ("heads", ctypes.c_int32), ("seq_len", ctypes.c_int32),
        ("head_dim", ctypes.c_int32), ("dout_dtype", ctypes.c_int32), ("out_dtype", ctypes.c_int32),
        ("eps", ctypes.c_float), ("dout", ctypes.c_void_p), ("dout_stride", _I64x4),
        ("out", ctypes.c_void_p), ("out_stride", _I64x4), ("z", ctypes.c_void_p), ("part", ctypes.c_void_p),
    ]


class FbHeadsArgs(ctypes.Structure):
    """Mirror of ``fb_heads_args`` (the layer's head epilogue)."""
    _fields_ = [
        ("batch", ctypes.c_int32), ("heads", ctypes.c_int32), ("seq_len", ctypes.c_int32),
        ("head_dim", ctypes.c_int32), ("dtype", ctypes.c_int32), ("eps", ctypes.c_float),
        ("o", ctypes.c_void_p), ("o_stride", _I64x4), ("v", ctypes.c_void_p), ("v_stride", _I64x4),
        ("xsa_alpha", ctypes.c_void_p), ("gate_x", ctypes.c_void_p), ("gate_channels", ctypes.c_int32),
        ("gate_w", ctypes.c_void_p), ("gate_b", ctypes.c_void_p), ("y", ctypes.c_void_p), ("dy", ctypes.c_void_p),
        ("grad_o", ctypes.c_void_p), ("grad_v", ctypes.c_void_p), ("dalpha", ctypes.c_void_p), ("du", ctypes.c_void_p),
    ]


# Every symbol the header declares, with its ctypes signature.
_PARGS = ctypes.POINTER(FbAttnArgs)
_PQKV = ctypes.POINTER(FbQkvArgs)
_PROWS = ctypes.POINTER(FbRowsArgs)
_PXENT = ctypes.POINTER(FbXentArgs)
SIGNATURES = {
    "fb_born_fwd": (ctypes.c_int, [_PARGS, ctypes.c_void_p]),
    "fb_born_bwd": (ctypes.c_int, [_PARGS, ctypes.c_void_p]),
    "fb_born_bwd_static_scratch": (ctypes.c_int, [_PARGS, ctypes.c_void_p]),
    "fb_born_bwd_term": (ctypes.c_int, [_PARGS, ctypes.c_void_p]),
    "fb_test_born_fwd_timeout": (ctypes.c_int, [_PARGS, ctypes.c_void_p, ctypes.c_uint32]),
    "fb_purified_born_fwd": (ctypes.c_int, [_PARGS, ctypes.c_void_p]),
    "fb_purified_born_bwd": (ctypes.c_int, [_PARGS, ctypes.c_void_p]),
    "fb_bwd_workspace_size": (ctypes.c_size_t, [_PARGS]),
    "fb_fwd_workspace_size": (ctypes.c_size_t, [_PARGS]),
    "fb_select_path": (ctypes.c_int, [_PARGS, ctypes.c_int]),
    "fb_last_launch_count": (ctypes.c_int, []),
    "fb_device_status": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int32)]),
    "fb_strerror": (ctypes.c_char_p, [ctypes.c_int]),
    "fb_last_cuda_error": (ctypes.c_char_p, []),
    "fb_abi_version": (ctypes.c_int, []),
    "fb_qkv_prologue_fwd": (ctypes.c_int, [_PQKV, ctypes.c_void_p]),
    "fb_qkv_prologue_bwd": (ctypes.c_int, [_PQKV, ctypes.c_void_p]),
    "fb_l2norm_rows_fwd": (ctypes.c_int, [_PROWS, ctypes.c_void_p]),
    "fb_l2norm_rows_bwd": (ctypes.c_int, [_PROWS, ctypes.c_void_p]),
    "fb_xent_fwd": (ctypes.c_int, [_PXENT, ctypes.c_void_p]),
    "fb_heads_epilogue_fwd": (ctypes.c_int, [ctypes.POINTER(FbHeadsArgs), ctypes.c_void_p]),
    "fb_heads_epilogue_bwd": (ctypes.c_int, [ctypes.POINTER(FbHeadsArgs), ctypes.c_void_p]),
    "fb_rotate_halves": (ctypes.c_int, [ctypes.POINTER(FbRotArgs), ctypes.c_void_p]),
    "fb_combine_terms": (ctypes.c_int, [ctypes.POINTER(FbCombineArgs), ctypes.c_void_p]),
    "fb_delta_terms": (ctypes.c_int, [ctypes.POINTER(FbDeltaArgs), ctypes.c_void_p]),
    "fb_xent_bwd": (ctypes.c_int, [_PXENT, ctypes.c_void_p]),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class FlashBornLibraryError(RuntimeError):
    """The native library is missing or returned an error status."""


def load() -> ctypes.CDLL:
    """Load (once) and return the native library; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise FlashBornLibraryError(
                    f"{LIB_PATH} is missing: build it with `python -m quantumdlblocks_b200.build` "
                    "(the flash-Born op has no fallback path)")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, argtypes) in SIGNATURES.items():
                if not hasattr(lib, name):
                    raise FlashBornLibraryError(f"{LIB_PATH} does not export {name}: rebuild it "
                                                "(`python -m quantumdlblocks_b200.build`)")
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = argtypes
            _lib = lib
    return _lib


def available() -> bool:
    """True when the library loads and exports every declared entry point (a stale build does not)."""
    try:
        load()
        return True
    except (OSError, AttributeError, FlashBornLibraryError):
        return False


def check(rc: int, what: str) -> None:
    if rc != FB_OK:
        lib = load()
        msg = lib.fb_strerror(rc).decode()
        if rc == FB_ERR_LAUNCH:
            msg += f" [{lib.fb_last_cuda_error().decode()}]"
        exc = ValueError if rc in (FB_ERR_SHAPE, FB_ERR_DTYPE, FB_ERR_ARG) else FlashBornLibraryError
        raise exc(f"{what}: {msg} (status {rc})")
