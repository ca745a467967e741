"""Flash-Born attention on B200 (sm_100a): the drop-in for ``qdlblocks.kernels.flash_born``.

Same public names, signatures, argument meaning, layout and error behaviour as the reference
module (``src/qdlblocks/kernels/flash_born.py``):

* ``flash_born_attention(q, k, v, scale, is_causal=True, eps=1e-12, window_size=0, doc_ids=None)``
  (reference ``:655-690``)
* ``flash_purified_born_attention(q, k, v, scale=None, tau=None, eps_base=0.05, is_causal=True,
  eps=1e-8, window_size=0, doc_ids=None, *, gamma_h=None, tau_h=None, causal=None)``
  (reference ``:1290-1341``)
* ``HAS_TRITON`` (here: "the fast CUDA path is available"), ``IS_HIP``,
  ``get_flash_born_launch_meta``, ``get_rdna4_autotune_configs`` (reference ``:21-75``)

The computation runs in the hand-written CUDA kernels of ``libflashborn_b200.so`` through its
C ABI; the autograd wiring is a ``torch.library`` custom op (``flashborn_b200::born_fwd`` /
``born_bwd``) so ``torch.compile`` can trace through it instead of breaking the graph
(the reference disables the compiler around its launch, ``:621``).  There is no CPU or eager
fallback: CPU tensors raise.
"""
from __future__ import annotations

import ctypes
from typing import Any, Optional

import torch

from .. import _lib

IS_HIP: bool = False
HAS_TRITON: bool = _lib.available()
"""True when the native B200 library is present (the name is kept for drop-in compatibility)."""

_DTYPE_CODE = {torch.float32: _lib.FB_F32, torch.float16: _lib.FB_F16, torch.bfloat16: _lib.FB_BF16}

# Kernel path override for tests and benchmarks: "auto", "tcgen05" or "general".
_PATH_CODE = {"auto": _lib.FB_PATH_AUTO, "tcgen05": _lib.FB_PATH_TCGEN05, "general": _lib.FB_PATH_GENERAL}
_forced_path = "auto"


def set_kernel_path(path: str) -> None:
    """Force the kernel family ("auto", "tcgen05", "general") for subsequent calls."""
    global _forced_path
    if path not in _PATH_CODE:
        raise ValueError(f"unknown kernel path {path!r}")
    _forced_path = path


def get_kernel_path() -> str:
    return _forced_path


def _next_pow2(n: int) -> int:
    return 1 << (max(1, int(n)) - 1).bit_length()


def get_flash_born_launch_meta(seq_len: int, is_hip: bool | None = None, head_dim: int = 64) -> dict[str, int]:
    """The reference's Triton launch metadata (``flash_born.py:31-65``), kept for drop-in callers.

    The B200 kernels do not read it (their tile plan is fixed per head dim; see
    ``fb_select_path``); it is reported unchanged because callers and tests inspect it.
    """
    use_hip = IS_HIP if is_hip is None else bool(is_hip)
    width = _next_pow2(head_dim)
    if width >= 256:
        bm = bn = 16
        stages = 1
    elif width >= 128:
        bm = bn = 32 if seq_len >= 32 else 16
        stages = 1
    else:
        bm = bn = 64 if seq_len >= 64 else (32 if seq_len >= 32 else 16)
        stages = 1 if use_hip else 2
    meta = {"BLOCK_M": bm, "BLOCK_N": bn, "num_warps": 4, "num_stages": 1 if use_hip else stages}
    if use_hip:
        meta.update(waves_per_eu=2, matrix_instr_nonkdim=16)
    return meta


def get_rdna4_autotune_configs() -> list[dict[str, int]]:
    """The reference's RDNA 4 autotune list (``flash_born.py:68-75``), kept for drop-in callers."""
    base = {"waves_per_eu": 2, "matrix_instr_nonkdim": 16, "num_stages": 1}
    return [
        dict(BLOCK_M=64, BLOCK_N=64, num_warps=4, **base),
        dict(BLOCK_M=64, BLOCK_N=32, num_warps=4, **base),
        dict(BLOCK_M=128, BLOCK_N=64, num_warps=8, **base),
        dict(BLOCK_M=32, BLOCK_N=32, num_warps=2, **{**base, "waves_per_eu": 4}),
    ]


# ------------------------------------------------------------------------------------------
# Argument packing
# ------------------------------------------------------------------------------------------


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _strides(t: torch.Tensor):
    return _lib._I64x4(*t.stride())


def _stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _prep(x: torch.Tensor) -> torch.Tensor:
    """Inner dimension must be unit-stride (the kernels read rows); copy otherwise."""
    return x if x.stride(-1) == 1 else x.contiguous()


def _fill_common(a: _lib.FbAttnArgs, q, k, v, out, z, scale_flat, tau_flat, doc, is_causal, eps, window_size,
                 eps_base) -> None:
    B, H, T, D = q.shape
    a.batch, a.heads, a.seq_len, a.head_dim = B, H, T, D
    a.dtype = _DTYPE_CODE[q.dtype]
    a.out_dtype = _DTYPE_CODE[out.dtype]
    a.is_causal = int(bool(is_causal))
    a.window_size = int(window_size)
    a.eps = float(eps)
    a.eps_base = float(eps_base)
    a.path = _PATH_CODE[_forced_path]
    # torch.use_deterministic_algorithms(True) asks for a backward without floating-point atomics
    # (the two-kernel tensor-core backward, or the general path); otherwise d=64 uses the fused
    # tensor-core backward, whose dQ reduce-adds may sum in a different order from run to run
    a.deterministic = int(torch.are_deterministic_algorithms_enabled())
    a.q, a.q_stride = _ptr(q), _strides(q)
    a.k, a.k_stride = _ptr(k), _strides(k)
    a.v, a.v_stride = _ptr(v), _strides(v)
    a.out, a.out_stride = _ptr(out), _strides(out)
    a.z = _ptr(z)
    a.scale, a.scale_numel = _ptr(scale_flat), scale_flat.numel()
    if tau_flat is not None:
        a.tau, a.tau_numel = _ptr(tau_flat), tau_flat.numel()
    if doc is not None:
        a.doc_ids = _ptr(doc)
        a.doc_stride = _lib._I64x2(*doc.stride())


def _check_inputs(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> None:
    if not (q.is_cuda and k.is_cuda and v.is_cuda):
        raise RuntimeError("flash-Born (B200): q, k, v must be CUDA tensors; this implementation has no CPU path")
    if q.dim() != 4 or q.shape != k.shape or q.shape != v.shape:
        raise ValueError(f"flash-Born expects q, k, v of one shape (B, H, T, D); got {tuple(q.shape)}, "
                         f"{tuple(k.shape)}, {tuple(v.shape)}")
    D = q.shape[-1]
    if D < 1 or D > 256:
        raise ValueError(f"flash-Born (B200) supports head_dim in [1, 256]; got {D}")


def _alloc_out(B: int, H: int, T: int, D: int, dtype: torch.dtype, device: torch.device,
               token_major: bool) -> torch.Tensor:
    """The forward output, shape (B, H, T, D).  token_major: memory laid out (B, T, H, D), so the
    caller's head merge ``out.transpose(1, 2).reshape(B, T, H * D)`` is a view; the kernels store
    O rows through their strides either way."""
    if token_major:
        return torch.empty((B, T, H, D), dtype=dtype, device=device).transpose(1, 2)
    return torch.empty((B, H, T, D), dtype=dtype, device=device)


# ------------------------------------------------------------------------------------------
# Custom ops
# ------------------------------------------------------------------------------------------


@torch.library.custom_op("flashborn_b200::born_fwd", mutates_args=())
def _born_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: torch.Tensor, tau: Optional[torch.Tensor],
              doc_ids: Optional[torch.Tensor], is_causal: bool, eps: float, window_size: int, eps_base: float,
              purified: bool, token_major: bool = False, f32_out: bool = False) -> tuple[torch.Tensor, torch.Tensor]:
    B, H, T, D = q.shape
    out_dtype = torch.float32 if (purified or f32_out) else q.dtype
    out = _alloc_out(B, H, T, D, out_dtype, q.device, token_major)
    z = torch.empty((B, H, T), dtype=torch.float32, device=q.device)
    lib = _lib.load()
    a = _lib.FbAttnArgs()
    _fill_common(a, q, k, v, out, z, scale, tau, doc_ids, is_causal, eps, window_size, eps_base)
    ws = None
    if doc_ids is not None:  # document spans for tile skipping
        ws_bytes = int(lib.fb_fwd_workspace_size(ctypes.byref(a)))
        if ws_bytes:
            ws = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device)
            a.workspace, a.workspace_bytes = _ptr(ws), ws_bytes
    with torch.cuda.device(q.device):
        fn = lib.fb_purified_born_fwd if purified else lib.fb_born_fwd
        _lib.check(fn(ctypes.byref(a), _stream_handle(q.device)), "flash-Born forward")
    return out, z


@_born_fwd.register_fake
def _born_fwd_fake(q, k, v, scale, tau, doc_ids, is_causal, eps, window_size, eps_base, purified, token_major=False,
                   f32_out=False):
    B, H, T, D = q.shape
    out = _alloc_out(B, H, T, D, torch.float32 if (purified or f32_out) else q.dtype, q.device, token_major)
    return out, q.new_empty((B, H, T), dtype=torch.float32)


@torch.library.custom_op("flashborn_b200::born_bwd", mutates_args=())
def _born_bwd(dout: torch.Tensor, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor,
              z: torch.Tensor, scale: torch.Tensor, tau: Optional[torch.Tensor], doc_ids: Optional[torch.Tensor],
              is_causal: bool, eps: float, window_size: int, eps_base: float,
              purified: bool) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    dq = torch.empty_like(q, memory_format=torch.contiguous_format)
    dk = torch.empty_like(k, memory_format=torch.contiguous_format)
    dv = torch.empty_like(v, memory_format=torch.contiguous_format)
    dscale = torch.zeros(scale.numel(), dtype=torch.float32, device=q.device)
    dtau = torch.zeros(tau.numel() if (purified and tau is not None) else 0, dtype=torch.float32, device=q.device)
    lib = _lib.load()
    a = _lib.FbAttnArgs()
    _fill_common(a, q, k, v, out, z, scale, tau if purified else None, doc_ids, is_causal, eps, window_size, eps_base)
    a.dout, a.dout_stride = _ptr(dout), _strides(dout)
    a.dq, a.dq_stride = _ptr(dq), _strides(dq)
    a.dk, a.dk_stride = _ptr(dk), _strides(dk)
    a.dv, a.dv_stride = _ptr(dv), _strides(dv)
    a.dscale = _ptr(dscale)
    a.dtau = _ptr(dtau) if purified else None
    ws_bytes = int(lib.fb_bwd_workspace_size(ctypes.byref(a)))
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=q.device)
    a.workspace, a.workspace_bytes = _ptr(ws), ws_bytes
    with torch.cuda.device(q.device):
        fn = lib.fb_purified_born_bwd if purified else lib.fb_born_bwd
        _lib.check(fn(ctypes.byref(a), _stream_handle(q.device)), "flash-Born backward")
    return dq, dk, dv, dscale, dtau


@_born_bwd.register_fake
def _born_bwd_fake(dout, q, k, v, out, z, scale, tau, doc_ids, is_causal, eps, window_size, eps_base, purified):
    n_tau = tau.numel() if (purified and tau is not None) else 0
    return (torch.empty_like(q), torch.empty_like(k), torch.empty_like(v),
            q.new_empty((scale.numel(),), dtype=torch.float32), q.new_empty((n_tau,), dtype=torch.float32))


def _setup_context(ctx, inputs, output):
    q, k, v, scale, tau, doc_ids, is_causal, eps, window_size, eps_base, purified = inputs[:11]
    out, z = output
    ctx.save_for_backward(q, k, v, out, z, scale, tau, doc_ids)
    ctx.is_causal = is_causal
    ctx.eps = eps
    ctx.window_size = window_size
    ctx.eps_base = eps_base
    ctx.purified = purified


def _backward(ctx, dout, dz):
    q, k, v, out, z, scale, tau, doc_ids = ctx.saved_tensors
    # the reference casts dO to the saved value dtype (flash_born.py:532)
    dout = _prep(dout.to(v.dtype))
    dq, dk, dv, dscale, dtau = _born_bwd(dout, q, k, v, out, z, scale, tau, doc_ids, ctx.is_causal, ctx.eps,
                                         ctx.window_size, ctx.eps_base, ctx.purified)
    dtau_out = dtau if (ctx.purified and tau is not None) else None
    return dq, dk, dv, dscale, dtau_out, None, None, None, None, None, None, None, None


torch.library.register_autograd("flashborn_b200::born_fwd", _backward, setup_context=_setup_context)


# ------------------------------------------------------------------------------------------
# Public entry points
# ------------------------------------------------------------------------------------------


def _target_dtype(q: torch.Tensor, v: torch.Tensor) -> torch.dtype:
    """Autocast GPU dtype when autocast is on, else v's dtype (flash_born.py:447)."""
    if q.is_cuda and torch.is_autocast_enabled("cuda"):
        return torch.get_autocast_dtype("cuda")
    return v.dtype


def _as_param(x: Any, device: torch.device) -> torch.Tensor:
    if isinstance(x, torch.Tensor):
        return x
    return torch.tensor(float(x), dtype=torch.float32, device=device)


def _flat_f32(t: torch.Tensor, device: torch.device) -> torch.Tensor:
    return t.reshape(-1).to(device=device, dtype=torch.float32).contiguous()


def _doc_i32(doc_ids: Optional[torch.Tensor], device: torch.device) -> Optional[torch.Tensor]:
    if doc_ids is None:
        return None
    return doc_ids.to(device=device, dtype=torch.int32).contiguous()


def flash_born_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    scale: float | torch.Tensor,
    is_causal: bool = True,
    eps: float = 1e-12,
    window_size: int = 0,
    doc_ids: torch.Tensor | None = None,
    *,
    token_major: bool = False,
) -> torch.Tensor:
    """Born attention ``O_i = sum_j p_ij v_j / (sum_j p_ij + eps)``, ``p = relu(scale q.k)^2``.

    Drop-in for ``qdlblocks.kernels.flash_born.flash_born_attention`` (``flash_born.py:655``):
    q, k, v are ``(B, H, T, D)`` CUDA tensors; ``scale`` is a float, a 0-d tensor, or a per-head
    tensor with ``H`` elements (``(H,)`` or ``(1, H, 1, 1)``), differentiable; ``window_size > 0``
    keeps keys with ``i - j < window_size``; ``doc_ids (B, T)`` masks across documents.
    Returns the output in the autocast dtype (or v's dtype) with gradients for q, k, v, scale.

    ``token_major=True`` (an addition; the reference has no such argument) returns the same
    values with memory laid out (B, T, H, D): the kernel stores each O row straight into its
    token's slot, so the head merge that follows the reference call
    (``out_heads.transpose(1, 2).contiguous().view(B, T, D)``, ``layers/attention.py:492``) is
    a view instead of a copy, and the incoming gradient of that merge reaches the backward
    kernels without a copy either.
    """
    _check_inputs(q, k, v)
    scale_t = _as_param(scale, q.device)
    dt = _target_dtype(q, v)
    if dt not in _DTYPE_CODE:
        raise ValueError(f"flash-Born (B200): unsupported dtype {dt}")
    qc, kc, vc = (_prep(x.to(dt)) for x in (q, k, v))
    if scale_t.numel() not in (1, q.shape[1]):
        raise ValueError(f"scale must have 1 or H={q.shape[1]} elements, got {scale_t.numel()}")
    out, _ = _born_fwd(qc, kc, vc, _flat_f32(scale_t, q.device), None, _doc_i32(doc_ids, q.device),
                       bool(is_causal), float(eps), int(window_size), 0.0, False, bool(token_major))
    return out


def flash_born_attention_token_major(q, k, v, scale, is_causal=True, eps=1e-12, window_size=0, doc_ids=None):
    """``flash_born_attention`` with ``token_major=True``: the binding that ``swap.install`` gives
    the reference's attention layer, whose only use of the result is the head merge of
    ``_finalize_heads`` (``layers/attention.py:478-493``)."""
    return flash_born_attention(q, k, v, scale, is_causal, eps, window_size, doc_ids, token_major=True)


def _run_triton_flash_born(q, k, v, scale_t, is_causal, eps, window_size=0, doc_ids=None):
    """Name kept from the reference (``flash_born.py:621``); routes to the B200 kernels."""
    return flash_born_attention(q, k, v, scale_t, is_causal, eps, window_size=window_size, doc_ids=doc_ids)


def flash_purified_born_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    scale: float | torch.Tensor | None = None,
    tau: float | torch.Tensor | None = None,
    eps_base: float = 0.05,
    is_causal: bool = True,
    eps: float = 1e-8,
    window_size: int = 0,
    doc_ids: torch.Tensor | None = None,
    *,
    gamma_h: float | torch.Tensor | None = None,
    tau_h: float | torch.Tensor | None = None,
    causal: bool | None = None,
) -> torch.Tensor:
    """Degree-4 coherence-thresholded ("purified") Born attention.

    Drop-in for ``qdlblocks.kernels.flash_born.flash_purified_born_attention``
    (``flash_born.py:1290``): ``p = relu(gamma (q.k - tau))^4 + eps_base relu(q.k)^2``; keyword
    aliases ``gamma_h``/``tau_h``/``causal`` and defaults ``gamma=8, tau=0.0625`` as there.
    The forward accumulates and stores the output in fp32 and returns it cast to the autocast
    dtype (or v's dtype), as the reference does (``:1102``, ``:1167``).
    """
    if scale is None:
        scale = gamma_h if gamma_h is not None else 8.0
    if tau is None:
        tau = tau_h if tau_h is not None else 0.0625
    if causal is not None:
        is_causal = bool(causal)
    _check_inputs(q, k, v)
    gamma_t = _as_param(scale, q.device)
    tau_t = _as_param(tau, q.device)
    dt = _target_dtype(q, v)
    if dt not in _DTYPE_CODE:
        raise ValueError(f"flash-Born (B200): unsupported dtype {dt}")
    H = q.shape[1]
    if gamma_t.numel() not in (1, H) or tau_t.numel() not in (1, H):
        raise ValueError(f"gamma/tau must have 1 or H={H} elements")
    qc, kc, vc = (_prep(x.to(dt)) for x in (q, k, v))
    out, _ = _born_fwd(qc, kc, vc, _flat_f32(gamma_t, q.device), _flat_f32(tau_t, q.device),
                       _doc_i32(doc_ids, q.device), bool(is_causal), float(eps), int(window_size),
                       float(eps_base), True)
    return out.to(dt)


def last_launch_count() -> int:
    """Kernel launches enqueued by the last flash-Born call on this thread."""
    return int(_lib.load().fb_last_launch_count())


def device_status(stream: Optional[torch.cuda.Stream] = None) -> tuple[int, int]:
    """(status, site) of the device status word (FB_OK or FB_ERR_TIMEOUT); clears it."""
    s = (stream or torch.cuda.current_stream()).cuda_stream
    detail = ctypes.c_int32(0)
    rc = _lib.load().fb_device_status(s, ctypes.byref(detail))
    return int(rc), int(detail.value)
