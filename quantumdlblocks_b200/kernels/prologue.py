"""The Born attention layer's operand prologue and row L2 normalisation as native kernels.

The reference layer (``layers/attention.py:508-589``) builds its attention operands with a chain of
PyTorch ops: ``psi = l2_normalize(x)`` (``functional.py:59``), then from the fused projection a
reshape / transpose / ``.contiguous()`` per operand (``:512-516``), ``apply_unitary_rope`` on Q and
K (``functional.py:104-121``) and ``l2_normalize`` again (``:588-589``).  Two op pairs replace it:

  ``qkv_rope_l2norm(qkv, cos, sin, heads, eps)``  qkv ``(B, T, 3 H hd)`` -> Q, K, V ``(B, H, T, hd)``
  ``l2_normalize(x, eps)``                        rows of the last dimension onto the unit sphere

both differentiable (``torch.library`` custom ops with registered backward kernels) and CUDA-only
(no fallback, like the attention op).  ``rope_tables(T, hd)`` gives the angle tables.
"""
from __future__ import annotations

import ctypes

import torch

from .. import _lib
from .flash_born import _DTYPE_CODE, _stream_handle

__all__ = ["qkv_rope_l2norm", "l2_normalize", "rope_tables"]

_SUPPORTED = (torch.bfloat16, torch.float32)


def rope_tables(seq_len: int, head_dim: int, base: float = 10000.0, device=None) -> tuple[torch.Tensor, torch.Tensor]:
    """``(T, hd/2)`` fp32 cos / sin of the angles ``t * base**(-i / (hd/2))``."""
    half = head_dim // 2
    inv = 1.0 / (base ** (torch.arange(half, dtype=torch.float32, device=device) / half))
    ang = torch.arange(seq_len, dtype=torch.float32, device=device)[:, None] * inv[None, :]
    return ang.cos().contiguous(), ang.sin().contiguous()


def _qkv_args(qkv, cos, sin, heads, eps, q, k, v, dqkv=None) -> _lib.FbQkvArgs:
    B, T, three_d = qkv.shape
    a = _lib.FbQkvArgs()
    a.batch, a.seq_len, a.heads, a.head_dim = B, T, heads, three_d // (3 * heads)
    a.dtype = _DTYPE_CODE[qkv.dtype]
    a.eps = float(eps)
    a.qkv, a.cos, a.sin = qkv.data_ptr(), cos.data_ptr(), sin.data_ptr()
    a.q, a.k, a.v = q.data_ptr(), k.data_ptr(), v.data_ptr()
    a.dqkv = None if dqkv is None else dqkv.data_ptr()
    return a


@torch.library.custom_op("flashborn_b200::qkv_prologue", mutates_args=())
def _qkv_prologue(qkv: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, heads: int,
                  eps: float) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    B, T, three_d = qkv.shape
    hd = three_d // (3 * heads)
    q, k, v = (torch.empty((B, heads, T, hd), dtype=qkv.dtype, device=qkv.device) for _ in range(3))
    a = _qkv_args(qkv, cos, sin, heads, eps, q, k, v)
    with torch.cuda.device(qkv.device):
        _lib.check(_lib.load().fb_qkv_prologue_fwd(ctypes.byref(a), _stream_handle(qkv.device)), "qkv prologue")
    return q, k, v


@_qkv_prologue.register_fake
def _qkv_prologue_fake(qkv, cos, sin, heads, eps):
    B, T, three_d = qkv.shape
    hd = three_d // (3 * heads)
    return tuple(qkv.new_empty((B, heads, T, hd)) for _ in range(3))


@torch.library.custom_op("flashborn_b200::qkv_prologue_bwd", mutates_args=())
def _qkv_prologue_bwd(qkv: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, dq: torch.Tensor, dk: torch.Tensor,
                      dv: torch.Tensor, heads: int, eps: float) -> torch.Tensor:
    dqkv = torch.empty_like(qkv)
    a = _qkv_args(qkv, cos, sin, heads, eps, dq, dk, dv, dqkv)
    with torch.cuda.device(qkv.device):
        _lib.check(_lib.load().fb_qkv_prologue_bwd(ctypes.byref(a), _stream_handle(qkv.device)),
                   "qkv prologue backward")
    return dqkv


@_qkv_prologue_bwd.register_fake
def _qkv_prologue_bwd_fake(qkv, cos, sin, dq, dk, dv, heads, eps):
    return torch.empty_like(qkv)


def _qkv_setup(ctx, inputs, output):
    qkv, cos, sin, heads, eps = inputs
    ctx.save_for_backward(qkv, cos, sin)
    ctx.heads, ctx.eps = heads, eps


def _qkv_backward(ctx, dq, dk, dv):
    qkv, cos, sin = ctx.saved_tensors
    B, T, three_d = qkv.shape
    shp = (B, ctx.heads, T, three_d // (3 * ctx.heads))

    def grad(g):
        return torch.zeros(shp, dtype=qkv.dtype, device=qkv.device) if g is None else g.to(qkv.dtype).contiguous()

    return _qkv_prologue_bwd(qkv, cos, sin, grad(dq), grad(dk), grad(dv), ctx.heads, ctx.eps), None, None, None, None


torch.library.register_autograd("flashborn_b200::qkv_prologue", _qkv_backward, setup_context=_qkv_setup)


def qkv_rope_l2norm(qkv: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, heads: int,
                    eps: float = 1e-12) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Q, K, V ``(B, H, T, hd)`` from a fused projection ``qkv (B, T, 3 H hd)``.

    ``Q = l2_normalize(apply_unitary_rope(q))``, likewise K, ``V = v``, where q, k, v are the three
    ``H hd`` slices of each token's row; ``cos`` / ``sin`` are ``(>= T, hd/2)`` angle tables
    (``rope_tables``).  hd is 64 or 128; bf16 or fp32.  Matches the reference's
    ``l2_normalize(apply_unitary_rope(X, cos, sin))`` of ``layers/attention.py:573-589`` with the
    rotation computed in fp32 (the reference rounds it to the activation dtype first).
    """
    if not qkv.is_cuda:
        raise RuntimeError("qkv_rope_l2norm: CUDA tensors required (no CPU path)")
    if qkv.dim() != 3 or qkv.shape[2] % (3 * heads) != 0:
        raise ValueError(f"qkv must be (B, T, 3 H hd); got {tuple(qkv.shape)} with H={heads}")
    if qkv.dtype not in _SUPPORTED:
        raise ValueError(f"qkv_rope_l2norm: dtype {qkv.dtype} not supported (bf16, fp32)")
    T, hd = qkv.shape[1], qkv.shape[2] // (3 * heads)
    if cos.shape[0] < T or cos.shape[1] != hd // 2 or sin.shape != cos.shape:
        raise ValueError(f"rope tables must be (>= {T}, {hd // 2}); got {tuple(cos.shape)}, {tuple(sin.shape)}")
    cos = cos[:T].to(device=qkv.device, dtype=torch.float32).contiguous()
    sin = sin[:T].to(device=qkv.device, dtype=torch.float32).contiguous()
    return _qkv_prologue(qkv.contiguous(), cos, sin, int(heads), float(eps))


def _rows_args(x, eps, y=None, dy=None, dx=None) -> _lib.FbRowsArgs:
    a = _lib.FbRowsArgs()
    a.rows, a.cols = x.numel() // x.shape[-1], x.shape[-1]
    a.dtype = _DTYPE_CODE[x.dtype]
    a.eps = float(eps)
    a.x = x.data_ptr()
    a.y = None if y is None else y.data_ptr()
    a.dy = None if dy is None else dy.data_ptr()
    a.dx = None if dx is None else dx.data_ptr()
    return a


@torch.library.custom_op("flashborn_b200::l2norm_rows", mutates_args=())
def _l2norm_rows(x: torch.Tensor, eps: float) -> torch.Tensor:
    y = torch.empty_like(x)
    a = _rows_args(x, eps, y=y)
    with torch.cuda.device(x.device):
        _lib.check(_lib.load().fb_l2norm_rows_fwd(ctypes.byref(a), _stream_handle(x.device)), "l2 normalise")
    return y


@_l2norm_rows.register_fake
def _l2norm_rows_fake(x, eps):
    return torch.empty_like(x)


@torch.library.custom_op("flashborn_b200::l2norm_rows_bwd", mutates_args=())
def _l2norm_rows_bwd(x: torch.Tensor, dy: torch.Tensor, eps: float) -> torch.Tensor:
    dx = torch.empty_like(x)
    a = _rows_args(x, eps, dy=dy, dx=dx)
    with torch.cuda.device(x.device):
        _lib.check(_lib.load().fb_l2norm_rows_bwd(ctypes.byref(a), _stream_handle(x.device)),
                   "l2 normalise backward")
    return dx


@_l2norm_rows_bwd.register_fake
def _l2norm_rows_bwd_fake(x, dy, eps):
    return torch.empty_like(x)


def _rows_setup(ctx, inputs, output):
    x, eps = inputs
    ctx.save_for_backward(x)
    ctx.eps = eps


def _rows_backward(ctx, dy):
    (x,) = ctx.saved_tensors
    return _l2norm_rows_bwd(x, dy.to(x.dtype).contiguous(), ctx.eps), None


torch.library.register_autograd("flashborn_b200::l2norm_rows", _rows_backward, setup_context=_rows_setup)


def l2_normalize(x: torch.Tensor, eps: float = 1e-12) -> torch.Tensor:
    """``x / sqrt(sum(x^2, -1) + eps)`` over the last dimension (``functional.py:59``), fp32 math.

    The last dimension must be a multiple of 8 (bf16) or 4 (fp32) elements.
    """
    if not x.is_cuda:
        raise RuntimeError("l2_normalize: CUDA tensors required (no CPU path)")
    if x.dtype not in _SUPPORTED:
        raise ValueError(f"l2_normalize: dtype {x.dtype} not supported (bf16, fp32)")
    return _l2norm_rows(x.contiguous(), float(eps))
