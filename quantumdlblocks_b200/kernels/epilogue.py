"""The Born attention layer's head epilogue as native kernels: ``_finalize_heads`` up to out_proj.

The reference layer (``layers/attention.py:478-493``) takes the attention output through the
gated XSA (``apply_gated_xsa``, ``layers/mudd_and_gates.py:45-61``), the input-driven per-head
output gate (``InputChannelGate``, ``:17-42``) and the head merge, each a PyTorch pass over
``(B, H, T, hd)`` tensors.  ``finalize_heads`` runs the three as one kernel forward and one
backward (``fb_heads_epilogue_fwd/bwd``); the parameter gradients are sums of per-(b, t, h)
scalars the backward kernel writes.  CUDA only, like every op here.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from .. import _lib
from .flash_born import _DTYPE_CODE, _ptr, _stream_handle, _strides

__all__ = ["finalize_heads"]


def _args(o, v, alpha, gx, gw, gb, eps) -> _lib.FbHeadsArgs:
    B, H, T, hd = o.shape
    a = _lib.FbHeadsArgs()
    a.batch, a.heads, a.seq_len, a.head_dim = B, H, T, hd
    a.dtype = _DTYPE_CODE[o.dtype]
    a.eps = float(eps)
    a.o, a.o_stride = _ptr(o), _strides(o)
    if v is not None:
        a.v, a.v_stride = _ptr(v), _strides(v)
    a.xsa_alpha = None if alpha is None else _ptr(alpha)
    if gx is not None:
        a.gate_x, a.gate_channels, a.gate_w, a.gate_b = _ptr(gx), gx.shape[-1], _ptr(gw), _ptr(gb)
    return a


def _run(fn, a, dev, what):
    with torch.cuda.device(dev):
        _lib.check(getattr(_lib.load(), fn)(ctypes.byref(a), _stream_handle(dev)), what)


class _FinalizeHeads(torch.autograd.Function):
    @staticmethod
    def forward(ctx, o, v, alpha, gx, gw, gb, eps):
        B, H, T, hd = o.shape
        y = torch.empty((B, T, H * hd), dtype=o.dtype, device=o.device)
        a = _args(o, v, alpha, gx, gw, gb, eps)
        a.y = _ptr(y)
        _run("fb_heads_epilogue_fwd", a, o.device, "heads epilogue")
        ctx.save_for_backward(o, v, alpha, gx, gw, gb)
        ctx.eps = eps
        return y

    @staticmethod
    def backward(ctx, dy):
        o, v, alpha, gx, gw, gb = ctx.saved_tensors
        B, H, T, hd = o.shape
        dy = dy.to(o.dtype).contiguous()
        grad_o = torch.empty((B, H, T, hd), dtype=o.dtype, device=o.device)
        grad_v = torch.empty_like(grad_o) if alpha is not None else None
        dalpha = torch.empty((B, T, H), dtype=torch.float32, device=o.device) if alpha is not None else None
        du = torch.empty((B, T, H), dtype=torch.float32, device=o.device) if gx is not None else None
        a = _args(o, v, alpha, gx, gw, gb, ctx.eps)
        a.dy, a.grad_o = _ptr(dy), _ptr(grad_o)
        a.grad_v = None if grad_v is None else _ptr(grad_v)
        a.dalpha = None if dalpha is None else _ptr(dalpha)
        a.du = None if du is None else _ptr(du)
        _run("fb_heads_epilogue_bwd", a, o.device, "heads epilogue backward")
        g_alpha = g_x = g_w = g_b = None
        if alpha is not None:
            g_alpha = dalpha.sum(dim=(0, 1))
        if gx is not None:
            du2 = du.reshape(B * T, H)
            g_w = du2.t() @ gx.reshape(B * T, -1)
            g_b = du2.sum(dim=0)
            g_x = (du2 @ gw).reshape(gx.shape)
        return grad_o, grad_v, g_alpha, g_x, g_w, g_b, None


def finalize_heads(
    out_heads: torch.Tensor,
    v: Optional[torch.Tensor] = None,
    xsa_alpha: Optional[torch.Tensor] = None,
    gate_input: Optional[torch.Tensor] = None,
    gate_weight: Optional[torch.Tensor] = None,
    gate_bias: Optional[torch.Tensor] = None,
    eps: float = 1e-12,
) -> torch.Tensor:
    """``(B, T, H hd)`` input of the layer's out_proj from the attention output ``out_heads``
    ``(B, H, T, hd)`` (any strides with a unit inner one; token-major from
    ``flash_born_attention(..., token_major=True)`` reads as well):

    * ``xsa_alpha`` ``(H,)`` with ``v``: ``r = y - tanh(alpha_h) (y . v) / (|v|^2 + eps) v``
      (``apply_gated_xsa``, ``layers/mudd_and_gates.py:45-61``);
    * ``gate_input`` ``(B, T, E)`` with ``gate_weight`` ``(H, c)``, ``gate_bias`` ``(H,)``: times
      ``2 sigmoid(gate_input[..., :c] W_h + b_h)`` (``InputChannelGate``, ``:17-42``, c <= 8);
    * heads merged: ``out[b, t, h hd + i]`` (``layers/attention.py:492``).

    Differentiable in every tensor argument; bf16 or fp32 ``out_heads`` (v the same), hd 32 / 64 /
    128; arithmetic in fp32.
    """
    if not out_heads.is_cuda:
        raise RuntimeError("finalize_heads (B200): out_heads must be a CUDA tensor; there is no CPU path")
    if out_heads.dim() != 4 or out_heads.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError(f"finalize_heads takes (B, H, T, hd) bf16 / fp32 heads; got {tuple(out_heads.shape)} "
                         f"{out_heads.dtype}")
    B, H, T, hd = out_heads.shape
    o = out_heads if out_heads.stride(-1) == 1 else out_heads.contiguous()
    vv = alpha = gx = gw = gb = None
    if xsa_alpha is not None:
        if v is None or v.shape != out_heads.shape:
            raise ValueError("gated XSA needs v of the heads' shape")
        vv = v.to(o.dtype)
        vv = vv if vv.stride(-1) == 1 else vv.contiguous()
        alpha = xsa_alpha.reshape(-1).to(torch.float32).contiguous()
        if alpha.numel() != H:
            raise ValueError(f"xsa_alpha must have H={H} elements")
    if gate_input is not None:
        c = min(gate_weight.shape[-1], gate_input.shape[-1])
        if c > 8 or gate_weight.shape[0] != H:
            raise ValueError("the output gate takes (H, c <= 8) weights")
        gx = gate_input[..., :c].to(torch.float32).contiguous()
        gw = gate_weight[:, :c].to(torch.float32).contiguous()
        gb = gate_bias.reshape(-1).to(torch.float32).contiguous()
    return _FinalizeHeads.apply(o, vv, alpha, gx, gw, gb, float(eps))
