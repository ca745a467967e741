"""Born attention families that the reference runs only as eager PyTorch: complex phase and
paired heads.  Both are sums of plain Born score families that share one normaliser, so each
runs as several calls of the tensor-core flash-Born kernels plus a combine, never as a T x T
tensor.

complex phase (``layers/attention.py:717-730``).  Q and K hold a complex vector as
``[re | im]`` halves; the layer forms ``s_re = Q_re K_re^T + Q_im K_im^T`` and
``s_im = Q_im K_re^T - Q_re K_im^T`` and ``p = relu(a s_re)^2 + relu(a s_im)^2``.  Since
``s_re = <q, k>`` and ``s_im = <q, rot k>`` with ``rot k = [-k_im | k_re]``, the two terms are
plain Born problems over (q, k, v) and (q, rot k, v).

paired heads (``layers/attention.py:591-626``).  With P = H / 2, the layer reshapes
(B, H, T, D) into (B, P, 2T, D) so that row 2t + a of pair c holds head c + aP at token t, and
masks by token (``idx // 2``): a query of either head of the pair attends the keys of both heads
at every visible token.  The four terms are plain Born problems over the head halves
(q_a, k_b, v_b), a, b in {0, 1}, with the token-level causal / window / document mask.

Combine.  Each term runs with eps / (number of terms) and fp32 output, so that for every query
row ``Z = sum_t Z_t`` is the family's ``sum p + eps`` and ``O = sum_t O_t Z_t / Z``.  The
backward runs ``fb_born_bwd_term`` per term with the combined O and Z (the term's share of
dQ, dK, dV) and forms the scale gradient from the closed form of a score homogeneous of
degree 2 in the scale, ``(2 / a_h) sum_{b,i} eps delta_i / Z_i`` with ``delta_i = dO_i . O_i``.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from .. import _lib
from .flash_born import (_DTYPE_CODE, _as_param, _born_fwd, _check_inputs, _doc_i32, _fill_common, _flat_f32,
                         _prep, _ptr, _stream_handle, _strides, _target_dtype)


def _born_bwd_term(dout, q, k, v, out, z, scale, doc, is_causal, eps, window_size):
    """dQ, dK, dV of one term through fb_born_bwd_term (out, z: the whole family's)."""
    dq = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    dk = torch.empty(k.shape, dtype=k.dtype, device=k.device)
    dv = torch.empty(v.shape, dtype=v.dtype, device=v.device)
    lib = _lib.load()
    a = _lib.FbAttnArgs()
    _fill_common(a, q, k, v, out, z, scale, None, doc, is_causal, eps, window_size, 0.0)
    a.dout, a.dout_stride = _ptr(dout), _strides(dout)
    a.dq, a.dq_stride = _ptr(dq), _strides(dq)
    a.dk, a.dk_stride = _ptr(dk), _strides(dk)
    a.dv, a.dv_stride = _ptr(dv), _strides(dv)
    a.dscale = None
    ws_bytes = int(lib.fb_bwd_workspace_size(ctypes.byref(a)))
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=q.device)
    a.workspace, a.workspace_bytes = _ptr(ws), ws_bytes
    with torch.cuda.device(q.device):
        _lib.check(lib.fb_born_bwd_term(ctypes.byref(a), _stream_handle(q.device)), "flash-Born backward term")
    return dq, dk, dv


def _combine(terms):
    """O = sum O_t Z_t / Z and Z = sum Z_t over terms [(O_t fp32, Z_t)]."""
    z = terms[0][1].clone()
    num = terms[0][0] * terms[0][1].unsqueeze(-1)
    for o_t, z_t in terms[1:]:
        z += z_t
        num.addcmul_(o_t, z_t.unsqueeze(-1))
    return num / z.unsqueeze(-1), z


def _scale_grad(dout, out, z, scale, eps, heads_of_row):
    """(2 / a_h) sum eps delta_i / Z_i per scale entry; heads_of_row maps the (B, H', T) rows'
    head axis to scale entries (identity for per-head scales)."""
    delta = (dout.float() * out).sum(-1)                     # (B, H', T)
    per_head = (eps * delta / z).sum(dim=(0, 2))             # (H',)
    if scale.numel() == 1:
        return (2.0 / scale) * per_head.sum().reshape(1)
    return (2.0 / scale) * heads_of_row(per_head)


def _rot(k: torch.Tensor) -> torch.Tensor:
    half = k.shape[-1] // 2
    return torch.cat((-k[..., half:], k[..., :half]), dim=-1)


def _rot_t(g: torch.Tensor) -> torch.Tensor:
    """Adjoint of _rot: the gradient for k of a gradient g for rot k."""
    half = g.shape[-1] // 2
    return torch.cat((g[..., half:], -g[..., :half]), dim=-1)


class _ComplexPhaseBorn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, scale, doc, is_causal, eps, window_size):
        kr = _rot(k).contiguous()
        terms = [_born_fwd(q, kk, v, scale, None, doc, is_causal, eps / 2, window_size, 0.0, False, False, True)
                 for kk in (k, kr)]
        out, z = _combine(terms)
        ctx.save_for_backward(q, k, kr, v, out, z, scale, doc)
        ctx.cfg = (is_causal, eps, window_size)
        return out.to(v.dtype)

    @staticmethod
    def backward(ctx, dout):
        q, k, kr, v, out, z, scale, doc = ctx.saved_tensors
        is_causal, eps, window_size = ctx.cfg
        dout = _prep(dout.to(v.dtype))
        dq1, dk1, dv1 = _born_bwd_term(dout, q, k, v, out, z, scale, doc, is_causal, eps / 2, window_size)
        dq2, dkr, dv2 = _born_bwd_term(dout, q, kr, v, out, z, scale, doc, is_causal, eps / 2, window_size)
        dk = dk1 + _rot_t(dkr)
        dscale = _scale_grad(dout, out, z, scale, eps, lambda x: x)
        return dq1 + dq2, dk, dv1 + dv2, dscale, None, None, None, None


def complex_phase_born_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    scale: float | torch.Tensor,
    is_causal: bool = True,
    eps: float = 1e-12,
    window_size: int = 0,
    doc_ids: torch.Tensor | None = None,
) -> torch.Tensor:
    """Complex-phase Born attention ``p = relu(a s_re)^2 + relu(a s_im)^2`` (the attention core of
    ``SubspaceProjectorBornAttention`` with ``complex_phase=True``, ``layers/attention.py:717-730``
    and the mask / normalisation that follow it, ``:737-758``).

    q, k, v are ``(B, H, T, D)`` CUDA tensors with D even (first half real, second imaginary);
    ``scale`` is a float, a 0-d tensor or ``H`` per-head values (the layer's
    ``clamp(head_scale, 1, 100)``); mask arguments as ``flash_born_attention``.  Returns
    ``(B, H, T, D)`` in the autocast dtype (or v's dtype), differentiable in q, k, v and scale.
    """
    _check_inputs(q, k, v)
    if q.shape[-1] % 2 != 0:
        raise ValueError(f"complex-phase Born needs an even head_dim; got {q.shape[-1]}")
    dt = _target_dtype(q, v)
    if dt not in _DTYPE_CODE:
        raise ValueError(f"flash-Born (B200): unsupported dtype {dt}")
    scale_t = _as_param(scale, q.device)
    if scale_t.numel() not in (1, q.shape[1]):
        raise ValueError(f"scale must have 1 or H={q.shape[1]} elements, got {scale_t.numel()}")
    qc, kc, vc = (_prep(x.to(dt)) for x in (q, k, v))
    return _ComplexPhaseBorn.apply(qc, kc, vc, _flat_f32(scale_t, q.device), _doc_i32(doc_ids, q.device),
                                   bool(is_causal), float(eps), int(window_size))


class _PairedHeadsBorn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, scale, doc, is_causal, eps, window_size):
        P = q.shape[1] // 2
        half = lambda x, a: x[:, a * P:(a + 1) * P]  # noqa: E731  head half a: (B, P, T, D) view
        outs, zs = [], []
        for a in (0, 1):
            terms = [_born_fwd(half(q, a), half(k, b), half(v, b), scale, None, doc, is_causal, eps / 2,
                               window_size, 0.0, False, False, True) for b in (0, 1)]
            o_a, z_a = _combine(terms)
            outs.append(o_a)
            zs.append(z_a)
        out, z = torch.cat(outs, dim=1), torch.cat(zs, dim=1)
        ctx.save_for_backward(q, k, v, out, z, scale, doc)
        ctx.cfg = (is_causal, eps, window_size)
        return out.to(v.dtype)

    @staticmethod
    def backward(ctx, dout):
        q, k, v, out, z, scale, doc = ctx.saved_tensors
        is_causal, eps, window_size = ctx.cfg
        P = q.shape[1] // 2
        dout = _prep(dout.to(v.dtype))
        half = lambda x, a: x[:, a * P:(a + 1) * P]  # noqa: E731
        dq, dk, dv = torch.zeros_like(q, dtype=torch.float32), torch.zeros_like(k, dtype=torch.float32), \
            torch.zeros_like(v, dtype=torch.float32)
        for a in (0, 1):
            o_a, z_a = out[:, a * P:(a + 1) * P], z[:, a * P:(a + 1) * P].contiguous()
            for b in (0, 1):
                gq, gk, gv = _born_bwd_term(half(dout, a), half(q, a), half(k, b), half(v, b), o_a, z_a, scale, doc,
                                            is_causal, eps / 2, window_size)
                half(dq, a).add_(gq)
                half(dk, b).add_(gk)
                half(dv, b).add_(gv)
        dscale = _scale_grad(dout, out, z, scale, eps, lambda x: x[:P] + x[P:])
        return dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype), dscale, None, None, None, None


def paired_heads_born_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    scale: float | torch.Tensor,
    is_causal: bool = True,
    eps: float = 1e-12,
    window_size: int = 0,
    doc_ids: torch.Tensor | None = None,
) -> torch.Tensor:
    """Paired-heads Born attention (the attention core of ``SubspaceProjectorBornAttention`` with
    ``use_paired_heads=True`` and plain Born weights, ``layers/attention.py:591-626``).

    q, k, v are ``(B, H, T, D)`` CUDA tensors with H even.  Pair c is heads c and c + H/2 (the
    grouping the layer's reshape makes); every query of the pair attends the keys of both heads
    at each visible token (causal / window / document masks by token).  ``scale`` is a float, a
    0-d tensor or H/2 per-pair values (the layer passes
    ``clamp(head_scale.view(1, H/2, 2, 1, 1).mean(2), 0.5, 100)``).  Returns ``(B, H, T, D)`` in
    the autocast dtype (or v's dtype), differentiable in q, k, v and scale.
    """
    _check_inputs(q, k, v)
    if q.shape[1] % 2 != 0:
        raise ValueError(f"paired heads need an even number of heads; got {q.shape[1]}")
    dt = _target_dtype(q, v)
    if dt not in _DTYPE_CODE:
        raise ValueError(f"flash-Born (B200): unsupported dtype {dt}")
    scale_t = _as_param(scale, q.device)
    if scale_t.numel() not in (1, q.shape[1] // 2):
        raise ValueError(f"scale must have 1 or H/2={q.shape[1] // 2} elements, got {scale_t.numel()}")
    qc, kc, vc = (_prep(x.to(dt)) for x in (q, k, v))
    return _PairedHeadsBorn.apply(qc, kc, vc, _flat_f32(scale_t, q.device), _doc_i32(doc_ids, q.device),
                                  bool(is_causal), float(eps), int(window_size))
