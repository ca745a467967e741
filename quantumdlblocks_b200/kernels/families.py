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
row ``Z = sum_t Z_t`` is the family's ``sum p + eps`` and ``O = sum_t O_t Z_t / Z``
(``fb_combine_terms``, one pass).  The backward runs ``fb_born_bwd_term`` per term with the
combined O and Z (the term's share of dQ, dK, dV) and forms the scale gradient from the closed
form of a score homogeneous of degree 2 in the scale, ``(2 / a_h) sum_{b,i} eps delta_i / Z_i``
with ``delta_i = dO_i . O_i`` (``fb_delta_terms``).  ``rot k`` and the adjoint rotation of its
gradient are ``fb_rotate_halves``.
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


def _combine(terms, out: torch.Tensor, z: torch.Tensor) -> None:
    """fb_combine_terms: out = sum O_t Z_t / sum Z_t, z = sum Z_t over terms [(O_t fp32, Z_t)];
    out (B, H', T, D) and z (B, H', T) may be strided views."""
    B, H, T, D = terms[0][0].shape
    a = _lib.FbCombineArgs()
    a.batch, a.heads, a.seq_len, a.head_dim = B, H, T, D
    a.n_terms = len(terms)
    a.out_dtype = _DTYPE_CODE[out.dtype]
    for i, (o_t, z_t) in enumerate(terms):
        a.o[i], a.z[i] = _ptr(o_t), _ptr(z_t)
    a.out, a.out_stride = _ptr(out), _strides(out)
    a.z_out = _ptr(z)
    a.z_stride = (ctypes.c_int64 * 3)(*z.stride())
    with torch.cuda.device(out.device):
        _lib.check(_lib.load().fb_combine_terms(ctypes.byref(a), _stream_handle(out.device)), "combine terms")


def _rotate(b: torch.Tensor, a: Optional[torch.Tensor] = None, adjoint: bool = False) -> torch.Tensor:
    """fb_rotate_halves: a + R b (adjoint: a + R^T b) per row of the last dimension."""
    b = b.contiguous()
    a = None if a is None else a.contiguous()  # held until the launch is enqueued
    dst = torch.empty_like(b)
    r = _lib.FbRotArgs()
    r.rows, r.head_dim = b.numel() // b.shape[-1], b.shape[-1]
    r.dtype, r.adjoint = _DTYPE_CODE[b.dtype], int(adjoint)
    r.a = None if a is None else _ptr(a)
    r.b, r.dst = _ptr(b), _ptr(dst)
    with torch.cuda.device(b.device):
        _lib.check(_lib.load().fb_rotate_halves(ctypes.byref(r), _stream_handle(b.device)), "rotate halves")
    return dst


def _scale_grad(dout, out, z, scale, eps, heads_of_row):
    """(2 / a_e) sum eps delta_i / Z_i per scale entry e (fb_delta_terms gives per-(b, h, 64-row) sums;
    heads_of_row maps the per-head sums onto scale entries)."""
    B, H, T, D = out.shape
    part = torch.empty((B, H, (T + 63) // 64), dtype=torch.float32, device=out.device)
    a = _lib.FbDeltaArgs()
    a.batch, a.heads, a.seq_len, a.head_dim = B, H, T, D
    a.dout_dtype, a.out_dtype = _DTYPE_CODE[dout.dtype], _DTYPE_CODE[out.dtype]
    a.eps = float(eps)
    a.dout, a.dout_stride = _ptr(dout), _strides(dout)
    a.out, a.out_stride = _ptr(out), _strides(out)
    a.z, a.part = _ptr(z), _ptr(part)
    with torch.cuda.device(out.device):
        _lib.check(_lib.load().fb_delta_terms(ctypes.byref(a), _stream_handle(out.device)), "scale gradient")
    per_head = part.sum(dim=(0, 2))
    if scale.numel() == 1:
        return (2.0 / scale) * per_head.sum().reshape(1)
    return (2.0 / scale) * heads_of_row(per_head)


class _ComplexPhaseBorn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, scale, doc, is_causal, eps, window_size):
        kr = _rotate(k)
        terms = [_born_fwd(q, kk, v, scale, None, doc, is_causal, eps / 2, window_size, 0.0, False, False, True)
                 for kk in (k, kr)]
        B, H, T, D = q.shape
        out = torch.empty((B, H, T, D), dtype=v.dtype, device=v.device)
        z = torch.empty((B, H, T), dtype=torch.float32, device=v.device)
        _combine(terms, out, z)
        ctx.save_for_backward(q, k, kr, v, out, z, scale, doc)
        ctx.cfg = (is_causal, eps, window_size)
        return out

    @staticmethod
    def backward(ctx, dout):
        q, k, kr, v, out, z, scale, doc = ctx.saved_tensors
        is_causal, eps, window_size = ctx.cfg
        dout = _prep(dout.to(v.dtype))
        dq1, dk1, dv1 = _born_bwd_term(dout, q, k, v, out, z, scale, doc, is_causal, eps / 2, window_size)
        dq2, dkr, dv2 = _born_bwd_term(dout, q, kr, v, out, z, scale, doc, is_causal, eps / 2, window_size)
        dk = _rotate(dkr, dk1, adjoint=True)
        dscale = _scale_grad(dout, out, z, scale, eps, lambda x: x)
        return dq1.add_(dq2), dk, dv1.add_(dv2), dscale, None, None, None, None


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
        B, H, T, D = q.shape
        P = H // 2
        half = lambda x, a: x[:, a * P:(a + 1) * P]  # noqa: E731  head half a: (B, P, T, D) view
        out = torch.empty((B, H, T, D), dtype=v.dtype, device=v.device)
        z = torch.empty((B, H, T), dtype=torch.float32, device=v.device)
        for a in (0, 1):
            terms = [_born_fwd(half(q, a), half(k, b), half(v, b), scale, None, doc, is_causal, eps / 2,
                               window_size, 0.0, False, False, True) for b in (0, 1)]
            _combine(terms, half(out, a), half(z, a))
        ctx.save_for_backward(q, k, v, out, z, scale, doc)
        ctx.cfg = (is_causal, eps, window_size)
        return out

    @staticmethod
    def backward(ctx, dout):
        q, k, v, out, z, scale, doc = ctx.saved_tensors
        is_causal, eps, window_size = ctx.cfg
        P = q.shape[1] // 2
        dout = _prep(dout.to(v.dtype))
        half = lambda x, a: x[:, a * P:(a + 1) * P]  # noqa: E731
        g = {}
        for a in (0, 1):
            for b in (0, 1):
                g[a, b] = _born_bwd_term(half(dout, a), half(q, a), half(k, b), half(v, b), half(out, a),
                                         half(z, a).contiguous(), scale, doc, is_causal, eps / 2, window_size)
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        for x in (0, 1):  # query half x gathers over key halves; key half x over query halves
            torch.add(g[x, 0][0], g[x, 1][0], out=half(dq, x))
            torch.add(g[0, x][1], g[1, x][1], out=half(dk, x))
            torch.add(g[0, x][2], g[1, x][2], out=half(dv, x))
        dscale = _scale_grad(dout, out, z, scale, eps, lambda x: x[:P] + x[P:])
        return dq, dk, dv, dscale, None, None, None, None


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
