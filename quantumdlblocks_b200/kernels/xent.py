"""The GPT training loss as native kernels: mean cross-entropy over bf16 logits.

Replaces ``F.cross_entropy(logits.reshape(-1, V), targets)`` of the reference's GPTs
(``models/born_gpt.py:1291``), which under bf16 autocast materialises an fp32 copy of the logits
and runs log-softmax forward and backward over it.  ``cross_entropy(logits, targets)`` reads the
bf16 logits once in the forward (per-row log-sum-exp) and once in the backward, where it writes
the bf16 gradient ``(softmax - onehot) * g / rows`` directly.  CUDA only, like every op here.
"""
from __future__ import annotations

import ctypes

import torch

from .. import _lib
from .flash_born import _stream_handle

__all__ = ["cross_entropy"]


def _args(logits: torch.Tensor, targets: torch.Tensor, lse: torch.Tensor) -> _lib.FbXentArgs:
    a = _lib.FbXentArgs()
    a.rows, a.vocab, a.ld = logits.shape[0], logits.shape[1], logits.stride(0)
    a.logits, a.targets, a.lse = logits.data_ptr(), targets.data_ptr(), lse.data_ptr()
    return a


class _CrossEntropy(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        lse = torch.empty(logits.shape[0], dtype=torch.float32, device=logits.device)
        loss = torch.empty_like(lse)
        a = _args(logits, targets, lse)
        a.loss = loss.data_ptr()
        with torch.cuda.device(logits.device):
            _lib.check(_lib.load().fb_xent_fwd(ctypes.byref(a), _stream_handle(logits.device)), "cross-entropy")
        ctx.save_for_backward(logits, targets, lse)
        return loss.mean()

    @staticmethod
    def backward(ctx, g: torch.Tensor):
        logits, targets, lse = ctx.saved_tensors
        grad = torch.empty_like(logits)
        gs = g.detach().to(torch.float32).reshape(1).contiguous()
        a = _args(logits, targets, lse)
        a.grad, a.gscale = grad.data_ptr(), gs.data_ptr()
        with torch.cuda.device(logits.device):
            _lib.check(_lib.load().fb_xent_bwd(ctypes.byref(a), _stream_handle(logits.device)),
                       "cross-entropy backward")
        return grad, None


def cross_entropy(logits: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
    """Mean cross-entropy of ``logits (N, V)`` bf16 (rows 16-byte aligned, V a multiple of 8;
    ``-inf`` columns take no probability) against ``targets (N,)`` int64, differentiable in the
    logits; the same value as ``F.cross_entropy(logits.float(), targets)``."""
    if not logits.is_cuda:
        raise RuntimeError("cross_entropy (B200): logits must be a CUDA tensor; there is no CPU path")
    if logits.dim() != 2 or logits.dtype != torch.bfloat16 or logits.stride(1) != 1:
        raise ValueError(f"cross_entropy (B200) takes 2-D bf16 logits with unit column stride; got "
                         f"{tuple(logits.shape)} {logits.dtype} strides {logits.stride()}")
    if targets.shape != (logits.shape[0],):
        raise ValueError(f"targets must have shape ({logits.shape[0]},); got {tuple(targets.shape)}")
    return _CrossEntropy.apply(logits, targets.to(torch.int64).contiguous())
