"""Torch-CPU restatement of the reference's eager flash-Born path -- TEST/BASELINE ONLY.

Used only by ``bench.py``'s CPU-baseline leg (``cpu_baseline`` and ``--impl reference``) to
time the reference's own CPU algorithm on the host cores; never by the product path.

It follows ``flash_born_attention``'s CPU branch (``src/qdlblocks/kernels/flash_born.py:681-690``):
``matmul(q, k^T) * scale -> relu -> square -> mask (:635-652) -> / (sum + eps) -> matmul(., v)``
with torch autograd for the backward, exactly as the reference computes on CPU.  To bound
memory at benchmark sizes it runs one (batch, head) unit at a time (the reference materialises
all units at once, which needs B*H*N^2 floats per intermediate).
"""
from __future__ import annotations

import torch


def eager_unit_fwd_bwd(q, k, v, do, scale: float, is_causal: bool = True, eps: float = 1e-12,
                       window_size: int = 0, doc_row=None):
    """Forward + backward of one (batch, head) unit: q, k, v, do are (T, D) CPU tensors."""
    q = q.detach().requires_grad_(True)
    k = k.detach().requires_grad_(True)
    v = v.detach().requires_grad_(True)
    T = q.shape[0]
    prob = torch.relu(torch.matmul(q, k.transpose(-1, -2)) * scale).square()
    if is_causal or window_size > 0 or doc_row is not None:
        idx = torch.arange(T)
        diff = idx[:, None] - idx[None, :]
        mask = (diff >= 0) if is_causal else torch.ones((T, T), dtype=torch.bool)
        if window_size > 0:
            mask = mask & (diff < window_size)
        if doc_row is not None:
            mask = mask & (doc_row[:, None] == doc_row[None, :])
        prob = prob * mask.to(prob.dtype)
    w = prob / (prob.sum(dim=-1, keepdim=True) + eps)
    out = torch.matmul(w, v)
    dq, dk, dv = torch.autograd.grad(out, (q, k, v), do)
    return out.detach(), dq, dk, dv
