"""CPU oracle for flash-Born attention -- TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline leg may import it.  The product path (``quantumdlblocks_b200``) runs
the CUDA library and raises when it is missing; it never calls into this file.

It restates, in numpy, the reference algorithm of QuantumDLBlocks (``qdlblocks``,
``src/qdlblocks/kernels/flash_born.py``), materialising one (batch, head) score matrix at a time
(optionally in query chunks) so that it also runs at the benchmark shapes:

* plain forward      -- eager path ``flash_born.py:681-690`` and the Triton forward ``:80-192``
* plain backward     -- the analytic gradient of the Triton backward kernels ``:194-322`` (dK, dV,
  dscale) and ``:324-430`` (dQ)
* purified forward   -- eager path ``flash_born.py:1329-1341``, Triton forward ``:695-811``
* purified backward  -- Triton kernels ``:813-947`` and ``:949-1061``
* masks              -- ``_apply_window_and_doc_mask`` ``flash_born.py:635-652``
* document ids       -- ``compute_document_ids`` ``src/qdlblocks/layers/attention.py:308-315``

Parity pin: ``tests/golden/`` holds outputs of the reference itself (its eager CPU path and
autograd, run in float64 by ``tests/golden/make_golden.py``); ``tests/test_oracle_golden.py``
checks this module against them.

All arithmetic runs in the dtype of the inputs (pass float64 arrays for the gate oracle).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

__all__ = [
    "valid_mask",
    "compute_document_ids",
    "born_forward",
    "born_backward",
    "purified_forward",
    "purified_backward",
    "count_valid_pairs",
    "BornGrads",
]


def compute_document_ids(idx: np.ndarray, eot_token_id: int = 50256) -> np.ndarray:
    """Document index per token: an EOT token belongs to the document it ends.

    Restates ``compute_document_ids`` (``layers/attention.py:308-315``):
    ``cumsum(is_eot) - is_eot`` as int32.
    """
    is_eot = (np.asarray(idx) == int(eot_token_id)).astype(np.int32)
    return (np.cumsum(is_eot, axis=-1, dtype=np.int32) - is_eot).astype(np.int32)


def valid_mask(
    rows: np.ndarray,
    cols: np.ndarray,
    is_causal: bool,
    window_size: int,
    doc_rows: np.ndarray | None = None,
    doc_cols: np.ndarray | None = None,
) -> np.ndarray:
    """Boolean (len(rows), len(cols)) mask ``valid(i, j)``.

    ``flash_born.py:635-652``: ``diff = i - j``; causal keeps ``diff >= 0``; a window keeps
    ``diff < window`` (so a non-causal window still sees the whole future); document ids must be
    equal.
    """
    diff = rows[:, None].astype(np.int64) - cols[None, :].astype(np.int64)
    mask = (diff >= 0) if is_causal else np.ones(diff.shape, dtype=bool)
    if window_size > 0:
        mask &= diff < int(window_size)
    if doc_rows is not None:
        mask &= doc_rows[:, None] == doc_cols[None, :]
    return mask


def _per_head(x, heads: int, dtype) -> np.ndarray:
    """Scalar or per-head parameter -> (H,) array (``numel() > 1`` means per head, ``:452``)."""
    arr = np.asarray(x, dtype=dtype).reshape(-1)
    if arr.size == 1:
        return np.full((heads,), arr[0], dtype=dtype)
    if arr.size != heads:
        raise ValueError(f"per-head parameter has {arr.size} elements for {heads} heads")
    return arr


def _chunks(T: int, chunk: int):
    for m0 in range(0, T, chunk):
        yield m0, min(T, m0 + chunk)


def _key_span(m0: int, m1: int, T: int, is_causal: bool, window_size: int) -> tuple[int, int]:
    """Keys ``[lo, hi)`` that can pair with queries ``[m0, m1)``: causal stops at ``m1``; a window
    starts at ``m0 - window + 1`` (``diff < window``, ``flash_born.py:635-652``).  Pairs outside the
    span are masked anyway, so restricting the columns to it changes no result, only the cost."""
    lo = max(0, m0 - int(window_size) + 1) if window_size > 0 else 0
    hi = m1 if is_causal else T
    return lo, max(lo, hi)


def count_valid_pairs(T: int, is_causal: bool, window_size: int, doc_ids_row: np.ndarray | None) -> int:
    """Number of (i, j) pairs with valid(i, j) for one (batch, head) -- the FLOP-count unit."""
    if doc_ids_row is None:
        if not is_causal and window_size <= 0:
            return T * T
        total = 0
        for i in range(T):
            lo = 0 if window_size <= 0 else max(0, i - window_size + 1)
            hi = (i + 1) if is_causal else T
            total += max(0, hi - lo)
        return total
    ids = np.asarray(doc_ids_row)
    total = 0
    for i in range(T):
        lo = 0 if window_size <= 0 else max(0, i - window_size + 1)
        hi = (i + 1) if is_causal else T
        if hi > lo:
            total += int(np.count_nonzero(ids[lo:hi] == ids[i]))
    return total


# --------------------------------------------------------------------------------------------
# Plain Born
# --------------------------------------------------------------------------------------------


def born_forward(q, k, v, scale, is_causal=True, eps=1e-12, window_size=0, doc_ids=None, chunk=1024):
    """Plain flash-Born forward. Returns ``(out, z)`` with ``z = sum_j p_ij + eps``.

    ``flash_born.py:681-690`` (eager) / ``:156-191`` (kernel): ``a = relu(scale * q.k) * valid``,
    ``p = a^2``, ``out = (p @ v) / (sum p + eps)``.
    """
    q, k, v = np.asarray(q), np.asarray(k), np.asarray(v)
    B, H, T, D = q.shape
    dt = q.dtype
    sc = _per_head(scale, H, dt)
    out = np.zeros_like(v)
    z = np.zeros((B, H, T), dtype=dt)
    for b in range(B):
        for h in range(H):
            for m0, m1 in _chunks(T, chunk):
                rows = np.arange(m0, m1)
                c0, c1 = _key_span(m0, m1, T, is_causal, window_size)
                cols = np.arange(c0, c1)
                mask = valid_mask(rows, cols, is_causal, window_size,
                                  None if doc_ids is None else doc_ids[b, m0:m1],
                                  None if doc_ids is None else doc_ids[b, c0:c1])
                raw = q[b, h, m0:m1] @ k[b, h, c0:c1].T
                a = np.where(mask, np.maximum(raw * sc[h], 0), 0).astype(dt)
                p = a * a
                zz = p.sum(axis=1) + dt.type(eps)
                out[b, h, m0:m1] = (p @ v[b, h, c0:c1]) / zz[:, None]
                z[b, h, m0:m1] = zz
    return out, z


@dataclass
class BornGrads:
    dq: np.ndarray
    dk: np.ndarray
    dv: np.ndarray
    dscale: np.ndarray  # (H,) per head (sum to a scalar for a shared scale)
    dtau: np.ndarray | None = None


def born_backward(q, k, v, out, z, dout, scale, is_causal=True, window_size=0, doc_ids=None, chunk=1024):
    """Plain flash-Born backward (analytic), ``flash_born.py:267-312`` and ``:398-427``.

    ``w = p / Z``; ``dV = w^T dO``; ``delta_i = sum_d dO_i O_i``; ``dP = (dO V^T - delta) / Z``;
    ``dS = 2 a dP`` (masked); ``dscale_h = sum dS * raw``; ``dK = dS^T Q scale``;
    ``dQ = dS K scale``.  Returns per-head dscale.
    """
    q, k, v, out, z, dout = (np.asarray(x) for x in (q, k, v, out, z, dout))
    B, H, T, D = q.shape
    dt = q.dtype
    sc = _per_head(scale, H, dt)
    dq = np.zeros_like(q)
    dk = np.zeros_like(k)
    dv = np.zeros_like(v)
    dscale = np.zeros((H,), dtype=dt)
    for b in range(B):
        for h in range(H):
            for m0, m1 in _chunks(T, chunk):
                rows = np.arange(m0, m1)
                c0, c1 = _key_span(m0, m1, T, is_causal, window_size)
                cols = np.arange(c0, c1)
                mask = valid_mask(rows, cols, is_causal, window_size,
                                  None if doc_ids is None else doc_ids[b, m0:m1],
                                  None if doc_ids is None else doc_ids[b, c0:c1])
                raw = q[b, h, m0:m1] @ k[b, h, c0:c1].T
                a = np.where(mask, np.maximum(raw * sc[h], 0), 0).astype(dt)
                zz = z[b, h, m0:m1][:, None]
                w = (a * a) / zz
                do = dout[b, h, m0:m1]
                dv[b, h, c0:c1] += w.T @ do
                delta = np.sum(do * out[b, h, m0:m1], axis=1)[:, None]
                dp = (do @ v[b, h, c0:c1].T - delta) / zz
                ds = np.where(mask, 2 * a * dp, 0).astype(dt)
                dscale[h] += np.sum(ds * raw)
                dk[b, h, c0:c1] += (ds.T @ q[b, h, m0:m1]) * sc[h]
                dq[b, h, m0:m1] = (ds @ k[b, h, c0:c1]) * sc[h]
    return BornGrads(dq, dk, dv, dscale)


# --------------------------------------------------------------------------------------------
# Purified Born (degree-4 coherence-thresholded)
# --------------------------------------------------------------------------------------------


def purified_forward(q, k, v, gamma, tau, eps_base=0.05, is_causal=True, eps=1e-8, window_size=0,
                     doc_ids=None, chunk=1024):
    """Purified forward, ``flash_born.py:1329-1341`` / ``:782-808``.

    ``u = relu(gamma (raw - tau))``, ``b = relu(raw)``, ``p = u^4 + eps_base b^2`` (masked),
    ``out = (p @ v) / (sum p + eps)``.
    """
    q, k, v = np.asarray(q), np.asarray(k), np.asarray(v)
    B, H, T, D = q.shape
    dt = q.dtype
    g = _per_head(gamma, H, dt)
    t = _per_head(tau, H, dt)
    out = np.zeros_like(v)
    z = np.zeros((B, H, T), dtype=dt)
    for b in range(B):
        for h in range(H):
            for m0, m1 in _chunks(T, chunk):
                rows = np.arange(m0, m1)
                c0, c1 = _key_span(m0, m1, T, is_causal, window_size)
                cols = np.arange(c0, c1)
                mask = valid_mask(rows, cols, is_causal, window_size,
                                  None if doc_ids is None else doc_ids[b, m0:m1],
                                  None if doc_ids is None else doc_ids[b, c0:c1])
                raw = q[b, h, m0:m1] @ k[b, h, c0:c1].T
                u = np.where(mask, np.maximum(g[h] * (raw - t[h]), 0), 0).astype(dt)
                bb = np.where(mask, np.maximum(raw, 0), 0).astype(dt)
                p = (u * u) * (u * u) + dt.type(eps_base) * (bb * bb)
                zz = p.sum(axis=1) + dt.type(eps)
                out[b, h, m0:m1] = (p @ v[b, h, c0:c1]) / zz[:, None]
                z[b, h, m0:m1] = zz
    return out, z


def purified_backward(q, k, v, out, z, dout, gamma, tau, eps_base=0.05, is_causal=True, window_size=0,
                      doc_ids=None, chunk=1024):
    """Purified backward, ``flash_born.py:913-941`` and ``:1044-1058``.

    ``dP = (dO V^T - delta) / Z``; ``d_raw = 4 u^3 dP gamma + 2 eps_base b dP`` (masked);
    ``dgamma = sum 4 u^3 dP (raw - tau)``; ``dtau = -sum 4 u^3 dP gamma``;
    ``dK = d_raw^T Q``; ``dQ = d_raw K``.
    """
    q, k, v, out, z, dout = (np.asarray(x) for x in (q, k, v, out, z, dout))
    B, H, T, D = q.shape
    dt = q.dtype
    g = _per_head(gamma, H, dt)
    t = _per_head(tau, H, dt)
    eb = dt.type(eps_base)
    dq = np.zeros_like(q)
    dk = np.zeros_like(k)
    dv = np.zeros_like(v)
    dgamma = np.zeros((H,), dtype=dt)
    dtau = np.zeros((H,), dtype=dt)
    for b in range(B):
        for h in range(H):
            for m0, m1 in _chunks(T, chunk):
                rows = np.arange(m0, m1)
                c0, c1 = _key_span(m0, m1, T, is_causal, window_size)
                cols = np.arange(c0, c1)
                mask = valid_mask(rows, cols, is_causal, window_size,
                                  None if doc_ids is None else doc_ids[b, m0:m1],
                                  None if doc_ids is None else doc_ids[b, c0:c1])
                raw = q[b, h, m0:m1] @ k[b, h, c0:c1].T
                u = np.where(mask, np.maximum(g[h] * (raw - t[h]), 0), 0).astype(dt)
                bb = np.where(mask, np.maximum(raw, 0), 0).astype(dt)
                p = (u * u) * (u * u) + eb * (bb * bb)
                zz = z[b, h, m0:m1][:, None]
                do = dout[b, h, m0:m1]
                dv[b, h, c0:c1] += (p / zz).T @ do
                delta = np.sum(do * out[b, h, m0:m1], axis=1)[:, None]
                dp = (do @ v[b, h, c0:c1].T - delta) / zz
                du = 4 * (u * u * u) * dp
                draw = np.where(mask, du * g[h] + 2 * eb * bb * dp, 0).astype(dt)
                dgamma[h] += np.sum(du * (raw - t[h]))
                dtau[h] += np.sum(-du * g[h])
                dk[b, h, c0:c1] += draw.T @ q[b, h, m0:m1]
                dq[b, h, m0:m1] = draw @ k[b, h, c0:c1]
    return BornGrads(dq, dk, dv, dgamma, dtau)
