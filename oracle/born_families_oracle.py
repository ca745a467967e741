"""Numpy restatement of the reference's complex-phase and paired-heads Born attention -- TEST
INFRASTRUCTURE ONLY (the checker of the CUDA path in tests/; never imported by the product).

Both live inside ``SubspaceProjectorBornAttention.forward`` of the reference as eager PyTorch:

  complex phase  ``layers/attention.py:717-730`` (two overlaps s_re, s_im of the [re | im] halves,
                 ``p = relu(a s_re)^2 + relu(a s_im)^2``), then the mask and normalisation of
                 ``:737-758`` (``w = p / (sum p + eps)``, ``out = w @ V``)
  paired heads   ``layers/attention.py:591-626`` (heads reshaped into (B, H/2, 2T, D), token mask
                 ``idx // 2``, ``p = relu(a s)^2``, same normalisation, reshaped back)

Dense float64 per (batch, head) unit with the analytic backward (the scale gradient summed
explicitly, ``sum dS * raw``); small sizes only.  Pinned against golden vectors that the
reference layer itself produced (tests/golden/make_golden_families.py).
"""
from __future__ import annotations

import numpy as np


def token_mask(tok: np.ndarray, is_causal: bool, window_size: int, doc_row) -> np.ndarray:
    """valid[i, j] for rows / columns at token positions tok (``layers/attention.py:741-752``)."""
    diff = tok[:, None] - tok[None, :]
    m = (diff >= 0) if is_causal else np.ones(diff.shape, dtype=bool)
    if window_size > 0:
        m = m & (diff < window_size)
    if doc_row is not None:
        d = np.asarray(doc_row)
        m = m & (d[:, None] == d[None, :])
    return m


def _unit(q, ks, v, do, a, mask, eps):
    """One (batch, head) unit of a sum of Born score families: q (T, D), ks the key matrices of
    the families, p = sum_f relu(a q ks_f^T)^2 masked.  Returns out, dq, [dk_f], dv, dscale."""
    raws = [q @ k.T for k in ks]
    amps = [np.maximum(a * r, 0.0) * mask for r in raws]
    p = sum(x * x for x in amps)
    z = p.sum(-1, keepdims=True)
    zz = z + eps
    w = p / zz
    out = w @ v
    dv = w.T @ do
    delta = (do * out).sum(-1, keepdims=True)
    dp = (do @ v.T - delta) / zz
    dq = np.zeros_like(q)
    dks, da = [], 0.0
    for r, am, k in zip(raws, amps, ks):
        ds = 2.0 * am * dp            # dL / d(a raw)
        da += float((ds * r).sum())
        dq += a * (ds @ k)
        dks.append(a * (ds.T @ q))
    return out, zz[:, 0], dq, dks, dv, da


def _scale_of(scale, n):
    s = np.asarray(scale, dtype=np.float64).reshape(-1)
    return s if s.size == n else np.full(n, float(s[0]))


def rot(k: np.ndarray) -> np.ndarray:
    """rot k = [-k_im | k_re], so <q, rot k> = q_im . k_re - q_re . k_im (``:726-728``)."""
    half = k.shape[-1] // 2
    return np.concatenate((-k[..., half:], k[..., :half]), axis=-1)


def rot_t(g: np.ndarray) -> np.ndarray:
    half = g.shape[-1] // 2
    return np.concatenate((g[..., half:], -g[..., :half]), axis=-1)


def complex_phase(q, k, v, do, scale, is_causal=True, eps=1e-12, window_size=0, doc_ids=None):
    """Forward and backward of complex-phase Born attention; q, k, v, do (B, H, T, D).
    Returns out, z, dq, dk, dv, dscale (shape of scale: 1 or H entries)."""
    B, H, T, D = q.shape
    sc = _scale_of(scale, H)
    out, dq, dk, dv = (np.zeros((B, H, T, D)) for _ in range(4))
    z = np.zeros((B, H, T))
    dsc = np.zeros(H)
    tok = np.arange(T)
    for b in range(B):
        m = token_mask(tok, is_causal, window_size, None if doc_ids is None else doc_ids[b])
        for h in range(H):
            kk = k[b, h]
            o, zz, gq, (gk1, gk2), gv, ga = _unit(q[b, h], [kk, rot(kk)], v[b, h], do[b, h], sc[h], m, eps)
            out[b, h], z[b, h], dq[b, h], dv[b, h] = o, zz, gq, gv
            dk[b, h] = gk1 + rot_t(gk2)
            dsc[h] += ga
    n = np.asarray(scale).size
    return out, z, dq, dk, dv, (dsc if n == H else np.array([dsc.sum()]))


def paired_heads(q, k, v, do, scale, is_causal=True, eps=1e-12, window_size=0, doc_ids=None):
    """Forward and backward of paired-heads Born attention; q, k, v, do (B, H, T, D), scale 1 or
    H/2 entries (one per pair).  Pair c interleaves heads c and c + H/2 token by token, as the
    reference's ``transpose(1, 2).reshape(B, 2T, H/2, D)`` does (``:595-597``)."""
    B, H, T, D = q.shape
    P = H // 2
    sc = _scale_of(scale, P)
    out, dq, dk, dv = (np.zeros((B, H, T, D)) for _ in range(4))
    dsc = np.zeros(P)
    tok = np.arange(2 * T) // 2

    def pair(x, b, c):  # (2T, D): row 2t + a = head c + aP at token t
        return np.stack((x[b, c], x[b, c + P]), axis=1).reshape(2 * T, D)

    def unpair(y):      # inverse of pair
        y = y.reshape(T, 2, D)
        return y[:, 0], y[:, 1]

    for b in range(B):
        doc2 = None if doc_ids is None else np.repeat(np.asarray(doc_ids[b]), 2)
        m = token_mask(tok, is_causal, window_size, doc2)
        for c in range(P):
            o, _, gq, (gk,), gv, ga = _unit(pair(q, b, c), [pair(k, b, c)], pair(v, b, c), pair(do, b, c), sc[c], m,
                                            eps)
            out[b, c], out[b, c + P] = unpair(o)
            dq[b, c], dq[b, c + P] = unpair(gq)
            dk[b, c], dk[b, c + P] = unpair(gk)
            dv[b, c], dv[b, c + P] = unpair(gv)
            dsc[c] += ga
    n = np.asarray(scale).size
    return out, dq, dk, dv, (dsc if n == P else np.array([dsc.sum()]))
