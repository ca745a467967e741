"""Flash-Born work split over ranks: one process per GPU, no collective on the data path.

Every (batch, head) unit of flash-Born attention is independent in the forward and in the
backward: the reference launches one program per (query tile, batch, head)
(``kernels/flash_born.py:121-123`` forward, ``:228-230`` and ``:354-356`` backward) and no
program reads another unit's rows.  A job over N GPUs therefore gives each rank a rectangle of
units, ``[b0, b1) x [h0, h1)``, runs the ordinary single-GPU op on that slice (strided views with
a unit inner stride are accepted as they are) and exchanges nothing while it computes.

The one cross-rank sum is the scale gradient: ``dscale_h`` is a sum over every batch row of head
``h`` (``flash_born.py:309`` and the per-head atomic at ``:319-322``), so a plan that splits the
batch leaves each rank a partial per-head sum; ``gather_param_grad`` adds the N partials (one
all-reduce of ``H`` floats), and with a head split it assembles the heads each rank owns.

Plans:
  * heads split evenly when ``H % world == 0`` (every head of a batch row has the same mask, so
    the split is exactly balanced, causal or document-masked, and no scale gradient is shared);
  * otherwise batch rows split into contiguous ranges that minimise the largest per-rank count of
    valid (query, key) pairs (document masks make rows unequal), which needs ``B >= world``.

``max_over_ranks`` is the timing rule of a multi-GPU measurement: a job takes as long as its
slowest rank.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

__all__ = ["Shard", "row_valid_pairs", "plan_shards", "shard_inputs", "gather_param_grad", "max_over_ranks"]


@dataclass(frozen=True)
class Shard:
    """Units ``[b0, b1) x [h0, h1)`` of rank ``rank``; ``pairs`` = valid (query, key) pairs in them."""

    rank: int
    b0: int
    b1: int
    h0: int
    h1: int
    pairs: int

    @property
    def units(self) -> int:
        return (self.b1 - self.b0) * (self.h1 - self.h0)


def _row_pairs_no_doc(T: int, is_causal: bool, window_size: int) -> int:
    i = np.arange(T, dtype=np.int64)
    hi = (i + 1) if is_causal else np.full(T, T, dtype=np.int64)
    lo = np.maximum(0, i - window_size + 1) if window_size > 0 else np.zeros(T, dtype=np.int64)
    return int(np.maximum(0, hi - lo).sum())


def row_valid_pairs(B: int, T: int, is_causal: bool = True, window_size: int = 0, doc_ids=None) -> np.ndarray:
    """Valid (query, key) pairs of one head of each batch row, ``(B,)`` int64.

    The mask is the reference's (``flash_born.py:169-178``): ``j <= i`` when causal,
    ``i - j < window`` when a window is set, equal document ids when ``doc_ids`` is given.
    """
    if doc_ids is None:
        return np.full(B, _row_pairs_no_doc(T, is_causal, window_size), dtype=np.int64)
    doc = doc_ids.detach().cpu().numpy() if isinstance(doc_ids, torch.Tensor) else np.asarray(doc_ids)
    if doc.shape != (B, T):
        raise ValueError(f"doc_ids must be (B, T) = ({B}, {T}), got {doc.shape}")
    out = np.zeros(B, dtype=np.int64)
    for b in range(B):
        row = doc[b]
        if window_size <= 0:
            # positions sharing an id form c(c+1)/2 causal pairs (c^2 without the causal mask),
            # whether or not the ids are sorted
            _, c = np.unique(row, return_counts=True)
            c = c.astype(np.int64)
            out[b] = int((c * (c + 1) // 2).sum()) if is_causal else int((c * c).sum())
            continue
        total = 0
        for t in range(T):
            lo = max(0, t - window_size + 1)
            hi = t + 1 if is_causal else T
            if hi > lo:
                total += int(np.count_nonzero(row[lo:hi] == row[t]))
        out[b] = total
    return out


def _linear_partition(costs: np.ndarray, parts: int) -> list[tuple[int, int]]:
    """Contiguous ranges of ``costs`` (``parts`` of them, none empty) minimising the largest sum."""
    n = len(costs)
    prefix = np.concatenate([[0], np.cumsum(costs, dtype=np.int64)])
    inf = np.iinfo(np.int64).max
    # best[k][i]: smallest max-sum splitting the first i items into k ranges
    best = np.full((parts + 1, n + 1), inf, dtype=np.int64)
    cut = np.zeros((parts + 1, n + 1), dtype=np.int64)
    best[0][0] = 0
    for k in range(1, parts + 1):
        for i in range(k, n - (parts - k) + 1):
            for j in range(k - 1, i):
                if best[k - 1][j] == inf:
                    continue
                v = max(best[k - 1][j], prefix[i] - prefix[j])
                if v < best[k][i]:
                    best[k][i] = v
                    cut[k][i] = j
    ranges, i = [], n
    for k in range(parts, 0, -1):
        j = int(cut[k][i])
        ranges.append((j, i))
        i = j
    return ranges[::-1]


def plan_shards(B: int, H: int, T: int, world: int, *, is_causal: bool = True, window_size: int = 0,
                doc_ids=None) -> list[Shard]:
    """One ``Shard`` per rank (index = rank); see the module docstring for the rule."""
    if world < 1:
        raise ValueError("world must be >= 1")
    rows = row_valid_pairs(B, T, is_causal, window_size, doc_ids)
    if H % world == 0:
        hs = H // world
        total = int(rows.sum())
        return [Shard(r, 0, B, r * hs, (r + 1) * hs, total * hs) for r in range(world)]
    if B >= world:
        return [Shard(r, b0, b1, 0, H, int(rows[b0:b1].sum()) * H)
                for r, (b0, b1) in enumerate(_linear_partition(rows, world))]
    raise ValueError(f"cannot split B={B} x H={H} units over {world} ranks: need H % world == 0 or B >= world")


def shard_inputs(shard: Shard, q, k, v, scale, doc_ids=None):
    """This rank's views of full ``(B, H, T, D)`` inputs: ``(q, k, v, scale, doc_ids)``.

    ``scale`` keeps its form: a float or single-element tensor is shared by every head; a per-head
    tensor (``(H,)`` or ``(1, H, 1, 1)``, ``flash_born.py:452``) is sliced to the shard's heads.
    """
    bs, hs = slice(shard.b0, shard.b1), slice(shard.h0, shard.h1)
    qs, ks, vs = (x[bs, hs] for x in (q, k, v))
    sc = scale
    if isinstance(scale, torch.Tensor) and scale.numel() > 1:
        sc = scale.reshape(-1)[hs].reshape(1, -1, 1, 1) if scale.dim() == 4 else scale.reshape(-1)[hs]
    doc = None if doc_ids is None else doc_ids[bs]
    return qs, ks, vs, sc, doc


def gather_param_grad(local: torch.Tensor, shard: Shard, H: int, per_head: bool = True, group=None) -> torch.Tensor:
    """The whole job's scale (or tau) gradient on every rank, from this rank's part.

    ``per_head``: ``local`` holds the shard's heads (``h1 - h0`` values); they are placed at their
    heads of an ``(H,)`` vector and summed over ranks, which assembles a head split and adds the
    partial sums over batch rows of a batch split.  Shared parameter: ``local`` is one value and
    the result is its sum over ranks, shape ``(1,)``.  One all-reduce either way.
    """
    import torch.distributed as dist

    flat = local.detach().reshape(-1).to(torch.float64)
    if per_head:
        if flat.numel() != shard.h1 - shard.h0:
            raise ValueError(f"expected {shard.h1 - shard.h0} per-head values, got {flat.numel()}")
        full = torch.zeros(H, dtype=torch.float64, device=flat.device)
        full[shard.h0:shard.h1] = flat
    else:
        if flat.numel() != 1:
            raise ValueError(f"a shared parameter has one gradient value, got {flat.numel()}")
        full = flat.clone()
    if dist.is_available() and dist.is_initialized():
        dist.all_reduce(full, op=dist.ReduceOp.SUM, group=group)
    return full


def max_over_ranks(values, device=None, group=None) -> list[float]:
    """Element-wise maximum over ranks of a list of floats (timings): one all-reduce."""
    import torch.distributed as dist

    t = torch.tensor([float(x) for x in values], dtype=torch.float64, device=device)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return [float(x) for x in t.tolist()]
