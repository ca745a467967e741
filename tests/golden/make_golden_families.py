"""Golden vectors for complex-phase and paired-heads Born attention, produced by the REFERENCE
attention layer itself (``qdlblocks.layers.attention.SubspaceProjectorBornAttention`` with
``complex_phase=True`` or ``use_paired_heads=True``), in float64 on CPU.

Run in a container where the reference source tree is available (it does not travel to GPU
machines):

    PYTHONPATH=<reference>/src python tests/golden/make_golden_families.py <reference>/src

The attention core sits inside the layer's forward, so this script records its operands and
result while the layer runs: the last two ``l2_normalize`` results before the head merge are the
normalised Q and K (``layers/attention.py:588-589``), and ``_finalize_heads`` receives the core's
output and V (``:478``).  The per-head scale is the layer's ``head_scale`` parameter
(``clamp(head_scale, 1, 100)`` for complex phase, ``:691-695``; the pair mean clamped to
[0.5, 100] for paired heads, ``:598-601``).  Gradients of ``sum(out * dO)`` with respect to Q, K,
V and ``head_scale`` come from torch autograd through the layer's own graph.  Writes
``tests/golden/families_<case>.npz`` (float64 results stored as float32).
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

CASES = {
    # name: (family, B, H, T, D, is_causal, window, with_docs, seed)
    "complex_causal_d64": ("complex", 1, 4, 80, 64, True, 0, False, 11),
    "complex_noncausal_window_doc_d16": ("complex", 2, 2, 40, 16, False, 7, True, 12),
    "paired_causal_d64": ("paired", 1, 4, 80, 64, True, 0, False, 13),
    "paired_window_doc_d16": ("paired", 1, 4, 40, 16, True, 5, True, 14),
}


def _run_case(attn_mod, family, B, H, T, D, is_causal, window, with_docs, seed):
    torch.manual_seed(seed)
    E = H * D
    layer = attn_mod.SubspaceProjectorBornAttention(
        embed_dim=E, num_heads=H, block_size=T, is_causal=is_causal, learnable_temperature=True,
        complex_phase=family == "complex", use_paired_heads=family == "paired").double()
    with torch.no_grad():  # per-head scales inside the clamps' pass-through range
        layer.head_scale.copy_(torch.linspace(2.0, 9.0, H, dtype=torch.float64).view(1, H, 1, 1))
    x = torch.randn(B, T, E, dtype=torch.float64)
    doc = None
    if with_docs:
        g = torch.Generator().manual_seed(seed)
        doc = torch.cumsum((torch.rand(B, T, generator=g) < 0.12).to(torch.int64), dim=1).to(torch.int32)

    seen: list[torch.Tensor] = []
    orig_l2n = attn_mod.l2_normalize

    def spy_l2n(t, *a, **kw):
        r = orig_l2n(t, *a, **kw)
        seen.append(r)
        return r

    got = {}

    def spy_finalize(out_heads, V, psi_in, B_, T_, D_):
        got["out"], got["v"] = out_heads, V
        got["q"], got["k"] = seen[-2], seen[-1]
        return out_heads.transpose(1, 2).contiguous().view(B_, T_, D_)

    attn_mod.l2_normalize = spy_l2n
    layer._finalize_heads = spy_finalize
    try:
        layer(x, window_size=window, doc_ids=doc)
    finally:
        attn_mod.l2_normalize = orig_l2n
    q, k, v, out = got["q"], got["k"], got["v"], got["out"]
    do = torch.randn(out.shape, dtype=torch.float64, generator=torch.Generator().manual_seed(seed + 100))
    dq, dk, dv, dhs = torch.autograd.grad(out, (q, k, v, layer.head_scale), do)
    f32 = lambda t: t.detach().numpy().astype(np.float32)  # noqa: E731
    return {
        "family": np.array(family), "is_causal": np.array(is_causal), "window_size": np.array(window),
        "eps": np.array(layer.eps), "doc_ids": np.array(0) if doc is None else doc.numpy(),
        "has_doc": np.array(doc is not None), "head_scale": layer.head_scale.detach().reshape(-1).numpy(),
        "q": f32(q), "k": f32(k), "v": f32(v), "do": f32(do),
        "ref_out": f32(out), "ref_dq": f32(dq), "ref_dk": f32(dk), "ref_dv": f32(dv),
        "ref_dhead_scale": dhs.reshape(-1).numpy(),
    }


def main(src: str) -> None:
    if src not in sys.path:
        sys.path.insert(0, src)
    import warnings

    warnings.filterwarnings("ignore")
    import qdlblocks.layers.attention as attn_mod

    for name, spec in CASES.items():
        arrays = _run_case(attn_mod, *spec)
        np.savez_compressed(os.path.join(HERE, f"families_{name}.npz"), **arrays)
        print(name, {k: v.shape for k, v in arrays.items() if v.ndim})


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden_families.py <reference>/src")
    main(sys.argv[1])
