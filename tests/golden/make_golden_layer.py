"""Golden vectors of the reference attention layer's own flash-Born call, produced by the REFERENCE
layer itself (``qdlblocks.layers.attention.SubspaceProjectorBornAttention``) in float64 on CPU.

Run in a container where the reference source tree is available (it does not travel to GPU
machines):

    PYTHONPATH=<reference>/src python tests/golden/make_golden_layer.py <reference>/src

The layer calls ``flash_born_attention(Q, K, V, scale=clamp(head_scale, 1, 100), is_causal,
eps=self.eps, window_size, doc_ids)`` (``layers/attention.py:691-713``) and hands the result to
``_finalize_heads`` (head merge + ``out_proj``, ``:478-493``).  This script wraps the module
attribute the layer calls, so the reference's own function runs (its CPU eager path) while the
wrapper records the call's operands exactly as the layer formed them: Q, K (L2-normalised), V (after
value-residual mixing), the scale (a ``(1, H, 1, 1)`` clamped tensor, or the python float
``sqrt(head_dim)`` without a learnable temperature), ``is_causal``, ``eps``, ``window_size`` and the
document ids of ``compute_document_ids`` (``:308-315``) over token ids with end-of-text tokens.
The purified layer on CPU computes its core with ``purified_born_attention_weights`` (``:674-686``;
the flash path needs CUDA tensors, ``:640-656``), which is wrapped the same way to record Q, K,
``gamma = clamp(head_scale, 0.5, 20)``, ``tau = tau_max * sigmoid(tau_raw)`` and ``eps``.

Then ``sum(y * dy)`` of the layer output y is back-propagated through the layer's own graph and
the gradients reaching Q, K, V, the scale tensor, the core output (``dO``) and ``head_scale`` are
stored, with ``out_proj``'s weight, dy and y, so a test can replay the core call and the head merge
with the B200 op.  Writes ``tests/golden/layer_<case>.npz`` (float64 results stored as float32,
the head_scale gradient as float64).
"""
from __future__ import annotations

import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

CASES = {
    # name: dict of layer arguments and call arguments
    # the reference's module-level test configuration (tests/test_flash_born.py:17-67): B=2, T=64,
    # embed 128, 4 heads of 32, value-residual mixing with psi_0, both temperatures and causalities
    "plain_causal_learnable_hd32": dict(B=2, T=64, E=128, H=4, causal=True, learnable=True, window=0, eot=False,
                                        purified=False, seed=42),
    "plain_noncausal_fixed_hd32": dict(B=2, T=64, E=128, H=4, causal=False, learnable=False, window=0, eot=False,
                                       purified=False, seed=43),
    # the GPT call: 64-dim heads, a 384-token sliding window and end-of-text document ids
    "plain_window384_eot_hd64": dict(B=2, T=448, E=128, H=2, causal=True, learnable=True, window=384, eot=True,
                                     purified=False, seed=44),
    "purified_causal_eot_hd64": dict(B=2, T=160, E=128, H=2, causal=True, learnable=True, window=0, eot=True,
                                     purified=True, seed=45),
}


def _tokens(B: int, T: int, seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    idx = torch.randint(0, 50000, (B, T), generator=g)
    eot = torch.rand(B, T, generator=g) < 0.02  # documents of ~50 tokens
    return torch.where(eot, torch.full_like(idx, 50256), idx)


def _run_case(attn_mod, B, T, E, H, causal, learnable, window, eot, purified, seed):
    torch.manual_seed(seed)
    layer = attn_mod.SubspaceProjectorBornAttention(
        embed_dim=E, num_heads=H, block_size=T, is_causal=causal, learnable_temperature=learnable,
        value_residual_mixing=True, use_flash_born=True, use_purified_attn=purified).double()
    hd = E // H
    if layer.head_scale is not None:
        with torch.no_grad():  # distinct per-head values, inside the clamps' pass-through range
            lo, hi = (4.0, 11.0) if purified else (0.8 * math.sqrt(hd), 1.3 * math.sqrt(hd))
            layer.head_scale.copy_(torch.linspace(lo, hi, H, dtype=torch.float64).view(1, H, 1, 1))
    x = attn_mod.l2_normalize(torch.randn(B, T, E, dtype=torch.float64), dim=-1).requires_grad_(True)
    psi0 = attn_mod.l2_normalize(torch.randn(B, T, E, dtype=torch.float64), dim=-1)
    doc = attn_mod.compute_document_ids(_tokens(B, T, seed)) if eot else None

    rec: dict = {}

    def keep(name, t):
        if isinstance(t, torch.Tensor) and t.requires_grad:
            t.retain_grad()
        rec[name] = t

    if purified:
        orig = attn_mod.purified_born_attention_weights

        def spy(q, k, gamma, tau, eps_base, causal, eps, window_size, doc_ids):
            keep("q", q), keep("k", k), keep("scale", gamma), keep("tau", tau)
            rec.update(eps_base=eps_base, is_causal=causal, eps=eps, window_size=window_size, doc_ids=doc_ids)
            return orig(q, k, gamma=gamma, tau=tau, eps_base=eps_base, causal=causal, eps=eps,
                        window_size=window_size, doc_ids=doc_ids)

        def spy_finalize(out_heads, V, psi_in, B_, T_, D_):
            keep("out", out_heads), keep("v", V)
            return orig_finalize(out_heads, V, psi_in, B_, T_, D_)

        attn_mod.purified_born_attention_weights = spy
    else:
        orig = attn_mod.flash_born_attention

        def spy(Q, K, V, scale, is_causal, eps, window_size, doc_ids):
            keep("q", Q), keep("k", K), keep("v", V), keep("scale", scale)
            rec.update(is_causal=is_causal, eps=eps, window_size=window_size, doc_ids=doc_ids)
            out = orig(Q, K, V, scale=scale, is_causal=is_causal, eps=eps, window_size=window_size, doc_ids=doc_ids)
            keep("out", out)
            return out

        attn_mod.flash_born_attention = spy
    orig_finalize = layer._finalize_heads
    if purified:
        layer._finalize_heads = spy_finalize
    try:
        y = layer(x, psi_0=psi0, window_size=window, doc_ids=doc)
    finally:
        if purified:
            attn_mod.purified_born_attention_weights = orig
        else:
            attn_mod.flash_born_attention = orig
    dy = torch.randn(y.shape, dtype=torch.float64, generator=torch.Generator().manual_seed(seed + 100))
    (y * dy).sum().backward()

    f32 = lambda t: t.detach().numpy().astype(np.float32)  # noqa: E731
    sc = rec["scale"]
    res = {
        "kind": np.array("purified" if purified else "plain"),
        "is_causal": np.array(bool(rec["is_causal"])), "window_size": np.array(int(rec["window_size"])),
        "eps": np.array(float(rec["eps"])),
        "has_doc": np.array(rec["doc_ids"] is not None),
        "doc_ids": np.array(0) if rec["doc_ids"] is None else rec["doc_ids"].numpy().astype(np.int32),
        "scale_is_tensor": np.array(isinstance(sc, torch.Tensor)),
        "scale": (sc.detach().numpy() if isinstance(sc, torch.Tensor) else np.array(sc)).astype(np.float64),
        "q": f32(rec["q"]), "k": f32(rec["k"]), "v": f32(rec["v"]),
        "ref_out": f32(rec["out"]), "ref_dout": f32(rec["out"].grad),
        "ref_dq": f32(rec["q"].grad), "ref_dk": f32(rec["k"].grad), "ref_dv": f32(rec["v"].grad),
        "out_proj_weight": f32(layer.out_proj.weight), "dy": f32(dy), "ref_y": f32(y),
    }
    if isinstance(sc, torch.Tensor):
        res["ref_dscale"] = sc.grad.detach().numpy().astype(np.float64)
        res["ref_dhead_scale"] = layer.head_scale.grad.detach().numpy().astype(np.float64)
    if purified:
        res["eps_base"] = np.array(float(rec["eps_base"]))
        res["tau"] = rec["tau"].detach().numpy().astype(np.float64)
        res["ref_dtau"] = rec["tau"].grad.detach().numpy().astype(np.float64)
    return res


def main(src: str) -> None:
    if src not in sys.path:
        sys.path.insert(0, src)
    import warnings

    warnings.filterwarnings("ignore")
    import qdlblocks.layers.attention as attn_mod

    for name, spec in CASES.items():
        arrays = _run_case(attn_mod, **spec)
        np.savez_compressed(os.path.join(HERE, f"layer_{name}.npz"), **arrays)
        print(name, {k: v.shape for k, v in arrays.items() if v.ndim})


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden_layer.py <reference>/src")
    main(sys.argv[1])
