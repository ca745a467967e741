"""GPU: the reference attention layer's own flash-Born calls replayed through the B200 op.

``tests/golden/make_golden_layer.py`` recorded, from ``SubspaceProjectorBornAttention`` itself
(``layers/attention.py:691-715``, float64), the operands of the layer's core call -- L2-normalised
Q and K, value-mixed V, the ``(1, H, 1, 1)`` clamped ``head_scale`` (or the python float
``sqrt(head_dim)`` without a learnable temperature), ``window_size`` 384, end-of-text document
ids -- plus ``out_proj``'s weight, the layer's output y and the upstream gradient dy.

Each case calls the binding ``swap.install()`` gives the layer module (the token-major
``flash_born_attention`` for the plain layer, ``flash_purified_born_attention`` for the purified
one) with the layer's exact keyword call, then runs the layer's head merge
(``out.transpose(1, 2).contiguous().view(B, T, D)``, ``:492``) and ``out_proj`` and
back-propagates ``sum(y * dy)``:

* fp32: y, the core output and the gradients of Q, K, V, the scale tensor (= the ``head_scale``
  gradient inside the clamp's range) and tau against the reference layer's own values;
* bf16 under autocast (how the GPTs call it): against the float64 oracle on the rounded operands.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from layer_cases import layer_case_names, load_layer_case
from oracle import flash_born_oracle as orc
from parity_util import check_all, fp32_gate, lowp_gate, round_to
from quantumdlblocks_b200 import swap
from quantumdlblocks_b200.kernels import flash_born as fbm

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("CUDA device required", allow_module_level=True)


def _binding(kind: str):
    if kind == "plain":
        return swap.LAYER_OVERRIDES[("qdlblocks.layers.attention", "flash_born_attention")]
    return swap.REPLACEMENTS["flash_purified_born_attention"]


def _replay(c: dict, dtype: torch.dtype):
    dev = "cuda"
    q, k, v = (torch.tensor(c[n], device=dev).requires_grad_(True) for n in ("q", "k", "v"))
    B, H, T, hd = q.shape
    scale = torch.tensor(c["scale"], dtype=torch.float32, device=dev).requires_grad_(True) \
        if c["scale_is_tensor"] else float(c["scale"])
    doc = None if c["doc_ids"] is None else torch.tensor(c["doc_ids"], device=dev)
    w = torch.tensor(c["out_proj_weight"], device=dev)
    dy = torch.tensor(c["dy"], device=dev)
    tau = None
    fn = _binding(c["kind"])
    with torch.autocast("cuda", dtype=torch.bfloat16, enabled=dtype == torch.bfloat16):
        if c["kind"] == "plain":
            out = fn(q, k, v, scale=scale, is_causal=c["is_causal"], eps=c["eps"], window_size=c["window_size"],
                     doc_ids=doc)
            assert out.transpose(1, 2).is_contiguous()  # token-major: the merge below is a view
        else:
            tau = torch.tensor(c["tau"], dtype=torch.float32, device=dev).requires_grad_(True)
            out = fn(q, k, v, scale=scale, tau=tau, eps_base=c["eps_base"], is_causal=c["is_causal"], eps=c["eps"],
                     window_size=c["window_size"], doc_ids=doc)
        out.retain_grad()
        merged = out.transpose(1, 2).contiguous().view(B, T, H * hd)
        y = torch.nn.functional.linear(merged, w.to(merged.dtype))
    (y.float() * dy).sum().backward()
    torch.cuda.synchronize()
    assert fbm.device_status() == (0, 0)
    res = {"y": y, "out": out, "dout": out.grad, "dq": q.grad, "dk": k.grad, "dv": v.grad}
    if isinstance(scale, torch.Tensor):
        res["dscale"] = scale.grad
    if tau is not None:
        res["dtau"] = tau.grad
    return {n: t.detach().double().cpu().numpy() for n, t in res.items()}


@pytest.mark.parametrize("name", layer_case_names())
def test_layer_call_fp32_matches_reference_layer(name):
    c = load_layer_case(name)
    got = _replay(c, torch.float32)
    for n in ("y", "out", "dq", "dk", "dv"):
        fp32_gate(got[n], c["ref_" + n], n)
    gscale = max(1.0, float(np.abs(c["ref_dq"]).max()), float(np.abs(c["ref_dk"]).max()))
    for n in ("dscale", "dtau"):
        if "ref_" + n in c:
            err = float(np.abs(got[n].reshape(c["ref_" + n].shape) - c["ref_" + n]).max())
            assert err <= 1e-4 * gscale, (n, err, gscale)
    if "ref_dhead_scale" in c:  # the layer parameter's gradient (clamp pass-through)
        err = float(np.abs(got["dscale"].reshape(c["ref_dhead_scale"].shape) - c["ref_dhead_scale"]).max())
        assert err <= 1e-4 * gscale


@pytest.mark.parametrize("name", layer_case_names())
def test_layer_call_bf16_autocast_matches_oracle(name):
    c = load_layer_case(name)
    got = _replay(c, torch.bfloat16)
    q, k, v = (round_to(c[n], torch.bfloat16) for n in ("q", "k", "v"))
    # the incoming core gradient of this run (bf16 merge + out_proj), rounded as the op consumes it
    do = round_to(got["dout"], torch.bfloat16)
    sc = np.asarray(c["scale"], np.float64)
    if c["kind"] == "plain":
        out, z = orc.born_forward(q, k, v, sc, c["is_causal"], c["eps"], c["window_size"], c["doc_ids"])
        g = orc.born_backward(q, k, v, out, z, do, sc, c["is_causal"], c["window_size"], c["doc_ids"])
    else:
        out, z = orc.purified_forward(q, k, v, sc, c["tau"], c["eps_base"], c["is_causal"], c["eps"],
                                      c["window_size"], c["doc_ids"])
        g = orc.purified_backward(q, k, v, out, z, do, sc, c["tau"], c["eps_base"], c["is_causal"],
                                  c["window_size"], c["doc_ids"])
    ref = {"out": out, "dq": g.dq, "dk": g.dk, "dv": g.dv}
    if c["scale_is_tensor"]:
        ref["dscale"] = g.dscale.reshape(c["ref_dscale"].shape)
    if c["kind"] == "purified":
        ref["dtau"] = g.dtau.reshape(c["ref_dtau"].shape)
    check_all(got, ref, lowp=True)
    # and the layer output itself against the reference layer's float64 y
    lowp_gate(got["y"], c["ref_y"], "y")
