"""Pin the oracle against the reference attention layer's own flash-Born calls (CPU).

``tests/golden/make_golden_layer.py`` ran ``SubspaceProjectorBornAttention`` (plain flash-Born and
purified configurations, float64) and recorded the operands of its core call as the layer formed
them -- L2-normalised Q and K, mixed V, the ``(1, H, 1, 1)`` clamped scale or the python float
``sqrt(head_dim)``, a 384-token window, end-of-text document ids -- with the gradients the
layer's backward delivered to each of them.  The oracle must reproduce the core's output and
gradients from those operands; the GPU replay of the same calls through the B200 op lives in
``test_gpu_layer_swap.py``.
"""
from __future__ import annotations

import numpy as np
import pytest

from layer_cases import layer_case_names, load_layer_case
from oracle import flash_born_oracle as orc

RTOL = 1e-5  # float32-stored fixtures; the purified layer forms its overlaps in float32


def _rel(x, r):
    x, r = np.asarray(x, np.float64), np.asarray(r, np.float64)
    return float(np.abs(x - r).max() / max(np.abs(r).max(), 1e-30))


def test_layer_cases_present():
    names = layer_case_names()
    assert {"plain_causal_learnable_hd32", "plain_window384_eot_hd64", "purified_causal_eot_hd64"} <= set(names)


@pytest.mark.parametrize("name", layer_case_names())
def test_oracle_reproduces_layer_core_call(name):
    c = load_layer_case(name)
    q, k, v, do = (c[n].astype(np.float64) for n in ("q", "k", "v", "ref_dout"))
    sc = np.asarray(c["scale"], np.float64)
    if c["kind"] == "plain":
        out, z = orc.born_forward(q, k, v, sc, c["is_causal"], c["eps"], c["window_size"], c["doc_ids"])
        g = orc.born_backward(q, k, v, out, z, do, sc, c["is_causal"], c["window_size"], c["doc_ids"])
    else:
        out, z = orc.purified_forward(q, k, v, sc, c["tau"], c["eps_base"], c["is_causal"], c["eps"],
                                      c["window_size"], c["doc_ids"])
        g = orc.purified_backward(q, k, v, out, z, do, sc, c["tau"], c["eps_base"], c["is_causal"],
                                  c["window_size"], c["doc_ids"])
    for n, got in (("out", out), ("dq", g.dq), ("dk", g.dk), ("dv", g.dv)):
        assert _rel(got, c["ref_" + n]) <= RTOL, (n, _rel(got, c["ref_" + n]))
    if c["scale_is_tensor"]:
        assert _rel(g.dscale.reshape(c["ref_dscale"].shape), c["ref_dscale"]) <= 1e-4
        # inside the clamp's pass-through range the layer parameter's gradient is the scale's
        np.testing.assert_allclose(c["ref_dhead_scale"], c["ref_dscale"], rtol=1e-12)
    if c["kind"] == "purified":
        assert _rel(g.dtau.reshape(c["ref_dtau"].shape), c["ref_dtau"]) <= 1e-4


def test_layer_merge_replays_out_proj():
    """The recorded head merge: y = out.transpose(1, 2).reshape(B, T, H*hd) @ W_out^T."""
    for name in layer_case_names():
        c = load_layer_case(name)
        B, H, T, hd = c["ref_out"].shape
        merged = c["ref_out"].astype(np.float64).transpose(0, 2, 1, 3).reshape(B, T, H * hd)
        y = merged @ c["out_proj_weight"].astype(np.float64).T
        assert _rel(y, c["ref_y"]) <= 1e-5, name
