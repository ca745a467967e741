"""Pin the complex-phase / paired-heads oracle against golden vectors that the reference
attention layer produced (tests/golden/make_golden_families.py)."""
from __future__ import annotations

import numpy as np
import pytest

from families_cases import family_case_names, head_scale_grad, layer_scale, load_family_case
from oracle import born_families_oracle as orc

# float64 results stored as float32; the oracle recomputes from the float32-rounded inputs
RTOL = 2e-5


def _close(x, ref, name):
    ref = np.asarray(ref, dtype=np.float64)
    err = np.abs(np.asarray(x, dtype=np.float64) - ref).max() / max(np.abs(ref).max(), 1e-30)
    assert err <= RTOL, f"{name}: max-rel {err:.3e}"


def test_fixtures_present():
    names = family_case_names()
    assert {n.split("_")[0] for n in names} == {"complex", "paired"}


@pytest.mark.parametrize("name", family_case_names())
def test_oracle_matches_reference_layer(name):
    c = load_family_case(name)
    q, k, v, do = (c[n].astype(np.float64) for n in ("q", "k", "v", "do"))
    sc = layer_scale(c)
    if c["family"] == "complex":
        out, _, dq, dk, dv, dsc = orc.complex_phase(q, k, v, do, sc, c["is_causal"], c["eps"], c["window_size"],
                                                    c["doc_ids"])
    else:
        out, dq, dk, dv, dsc = orc.paired_heads(q, k, v, do, sc, c["is_causal"], c["eps"], c["window_size"],
                                                c["doc_ids"])
    for n, x in (("out", out), ("dq", dq), ("dk", dk), ("dv", dv)):
        _close(x, c["ref_" + n], n)
    np.testing.assert_allclose(head_scale_grad(c, dsc), c["ref_dhead_scale"], rtol=1e-4, atol=1e-9)


def test_rot_is_the_imaginary_overlap():
    rng = np.random.default_rng(0)
    q, k = rng.standard_normal((2, 5, 8))
    half = 4
    s_im = q[:, :half] @ k[:, half:].T * 0 + q[:, half:] @ k[:, :half].T - q[:, :half] @ k[:, half:].T
    np.testing.assert_allclose(q @ orc.rot(k).T, s_im, rtol=1e-12, atol=1e-12)
    g = rng.standard_normal((5, 8))
    # rot_t is the adjoint of rot: <rot k, g> = <k, rot_t g>
    np.testing.assert_allclose((orc.rot(k) * g).sum(), (k * orc.rot_t(g)).sum(), rtol=1e-12)
