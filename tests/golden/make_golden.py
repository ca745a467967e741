"""Generate golden vectors for flash-Born from the REFERENCE implementation itself.

Run in a container where the reference source tree is available (it is read-only there and
does not travel to GPU machines):

    PYTHONPATH=<reference>/src python tests/golden/make_golden.py <reference>/src

For every case this script draws seeded inputs, runs the reference's public entry points
``qdlblocks.kernels.flash_born.flash_born_attention`` / ``flash_purified_born_attention`` on CPU
tensors (their eager path, ``flash_born.py:681-690`` and ``:1329-1341``) in float64, takes
gradients with torch autograd, and writes inputs + outputs to ``tests/golden/<case>.npz``.
It also writes checksums of configuration C1 (B=2, H=4, N=256, d=64, fp32, causal, per-head
scale 8, eps 1e-12, Q/K/V from torch seed 0, dO from seed 1) in float32 and float64.

The committed .npz files are what the tests read; this script is only needed to regenerate them.
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _import_reference(src: str):
    if src not in sys.path:
        sys.path.insert(0, src)
    import warnings

    warnings.filterwarnings("ignore")
    from qdlblocks.kernels.flash_born import flash_born_attention, flash_purified_born_attention
    from qdlblocks.layers.attention import compute_document_ids

    return flash_born_attention, flash_purified_born_attention, compute_document_ids


def _l2n(x: np.ndarray) -> np.ndarray:
    return x / np.maximum(np.linalg.norm(x, axis=-1, keepdims=True), 1e-12)


def _run(fn, q, k, v, do, params: dict, grad_params: tuple[str, ...]):
    """Run the reference in float64 with autograd; return dict of numpy outputs."""
    qt = torch.tensor(q, dtype=torch.float64, requires_grad=True)
    kt = torch.tensor(k, dtype=torch.float64, requires_grad=True)
    vt = torch.tensor(v, dtype=torch.float64, requires_grad=True)
    kw = {}
    leaves = {}
    for name, val in params.items():
        if isinstance(val, np.ndarray) and name != "doc_ids":
            t = torch.tensor(val, dtype=torch.float64, requires_grad=name in grad_params)
            kw[name] = t
            leaves[name] = t
        elif name == "doc_ids" and val is not None:
            kw[name] = torch.tensor(val, dtype=torch.int32)
        else:
            kw[name] = val
    out = fn(qt, kt, vt, **kw)
    (out * torch.tensor(do, dtype=torch.float64)).sum().backward()
    res = {"out": out.detach().numpy(), "dq": qt.grad.numpy(), "dk": kt.grad.numpy(), "dv": vt.grad.numpy()}
    for name in grad_params:
        res["d" + name] = leaves[name].grad.numpy()
    return res


def main(src: str) -> None:
    fb, fpb, cdi = _import_reference(src)
    cases = {}

    # g_causal: fp32-valued inputs, causal, shared scale (python float), D=32
    rng = np.random.default_rng(101)
    B, H, T, D = 2, 2, 64, 32
    q, k, v, do = (rng.standard_normal((B, H, T, D)).astype(np.float32) for _ in range(4))
    cases["plain_causal_d32"] = dict(
        kind="plain", q=q, k=k, v=v, do=do,
        params=dict(scale=np.array(0.75, dtype=np.float32), is_causal=True, eps=1e-12, window_size=0, doc_ids=None),
        grad=("scale",))

    # non-causal, per-head (H,) scale, D=64, L2-normalised q/k (the caller's contract)
    rng = np.random.default_rng(202)
    B, H, T, D = 1, 3, 48, 64
    q = _l2n(rng.standard_normal((B, H, T, D))).astype(np.float32)
    k = _l2n(rng.standard_normal((B, H, T, D))).astype(np.float32)
    v, do = (rng.standard_normal((B, H, T, D)).astype(np.float32) for _ in range(2))
    cases["plain_noncausal_perhead_d64"] = dict(
        kind="plain", q=q, k=k, v=v, do=do,
        params=dict(scale=np.array([6.0, 8.0, 11.0], dtype=np.float32), is_causal=False, eps=1e-12,
                    window_size=0, doc_ids=None),
        grad=("scale",))

    # ragged T, D=48, causal + window 20, (1,H,1,1) scale
    rng = np.random.default_rng(303)
    B, H, T, D = 1, 2, 77, 48
    q, k, v, do = (rng.standard_normal((B, H, T, D)).astype(np.float32) for _ in range(4))
    cases["plain_window_ragged_d48"] = dict(
        kind="plain", q=q, k=k, v=v, do=do,
        params=dict(scale=np.array([0.5, 0.3], dtype=np.float32).reshape(1, 2, 1, 1), is_causal=True, eps=1e-12,
                    window_size=20, doc_ids=None),
        grad=("scale",))

    # window 4 + EOT document ids (the reference's own mask test, shapes b=2 h=4 t=8 d=16)
    idx = torch.tensor([[10, 20, 50256, 30, 40, 50256, 50, 60], [11, 50256, 22, 33, 44, 55, 66, 77]])
    doc = cdi(idx, eot_token_id=50256).numpy().astype(np.int32)
    rng = np.random.default_rng(404)
    B, H, T, D = 2, 4, 8, 16
    q = _l2n(rng.standard_normal((B, H, T, D)))
    k = _l2n(0.85 * q + 0.15 * rng.standard_normal((B, H, T, D)))
    v = _l2n(rng.standard_normal((B, H, T, D)))
    q, k, v = (x.astype(np.float32) for x in (q, k, v))
    do = rng.standard_normal((B, H, T, D)).astype(np.float32)
    cases["plain_window4_doc_t8"] = dict(
        kind="plain", q=q, k=k, v=v, do=do,
        params=dict(scale=np.array(10.0, dtype=np.float32), is_causal=True, eps=1e-12, window_size=4, doc_ids=doc),
        grad=("scale",))
    cases["purified_window4_doc_t8"] = dict(
        kind="purified", q=q, k=k, v=v, do=do,
        params=dict(scale=np.full((H,), 8.0, dtype=np.float32), tau=np.zeros((H,), dtype=np.float32),
                    eps_base=0.05, is_causal=True, eps=1e-8, window_size=4, doc_ids=doc),
        grad=("scale", "tau"))

    # document mask over a longer row (geometric doc lengths), causal, D=64, T=200
    rng = np.random.default_rng(505)
    B, H, T, D = 2, 1, 160, 32
    lens = []
    doc = np.zeros((B, T), dtype=np.int32)
    for b in range(B):
        t, d = 0, 0
        while t < T:
            L = int(rng.geometric(1.0 / 40.0))
            doc[b, t:t + L] = d
            t += L
            d += 1
    q, k, v, do = (rng.standard_normal((B, H, T, D)).astype(np.float32) for _ in range(4))
    q = (_l2n(q) * 4.0).astype(np.float32)
    k = (_l2n(k) * 4.0).astype(np.float32)
    cases["plain_doc_geometric_t160"] = dict(
        kind="plain", q=q, k=k, v=v, do=do,
        params=dict(scale=np.array([2.0], dtype=np.float32), is_causal=True, eps=1e-12, window_size=0,
                    doc_ids=doc),
        grad=("scale",))

    # purified, causal, per-head gamma/tau (the reference's bf16 parity shape family, fp64 here)
    rng = np.random.default_rng(606)
    B, H, T, D = 1, 3, 96, 64
    q = _l2n(rng.standard_normal((B, H, T, D))).astype(np.float32)
    k = _l2n(rng.standard_normal((B, H, T, D))).astype(np.float32)
    v = _l2n(rng.standard_normal((B, H, T, D))).astype(np.float32)
    do = rng.standard_normal((B, H, T, D)).astype(np.float32)
    cases["purified_causal_perhead_d64"] = dict(
        kind="purified", q=q, k=k, v=v, do=do,
        params=dict(scale=np.linspace(4.0, 11.0, H).astype(np.float32).reshape(1, H, 1, 1),
                    tau=np.linspace(0.03, 0.09, H).astype(np.float32).reshape(1, H, 1, 1),
                    eps_base=0.05, is_causal=True, eps=1e-8, window_size=0, doc_ids=None),
        grad=("scale", "tau"))

    # purified, non-causal, scalar gamma/tau, ragged T, D=128
    rng = np.random.default_rng(707)
    B, H, T, D = 1, 1, 45, 128
    q = _l2n(rng.standard_normal((B, H, T, D))).astype(np.float32)
    k = _l2n(q + 0.5 * rng.standard_normal((B, H, T, D))).astype(np.float32)
    v, do = (rng.standard_normal((B, H, T, D)).astype(np.float32) for _ in range(2))
    cases["purified_noncausal_d128"] = dict(
        kind="purified", q=q, k=k, v=v, do=do,
        params=dict(scale=np.array(8.0, dtype=np.float32), tau=np.array(0.0625, dtype=np.float32),
                    eps_base=0.05, is_causal=False, eps=1e-8, window_size=0, doc_ids=None),
        grad=("scale", "tau"))

    # zero-overlap rows: q rows orthogonal-ish with negative overlaps -> Z == eps rows
    rng = np.random.default_rng(808)
    B, H, T, D = 1, 1, 33, 16
    q = rng.standard_normal((B, H, T, D)).astype(np.float32)
    k = (-q + 0.01 * rng.standard_normal((B, H, T, D))).astype(np.float32)
    v, do = (rng.standard_normal((B, H, T, D)).astype(np.float32) for _ in range(2))
    cases["plain_zero_rows_d16"] = dict(
        kind="plain", q=q, k=k, v=v, do=do,
        params=dict(scale=np.array(1.0, dtype=np.float32), is_causal=True, eps=1e-12, window_size=0, doc_ids=None),
        grad=("scale",))

    # eps large enough that the parameter gradients are far from zero, so the closed forms of the
    # B200 backward (dscale = (2 / scale) sum eps delta / Z, dgamma = (4 / gamma)(sum eps delta / Z
    # - sum eps_base b^2 dP)) are gated relative to their own size.  The first mirrors the shape,
    # seed, eps 1e-6 and per-head (H,) scale of the reference's JAX parity test
    # (tests/test_jax_haliax.py:74-135, torch side).
    rng = np.random.default_rng(123)
    B, H, T, D = 2, 2, 16, 8
    q, k, v, do = (rng.standard_normal((B, H, T, D)).astype(np.float32) for _ in range(4))
    cases["plain_eps1e-6_perhead_d8"] = dict(
        kind="plain", q=q, k=k, v=v, do=do,
        params=dict(scale=np.array([2.5, 3.2], dtype=np.float32), is_causal=True, eps=1e-6, window_size=0,
                    doc_ids=None),
        grad=("scale",))
    rng = np.random.default_rng(1)
    B, H, T, D = 1, 3, 200, 64
    q = _l2n(rng.standard_normal((B, H, T, D))).astype(np.float32)
    k = _l2n(rng.standard_normal((B, H, T, D))).astype(np.float32)
    v, do = (rng.standard_normal((B, H, T, D)).astype(np.float32) for _ in range(2))
    cases["plain_eps1e-2_perhead_d64"] = dict(
        kind="plain", q=q, k=k, v=v, do=do,
        params=dict(scale=np.array([2.0, 4.0, 8.0], dtype=np.float32).reshape(1, H, 1, 1), is_causal=True,
                    eps=1e-2, window_size=0, doc_ids=None),
        grad=("scale",))
    rng = np.random.default_rng(3)
    B, H, T, D = 2, 2, 150, 64
    q = _l2n(rng.standard_normal((B, H, T, D))).astype(np.float32)
    k = _l2n(rng.standard_normal((B, H, T, D))).astype(np.float32)
    v, do = (rng.standard_normal((B, H, T, D)).astype(np.float32) for _ in range(2))
    cases["plain_eps0.5_window_shared_d64"] = dict(
        kind="plain", q=q, k=k, v=v, do=do,
        params=dict(scale=np.array(3.0, dtype=np.float32), is_causal=False, eps=0.5, window_size=40,
                    doc_ids=None),
        grad=("scale",))
    rng = np.random.default_rng(2)
    B, H, T, D = 1, 3, 200, 64
    q = _l2n(rng.standard_normal((B, H, T, D))).astype(np.float32)
    k = _l2n(rng.standard_normal((B, H, T, D))).astype(np.float32)
    v, do = (rng.standard_normal((B, H, T, D)).astype(np.float32) for _ in range(2))
    cases["purified_eps0.3_perhead_d64"] = dict(
        kind="purified", q=q, k=k, v=v, do=do,
        params=dict(scale=np.array([4.0, 8.0, 11.0], dtype=np.float32),
                    tau=np.array([0.02, 0.05, 0.08], dtype=np.float32),
                    eps_base=0.05, is_causal=True, eps=0.3, window_size=0, doc_ids=None),
        grad=("scale", "tau"))

    manifest = {}
    for name, c in cases.items():
        fn = fb if c["kind"] == "plain" else fpb
        res = _run(fn, c["q"], c["k"], c["v"], c["do"], c["params"], c["grad"])
        arrays = {"q": c["q"], "k": c["k"], "v": c["v"], "do": c["do"]}
        meta = {"kind": c["kind"]}
        for pn, pv in c["params"].items():
            if isinstance(pv, np.ndarray) and pn != "doc_ids":
                arrays["param_" + pn] = pv
            elif pn == "doc_ids":
                if pv is not None:
                    arrays["doc_ids"] = pv
            else:
                meta[pn] = pv
        for rn, rv in res.items():
            # computed in float64 by the reference; stored rounded to float32 to keep fixtures small
            arrays["ref_" + rn] = rv.astype(np.float32)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **arrays)
        manifest[name] = meta

    # C1 checksums (fp32 and fp64 runs of the reference on the seeded C1 inputs)
    torch.manual_seed(0)
    q = torch.randn(2, 4, 256, 64)
    k = torch.randn(2, 4, 256, 64)
    v = torch.randn(2, 4, 256, 64)
    torch.manual_seed(1)
    do = torch.randn(2, 4, 256, 64)
    c1 = {}
    sample_rng = np.random.default_rng(9)
    sample_idx = sample_rng.integers(0, 2 * 4 * 256 * 64, size=64)
    for dt_name, dt in (("f32", torch.float32), ("f64", torch.float64)):
        qt, kt, vt = (x.to(dt).clone().requires_grad_(True) for x in (q, k, v))
        sc = torch.full((1, 4, 1, 1), 8.0, dtype=dt, requires_grad=True)
        out = fb(qt, kt, vt, scale=sc, is_causal=True, eps=1e-12)
        (out * do.to(dt)).sum().backward()
        entry = {}
        for nm, tns in (("out", out), ("dq", qt.grad), ("dk", kt.grad), ("dv", vt.grad)):
            a = tns.detach().to(torch.float64).numpy().reshape(-1)
            entry[nm] = {"sum": float(a.sum()), "sumsq": float((a * a).sum()), "maxabs": float(np.abs(a).max()),
                         "sample": [float(a[i]) for i in sample_idx]}
        entry["dscale"] = [float(x) for x in sc.grad.reshape(-1).to(torch.float64).numpy()]
        c1[dt_name] = entry
    c1["sample_idx"] = [int(i) for i in sample_idx]
    manifest["C1"] = {"kind": "plain", "shape": [2, 4, 256, 64], "scale": 8.0, "eps": 1e-12, "is_causal": True,
                      "checksums": c1}
    with open(os.path.join(HERE, "manifest.json"), "w") as f:
        json.dump(manifest, f, indent=1, sort_keys=True)
    print("wrote", len(cases), "cases + C1 checksums to", HERE)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("QDL_REFERENCE_SRC", ""))
