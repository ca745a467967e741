"""GPU: the tcgen05 tensor-core kernels against the float64 oracle and the general CUDA path,
forced explicitly (FB_PATH_TCGEN05), across masks, ragged lengths, both head dims and both maps."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import flash_born_oracle as orc
from parity_util import lowp_gate, round_to
from quantumdlblocks_b200.kernels import flash_born as fbm

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("CUDA device required", allow_module_level=True)


def _fwd(q, k, v, scale, tau, doc, causal, window, purified, path):
    prev = fbm.get_kernel_path()
    fbm.set_kernel_path(path)
    try:
        out, z = torch.ops.flashborn_b200.born_fwd(q, k, v, scale, tau, doc, causal, 1e-12 if not purified else 1e-8,
                                                   window, 0.05, purified)
        launches = fbm.last_launch_count()
        torch.cuda.synchronize()
    finally:
        fbm.set_kernel_path(prev)
    return out, z, launches


def make_docs(rng, B, T, doc_mean):
    """Document ids: doc_mean > 0 packs documents of geometric length (ids rising along the
    sequence, as the reference's running count of end-of-text tokens gives); doc_mean < 0 packs
    row 0 that way and gives the other rows runs of ids drawn from {0, 1, 2}, so one id comes back
    after others (the kernels then compare ids pair by pair instead of using runs)."""
    if doc_mean is None:
        return None
    doc = np.zeros((B, T), np.int32)
    for b in range(B):
        t, d = 0, 0
        while t < T:
            L = int(rng.geometric(1 / abs(doc_mean)))
            doc[b, t:t + L] = d if (doc_mean > 0 or b == 0) else int(rng.integers(0, 3))
            t, d = t + L, d + 1
    return doc


CASES = [
    # B, H, T, D, causal, window, doc_mean (negative: ids that come back, see make_docs)
    (1, 1, 128, 64, True, 0, None),
    (1, 2, 1, 64, True, 0, None),
    (2, 2, 77, 64, True, 0, None),
    (1, 2, 300, 128, True, 0, None),
    (2, 3, 1000, 64, True, 0, None),
    (1, 2, 513, 64, False, 0, None),
    (1, 2, 700, 64, True, 100, None),
    (1, 2, 700, 128, False, 260, None),
    (2, 2, 900, 64, True, 0, 120.0),
    (1, 2, 640, 128, True, 0, 60.0),
    # long documents: most tiles lie inside one document and take the unmasked fast path
    (2, 2, 1500, 64, True, 0, 600.0),
    (1, 2, 1100, 128, True, 0, 500.0),
    # documents with a window, without the causal mask, and ids that come back in a later run
    (2, 2, 800, 64, True, 200, 150.0),
    (2, 2, 600, 64, False, 0, 150.0),
    (2, 2, 900, 64, True, 0, -120.0),
    (2, 2, 700, 128, True, 0, -80.0),
]


@pytest.mark.parametrize("purified", [False, True])
@pytest.mark.parametrize("case", CASES, ids=[str(c) for c in CASES])
def test_tc_forward_matches_oracle_and_general(case, purified):
    B, H, T, D, causal, window, doc_mean = case
    rng = np.random.default_rng(B * 7 + T + D)
    q, k, v = (rng.standard_normal((B, H, T, D)) for _ in range(3))
    if purified:
        q /= np.linalg.norm(q, axis=-1, keepdims=True)
        k /= np.linalg.norm(k, axis=-1, keepdims=True)
    q, k, v = (round_to(x, torch.bfloat16) for x in (q, k, v))
    doc = make_docs(rng, B, T, doc_mean)
    scale = np.linspace(6.0, 9.0, H).astype(np.float32) if purified else np.linspace(0.3, 0.5, H).astype(np.float32)
    tau = np.linspace(0.02, 0.08, H).astype(np.float32) if purified else None
    dev = "cuda"
    qt, kt, vt = (torch.tensor(x, dtype=torch.float32, device=dev).to(torch.bfloat16) for x in (q, k, v))
    st = torch.tensor(scale, device=dev)
    tt = None if tau is None else torch.tensor(tau, device=dev)
    dt = None if doc is None else torch.tensor(doc, device=dev)
    o_tc, z_tc, n_tc = _fwd(qt, kt, vt, st, tt, dt, causal, window, purified, "tcgen05")
    o_ge, z_ge, _ = _fwd(qt, kt, vt, st, tt, dt, causal, window, purified, "general")
    assert n_tc == (3 if doc is not None else 1)  # + the two document-span launches
    assert fbm.device_status() == (0, 0)
    if purified:
        ref, zref = orc.purified_forward(q, k, v, scale, tau, 0.05, causal, 1e-8, window, doc)
    else:
        ref, zref = orc.born_forward(q, k, v, scale, causal, 1e-12, window, doc)
    o_tc_np = o_tc.double().cpu().numpy()
    lowp_gate(o_tc_np, ref, "out(tcgen05)")
    lowp_gate(o_ge.double().cpu().numpy(), ref, "out(general)")
    # Z (saved for the backward, not returned): the tensor-core forward sums the bf16-rounded p that
    # its PV product consumes, so each term carries up to 2^-9 relative rounding
    np.testing.assert_allclose(z_tc.double().cpu().numpy(), zref, rtol=5e-3, atol=1e-30)
    np.testing.assert_allclose(z_tc.cpu().numpy(), z_ge.cpu().numpy(), rtol=5e-3)


def test_tc_forward_is_selected_for_bf16_d64_d128():
    x = torch.randn(1, 1, 64, 64, device="cuda", dtype=torch.bfloat16)
    fbm.flash_born_attention(x, x, x, 1.0)
    assert fbm.last_launch_count() == 1
    import ctypes

    from quantumdlblocks_b200 import _lib

    a = _lib.FbAttnArgs()
    a.batch, a.heads, a.seq_len, a.head_dim = 1, 1, 64, 64
    a.dtype = a.out_dtype = _lib.FB_BF16
    a.scale, a.scale_numel = x.data_ptr(), 1
    a.z = x.data_ptr()
    for n in ("q", "k", "v", "out"):
        setattr(a, n, x.data_ptr())
        setattr(a, n + "_stride", _lib._I64x4(*x.stride()))
    assert _lib.load().fb_select_path(ctypes.byref(a), 0) == _lib.FB_PATH_TCGEN05
    a.dtype = a.out_dtype = _lib.FB_F16
    assert _lib.load().fb_select_path(ctypes.byref(a), 0) == _lib.FB_PATH_GENERAL


# every forward case, plus shapes where CTAs walk several work items (windows of heads in the
# key-major kernel, LPT rounds in the query-major one) for both head dims
BWD_CASES = CASES + [
    (4, 8, 1024, 64, True, 0, None),
    (2, 3, 1536, 128, True, 0, None),
    (3, 5, 640, 64, False, 0, None),
]


@pytest.mark.parametrize("deterministic", [False, True], ids=["fused", "deterministic"])
@pytest.mark.parametrize("purified", [False, True])
@pytest.mark.parametrize("case", BWD_CASES, ids=[str(c) for c in BWD_CASES])
def test_tc_backward_matches_oracle(case, purified, deterministic):
    """Forward and backward both forced onto the tcgen05 kernels, against the oracle: d=64 through
    the fused backward and (deterministic mode) the two-kernel one; d=128 always takes the latter."""
    from parity_util import check_all, run_cuda, run_oracle

    B, H, T, D, causal, window, doc_mean = case
    if deterministic and D != 64:
        pytest.skip("d=128 always uses the two-kernel backward")
    rng = np.random.default_rng(B * 11 + T + D)
    q, k, v, do = (rng.standard_normal((B, H, T, D)) for _ in range(4))
    if purified:
        q /= np.linalg.norm(q, axis=-1, keepdims=True)
        k /= np.linalg.norm(k, axis=-1, keepdims=True)
    q, k, v, do = (round_to(x, torch.bfloat16) for x in (q, k, v, do))
    doc = make_docs(rng, B, T, doc_mean)
    scale = np.linspace(6.0, 9.0, H).astype(np.float32) if purified else np.linspace(0.3, 0.5, H).astype(np.float32)
    kw = dict(is_causal=causal, window_size=window, doc_ids=doc)
    if purified:
        kw["tau"] = np.linspace(0.02, 0.08, H).astype(np.float32)
    got = run_cuda("purified" if purified else "plain", q, k, v, do, scale, dtype=torch.bfloat16, path="tcgen05",
                   deterministic=deterministic, **kw)
    assert fbm.device_status() == (0, 0)
    ref = run_oracle("purified" if purified else "plain", q, k, v, do, scale, **kw)
    check_all(got, ref, lowp=True)


@pytest.mark.parametrize("D", [64, 128])
def test_tc_backward_deterministic_mode_is_bitwise_repeatable(D):
    """Under torch.use_deterministic_algorithms(True) two backward runs give identical bits."""
    from parity_util import run_cuda

    rng = np.random.default_rng(5)
    q, k, v, do = (round_to(rng.standard_normal((2, 3, 700, D)), torch.bfloat16) for _ in range(4))
    scale = np.full(3, 0.4, np.float32)
    a = run_cuda("plain", q, k, v, do, scale, dtype=torch.bfloat16, path="tcgen05", deterministic=True)
    b = run_cuda("plain", q, k, v, do, scale, dtype=torch.bfloat16, path="tcgen05", deterministic=True)
    for name in ("dq", "dk", "dv", "dscale"):
        assert np.array_equal(a[name], b[name]), name


@pytest.mark.parametrize("purified", [False, True])
@pytest.mark.parametrize("shape,doc_mean", [((8, 16, 2048, 64), None), ((2, 16, 4096, 64), 300.0)],
                         ids=["c2", "doc-masked"])
def test_fused_and_deterministic_backward_agree_at_full_size(shape, doc_mean, purified):
    """Benchmark-sized problems put many work items on every CTA (the cases above hold at most a
    few), which exercises the cross-item pipelines: the fused backward must finish with a clean
    device status and agree with the two-kernel deterministic backward."""
    B, H, T, D = shape
    g = torch.Generator().manual_seed(9)
    q, k, v, do = (torch.randn(B, H, T, D, generator=g) for _ in range(4))
    if purified:
        q, k = (x / x.norm(dim=-1, keepdim=True) for x in (q, k))
    q, k, v, do = (x.to("cuda", torch.bfloat16) for x in (q, k, v, do))
    doc = None
    if doc_mean is not None:
        rng = np.random.default_rng(3)
        d = np.zeros((B, T), np.int32)
        for b in range(B):
            t, n = 0, 0
            while t < T:
                L = int(rng.geometric(1 / doc_mean))
                d[b, t:t + L] = n
                t, n = t + L, n + 1
        doc = torch.tensor(d, device="cuda")
    scale = torch.linspace(6.0, 9.0, H, device="cuda") if purified else torch.full((H,), 8.0, device="cuda")
    tau = torch.linspace(0.02, 0.08, H, device="cuda") if purified else None
    eps = 1e-8 if purified else 1e-12
    fwd, bwd = torch.ops.flashborn_b200.born_fwd, torch.ops.flashborn_b200.born_bwd
    out, z = fwd(q, k, v, scale, tau, doc, True, eps, 0, 0.05, purified)
    prev = torch.are_deterministic_algorithms_enabled()
    res = {}
    try:
        for det in (False, True):
            torch.use_deterministic_algorithms(det)
            res[det] = bwd(do, q, k, v, out, z, scale, tau, doc, True, eps, 0, 0.05, purified)
            torch.cuda.synchronize()
            assert fbm.device_status() == (0, 0), f"device status after the {'split' if det else 'fused'} backward"
    finally:
        torch.use_deterministic_algorithms(prev)
    for idx, name in enumerate(("dq", "dk", "dv")):
        a, b = res[False][idx].float(), res[True][idx].float()
        assert torch.isfinite(a).all(), name
        err = (a - b).abs().max().item()
        assert err <= 1e-2 * b.abs().max().item(), (name, err, b.abs().max().item())
