"""GPU parity of the complex-phase and paired-heads Born attention (sums of plain Born terms run
on the flash-Born kernels, backward through fb_born_bwd_term) against the reference layer's
golden vectors and the float64 oracle, and of the token-major output layout of the plain op."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from families_cases import family_case_names, head_scale_grad, layer_scale, load_family_case
from oracle import born_families_oracle as orc
from parity_util import check_all, round_to

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # collected on CPU hosts, skipped there
    pytest.skip("CUDA device required", allow_module_level=True)

from quantumdlblocks_b200 import (complex_phase_born_attention, flash_born_attention,  # noqa: E402
                                  paired_heads_born_attention)
from quantumdlblocks_b200 import _lib  # noqa: E402
from quantumdlblocks_b200.kernels import flash_born as fbm  # noqa: E402

FAMILY_FN = {"complex": complex_phase_born_attention, "paired": paired_heads_born_attention}


def _run(family, q, k, v, do, scale, dtype, path="auto", **kw):
    dev = torch.device("cuda")
    t = [torch.tensor(np.asarray(x), dtype=torch.float32, device=dev).to(dtype).requires_grad_(True)
         for x in (q, k, v)]
    sc = torch.tensor(np.asarray(scale, dtype=np.float32), device=dev).requires_grad_(True)
    doc = kw.pop("doc_ids", None)
    if doc is not None:
        doc = torch.tensor(np.asarray(doc), dtype=torch.int32, device=dev)
    prev = fbm.get_kernel_path()
    fbm.set_kernel_path(path)
    try:
        out = FAMILY_FN[family](*t, sc, doc_ids=doc, **kw)
        g = torch.autograd.grad(out, (*t, sc), torch.tensor(np.asarray(do), dtype=torch.float32,
                                                           device=dev).to(out.dtype))
        torch.cuda.synchronize()
    finally:
        fbm.set_kernel_path(prev)
    rc, site = fbm.device_status()
    assert rc == 0, f"device status {rc} at site {site}"
    res = dict(zip(("out", "dq", "dk", "dv", "dscale"), (out, *g)))
    return {n: x.detach().to(torch.float64).cpu().numpy() for n, x in res.items()}


def _oracle(family, q, k, v, do, scale, **kw):
    if family == "complex":
        out, _, dq, dk, dv, dsc = orc.complex_phase(q, k, v, do, scale, **kw)
    else:
        out, dq, dk, dv, dsc = orc.paired_heads(q, k, v, do, scale, **kw)
    return dict(out=out, dq=dq, dk=dk, dv=dv, dscale=dsc)


def _kw(c):
    return dict(is_causal=c["is_causal"], eps=c["eps"], window_size=c["window_size"], doc_ids=c["doc_ids"])


@pytest.mark.parametrize("name", family_case_names())
def test_family_golden_fp32(name):
    """fp32 inputs (general kernels, given-normaliser backward) against the reference layer's own
    float64 results, through the layer's head_scale chain rule."""
    c = load_family_case(name)
    sc = layer_scale(c)
    got = _run(c["family"], c["q"], c["k"], c["v"], c["do"], sc, torch.float32, **_kw(c))
    ref = {n: c["ref_" + n] for n in ("out", "dq", "dk", "dv")}
    check_all(got, ref, lowp=False)
    gscale = max(1.0, float(np.abs(ref["dq"]).max()), float(np.abs(ref["dk"]).max()))
    np.testing.assert_allclose(head_scale_grad(c, got["dscale"]), c["ref_dhead_scale"], rtol=0, atol=1e-4 * gscale)


@pytest.mark.parametrize("path", ["auto", "general"])
@pytest.mark.parametrize("name", family_case_names())
def test_family_golden_bf16(name, path):
    """bf16 inputs (tensor-core kernels for head_dim 64) against the float64 oracle on the rounded
    inputs."""
    c = load_family_case(name)
    q, k, v, do = (round_to(c[n], torch.bfloat16) for n in ("q", "k", "v", "do"))
    sc = layer_scale(c)
    got = _run(c["family"], q, k, v, do, sc, torch.bfloat16, path=path, **_kw(c))
    check_all(got, _oracle(c["family"], q, k, v, do, sc, **_kw(c)), lowp=True,
              names=("out", "dq", "dk", "dv", "dscale"))


@pytest.mark.parametrize("family", ["complex", "paired"])
@pytest.mark.parametrize("D,T,window,docs,shared", [(64, 300, 0, False, False), (128, 200, 0, True, False),
                                                     (64, 257, 33, True, True)])
def test_family_tensor_core_shapes(family, D, T, window, docs, shared):
    """Ragged sequence lengths, head_dim 64 and 128, window and document masks, shared and
    per-head (per-pair) scales, on the tensor-core path."""
    rng = np.random.default_rng(D + T)
    B, H = 2, 4
    q, k = (rng.standard_normal((B, H, T, D)) for _ in range(2))
    q /= np.linalg.norm(q, axis=-1, keepdims=True)
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v, do = (rng.standard_normal((B, H, T, D)) for _ in range(2))
    q, k, v, do = (round_to(x, torch.bfloat16) for x in (q, k, v, do))
    n_sc = 1 if shared else (H if family == "complex" else H // 2)
    sc = np.linspace(3.0, 8.0, n_sc)
    doc = np.cumsum(rng.random((B, T)) < 0.02, axis=1).astype(np.int32) if docs else None
    kw = dict(is_causal=True, eps=1e-12, window_size=window, doc_ids=doc)
    got = _run(family, q, k, v, do, sc, torch.bfloat16, **kw)
    check_all(got, _oracle(family, q, k, v, do, sc, **kw), lowp=True, names=("out", "dq", "dk", "dv", "dscale"))


def test_term_backward_needs_no_scale_gradient_buffer():
    """fb_born_bwd_term accepts dscale = NULL (it never writes parameter gradients), where
    fb_born_bwd refuses it."""
    lib = _lib.load()
    dev = torch.device("cuda")
    B, H, T, D = 1, 2, 128, 64
    q, k, v, do = (torch.randn(B, H, T, D, device=dev).to(torch.bfloat16) for _ in range(4))
    sc = torch.full((H,), 4.0, device=dev)
    out, z = torch.ops.flashborn_b200.born_fwd(q, k, v, sc, None, None, True, 1e-12, 0, 0.0, False)
    a = _lib.FbAttnArgs()
    fbm._fill_common(a, q, k, v, out, z, sc, None, None, True, 1e-12, 0, 0.0)
    dq, dk, dv = (torch.empty_like(q) for _ in range(3))
    a.dout, a.dout_stride = fbm._ptr(do), fbm._strides(do)
    a.dq, a.dq_stride = fbm._ptr(dq), fbm._strides(dq)
    a.dk, a.dk_stride = fbm._ptr(dk), fbm._strides(dk)
    a.dv, a.dv_stride = fbm._ptr(dv), fbm._strides(dv)
    a.dscale = None
    ws_bytes = int(lib.fb_bwd_workspace_size(ctypes.byref(a)))
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
    a.workspace, a.workspace_bytes = fbm._ptr(ws), ws_bytes
    s = torch.cuda.current_stream().cuda_stream
    assert lib.fb_born_bwd(ctypes.byref(a), s) == _lib.FB_ERR_ARG
    assert lib.fb_born_bwd_term(ctypes.byref(a), s) == _lib.FB_OK
    # a single term with its own O and Z is the plain backward
    dq2, dk2, dv2, _, _ = torch.ops.flashborn_b200.born_bwd(do, q, k, v, out, z, sc, None, None, True, 1e-12, 0,
                                                            0.0, False)
    torch.cuda.synchronize()
    for x, y in ((dq, dq2), (dk, dk2), (dv, dv2)):
        e = (x.float() - y.float()).abs().max() / y.float().abs().max()
        assert e < 1e-2, float(e)


@pytest.mark.parametrize("D", [64, 128])
def test_token_major_output(D):
    """token_major=True: the same values, memory (B, T, H, D), so the head merge is a view; the
    backward takes the merge's strided gradient without a copy and gives the same gradients."""
    torch.manual_seed(0)
    dev = torch.device("cuda")
    B, H, T = 2, 4, 384
    base = [torch.randn(B, H, T, D, device=dev).to(torch.bfloat16) for _ in range(3)]
    sc = torch.full((1, H, 1, 1), 6.0, device=dev)
    dmerged = torch.randn(B, T, H * D, device=dev).to(torch.bfloat16)
    res = []
    for tm in (False, True):
        q, k, v = (x.detach().clone().requires_grad_(True) for x in base)
        s = sc.clone().requires_grad_(True)
        o = flash_born_attention(q, k, v, s, token_major=tm)
        merged = o.transpose(1, 2).contiguous().view(B, T, H * D)
        if tm:
            assert o.stride() == (T * H * D, D, H * D, 1)
            assert merged.data_ptr() == o.data_ptr()  # the merge copied nothing
        g = torch.autograd.grad(merged, (q, k, v, s), dmerged)
        res.append((o.detach(), g))
    torch.cuda.synchronize()
    assert torch.equal(res[0][0], res[1][0])
    for a, b in zip(res[0][1][:3], res[1][1][:3]):
        e = (a.float() - b.float()).abs().max() / b.float().abs().max()
        assert e < 1e-2, float(e)
