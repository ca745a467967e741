"""GPU parity: the CUDA kernels (through the custom op and the C ABI) against the reference's
golden vectors and the float64 oracle, on both kernel paths, with the reference's edge cases."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from golden_cases import c1_inputs, case_names, load_case, manifest
from parity_util import check_all, fp32_gate, lowp_gate, round_to, run_cuda, run_oracle

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # collected on CPU hosts, skipped there
    pytest.skip("CUDA device required", allow_module_level=True)


def _case_kwargs(c):
    kw = dict(is_causal=c["is_causal"], eps=c["eps"], window_size=c["window_size"], doc_ids=c["doc_ids"])
    if c["kind"] == "purified":
        kw.update(tau=c["param_tau"], eps_base=c["eps_base"])
    return kw


@pytest.mark.parametrize("name", case_names())
def test_golden_fp32(name):
    """fp32 inputs against the reference's own float64 outputs (general path)."""
    c = load_case(name)
    got = run_cuda(c["kind"], c["q"], c["k"], c["v"], c["do"], c["param_scale"], dtype=torch.float32,
                   **_case_kwargs(c))
    ref = {n: c["ref_" + n] for n in ("out", "dq", "dk", "dv", "dscale")}
    if c["kind"] == "purified":
        ref["dtau"] = c["ref_dtau"]
    check_all(got, ref, lowp=False)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("path", ["auto", "general"])
@pytest.mark.parametrize("name", case_names())
def test_golden_lowp(name, dtype, path):
    """bf16/fp16 inputs against the float64 oracle on the rounded inputs."""
    c = load_case(name)
    q, k, v, do = (round_to(c[n], dtype) for n in ("q", "k", "v", "do"))
    kw = _case_kwargs(c)
    got = run_cuda(c["kind"], q, k, v, do, c["param_scale"], dtype=dtype, path=path, **kw)
    ref = run_oracle(c["kind"], q, k, v, do, c["param_scale"], **kw)
    check_all(got, ref, lowp=True)


def test_c1_fp32_against_reference_checksums():
    """C1 (B=2,H=4,N=256,d=64 fp32 causal, per-head scale 8): gate + the reference's checksums."""
    q, k, v, do = (x.numpy() for x in c1_inputs())
    scale = np.full((1, 4, 1, 1), 8.0, dtype=np.float32)
    got = run_cuda("plain", q, k, v, do, scale, dtype=torch.float32)
    ref = run_oracle("plain", q, k, v, do, scale)
    check_all(got, ref, lowp=False)
    m = manifest()["C1"]["checksums"]["f64"]
    idx = np.array(manifest()["C1"]["checksums"]["sample_idx"])
    for n in ("out", "dq", "dk", "dv"):
        fp32_gate(got[n].reshape(-1)[idx], np.array(m[n]["sample"]), n + " (reference sample)")


@pytest.mark.parametrize("T", [1, 15, 17, 63, 65, 127, 129, 200])
@pytest.mark.parametrize("D", [16, 48, 64, 128])
def test_ragged_shapes_bf16(T, D):
    rng = np.random.default_rng(T * 1000 + D)
    B, H = 2, 2
    q, k, v, do = (round_to(rng.standard_normal((B, H, T, D)), torch.bfloat16) for _ in range(4))
    scale = np.array([0.4, 0.25], dtype=np.float32)
    got = run_cuda("plain", q, k, v, do, scale, dtype=torch.bfloat16)
    ref = run_oracle("plain", q, k, v, do, scale)
    check_all(got, ref, lowp=True)


@pytest.mark.parametrize("D", [32, 96, 256])
def test_other_head_dims_fp32(D):
    rng = np.random.default_rng(D)
    q, k, v, do = (rng.standard_normal((1, 2, 70, D)).astype(np.float32) for _ in range(4))
    q /= np.linalg.norm(q, axis=-1, keepdims=True)
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    got = run_cuda("plain", q, k, v, do, np.float32(9.0), dtype=torch.float32, window_size=33)
    ref = run_oracle("plain", q, k, v, do, np.float32(9.0), window_size=33)
    check_all(got, ref, lowp=False)


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("window", [0, 1, 64, 300])
def test_window_and_causality_bf16(causal, window):
    rng = np.random.default_rng(7 + window)
    B, H, T, D = 1, 2, 320, 64
    q, k, v, do = (round_to(rng.standard_normal((B, H, T, D)), torch.bfloat16) for _ in range(4))
    scale = np.float32(0.3)
    got = run_cuda("plain", q, k, v, do, scale, dtype=torch.bfloat16, is_causal=causal, window_size=window)
    ref = run_oracle("plain", q, k, v, do, scale, is_causal=causal, window_size=window)
    # causal window 1: every row has exactly one key, so dQ/dK are analytically
    # 2 a dO.v eps / (p + eps)^2 -- O(eps / a^3), below the resolution of fp32 sums of p; they are
    # held to an absolute bound of 1e-2 x the output scale (floor 0.5 x scale) instead of max-rel.
    check_all(got, ref, lowp=True, floor_rel=0.5 if (causal and window == 1) else 1e-3)


@pytest.mark.parametrize("kind", ["plain", "purified"])
def test_document_mask_bf16(kind):
    rng = np.random.default_rng(11)
    B, H, T, D = 2, 2, 600, 64
    doc = np.zeros((B, T), dtype=np.int32)
    for b in range(B):
        t, d = 0, 0
        while t < T:
            L = int(rng.geometric(1 / 90))
            doc[b, t:t + L] = d
            t, d = t + L, d + 1
    q, k, v, do = (rng.standard_normal((B, H, T, D)) for _ in range(4))
    if kind == "purified":
        q /= np.linalg.norm(q, axis=-1, keepdims=True)
        k /= np.linalg.norm(k, axis=-1, keepdims=True)
    q, k, v, do = (round_to(x, torch.bfloat16) for x in (q, k, v, do))
    kw = dict(doc_ids=doc)
    scale = np.array([0.5, 0.35], dtype=np.float32) if kind == "plain" else np.array([6.0, 9.0], np.float32)
    if kind == "purified":
        kw.update(tau=np.array([0.03, 0.06], np.float32))
    got = run_cuda(kind, q, k, v, do, scale, dtype=torch.bfloat16, **kw)
    ref = run_oracle(kind, q, k, v, do, scale, **kw)
    check_all(got, ref, lowp=True)


def test_c2_shape_subset_bf16():
    """C2 shape (N=2048, d=64, causal, scale 8) on 2 (b,h) units against the float64 oracle."""
    torch.manual_seed(0)
    q, k, v = (torch.randn(1, 2, 2048, 64).to(torch.bfloat16).double().numpy() for _ in range(3))
    torch.manual_seed(1)
    do = torch.randn(1, 2, 2048, 64).to(torch.bfloat16).double().numpy()
    scale = np.full((1, 2, 1, 1), 8.0, dtype=np.float32)
    got = run_cuda("plain", q, k, v, do, scale, dtype=torch.bfloat16)
    ref = run_oracle("plain", q, k, v, do, scale)
    check_all(got, ref, lowp=True)


def test_noncontiguous_inputs_match_contiguous():
    """(B,T,H,D) storage viewed as (B,H,T,D): strided inputs give the same result as contiguous."""
    torch.manual_seed(3)
    B, H, T, D = 2, 3, 130, 64
    base = [torch.randn(B, T, H, D, device="cuda", dtype=torch.bfloat16) for _ in range(3)]
    strided = [x.transpose(1, 2) for x in base]
    contig = [x.contiguous() for x in strided]
    from quantumdlblocks_b200 import flash_born_attention
    o1 = flash_born_attention(*strided, 0.4)
    o2 = flash_born_attention(*contig, 0.4)
    torch.testing.assert_close(o1, o2, atol=0, rtol=0)


def test_scale_forms_and_autocast():
    from quantumdlblocks_b200 import flash_born_attention
    torch.manual_seed(4)
    q, k, v = (torch.randn(2, 4, 96, 64, device="cuda") for _ in range(3))
    ref = flash_born_attention(q, k, v, 0.5)
    for sc in (torch.tensor(0.5, device="cuda"), torch.full((4,), 0.5, device="cuda"),
               torch.full((1, 4, 1, 1), 0.5, device="cuda")):
        torch.testing.assert_close(flash_born_attention(q, k, v, sc), ref, atol=0, rtol=0)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        ob = flash_born_attention(q, k, v, 0.5)
    assert ob.dtype == torch.bfloat16
    lowp_gate(ob.float().cpu().numpy(), ref.cpu().numpy(), "autocast")
    sc = torch.full((1, 4, 1, 1), 0.5, device="cuda", requires_grad=True)
    flash_born_attention(q, k, v, sc).sum().backward()
    assert sc.grad.shape == sc.shape and sc.grad.dtype == sc.dtype


def test_empty_sequence():
    from quantumdlblocks_b200 import flash_born_attention
    q = torch.randn(2, 2, 0, 64, device="cuda", requires_grad=True)
    out = flash_born_attention(q, q, q, 1.0)
    assert out.shape == q.shape
    out.sum().backward()
    assert q.grad.shape == q.shape


def test_zero_rows_stay_finite_bf16():
    """Rows whose every overlap is <= 0 give Z = eps and O = 0; gradients stay finite."""
    c = load_case("plain_zero_rows_d16")
    q, k, v, do = (round_to(c[n], torch.bfloat16) for n in ("q", "k", "v", "do"))
    got = run_cuda("plain", q, k, v, do, c["param_scale"], dtype=torch.bfloat16)
    for n in ("out", "dq", "dk", "dv"):
        assert np.isfinite(got[n]).all(), n
    ref = run_oracle("plain", q, k, v, do, c["param_scale"])
    lowp_gate(got["out"], ref["out"], "out")
