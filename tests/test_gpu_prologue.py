"""GPU: the fused Q / K / V prologue and row L2 normalisation against plain fp32 PyTorch
restatements of the reference ops (``functional.py:59-121``: l2_normalize, apply_unitary_rope;
``layers/attention.py:512-516, 588-589``), forward and backward."""
from __future__ import annotations

import pytest
import torch

from quantumdlblocks_b200.kernels import flash_born as fbm
from quantumdlblocks_b200.kernels.prologue import l2_normalize, qkv_rope_l2norm, rope_tables

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("CUDA device required", allow_module_level=True)


def ref_l2n(x, eps):
    return x / torch.sqrt(x.square().sum(-1, keepdim=True) + eps)


def ref_rope(x, cos, sin):
    d = x.shape[-1]
    x1, x2 = x[..., :d // 2], x[..., d // 2:]
    return torch.cat([x1 * cos - x2 * sin, x1 * sin + x2 * cos], dim=-1)


def ref_prologue(qkv, cos, sin, H, eps):
    B, T, three_d = qkv.shape
    hd = three_d // (3 * H)
    q, k, v = (qkv.view(B, T, 3, H, hd)[:, :, i].transpose(1, 2) for i in range(3))
    return ref_l2n(ref_rope(q, cos, sin), eps), ref_l2n(ref_rope(k, cos, sin), eps), v


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 2e-6), (torch.bfloat16, 1e-2)], ids=["fp32", "bf16"])
@pytest.mark.parametrize("B,T,H,hd", [(2, 37, 3, 64), (1, 300, 16, 64), (3, 17, 2, 128)])
def test_qkv_prologue_matches_reference(B, T, H, hd, dtype, tol):
    g = torch.Generator().manual_seed(B * 100 + T + hd)
    qkv = (torch.randn(B, T, 3 * H * hd, generator=g) * 3).to("cuda", dtype).requires_grad_(True)
    cos, sin = rope_tables(T + 5, hd, device="cuda")  # longer tables are sliced to T
    gq, gk, gv = (torch.randn(B, H, T, hd, generator=g).to("cuda", dtype) for _ in range(3))
    q, k, v = qkv_rope_l2norm(qkv, cos, sin, H, eps=1e-12)
    assert q.is_contiguous() and k.is_contiguous() and v.is_contiguous() and q.shape == (B, H, T, hd)
    ((q.float() * gq.float()).sum() + (k.float() * gk.float()).sum() + (v.float() * gv.float()).sum()).backward()
    torch.cuda.synchronize()
    assert fbm.device_status() == (0, 0)
    x = qkv.detach().float().requires_grad_(True)
    rq, rk, rv = ref_prologue(x, cos[:T], sin[:T], H, 1e-12)
    ((rq * gq.float()).sum() + (rk * gk.float()).sum() + (rv * gv.float()).sum()).backward()
    for got, want in ((q, rq), (k, rk), (v, rv)):
        assert (got.float() - want.detach()).abs().max().item() <= tol * want.abs().max().item()
    err = (qkv.grad.float() - x.grad).abs().max().item()
    assert err <= tol * x.grad.abs().max().item() * 4, err
    assert torch.equal(v, qkv.detach().view(B, T, 3, H, hd)[:, :, 2].transpose(1, 2))  # V is copied exactly


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 2e-6), (torch.bfloat16, 1e-2)], ids=["fp32", "bf16"])
@pytest.mark.parametrize("shape", [(5, 7, 1024), (3, 64), (1, 8)])
def test_l2_normalize_matches_reference(shape, dtype, tol):
    g = torch.Generator().manual_seed(len(shape) + shape[-1])
    x = (torch.randn(*shape, generator=g) * 2).to("cuda", dtype).requires_grad_(True)
    dy = torch.randn(*shape, generator=g).to("cuda", dtype)
    y = l2_normalize(x, eps=1e-12)
    (y.float() * dy.float()).sum().backward()
    torch.cuda.synchronize()
    xr = x.detach().float().requires_grad_(True)
    yr = ref_l2n(xr, 1e-12)
    (yr * dy.float()).sum().backward()
    assert (y.float() - yr.detach()).abs().max().item() <= tol * yr.abs().max().item()
    assert (x.grad.float() - xr.grad).abs().max().item() <= 2 * tol * xr.grad.abs().max().item()


def test_zero_rows_stay_finite():
    x = torch.zeros(4, 64, device="cuda", requires_grad=True)
    y = l2_normalize(x)
    y.sum().backward()
    assert torch.isfinite(y).all() and torch.isfinite(x.grad).all() and y.abs().max() == 0
