"""GPU: the fused cross-entropy (the GPT training loss) against PyTorch's fp32 cross-entropy on
the same bf16 logits (the reference GPTs' ``F.cross_entropy``, ``models/born_gpt.py:1291``)."""
from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("CUDA device required", allow_module_level=True)

from quantumdlblocks_b200.kernels import flash_born as fbm  # noqa: E402
from quantumdlblocks_b200.kernels.xent import cross_entropy  # noqa: E402


@pytest.mark.parametrize("N,V,pad,gscale", [(37, 64, 0, 1.0), (300, 50304, 47, 1.0), (129, 2056, 8, 2.5)])
def test_cross_entropy_matches_torch(N, V, pad, gscale):
    g = torch.Generator(device="cuda").manual_seed(N + V)
    x = (torch.randn(N, V, generator=g, device="cuda") * 3).to(torch.bfloat16)
    if pad:
        x[:, V - pad:] = float("-inf")  # the GPT's padded head rows
    t = torch.randint(0, V - pad, (N,), generator=g, device="cuda")
    a = x.clone().requires_grad_(True)
    loss = cross_entropy(a, t)
    (loss * gscale).backward()
    torch.cuda.synchronize()
    assert fbm.device_status() == (0, 0)
    r = x.float().requires_grad_(True)
    ref = F.cross_entropy(r, t)
    (ref * gscale).backward()
    assert abs(loss.item() - ref.item()) <= 1e-5 * max(1.0, abs(ref.item()))
    err = (a.grad.float() - r.grad).abs().max().item()
    assert err <= 1e-2 * r.grad.abs().max().item(), err  # the gradient is stored in bf16
    if pad:
        assert torch.all(a.grad[:, V - pad:] == 0)


def test_cross_entropy_strided_rows_and_checks():
    x = torch.randn(8, 72, device="cuda").to(torch.bfloat16)[:, :64]  # row stride 72 > vocab 64
    t = torch.randint(0, 64, (8,), device="cuda")
    a = x.clone().requires_grad_(True)  # clone() keeps the dense layout; test the strided view too
    got = cross_entropy(x, t)
    ref = F.cross_entropy(x.float(), t)
    assert abs(got.item() - ref.item()) <= 1e-5 * max(1.0, abs(ref.item()))
    cross_entropy(a, t).backward()
    with pytest.raises(ValueError):
        cross_entropy(x.float(), t)
    with pytest.raises(ValueError):
        cross_entropy(x, t[:4])
