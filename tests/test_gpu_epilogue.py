"""GPU: the fused head epilogue (gated XSA, output gate, head merge) against a plain fp32 PyTorch
restatement of the reference ops (``layers/mudd_and_gates.py:17-61``, ``layers/attention.py:478-493``),
forward and backward."""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("CUDA device required", allow_module_level=True)

from quantumdlblocks_b200.kernels import flash_born as fbm  # noqa: E402
from quantumdlblocks_b200.kernels.epilogue import finalize_heads  # noqa: E402


def ref_finalize(o, v, alpha, x, w, b, eps):
    """apply_gated_xsa -> InputChannelGate -> transpose / merge, all in fp32."""
    y = o
    if alpha is not None:
        gate = torch.tanh(alpha).view(1, -1, 1, 1)
        n = v.square().sum(-1, keepdim=True) + eps
        y = y - gate * ((y * v).sum(-1, keepdim=True) / n) * v
    if x is not None:
        c = w.shape[1]
        g = 2.0 * torch.sigmoid(torch.nn.functional.linear(x[..., :c], w, b))  # (B, T, H)
        y = g.transpose(1, 2).unsqueeze(-1) * y
    B, H, T, hd = o.shape
    return y.transpose(1, 2).reshape(B, T, H * hd)


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-5), (torch.bfloat16, 2e-2)], ids=["fp32", "bf16"])
@pytest.mark.parametrize("B,H,T,hd,xsa,gate,token_major", [
    (2, 16, 64, 64, True, True, False), (1, 3, 37, 64, True, True, True), (2, 4, 50, 128, True, False, False),
    (1, 6, 33, 32, False, True, True), (2, 5, 17, 128, False, False, False)])
def test_finalize_heads_matches_reference_ops(B, H, T, hd, xsa, gate, token_major, dtype, tol):
    g = torch.Generator(device="cuda").manual_seed(B * 1000 + H * 10 + hd)
    E = H * hd
    shape = (B, T, H, hd) if token_major else (B, H, T, hd)
    o = torch.randn(shape, generator=g, device="cuda").to(dtype)
    o = o.transpose(1, 2) if token_major else o
    v = torch.randn(B, H, T, hd, generator=g, device="cuda").to(dtype)
    alpha = (torch.randn(H, generator=g, device="cuda") * 0.7) if xsa else None
    x = torch.randn(B, T, E, generator=g, device="cuda") if gate else None
    w = (torch.randn(H, 6, generator=g, device="cuda") * 0.5) if gate else None
    b = (torch.randn(H, generator=g, device="cuda") * 0.5) if gate else None
    dy = torch.randn(B, T, E, generator=g, device="cuda").to(dtype)
    leaves = [t for t in (o, v, alpha, x, w, b) if t is not None]
    got_in = [t.detach().clone().requires_grad_(True) for t in leaves]
    ref_in = [t.detach().float().clone().requires_grad_(True) for t in leaves]

    def unpack(ts):
        it = iter(ts)
        oo, vv = next(it), next(it)
        aa = next(it) if xsa else None
        xx, ww, bb = (next(it), next(it), next(it)) if gate else (None, None, None)
        return oo, vv, aa, xx, ww, bb

    go, gv, ga, gx, gw, gb = unpack(got_in)
    out = finalize_heads(go, gv if xsa else None, ga, gx, gw, gb, eps=1e-12)
    out.backward(dy)
    torch.cuda.synchronize()
    assert fbm.device_status() == (0, 0)
    ref = ref_finalize(*unpack(ref_in), eps=1e-12)
    ref.backward(dy.float())
    assert out.shape == (B, T, E) and out.dtype == dtype
    assert (out.float() - ref).abs().max().item() <= tol * ref.abs().max().item()
    for got, want, name in zip(got_in, ref_in, ["o", "v", "alpha", "x", "w", "b"] if xsa and gate else
                               ["o", "v", "alpha"] if xsa else ["o", "v", "x", "w", "b"] if gate else ["o", "v"]):
        if want.grad is None:
            assert got.grad is None or got.grad.abs().max().item() == 0, name
            continue
        err = (got.grad.float() - want.grad).abs().max().item()
        assert err <= tol * max(want.grad.abs().max().item(), 1e-6) * 2, f"{name}: {err}"


def test_finalize_heads_identity_without_gates_is_the_merge():
    o = torch.randn(2, 4, 10, 64, device="cuda").to(torch.bfloat16)
    out = finalize_heads(o)
    assert torch.equal(out, o.transpose(1, 2).reshape(2, 10, 256))
