"""GPU: the C5 GPT with the native flash-Born op against the same GPT (same weights) with a plain
fp32 PyTorch Born attention: loss and parameter gradients, in fp32 (general kernels) and under
bf16 autocast (tensor-core kernels, strided Q / K / V views of the fused projection)."""
from __future__ import annotations

import copy

import pytest
import torch

from quantumdlblocks_b200 import flash_born_attention
from quantumdlblocks_b200.gpt import BornGPT, GPTConfig, train_step, zipf_tokens
from quantumdlblocks_b200.kernels import flash_born as fbm
from test_gpt_cpu import born_eager

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("CUDA device required", allow_module_level=True)

CFG = GPTConfig(vocab_size=211, d_model=256, n_layers=2, n_heads=4, seq_len=320)


def _loss_and_grads(attention, autocast_dtype):
    torch.manual_seed(0)
    model = BornGPT(CFG, attention=attention).cuda()
    tok = torch.from_numpy(zipf_tokens(3, CFG.seq_len, CFG.vocab_size, seed=7)).cuda()
    with torch.autocast("cuda", dtype=autocast_dtype or torch.float32, enabled=autocast_dtype is not None):
        loss = model(tok[:, :-1], tok[:, 1:])
    loss.backward()
    torch.cuda.synchronize()
    return loss.item(), {n: p.grad.detach().float() for n, p in model.named_parameters()}


@pytest.mark.parametrize("autocast_dtype,tol", [(None, 1e-4), (torch.bfloat16, 3e-2)], ids=["fp32", "bf16"])
def test_gpt_native_attention_matches_eager(autocast_dtype, tol):
    loss_n, g_n = _loss_and_grads(flash_born_attention, autocast_dtype)
    assert fbm.device_status() == (0, 0)
    loss_e, g_e = _loss_and_grads(born_eager, autocast_dtype)
    assert abs(loss_n - loss_e) <= tol * abs(loss_e)
    # the head-scale gradient is analytically ~0 here (2 eps sum delta / (scale Z) with eps 1e-12):
    # eager autograd returns its cancellation noise, the native op its closed form, so gradients
    # are compared against a floor of 1e-3 of the model's largest gradient
    floor = 1e-3 * max(g.abs().max().item() for g in g_e.values())
    for name in g_e:
        a, b = g_n[name], g_e[name]
        err = (a - b).abs().max().item()
        assert err <= tol * max(b.abs().max().item(), floor), (name, err, b.abs().max().item())


def test_gpt_train_step_runs_and_learns():
    torch.manual_seed(0)
    model = BornGPT(CFG).cuda()
    opt = torch.optim.AdamW(model.parameters(), lr=3e-3)
    tok = torch.from_numpy(zipf_tokens(4, CFG.seq_len, CFG.vocab_size, seed=11)).cuda()
    losses = [train_step(model, opt, tok).item() for _ in range(8)]
    assert fbm.device_status() == (0, 0)
    assert all(map(lambda x: x == x, losses)) and losses[-1] < losses[0]
