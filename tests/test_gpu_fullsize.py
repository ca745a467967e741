"""GPU: the benchmark configurations at full size, checked against the float64 oracle.

Each test builds the exact inputs ``bench.py`` times (``bench.make_inputs``: C2 B=8 H=16 N=2048
d=64; C3 B=1 H=32 N=16384 d=128 with unit-norm * sqrt(d) Q/K; C4 B=4 H=16 N=8192 d=64 with seed-3
geometric documents), runs forward + backward through the public API (``flash_born_attention`` +
autograd, as the benchmark step does), so the persistent kernels walk their full work lists, the
cross-item pipelines and the L2-window schedule.  The first and last (batch, head) units and a few
seeded random ones are then recomputed one unit at a time by the float64 oracle on the same
bf16-rounded inputs and gated at max-rel 2e-2 (``parity_util.check_all``).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import bench
from oracle import flash_born_oracle as orc
from parity_util import check_all
from quantumdlblocks_b200 import flash_born_attention
from quantumdlblocks_b200.kernels import flash_born as fbm

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("CUDA device required", allow_module_level=True)


def _units(B: int, H: int, n_random: int, seed: int) -> list[tuple[int, int]]:
    picks = [(0, 0), (B - 1, H - 1)]
    rng = np.random.default_rng(seed)
    while len(picks) < 2 + n_random:
        u = (int(rng.integers(B)), int(rng.integers(H)))
        if u not in picks:
            picks.append(u)
    return picks


@pytest.mark.parametrize("workload,n_random", [("c2", 4), ("c4", 2), ("c3", 1)])
def test_full_size_units_match_oracle(workload, n_random):
    B, H, N, D, causal, _ = bench.WORKLOADS[workload]
    q_cpu, k_cpu, v_cpu, do_cpu, doc_np, scale_val = bench.make_inputs(workload, 0)
    bf = torch.bfloat16
    q, k, v = (x.to(bf).cuda().requires_grad_(True) for x in (q_cpu, k_cpu, v_cpu))
    do = do_cpu.to(bf).cuda()
    doc = None if doc_np is None else torch.from_numpy(doc_np).cuda()
    scale = torch.full((1, H, 1, 1), scale_val, device="cuda", requires_grad=True)
    out = flash_born_attention(q, k, v, scale, is_causal=causal, eps=1e-12, doc_ids=doc)
    gq, gk, gv, gs = torch.autograd.grad(out, (q, k, v, scale), do)
    torch.cuda.synchronize()
    assert fbm.device_status() == (0, 0)
    assert torch.isfinite(gs).all()
    for b, h in _units(B, H, n_random, seed=B * H + N):
        qu, ku, vu, du = (x[b, h][None, None].to(bf).double().numpy() for x in (q_cpu, k_cpu, v_cpu, do_cpu))
        dr = None if doc_np is None else doc_np[b:b + 1]
        ref_o, ref_z = orc.born_forward(qu, ku, vu, scale_val, causal, 1e-12, 0, dr)
        g = orc.born_backward(qu, ku, vu, ref_o, ref_z, du, scale_val, causal, 0, dr)
        got = {n: t[b, h][None, None].detach().double().cpu().numpy()
               for n, t in (("out", out), ("dq", gq), ("dk", gk), ("dv", gv))}
        ref = {"out": ref_o, "dq": g.dq, "dk": g.dk, "dv": g.dv}
        try:
            check_all(got, ref, lowp=True)
        except AssertionError as e:
            raise AssertionError(f"{workload} unit (b={b}, h={h}): {e}") from None
