"""GPU: a problem split into shards (the multi-GPU unit split, emulated on one GPU) gives the
whole problem's result.  Each shard runs the ordinary op on strided views of the full tensors;
the forward output and, in deterministic mode, dQ / dK / dV are bitwise the whole problem's
(every (batch, head) unit is computed independently), and the per-head scale gradient assembled
from the shards' parts matches."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from quantumdlblocks_b200 import flash_born_attention, sharding

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("CUDA device required", allow_module_level=True)


@pytest.mark.parametrize("B,H,world,with_doc", [(2, 8, 4, False), (4, 3, 2, True), (3, 5, 3, False)],
                         ids=["heads", "batch-doc", "batch"])
def test_shards_reassemble_the_whole_problem(B, H, world, with_doc):
    T, D = 700, 64
    g = torch.Generator().manual_seed(5)
    q, k, v, do = (torch.randn(B, H, T, D, generator=g).to("cuda", torch.bfloat16) for _ in range(4))
    doc = None
    if with_doc:
        doc = torch.sort(torch.randint(0, 6, (B, T), generator=g), dim=1).values.to(torch.int32).cuda()
    scale = torch.linspace(0.3, 0.5, H, device="cuda")
    prev = torch.are_deterministic_algorithms_enabled()
    torch.use_deterministic_algorithms(True)
    try:
        qf, kf, vf = (x.clone().requires_grad_(True) for x in (q, k, v))
        sf = scale.clone().requires_grad_(True)
        out = flash_born_attention(qf, kf, vf, sf, is_causal=True, doc_ids=doc)
        out.backward(do)

        plan = sharding.plan_shards(B, H, T, world, doc_ids=doc)
        qs, ks, vs = (x.clone().requires_grad_(True) for x in (q, k, v))
        outs = torch.zeros_like(out)
        dscale = torch.zeros(H, dtype=torch.float64, device="cuda")
        for sh in plan:
            sq, sk, sv, _, sdoc = sharding.shard_inputs(sh, qs, ks, vs, scale, doc)
            ss = scale[sh.h0:sh.h1].clone().requires_grad_(True)
            o = flash_born_attention(sq, sk, sv, ss, is_causal=True, doc_ids=sdoc)
            o.backward(do[sh.b0:sh.b1, sh.h0:sh.h1])
            outs[sh.b0:sh.b1, sh.h0:sh.h1] = o.detach()
            dscale += sharding.gather_param_grad(ss.grad, sh, H)  # no process group: this shard's part
        torch.cuda.synchronize()
    finally:
        torch.use_deterministic_algorithms(prev)
    assert torch.equal(outs, out.detach())
    assert torch.equal(qs.grad, qf.grad)
    assert torch.equal(ks.grad, kf.grad)
    assert torch.equal(vs.grad, vf.grad)
    ref = sf.grad.double()
    np.testing.assert_allclose(dscale.cpu().numpy(), ref.cpu().numpy(), rtol=1e-5,
                               atol=1e-5 * float(ref.abs().max()))
