"""GPU: one forward + backward step through the public API, captured as a CUDA graph and replayed,
gives the eager step's results.  The op allocates its outputs and workspaces through PyTorch and
launches on the current stream, so the capture holds the same kernels (and the zero fill of the
scale gradient); replays recompute everything from the captured inputs.  Deterministic mode
(split backward) is compared bitwise, the fused backward (dQ additions in run order) and the
document-masked path within the bf16 gate."""
from __future__ import annotations

import pytest
import torch

from quantumdlblocks_b200 import flash_born_attention

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("CUDA device required", allow_module_level=True)


def _step(q, k, v, scale, do, doc):
    out = flash_born_attention(q, k, v, scale, is_causal=True, doc_ids=doc)
    return (out,) + torch.autograd.grad(out, (q, k, v, scale), do)


@pytest.mark.parametrize("deterministic,with_doc", [(True, False), (False, False), (False, True)],
                         ids=["deterministic", "fused", "fused-doc"])
def test_graph_replay_matches_eager_step(deterministic, with_doc):
    B, H, T, D = 2, 4, 700, 64
    g = torch.Generator().manual_seed(11)
    q, k, v, do = (torch.randn(B, H, T, D, generator=g).to("cuda", torch.bfloat16) for _ in range(4))
    q, k, v = (x.requires_grad_(True) for x in (q, k, v))
    scale = torch.linspace(6.0, 9.0, H, device="cuda").reshape(1, H, 1, 1).requires_grad_(True)
    doc = None
    if with_doc:
        doc = torch.sort(torch.randint(0, 5, (B, T), generator=g), dim=1).values.to(torch.int32).cuda()
    prev = torch.are_deterministic_algorithms_enabled()
    torch.use_deterministic_algorithms(deterministic)
    try:
        eager = [x.clone() for x in _step(q, k, v, scale, do, doc)]
        # fresh leaves for the captured step: the eager step's leaves carry autograd state made
        # on the default stream
        q, k, v, scale = (x.detach().clone().requires_grad_(True) for x in (q, k, v, scale))
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(2):
                _step(q, k, v, scale, do, doc)
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            static = _step(q, k, v, scale, do, doc)
        for _ in range(2):  # every replay recomputes the whole step
            for x in static:
                x.zero_()
            graph.replay()
            torch.cuda.synchronize()
            for name, got, ref in zip(("out", "dq", "dk", "dv", "dscale"), static, eager):
                if deterministic and name != "dscale":
                    assert torch.equal(got, ref), name
                else:
                    err = ((got.float() - ref.float()).abs().max() / ref.float().abs().max().clamp_min(1e-30)).item()
                    assert err <= 2e-2, (name, err)
    finally:
        torch.use_deterministic_algorithms(prev)
