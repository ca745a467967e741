"""fb_born_bwd_static_scratch: the backward entry point that allocates nothing.

Some callers cannot allocate device memory -- a host runtime that binds only this library's C
functions and has no device allocator, or a training step that must not call cudaMalloc (it can
synchronise the device, and fails once another framework's pool holds the GPU).  They call
fb_born_bwd_static_scratch, which takes no workspace and runs the backward out of a fixed device
array inside the library.  These tests call it through the C ABI on each backward kernel family (fused and split
tensor-core, general CUDA-core), with a different masked problem in between two checked calls so
the shared array holds other data, and compare its gradients with fb_born_bwd given a
caller-allocated workspace; they also check that purified arguments and a problem needing more
scratch than the array holds are refused.  The file name makes pytest collect it last.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from quantumdlblocks_b200 import _lib
from quantumdlblocks_b200.kernels import flash_born as fbm

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("CUDA device required", allow_module_level=True)

MAX_REL = 2e-2  # the bf16 gate used by every other parity test


def _problem(dtype, B=2, H=4, T=640, D=64, seed=0, window=0, doc_mean=None):
    g = torch.Generator().manual_seed(seed)
    q, k, v, do = (torch.randn(B, H, T, D, generator=g).to(dtype).cuda() for _ in range(4))
    scale = torch.linspace(0.3, 0.5, H).cuda()
    doc = None
    if doc_mean is not None:
        rng = np.random.default_rng(seed)
        d = np.zeros((B, T), np.int32)
        for b in range(B):
            t, n = 0, 0
            while t < T:
                L = int(rng.geometric(1 / doc_mean))
                d[b, t:t + L] = n
                t, n = t + L, n + 1
        doc = torch.tensor(d, device="cuda")
    out, z = torch.ops.flashborn_b200.born_fwd(q, k, v, scale, None, doc, True, 1e-12, window, 0.0, False)
    return dict(q=q, k=k, v=v, do=do, scale=scale, out=out, z=z, doc=doc, window=window)


def _args(p, dq, dk, dv, dscale, workspace=None):
    a = _lib.FbAttnArgs()
    fbm._fill_common(a, p["q"], p["k"], p["v"], p["out"], p["z"], p["scale"], None, p["doc"], True, 1e-12,
                     p["window"], 0.0)
    a.dout, a.dout_stride = p["do"].data_ptr(), _lib._I64x4(*p["do"].stride())
    a.dq, a.dq_stride = dq.data_ptr(), _lib._I64x4(*dq.stride())
    a.dk, a.dk_stride = dk.data_ptr(), _lib._I64x4(*dk.stride())
    a.dv, a.dv_stride = dv.data_ptr(), _lib._I64x4(*dv.stride())
    a.dscale = dscale.data_ptr()
    if workspace is not None:
        a.workspace, a.workspace_bytes = workspace.data_ptr(), workspace.numel()
    return a


def _grads(p, fn, with_workspace, deterministic=False):
    """One backward through the C ABI; deterministic selects the split tensor-core backward (as
    torch.use_deterministic_algorithms(True) does through fb_attn_args.deterministic)."""
    lib = _lib.load()
    dq, dk, dv = (torch.empty_like(p["q"]) for _ in range(3))
    dscale = torch.zeros(p["scale"].numel(), device="cuda")
    prev = torch.are_deterministic_algorithms_enabled()
    torch.use_deterministic_algorithms(deterministic)
    try:
        a = _args(p, dq, dk, dv, dscale)
        if with_workspace:
            ws = torch.empty(max(1, int(lib.fb_bwd_workspace_size(ctypes.byref(a)))), dtype=torch.uint8,
                             device="cuda")
            a = _args(p, dq, dk, dv, dscale, ws)
    finally:
        torch.use_deterministic_algorithms(prev)
    rc = fn(ctypes.byref(a), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert rc == _lib.FB_OK, lib.fb_strerror(rc).decode()
    return [t.double().cpu().numpy() for t in (dq, dk, dv, dscale)]


def _check(got, ref, what):
    scale_of_grads = max(float(np.abs(ref[0]).max()), float(np.abs(ref[1]).max()), 1.0)
    for name, x, r in zip(("dq", "dk", "dv"), got[:3], ref[:3]):
        err = float(np.abs(x - r).max() / max(np.abs(r).max(), 1e-30))
        assert err <= MAX_REL, f"{what} {name}: max-rel {err:.3e}"
    assert float(np.abs(got[3] - ref[3]).max()) <= MAX_REL * 1e-2 * scale_of_grads, f"{what} dscale"


# (dtype, head dim, deterministic): the fused tensor-core backward (bf16, d=64), the split
# tensor-core backward (deterministic d=64, and d=128), and the general CUDA-core backward (fp32);
# each lays out its scratch differently
PATHS = [(torch.bfloat16, 64, False), (torch.bfloat16, 64, True), (torch.bfloat16, 128, False),
         (torch.float32, 64, False)]


@pytest.mark.parametrize("dtype,D,deterministic", PATHS, ids=["fused-d64", "split-d64", "split-d128", "general-f32"])
def test_static_scratch_backward_matches_workspace_backward(dtype, D, deterministic):
    lib = _lib.load()
    p = _problem(dtype, D=D)
    ref = _grads(p, lib.fb_born_bwd, with_workspace=True, deterministic=deterministic)
    got = _grads(p, lib.fb_born_bwd_static_scratch, with_workspace=False, deterministic=deterministic)
    _check(got, ref, "first call")
    # a different problem (other shape, a window, document ids) leaves other data in the array
    other = _problem(dtype, B=1, H=3, T=900, D=D, seed=1, window=300, doc_mean=150.0)
    ref_o = _grads(other, lib.fb_born_bwd, with_workspace=True, deterministic=deterministic)
    got_o = _grads(other, lib.fb_born_bwd_static_scratch, with_workspace=False, deterministic=deterministic)
    _check(got_o, ref_o, "masked call")
    # the first problem again, over the other problem's leftovers
    got = _grads(p, lib.fb_born_bwd_static_scratch, with_workspace=False, deterministic=deterministic)
    _check(got, ref, "repeat call")
    assert fbm.device_status() == (0, 0)


def test_static_scratch_refuses_purified_arguments():
    lib = _lib.load()
    p = _problem(torch.bfloat16, B=1, H=1, T=128)
    dq, dk, dv = (torch.empty_like(p["q"]) for _ in range(3))
    dscale = torch.zeros(1, device="cuda")
    a = _args(p, dq, dk, dv, dscale)
    tau = torch.zeros(1, device="cuda")
    a.tau, a.tau_numel = tau.data_ptr(), 1
    rc = lib.fb_born_bwd_static_scratch(ctypes.byref(a), torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.FB_ERR_ARG


def test_static_scratch_refuses_problems_over_the_limit():
    lib = _lib.load()
    p = _problem(torch.bfloat16, B=1, H=1, T=128)
    dq, dk, dv = (torch.empty_like(p["q"]) for _ in range(3))
    dscale = torch.zeros(1, device="cuda")
    a = _args(p, dq, dk, dv, dscale)
    # claim B=8, H=16, N=32768: its backward needs ~34 MB of scratch (two fp32 vectors per query
    # row and the parameter partials); refused before any launch
    a.batch, a.heads, a.seq_len = 8, 16, 32768
    assert lib.fb_bwd_workspace_size(ctypes.byref(a)) > _lib.FB_STATIC_SCRATCH_BYTES
    rc = lib.fb_born_bwd_static_scratch(ctypes.byref(a), torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.FB_ERR_SCRATCH_LIMIT
    assert "static" in lib.fb_strerror(rc).decode()
