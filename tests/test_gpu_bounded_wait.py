"""GPU: a bounded device-side wait that runs out, and the context afterwards.

Every pipeline wait of the tensor-core kernels is bounded: a wait that reaches its bound raises
the CTA's abort flag and the device status word (FB_ERR_TIMEOUT with the wait's site), lets the
copies and products already in flight land, frees tensor memory and returns -- the failure
detection of the kernels, which never trap.  ``fb_test_born_fwd_timeout`` makes one such wait run
out on purpose: the forward runs with a 2 ms bound and CTA 0's producer never requests its first
K tile.  Nothing faults or hangs; the test checks the status word, then that a normal forward and
backward in the same process still match the oracle.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from parity_util import check_all, round_to, run_cuda, run_oracle
from quantumdlblocks_b200 import _lib
from quantumdlblocks_b200.kernels import flash_born as fbm

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("CUDA device required", allow_module_level=True)

# wait sites of the tensor-core forward (the argument `site` of its mbar_wait calls)
FORWARD_SITES = set(range(1, 14))


def _fwd_args(q, k, v, out, z, scale):
    a = _lib.FbAttnArgs()
    fbm._fill_common(a, q, k, v, out, z, scale, None, None, True, 1e-12, 0, 0.0)
    return a


def test_wait_bound_runs_out_and_the_context_stays_usable():
    lib = _lib.load()
    assert fbm.device_status() == (0, 0)  # clean to begin with
    g = torch.Generator(device="cuda").manual_seed(0)
    B, H, T, D = 1, 2, 512, 64
    q, k, v = (torch.randn(B, H, T, D, generator=g, device="cuda").to(torch.bfloat16) for _ in range(3))
    scale = torch.full((H,), 0.4, device="cuda")
    out = torch.empty_like(q)
    z = torch.empty(B, H, T, device="cuda")
    a = _fwd_args(q, k, v, out, z, scale)
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.fb_test_born_fwd_timeout(ctypes.byref(a), stream, 2000)  # 2 ms bound
    assert rc == _lib.FB_OK, lib.fb_strerror(rc).decode()
    torch.cuda.synchronize()  # returns: the aborted CTA stopped within its bounds
    status, site = fbm.device_status()
    assert status == _lib.FB_ERR_TIMEOUT, status
    assert site in FORWARD_SITES, site
    assert fbm.device_status() == (0, 0)  # reading the word cleared it

    # the same process, the same library: a normal forward + backward is correct
    rng = np.random.default_rng(1)
    qn, kn, vn, don = (round_to(rng.standard_normal((2, 2, 300, 64)), torch.bfloat16) for _ in range(4))
    sc = np.array([0.35, 0.45], np.float32)
    got = run_cuda("plain", qn, kn, vn, don, sc, dtype=torch.bfloat16, path="tcgen05")
    assert fbm.device_status() == (0, 0)
    check_all(got, run_oracle("plain", qn, kn, vn, don, sc), lowp=True)


def test_timeout_hook_refuses_what_it_does_not_cover():
    lib = _lib.load()
    q = torch.randn(1, 1, 64, 48, device="cuda", dtype=torch.bfloat16)  # d=48: no tensor-core path
    out, z = torch.empty_like(q), torch.empty(1, 1, 64, device="cuda")
    scale = torch.ones(1, device="cuda")
    a = _fwd_args(q, q, q, out, z, scale)
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.fb_test_born_fwd_timeout(ctypes.byref(a), stream, 2000) == _lib.FB_ERR_UNSUPPORTED
    assert lib.fb_test_born_fwd_timeout(ctypes.byref(a), stream, 0) == _lib.FB_ERR_ARG
    assert fbm.device_status() == (0, 0)
