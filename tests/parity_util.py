"""Helpers shared by the GPU parity tests: run the CUDA op, run the oracle, apply the gates.

Gates (from the task's tolerance statement):
* fp32 inputs: max |x - r| <= 1e-4 * max(1, max |r|) per tensor (absolute 1e-4 for O(1) tensors;
  gradients larger than 1 are held to the same relative resolution).
* bf16 / fp16 inputs: max-rel error ``max |x - r| / max |r|`` <= 2e-2 per tensor, against the
  float64 oracle evaluated on the rounded inputs.
* parameter gradients (dscale, dgamma, dtau): bf16/fp16 -- max-rel 2e-2 against their own size,
  floored at 1e-2 of the dQ/dK scale (the plain dscale is analytically sum_i 2 eps delta_i /
  (scale Z_i) ~ 0); fp32 -- absolute 1e-4 of the dQ/dK scale.
* a tensor that is analytically zero (dQ/dK when every row has a single valid key: then
  dO.v_j - delta_i = 0 exactly) is compared against an absolute floor: the max-rel denominator
  is at least 1e-3 x max(|out|, |dV|) of the same problem.
"""
from __future__ import annotations

import numpy as np
import torch

from oracle import flash_born_oracle as orc
from quantumdlblocks_b200 import flash_born_attention, flash_purified_born_attention
from quantumdlblocks_b200.kernels import flash_born as fbm

FP32_ABS = 1e-4
LOWP_REL = 2e-2


def max_rel(x, r) -> float:
    x = np.asarray(x, dtype=np.float64)
    r = np.asarray(r, dtype=np.float64)
    return float(np.abs(x - r).max() / max(np.abs(r).max(), 1e-30))


def fp32_gate(x, r, name="") -> None:
    x = np.asarray(x, dtype=np.float64)
    r = np.asarray(r, dtype=np.float64)
    err = float(np.abs(x - r).max())
    bound = FP32_ABS * max(1.0, float(np.abs(r).max()))
    assert err <= bound, f"{name}: max-abs {err:.3e} > {bound:.3e}"


def lowp_gate(x, r, name="", tol=LOWP_REL, floor=1e-30) -> None:
    x = np.asarray(x, dtype=np.float64)
    r = np.asarray(r, dtype=np.float64)
    e = float(np.abs(x - r).max() / max(np.abs(r).max(), floor))
    assert e <= tol, f"{name}: max-rel {e:.3e} > {tol:.1e}"


def run_cuda(kind, q, k, v, do, scale, tau=None, eps_base=0.05, is_causal=True, eps=None, window_size=0,
             doc_ids=None, dtype=torch.float32, path="auto", device="cuda", deterministic=False):
    """Run the CUDA op fwd+bwd; return dict of float64 numpy arrays (out, dq, dk, dv, dscale[, dtau]).

    deterministic=True runs under torch.use_deterministic_algorithms(True), which selects the
    backward without floating-point atomics."""
    qt, kt, vt = (torch.as_tensor(np.asarray(x), dtype=torch.float32).to(device=device, dtype=dtype)
                  .requires_grad_(True) for x in (q, k, v))
    dot = torch.as_tensor(np.asarray(do), dtype=torch.float32).to(device=device, dtype=dtype)
    sc = torch.as_tensor(np.asarray(scale, dtype=np.float32), device=device).requires_grad_(True)
    doc = None if doc_ids is None else torch.as_tensor(np.asarray(doc_ids), device=device)
    prev = fbm.get_kernel_path()
    prev_det = torch.are_deterministic_algorithms_enabled()
    fbm.set_kernel_path(path)
    torch.use_deterministic_algorithms(deterministic)
    try:
        if kind == "plain":
            out = flash_born_attention(qt, kt, vt, sc, is_causal=is_causal, eps=1e-12 if eps is None else eps,
                                       window_size=window_size, doc_ids=doc)
            ta = None
        else:
            ta = torch.as_tensor(np.asarray(tau, dtype=np.float32), device=device).requires_grad_(True)
            out = flash_purified_born_attention(qt, kt, vt, sc, ta, eps_base=eps_base, is_causal=is_causal,
                                                eps=1e-8 if eps is None else eps, window_size=window_size,
                                                doc_ids=doc)
        (out * dot).sum().backward()
        torch.cuda.synchronize()
    finally:
        fbm.set_kernel_path(prev)
        torch.use_deterministic_algorithms(prev_det)
    res = {"out": out, "dq": qt.grad, "dk": kt.grad, "dv": vt.grad, "dscale": sc.grad}
    if ta is not None:
        res["dtau"] = ta.grad
    return {n: t.detach().to(torch.float64).cpu().numpy() for n, t in res.items()}


def run_oracle(kind, q, k, v, do, scale, tau=None, eps_base=0.05, is_causal=True, eps=None, window_size=0,
               doc_ids=None):
    """Float64 oracle on the given (already rounded) inputs; param grads folded to scale's shape."""
    q, k, v, do = (np.asarray(x, dtype=np.float64) for x in (q, k, v, do))
    scale = np.asarray(scale, dtype=np.float64)
    H = q.shape[1]
    if kind == "plain":
        out, z = orc.born_forward(q, k, v, scale, is_causal, 1e-12 if eps is None else eps, window_size, doc_ids)
        g = orc.born_backward(q, k, v, out, z, do, scale, is_causal, window_size, doc_ids)
    else:
        tau = np.asarray(tau, dtype=np.float64)
        out, z = orc.purified_forward(q, k, v, scale, tau, eps_base, is_causal, 1e-8 if eps is None else eps,
                                      window_size, doc_ids)
        g = orc.purified_backward(q, k, v, out, z, do, scale, tau, eps_base, is_causal, window_size, doc_ids)

    def fold(ph, shape):
        return ph.sum().reshape(shape) if int(np.prod(shape)) == 1 else ph.reshape(shape)

    res = {"out": out, "dq": g.dq, "dk": g.dk, "dv": g.dv, "dscale": fold(g.dscale, scale.shape)}
    if kind != "plain":
        res["dtau"] = fold(g.dtau, tau.shape)
    return res


def round_to(x, dtype) -> np.ndarray:
    return torch.as_tensor(np.asarray(x), dtype=torch.float32).to(dtype).to(torch.float64).numpy()


def check_all(got, ref, lowp: bool, names=("out", "dq", "dk", "dv"), floor_rel: float = 1e-3) -> None:
    floor = floor_rel * max(float(np.abs(ref["out"]).max()), float(np.abs(ref["dv"]).max()))
    for n in names:
        if lowp:
            lowp_gate(got[n], ref[n], n, floor=floor)
        else:
            fp32_gate(got[n], ref[n], n)
    gscale = max(1.0, float(np.abs(ref["dq"]).max()), float(np.abs(ref["dk"]).max()))
    for n in ("dscale", "dtau"):
        if n in ref:
            err = float(np.abs(got[n].reshape(ref[n].shape) - ref[n]).max())
            if lowp:
                # max-rel against the parameter gradient's own size, floored for the plain dscale
                # (analytically 2 eps sum delta / (scale Z) ~ 0) at 1e-2 of the dQ/dK scale
                bound = LOWP_REL * max(float(np.abs(ref[n]).max()), 1e-2 * gscale)
            else:
                bound = FP32_ABS * gscale
            assert err <= bound, f"{n}: {err:.3e} > {bound:.3e}"
