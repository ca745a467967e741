"""Shared loaders for the complex-phase / paired-heads golden fixtures (tests/golden/families_*.npz,
written by tests/golden/make_golden_families.py from the reference attention layer)."""
from __future__ import annotations

import glob
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def family_case_names() -> list[str]:
    return sorted(os.path.basename(p)[len("families_"):-4] for p in glob.glob(os.path.join(GOLDEN, "families_*.npz")))


def load_family_case(name: str) -> dict:
    z = np.load(os.path.join(GOLDEN, f"families_{name}.npz"))
    c = {k: z[k] for k in z.files}
    c["family"] = str(c["family"])
    for k in ("is_causal", "has_doc"):
        c[k] = bool(c[k])
    c["window_size"] = int(c["window_size"])
    c["eps"] = float(c["eps"])
    if not c["has_doc"]:
        c["doc_ids"] = None
    return c


def layer_scale(c: dict) -> np.ndarray:
    """The scale the layer hands the attention core: clamp(head_scale, 1, 100) per head for
    complex phase (layers/attention.py:691-695); the pair mean of head_scale clamped to
    [0.5, 100] for paired heads (:598-601)."""
    hs = c["head_scale"].astype(np.float64)
    if c["family"] == "complex":
        return np.clip(hs, 1.0, 100.0)
    return np.clip(hs.reshape(-1, 2).mean(axis=1), 0.5, 100.0)


def head_scale_grad(c: dict, dscale: np.ndarray) -> np.ndarray:
    """Chain rule from the core's scale gradient to head_scale (clamps pass through: every
    head_scale of the fixtures lies inside them)."""
    if c["family"] == "complex":
        return np.asarray(dscale, dtype=np.float64)
    return np.repeat(np.asarray(dscale, dtype=np.float64) / 2.0, 2)
