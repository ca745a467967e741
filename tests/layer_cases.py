"""Loader for the reference attention layer's recorded flash-Born calls (tests/golden/layer_*.npz,
made by tests/golden/make_golden_layer.py)."""
from __future__ import annotations

import glob
import os

import numpy as np

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def layer_case_names() -> list[str]:
    return sorted(os.path.basename(p)[len("layer_"):-len(".npz")] for p in glob.glob(os.path.join(GOLDEN_DIR, "layer_*.npz")))


def load_layer_case(name: str) -> dict:
    with np.load(os.path.join(GOLDEN_DIR, f"layer_{name}.npz")) as z:
        c = {k: z[k] for k in z.files}
    for k in ("kind",):
        c[k] = str(c[k])
    for k in ("is_causal", "has_doc", "scale_is_tensor"):
        c[k] = bool(c[k])
    c["window_size"] = int(c["window_size"])
    c["eps"] = float(c["eps"])
    if "eps_base" in c:
        c["eps_base"] = float(c["eps_base"])
    if not c["has_doc"]:
        c["doc_ids"] = None
    return c
