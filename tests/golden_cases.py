"""Loader for the golden vectors in tests/golden (made by tests/golden/make_golden.py)."""
from __future__ import annotations

import json
import os

import numpy as np

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def manifest() -> dict:
    with open(os.path.join(GOLDEN_DIR, "manifest.json")) as f:
        return json.load(f)


def case_names() -> list[str]:
    return sorted(k for k in manifest() if k != "C1")


def load_case(name: str) -> dict:
    meta = manifest()[name]
    with np.load(os.path.join(GOLDEN_DIR, f"{name}.npz")) as z:
        arrays = {k: z[k] for k in z.files}
    case = dict(meta)
    case.update(arrays)
    case["doc_ids"] = arrays.get("doc_ids")
    return case


def c1_inputs():
    """C1 inputs exactly as the benchmark config defines them (torch CPU generator)."""
    import torch

    torch.manual_seed(0)
    q = torch.randn(2, 4, 256, 64)
    k = torch.randn(2, 4, 256, 64)
    v = torch.randn(2, 4, 256, 64)
    torch.manual_seed(1)
    do = torch.randn(2, 4, 256, 64)
    return q, k, v, do
