"""Swap the B200 flash-Born kernels into an existing QuantumDLBlocks (``qdlblocks``) install.

The reference binds the kernel names at import time in several modules
(``src/qdlblocks/layers/attention.py:20`` imports ``flash_born_attention`` and
``flash_purified_born_attention`` from ``..kernels``; ``qdlblocks/__init__.py`` and
``qdlblocks/kernels/__init__.py`` re-export them).  ``install()`` rebinds every one of those
module attributes to this package's implementation, so the reference's layers and GPTs
(``SubspaceProjectorBornAttention`` and the models built on it) call the B200 kernels unchanged.
``uninstall()`` restores the originals.

The attention layer's own binding gets the token-major variant: the layer's only use of the
result is ``_finalize_heads``' head merge (``layers/attention.py:492``), which then costs no copy.
"""
from __future__ import annotations

import importlib
import sys
from types import ModuleType

from .kernels import flash_born as _fb

# module -> names that hold the reference's kernel entry points
TARGETS = {
    "qdlblocks.kernels.flash_born": ("flash_born_attention", "flash_purified_born_attention", "_run_triton_flash_born"),
    "qdlblocks.kernels": ("flash_born_attention", "flash_purified_born_attention"),
    "qdlblocks.layers.attention": ("flash_born_attention", "flash_purified_born_attention"),
    "qdlblocks": ("flash_born_attention", "flash_purified_born_attention"),
}

REPLACEMENTS = {
    "flash_born_attention": _fb.flash_born_attention,
    "flash_purified_born_attention": _fb.flash_purified_born_attention,
    "_run_triton_flash_born": _fb._run_triton_flash_born,
}

# (module, name) bindings that get a different implementation from REPLACEMENTS[name]
LAYER_OVERRIDES = {
    ("qdlblocks.layers.attention", "flash_born_attention"): _fb.flash_born_attention_token_major,
}

_saved: dict[tuple[str, str], object] = {}


def _module(name: str, import_missing: bool) -> ModuleType | None:
    mod = sys.modules.get(name)
    if mod is None and import_missing:
        try:
            mod = importlib.import_module(name)
        except ImportError:
            mod = None
    return mod


def install(import_missing: bool = True) -> list[str]:
    """Rebind the reference's flash-Born names to the B200 kernels; returns the patched names."""
    patched = []
    for modname, names in TARGETS.items():
        mod = _module(modname, import_missing)
        if mod is None:
            continue
        for name in names:
            if hasattr(mod, name):
                _saved.setdefault((modname, name), getattr(mod, name))
                setattr(mod, name, LAYER_OVERRIDES.get((modname, name), REPLACEMENTS[name]))
                patched.append(f"{modname}.{name}")
    return patched


def uninstall() -> None:
    """Restore every attribute that install() replaced."""
    for (modname, name), orig in list(_saved.items()):
        mod = sys.modules.get(modname)
        if mod is not None:
            setattr(mod, name, orig)
        del _saved[(modname, name)]
