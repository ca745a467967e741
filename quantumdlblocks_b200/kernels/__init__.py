"""B200 flash-Born kernels: the import surface of ``qdlblocks.kernels`` for this path.

Mirrors the names the reference re-exports for flash-Born (``src/qdlblocks/kernels/__init__.py:3-10``).
"""
from .families import complex_phase_born_attention, paired_heads_born_attention
from .flash_born import (
    HAS_TRITON,
    IS_HIP,
    flash_born_attention,
    flash_born_attention_token_major,
    flash_purified_born_attention,
    get_flash_born_launch_meta,
    get_rdna4_autotune_configs,
)

__all__ = [
    "HAS_TRITON",
    "IS_HIP",
    "complex_phase_born_attention",
    "flash_born_attention",
    "flash_born_attention_token_major",
    "flash_purified_born_attention",
    "get_flash_born_launch_meta",
    "get_rdna4_autotune_configs",
    "paired_heads_born_attention",
]
