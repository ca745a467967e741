"""quantumdlblocks_b200 -- B200-native (sm_100a) flash-Born attention for QuantumDLBlocks.

The hot path of QuantumDLBlocks' Born-attention GPTs (``qdlblocks.flash_born_attention`` and
``qdlblocks.flash_purified_born_attention``) rebuilt as hand-written CUDA behind a C ABI
(``include/flashborn_b200.h``, ``libflashborn_b200.so``), with the reference's Python call
signatures and tensor layout so callers swap it in unchanged (see ``swap``).
"""
from .kernels import (
    HAS_TRITON,
    IS_HIP,
    complex_phase_born_attention,
    flash_born_attention,
    flash_born_attention_token_major,
    flash_purified_born_attention,
    get_flash_born_launch_meta,
    get_rdna4_autotune_configs,
    paired_heads_born_attention,
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
