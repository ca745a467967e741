"""Host-side logic of the drop-in module (no GPU)."""
from __future__ import annotations

import pytest
import torch

import quantumdlblocks_b200 as fbk
from quantumdlblocks_b200.kernels import flash_born as fbm


def test_public_names_match_reference_surface():
    # qdlblocks.kernels re-exports these names for flash-Born (kernels/__init__.py:3-10)
    for name in ("HAS_TRITON", "IS_HIP", "flash_born_attention", "flash_purified_born_attention",
                 "get_flash_born_launch_meta", "get_rdna4_autotune_configs"):
        assert hasattr(fbk, name)
        assert hasattr(fbk.kernels, name)
    assert fbk.IS_HIP is False
    assert fbk.HAS_TRITON is True  # the library is built in-tree


def test_launch_metadata_pins_of_the_reference_tests():
    # tests/test_flash_born.py:70-83 of the reference
    hip = fbk.get_flash_born_launch_meta(64, is_hip=True)
    assert hip["num_warps"] == 4 and hip["waves_per_eu"] == 2
    cuda = fbk.get_flash_born_launch_meta(64, is_hip=False)
    assert cuda["num_warps"] == 4 and "waves_per_eu" not in cuda
    cfgs = fbk.get_rdna4_autotune_configs()
    assert len(cfgs) == 4
    assert all(c["matrix_instr_nonkdim"] == 16 and c["waves_per_eu"] in (2, 4) for c in cfgs)
    # tests/test_plan049_...py:308-319 of the reference
    assert fbk.get_flash_born_launch_meta(512, head_dim=64)["BLOCK_M"] == 64
    assert fbk.get_flash_born_launch_meta(512, head_dim=64)["BLOCK_N"] == 64
    for hd in (48, 80, 96, 112):
        assert fbk.get_flash_born_launch_meta(512, head_dim=hd)["BLOCK_M"] in (32, 64)


def test_cpu_tensors_raise_no_fallback():
    x = torch.randn(1, 2, 8, 16)
    with pytest.raises(RuntimeError, match="CUDA"):
        fbk.flash_born_attention(x, x, x, 1.0)
    with pytest.raises(RuntimeError, match="CUDA"):
        fbk.flash_purified_born_attention(x, x, x)


def test_kernel_path_override():
    assert fbm.get_kernel_path() == "auto"
    fbm.set_kernel_path("general")
    try:
        assert fbm.get_kernel_path() == "general"
    finally:
        fbm.set_kernel_path("auto")
    with pytest.raises(ValueError):
        fbm.set_kernel_path("triton")


def test_swap_rebinds_reference_names_and_restores_them(monkeypatch):
    """install() patches every module attribute the reference binds the kernels to."""
    import sys
    import types

    from quantumdlblocks_b200 import swap

    orig = object()
    fake = {}
    for modname, names in swap.TARGETS.items():
        m = types.ModuleType(modname)
        for n in names:
            setattr(m, n, orig)
        fake[modname] = m
        monkeypatch.setitem(sys.modules, modname, m)
    patched = swap.install(import_missing=False)
    assert len(patched) == sum(len(v) for v in swap.TARGETS.values())
    assert sys.modules["qdlblocks.layers.attention"].flash_born_attention is fbm.flash_born_attention_token_major
    assert sys.modules["qdlblocks.kernels"].flash_born_attention is fbk.flash_born_attention
    assert sys.modules["qdlblocks.kernels.flash_born"]._run_triton_flash_born is fbm._run_triton_flash_born
    swap.uninstall()
    assert all(getattr(fake[m], n) is orig for m, ns in swap.TARGETS.items() for n in ns)


def test_prologue_ops_raise_on_cpu_and_check_shapes():
    from quantumdlblocks_b200.kernels.prologue import l2_normalize, qkv_rope_l2norm, rope_tables

    cos, sin = rope_tables(8, 64)
    assert cos.shape == (8, 32) and torch.allclose(cos[0], torch.ones(32)) and torch.allclose(sin[0], torch.zeros(32))
    with pytest.raises(RuntimeError, match="CUDA"):
        qkv_rope_l2norm(torch.zeros(1, 8, 3 * 64), cos, sin, 1)
    with pytest.raises(RuntimeError, match="CUDA"):
        l2_normalize(torch.zeros(2, 8))


def test_family_and_loss_ops_raise_on_cpu():
    """No CPU fallback: the families and the loss refuse CPU tensors, and check their shapes."""
    from quantumdlblocks_b200 import complex_phase_born_attention, paired_heads_born_attention
    from quantumdlblocks_b200.kernels.xent import cross_entropy

    x = torch.zeros(1, 2, 8, 16)
    for fn in (complex_phase_born_attention, paired_heads_born_attention):
        with pytest.raises(RuntimeError, match="CUDA"):
            fn(x, x, x, 4.0)
    with pytest.raises(RuntimeError, match="CUDA"):
        cross_entropy(torch.zeros(4, 64, dtype=torch.bfloat16), torch.zeros(4, dtype=torch.int64))


def test_finalize_heads_raises_on_cpu():
    from quantumdlblocks_b200.kernels.epilogue import finalize_heads

    with pytest.raises(RuntimeError, match="CUDA"):
        finalize_heads(torch.zeros(1, 2, 4, 64))
