"""The C ABI without a GPU: the library loads, exports every declared symbol, its struct layout
matches the header, and host-side validation returns status codes (no device work)."""
from __future__ import annotations

import ctypes
import os
import re
import shutil
import subprocess

import pytest

from quantumdlblocks_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "flashborn_b200.h")


def declared_symbols() -> list[str]:
    text = open(HEADER).read()
    return sorted(set(re.findall(r"FB_API\s+[\w\s\*]+?\b(fb_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    syms = declared_symbols()
    assert len(syms) >= 11
    for name in syms:
        assert hasattr(lib, name), name
    assert set(syms) == set(_lib.SIGNATURES), "ctypes signature table out of sync with the header"


def test_abi_version_and_strerror():
    lib = _lib.load()
    assert lib.fb_abi_version() == 4
    for code in range(0, 10):
        msg = lib.fb_strerror(code).decode()
        assert msg and (code == 0 or msg.startswith("flashborn:"))
    assert b"unknown" in lib.fb_strerror(1234)


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc needed for the layout probe")
def test_struct_layout_matches_header(tmp_path):
    fields = [f[0] for f in _lib.FbAttnArgs._fields_]
    src = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{HEADER}"', "int main(void){",
           'printf("size %zu\\n", sizeof(fb_attn_args));']
    for f in fields:
        src.append(f'printf("{f} %zu\\n", offsetof(fb_attn_args, {f}));')
    src.append("return 0;}")
    c = tmp_path / "probe.c"
    c.write_text("\n".join(src))
    exe = tmp_path / "probe"
    subprocess.run(["gcc", "-std=c99", str(c), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split("\n")
    got = dict(line.split() for line in out if line.strip())
    assert int(got["size"]) == ctypes.sizeof(_lib.FbAttnArgs)
    for f in fields:
        assert int(got[f]) == getattr(_lib.FbAttnArgs, f).offset, f


def _args(**kw) -> _lib.FbAttnArgs:
    a = _lib.FbAttnArgs()
    a.batch, a.heads, a.seq_len, a.head_dim = 2, 4, 64, 64
    a.dtype = a.out_dtype = _lib.FB_BF16
    a.is_causal = 1
    a.eps = 1e-12
    fake = 0x10000  # never dereferenced: validation fails or nothing is launched
    for name in ("q", "k", "v", "out", "z", "scale", "dout", "dq", "dk", "dv", "dscale", "workspace"):
        setattr(a, name, fake)
    a.scale_numel = 1
    for n in ("q", "k", "v", "out", "dout", "dq", "dk", "dv"):
        setattr(a, n + "_stride", _lib._I64x4(4 * 64 * 64, 64 * 64, 64, 1))
    for k_, v_ in kw.items():
        setattr(a, k_, v_)
    return a


@pytest.mark.parametrize(
    "kw,code",
    [
        (dict(head_dim=0), _lib.FB_ERR_SHAPE),
        (dict(head_dim=257), _lib.FB_ERR_SHAPE),
        (dict(seq_len=-1), _lib.FB_ERR_SHAPE),
        (dict(dtype=7), _lib.FB_ERR_DTYPE),
        (dict(out_dtype=_lib.FB_F16), _lib.FB_ERR_DTYPE),  # plain out: the input dtype or fp32
        (dict(scale=None), _lib.FB_ERR_ARG),
        (dict(scale_numel=3), _lib.FB_ERR_ARG),
        (dict(window_size=-2), _lib.FB_ERR_ARG),
        (dict(q=None), _lib.FB_ERR_ARG),
        (dict(z=None), _lib.FB_ERR_ARG),
        (dict(path=9), _lib.FB_ERR_ARG),
    ],
)
def test_forward_validation_without_gpu(kw, code):
    lib = _lib.load()
    assert lib.fb_born_fwd(ctypes.byref(_args(**kw)), None) == code


def test_purified_validation_without_gpu():
    lib = _lib.load()
    a = _args(out_dtype=_lib.FB_F32)
    assert lib.fb_purified_born_fwd(ctypes.byref(a), None) == _lib.FB_ERR_ARG  # tau missing
    a.tau, a.tau_numel = 0x10000, 5
    assert lib.fb_purified_born_fwd(ctypes.byref(a), None) == _lib.FB_ERR_ARG  # tau length
    a.tau_numel = 4
    a.dtau = None
    assert lib.fb_purified_born_bwd(ctypes.byref(a), None) == _lib.FB_ERR_ARG  # dtau missing


def test_backward_validation_without_gpu():
    lib = _lib.load()
    assert lib.fb_born_bwd(ctypes.byref(_args(dscale=None)), None) == _lib.FB_ERR_ARG
    assert lib.fb_born_bwd(ctypes.byref(_args(dq=None)), None) == _lib.FB_ERR_ARG
    a = _args()
    need = lib.fb_bwd_workspace_size(ctypes.byref(a))
    assert need > 0
    a.workspace_bytes = need - 1
    assert lib.fb_born_bwd(ctypes.byref(a), None) == _lib.FB_ERR_WORKSPACE


def test_empty_problem_is_a_noop():
    lib = _lib.load()
    for kw in (dict(seq_len=0), dict(batch=0), dict(heads=0)):
        a = _args(**kw)
        assert lib.fb_born_fwd(ctypes.byref(a), None) == _lib.FB_OK
        assert lib.fb_last_launch_count() == 0


def test_path_selection_is_host_only():
    lib = _lib.load()
    # fp32 never takes the tensor-core path; forcing it is refused with a status code
    a = _args(dtype=_lib.FB_F32, out_dtype=_lib.FB_F32)
    assert lib.fb_select_path(ctypes.byref(a), 0) == _lib.FB_PATH_GENERAL
    a.path = _lib.FB_PATH_TCGEN05
    assert lib.fb_select_path(ctypes.byref(a), 0) == -_lib.FB_ERR_UNSUPPORTED
    assert lib.fb_born_fwd(ctypes.byref(a), None) == _lib.FB_ERR_UNSUPPORTED
    a.path = _lib.FB_PATH_GENERAL
    assert lib.fb_select_path(ctypes.byref(a), 1) == _lib.FB_PATH_GENERAL


def test_cross_entropy_validation_without_gpu():
    lib = _lib.load()
    a = _lib.FbXentArgs()
    a.rows, a.vocab, a.ld = 4, 64, 64
    a.logits = a.targets = a.lse = a.loss = 0x10000  # never dereferenced: validation fails first
    for field, val, code in (("vocab", 63, _lib.FB_ERR_SHAPE), ("ld", 32, _lib.FB_ERR_SHAPE),
                             ("logits", None, _lib.FB_ERR_ARG), ("logits", 0x10008, _lib.FB_ERR_ALIGN)):
        b = _lib.FbXentArgs.from_buffer_copy(a)
        setattr(b, field, val)
        assert lib.fb_xent_fwd(ctypes.byref(b), None) == code, field
    assert lib.fb_xent_bwd(ctypes.byref(a), None) == _lib.FB_ERR_ARG  # grad / gscale missing


def test_heads_epilogue_validation_without_gpu():
    lib = _lib.load()
    a = _lib.FbHeadsArgs()
    a.batch, a.heads, a.seq_len, a.head_dim, a.dtype = 1, 2, 4, 64, _lib.FB_BF16
    a.o, a.y = 0x10000, 0x10000  # never dereferenced: validation fails first
    a.o_stride = _lib._I64x4(512, 256, 64, 1)
    b = _lib.FbHeadsArgs.from_buffer_copy(a)
    b.head_dim = 48
    assert lib.fb_heads_epilogue_fwd(ctypes.byref(b), None) == _lib.FB_ERR_SHAPE
    b = _lib.FbHeadsArgs.from_buffer_copy(a)
    b.xsa_alpha = 0x10000  # XSA without v
    assert lib.fb_heads_epilogue_fwd(ctypes.byref(b), None) == _lib.FB_ERR_ARG
    b = _lib.FbHeadsArgs.from_buffer_copy(a)
    b.o_stride = _lib._I64x4(512, 256, 63, 1)
    assert lib.fb_heads_epilogue_fwd(ctypes.byref(b), None) == _lib.FB_ERR_ALIGN
    b = _lib.FbHeadsArgs.from_buffer_copy(a)
    b.gate_x, b.gate_channels = 0x10000, 9  # more gate channels than the kernel holds
    assert lib.fb_heads_epilogue_fwd(ctypes.byref(b), None) == _lib.FB_ERR_ARG
    assert lib.fb_heads_epilogue_bwd(ctypes.byref(a), None) == _lib.FB_ERR_ARG  # dy / grad_o missing
