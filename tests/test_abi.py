"""The C-ABI library: it loads, exports every entry point declared in
include/pasa_b200.h, and validates arguments on the host (no GPU needed)."""
import ctypes
import math
import re

import pytest

from conftest import ROOT
from pasa_b200 import _lib

HEADER = (ROOT / "include" / "pasa_b200.h").read_text()


def declared_symbols():
    return sorted(set(re.findall(r"^PASA_API\s+[\w\s\*]+?\b(pasa_\w+)\s*\(", HEADER, flags=re.M)))


def test_library_loads_and_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_symbols()
    assert len(names) >= 9
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(_lib.EXPORTS)
    assert lib.pasa_abi_version() == 1


def test_status_strings():
    for code in range(0, 10):
        assert _lib.status_string(code)
    assert "unknown" in _lib.status_string(1234)


@pytest.mark.parametrize("T,density", [(1024, 0.25), (1000, 0.3), (75600, 0.1), (119056, 0.1), (32760, 0.15),
                                       (640, 0.01), (700, 1.0), (64, 0.5), (65, 2.0), (3000, 0.0),
                                       (3000, -1.0), (4096, 0.123456)])
def test_derive_matches_reference_formula(T, density):
    NT = math.ceil(T / 64)
    ref_ns = min(max(1, int(density * NT)), NT)  # group_pisa_attention.py:373
    nt, ng, ns = _lib.derive(T, density)
    assert (nt, ng, ns) == (NT, math.ceil(NT / 32), ref_ns)


def test_derive_rejects_bad_arguments():
    with pytest.raises(ValueError):
        _lib.derive(1024, float("nan"))
    with pytest.raises(ValueError):
        _lib.derive(0, 0.1)
    with pytest.raises(ValueError):
        _lib.derive(1024, 0.1, block=128)


def test_workspace_size_grows_with_problem():
    a = _lib.workspace_size(1, 4, 1024, 64, _lib.F32, 4)
    b = _lib.workspace_size(1, 40, 75600, 128, _lib.BF16, 118)
    assert 0 < a < b
    assert b % 256 == 0
    with pytest.raises(ValueError):
        _lib.workspace_size(1, 4, 1024, 96, _lib.BF16, 4)  # head_dim 96 unsupported
    with pytest.raises(ValueError):
        _lib.workspace_size(1, 4, 1024, 64, 7, 4)  # bad dtype code
    with pytest.raises(ValueError):
        _lib.workspace_size(1, 4, 1024, 64, _lib.BF16, 17)  # ns > NT


def test_entry_points_validate_before_touching_the_device():
    lib = _lib.load()
    p = ctypes.c_void_p(4096)          # aligned fake pointer: never dereferenced
    bad = ctypes.c_void_p(4096 + 8)    # misaligned
    assert lib.pasa_prep(None, p, p, p, 1, 1, 128, 96, _lib.BF16, 64, 32, p, p, p, p, p) == _lib.ERR_UNSUPPORTED
    assert lib.pasa_prep(None, p, p, p, 1, 1, 128, 64, 5, 64, 32, p, p, p, p, p) == _lib.ERR_DTYPE
    assert lib.pasa_prep(None, bad, p, p, 1, 1, 128, 64, _lib.BF16, 64, 32, p, p, p, p, p) == _lib.ERR_ALIGN
    assert lib.pasa_prep(None, None, p, p, 1, 1, 128, 64, _lib.BF16, 64, 32, p, p, p, p, p) == _lib.ERR_NULL
    assert lib.pasa_prep(None, p, p, p, 1, 1, 0, 64, _lib.BF16, 64, 32, p, p, p, p, p) == _lib.ERR_SHAPE
    assert lib.pasa_select(None, p, p, p, None, 1, 16, 64, _lib.BF16, 0.125, 1, 17, p, p) == _lib.ERR_SHAPE
    assert lib.pasa_select(None, p, p, None, None, 1, 16, 64, _lib.BF16, 0.125, 1, 4, p, p) == _lib.ERR_NULL
    assert lib.pasa_attn(None, p, p, p, p, p, p, p, p, 1, 1024, 64, _lib.F32, 0.125, 4, p, None,
                         _lib.ATTN_TCGEN05) != _lib.OK
    assert lib.pasa_forward(None, p, p, p, 1, 1, 1024, 64, _lib.BF16, float("inf"), 0.125, 1, None, p, 1 << 30,
                            p, 0) == _lib.ERR_DENSITY
    assert lib.pasa_forward(None, p, p, p, 1, 1, 1024, 64, _lib.BF16, 0.25, 0.125, 1, None, p, 16, p,
                            0) == _lib.ERR_WORKSPACE
    # placement: seq_len must be context + frames * frame_size (placement.py:128)
    assert lib.pasa_place(None, p, p, p, 1, 2, 100, 64, _lib.BF16, 4, 3, 30, 0) == _lib.ERR_SHAPE
    # DiT row kernels: cols a multiple of 8 and at most 8192, known norm mode,
    # gate only with add, scale and shift together, 16-byte alignment
    rn = lambda x, add, gate, scale, shift, rows, brows, cols, norm: lib.pasa_dit_row_norm(
        None, x, add, gate, None, None, None, scale, shift, rows, brows, cols, 1e-6, norm, p)
    assert rn(p, None, None, None, None, 4, 4, 5121, 1) == _lib.ERR_SHAPE
    assert rn(p, None, None, None, None, 4, 4, 8200, 1) == _lib.ERR_SHAPE
    assert rn(p, None, None, None, None, 4, 3, 64, 1) == _lib.ERR_SHAPE       # rows % batch_rows
    assert rn(p, None, None, None, None, 4, 4, 64, 3) == _lib.ERR_UNSUPPORTED
    assert rn(p, None, p, None, None, 4, 4, 64, 1) == _lib.ERR_NULL           # gate without add
    assert rn(p, None, None, p, None, 4, 4, 64, 1) == _lib.ERR_NULL           # scale without shift
    assert rn(bad, None, None, None, None, 4, 4, 64, 1) == _lib.ERR_ALIGN
    qr = lambda xq, xk, wk, cos, sin, heads, hd: lib.pasa_dit_qkv_rope(
        None, xq, xk, None, p, wk, cos, sin, 1, 16, heads, hd, 1e-6, 1, p, p, None)
    assert qr(p, None, None, None, None, 40, 12) == _lib.ERR_SHAPE            # head_dim % 8
    assert qr(p, None, None, None, None, 80, 128) == _lib.ERR_SHAPE           # cols > 8192
    assert qr(p, p, None, None, None, 40, 128) == _lib.ERR_NULL               # xk without wk
    assert qr(p, None, None, p, None, 40, 128) == _lib.ERR_NULL               # cos without sin
    assert qr(bad, None, None, None, None, 40, 128) == _lib.ERR_ALIGN
