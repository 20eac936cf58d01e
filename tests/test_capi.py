"""The C-ABI library: it loads without a GPU, exports every symbol include/nemicli_qmv.h declares,
and refuses bad arguments before any CUDA work (no compute calls here)."""
import ctypes
import os
import re

import pytest

from nemicli_terminal_b200 import _lib
from nemicli_terminal_b200.formats import FORMATS, TYPE_ID

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "nemicli_qmv.h")


def declared():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\**(qmv_\w+)\s*\(", text, re.M)))


def test_header_declares_the_bound_symbols():
    assert declared() == sorted(_lib.exported_symbols())


def test_library_exports_every_declared_symbol():
    L = _lib.load()
    for name in declared():
        assert hasattr(L, name), name


def test_abi_and_status_strings():
    L = _lib.load()
    assert L.qmv_abi_version() == _lib.ABI_VERSION
    for st in range(8):
        assert L.qmv_status_string(st)
    assert L.qmv_status_string(0) == b"ok"


@pytest.mark.parametrize("fmt", list(FORMATS))
def test_block_geometry_matches_format_table(fmt):
    L = _lib.load()
    bv, bb = FORMATS[fmt]
    assert L.qmv_block_values(TYPE_ID[fmt]) == bv
    assert L.qmv_block_bytes(TYPE_ID[fmt]) == bb
    assert L.qmv_supported(TYPE_ID[fmt], bv * 3) == 1
    assert L.qmv_supported(TYPE_ID[fmt], bv * 3 + 16) == 0
    assert L.qmv_supported(TYPE_ID[fmt], 0) == 0
    # the unit of the int32 sums (the buffers qmv_block_sums writes are sized from it)
    from oracle import oracle as O
    assert L.qmv_unit_values(TYPE_ID[fmt]) == O.unit_values(fmt)


def test_unknown_formats_are_refused():
    L = _lib.load()
    for t in (0, 1, 9, 15, 24, 30, 144):          # F32, F16, Q8_1, Q8_K, I8, BF16 and an unassigned id
        assert L.qmv_supported(t, 4096) == 0
        assert L.qmv_block_values(t) == 0
        assert L.qmv_unit_values(t) == 0
    st = L.qmv_mv(15, ctypes.c_void_p(16), 1, 256, ctypes.c_void_p(16), ctypes.c_void_p(16),
                  ctypes.c_void_p(16), ctypes.c_void_p(16), 1, ctypes.c_void_p(16), None)
    assert st == 1


def test_argument_checks_precede_any_launch():
    L = _lib.load()
    a = ctypes.c_void_p(4096)           # never dereferenced: every call below is refused first
    Q4K = TYPE_ID["Q4_K"]
    assert L.qmv_mv(Q4K, None, 1, 256, a, a, a, a, 1, a, None) == 6                 # null
    assert L.qmv_mv(Q4K, a, 0, 256, a, a, a, a, 1, a, None) == 2                    # n_out
    assert L.qmv_mv(Q4K, a, 4, 100, a, a, a, a, 1, a, None) == 2                    # n_in
    assert L.qmv_mv(Q4K, a, 4, 256, a, a, a, a, 0, a, None) == 4                    # tokens
    assert L.qmv_mv(Q4K, ctypes.c_void_p(4098), 4, 256, a, a, a, a, 1, a, None) == 3   # Q4_K wants 16 B
    assert L.qmv_mv(Q4K, a, 4, 256, ctypes.c_void_p(4097), a, a, a, 1, a, None) == 3   # xq alignment
    assert L.qmv_mv_experts(Q4K, a, 144, 4, None, 1, a, a, a, a, 1, a, 1, 256, None) == 6
    assert L.qmv_mv_experts(Q4K, a, 144, 4, a, 0, a, a, a, a, 1, a, 1, 256, None) == 4
    assert L.qmv_mv_experts(Q4K, a, 144, 0, a, 1, a, a, a, a, 1, a, 1, 256, None) == 2
    assert L.qmv_mv_experts(Q4K, a, 100, 4, a, 1, a, a, a, a, 1, a, 1, 256, None) == 2   # expert too small
    assert L.qmv_mv_experts(Q4K, a, 144, 4, a, 1, a, a, a, a, 0, a, 1, 256, None) == 2   # x_group
    assert L.qmv_quant_q8(a, 1, a, a, a, a, 33, None) == 2
    assert L.qmv_quant_q8(None, 1, a, a, a, a, 32, None) == 6
    assert L.qmv_block_sums(Q4K, a, 4, 300, a, a, a, a, None) == 2


def test_moe_argument_checks():
    """qmv_moe_ffn refuses before any launch: null pointers, too many pairs or experts, shapes off the
    block grid, experts smaller than their matrices, misaligned workspace."""
    L = _lib.load()
    a = ctypes.c_void_p(4096)
    Q4K = TYPE_ID["Q4_K"]
    per = 256 * 144                     # 256 rows of one Q4_K superblock

    def call(**kw):
        arg = dict(gt=Q4K, gate=a, up=a, gper=per, dt=Q4K, down=a, dper=per, n_exp=8, ids=a, wts=a, L=4, k=2,
                   x=a, f32=1, stride=256, dim=256, ff=256, ws=a, out=a)
        arg.update(kw)
        return L.qmv_moe_ffn(arg["gt"], arg["gate"], arg["up"], arg["gper"], arg["dt"], arg["down"], arg["dper"],
                             arg["n_exp"], arg["ids"], arg["wts"], arg["L"], arg["k"], arg["x"], arg["f32"],
                             arg["stride"], arg["dim"], arg["ff"], arg["ws"], arg["out"], None)
    assert call(gt=15) == 1
    assert call(ids=None) == 6
    assert call(L=513) == 4                                   # 1026 pairs
    assert call(L=0) == 4
    assert call(n_exp=1025) == 2
    assert call(dim=288, stride=288) == 2                     # not a whole Q4_K superblock
    assert call(stride=128) == 2                              # rows overlap
    assert call(gper=per - 16) == 2
    assert call(ws=ctypes.c_void_p(4096 + 128)) == 3
    assert L.qmv_moe_workspace_bytes(4, 2, 256, 256) > 0
    assert L.qmv_moe_workspace_bytes(4, 2, 250, 256) == 0


def test_multi_matrix_entry_checks():
    """qmv_mv_multi_tok and qmv_mv_multi_ep refuse before any launch: null pointers, job counts, token
    counts, the epilogue's kind, jobs and 32-row groups, misaligned buffers."""
    L = _lib.load()
    a = ctypes.c_void_p(4096)
    Q4K = TYPE_ID["Q4_K"]
    w2 = (ctypes.c_void_p * 2)(4096, 8192)
    y2 = (ctypes.c_void_p * 2)(4096, 8192)
    n2 = (ctypes.c_int * 2)(512, 512)
    n_odd = (ctypes.c_int * 2)(500, 512)
    n_diff = (ctypes.c_int * 2)(512, 256)
    assert L.qmv_mv_multi_tok(Q4K, 2, None, n2, y2, 4096, a, a, a, a, 4, None) == 6
    assert L.qmv_mv_multi_tok(Q4K, 5, w2, n2, y2, 4096, a, a, a, a, 4, None) == 4   # > 4 matrices
    assert L.qmv_mv_multi_tok(Q4K, 2, w2, n2, y2, 4096, a, a, a, a, 0, None) == 4   # tokens
    assert L.qmv_mv_multi_tok(Q4K, 2, w2, n2, y2, 4000, a, a, a, a, 4, None) == 2   # row length

    def ep(kind=1, j0=0, j1=1, n=n2, cnt=a, xq=a, ea=a, n_in=4096):
        return L.qmv_mv_multi_ep(Q4K, 2, w2, n, y2, n_in, a, a, a, a, kind, j0, j1, cnt, xq, a, a, a, ea, None)
    assert ep(cnt=None) == 6
    assert ep(kind=3) == 2
    assert ep(j0=2) == 2
    assert ep(kind=2, j1=0) == 2                                # the same matrix twice
    assert ep(kind=2, ea=None) == 6                             # silu_mul needs its fp32 output
    assert ep(n=n_odd) == 2                                     # not whole 32-row groups
    assert ep(kind=2, n=n_diff) == 2                            # gate and up of different sizes
    assert ep(xq=ctypes.c_void_p(4097)) == 3
    assert ep(n_in=4000) == 2
