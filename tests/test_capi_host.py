"""Host-side checks of the C ABI (CPU only, no kernel launches): the library
loads, exports every function include/*.h declares, derives the
reference's block counts, lays out its workspace consistently and rejects
invalid problems with the documented status codes."""
import ctypes
import os
import re

import pytest

from in_context_sparse_attention import _capi
from oracle import icsa_oracle as orc

INCLUDE = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include")


def declared_functions():
    names = set()
    for h in sorted(os.listdir(INCLUDE)):
        if h.endswith(".h"):
            text = open(os.path.join(INCLUDE, h)).read()
            names |= set(re.findall(r"ICSA_API\s+[\w\s\*]+?\b(icsa_\w+)\s*\(", text))
    return sorted(names)


def test_library_exports_every_declared_function():
    lib = _capi.load()
    names = declared_functions()
    assert len(names) >= 10
    for name in names:
        assert hasattr(lib, name), f"libicsa.so does not export {name}"
    assert b"sm_100a" in lib.icsa_version()


@pytest.mark.parametrize("shape", [
    (1, 8192, 2, 64, 4096),          # configuration 1
    (1, 65536, 40, 128, 32768),      # 480p
    (1, 151296, 40, 128, 75648),     # 720p
    (2, 64 * 37, 3, 128, 64 * 20),   # odd counts, batch 2
    (1, 5000, 2, 128, 2500),         # unaligned t_seq_len and S
])
def test_counts_match_reference_formulas(shape):
    B, S, H, D, t = shape
    p = _capi.problem(B, S, H, D, t)
    c = orc.Counts.make(B, S, H, D, t)
    got = (p.num_blocks, p.n_t, p.n_s, p.topK, p.num_flat, p.k_sparsity, p.tkv, p.nkv, p.top_k)
    want = (c.NB, c.n_t, c.n_s, c.topK, c.num_flat, c.k_sparsity, c.tkv, c.nkv, c.top_k)
    assert got == want


def test_ratios_generalise_the_hard_coded_fractions():
    for sr in (0.0625, 0.125, 0.25):
        for fr in (0.0, 0.5, 1.0):
            p = _capi.problem(1, 16384, 4, 128, 8192, 0.0625, sr, fr)
            c = orc.Counts.make(1, 16384, 4, 128, 8192, 0.0625, sr, fr)
            assert (p.topK, p.num_flat, p.nkv, p.top_k) == (c.topK, c.num_flat, c.nkv, c.top_k)


def test_workspace_layout_is_disjoint_and_aligned():
    for dt in (_capi.ICSA_BF16, _capi.ICSA_F32):
        p = _capi.problem(1, 5000, 2, 128, 2500)
        p.q_dtype = p.k_dtype = dt
        p.debug_keys = 1
        L = _capi.workspace_layout(p)
        size = _capi.load().icsa_workspace_size(ctypes.byref(p))
        assert size == L.total
        offs = sorted(getattr(L, n) for n, _ in _capi.WorkspaceLayout._fields_
                      if n not in ("total", "nkv_pad", "n_sparse") and getattr(L, n))
        assert all(o % 256 == 0 for o in offs)
        assert len(offs) == len(set(offs)) and offs[-1] < L.total
        assert L.nkv_pad % 128 == 0 and L.nkv_pad >= p.nkv
        assert (L.qbf != 0) == (dt == _capi.ICSA_F32)
        assert L.newk != 0  # t_seq_len % 64 != 0 materialises the extended KV


def _status(fn):
    with pytest.raises(_capi.IcsaError) as e:
        fn()
    return e.value.code


def test_invalid_problems_are_rejected():
    assert _status(lambda: _capi.problem(1, 4096, 2, 96, 2048)) == 2       # D outside {64, 128}
    assert _status(lambda: _capi.problem(1, 4096, 2, 128, 5000)) == 1      # t_seq_len > S
    assert _status(lambda: _capi.problem(0, 4096, 2, 128, 2048)) == 1      # empty batch
    assert _status(lambda: _capi.problem(1, 64, 2, 128, 0)) == 1           # empty extended KV
    assert _status(lambda: _capi.problem(1, 4096, 2, 128, 2048, 2.0)) == 1  # top_k > nkv


def test_forward_checks_arguments_before_any_launch():
    lib = _capi.load()
    p = _capi.problem(1, 4096, 2, 128, 2048)
    need = lib.icsa_workspace_size(ctypes.byref(p))
    # undersized workspace
    rc = lib.icsa_forward(ctypes.byref(p), 16, 16, 16, None, 16, 256, need - 1, None)
    assert rc == 4 and b"workspace" in lib.icsa_last_error()
    # misaligned workspace
    rc = lib.icsa_forward(ctypes.byref(p), 16, 16, 16, None, 16, 257, need, None)
    assert rc == 1
    # missing inputs
    rc = lib.icsa_forward(ctypes.byref(p), None, 16, 16, None, 16, 256, need, None)
    assert rc == 1
    # inconsistent hand-edited counts
    p.topK += 1
    assert lib.icsa_workspace_size(ctypes.byref(p)) == 0
