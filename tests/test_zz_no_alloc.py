"""icsa_forward_static: the allocation-free entry point.

Some callers cannot allocate device memory where they call the library: a
plugin host that owns every allocation and hands none out, a runtime that
works inside a fixed memory budget, or a foreign-language caller (cgo, JNI)
that has no CUDA allocator at hand.  For them icsa_forward_static keeps its
scratch in a fixed 64 MiB array inside the library; the caller passes only
q, k, v and the output.

This file is collected last on purpose (test_zz_*): if it fails, a run that
stops at the first failure has already run every other test.  It passes run
alone in a fresh process as well as after the other tests.
"""
import ctypes

import pytest
import torch

from in_context_sparse_attention import _capi

pytestmark = pytest.mark.gpu

MAX_ABS_BF16, MEAN_ABS_BF16 = 2e-2, 1e-3


def _lib():
    lib = _capi.load()
    lib.icsa_forward_static.argtypes = [ctypes.POINTER(_capi.Problem)] + [ctypes.c_void_p] * 6
    lib.icsa_forward_static.restype = ctypes.c_int
    lib.icsa_static_scratch_bytes.argtypes = []
    lib.icsa_static_scratch_bytes.restype = ctypes.c_size_t
    lib.icsa_static_device_status.argtypes = [ctypes.c_void_p]
    lib.icsa_static_device_status.restype = ctypes.c_int
    return lib


def _inputs(seed, B, S, H, D, t):
    g = torch.Generator().manual_seed(seed)
    q, k, v = (torch.randn(B, S, H, D, generator=g) for _ in range(3))
    k[:, t:] = 0.8 * k[:, :S - t] + 0.6 * torch.randn(B, S - t, H, D, generator=g)
    return tuple(x.to(torch.bfloat16).cuda() for x in (q, k, v))


def test_static_scratch_matches_workspace_entry_point(cuda_device):
    """Two calls in a row (different inputs, so the second one starts from the
    first one's leftovers) give the same bytes as icsa_forward with its own
    workspace: both run the same deterministic kernels (every reduction in a
    fixed order), so the comparison is exact rather than within the bf16
    tolerance.  The scratch's device status word reports no timeout."""
    lib = _lib()
    B, S, H, D, t = 1, 4096, 2, 128, 2048
    p = _capi.problem(B, S, H, D, t)
    need = lib.icsa_workspace_size(ctypes.byref(p))
    assert 0 < need <= lib.icsa_static_scratch_bytes()
    stream = torch.cuda.current_stream().cuda_stream
    for seed in (101, 202):
        q, k, v = _inputs(seed, B, S, H, D, t)
        ws = torch.empty(need, dtype=torch.uint8, device="cuda")
        ref = torch.empty_like(q)
        _capi.check(lib.icsa_forward(ctypes.byref(p), q.data_ptr(), k.data_ptr(), v.data_ptr(), None, ref.data_ptr(),
                                     ws.data_ptr(), need, stream), "icsa_forward")
        out = torch.empty_like(q)
        _capi.check(lib.icsa_forward_static(ctypes.byref(p), q.data_ptr(), k.data_ptr(), v.data_ptr(), None,
                                            out.data_ptr(), stream), "icsa_forward_static")
        torch.cuda.synchronize()
        d = (out.float() - ref.float()).abs()
        assert float(d.max()) <= MAX_ABS_BF16 and float(d.mean()) <= MEAN_ABS_BF16
        assert torch.equal(out, ref)
        assert lib.icsa_static_device_status(stream) == 0, lib.icsa_last_error()


def test_static_scratch_rejects_oversized_problem(cuda_device):
    lib = _lib()
    p = _capi.problem(1, 65536, 40, 128, 32768)
    assert lib.icsa_workspace_size(ctypes.byref(p)) > lib.icsa_static_scratch_bytes()
    dummy = torch.empty(16, device="cuda")
    rc = lib.icsa_forward_static(ctypes.byref(p), dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(), None,
                                 dummy.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 4  # ICSA_ERR_WORKSPACE
    assert b"static scratch" in lib.icsa_last_error()
