"""Device-side timeouts reach the caller, and side streams under capture.

Every wait inside the kernels is bounded: one that gives up records a status
code and the kernel returns.  These tests make a wait run out without any
fault -- icsa_wait_selftest waits on an mbarrier that nothing arrives at --
and check that each product path then raises instead of returning as if the
call had succeeded:
* the per-device record read by icsa_last_status (and device_status());
* the drop-in on CUDA tensors with check=True;
* the drop-in on pinned host tensors (always checked when blocking).
A last test makes an eager call on one stream while a call on another stream
is being captured into a CUDA graph; the library's side streams keep the two
apart.
"""
import ctypes

import pytest
import torch

from in_context_sparse_attention import IcsaError, _capi, device_status, editing_sparse_attention

pytestmark = pytest.mark.gpu

B, S, H, D, T = 1, 4096, 2, 128, 2048


def _inputs(seed):
    g = torch.Generator().manual_seed(seed)
    return tuple(torch.randn(B, S, H, D, generator=g).to(torch.bfloat16) for _ in range(3))


def _timeout_once(lib):
    """Runs the self-test: one bounded wait gives up after about a second."""
    ws = torch.zeros(256, dtype=torch.uint8, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    assert lib.icsa_wait_selftest(ws.data_ptr(), st) == 0
    torch.cuda.synchronize()
    return ws


def test_sticky_record_reports_and_clears(cuda_device):
    lib = _capi.load()
    st = torch.cuda.current_stream().cuda_stream
    lib.icsa_last_status(st, 1)  # start from a clear record
    _timeout_once(lib)
    assert lib.icsa_last_status(st, 0) == 5  # ICSA_ERR_DEVICE_TIMEOUT, kept
    assert b"gave up" in lib.icsa_last_error()
    with pytest.raises(IcsaError) as e:
        device_status()
    assert e.value.code == 5
    assert lib.icsa_last_status(st, 1) == 0  # device_status() cleared it
    device_status()


def test_checked_device_call_raises_after_a_timeout(cuda_device):
    lib = _capi.load()
    q, k, v = (x.cuda() for x in _inputs(1))
    want = editing_sparse_attention(q, k, v, T, S - T, check=True)
    _timeout_once(lib)
    with pytest.raises(IcsaError) as e:
        editing_sparse_attention(q, k, v, T, S - T, check=True)
    assert e.value.code == 5
    again = editing_sparse_attention(q, k, v, T, S - T, check=True)  # the record was cleared
    assert torch.equal(again, want)


def test_pinned_host_call_raises_after_a_timeout(cuda_device):
    lib = _capi.load()
    hq, hk, hv = (x.pin_memory() for x in _inputs(2))
    want = editing_sparse_attention(hq, hk, hv, T, S - T)
    _timeout_once(lib)
    with pytest.raises(IcsaError) as e:
        editing_sparse_attention(hq, hk, hv, T, S - T)
    assert e.value.code == 5
    assert torch.equal(editing_sparse_attention(hq, hk, hv, T, S - T), want)


def test_eager_call_on_another_stream_during_a_capture(cuda_device):
    """While stream A is being captured (its side work joins the capture), an
    eager call on stream B runs to the right result on side streams of its
    own, and the captured graph replays to the right result afterwards."""
    lib = _capi.load()
    qa, ka, va = (x.cuda() for x in _inputs(3))
    qb, kb, vb = (x.cuda() for x in _inputs(4))
    want_a = editing_sparse_attention(qa, ka, va, T, S - T)
    want_b = editing_sparse_attention(qb, kb, vb, T, S - T)
    p = _capi.problem(B, S, H, D, T)
    size = lib.icsa_workspace_size(ctypes.byref(p))
    ws_b = torch.empty(size, dtype=torch.uint8, device="cuda")
    out_b = torch.empty_like(qb)
    sb = torch.cuda.Stream()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out_a = editing_sparse_attention(qa, ka, va, T, S - T)
        # eager, on stream B, with buffers allocated before the capture
        rc = lib.icsa_forward(ctypes.byref(p), qb.data_ptr(), kb.data_ptr(), vb.data_ptr(), None, out_b.data_ptr(),
                              ws_b.data_ptr(), size, sb.cuda_stream)
    assert rc == 0, lib.icsa_last_error()
    sb.synchronize()
    assert torch.equal(out_b, want_b)
    out_a.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out_a, want_a)
    assert lib.icsa_device_status(ws_b.data_ptr(), sb.cuda_stream) == 0
    del g
