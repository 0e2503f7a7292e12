"""Drop-in replacement of the reference's
``in_context_sparse_attention.editing_sparse_attention``
(in_context_sparse_attention/editing_sparse_attention.py:67-232 of the
reference), running every stage on the B200 through libicsa.so.

Same positional/keyword signature, same result shape and dtype rules:

    x = editing_sparse_attention(q, k, v, t_seq_len, s_seq_len,
                                 alpha_2=1.0, alpha_3=1.0, SPARSITY_RATIO=0.0625,
                                 backend='b200')

* q, k, v: [B, S, H, D] CUDA tensors (bf16 or fp32), D in {64, 128}; or
  pinned (page-locked) CPU tensors, which are streamed through the current
  CUDA device by groups of heads (copy in, compute and copy out overlap on
  three streams) and give a pinned CPU result.  Ordinary CPU tensors are
  refused: there is no CPU fallback.
* t_seq_len: target-video tokens.  s_seq_len and alpha_3 are accepted and
  unused, exactly as in the reference (only t_seq_len and S enter the
  computation).
* alpha_2: python number or a tensor broadcastable to [B, S, H, D] (the DiT
  passes a per-token gate of shape [B, S, 1, 1]).
* backend: ``'b200'``.  The reference's names ``'tilelang'`` and ``'triton'``
  are accepted so that an unchanged ``attention.backend`` entry of
  inference.yaml keeps working; all three run the same kernels, which
  reproduce the tilelang backend's semantics (BN = 64 interval term).  Any
  other name raises ValueError like Backend.validate of the reference.
* keyword-only select_ratio / flat_ratio generalise the reference's
  hard-coded ``n_s // 8`` retrieved source blocks and ``NB // 2`` flat blocks
  (defaults reproduce them).

With CUDA inputs the call is asynchronous on the current CUDA stream,
performs no host synchronisation and allocates only its output and one
workspace from the PyTorch caching allocator, so it can be captured in a CUDA
graph.  With pinned CPU inputs it returns once the result is in host memory,
unless ``non_blocking=True`` (then synchronise the current stream before
reading the result); ``out=`` takes a preallocated pinned result tensor.

Device-side timeouts.  Every wait inside the kernels is bounded (about one
second); a wait that gives up records a status code instead of hanging, and
the kernel returns with an unfinished result.  The reference raises on
failure (its host asserts, tilelang_host.py:251-260), so this package raises
IcsaError (a RuntimeError) when such a code is found:
* pinned CPU inputs with ``non_blocking=False``: always, after the result has
  reached host memory;
* CUDA inputs: with ``check=True`` (or the environment variable
  ICSA_CHECK_STATUS=1), which synchronises the stream after the call; the
  check is skipped while the stream is being captured into a CUDA graph;
* otherwise: ``device_status()``, which synchronises and reports a wait that
  gave up in any call on the device since the last check.
"""
from __future__ import annotations

import ctypes
import numbers
import os

import torch

from . import _capi

BLOCK_M = 64
_CHECK_DEFAULT = os.environ.get("ICSA_CHECK_STATUS", "0") not in ("", "0")


def _check_status(lib, ws_ptr, stream_handle, where):
    """Synchronises `stream_handle` and raises IcsaError if a device-side
    wait gave up: the per-device record (icsa_last_status, cleared by this
    check) covers every call on the device since the last check, the
    workspace status word `ws_ptr` (when given) this call."""
    rc = lib.icsa_last_status(stream_handle, 1)
    _capi.check(rc, where)
    if ws_ptr:
        _capi.check(lib.icsa_device_status(ws_ptr, stream_handle), where)


def device_status(device=None):
    """Synchronises the current stream of `device` (default: the current
    CUDA device) and raises IcsaError if a device-side wait of any call on
    that device gave up since the last check; clears the record."""
    lib = _capi.load()
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(dev):
        _check_status(lib, None, torch.cuda.current_stream(dev).cuda_stream, "device_status")


class Backend:
    """Backend names.  B200 is the implementation; TILELANG and TRITON are the
    reference's names, accepted as aliases of it."""
    B200 = "b200"
    TILELANG = "tilelang"
    TRITON = "triton"

    @classmethod
    def validate(cls, backend: str) -> str:
        if backend not in (cls.B200, cls.TILELANG, cls.TRITON):
            raise ValueError(f"Unknown backend '{backend}'.  Valid: {cls.B200}, {cls.TILELANG}, {cls.TRITON}")
        return backend


_DT = {torch.bfloat16: _capi.ICSA_BF16, torch.float32: _capi.ICSA_F32}


def _result_dtypes(q_dtype, k_dtype, v_dtype, alpha):
    """dtypes the reference produces (torch type promotion): out_compress is
    bf16 when any input is bf16 (mixed fp32 q/k with bf16 v only runs under
    CUDA autocast, where the compressed matmuls are bf16); out_compress*alpha
    follows promotion with a tensor alpha; the output is promote(q, that)."""
    autocast_bf16 = torch.is_autocast_enabled("cuda") and torch.get_autocast_dtype("cuda") == torch.bfloat16
    outc = torch.bfloat16 if (torch.bfloat16 in (q_dtype, k_dtype, v_dtype) or autocast_bf16) else torch.float32
    ca = torch.promote_types(outc, alpha.dtype) if isinstance(alpha, torch.Tensor) else outc
    out = torch.promote_types(q_dtype, ca)
    return outc, ca, out


def _is_host(x) -> bool:
    """True for a pinned CPU tensor (streamed through the GPU); raises for
    any other non-CUDA tensor."""
    if x.is_cuda:
        return False
    if x.device.type == "cpu" and x.is_pinned():
        return True
    raise RuntimeError(f"tensor is on {x.device}: the b200 backend computes on CUDA only (there is no CPU "
                       "fallback); pass CUDA tensors, or pinned CPU tensors to stream them through the GPU")


def _default_group_heads(H: int) -> int:
    """Heads per streamed group: about eight groups, at least four heads per
    group when H allows it (smaller groups leave SMs idle at the tail)."""
    cap = max(4, H // 8)
    return max(d for d in range(1, H + 1) if H % d == 0 and d <= cap)


def _prepare(q, k, v, t_seq_len, alpha_2, SPARSITY_RATIO, select_ratio, flat_ratio, debug_keys=False):
    for name, x in (("q", q), ("k", k), ("v", v)):
        if not isinstance(x, torch.Tensor) or x.dim() != 4:
            raise ValueError(f"{name} must be a 4-D [B, S, H, D] tensor")
        _is_host(x)
        if x.dtype not in _DT:
            raise ValueError(f"{name} has dtype {x.dtype}; supported: bfloat16, float32")
    if q.shape != k.shape or q.shape[:3] != v.shape[:3] or v.shape[3] != q.shape[3]:
        raise ValueError(f"q, k, v shapes differ: {tuple(q.shape)}, {tuple(k.shape)}, {tuple(v.shape)}")
    if not (q.device == k.device == v.device):
        raise ValueError("q, k, v must be on one device")
    B, S, H, D = q.shape
    outc_dt, ca_dt, out_dt = _result_dtypes(q.dtype, k.dtype, v.dtype, alpha_2)
    if out_dt not in _DT:
        raise ValueError(f"unsupported output dtype {out_dt}")

    p = _capi.problem(B, S, H, D, int(t_seq_len), float(SPARSITY_RATIO), float(select_ratio), float(flat_ratio))
    p.q_dtype, p.k_dtype, p.v_dtype = _DT[q.dtype], _DT[k.dtype], _DT[v.dtype]
    p.out_dtype = _DT[out_dt]
    p.outc_bf16 = int(outc_dt == torch.bfloat16)
    p.ca_bf16 = int(ca_dt == torch.bfloat16)
    p.debug_keys = int(debug_keys)
    alpha_t = None
    if isinstance(alpha_2, torch.Tensor):
        a = alpha_2
        if a.dtype not in _DT:
            a = a.float()
        dev = q.device if q.is_cuda else torch.device("cuda", torch.cuda.current_device())
        if a.device != dev:
            a = a.to(dev)
        a = a.expand(B, S, H, D) if a.dim() <= 4 else None
        if a is None:
            raise ValueError("alpha_2 must broadcast to [B, S, H, D]")
        p.alpha_mode = _capi.ICSA_ALPHA_TENSOR
        p.alpha_dtype = _DT[a.dtype]
        for i in range(4):
            p.alpha_strides[i] = a.stride(i) if a.shape[i] > 1 else 0
        alpha_t = a
    elif isinstance(alpha_2, numbers.Number):
        p.alpha_mode = _capi.ICSA_ALPHA_SCALAR
        p.alpha_scalar = float(alpha_2)
    else:
        raise ValueError("alpha_2 must be a number or a tensor")
    return p, out_dt, alpha_t


def _streamed(lib, p, q, k, v, alpha_t, out_dt, out, group_heads, non_blocking):
    """Pinned host q, k, v -> pinned host result through icsa_forward_host."""
    B, S, H, D = q.shape
    hg = group_heads or _default_group_heads(H)
    if out is None:
        out = torch.empty(B, S, H, D, dtype=out_dt, pin_memory=True)
    elif (not isinstance(out, torch.Tensor) or out.shape != q.shape or out.dtype != out_dt or out.is_cuda
          or not out.is_pinned() or not out.is_contiguous()):
        raise ValueError(f"out must be a contiguous pinned CPU tensor of shape {tuple(q.shape)} and dtype {out_dt}")
    dev = torch.device("cuda", torch.cuda.current_device())
    with torch.cuda.device(dev):
        size = lib.icsa_host_workspace_size(ctypes.byref(p), hg)
        if size == 0:
            _capi.check(1, "icsa_host_workspace_size")
        ws = torch.empty(size, dtype=torch.uint8, device=dev)
        stream = torch.cuda.current_stream(dev)
        rc = lib.icsa_forward_host(ctypes.byref(p), hg, q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                   alpha_t.data_ptr() if alpha_t is not None else None, out.data_ptr(),
                                   ws.data_ptr(), size, stream.cuda_stream)
        _capi.check(rc, "icsa_forward_host")
        ws.record_stream(stream)
        if not non_blocking:
            _check_status(lib, ws.data_ptr(), stream.cuda_stream, "editing_sparse_attention (pinned host)")
    return out


def editing_sparse_attention(q, k, v, t_seq_len, s_seq_len=None, alpha_2=1.0, alpha_3=1.0, SPARSITY_RATIO=0.0625,
                             backend=Backend.B200, *, select_ratio=0.125, flat_ratio=0.5, out=None,
                             group_heads=None, non_blocking=False, check=None, _debug=None):
    """In-context sparse attention (see the module docstring).  Returns x
    [B, S, H, D].  `out`, `group_heads` and `non_blocking` apply to pinned
    CPU inputs only; `check` (default: ICSA_CHECK_STATUS) to CUDA inputs.
    `_debug`, when a dict, receives the workspace and its layout (used by the
    parity tests to read selections and keys)."""
    Backend.validate(backend)
    lib = _capi.load()
    p, out_dt, alpha_t = _prepare(q, k, v, t_seq_len, alpha_2, SPARSITY_RATIO, select_ratio, flat_ratio,
                                  debug_keys=_debug is not None)
    hosts = {_is_host(x) for x in (q, k, v)}
    if len(hosts) != 1:
        raise ValueError("q, k, v must all be CUDA tensors or all pinned CPU tensors")
    if hosts.pop():
        if _debug is not None:
            raise ValueError("_debug is only available for CUDA inputs")
        return _streamed(lib, p, q.contiguous(), k.contiguous(), v.contiguous(), alpha_t, out_dt, out, group_heads,
                         non_blocking)
    if out is not None:
        raise ValueError("out= is only supported for pinned CPU inputs")
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    B, S, H, D = q.shape
    with torch.cuda.device(q.device):
        size = lib.icsa_workspace_size(ctypes.byref(p))
        if size == 0:
            _capi.check(1, "icsa_workspace_size")
        ws = torch.empty(size, dtype=torch.uint8, device=q.device)
        out = torch.empty(B, S, H, D, dtype=out_dt, device=q.device)
        stream = torch.cuda.current_stream(q.device).cuda_stream
        rc = lib.icsa_forward(ctypes.byref(p), q.data_ptr(), k.data_ptr(), v.data_ptr(),
                              alpha_t.data_ptr() if alpha_t is not None else None, out.data_ptr(),
                              ws.data_ptr(), size, stream)
        _capi.check(rc, "icsa_forward")
        if (_CHECK_DEFAULT if check is None else check) and not torch.cuda.is_current_stream_capturing():
            _check_status(lib, ws.data_ptr(), stream, "editing_sparse_attention")
    if _debug is not None:
        _debug.update(workspace=ws, layout=_capi.workspace_layout(p), problem=p, inputs=(q, k, v))
    return out


# Backward-compatible alias of the reference (:235-236).
editing_sparse_attention_tilelang = editing_sparse_attention
