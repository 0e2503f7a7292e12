"""B200 (sm_100a) implementation of LIVEditor's in-context sparse attention.

Same package name and exports as the reference package
(in_context_sparse_attention/__init__.py:1-11), plus the `'b200'` backend
name.  Put the directory containing this package on sys.path (or install
it) and the Wan 2.2 DiT's call site `editing_sparse_attention(q, k, v,
t_seq_len, s_seq_len, alpha_2=..., backend=...)` runs unchanged.
"""
from ._capi import IcsaError
from .editing_sparse_attention import (
    Backend,
    device_status,  # not in the reference: reports device-side timeouts (see its docstring)
    editing_sparse_attention,
    editing_sparse_attention_tilelang,  # backward-compatible alias
)

__all__ = [
    "Backend",
    "IcsaError",
    "device_status",
    "editing_sparse_attention",
    "editing_sparse_attention_tilelang",
]
