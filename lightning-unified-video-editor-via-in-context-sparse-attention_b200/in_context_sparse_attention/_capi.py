"""ctypes binding of libicsa.so (declared in include/icsa.h).

Loading is explicit and loud: if the shared library is missing or does not
export the expected symbols, an ImportError/OSError is raised.  There is no
CPU or pure-PyTorch fallback anywhere in this package.
"""
from __future__ import annotations

import ctypes
import os
import threading

_PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.environ.get("ICSA_LIB", os.path.join(_PKG_DIR, "libicsa.so"))

ICSA_BF16, ICSA_F32 = 0, 1
ICSA_ALPHA_SCALAR, ICSA_ALPHA_TENSOR = 0, 1
STATUS = {0: "ICSA_OK", 1: "ICSA_ERR_INVALID", 2: "ICSA_ERR_UNSUPPORTED", 3: "ICSA_ERR_CUDA",
          4: "ICSA_ERR_WORKSPACE", 5: "ICSA_ERR_DEVICE_TIMEOUT"}

EXPORTED = ("icsa_last_error", "icsa_version", "icsa_problem_init", "icsa_workspace_size",
            "icsa_get_workspace_layout", "icsa_forward", "icsa_pool", "icsa_select", "icsa_attend",
            "icsa_attend_dense", "icsa_attend_sparse", "icsa_host_workspace_size", "icsa_forward_host", "icsa_wait_selftest",
            "icsa_device_status", "icsa_last_status", "icsa_forward_static", "icsa_static_scratch_bytes",
            "icsa_static_device_status")


class Problem(ctypes.Structure):
    """Mirror of struct icsa_problem."""
    _fields_ = [
        ("B", ctypes.c_int), ("S", ctypes.c_int), ("H", ctypes.c_int), ("D", ctypes.c_int),
        ("t_seq_len", ctypes.c_int),
        ("num_blocks", ctypes.c_int), ("n_t", ctypes.c_int), ("n_s", ctypes.c_int), ("topK", ctypes.c_int),
        ("num_flat", ctypes.c_int), ("k_sparsity", ctypes.c_int), ("tkv", ctypes.c_int), ("nkv", ctypes.c_int),
        ("top_k", ctypes.c_int),
        ("q_dtype", ctypes.c_int), ("k_dtype", ctypes.c_int), ("v_dtype", ctypes.c_int), ("out_dtype", ctypes.c_int),
        ("outc_bf16", ctypes.c_int),
        ("alpha_mode", ctypes.c_int), ("alpha_dtype", ctypes.c_int), ("alpha_scalar", ctypes.c_float),
        ("alpha_strides", ctypes.c_int64 * 4),
        ("ca_bf16", ctypes.c_int),
        ("debug_keys", ctypes.c_int),
    ]


class WorkspaceLayout(ctypes.Structure):
    """Mirror of struct icsa_workspace_layout."""
    _fields_ = [(n, ctypes.c_size_t) for n in (
        "total", "err", "qsum", "ksum", "vsum", "qmean", "kmean", "vmean", "scores", "rowmax", "rowsum", "sharp",
        "colsum", "outc", "sel", "order", "kv_rows", "kc", "vc", "sparse_idx", "sel_mask", "blockscore",
        "qbf", "kbf", "vbf", "newk", "newv")] + [("nkv_pad", ctypes.c_int), ("n_sparse", ctypes.c_int)]


class IcsaError(RuntimeError):
    def __init__(self, code: int, where: str, msg: str):
        super().__init__(f"{where}: {STATUS.get(code, code)}: {msg}")
        self.code = code


_lib = None
_lock = threading.Lock()


def load(path: str = None) -> ctypes.CDLL:
    """Load libicsa.so once and declare the signatures."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        p = path or LIB_PATH
        if not os.path.exists(p):
            raise ImportError(f"libicsa.so not found at {p}; build it with `python build.py` "
                              "(there is no CPU fallback)")
        lib = ctypes.CDLL(p)
        for name in EXPORTED:
            if not hasattr(lib, name):
                raise ImportError(f"{p} does not export {name}")
        vp, sz, i = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int
        pp = ctypes.POINTER(Problem)
        lib.icsa_last_error.restype = ctypes.c_char_p
        lib.icsa_version.restype = ctypes.c_char_p
        lib.icsa_problem_init.argtypes = [pp, i, i, i, i, i, ctypes.c_double, ctypes.c_double, ctypes.c_double]
        lib.icsa_problem_init.restype = i
        lib.icsa_workspace_size.argtypes = [pp]
        lib.icsa_workspace_size.restype = sz
        lib.icsa_get_workspace_layout.argtypes = [pp, ctypes.POINTER(WorkspaceLayout)]
        lib.icsa_get_workspace_layout.restype = i
        lib.icsa_forward.argtypes = [pp, vp, vp, vp, vp, vp, vp, sz, vp]
        lib.icsa_forward.restype = i
        lib.icsa_pool.argtypes = [pp, vp, vp, vp, vp, sz, vp]
        lib.icsa_pool.restype = i
        lib.icsa_select.argtypes = [pp, vp, vp, vp, sz, vp]
        lib.icsa_select.restype = i
        lib.icsa_attend.argtypes = [pp, vp, vp, vp, vp, vp, vp, sz, vp]
        lib.icsa_attend.restype = i
        for name in ("icsa_attend_dense", "icsa_attend_sparse"):
            getattr(lib, name).argtypes = [pp, vp, vp, vp, vp, vp, vp, sz, vp]
            getattr(lib, name).restype = i
        lib.icsa_host_workspace_size.argtypes = [pp, i]
        lib.icsa_host_workspace_size.restype = sz
        lib.icsa_forward_host.argtypes = [pp, i, vp, vp, vp, vp, vp, vp, sz, vp]
        lib.icsa_forward_host.restype = i
        lib.icsa_wait_selftest.argtypes = [vp, vp]
        lib.icsa_wait_selftest.restype = i
        lib.icsa_device_status.argtypes = [vp, vp]
        lib.icsa_device_status.restype = i
        lib.icsa_last_status.argtypes = [vp, i]
        lib.icsa_last_status.restype = i
        lib.icsa_forward_static.argtypes = [pp, vp, vp, vp, vp, vp, vp]
        lib.icsa_forward_static.restype = i
        lib.icsa_static_scratch_bytes.argtypes = []
        lib.icsa_static_scratch_bytes.restype = sz
        lib.icsa_static_device_status.argtypes = [vp]
        lib.icsa_static_device_status.restype = i
        _lib = lib
        return lib


def check(code: int, where: str):
    if code != 0:
        raise IcsaError(code, where, load().icsa_last_error().decode(errors="replace"))


def problem(B, S, H, D, t_seq_len, sparsity=0.0625, select_ratio=0.125, flat_ratio=0.5) -> Problem:
    p = Problem()
    check(load().icsa_problem_init(ctypes.byref(p), B, S, H, D, t_seq_len, sparsity, select_ratio, flat_ratio),
          "icsa_problem_init")
    return p


def workspace_layout(p: Problem) -> WorkspaceLayout:
    L = WorkspaceLayout()
    check(load().icsa_get_workspace_layout(ctypes.byref(p), ctypes.byref(L)), "icsa_get_workspace_layout")
    return L
