"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run in a container where the reference is importable (its source tree path is
given by --reference).  Writes tests/golden/*.pt.  The GPU box never runs
this script; tests only read the fixtures it produced.

1. config1_reference.pt -- BASELINE configuration 1 (B=1, H=2, D=64, fp32,
   t = s = 4096) run through the reference's own `editing_sparse_attention`
   (in_context_sparse_attention/editing_sparse_attention.py:67-232) on the CPU.
   Its two GPU-only calls are replaced by the oracle's restatements
   (oracle.icsa_oracle.sparse_backend for the tilelang host,
   oracle.icsa_oracle.dense_attention for flash_attn_func); every other line
   is the reference's.  The selections it makes (torch.topk / torch.argsort
   calls) and its output are recorded.
2. triton_interval_pin.pt -- the reference's own Triton sparse kernel
   (triton_kernels.py:122-263) run by the Triton interpreter on the CPU in
   fp32 with BN = 64, on seeded inputs, next to the indices it was given.
   This pins the oracle's restatement of the exact + interval term.

Inputs are regenerated from seeds by the tests; checksums recorded here guard
against a change of the random generator.
"""
import argparse
import importlib
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
sys.path.insert(0, os.path.join(REPO, "lightning-unified-video-editor-via-in-context-sparse-attention_b200"))

from oracle import icsa_oracle as orc  # noqa: E402
from in_context_sparse_attention import synthetic  # noqa: E402


def import_reference(ref_root, module):
    """Import `module` from the reference tree under its own package name,
    shadowing this repository's package of the same name."""
    for name in list(sys.modules):
        if name == "in_context_sparse_attention" or name.startswith("in_context_sparse_attention."):
            del sys.modules[name]
    sys.path[:] = [ref_root] + [p for p in sys.path if not p.endswith("_b200") and p != ref_root]
    return importlib.import_module(module)


def checksum(t):
    t = t.double()
    return [float(t.sum()), float(t.abs().sum()), float((t * t).sum())]


class TorchProxy:
    """Stands in for the `torch` module inside the reference module and
    records the selection calls it makes."""

    def __init__(self, log):
        self._log = log

    def __getattr__(self, name):
        return getattr(torch, name)

    def topk(self, x, k, *a, **kw):
        r = torch.topk(x, k, *a, **kw)
        self._log.append(("topk", x.detach().clone(), r.indices.clone()))
        return r

    def argsort(self, x, *a, **kw):
        r = torch.argsort(x, *a, **kw)
        self._log.append(("argsort", x.detach().clone(), r.clone()))
        return r


def run_reference_config1(ref_root):
    import_reference(ref_root, "in_context_sparse_attention")
    esa = sys.modules["in_context_sparse_attention.editing_sparse_attention"]
    log = []
    esa.torch = TorchProxy(log)

    def sparse_cpu(q, k, v, sparsity=0.1, block_size=64):
        # tilelang_host.py:229-274 asserts, then the restated pipeline
        assert q.dtype == k.dtype == v.dtype == torch.bfloat16 and block_size == 64
        return orc.sparse_backend(q, k, v, sparsity)

    def flash_cpu(q, k, v):
        return orc.dense_attention(q, k, v)

    esa.sparse_piecewise_attn_1st_intervals_tilelang = sparse_cpu
    esa.flash_attn_func = flash_cpu
    w = synthetic.CONFIG1
    q, k, v = synthetic.make_inputs(w)
    torch.set_num_threads(os.cpu_count())
    x = esa.editing_sparse_attention(q, k, v, w.t_seq_len, w.t_seq_len, alpha_2=1.0, SPARSITY_RATIO=0.0625,
                                     backend="tilelang")
    return w, (q, k, v), x, log


def make_config1(ref_root):
    w, (q, k, v), x, log = run_reference_config1(ref_root)
    topk_calls = [e for e in log if e[0] == "topk"]
    argsort_calls = [e for e in log if e[0] == "argsort"]
    c = orc.Counts.make(w.B, w.S, w.H, w.D, w.t_seq_len)
    colsum_ref, topk_idx = topk_calls[0][1], topk_calls[0][2]
    sharp_ref, order_ref = argsort_calls[0][1], argsort_calls[0][2]
    sel_ref = topk_idx[..., :c.topK]
    # the oracle's own, independent orchestration of the same inputs
    o = orc.editing_sparse_attention(q, k, v, w.t_seq_len)
    diff = (o.out.double() - x.double()).abs()
    print(f"config1: reference vs oracle max|d|={float(diff.max()):.3e} mean|d|={float(diff.mean()):.3e}")
    print("config1: sel equal:", bool(torch.equal(o.sel, sel_ref)),
          " split equal:", bool(torch.equal(o.order[..., :c.num_flat].sort(-1).values,
                                             order_ref[..., :c.num_flat].sort(-1).values)))
    NB = c.NB
    blocksum = x.double().view(w.B, NB, 64, w.H, w.D).sum(2)
    fx = {
        "workload": w.name, "counts": vars(c),
        "input_checksums": [checksum(t) for t in (q, k, v)],
        "sel": sel_ref.clone(), "order": order_ref.clone(),
        "colsum": colsum_ref.float().clone(), "sharp": sharp_ref.float().clone(),
        "out_rows": x[:, ::13].clone(), "out_blocksum": blocksum.clone(),
        "out_checksum": checksum(x),
        "oracle_vs_reference_maxdiff": float(diff.max()),
    }
    torch.save(fx, os.path.join(HERE, "config1_reference.pt"))


def make_triton_pin(ref_root):
    os.environ["TRITON_INTERPRET"] = "1"
    tk = import_reference(ref_root, "in_context_sparse_attention.triton_kernels")
    g = torch.Generator().manual_seed(1234)
    B, H, TQ, TKV, D, sparsity = 1, 1, 256, 640, 64, 0.3
    q = torch.randn(B, H, TQ, D, generator=g)
    k = torch.randn(B, H, TKV, D, generator=g)
    v = torch.randn(B, H, TKV, D, generator=g)
    NQ, NKV = TQ // 64, TKV // 64
    # block sums kept in fp32: the interpreter mishandles bf16 buffers
    qc = torch.empty(B, H, NQ, D)
    kc = torch.empty(B, H, NKV, D)
    vc = torch.empty(B, H, NKV, D)
    kvc = torch.empty(B, H, NKV, D, D)
    tk.chunk_reduce_q_kernel.fn[(1, NQ, B * H)](q, qc, TQ, NQ, D, 64, D)
    tk.chunk_reduce_kv_kernel.fn[(1, NKV, B * H)](k, v, kc, vc, kvc, TKV, NKV, D, D, 64, D, D)
    top_k = max(1, int(sparsity * NKV))
    p = torch.einsum("bhik,bhjk->bhij", qc, kc)
    idx = torch.topk(p, k=top_k, dim=-1).indices.to(torch.int32)
    o = torch.empty(B, H, TQ, D)
    lse = torch.empty(B, H, TQ)
    tk.sparse_piecewise_attn_1st_intervals_kernel.fn[(1, NQ, B * H)](
        q, k, v, kc, vc, kvc, o, lse, idx, D ** -0.5, TQ, TKV, D, D, 64, D, D, NQ, NKV, top_k, BN=64)
    mine = orc.sparse_kernel(q[0, 0].view(NQ, 64, D), k[0, 0], v[0, 0], kc[0, 0], vc[0, 0], idx[0, 0], NKV,
                             round_p_bf16=False)
    d = float((mine.reshape(TQ, D) - o[0, 0]).abs().max())
    print(f"triton pin: oracle vs reference Triton kernel max|d|={d:.3e}")
    torch.save({"seed": 1234, "shape": (B, H, TQ, TKV, D), "sparsity": sparsity,
                "input_checksums": [checksum(t) for t in (q, k, v)], "idx": idx.clone(),
                "kc": kc.clone(), "vc": vc.clone(), "out": o.clone(), "oracle_maxdiff": d},
               os.path.join(HERE, "triton_interval_pin.pt"))


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("ICSA_REFERENCE"), required="ICSA_REFERENCE" not in os.environ,
                    help="source tree of the reference (the directory holding in_context_sparse_attention/)")
    a = ap.parse_args()
    make_triton_pin(a.reference)
    make_config1(a.reference)
