"""Shared helpers of the parity tests: run the C-ABI path with its workspace
kept, read named workspace regions, and compare with the CPU oracle."""
import json
import os

import torch

from in_context_sparse_attention import editing_sparse_attention
from oracle import icsa_oracle as orc


def region(dbg, name, dtype, shape):
    """View of a named workspace region (see icsa_workspace_layout)."""
    ws, L = dbg["workspace"], dbg["layout"]
    off = getattr(L, name)
    n = 1
    for s in shape:
        n *= s
    nbytes = n * torch.empty((), dtype=dtype).element_size()
    return ws[off:off + nbytes].view(dtype).view(*shape)


def run_gpu(q, k, v, t_seq_len, alpha=1.0, sparsity=0.0625, select_ratio=0.125, flat_ratio=0.5):
    dbg = {}
    out = editing_sparse_attention(q, k, v, t_seq_len, q.shape[1] - t_seq_len, alpha_2=alpha,
                                   SPARSITY_RATIO=sparsity, select_ratio=select_ratio, flat_ratio=flat_ratio,
                                   _debug=dbg)
    torch.cuda.synchronize()
    return out, dbg


def gpu_selections(dbg):
    """Selections and keys the GPU made, on the CPU, shaped like the oracle's."""
    p, L = dbg["problem"], dbg["layout"]
    B, H, NB = p.B, p.H, p.num_blocks
    n_sp = L.n_sparse
    sel = region(dbg, "sel", torch.int32, (B, H, p.topK)).long().cpu() if p.topK > 0 else torch.zeros(B, H, 0).long()
    order = region(dbg, "order", torch.int32, (B, H, NB)).long().cpu()
    sparse_idx = (region(dbg, "sparse_idx", torch.int32, (B, H, n_sp, p.top_k)).long().cpu()
                  if n_sp > 0 else torch.zeros(B, H, 0, p.top_k).long())
    colsum = region(dbg, "colsum", torch.float32, (B, H, p.n_s)).cpu() if p.n_s > 0 else None
    sharp = region(dbg, "sharp", torch.float32, (B, H, NB)).cpu()
    blockscore = region(dbg, "blockscore", torch.float32, (B, H, n_sp, p.nkv)).cpu() if n_sp > 0 else None
    outc = region(dbg, "outc", torch.float32, (B, H, NB, p.D)).cpu()
    return dict(sel=sel, order=order, sparse_idx=sparse_idx, colsum=colsum, sharp=sharp, blockscore=blockscore,
                outc=outc)


def record(name, **fields):
    """Appends one JSON line of measured errors to the file named by the
    ICSA_PARITY_LOG environment variable (pytest -q hides prints)."""
    path = os.environ.get("ICSA_PARITY_LOG")
    if path:
        with open(path, "a") as f:
            f.write(json.dumps({"case": name, **fields}) + "\n")


def oracle_forced(q, k, v, t_seq_len, sels, alpha=1.0, **kw):
    """Oracle output with the GPU's selections forced."""
    a = alpha.cpu() if isinstance(alpha, torch.Tensor) else alpha
    forced = dict(sel=sels["sel"], order=sels["order"], sparse_idx=sels["sparse_idx"])
    return orc.editing_sparse_attention(q.cpu(), k.cpu(), v.cpu(), t_seq_len, alpha_2=a, forced=forced, **kw)


def errors(a, b):
    d = (a.double().cpu() - b.double().cpu()).abs()
    return float(d.max()), float(d.mean())


def bf16_ulp(x):
    """Spacing of bf16 numbers at |x| (8 significant bits): 2^(e - 7) for
    2^e <= |x| < 2^(e+1)."""
    e = torch.floor(torch.log2(x.double().abs().clamp_min(2.0 ** -126)))
    return torch.exp2(e - 7)


def excess_over_bf16_bound(out, ref, max_abs):
    """Largest amount by which |out - ref| exceeds max(max_abs, two bf16 units
    of ref), and the reference value there.  Both sides are rounded to bf16
    twice, as the reference rounds them: the attention output, then
    x = attention + out_compress * alpha_2.  Where the two fp32 accumulations
    straddle a rounding boundary, each rounding can move the result by one
    unit, so two units of |x| is the smallest element-wise bound; it exceeds
    2e-2 only for |x| >= 2 (one unit is 2^-6 there)."""
    o, r = out.double().cpu(), ref.double().cpu()
    d = (o - r).abs()
    ex = d - torch.clamp(2 * bf16_ulp(r), min=max_abs)
    i = int(torch.argmax(ex))
    return float(ex.flatten()[i]), float(r.flatten()[i]), float(d.flatten()[i])
