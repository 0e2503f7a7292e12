"""CPU oracle for the in-context sparse attention call.

TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the
cpu_baseline / --impl reference legs of bench.py may import this module; the
product path (libicsa.so and the in_context_sparse_attention package) never
does and has no CPU fallback.

A restatement, in torch on the CPU, of what the reference computes:

* orchestration: in_context_sparse_attention/editing_sparse_attention.py:67-232
  (pooling :107-111 + compress_seq :37-55, compressed attention torch_attention
  :58-64 / :113-123, in-context top-K :125-136, extended KV :138-159,
  sharpness split :161-172, gathers :174-184, scatter + residual :217-232);
* the sparse backend (tilelang default): tilelang_host.py:121-206 (block sums,
  host top-k, fused kernel) and the fused kernel
  tilelang_kernels.py:681-997 -- exact online softmax over the top_k indexed
  blocks with bf16 P, then the interval term in chunks of BN = 64 pooled
  blocks whose g_acc / g_l are never rescaled;
* the dense part, flash_attn_func (:211-215), a third-party library
  (flash-attn, requirements.txt:4 "flash-attn>=2.7.0"): exact softmax
  attention with the default 1/sqrt(D) scale, computed here in fp64.

Selections follow the contract of this build: every top-k / sort is a total
order on (value descending, index ascending), evaluated on fp32 keys.

Pins (see tests/golden/make_golden.py):
* the orchestration is pinned against the reference's own
  editing_sparse_attention run on the CPU (fp32) with the
  two GPU-only calls replaced by the restatements below;
* the sparse restatement is pinned against the reference's own Triton kernel
  (triton_kernels.py:122-263, BN = 64) run by the Triton interpreter on the CPU
  in fp32.  For 64-aligned extended KV (every configuration benchmarked) the
  Triton and TileLang kernels compute the same function.
* flash_attn_func is not runnable here; parity of the dense part is
  "unpinned" beyond exact-softmax semantics and is checked with a tolerance.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

BLOCK = 64
LOG2E = 1.44269504  # the constant used by tilelang_kernels.py:708


# ---------------------------------------------------------------------------
# counts (editing_sparse_attention.py:90,126-129,139,164,170; tilelang_host.py:151-171)
# ---------------------------------------------------------------------------
@dataclass
class Counts:
    B: int
    S: int
    H: int
    D: int
    t_seq_len: int
    NB: int = 0
    n_t: int = 0
    n_s: int = 0
    topK: int = 0
    num_flat: int = 0
    n_sparse: int = 0
    k_sparsity: int = 0
    tkv: int = 0
    nkv: int = 0
    top_k: int = 0

    @staticmethod
    def make(B, S, H, D, t_seq_len, sparsity=0.0625, select_ratio=0.125, flat_ratio=0.5) -> "Counts":
        c = Counts(B, S, H, D, t_seq_len)
        c.NB = (S + BLOCK - 1) // BLOCK
        c.n_t = t_seq_len // BLOCK
        c.n_s = c.NB - c.n_t
        c.topK = int(c.n_s * select_ratio)
        c.num_flat = int(c.NB * flat_ratio)
        c.n_sparse = c.NB - c.num_flat
        c.k_sparsity = max(1, int(c.n_t * sparsity))
        c.tkv = t_seq_len + c.topK * BLOCK
        c.nkv = (c.tkv + BLOCK - 1) // BLOCK
        c.top_k = max(1, int(sparsity * c.nkv))
        return c


# ---------------------------------------------------------------------------
# selection primitive
# ---------------------------------------------------------------------------
def select_desc(keys: torch.Tensor, k: int) -> torch.Tensor:
    """Indices of the k largest entries of each row of `keys` (last dim),
    ordered by value descending with ties broken towards the lower index."""
    keys = keys.float() + 0.0  # fold -0.0 onto +0.0
    order = torch.sort(-keys, dim=-1, stable=True).indices
    return order[..., :k]


# ---------------------------------------------------------------------------
# stage 1: pooling (editing_sparse_attention.py:37-55,107-111; tilelang_kernels.py:33-120)
# ---------------------------------------------------------------------------
def block_means(x: torch.Tensor) -> torch.Tensor:
    """[B,S,H,D] -> [B,NB,H,D] block means in x.dtype arithmetic (the reference's
    compress_seq; the last block may be partial)."""
    B, S, H, D = x.shape
    NB = (S + BLOCK - 1) // BLOCK
    sizes = torch.full((NB,), BLOCK, dtype=torch.int32)
    sizes[-1] = S - (NB - 1) * BLOCK
    pad = NB * BLOCK - S
    xp = torch.nn.functional.pad(x, (0, 0, 0, 0, 0, pad)) if pad else x
    s = xp.view(B, NB, BLOCK, H, D).float().sum(dim=2).to(x.dtype)
    return (s / sizes.view(1, -1, 1, 1)).to(x.dtype)


def block_sums_bf16(x: torch.Tensor) -> torch.Tensor:
    """[B,T,H,D] (T % 64 == 0 after zero padding) -> [B,H,T/64,D] bf16 sums of the
    bf16-cast rows with fp32 accumulation (reduce_q_kernel / reduce_kv_kernel)."""
    B, T, H, D = x.shape
    pad = (-T) % BLOCK
    xb = x.to(torch.bfloat16).float()
    if pad:
        xb = torch.nn.functional.pad(xb, (0, 0, 0, 0, 0, pad))
    n = xb.shape[1] // BLOCK
    return xb.view(B, n, BLOCK, H, D).sum(dim=2).to(torch.bfloat16).permute(0, 2, 1, 3).contiguous()


# ---------------------------------------------------------------------------
# stage 2: compressed attention and keys (editing_sparse_attention.py:58-64,113-172)
# ---------------------------------------------------------------------------
def compressed_attention(qm, km, vm):
    """qm/km/vm [B,H,NB,D] (any float dtype) -> scores, P (fp32), out_c (fp32).
    scores = q.k / sqrt(D) (QK /= sqrt(D)), P = softmax over all NB columns."""
    D = qm.shape[-1]
    s = torch.matmul(qm.float(), km.float().transpose(-1, -2)) / float(math.sqrt(D))
    P = torch.softmax(s, dim=-1)
    out_c = torch.matmul(P, vm.float())
    return s, P, out_c


def incontext_keys(P: torch.Tensor, n_t: int) -> torch.Tensor:
    """Column sums of P over target query rows, source columns: [B,H,n_s]."""
    return P[:, :, :n_t, n_t:].sum(dim=-2)


def sharpness_keys(P: torch.Tensor, n_t: int, k_sparsity: int) -> torch.Tensor:
    """Sum of the k_sparsity largest P[row, :n_t] per row: [B,H,NB]."""
    sub = P[..., :n_t]
    if n_t == 0:
        return torch.zeros(P.shape[:-1])
    top = torch.sort(sub, dim=-1, descending=True).values[..., :k_sparsity]
    return top.sum(dim=-1)


# ---------------------------------------------------------------------------
# extended KV (editing_sparse_attention.py:138-159)
# ---------------------------------------------------------------------------
def extended_kv(x: torch.Tensor, t_seq_len: int, sel: torch.Tensor) -> torch.Tensor:
    """x [B,S,H,D], sel [B,H,topK] -> [B,H,tkv,D]: target rows then the selected
    source blocks gathered from the zero-padded x at offset (t // 64) * 64."""
    B, S, H, D = x.shape
    NB = (S + BLOCK - 1) // BLOCK
    xp = torch.nn.functional.pad(x, (0, 0, 0, 0, 0, NB * BLOCK - S))
    topK = sel.shape[-1]
    rows = (sel[..., None] * BLOCK + torch.arange(BLOCK) + (t_seq_len // BLOCK) * BLOCK).reshape(B, H, topK * BLOCK)
    out = torch.empty(B, H, t_seq_len + topK * BLOCK, D, dtype=x.dtype)
    out[:, :, :t_seq_len] = x[:, :t_seq_len].permute(0, 2, 1, 3)
    for b in range(B):
        for h in range(H):
            out[b, h, t_seq_len:] = xp[b, rows[b, h], h]
    return out


# ---------------------------------------------------------------------------
# the sparse kernel: tilelang_kernels.py:681-997 (BN = 64)
# ---------------------------------------------------------------------------
def sparse_kernel(q, k, v, kc, vc, idx, nkv_real: int, round_p_bf16: bool = True):
    """One (b,h): q [NQ,64,D], k/v [NKV*64, D] (extended KV, zero padded to a
    multiple of 64), kc/vc [NKV, D] block sums, idx [NQ, top_k] -> out [NQ,64,D] fp32.

    Follows the fused kernel step by step: exact online softmax over idx (in
    list order) with P rounded to bf16 for the P.V product; then, per chunk of
    64 pooled blocks, scores q.kc/64 with the selected and >= nkv_real blocks
    masked, a running-max update that rescales acc/l, and g_acc/g_l that are
    accumulated relative to the running max of their chunk and never rescaled.
    """
    NQ, BT, D = q.shape
    scale = (1.0 / D) ** 0.5 * LOG2E
    qf = q.float()
    kf = k.float().view(-1, BT, D)
    vf = v.float().view(-1, BT, D)
    cast = (lambda t: t.to(torch.bfloat16).float()) if round_p_bf16 else (lambda t: t)
    m = torch.full((NQ, BT), -math.inf)
    l = torch.zeros(NQ, BT)
    acc = torch.zeros(NQ, BT, D)
    ar = torch.arange(NQ)
    for i in range(idx.shape[1]):
        blk = idx[:, i].long()
        s = torch.einsum("qrd,qcd->qrc", qf, kf[blk])
        m_new = torch.maximum(m, s.max(dim=-1).values)
        alpha = torch.exp2(m * scale - m_new * scale)
        p = torch.exp2(s * scale - m_new[..., None] * scale)
        l = l * alpha + p.sum(-1)
        acc = acc * alpha[..., None] + torch.einsum("qrc,qcd->qrd", cast(p), vf[blk])
        m = m_new
    nkv_pad = ((kc.shape[0] + 63) // 64) * 64
    kcp = torch.nn.functional.pad(kc.float(), (0, 0, 0, nkv_pad - kc.shape[0]))
    vcp = torch.nn.functional.pad(vc.float(), (0, 0, 0, nkv_pad - vc.shape[0]))
    selected = torch.zeros(NQ, nkv_pad, dtype=torch.bool)
    selected[ar[:, None], idx.long()] = True
    g_acc = torch.zeros(NQ, BT, D)
    g_l = torch.zeros(NQ, BT)
    for c0 in range(0, nkv_pad, 64):
        s = torch.einsum("qrd,cd->qrc", qf, kcp[c0:c0 + 64]) / BT
        blk = torch.arange(c0, c0 + 64)
        invalid = (blk >= nkv_real)[None, :] | selected[:, c0:c0 + 64]
        s = torch.where(invalid[:, None, :], torch.tensor(-math.inf), s)
        m_new = torch.maximum(m, s.max(dim=-1).values)
        sc = torch.exp2(m * scale - m_new * scale)
        acc = acc * sc[..., None]
        l = l * sc
        m = m_new
        p = torch.exp2(s * scale - m[..., None] * scale)
        g_l = g_l + p.sum(-1) * BT
        g_acc = g_acc + torch.einsum("qrc,cd->qrd", cast(p), vcp[c0:c0 + 64])
    l = l + g_l
    acc = acc + g_acc
    out = torch.where(l[..., None] == 0, torch.zeros(()), acc / l[..., None])
    return out


def sparse_backend(q_sharp, new_k, new_v, sparsity, forced_idx=None, return_keys=False):
    """sparse_piecewise_attn_1st_intervals_tilelang (tilelang_host.py:229-274)
    restated: q_sharp [B,H,TQ,D], new_k/new_v [B,H,TKV,D] (TKV % 64 == 0) ->
    [B,H,TQ,D] (bf16 values in fp32).  forced_idx [B,H,NQ,top_k] replaces the
    host top-k (used to evaluate with a selection computed elsewhere)."""
    B, H, TQ, D = q_sharp.shape
    TKV = new_k.shape[2]
    NQ, NKV = TQ // BLOCK, TKV // BLOCK
    top_k = max(1, int(sparsity * NKV))
    qc = block_sums_bf16(q_sharp.permute(0, 2, 1, 3))      # [B,H,NQ,D]
    kc = block_sums_bf16(new_k.permute(0, 2, 1, 3))
    vc = block_sums_bf16(new_v.permute(0, 2, 1, 3))
    scores = torch.matmul(qc.float(), kc.float().transpose(-1, -2))  # fp32 keys
    idx = select_desc(scores, top_k) if forced_idx is None else forced_idx
    out = torch.empty(B, H, TQ, D)
    for b in range(B):
        for h in range(H):
            o = sparse_kernel(q_sharp[b, h].to(torch.bfloat16).view(NQ, BLOCK, D),
                              new_k[b, h].to(torch.bfloat16), new_v[b, h].to(torch.bfloat16),
                              kc[b, h], vc[b, h], idx[b, h], NKV)
            out[b, h] = o.reshape(TQ, D)
    out = out.to(torch.bfloat16).float()
    if return_keys:
        return out, scores, idx
    return out


def dense_attention(q, k, v, dtype=torch.float64, chunk=1024):
    """flash_attn_func(q, k, v) restated: [B,T,H,D] bf16 -> exact softmax
    attention in `dtype` arithmetic (fp64 for parity checks), returned as bf16
    values in fp32.  Queries are taken `chunk` at a time, so the score matrix
    held at once is chunk x Tkv per (b, h) whatever the sequence length."""
    B, T, H, D = q.shape
    out = torch.empty(B, H, T, D, dtype=torch.float32)
    for b in range(B):
        for h in range(H):
            qd, kd, vd = (t[b, :, h].to(dtype).contiguous() for t in (q, k, v))
            kt = kd.t().contiguous()
            for i in range(0, T, chunk):
                s = torch.matmul(qd[i:i + chunk], kt) / math.sqrt(D)
                out[b, h, i:i + chunk] = torch.matmul(torch.softmax(s, dim=-1), vd).to(torch.bfloat16).float()
    return out.permute(0, 2, 1, 3)


# ---------------------------------------------------------------------------
# the whole call
# ---------------------------------------------------------------------------
@dataclass
class OracleResult:
    out: torch.Tensor
    counts: Counts
    sel: torch.Tensor = None          # [B,H,topK]
    order: torch.Tensor = None        # [B,H,NB]
    colsum: torch.Tensor = None
    sharp: torch.Tensor = None
    out_c: torch.Tensor = None        # [B,H,NB,D] fp32
    blockscore: torch.Tensor = None   # [B,H,n_sparse,nkv]
    sparse_idx: torch.Tensor = None   # [B,H,n_sparse,top_k]
    extra: dict = field(default_factory=dict)


def result_dtypes(q_dtype, k_dtype, v_dtype, alpha):
    """dtypes of out_compress, of out_compress*alpha and of the output, by the
    reference's torch type promotion (mixed q/k vs v means CUDA autocast)."""
    outc = torch.bfloat16 if torch.bfloat16 in (q_dtype, k_dtype, v_dtype) else torch.float32
    if isinstance(alpha, torch.Tensor):
        ca = torch.promote_types(outc, alpha.dtype)
    else:
        ca = outc
    out = torch.promote_types(q_dtype, ca)
    return outc, ca, out


def editing_sparse_attention(q, k, v, t_seq_len, alpha_2=1.0, sparsity=0.0625, select_ratio=0.125,
                             flat_ratio=0.5, forced=None, means=None, dense_dtype=torch.float64) -> OracleResult:
    """The whole call on the CPU.  forced: optional dict with 'sel', 'order',
    'sparse_idx' from another implementation; when given, those selections are
    used instead of the oracle's own (so outputs can be compared without
    near-tie selection differences).  means: optional (qm, km) [B, NB, H, D]
    block means of the float32 q and k that the given bf16 q and k were
    rounded from (a sequence-parallel caller pools before it exchanges the
    bf16 tensors); they replace the means of q and k.  dense_dtype: the
    arithmetic of the dense (flash_attn_func) part; fp64 for parity checks,
    fp32 (flash-attn's accumulation type) when the call is timed.  Memory is
    bounded at any sequence length: the dense part takes its queries in
    chunks, and every other stage holds at most [NB, NB] or [n_sparse, 64,
    64] scores per (b, h)."""
    B, S, H, D = q.shape
    c = Counts.make(B, S, H, D, t_seq_len, sparsity, select_ratio, flat_ratio)
    outc_dt, ca_dt, out_dt = result_dtypes(q.dtype, k.dtype, v.dtype, alpha_2)

    qm, km, vm = block_means(q), block_means(k), block_means(v)
    if means is not None:
        qm, km = means
    cast = (lambda t: t.to(torch.bfloat16)) if outc_dt == torch.bfloat16 else (lambda t: t)
    s, P, out_c = compressed_attention(*(cast(t).permute(0, 2, 1, 3) for t in (qm, km, vm)))
    colsum = incontext_keys(P, c.n_t)
    sharp = sharpness_keys(P, c.n_t, c.k_sparsity)
    sel = select_desc(colsum, c.topK) if forced is None else forced["sel"]
    order = select_desc(sharp, c.NB) if forced is None else forced["order"]
    flat_blocks = order[..., :c.num_flat]
    sparse_blocks = order[..., c.num_flat:]

    new_k = extended_kv(k, t_seq_len, sel)
    new_v = extended_kv(v, t_seq_len, sel)
    tkv_pad = c.nkv * BLOCK
    pad = tkv_pad - c.tkv
    new_k_sp = torch.nn.functional.pad(new_k, (0, 0, 0, pad)) if pad else new_k
    new_v_sp = torch.nn.functional.pad(new_v, (0, 0, 0, pad)) if pad else new_v

    NBp = c.NB * BLOCK
    qp = torch.nn.functional.pad(q, (0, 0, 0, 0, 0, NBp - S)).permute(0, 2, 1, 3).reshape(B, H, c.NB, BLOCK, D)

    def gather(blocks):
        return torch.stack([torch.stack([qp[b, h, blocks[b, h]] for h in range(H)]) for b in range(B)])

    out_blocks = torch.zeros(B, H, c.NB, BLOCK, D)
    blockscore = sparse_idx = None
    if c.n_sparse > 0:
        qs = gather(sparse_blocks).reshape(B, H, c.n_sparse * BLOCK, D)
        o_s, blockscore, sparse_idx = sparse_backend(
            qs.to(torch.bfloat16), new_k_sp, new_v_sp, sparsity,
            forced_idx=None if forced is None else forced["sparse_idx"], return_keys=True)
        o_s = o_s.view(B, H, c.n_sparse, BLOCK, D)
        for b in range(B):
            for h in range(H):
                out_blocks[b, h, sparse_blocks[b, h]] = o_s[b, h]
    if c.num_flat > 0:
        qf = gather(flat_blocks).reshape(B, H, c.num_flat * BLOCK, D)
        o_f = dense_attention(qf.permute(0, 2, 1, 3).to(torch.bfloat16), new_k.permute(0, 2, 1, 3).to(torch.bfloat16),
                              new_v.permute(0, 2, 1, 3).to(torch.bfloat16), dtype=dense_dtype)
        o_f = o_f.permute(0, 2, 1, 3).reshape(B, H, c.num_flat, BLOCK, D)
        for b in range(B):
            for h in range(H):
                out_blocks[b, h, flat_blocks[b, h]] = o_f[b, h]

    x = out_blocks.view(B, H, NBp, D).permute(0, 2, 1, 3)[:, :S].to(q.dtype)
    oc = out_c.to(outc_dt).permute(0, 2, 1, 3).repeat_interleave(BLOCK, dim=1)[:, :S]
    x = x + oc * alpha_2
    return OracleResult(out=x.to(out_dt), counts=c, sel=sel, order=order, colsum=colsum, sharp=sharp, out_c=out_c,
                        blockscore=blockscore, sparse_idx=sparse_idx)
