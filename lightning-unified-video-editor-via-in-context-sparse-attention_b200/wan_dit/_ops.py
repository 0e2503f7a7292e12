"""Operations of one Wan 2.2 DiT block, as the model in this package calls them.

`CudaOps` is the implementation: the fused elementwise passes and the
in-context sparse attention and the cross-attention over the text tokens
(the reference's flash_attention call, wanx/attention.py:18-85) run in
libicsa.so (include/icsa_dit.h, include/icsa.h); the projections are library
GEMMs (torch.nn.functional.linear, i.e. cuBLAS, bf16 in / bf16 out with f32
accumulation, which is what the reference's nn.Linear computes under CUDA
autocast).
Constructing it loads libicsa.so and raises if it is missing: there is no CPU
fallback.

Every method takes and returns torch tensors on the current CUDA device and
runs on the current stream.
"""
from __future__ import annotations

import ctypes

import torch
import torch.nn.functional as F

from in_context_sparse_attention import _capi

DIT_EXPORTED = ("icsa_dit_modulated_norm", "icsa_dit_norm_rope", "icsa_dit_norm_rope_pool",
                "icsa_dit_gated_residual", "icsa_dit_cross_attention", "icsa_dit_linear_residual")

_DT = {torch.bfloat16: _capi.ICSA_BF16, torch.float32: _capi.ICSA_F32}


class NormRopeDesc(ctypes.Structure):
    """Mirror of struct icsa_dit_norm_rope_desc."""
    _fields_ = [
        ("rows", ctypes.c_int), ("C", ctypes.c_int), ("D", ctypes.c_int),
        ("ld", ctypes.c_int64),
        ("rows_per_batch", ctypes.c_int), ("token_offset", ctypes.c_int),
        ("eps", ctypes.c_float),
        ("count", ctypes.c_int),
        ("src", ctypes.c_void_p * 3), ("norm_weight", ctypes.c_void_p * 3), ("rope", ctypes.c_int * 3),
        ("dst", ctypes.c_void_p * 3), ("dst_dtype", ctypes.c_int * 3),
        ("heads_per_group", ctypes.c_int),
        ("dst_batch_stride", ctypes.c_int64), ("dst_group_stride", ctypes.c_int64),
        ("dst_token_stride", ctypes.c_int64),
        ("rope_table", ctypes.c_void_p), ("rope_positions", ctypes.c_int),
        ("token_pos", ctypes.c_void_p), ("token_count", ctypes.c_int),
        ("rope_split1", ctypes.c_int), ("rope_split2", ctypes.c_int),
        ("gate_src", ctypes.c_void_p), ("gate_dst", ctypes.c_void_p),
    ]


class NormRopePoolDesc(ctypes.Structure):
    """Mirror of struct icsa_dit_norm_rope_pool_desc."""
    _fields_ = [
        ("base", NormRopeDesc),
        ("mean", ctypes.c_void_p * 3),
        ("mean_batch_stride", ctypes.c_int64), ("mean_group_stride", ctypes.c_int64),
        ("round_mean_bf16", ctypes.c_int),
        ("rs_scratch", ctypes.c_void_p),
        ("sum", ctypes.c_void_p * 3),
        ("bf16_mean", ctypes.c_int * 3),
    ]


def _load():
    lib = _capi.load()
    for name in DIT_EXPORTED:
        if not hasattr(lib, name):
            raise ImportError(f"{_capi.LIB_PATH} does not export {name}; rebuild it with `python build.py`")
    vp, i, i64, f = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float
    lib.icsa_dit_modulated_norm.argtypes = [vp, i, i64, i, i, i, vp, i64, vp, i64, f, i, vp, vp]
    lib.icsa_dit_modulated_norm.restype = i
    lib.icsa_dit_norm_rope.argtypes = [ctypes.POINTER(NormRopeDesc), vp]
    lib.icsa_dit_norm_rope.restype = i
    lib.icsa_dit_norm_rope_pool.argtypes = [ctypes.POINTER(NormRopePoolDesc), vp]
    lib.icsa_dit_norm_rope_pool.restype = i
    lib.icsa_dit_gated_residual.argtypes = [vp, vp, i64, i, i, i, vp, i64, vp]
    lib.icsa_dit_gated_residual.restype = i
    lib.icsa_dit_cross_attention.argtypes = [vp, i64, vp, i64, vp, i64, vp, i, i, i, i, i, vp]
    lib.icsa_dit_cross_attention.restype = i
    lib.icsa_dit_linear_residual.argtypes = [vp, i64, vp, i64, vp, vp, i64, i, i, i, i, vp, i64, vp]
    lib.icsa_dit_linear_residual.restype = i
    return lib


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _rows(x: torch.Tensor):
    """(rows, leading dimension) of a 2-D row-major view."""
    if x.dim() != 2 or x.stride(1) != 1:
        raise ValueError(f"expected a 2-D row-major view, got shape {tuple(x.shape)} strides {x.stride()}")
    return x.shape[0], x.stride(0)


class CudaOps:
    """The B200 implementation of the block's operations."""

    def __init__(self):
        self.lib = _load()

    # --- library GEMMs and activations -----------------------------------
    @staticmethod
    def linear(x, w, b=None):
        return F.linear(x, w, b)

    @staticmethod
    def gelu_tanh(x):
        return F.gelu(x, approximate="tanh")

    # --- fused elementwise passes ----------------------------------------
    def modulated_norm(self, x, scale, shift, rows_per_batch, eps, round_norm=False):
        """bf16 [rows, C] = LayerNorm(x) * scale[b] + shift[b] (include/icsa_dit.h).
        scale / shift: f32 [B, C] or [C] (shared by all rows)."""
        rows, ld = _rows(x)
        C = x.shape[1]
        nb = -(-rows // rows_per_batch)
        for t in (scale, shift):
            if t.dtype != torch.float32 or t.shape[-1] != C or t.stride(-1) != 1 or (t.dim() == 2 and t.shape[0] < nb):
                raise ValueError(f"modulated_norm: scale/shift must be f32 [{nb}, {C}] or [{C}]")
        out = torch.empty(rows, C, dtype=torch.bfloat16, device=x.device)
        sbs = scale.stride(0) if scale.dim() == 2 else 0
        hbs = shift.stride(0) if shift.dim() == 2 else 0
        _capi.check(self.lib.icsa_dit_modulated_norm(
            x.data_ptr(), _DT[x.dtype], ld, rows, C, rows_per_batch, scale.data_ptr(), sbs, shift.data_ptr(), hbs,
            float(eps), int(bool(round_norm)), out.data_ptr(), _stream()), "icsa_dit_modulated_norm")
        return out

    def norm_rope(self, jobs, rows_per_batch, eps, token_offset=0, table=None, token_pos=None, splits=(0, 0),
                  gate=None):
        """jobs: up to three (src [rows, C] bf16 view, norm weight or None,
        rope flag, out [B, G, s, hp, D] contiguous).  gate: optional
        (src [rows] bf16 column view, out bf16 [rows])."""
        d = self._norm_rope_desc(jobs, rows_per_batch, eps, token_offset, table, token_pos, splits, gate)
        _capi.check(self.lib.icsa_dit_norm_rope(ctypes.byref(d), _stream()), "icsa_dit_norm_rope")

    def norm_rope_pool(self, jobs, means, rows_per_batch, eps, token_offset=0, table=None, token_pos=None,
                       splits=(0, 0), gate=None, round_mean=True, sums=None, bf16_mean=(False, False, False)):
        """norm_rope with bf16 outputs and, for each job whose entry of
        `means` is a tensor, the f32 means of its 64-token blocks, laid out
        [B, G, hp, s/64, D] (include/icsa_dit.h, icsa_dit_norm_rope_pool).
        sums: optional bf16 tensors of the same shape for the block sums of
        the bf16 outputs; bf16_mean[j]: mean j in the bf16 arithmetic of a
        bf16 vector (the attention's pooling of v)."""
        base = self._norm_rope_desc(jobs, rows_per_batch, eps, token_offset, table, token_pos, splits, gate)
        B, G, s, hp, D = jobs[0][3].shape
        if s % 64:
            raise ValueError(f"norm_rope_pool: {s} tokens per batch element are not whole 64-token blocks")
        d = NormRopePoolDesc()
        d.base = base
        shape = (B, G, hp, s // 64, D)
        ref = None
        for j, m in enumerate(means):
            if m is None:
                continue
            if m.shape != shape or m.dtype != torch.float32 or not m.is_contiguous():
                raise ValueError(f"norm_rope_pool: mean {j} must be contiguous f32 {shape}")
            d.mean[j] = m.data_ptr()
            d.bf16_mean[j] = int(bool(bf16_mean[j]))
            ref = m
        for j, m in enumerate(sums or ()):
            if m is None:
                continue
            if m.shape != shape or m.dtype != torch.bfloat16 or not m.is_contiguous():
                raise ValueError(f"norm_rope_pool: sum {j} must be contiguous bf16 {shape}")
            d.sum[j] = m.data_ptr()
            ref = m if ref is None else ref
        if ref is not None:
            d.mean_batch_stride, d.mean_group_stride = ref.stride(0), ref.stride(1)
        d.round_mean_bf16 = int(bool(round_mean))
        rs = torch.empty(len(jobs) * B * s, dtype=torch.float32, device=jobs[0][0].device)
        d.rs_scratch = rs.data_ptr()
        _capi.check(self.lib.icsa_dit_norm_rope_pool(ctypes.byref(d), _stream()), "icsa_dit_norm_rope_pool")

    @staticmethod
    def _norm_rope_desc(jobs, rows_per_batch, eps, token_offset, table, token_pos, splits, gate):
        d = NormRopeDesc()
        src0 = jobs[0][0]
        rows, ld = _rows(src0)
        out0 = jobs[0][3]
        B, G, s, hp, D = out0.shape
        if s != rows_per_batch or rows != B * s or G * hp * D != src0.shape[1]:
            raise ValueError(f"norm_rope: output layout {tuple(out0.shape)} does not hold {rows} rows of "
                             f"{src0.shape[1]} values in batches of {rows_per_batch}")
        if table is not None and (token_pos.shape[1] != 4 or token_pos.dtype != torch.int32
                                  or token_offset + s > token_pos.shape[0] or not token_pos.is_contiguous()):
            raise ValueError("norm_rope: token_pos must be contiguous int32 [tokens, 4] covering this shard")
        if table is not None and (table.dtype != torch.float64 or table.shape[1:] != (D // 2, 2)
                                  or not table.is_contiguous()):
            raise ValueError(f"norm_rope: the rotary table must be contiguous f64 [positions, {D // 2}, 2]")
        if gate is not None and (gate[1].numel() < rows or gate[1].dtype != torch.bfloat16):
            raise ValueError(f"norm_rope: the gate output must be bf16 with {rows} entries")
        d.rows, d.C, d.D, d.ld = rows, src0.shape[1], D, ld
        d.rows_per_batch, d.token_offset, d.eps, d.count = rows_per_batch, token_offset, float(eps), len(jobs)
        for j, (src, w, rope, out) in enumerate(jobs):
            if _rows(src) != (rows, ld) or out.shape != out0.shape or not out.is_contiguous():
                raise ValueError("norm_rope: all vectors must share rows, leading dimension and output layout")
            d.src[j] = src.data_ptr()
            d.norm_weight[j] = w.data_ptr() if w is not None else None
            d.rope[j] = int(bool(rope))
            d.dst[j] = out.data_ptr()
            d.dst_dtype[j] = _DT[out.dtype]
        d.heads_per_group = hp
        d.dst_batch_stride, d.dst_group_stride, d.dst_token_stride = out0.stride(0), out0.stride(1), out0.stride(2)
        if table is not None:
            d.rope_table, d.rope_positions = table.data_ptr(), table.shape[0]
            d.token_pos, d.token_count = token_pos.data_ptr(), token_pos.shape[0]
            d.rope_split1, d.rope_split2 = splits
        if gate is not None:
            gsrc, gout = gate
            if gsrc.stride(0) != ld:
                raise ValueError("norm_rope: the gate column must share the rows' leading dimension")
            d.gate_src, d.gate_dst = gsrc.data_ptr(), gout.data_ptr()
        return d

    def gated_residual_(self, x, y, gate, rows_per_batch):
        """x (f32 [rows, C], in place) += y (bf16 [rows, C] view) * gate[b] (f32 [B, C] or None)."""
        if x.dtype != torch.float32 or not x.is_contiguous():
            raise ValueError("gated_residual_: x must be a contiguous f32 tensor")
        rows, ldy = _rows(y)
        C = x.shape[-1]
        if x.shape != (rows, y.shape[1]):
            raise ValueError(f"gated_residual_: x {tuple(x.shape)} and y {tuple(y.shape)} differ")
        if gate is not None and (gate.dtype != torch.float32 or gate.shape[-1] != C or gate.stride(-1) != 1
                                 or gate.shape[0] < -(-rows // rows_per_batch)):
            raise ValueError("gated_residual_: gate must be f32 [batches, C]")
        gp, gbs = (gate.data_ptr(), gate.stride(0)) if gate is not None else (None, 0)
        _capi.check(self.lib.icsa_dit_gated_residual(x.data_ptr(), y.data_ptr(), ldy, rows, C, rows_per_batch, gp, gbs,
                                                     _stream()), "icsa_dit_gated_residual")
        return x

    def linear_residual_(self, x, a, w, b, gate, rows_per_batch):
        """x (f32 [rows, N], in place) += bf16(a @ w^T + b) * gate[row // rows_per_batch]
        (gate None: + bf16(...)): the output projection and its residual
        update in one tcgen05 GEMM whose epilogue reads and writes x
        (icsa_dit_linear_residual); a: bf16 [rows, K] row-major view,
        w: bf16 [N, K] (nn.Linear weight), b: bf16 [N] or None."""
        rows, lda = _rows(a)
        N, K = w.shape
        if x.dtype != torch.float32 or not x.is_contiguous() or x.shape != (rows, N):
            raise ValueError(f"linear_residual_: x must be contiguous f32 [{rows}, {N}]")
        if a.dtype != torch.bfloat16 or w.dtype != torch.bfloat16 or a.shape[1] != K or w.stride(1) != 1:
            raise ValueError("linear_residual_: a and w must be bf16 with matching K")
        if b is not None and (b.dtype != torch.bfloat16 or b.shape != (N,) or not b.is_contiguous()):
            raise ValueError(f"linear_residual_: bias must be bf16 [{N}]")
        if gate is not None and (gate.dtype != torch.float32 or gate.shape[-1] != N or gate.stride(-1) != 1
                                 or gate.shape[0] < -(-rows // rows_per_batch)):
            raise ValueError("linear_residual_: gate must be f32 [batches, N]")
        gp, gbs = (gate.data_ptr(), gate.stride(0)) if gate is not None else (None, 0)
        _capi.check(self.lib.icsa_dit_linear_residual(
            a.data_ptr(), lda, w.data_ptr(), w.stride(0), b.data_ptr() if b is not None else None, x.data_ptr(),
            x.stride(0), rows, N, K, rows_per_batch, gp, gbs, _stream()), "icsa_dit_linear_residual")
        return x

    # --- attention ---------------------------------------------------------
    def self_attention(self, q, k, v, alpha, t_seq_len, means=None):
        """In-context sparse attention of the reference's WanSelfAttention
        (model.py:172-173) for q, k f32 and v bf16 [B, S, h, D] and the bf16
        gate alpha [B, S], returned as the bf16 operand of the output
        projection (the reference's f32 result rounded once to bf16, which is
        what its autocast o-projection reads).

        means: optional (qmean, kmean) f32 [B, h, NB, D], the block means of
        the f32 q and k that were rounded to the bf16 q and k passed here
        (icsa_dit_norm_rope_pool computes them before the exchange).  The
        pool stage then runs on the bf16 tensors, its q / k means are
        replaced by these, and the result is bit for bit the one of the f32
        call.  With six arrays, (qmean, kmean, vmean, qsum, ksum, vsum)
        (f32 means, bf16 sums, all [B, h, NB, D]), the pool stage does not
        run at all: these are every block statistic it would produce."""
        if means is not None:
            return self._self_attention_premeaned(q, k, v, alpha, t_seq_len, means)
        B, S, H, D = q.shape
        p = self._problem(q, k, v, alpha, t_seq_len, _DT[q.dtype], _DT[k.dtype])
        lib = self.lib
        size = lib.icsa_workspace_size(ctypes.byref(p))
        if size == 0:
            _capi.check(1, "icsa_workspace_size")
        ws = torch.empty(size, dtype=torch.uint8, device=q.device)
        out = torch.empty(B, S, H, D, dtype=torch.bfloat16, device=q.device)
        _capi.check(lib.icsa_forward(ctypes.byref(p), q.data_ptr(), k.data_ptr(), v.data_ptr(), alpha.data_ptr(),
                                     out.data_ptr(), ws.data_ptr(), size, _stream()), "icsa_forward")
        return out

    def _problem(self, q, k, v, alpha, t_seq_len, q_dtype, k_dtype):
        B, S, H, D = q.shape
        p = _capi.problem(B, S, H, D, int(t_seq_len))
        p.q_dtype, p.k_dtype, p.v_dtype = q_dtype, k_dtype, _DT[v.dtype]
        p.out_dtype = _capi.ICSA_BF16
        p.outc_bf16, p.ca_bf16 = 1, 1
        p.alpha_mode, p.alpha_dtype = _capi.ICSA_ALPHA_TENSOR, _DT[alpha.dtype]
        for i, st in enumerate((alpha.stride(0), alpha.stride(1), 0, 0)):
            p.alpha_strides[i] = st
        return p

    def _self_attention_premeaned(self, q, k, v, alpha, t_seq_len, means):
        B, S, H, D = q.shape
        if q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16:
            raise ValueError("self_attention with means: q and k must be the bf16 tensors")
        p = self._problem(q, k, v, alpha, t_seq_len, _capi.ICSA_BF16, _capi.ICSA_BF16)
        L = _capi.workspace_layout(p)
        NB = p.num_blocks
        if len(means) not in (2, 6) or any(m.shape != (B, H, NB, D) for m in means):
            raise ValueError(f"self_attention means must be 2 or 6 arrays [{B}, {H}, {NB}, {D}]")
        lib, st = self.lib, _stream()
        size = L.total
        ws = torch.empty(size, dtype=torch.uint8, device=q.device)
        out = torch.empty(B, S, H, D, dtype=torch.bfloat16, device=q.device)
        pp = ctypes.byref(p)
        a = (q.data_ptr(), k.data_ptr(), v.data_ptr())
        n = B * H * NB * D
        regions = [(L.qmean, torch.float32), (L.kmean, torch.float32)]
        if len(means) == 6:
            # every block statistic of the pool stage is given: it does not run
            regions += [(L.vmean, torch.float32), (L.qsum, torch.bfloat16), (L.ksum, torch.bfloat16),
                        (L.vsum, torch.bfloat16)]
        else:
            _capi.check(lib.icsa_pool(pp, *a, ws.data_ptr(), size, st), "icsa_pool")
        for (off, dt), m in zip(regions, means):
            if m.dtype != dt:
                raise ValueError(f"self_attention: block statistic of dtype {m.dtype}, expected {dt}")
            ws[off:off + n * m.element_size()].view(dt).copy_(m.reshape(-1))
        _capi.check(lib.icsa_select(pp, a[1], a[2], ws.data_ptr(), size, st), "icsa_select")
        _capi.check(lib.icsa_attend(pp, *a, alpha.data_ptr(), out.data_ptr(), ws.data_ptr(), size, st),
                    "icsa_attend")
        return out

    def cross_attention(self, q, k, v):
        """Softmax attention of bf16 q [B, L, H, D] over k, v [B, Lk, H, D]
        with the default 1/sqrt(D) scale; bf16 [B, L, H, D].  This library's
        tcgen05 dense attention kernel (icsa_dit_cross_attention); each of
        q, k, v may have any token stride (rows of a wider GEMM output) as
        long as its heads and features are contiguous."""
        B, L, H, D = q.shape
        Lk = k.shape[1]
        args = []
        for name, t, n in (("q", q, L), ("k", k, Lk), ("v", v, Lk)):
            if t.dtype != torch.bfloat16 or t.shape != (B, n, H, D):
                raise ValueError(f"cross_attention: {name} must be bf16 [{B}, {n}, {H}, {D}]")
            if t.stride(3) != 1 or t.stride(2) != D or t.stride(0) != n * t.stride(1):
                t = t.contiguous()
            args += [t.data_ptr(), t.stride(1)]
        out = torch.empty(B, L, H, D, dtype=torch.bfloat16, device=q.device)
        _capi.check(self.lib.icsa_dit_cross_attention(*args, out.data_ptr(), B, L, Lk, H, D, _stream()),
                    "icsa_dit_cross_attention")
        return out
