"""A Wan 2.2 A14B-shaped DiT for one LIVEditor denoising step on B200s.

This is the model around the in-context sparse attention call: the
reference's WanModel (model.py:308-464) with its WanAttentionBlock
(model.py:225-269), restated as explicit tensor code so that each stage runs
as one of the fused passes of `_ops.CudaOps`, and so that the self-attention
can be run with Ulysses sequence parallelism:

* the residual stream is sequence-sharded: rank r holds tokens
  [r*s, (r+1)*s) of both CFG branches (s = S / world), in f32 (the
  reference's residual stream is f32 from the first `x + y * e[2]` on);
* q, k, v leave the fused RMSNorm + RoPE pass already in the layout of the
  all-to-all's send buffer, [B, world, s, H/world, D]; one NCCL
  all_to_all_single per tensor and batch element turns them into
  [B, S, H/world, D], the head shard the attention needs; the per-token gate
  alpha_1 is all-gathered; the bf16 attention output goes back the same way;
* cross-attention and the FFN are local to the sequence shard.

With one rank the exchanges vanish and the step is the plain model.

CFG runs as a batch of two (unconditional, conditional) sharing the latent,
which is what the reference's two model calls per step compute
(inference.py:266-281).  Weights are random (N(0, 0.02) for the projections,
the reference's own initialisation for modulation tables and norms); nothing
is loaded from a checkpoint.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import rope as rope_mod


@dataclass
class WanDiTConfig:
    """Shape of the DiT; defaults are the Wan 2.2 A14B expert of the
    reference's inference.yaml (configs/inference.yaml:14-24)."""
    dim: int = 5120
    ffn_dim: int = 13824
    num_heads: int = 40
    num_layers: int = 40
    freq_dim: int = 256
    text_dim: int = 4096
    text_len: int = 512
    in_dim: int = 16
    out_dim: int = 16
    patch_size: tuple = (1, 2, 2)
    eps: float = 1e-6
    init_std: float = 0.02

    @property
    def head_dim(self) -> int:
        return self.dim // self.num_heads


def sinusoidal_embedding_1d(dim: int, position: torch.Tensor) -> torch.Tensor:
    """[N, dim] f64: cos | sin of position * 10000**(-i/half) (model.py:24-30)."""
    half = dim // 2
    position = position.to(torch.float64)
    sinusoid = torch.outer(position, torch.pow(10000, -torch.arange(half, dtype=torch.float64,
                                                                      device=position.device).div(half)))
    return torch.cat([torch.cos(sinusoid), torch.sin(sinusoid)], dim=1)


class _Block:
    """Weights of one WanAttentionBlock (model.py:225-245).  The q, k, v and
    alpha_1 projections of the self-attention are stacked into one [3C + 8, C]
    GEMM (row 3C is alpha_1, rows 3C+1.. are zero padding that keeps the
    output rows 16-byte aligned)."""

    def __init__(self, cfg: WanDiTConfig, g: torch.Generator, device):
        C, Fd = cfg.dim, cfg.ffn_dim

        def w(o, i):
            return (torch.randn(o, i, generator=g, device=device) * cfg.init_std).to(torch.bfloat16)

        def zeros(n):
            return torch.zeros(n, dtype=torch.bfloat16, device=device)

        def ones(n):
            return torch.ones(n, dtype=torch.bfloat16, device=device)

        self.w_qkv = torch.cat([w(3 * C, C), w(1, C), torch.zeros(7, C, dtype=torch.bfloat16, device=device)])
        self.b_qkv = zeros(3 * C + 8)
        self.norm_q, self.norm_k = ones(C), ones(C)
        self.w_o, self.b_o = w(C, C), zeros(C)
        self.norm3_w = torch.ones(C, device=device)     # f32 copies of the affine LayerNorm
        self.norm3_b = torch.zeros(C, device=device)
        self.wc_q, self.bc_q = w(C, C), zeros(C)
        self.wc_kv, self.bc_kv = w(2 * C, C), zeros(2 * C)
        self.cnorm_q, self.cnorm_k = ones(C), ones(C)
        self.wc_o, self.bc_o = w(C, C), zeros(C)
        self.w1, self.b1 = w(Fd, C), zeros(Fd)
        self.w2, self.b2 = w(C, Fd), zeros(C)
        # modulation: randn / sqrt(dim) (model.py:246), kept in bf16 like the model's parameters
        self.modulation = (torch.randn(6, C, generator=g, device=device) / C ** 0.5).to(torch.bfloat16)


class WanDiT:
    """Random-init Wan 2.2 DiT whose self-attention is the in-context sparse
    attention of this package.

    ops:       the block operations (default: `_ops.CudaOps`, which needs
               libicsa.so and a CUDA device).
    group:     process group of the Ulysses ranks (default: the default group
               when torch.distributed is initialised, else a single rank).
    pipelined: with several ranks, overlap each batch element's exchanges
               with the other's computation (`_self_attention_pipelined`);
               False runs one exchange per tensor for the whole batch.
    pooled_exchange: in the pipelined exchanges, send q and k as bf16 with
               the f32 means of their 64-token blocks (pooled before the
               exchange) instead of as f32: a third less NVLink traffic, and
               the attention's result is bit for bit the same.
    """

    def __init__(self, cfg: WanDiTConfig = WanDiTConfig(), device=None, seed: int = 0, ops=None, group=None,
                 pipelined: bool = True, pooled_exchange: bool = True):
        if ops is None:
            from ._ops import CudaOps
            ops = CudaOps()
        self.ops = ops
        self.cfg = cfg
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.group = group
        self.pipelined = pipelined
        self.pooled_exchange = pooled_exchange
        self.dist = dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size(group) if self.dist else 1
        self.rank = dist.get_rank(group) if self.dist else 0
        if cfg.num_heads % self.world:
            raise ValueError(f"{cfg.num_heads} heads do not split over {self.world} ranks")
        C, D = cfg.dim, cfg.head_dim
        if D not in (64, 128):
            raise ValueError(f"head dim {D}: the attention supports 64 and 128")
        g = torch.Generator(device=self.device).manual_seed(seed)
        std = cfg.init_std

        def w(o, i):
            return (torch.randn(o, i, generator=g, device=self.device) * std).to(torch.bfloat16)

        def zeros(n):
            return torch.zeros(n, dtype=torch.bfloat16, device=self.device)

        p = math.prod(cfg.patch_size)
        # patch embeddings (Conv3d with kernel = stride = patch_size, model.py:356-358) as GEMMs
        self.w_patch, self.b_patch = w(C, cfg.in_dim * p), zeros(C)
        self.w_patch_src, self.b_patch_src = w(C, cfg.in_dim * p), zeros(C)
        self.w_text1, self.b_text1 = w(C, cfg.text_dim), zeros(C)
        self.w_text2, self.b_text2 = w(C, C), zeros(C)
        self.w_time1, self.b_time1 = w(C, cfg.freq_dim), zeros(C)
        self.w_time2, self.b_time2 = w(C, C), zeros(C)
        self.w_tproj, self.b_tproj = w(6 * C, C), zeros(6 * C)
        self.blocks = [_Block(cfg, g, self.device) for _ in range(cfg.num_layers)]
        self.w_head, self.b_head = w(cfg.out_dim * p, C), zeros(cfg.out_dim * p)
        self.head_modulation = (torch.randn(2, C, generator=g, device=self.device) / C ** 0.5).to(torch.bfloat16)
        self.rope_table = rope_mod.rope_table(D).to(self.device)
        self.rope_splits = rope_mod.head_dim_splits(D)
        self._pos_key = None
        self._time_f32 = None

    # ------------------------------------------------------------------
    # embeddings
    # ------------------------------------------------------------------
    def _patchify(self, latent: torch.Tensor):
        """[C_in, F, H, W] -> ([F*H/ph*W/pw, C_in*pf*ph*pw] bf16, grid), the
        patch vector in Conv3d weight order (channel, kt, kh, kw)."""
        pf, ph, pw = self.cfg.patch_size
        c, f, h, w = latent.shape
        x = latent.to(torch.bfloat16).view(c, f // pf, pf, h // ph, ph, w // pw, pw)
        x = x.permute(1, 3, 5, 0, 2, 4, 6).reshape((f // pf) * (h // ph) * (w // pw), c * pf * ph * pw)
        return x, (f // pf, h // ph, w // pw)

    def embed(self, latent, source_latent, seq_len: int):
        """Joint token sequence [target | source | zeros] (model.py:413-432) as
        bf16 [seq_len, C], with the grids and per-token RoPE positions."""
        xt, grid = self._patchify(latent)
        xs, sgrid = self._patchify(source_latent)
        t = self.ops.linear(xt, self.w_patch, self.b_patch)
        s = self.ops.linear(xs, self.w_patch_src, self.b_patch_src)
        n = t.shape[0] + s.shape[0]
        if n > seq_len:
            raise ValueError(f"{n} tokens exceed seq_len={seq_len}")
        pad = torch.zeros(seq_len - n, self.cfg.dim, dtype=t.dtype, device=t.device)
        key = (grid, sgrid, seq_len)
        if self._pos_key != key:
            self.token_pos = rope_mod.token_positions(grid, sgrid, seq_len).to(self.device)
            self._pos_key = key
        return torch.cat([t, s, pad]), grid, sgrid

    def time_embed(self, t: torch.Tensor):
        """e [N, C] and e0 [N, 6, C] in f32 (model.py:434-437)."""
        lin = torch.nn.functional.linear
        if self._time_f32 is None:   # f32 copies of the time MLP, made once (the reference runs it in f32)
            self._time_f32 = [w.float() for w in (self.w_time1, self.b_time1, self.w_time2, self.b_time2,
                                                  self.w_tproj, self.b_tproj)]
        w1, b1, w2, b2, wp, bp = self._time_f32
        x = sinusoidal_embedding_1d(self.cfg.freq_dim, t).float()
        e = lin(torch.nn.functional.silu(lin(x, w1, b1)), w2, b2)
        e0 = lin(torch.nn.functional.silu(e), wp, bp)
        return e, e0.unflatten(1, (6, self.cfg.dim))

    def text_embed(self, context: torch.Tensor):
        """[B, text_len, C] bf16: Linear, GELU(tanh), Linear (model.py:359-360, :439-440)."""
        B, L, _ = context.shape
        x = self.ops.linear(context.reshape(B * L, -1).to(torch.bfloat16), self.w_text1, self.b_text1)
        x = self.ops.linear(self.ops.gelu_tanh(x), self.w_text2, self.b_text2)
        return x.view(B, L, self.cfg.dim)

    # ------------------------------------------------------------------
    # Ulysses exchanges
    # ------------------------------------------------------------------
    def _exchange_in(self, q, k, v, gate):
        """[B, n, s, hp, D] per rank -> [B, S, hp, D]; gate [B*s] -> [B, S]."""
        B, n, s, hp, D = q.shape
        if n == 1:
            return q.view(B, s, hp, D), k.view(B, s, hp, D), v.view(B, s, hp, D), gate.view(B, s)
        outs = []
        for t in (q, k, v):
            r = torch.empty(B, n * s, hp, D, dtype=t.dtype, device=t.device)
            for b in range(B):
                dist.all_to_all_single(r[b], t[b], group=self.group)
            outs.append(r)
        g = torch.empty(n * B * s, dtype=gate.dtype, device=gate.device)
        dist.all_gather_into_tensor(g, gate, group=self.group)
        alpha = g.view(n, B, s).permute(1, 0, 2).reshape(B, n * s)
        return outs[0], outs[1], outs[2], alpha

    def _exchange_out(self, o):
        """[B, S, hp, D] per rank -> [B*s, H*D] (this rank's tokens, all heads)."""
        B, S, hp, D = o.shape
        n = self.world
        if n == 1:
            return o.view(B * S, hp * D)
        s = S // n
        r = torch.empty(B, n, s, hp, D, dtype=o.dtype, device=o.device)
        for b in range(B):
            dist.all_to_all_single(r[b], o[b], group=self.group)
        return r.permute(0, 2, 1, 3, 4).reshape(B * s, n * hp * D)

    # ------------------------------------------------------------------
    # one block
    # ------------------------------------------------------------------
    def block_forward(self, blk: _Block, x, e0, ctx, t_seq_len: int, first: bool = False):
        """WanAttentionBlock.forward (model.py:248-269) on this rank's tokens.
        x: f32 [B*s, C] (bf16 for the first block, whose LayerNorm output the
        reference rounds to the residual stream's bf16); returns the new f32
        residual stream."""
        cfg, ops = self.cfg, self.ops
        C, H, D = cfg.dim, cfg.num_heads, cfg.head_dim
        B = e0.shape[0]
        s = x.shape[0] // B
        n, hp = self.world, H // self.world
        e = self.e_block(blk, e0)

        # self-attention (model.py:255-259); the output projection and the
        # residual update x + y * e[2] are one GEMM with a fused epilogue
        xin = ops.modulated_norm(x, e["scale0"], e["shift0"], s, cfg.eps, round_norm=first)
        dev = x.device
        if x.dtype != torch.float32:
            x = x.float()
        if n > 1 and self.pipelined:
            self._self_attention_pipelined(blk, xin, B, s, t_seq_len, x, e["gate0"])
        elif n == 1 and self.pooled_exchange and s % 64 == 0:
            self._self_attention_local_pooled(blk, xin, B, s, t_seq_len, x, e["gate0"])
        else:
            qkv = ops.linear(xin, blk.w_qkv, blk.b_qkv)
            q, k, v, gate = self._qkv(blk, qkv, B, s)
            del xin, qkv
            qf, kf, vf, alpha = self._exchange_in(q, k, v, gate)
            del q, k, v
            o = ops.self_attention(qf, kf, vf, alpha, t_seq_len)
            del qf, kf, vf
            ops.linear_residual_(x, self._exchange_out(o), blk.w_o, blk.b_o, e["gate0"], s)
            del o

        # cross-attention (model.py:262, WanT2VCrossAttention :181-188)
        xn = ops.modulated_norm(x, blk.norm3_w, blk.norm3_b, s, cfg.eps)
        qc = ops.linear(xn, blk.wc_q, blk.bc_q)
        L = ctx.shape[1]
        kv = ops.linear(ctx.reshape(B * L, C), blk.wc_kv, blk.bc_kv)
        qn = torch.empty(B, 1, s, H, D, dtype=torch.bfloat16, device=dev)
        kn = torch.empty(B, 1, L, H, D, dtype=torch.bfloat16, device=dev)
        ops.norm_rope([(qc, blk.cnorm_q, False, qn)], rows_per_batch=s, eps=cfg.eps)
        ops.norm_rope([(kv[:, :C], blk.cnorm_k, False, kn)], rows_per_batch=L, eps=cfg.eps)
        oc = ops.cross_attention(qn.view(B, s, H, D), kn.view(B, L, H, D), kv[:, C:].view(B, L, H, D))
        ops.linear_residual_(x, oc.reshape(B * s, C), blk.wc_o, blk.bc_o, None, s)

        # FFN (model.py:263-265)
        xn = ops.modulated_norm(x, e["scale1"], e["shift1"], s, cfg.eps)
        h = ops.gelu_tanh(ops.linear(xn, blk.w1, blk.b1))
        ops.linear_residual_(x, h, blk.w2, blk.b2, e["gate1"], s)
        del h
        return x

    def _qkv(self, blk: _Block, qkv, B, s):
        """RMSNorm + RoPE of q and k, v passed through, all written into the
        all-to-all send layout [B, world, s, H/world, D], and the gate alpha_1
        (model.py:153-170), from the fused projection output qkv [B*s, 3C+8]."""
        cfg = self.cfg
        C, D, n = cfg.dim, cfg.head_dim, self.world
        hp = cfg.num_heads // n
        q = torch.empty(B, n, s, hp, D, dtype=torch.float32, device=qkv.device)
        k = torch.empty_like(q)
        v = torch.empty(B, n, s, hp, D, dtype=torch.bfloat16, device=qkv.device)
        gate = torch.empty(B * s, dtype=torch.bfloat16, device=qkv.device)
        self.ops.norm_rope([(qkv[:, :C], blk.norm_q, True, q), (qkv[:, C:2 * C], blk.norm_k, True, k),
                            (qkv[:, 2 * C:3 * C], None, False, v)], rows_per_batch=s, eps=cfg.eps,
                           token_offset=self.rank * s, table=self.rope_table, token_pos=self.token_pos,
                           splits=self.rope_splits, gate=(qkv[:, 3 * C], gate))
        return q, k, v, gate

    def _qkv_pooled(self, blk: _Block, qkv, s):
        """`_qkv` for one batch element with bf16 q, k, v and every block
        statistic of the attention's first stage (editing_sparse_attention.py:
        37-55, :107-111, and the block sums of tilelang_kernels.py:33-120),
        [1, world, H/world, s/64, D] each, computed before the exchange: the
        f32 means of the f32 q and k, the bf16-arithmetic mean of v, and the
        bf16 block sums of q, k and v.  The attention then skips its pooling
        pass over q, k and v."""
        cfg = self.cfg
        C, D, n = cfg.dim, cfg.head_dim, self.world
        hp = cfg.num_heads // n
        dev = qkv.device
        q = torch.empty(1, n, s, hp, D, dtype=torch.bfloat16, device=dev)
        k = torch.empty_like(q)
        v = torch.empty_like(q)
        means = [torch.empty(1, n, hp, s // 64, D, dtype=torch.float32, device=dev) for _ in range(3)]
        sums = [torch.empty(1, n, hp, s // 64, D, dtype=torch.bfloat16, device=dev) for _ in range(3)]
        gate = torch.empty(s, dtype=torch.bfloat16, device=dev)
        self.ops.norm_rope_pool([(qkv[:, :C], blk.norm_q, True, q), (qkv[:, C:2 * C], blk.norm_k, True, k),
                                 (qkv[:, 2 * C:3 * C], None, False, v)], means, rows_per_batch=s,
                                eps=cfg.eps, token_offset=self.rank * s, table=self.rope_table,
                                token_pos=self.token_pos, splits=self.rope_splits, gate=(qkv[:, 3 * C], gate),
                                sums=sums, bf16_mean=(False, False, True))
        return q, k, v, gate, means + sums

    def _self_attention_local_pooled(self, blk: _Block, xin, B, s, t_seq_len, x, res_gate):
        """Self-attention on one rank holding the whole sequence, per batch
        element: the producer pass writes bf16 q, k, v and every block
        statistic of the attention's pooling stage, so the attention reads
        bf16 operands and skips its pooling pass (the same bits as the f32
        q / k call, as in the sequence-parallel path)."""
        ops, cfg = self.ops, self.cfg
        C, H, D = cfg.dim, cfg.num_heads, cfg.head_dim
        for b in range(B):
            qkv = ops.linear(xin[b * s:(b + 1) * s], blk.w_qkv, blk.b_qkv)
            q, k, v, gate, stats = self._qkv_pooled(blk, qkv, s)
            del qkv
            # [1, 1, H, s/64, D] -> [1, H, s/64, D]
            means = tuple(m[:, 0] for m in stats)
            o = ops.self_attention(q.view(1, s, H, D), k.view(1, s, H, D), v.view(1, s, H, D), gate.view(1, s),
                                   t_seq_len, means=means)
            del q, k, v
            ops.linear_residual_(x[b * s:(b + 1) * s], o.view(s, C), blk.w_o, blk.b_o, res_gate[b:b + 1], s)

    def _self_attention_pipelined(self, blk: _Block, xin, B, s, t_seq_len, x, res_gate):
        """Ulysses self-attention with the exchanges of one batch element
        overlapping the computation of the other: NCCL runs the all-to-alls on
        its own stream, each launched as soon as its operand is written, and
        the compute stream waits for an exchange only right before its result
        is read:

            projection+RoPE b0 | projection+RoPE b1 | attention b0 | attention b1 | o-proj b0 | o-proj b1
                               | exchange-in b0     | exchange-in b1 | exchange-out b0 | exchange-out b1

        The o-projection of batch element b updates its rows of the residual
        stream x in place (x + o(y) * res_gate[b]).  Every rank issues the same
        collectives in the same order."""
        ops, g = self.ops, self.group
        cfg = self.cfg
        C, D, n = cfg.dim, cfg.head_dim, self.world
        hp = cfg.num_heads // n
        S = n * s
        dev = xin.device
        # pooled exchange: q and k cross as bf16 with the f32 means of their
        # 64-token blocks (whole blocks only), instead of as f32
        pooled = self.pooled_exchange and s % 64 == 0
        qdt = torch.bfloat16 if pooled else torch.float32
        inbound = []
        for b in range(B):
            qkv = ops.linear(xin[b * s:(b + 1) * s], blk.w_qkv, blk.b_qkv)
            if pooled:
                q, k, v, gate, stats = self._qkv_pooled(blk, qkv, s)
            else:
                q, k, v, gate = self._qkv(blk, qkv, 1, s)
            del qkv
            qf = torch.empty(1, S, hp, D, dtype=qdt, device=dev)
            kf = torch.empty_like(qf)
            vf = torch.empty(1, S, hp, D, dtype=torch.bfloat16, device=dev)
            alpha = torch.empty(1, S, dtype=torch.bfloat16, device=dev)
            works = [dist.all_to_all_single(qf[0], q[0], group=g, async_op=True),
                     dist.all_to_all_single(kf[0], k[0], group=g, async_op=True),
                     dist.all_to_all_single(vf[0], v[0], group=g, async_op=True),
                     dist.all_gather_into_tensor(alpha.view(-1), gate, group=g, async_op=True)]
            means = None
            if pooled:
                # qmean, kmean, vmean (f32), qsum, ksum, vsum (bf16): [source rank, head, block, D]
                means = tuple(torch.empty(n, hp, s // 64, D, dtype=x.dtype, device=dev) for x in stats)
                works += [dist.all_to_all_single(r, x[0], group=g, async_op=True) for r, x in zip(means, stats)]
            inbound.append((works, qf, kf, vf, alpha, means))
        outbound = []
        for b in range(B):
            works, qf, kf, vf, alpha, means = inbound[b]
            for w in works:
                w.wait()
            if means is not None:
                # [source rank, head, block, D] -> [1, head, global block, D]
                means = tuple(m.permute(1, 0, 2, 3).reshape(1, hp, n * (s // 64), D) for m in means)
                o = ops.self_attention(qf, kf, vf, alpha, t_seq_len, means=means)
            else:
                o = ops.self_attention(qf, kf, vf, alpha, t_seq_len)
            inbound[b] = None
            r = torch.empty(n, s, hp, D, dtype=torch.bfloat16, device=xin.device)
            outbound.append((dist.all_to_all_single(r, o[0], group=g, async_op=True), r))
        for b in range(B):
            work, r = outbound[b]
            work.wait()
            ops.linear_residual_(x[b * s:(b + 1) * s], r.permute(1, 0, 2, 3).reshape(s, C), blk.w_o, blk.b_o,
                                 res_gate[b:b + 1], s)

    @staticmethod
    def e_block(blk: _Block, e0):
        """(modulation + e0).chunk(6) in f32 (model.py:252), with 1 + scale
        formed once per block."""
        e = blk.modulation.float().unsqueeze(0) + e0
        return {"shift0": e[:, 0].contiguous(), "scale0": (1 + e[:, 1]).contiguous(), "gate0": e[:, 2].contiguous(),
                "shift1": e[:, 3].contiguous(), "scale1": (1 + e[:, 4]).contiguous(), "gate1": e[:, 5].contiguous()}

    # ------------------------------------------------------------------
    # whole model
    # ------------------------------------------------------------------
    def forward(self, latent, source_latent, t, context, seq_len: int):
        """Noise prediction for a batch of CFG branches sharing one latent.

        latent, source_latent: f32 [C_in, F, H, W] (replicated on every rank);
        t: timestep (python number or 0-d tensor); context: [B, text_len,
        text_dim] (one text embedding per branch); seq_len: joint tokens,
        divisible by the world size.  Returns f32 [B, out_dim, F, H, W] on
        every rank (model.py:410-451)."""
        cfg = self.cfg
        B = context.shape[0]
        if seq_len % self.world:
            raise ValueError(f"seq_len={seq_len} does not split over {self.world} ranks")
        x_all, grid, sgrid = self.embed(latent, source_latent, seq_len)
        t_seq_len = math.prod(grid)
        s = seq_len // self.world
        x = x_all[self.rank * s:(self.rank + 1) * s].unsqueeze(0).expand(B, s, cfg.dim).reshape(B * s, cfg.dim)
        del x_all
        tt = torch.as_tensor(t, dtype=torch.float64, device=self.device).reshape(1)
        e, e0 = self.time_embed(tt)
        e, e0 = e.expand(B, -1), e0.expand(B, -1, -1)
        ctx = self.text_embed(context)
        for i, blk in enumerate(self.blocks):
            x = self.block_forward(blk, x, e0, ctx, t_seq_len, first=(i == 0))
        return self.head(x, e, B, s, grid, seq_len)

    def head(self, x, e, B, s, grid, seq_len):
        """Head (model.py:278-289) on this rank's tokens, then the target
        tokens of all ranks gathered and unpatchified (model.py:448-450, :456-464)."""
        cfg = self.cfg
        m = self.head_modulation.float().unsqueeze(0) + e.unsqueeze(1)   # [B, 2, C]
        xn = self.ops.modulated_norm(x, (1 + m[:, 1]).contiguous(), m[:, 0].contiguous(), s, cfg.eps)
        y = self.ops.linear(xn, self.w_head, self.b_head).float().view(B, s, -1)
        if self.world > 1:
            P = y.shape[-1]
            parts = torch.empty(self.world * B * s * P, dtype=y.dtype, device=y.device)
            dist.all_gather_into_tensor(parts, y.reshape(-1), group=self.group)
            y = parts.view(self.world, B, s, P).permute(1, 0, 2, 3).reshape(B, seq_len, P)
        f, h, w = grid
        pf, ph, pw = cfg.patch_size
        u = y[:, :f * h * w].reshape(B, f, h, w, pf, ph, pw, cfg.out_dim)
        u = torch.einsum("bfhwpqrc->bcfphqwr", u)
        return u.reshape(B, cfg.out_dim, f * pf, h * ph, w * pw)

    def denoise_step(self, latent, source_latent, t, sigma, sigma_next, context, seq_len, guidance_scale=2.5,
                     check_status=True):
        """One denoising step of the reference's loop (inference.py:266-291):
        both CFG branches in one batch (context[0] unconditional, context[1]
        conditional), noise = uncond + g * (cond - uncond), then a
        flow-matching Euler update latent + (sigma_next - sigma) * noise,
        which stands in for the reference's UniPC solver (a few elementwise
        ops on the latent).

        check_status: after the step, synchronise and raise IcsaError if a
        bounded wait inside any attention kernel of the step gave up (the
        per-device record of icsa_last_status); skipped while the stream is
        being captured into a CUDA graph."""
        out = self.forward(latent, source_latent, t, context, seq_len)
        noise = out[0] + guidance_scale * (out[1] - out[0])
        new = latent + (sigma_next - sigma) * noise
        if check_status and not torch.cuda.is_current_stream_capturing():
            from in_context_sparse_attention import device_status
            device_status(new.device)
        return new
