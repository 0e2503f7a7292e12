"""TEST INFRASTRUCTURE ONLY: a torch restatement of the reference's DiT block
math (model.py of the reference), with the same interface as
wan_dit._ops.CudaOps so that wan_dit.WanDiT can run on either.

Each method recomputes what the reference computes under CUDA autocast
(bf16 GEMMs, f32 residual stream), in the reference's own order of tensor
ops:

* LayerNorm:  F.layer_norm(x.float()) (WanLayerNorm, model.py:116-121), then
  `.float() * (1 + e[1]) + e[0]` (model.py:256, :263) and the Linear's bf16
  cast;
* RMSNorm:    `self._norm(x.float()).type_as(x) * self.weight`
  (WanRMSNorm, model.py:102-113);
* RoPE:       rope_params (model.py:54-59) and rope_apply (model.py:69-95),
  complex128 multiply of the (frame | row | column) frequency table, ones for
  padding tokens, result `.float()`;
* alpha_1:    `(Linear(x).sigmoid() - 0.5) * 0.5` on a bf16 tensor (:162);
* residual:   `x + y * e` with f32 e (:259, :262, :265);
* self-attention: the CPU oracle of this repository (oracle/icsa_oracle.py)
  on q, k f32 and v bf16, its f32 result cast to bf16 (the o-projection's
  autocast input);
* cross-attention: exact softmax attention in f32 (flash_attention,
  wanx/attention.py:18-85), cast to bf16.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from oracle import icsa_oracle


def rope_params(max_seq_len, dim, theta=10000):
    """complex128 [max_seq_len, dim/2] (model.py:54-59)."""
    freqs = torch.outer(torch.arange(max_seq_len),
                        1.0 / torch.pow(theta, torch.arange(0, dim, 2).to(torch.float64).div(dim)))
    return torch.polar(torch.ones_like(freqs), freqs)


def reference_freqs(D, positions=1024):
    """The model's concatenated table (model.py:380-384)."""
    return torch.cat([rope_params(positions, D - 4 * (D // 6)), rope_params(positions, 2 * (D // 6)),
                      rope_params(positions, 2 * (D // 6))], dim=1)


def rope_apply_tokens(x, token_pos, freqs):
    """rope_apply (model.py:69-95) for x [B, s, H, D] whose tokens have the
    positions token_pos [s, 4] (frame, row, column, rotate): complex128
    multiply, f32 result."""
    B, s, H, D = x.shape
    c = D // 2
    parts = freqs.split([c - 2 * (c // 3), c // 3, c // 3], dim=1)
    pos = token_pos.long().cpu()
    f = torch.cat([parts[0][pos[:, 0]], parts[1][pos[:, 1]], parts[2][pos[:, 2]]], dim=1)   # [s, c]
    f = torch.where(pos[:, 3:4].bool(), f, torch.ones_like(f))
    xc = torch.view_as_complex(x.to(torch.float64).cpu().reshape(B, s, H, c, 2))
    out = torch.view_as_real(xc * f.view(1, s, 1, c)).flatten(3)
    return out.float().to(x.device)


class ReferenceOps:
    """The reference's block math in torch (see the module docstring)."""

    def __init__(self, attention=None):
        self._attention = attention

    @staticmethod
    def linear(x, w, b=None):
        return F.linear(x, w, b)

    @staticmethod
    def gelu_tanh(x):
        return F.gelu(x, approximate="tanh")

    @staticmethod
    def _per_row(t, rows, rows_per_batch):
        if t.dim() == 1:
            return t.unsqueeze(0)
        idx = torch.arange(rows, device=t.device) // rows_per_batch
        return t[idx]

    def modulated_norm(self, x, scale, shift, rows_per_batch, eps, round_norm=False):
        rows, C = x.shape
        n = F.layer_norm(x.float(), (C,), eps=eps)
        if round_norm:
            n = n.to(x.dtype).float()
        y = n * self._per_row(scale, rows, rows_per_batch)
        y = y + self._per_row(shift, rows, rows_per_batch)
        return y.to(torch.bfloat16)

    def norm_rope(self, jobs, rows_per_batch, eps, token_offset=0, table=None, token_pos=None, splits=(0, 0),
                  gate=None):
        for src, w, rope, out in jobs:
            B, G, s, hp, D = out.shape
            x = src
            if w is not None:
                xf = x.float()
                x = (xf * torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + eps)).type_as(src) * w
            x = x.reshape(B, s, G * hp, D)
            if rope:
                freqs = reference_freqs(D, table.shape[0])
                pos = token_pos[token_offset:token_offset + s]
                x = rope_apply_tokens(x, pos, freqs)
            out.copy_(x.reshape(B, s, G, hp, D).permute(0, 2, 1, 3, 4).to(out.dtype))
        if gate is not None:
            gsrc, gout = gate
            gout.copy_((gsrc.sigmoid() - 0.5) * 0.5)

    def norm_rope_pool(self, jobs, means, rows_per_batch, eps, token_offset=0, table=None, token_pos=None,
                       splits=(0, 0), gate=None, round_mean=True, sums=None, bf16_mean=(False, False, False)):
        """norm_rope computed in f32, written as bf16, and the 64-token block
        means of the f32 values (compress_seq, editing_sparse_attention.py:
        37-55 of the reference), laid out [B, G, hp, s/64, D]; optionally the
        bf16 block sums of the bf16 outputs (rows summed in order in f32) and,
        with bf16_mean[j], mean j as bf16(bf16(sum) / 64) of the bf16 outputs."""
        f32 = []
        for src, w, rope, out in jobs:
            tmp = torch.empty(out.shape, dtype=torch.float32, device=out.device)
            f32.append(tmp)
            self.norm_rope([(src, w, rope, tmp)], rows_per_batch, eps, token_offset, table, token_pos, splits)
            out.copy_(tmp.to(out.dtype))
        if gate is not None:
            gsrc, gout = gate
            gout.copy_((gsrc.sigmoid() - 0.5) * 0.5)
        sums = list(sums) if sums is not None else [None] * len(jobs)

        def block_sum_in_order(x):
            # [B, G, s, hp, D] -> [B, G, s/64, hp, D], rows of a block added one by one
            B, G, s, hp, D = x.shape
            xb = x.reshape(B, G, s // 64, 64, hp, D)
            acc = torch.zeros(B, G, s // 64, hp, D, dtype=torch.float32, device=x.device)
            for r in range(64):
                acc = acc + xb[:, :, :, r]
            return acc

        for j, x in enumerate(f32):
            m, sm = means[j] if j < len(means) else None, sums[j]
            if m is None and sm is None:
                continue
            xb16 = x.to(torch.bfloat16).float()
            sum_bf = block_sum_in_order(xb16)
            if sm is not None:
                sm.copy_(sum_bf.to(torch.bfloat16).permute(0, 1, 3, 2, 4))
            if m is None:
                continue
            if bf16_mean[j]:
                mm = (sum_bf.to(torch.bfloat16).float() / 64.0).to(torch.bfloat16).float()
            else:
                mm = block_sum_in_order(x) / 64.0
                if round_mean:
                    mm = mm.to(torch.bfloat16).float()
            m.copy_(mm.permute(0, 1, 3, 2, 4))

    def gated_residual_(self, x, y, gate, rows_per_batch):
        if gate is None:
            x.copy_(x + y)
        else:
            x.copy_(x + y * self._per_row(gate, x.shape[0], rows_per_batch))
        return x

    def linear_residual_(self, x, a, w, b, gate, rows_per_batch):
        return self.gated_residual_(x, self.linear(a, w, b), gate, rows_per_batch)

    def self_attention(self, q, k, v, alpha, t_seq_len, means=None):
        if self._attention is not None:
            if means is not None:
                return self._attention(q, k, v, alpha, t_seq_len, means=means)
            return self._attention(q, k, v, alpha, t_seq_len)
        # the q / k means; the other block statistics of a six-array `means`
        # are what the oracle's pooling computes from the bf16 tensors anyway
        m = None if means is None else tuple(x.cpu().permute(0, 2, 1, 3) for x in means[:2])
        r = icsa_oracle.editing_sparse_attention(q.cpu(), k.cpu(), v.cpu(), t_seq_len,
                                                 alpha_2=alpha.cpu()[:, :, None, None], means=m)
        return r.out.to(torch.bfloat16).to(q.device).contiguous()

    @staticmethod
    def cross_attention(q, k, v):
        D = q.shape[-1]
        s = torch.einsum("blhd,bkhd->bhlk", q.float(), k.float()) / D ** 0.5
        return torch.einsum("bhlk,bkhd->blhd", s.softmax(-1), v.float()).to(torch.bfloat16)
