"""Seeded synthetic inputs with the shapes and statistics of the benchmark
configurations (the reference's EditVerse videos and Wan 2.2 weights are not
available; these stand in for them).

Two recipes:

* ``"gaussian"`` (configuration 1): q, k, v ~ N(0, 1); the source half of k and
  v is ``0.8 * target + 0.6 * N(0, 1)`` so that in-context retrieval is
  non-trivial.
* ``"blurred"`` (480p / 720p configurations): per tensor, a target field that is
  a Gaussian blur (sigma = 2 tokens along frames, rows and columns of the
  latent grid, separable, reflect padding) of N(0, 1), renormalised to unit
  variance, plus 0.5 * N(0, 1) noise; the source half is
  ``0.8 * target + 0.6 * independent field``.  Each half is the flattened
  latent grid padded with fresh N(0, 1) rows up to a multiple of 64.

Every (tensor, head) pair draws from its own seeded generator, so any subset
of heads (a rank's shard) is bit-identical to the same heads of the full
tensor.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

BLOCK = 64


@dataclass(frozen=True)
class Workload:
    name: str
    B: int
    H: int
    D: int
    grid: tuple            # latent grid (frames, rows, cols) of one video
    recipe: str            # "gaussian" | "blurred"
    dtype: torch.dtype
    half_len: int = 0      # tokens per video after padding (0: from grid)

    @property
    def t_seq_len(self) -> int:
        if self.half_len:
            return self.half_len
        n = self.grid[0] * self.grid[1] * self.grid[2]
        return (n + BLOCK - 1) // BLOCK * BLOCK

    @property
    def S(self) -> int:
        return 2 * self.t_seq_len


CONFIG1 = Workload("config1_cpu_fp32", 1, 2, 64, (1, 64, 64), "gaussian", torch.float32, half_len=4096)
WAN480P = Workload("wan22_480p_joint65k", 1, 40, 128, (21, 30, 52), "blurred", torch.bfloat16)
WAN720P = Workload("wan22_720p_joint151k", 1, 40, 128, (21, 45, 80), "blurred", torch.bfloat16)

# stream ids of the per-(tensor, head) generators
_STREAMS = {("q", "t"): 0, ("k", "t"): 1, ("v", "t"): 2, ("q", "s"): 3, ("k", "s"): 4, ("v", "s"): 5}


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def _blur_axis(x: torch.Tensor, dim: int, kernel: torch.Tensor) -> torch.Tensor:
    r = (kernel.numel() - 1) // 2
    xm = x.movedim(dim, -1)
    shp = xm.shape
    flat = xm.reshape(-1, 1, shp[-1])
    flat = torch.nn.functional.pad(flat, (r, r), mode="reflect")
    out = torch.nn.functional.conv1d(flat, kernel.view(1, 1, -1))
    return out.reshape(shp).movedim(-1, dim)


def _blurred_field(g: torch.Generator, C: int, grid, device) -> torch.Tensor:
    """[C, F, Hh, W] unit-variance Gaussian-blurred N(0,1) field."""
    sigma = 2.0
    r = int(math.ceil(3 * sigma))
    xs = torch.arange(-r, r + 1, dtype=torch.float32, device=device)
    kernel = torch.exp(-0.5 * (xs / sigma) ** 2)
    kernel = kernel / kernel.sum()
    f = torch.randn(C, *grid, generator=g, device=device, dtype=torch.float32)
    for dim in (1, 2, 3):
        if f.shape[dim] > r:
            f = _blur_axis(f, dim, kernel)
    return f / f.std()


def _half_blurred(g: torch.Generator, C: int, grid, half_len: int, device) -> torch.Tensor:
    """[half_len, C]: field + 0.5 noise over the grid tokens, fresh N(0,1) tail."""
    n = grid[0] * grid[1] * grid[2]
    f = _blurred_field(g, C, grid, device).reshape(C, n).t()
    f = f + 0.5 * torch.randn(n, C, generator=g, device=device)
    if half_len > n:
        f = torch.cat([f, torch.randn(half_len - n, C, generator=g, device=device)], dim=0)
    return f


def make_head(w: Workload, tensor: str, head: int, seed_base: int = 0, device="cpu") -> torch.Tensor:
    """[B, S, D] fp32 values of one head of q, k or v."""
    T = w.t_seq_len
    out = torch.empty(w.B, 2 * T, w.D, device=device)
    for b in range(w.B):
        gt = _gen(seed_base + 1000003 * b + 7919 * _STREAMS[(tensor, "t")] + head, device)
        gs = _gen(seed_base + 1000003 * b + 7919 * _STREAMS[(tensor, "s")] + head, device)
        if w.recipe == "gaussian":
            tgt = torch.randn(T, w.D, generator=gt, device=device)
            if tensor == "q":
                src = torch.randn(T, w.D, generator=gs, device=device)
            else:
                src = 0.8 * tgt + 0.6 * torch.randn(T, w.D, generator=gs, device=device)
        else:
            tgt = _half_blurred(gt, w.D, w.grid, T, device)
            src = 0.8 * tgt + 0.6 * _half_blurred(gs, w.D, w.grid, T, device)
        out[b, :T] = tgt
        out[b, T:] = src
    return out


def make_inputs(w: Workload, heads=None, seed_base: int = 0, device="cpu", dtype=None):
    """q, k, v as [B, S, len(heads), D] tensors of `dtype` (default w.dtype)."""
    heads = list(range(w.H)) if heads is None else list(heads)
    dtype = w.dtype if dtype is None else dtype
    res = []
    for name in ("q", "k", "v"):
        x = torch.empty(w.B, w.S, len(heads), w.D, device=device, dtype=dtype)
        for i, h in enumerate(heads):
            x[:, :, i] = make_head(w, name, h, seed_base, device).to(dtype)
        res.append(x)
    return tuple(res)
