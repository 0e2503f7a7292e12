"""Wan 2.2 DiT around the in-context sparse attention (the reference's
model.py), for one denoising step on B200s with Ulysses sequence parallelism.
"""
from .model import WanDiT, WanDiTConfig, sinusoidal_embedding_1d  # noqa: F401
from .rope import head_dim_splits, rope_table, token_positions  # noqa: F401

__all__ = ["WanDiT", "WanDiTConfig", "sinusoidal_embedding_1d", "head_dim_splits", "rope_table", "token_positions"]
