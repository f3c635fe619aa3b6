"""Tile-contiguous HBM layout of expert weights (the layout every bank and store holds).

A K-major weight matrix ``W [N, K]`` (N output rows, K reduction) is stored as
``[N/128][K/64][128][64]``: each 128-row x 64-column tile (16 KiB of bf16, one 128-byte
swizzle row per matrix row) is contiguous. One TMA box of the tcgen05 GEMM is then a single
16 KiB sequential read, and the decode GEMV's 8-row loads fall inside one 1 KiB span,
instead of 128-byte fragments 2*K bytes apart. The tensor keeps its logical shape
``[E, N, K]`` (same byte size, so whole-expert copies are layout-agnostic); only the element
order changes.

Shapes whose N is not a multiple of 128 or K not a multiple of 64 are left in row order
(tiny host-logic tests); the CUDA entry points require the tiled order.
"""

from __future__ import annotations

import torch

TILE_N = 128
TILE_K = 64


def tileable(n: int, k: int) -> bool:
    return n % TILE_N == 0 and k % TILE_K == 0


def to_tiled(w: torch.Tensor) -> torch.Tensor:
    """Row-major ``[..., N, K]`` -> tile-contiguous order, same shape."""
    *lead, n, k = w.shape
    if not tileable(n, k):
        raise ValueError(f"weight [{n}, {k}] is not a multiple of [{TILE_N}, {TILE_K}]")
    v = w.reshape(-1, n // TILE_N, TILE_N, k // TILE_K, TILE_K)
    return v.permute(0, 1, 3, 2, 4).contiguous().reshape(*lead, n, k)


def from_tiled(w: torch.Tensor) -> torch.Tensor:
    """Inverse of :func:`to_tiled`."""
    *lead, n, k = w.shape
    v = w.reshape(-1, n // TILE_N, k // TILE_K, TILE_N, TILE_K)
    return v.permute(0, 1, 3, 2, 4).contiguous().reshape(*lead, n, k)


def maybe_tiled(w: torch.Tensor) -> tuple[torch.Tensor, bool]:
    n, k = w.shape[-2:]
    if tileable(n, k):
        return to_tiled(w), True
    return w, False
