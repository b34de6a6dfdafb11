"""Seeded inputs of the two kernel microbenches (BASELINE configs 2 and 3).

Neither microbench has a reference kernel; they exercise the same operations
as the network at the shapes BASELINE names:

- attention: B positions x L = 61 tokens (the radius-4 disk) x H = 8 heads x
  d = 32, bf16 Q/K/V ~ N(0, 1) in (B, L, H*d), an fp32 bias table over the
  exact hex offsets of radius 8 (217 rows; radius 16 gives 817) ~ N(0, 0.5),
  indexed by the (L, L) offset-id map of key - query;
- 19-tap ray conv: B positions x N = 61 cells x C = 128, bf16 x ~ N(0, 1),
  bf16 weights (19 C, C) ~ N(0, 1/sqrt(19 C)), fp32 bias, neighbour table of
  `geometry.raytap_neighbors`.

Each position's rows come from a generator seeded by (config seed, position
index), so a shard or a sample holds exactly the rows it holds in the full
batch; the shared tables use the config seed alone.
"""

from __future__ import annotations

import math

import torch

from . import geometry

ATTN_MICRO = dict(batch=4096, disk=4, heads=8, head_dim=32, table_radius=8, seed=2)
CONV19_MICRO = dict(batch=4096, disk=4, channels=128, seed=3)


def disk_cells(radius: int) -> int:
    """Cells of the radius-`radius` hex disk, 3 r (r + 1) + 1."""

    return 3 * radius * (radius + 1) + 1


def _position_generator(seed: int, index: int) -> torch.Generator:
    return torch.Generator().manual_seed(seed * 1_000_003 + index)


def attention_inputs(cfg: dict, count: int, start: int = 0) -> dict:
    """q, k, v (count, L, H*d) bf16; table (rows, H) f32; offset_map (L, L) int32."""

    n = disk_cells(cfg["disk"])
    hd = cfg["heads"] * cfg["head_dim"]
    g = torch.Generator().manual_seed(cfg["seed"])
    rows = disk_cells(cfg["table_radius"])
    table = torch.randn(rows, cfg["heads"], generator=g) * 0.5
    offset_map = torch.from_numpy(geometry.offset_id_map(cfg["disk"], cfg["table_radius"]))
    qkv = torch.empty(3, count, n, hd)
    for i in range(count):
        qkv[:, i] = torch.randn(3, n, hd, generator=_position_generator(cfg["seed"], start + i))
    q, k, v = (t.bfloat16() for t in qkv)
    return {"q": q, "k": k, "v": v, "table": table, "offset_map": offset_map}


def conv19_inputs(cfg: dict, count: int, start: int = 0) -> dict:
    """x (count, N, C) bf16; nbr (N, 19) int32 (-1 = off the disk); weight
    (19 C, C) bf16 with row t*C + c the input channel c of tap t; bias (C,) f32."""

    n = disk_cells(cfg["disk"])
    c = cfg["channels"]
    taps = geometry.RAY_TAPS
    g = torch.Generator().manual_seed(cfg["seed"])
    weight = (torch.randn(taps * c, c, generator=g) / math.sqrt(taps * c)).bfloat16()
    bias = torch.randn(c, generator=g) * 0.1
    x = torch.empty(count, n, c)
    for i in range(count):
        x[i] = torch.randn(n, c, generator=_position_generator(cfg["seed"], start + i))
    return {"x": x.bfloat16(), "nbr": torch.from_numpy(geometry.raytap_neighbors(cfg["disk"])), "weight": weight,
            "bias": bias}


__all__ = ["ATTN_MICRO", "CONV19_MICRO", "disk_cells", "attention_inputs", "conv19_inputs"]
