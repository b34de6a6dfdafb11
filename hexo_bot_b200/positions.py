"""Seeded synthetic Hexo positions for tests and benchmarks.

The reference draws positions from uniform-random legal play through its Rust
rules engine (tests/shrimp_testkit.py:22-49). That engine is not available
here, so this module restates the rules that matter for featurization:

- the opening stone is forced to (0, 0) (hexo_engine rules.rs:16-23);
- player 1 then places two stones, player 0 two, and so on
  (state.rs:316-335); placement_index is 1-based (state.rs:266-272);
- a placement is legal when the cell is empty and within hex distance
  LEGAL_RADIUS of some stone (legal.rs:17, rules.rs:35-45).

Placements are drawn uniformly from the legal set (optionally restricted to a
fixed disk about the origin). A placement that would complete six in a row
for the mover is redrawn, so every generated position is a decision state.
"""

from __future__ import annotations

import random
from dataclasses import replace

from . import constants as K
from .featurize import (
    build_disk_support,
    build_features,
    build_support,
    collate_rows,
    facts_from_records,
    record_player,
)
from .geometry import disk_offsets

_AXES = ((1, 0), (0, 1), (1, -1))
_NEAR = tuple(disk_offsets(K.LEGAL_RADIUS))


def _wins(owner: dict, cell: tuple[int, int], player: int) -> bool:
    q, r = cell
    for dq, dr in _AXES:
        run = 1
        for sgn in (1, -1):
            k = 1
            while owner.get((q + sgn * k * dq, r + sgn * k * dr)) == player:
                run += 1
                k += 1
        if run >= 6:
            return True
    return False


def play_random(rng: random.Random, plies: int, disk_radius: int | None = None) -> list[tuple]:
    """Records (q, r, owner, placement_index) of `plies` random legal
    placements. With `disk_radius`, placements stay inside that disk."""

    allowed = set(disk_offsets(disk_radius)) if disk_radius is not None else None
    owner: dict = {}
    legal: set = set()
    records: list[tuple] = []
    for ply in range(plies):
        player = record_player(ply)
        if ply == 0:
            choices = [(0, 0)]
        else:
            choices = sorted(legal)
        placed = None
        while choices:
            cell = choices[rng.randrange(len(choices))] if len(choices) > 1 else choices[0]
            owner[cell] = player
            if ply > 0 and _wins(owner, cell, player):
                del owner[cell]
                choices = [c for c in choices if c != cell]
                continue
            placed = cell
            break
        if placed is None:
            break
        records.append((placed[0], placed[1], player, ply + 1))
        legal.discard(placed)
        for dq, dr in _NEAR:
            c = (placed[0] + dq, placed[1] + dr)
            if c not in owner and (allowed is None or c in allowed):
                legal.add(c)
    return records


def disk_position(seed: int, index: int, max_plies: int, disk_radius: int):
    """(Support, feats, facts) of one fixed-disk position; plies ~ U{0..max_plies}."""

    rng = random.Random(seed * 1_000_003 + index)
    plies = rng.randint(0, max_plies)
    records = play_random(rng, plies, disk_radius)
    facts = facts_from_records(records)
    sup = build_disk_support(facts.stones(), disk_radius)
    # Hot / win cells can fall outside the disk (a window may extend past it);
    # the fixed-disk regime drops those, as the support has no row for them.
    inside = sup.index.__contains__
    facts = replace(
        facts,
        own_hot=tuple(c for c in facts.own_hot if inside(c)),
        opp_hot=tuple(c for c in facts.opp_hot if inside(c)),
        own_win=tuple(c for c in facts.own_win if inside(c)),
        opp_win=tuple(c for c in facts.opp_win if inside(c)),
    )
    return sup, build_features(facts, sup), facts


def support_position(seed: int, index: int, max_plies: int, radius: int):
    """(Support, feats, facts) of one reference-support position (variable N)."""

    rng = random.Random(seed * 1_000_003 + index)
    plies = rng.randint(0, max_plies)
    records = play_random(rng, plies, None)
    facts = facts_from_records(records)
    sup = build_support(facts.stones(), radius)
    return sup, build_features(facts, sup), facts


def disk_batch(batch: int, seed: int, max_plies: int, disk_radius: int, start: int = 0):
    """Collated fixed-disk batch (all rows have N = |disk|, no padding)."""

    rows = [disk_position(seed, start + i, max_plies, disk_radius)[:2] for i in range(batch)]
    return collate_rows(rows)


def support_batch(batch: int, seed: int, max_plies: int, radius: int, pad_to: int | None = None):
    """Collated reference-support batch, padded to the largest row (or pad_to)."""

    rows = [support_position(seed, i, max_plies, radius)[:2] for i in range(batch)]
    return collate_rows(rows, pad_to=pad_to)


def tile_batch(batch: dict, copies: int) -> dict:
    """Repeat a collated batch `copies` times along the batch axis."""

    return {k: v.repeat((copies,) + (1,) * (v.dim() - 1)) for k, v in batch.items()}


__all__ = ["play_random", "disk_position", "support_position", "disk_batch", "support_batch", "tile_batch"]
