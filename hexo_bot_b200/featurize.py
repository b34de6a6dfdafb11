"""Host-side featurization: support sets, the 15 node-feature planes, batching.

This is the input side of the Shrimp forward: it turns a position (placement
history + side to move) into the four tensors the network consumes
(feats, nbr, mask, coords). It restates the reference's featurizer so batches
built here are interchangeable with the reference's:

- ``build_support``  -> packages/shrimp/python/shrimp/support.py:144-205
- ``window_scan``    -> packages/shrimp/python/shrimp/features.py:99-159
- ``build_features`` -> packages/shrimp/python/shrimp/features.py:165-231
- ``collate_rows``   -> packages/shrimp/python/shrimp/batching.py:45-80

``build_disk_support`` is the fixed-disk regime used for the benchmark
configurations (every position has the same N = |disk| cells, ordered
[legal | stones | rest]); its neighbour table and features come from the same
code as the reference support.

Pure numpy / Python; nothing here runs on the GPU.
"""

from __future__ import annotations

import os
from collections import deque
from dataclasses import dataclass

import numpy as np
import torch

from . import constants as K
from .geometry import disk_offsets, hex_dist

PHASE_OPENING = "Opening"
PHASE_FIRST = "FirstStone"
PHASE_SECOND = "SecondStone"

AXES: tuple[tuple[int, int], ...] = ((1, 0), (0, 1), (1, -1))  # Q, R, QR


def support_radius_from_env() -> int:
    raw = os.environ.get("SHRIMP_SUPPORT_RADIUS", "").strip()
    return int(raw) if raw else K.LEGAL_RADIUS


@dataclass(frozen=True)
class Support:
    """One position's node set in node order.

    coords (N, 2) int32 axial; dist (N,) int32 distance to the nearest stone;
    nbr (N, 6) int32 row-local neighbour per DIRECTIONS, -1 when absent;
    index maps (q, r) -> row. Rows [0, legal_count) are the legal cells."""

    coords: np.ndarray
    legal_count: int
    stone_count: int
    halo_count: int
    dist: np.ndarray
    nbr: np.ndarray
    index: dict

    @property
    def num_nodes(self) -> int:
        return int(self.coords.shape[0])


def neighbor_table(ordered: list[tuple[int, int]], index: dict) -> np.ndarray:
    """(N, 6) int32 row-local neighbour rows along DIRECTIONS, -1 if absent
    (support.py:196-205)."""

    nbr = np.full((len(ordered), 6), -1, dtype=np.int32)
    for row, (q, r) in enumerate(ordered):
        for k, (dq, dr) in enumerate(K.DIRECTIONS):
            j = index.get((q + dq, r + dr))
            if j is not None:
                nbr[row, k] = j
    return nbr


def _make_support(legal, stones, rest, dist_of) -> Support:
    ordered = list(legal) + list(stones) + list(rest)
    index = {c: i for i, c in enumerate(ordered)}
    return Support(
        coords=np.asarray(ordered, dtype=np.int32).reshape(-1, 2),
        legal_count=len(legal),
        stone_count=len(stones),
        halo_count=len(rest),
        dist=np.asarray([dist_of(c) for c in ordered], dtype=np.int32),
        nbr=neighbor_table(ordered, index),
        index=index,
    )


def build_support(stones: list[tuple[int, int]], radius: int | None = None) -> Support:
    """Reference support: legal cells (empty, within `radius` of a stone),
    stones, then the distance-(radius+1) halo; each segment ascending (q, r).
    With no stones the support is the origin (legal) plus its six neighbours
    (support.py:144-166). One multi-source BFS gives membership and dist."""

    radius = support_radius_from_env() if radius is None else int(radius)
    if not stones:
        halo = sorted(K.DIRECTIONS)
        return _make_support([(0, 0)], [], halo, lambda c: 0)

    stone_set = set(stones)
    dist = {c: 0 for c in stone_set}
    queue = deque(stone_set)
    halo_d = radius + 1
    while queue:
        cell = queue.popleft()
        d = dist[cell]
        if d >= halo_d:
            continue
        for dq, dr in K.DIRECTIONS:
            nxt = (cell[0] + dq, cell[1] + dr)
            if nxt not in dist:
                dist[nxt] = d + 1
                queue.append(nxt)
    legal = sorted(c for c, d in dist.items() if 0 < d <= radius)
    halo = sorted(c for c, d in dist.items() if d == halo_d)
    return _make_support(legal, sorted(stone_set), halo, dist.__getitem__)


def build_disk_support(stones: list[tuple[int, int]], disk_radius: int) -> Support:
    """Fixed-disk support: every cell of the radius-`disk_radius` disk about the
    origin, ordered [legal | stones | rest]. Legal = empty disk cells within
    LEGAL_RADIUS of a stone (only the origin before the first stone); rest =
    the remaining empty disk cells. dist = hex distance to the nearest stone
    (0 everywhere before the first stone)."""

    cells = disk_offsets(disk_radius)
    stone_set = set(stones)
    if not stone_set:
        legal = [(0, 0)]
        rest = [c for c in cells if c != (0, 0)]
        return _make_support(legal, [], rest, lambda c: 0)

    st = np.asarray(sorted(stone_set), dtype=np.int64).reshape(-1, 2)

    def nearest(c):
        dq = st[:, 0] - c[0]
        dr = st[:, 1] - c[1]
        return int(np.max(np.stack([np.abs(dq), np.abs(dr), np.abs(dq + dr)]), axis=0).min())

    dmap = {c: nearest(c) for c in cells}
    for s in stone_set:
        dmap.setdefault(s, 0)
    legal = [c for c in cells if c not in stone_set and dmap[c] <= K.LEGAL_RADIUS]
    rest = [c for c in cells if c not in stone_set and dmap[c] > K.LEGAL_RADIUS]
    return _make_support(legal, sorted(stone_set), rest, dmap.__getitem__)


# --- position facts ------------------------------------------------------------


@dataclass(frozen=True)
class PositionFacts:
    """One decision state (features.py:51-75). records are (q, r, owner,
    placement_index) in play order with 1-based placement_index; hot / win
    cell lists are relative to current_player."""

    records: tuple
    current_player: int
    phase: str
    first_stone: tuple | None
    own_hot: tuple
    opp_hot: tuple
    own_win: tuple
    opp_win: tuple

    @property
    def placements_made(self) -> int:
        return len(self.records)

    def stones(self) -> list[tuple[int, int]]:
        return [(q, r) for q, r, _o, _i in self.records]


def record_phase(ordinal: int) -> str:
    """Phase of the ordinal-th placement: one opening stone, then pairs
    (features.py:80-85)."""

    if ordinal == 0:
        return PHASE_OPENING
    return PHASE_FIRST if (ordinal - 1) % 2 == 0 else PHASE_SECOND


def record_player(ordinal: int) -> int:
    """Player of the ordinal-th placement: player 0 opens, then player 1 plays
    two stones, player 0 two, ... (features.py:88-93)."""

    if ordinal == 0:
        return 0
    return 1 if ((ordinal - 1) // 2) % 2 == 0 else 0


def side_to_move(placements_made: int) -> tuple[int, str]:
    """(current_player, phase) after `placements_made` placements."""

    return record_player(placements_made), record_phase(placements_made)


def window_scan(records, current_player: int, placements_made: int):
    """(own_hot, opp_hot, own_win, opp_win) from every length-6 window along the
    three axes that contains at least one stone (features.py:99-159).

    Windows with both colours are ignored. A single-colour window with exactly
    WIN_NOW_COUNT stones marks its one empty cell as a standing win; with
    >= HOT_MIN_COUNT stones (once HOT_MIN_PLACEMENTS placements are made) all
    its empty cells are hot. Lists are sorted by (q, r)."""

    owner = {(q, r): o for q, r, o, _i in records}
    starts = set()
    for (q, r) in owner:
        for ax, (dq, dr) in enumerate(AXES):
            for back in range(K.WINDOW_LEN):
                starts.add((q - back * dq, r - back * dr, ax))
    hot_ok = placements_made >= K.HOT_MIN_PLACEMENTS
    out = {"own_hot": set(), "opp_hot": set(), "own_win": set(), "opp_win": set()}
    for sq, sr, ax in starts:
        dq, dr = AXES[ax]
        cells = [(sq + i * dq, sr + i * dr) for i in range(K.WINDOW_LEN)]
        owners = [owner.get(c) for c in cells]
        present = {o for o in owners if o is not None}
        if len(present) != 1:
            continue
        (who,) = present
        count = sum(o is not None for o in owners)
        empties = [c for c, o in zip(cells, owners) if o is None]
        side = "own" if who == current_player else "opp"
        if count == K.WIN_NOW_COUNT:
            out[f"{side}_win"].update(empties)
        if count >= K.HOT_MIN_COUNT and hot_ok:
            out[f"{side}_hot"].update(empties)
    return tuple(tuple(sorted(out[k])) for k in ("own_hot", "opp_hot", "own_win", "opp_win"))


def facts_from_records(records) -> PositionFacts:
    """PositionFacts for the decision state after `records` (q, r, owner,
    placement_index) were played; the hot / win lists come from window_scan."""

    records = tuple(tuple(int(v) for v in rec) for rec in records)
    n = len(records)
    player, phase = side_to_move(n)
    first = (records[-1][0], records[-1][1]) if phase == PHASE_SECOND else None
    own_hot, opp_hot, own_win, opp_win = window_scan(records, player, n)
    return PositionFacts(records, player, phase, first, own_hot, opp_hot, own_win, opp_win)


def _opp_last_turn_cells(facts: PositionFacts) -> list[tuple[int, int]]:
    """Cells of the opponent's most recent complete turn (features.py:234-254)."""

    opponent = 1 - facts.current_player
    recs = facts.records
    for ordinal in range(len(recs) - 1, -1, -1):
        if record_player(ordinal) != opponent:
            continue
        phase = record_phase(ordinal)
        if phase == PHASE_SECOND:
            return [(recs[ordinal - 1][0], recs[ordinal - 1][1]), (recs[ordinal][0], recs[ordinal][1])]
        if phase == PHASE_OPENING:
            return [(recs[ordinal][0], recs[ordinal][1])]
    return []


def build_features(facts: PositionFacts, sup: Support) -> np.ndarray:
    """(N, 15) float32 node features in support order (features.py:165-231)."""

    n = sup.num_nodes
    f = np.zeros((n, K.NUM_FEATURES), dtype=np.float32)
    made = facts.placements_made
    for q, r, owner, pidx in facts.records:
        row = sup.index[(q, r)]
        own = owner == facts.current_player
        f[row, K.F_OWN_STONE if own else K.F_OPP_STONE] = 1.0
        plane = K.F_OWN_RECENCY if own else K.F_OPP_RECENCY
        f[row, plane] = max(f[row, plane], 1.0 / (1.0 + float(made - pidx)))
    f[:, K.F_EMPTY] = 1.0 - f[:, K.F_OWN_STONE] - f[:, K.F_OPP_STONE]
    f[: sup.legal_count, K.F_LEGAL] = 1.0
    if facts.phase == PHASE_SECOND:
        f[:, K.F_PHASE_SECOND] = 1.0
        if facts.first_stone is not None:
            f[sup.index[tuple(facts.first_stone)], K.F_FIRST_STONE] = 1.0
    if facts.current_player == 0:
        f[:, K.F_PLAYER_COLOUR] = 1.0
    for plane, cells in (
        (K.F_OPP_HOT, facts.opp_hot),
        (K.F_OWN_HOT, facts.own_hot),
        (K.F_OPP_WIN_NOW, facts.opp_win),
        (K.F_OWN_WIN_NOW, facts.own_win),
    ):
        for c in cells:
            f[sup.index[tuple(c)], plane] = 1.0
    f[:, K.F_DIST_TO_STONE] = sup.dist.astype(np.float32) / K.DIST_SCALE
    for c in _opp_last_turn_cells(facts):
        f[sup.index[c], K.F_OPP_LAST_TURN] = 1.0
    return f


def collate_rows(rows, pad_to: int | None = None) -> dict[str, torch.Tensor]:
    """Pad (Support, feats) rows into one batch (batching.py:45-80): zero pad
    features, pad neighbours -> Npad (the appended zero row), mask False on
    pad rows, zero pad coords. int64 nbr / coords like the reference."""

    npad = max(sup.num_nodes for sup, _ in rows)
    if pad_to is not None:
        if pad_to < npad:
            raise ValueError(f"pad_to {pad_to} < largest row {npad}")
        npad = pad_to
    b = len(rows)
    feats = np.zeros((b, npad, K.NUM_FEATURES), dtype=np.float32)
    nbr = np.full((b, npad, 6), npad, dtype=np.int64)
    mask = np.zeros((b, npad), dtype=np.bool_)
    coords = np.zeros((b, npad, 2), dtype=np.int64)
    legal = np.zeros(b, dtype=np.int64)
    for g, (sup, fr) in enumerate(rows):
        n = sup.num_nodes
        feats[g, :n] = fr
        nbr[g, :n] = np.where(sup.nbr >= 0, sup.nbr, npad)
        mask[g, :n] = True
        coords[g, :n] = sup.coords
        legal[g] = sup.legal_count
    return {
        "feats": torch.from_numpy(feats),
        "nbr": torch.from_numpy(nbr),
        "mask": torch.from_numpy(mask),
        "coords": torch.from_numpy(coords),
        "legal_counts": torch.from_numpy(legal),
    }


def hex_distance_array(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Vectorised hex distance between (…, 2) coordinate arrays."""

    d = b.astype(np.int64) - a.astype(np.int64)
    return np.max(np.abs(np.stack([d[..., 0], d[..., 1], d[..., 0] + d[..., 1]])), axis=0)


__all__ = [
    "Support",
    "PositionFacts",
    "build_support",
    "build_disk_support",
    "neighbor_table",
    "window_scan",
    "facts_from_records",
    "build_features",
    "collate_rows",
    "record_phase",
    "record_player",
    "side_to_move",
    "hex_dist",
]
