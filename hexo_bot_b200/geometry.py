"""Hex-lattice index math used to build the device-side lookup tables.

Axial coordinates (q, r); the third cube axis is s = -q - r. Everything here is
exact integer arithmetic. The functions restate the reference's geometry
(packages/shrimp/python/shrimp/geometry.py:24-131) so the bias-row table the
CUDA kernels consume is bit-identical to the one the reference gathers from.
"""

from __future__ import annotations

from functools import lru_cache

import numpy as np

from . import constants as K


def hex_dist(dq: int, dr: int) -> int:
    """Hex distance of an axial offset, max(|dq|, |dr|, |dq + dr|) (geometry.py:24-27)."""

    return max(abs(dq), abs(dr), abs(dq + dr))


def on_win_axis(dq: int, dr: int) -> bool:
    """Offset lies on one of the three win axes Q, R or QR (geometry.py:85-92)."""

    return dq == 0 or dr == 0 or dq + dr == 0


def disk_offsets(radius: int) -> list[tuple[int, int]]:
    """Offsets within `radius`, ascending by (dq, dr) (geometry.py:97-109)."""

    out = []
    for dq in range(-radius, radius + 1):
        lo = max(-radius, -radius - dq)
        hi = min(radius, radius - dq)
        out.extend((dq, dr) for dr in range(lo, hi + 1))
    return out


@lru_cache(maxsize=None)
def _exact_rows() -> dict[tuple[int, int], int]:
    rows = {off: i for i, off in enumerate(disk_offsets(K.BIAS_DISK_RADIUS))}
    assert len(rows) == K.BIAS_EXACT_ROWS
    return rows


def rel_bias_index(dq: int, dr: int) -> int:
    """Bias-table row of a (key - query) cell offset (geometry.py:115-131).

    Exact row for distance <= 8; distance 9..16 maps to an on-axis or
    off-axis ring row; anything further is the far row."""

    d = hex_dist(dq, dr)
    if d <= K.BIAS_DISK_RADIUS:
        return _exact_rows()[(dq, dr)]
    if d <= K.BIAS_RING_MAX:
        base = K.BIAS_ON_AXIS_BASE if on_win_axis(dq, dr) else K.BIAS_OFF_AXIS_BASE
        return base + d - K.BIAS_RING_MIN
    return K.BIAS_FAR_ROW


@lru_cache(maxsize=None)
def cell_bias_lut() -> np.ndarray:
    """(LUT_W * LUT_W,) uint8: entry (dq+M)*W + (dr+M) = rel_bias_index(dq, dr)
    for |dq|, |dr| <= M (model.py:625-641). Offsets are clamped to +-M before
    the lookup, which sends every offset beyond the rings to the far row."""

    m, w = K.LUT_M, K.LUT_W
    lut = np.empty(w * w, dtype=np.uint8)
    for dq in range(-m, m + 1):
        for dr in range(-m, m + 1):
            lut[(dq + m) * w + dr + m] = rel_bias_index(dq, dr)
    lut.flags.writeable = False
    return lut


# --- microbench tables (BASELINE configs 2 and 3; no reference kernel) -----------

# Win axes in the order [Q, R, QR] (hexfield_eq features.py:79 AXIS_DELTAS).
RAY_AXES = ((1, 0), (0, 1), (1, -1))
RAY_STEPS = 3
RAY_TAPS = 1 + len(RAY_AXES) * 2 * RAY_STEPS  # 19


def raytap_neighbors(disk_radius: int) -> np.ndarray:
    """(N, 19) int32 over the radius-`disk_radius` disk in `disk_offsets` order:
    tap 0 is the cell itself; tap 1 + axis*6 + dir*3 + (k-1) is the cell at
    offset (+k or -k for dir 0 / 1) x axis, -1 when that cell is off the disk
    (the ray packing of hexfield_eq _raytap.py:84-96 with three steps)."""

    cells = disk_offsets(disk_radius)
    index = {c: i for i, c in enumerate(cells)}
    out = np.full((len(cells), RAY_TAPS), -1, dtype=np.int32)
    for i, (q, r) in enumerate(cells):
        out[i, 0] = i
        for a, (aq, ar) in enumerate(RAY_AXES):
            for d, sgn in enumerate((1, -1)):
                for k in range(1, RAY_STEPS + 1):
                    out[i, 1 + a * 6 + d * 3 + (k - 1)] = index.get((q + sgn * k * aq, r + sgn * k * ar), -1)
    return out


def offset_id_map(disk_radius: int, table_radius: int) -> np.ndarray:
    """(N, N) int32 offset-id map over the radius-`disk_radius` disk: entry
    (query, key) is the index of the exact offset key - query in
    `disk_offsets(table_radius)` (217 ids at radius 8, 817 at radius 16)."""

    cells = disk_offsets(disk_radius)
    ids = {off: i for i, off in enumerate(disk_offsets(table_radius))}
    out = np.empty((len(cells), len(cells)), dtype=np.int32)
    for i, (qq, qr) in enumerate(cells):
        for j, (kq, kr) in enumerate(cells):
            out[i, j] = ids[(kq - qq, kr - qr)]
    return out


# --- D6 about the origin (geometry.py:52-82) -------------------------------------


def rot60(q: int, r: int) -> tuple[int, int]:
    return -r, q + r


def reflect(q: int, r: int) -> tuple[int, int]:
    return q, -q - r


def apply_d6(index: int, q: int, r: int) -> tuple[int, int]:
    """Transform 0..5 rotates by index*60 degrees; 6..11 reflect first."""

    if not 0 <= index < 12:
        raise ValueError(f"D6 index out of range: {index}")
    if index >= 6:
        q, r = reflect(q, r)
        index -= 6
    for _ in range(index):
        q, r = rot60(q, r)
    return q, r


def d6_inverse(index: int) -> int:
    if not 0 <= index < 12:
        raise ValueError(f"D6 index out of range: {index}")
    return index if index >= 6 else (6 - index) % 6


def pack_action_id(q: int, r: int) -> int:
    """((q + 2^15) << 16) | (r + 2^15); integer order equals (q, r) order."""

    lo, hi = -(1 << 15), (1 << 15) - 1
    if not (lo <= q <= hi and lo <= r <= hi):
        raise ValueError(f"coordinate out of i16 range: ({q}, {r})")
    return ((q + K.COORD_OFFSET) << 16) | (r + K.COORD_OFFSET)


def unpack_action_id(action_id: int) -> tuple[int, int]:
    return ((action_id >> 16) & 0xFFFF) - K.COORD_OFFSET, (action_id & 0xFFFF) - K.COORD_OFFSET
