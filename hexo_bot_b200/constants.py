"""Shrimp model constants: node-feature planes, geometry radii, bias-table rows.

The values mirror the reference's contract (packages/shrimp/python/shrimp/
constants.py:1-126) because checkpoints, featurized inputs and the bias-table
row layout must be interchangeable with it. Architecture defaults are read from
the same environment variables at import time (SHRIMP_CHANNELS,
SHRIMP_ATTENTION_HEADS, SHRIMP_TRUNK; constants.py:81-104), and can be
overridden per model through the ShrimpNet constructor.
"""

from __future__ import annotations

import os

# Legal placements: empty cells within this hex distance of any stone
# (reference constants.py:14-15, engine legal.rs). The halo is one ring further.
LEGAL_RADIUS = 8
HALO_DIST = LEGAL_RADIUS + 1

# Neighbour direction order: the rotate-60 orbit of (1, 0). Tap k+1 of every
# hex convolution reads the neighbour at DIRECTIONS[k] (constants.py:20-27).
DIRECTIONS: tuple[tuple[int, int], ...] = (
    (1, 0),
    (0, 1),
    (-1, 1),
    (-1, 0),
    (0, -1),
    (1, -1),
)

COORD_OFFSET = 1 << 15
NBR_SENTINEL_U16 = 0xFFFF

# Node feature planes (constants.py:40-56).
F_OWN_STONE = 0
F_OPP_STONE = 1
F_EMPTY = 2
F_LEGAL = 3
F_PHASE_SECOND = 4
F_FIRST_STONE = 5
F_PLAYER_COLOUR = 6
F_OWN_RECENCY = 7
F_OPP_RECENCY = 8
F_OPP_HOT = 9
F_OWN_HOT = 10
F_DIST_TO_STONE = 11
F_OPP_LAST_TURN = 12
F_OPP_WIN_NOW = 13
F_OWN_WIN_NOW = 14
NUM_FEATURES = 15

HOT_MIN_COUNT = 4
WIN_NOW_COUNT = 5
HOT_MIN_PLACEMENTS = 7
WINDOW_LEN = 6

DIST_SCALE = float(LEGAL_RADIUS)
HALO_DIST_FEATURE = HALO_DIST / DIST_SCALE

VALUE_BINS = 65
MOVES_LEFT_CAP = 209

NUM_TOKENS = 8
MLP_RATIO = 2


def _env_int(name: str, default: int) -> int:
    raw = os.environ.get(name, "").strip()
    return int(raw) if raw else default


CHANNELS = _env_int("SHRIMP_CHANNELS", 96)
ATTENTION_HEADS = _env_int("SHRIMP_ATTENTION_HEADS", 4)
TRUNK_LAYOUT = os.environ.get("SHRIMP_TRUNK", "").strip() or "CCCACCCACCA"


def validate_layout(layout: str) -> str:
    """A trunk layout is a non-empty C/A string ending in 'A' (constants.py:96-104)."""

    if not layout or set(layout) - {"C", "A"} or not layout.endswith("A"):
        raise ValueError(f"invalid trunk layout {layout!r}: need C/A letters ending with 'A'")
    return layout


if CHANNELS % ATTENTION_HEADS != 0:
    raise ValueError(
        f"SHRIMP_CHANNELS={CHANNELS} not divisible by SHRIMP_ATTENTION_HEADS={ATTENTION_HEADS}"
    )
validate_layout(TRUNK_LAYOUT)

# Relative-position bias table rows (constants.py:106-126):
#   0..216   exact offsets with hex distance <= 8, ascending (dq, dr)
#   217..224 on-win-axis rings, distance 9..16
#   225..232 off-axis rings, distance 9..16
#   233      far (distance >= 17)
#   234/235/236 cell->token, token->cell, token->token
BIAS_DISK_RADIUS = LEGAL_RADIUS
BIAS_EXACT_ROWS = 217
BIAS_RING_MIN = 9
BIAS_RING_MAX = 16
BIAS_ON_AXIS_BASE = 217
BIAS_OFF_AXIS_BASE = 225
BIAS_FAR_ROW = 233
BIAS_CELL_TOKEN_ROW = 234
BIAS_TOKEN_CELL_ROW = 235
BIAS_TOKEN_TOKEN_ROW = 236
BIAS_ROWS = 237
# Extra row used by the uint8 pair table for dead (padded) keys.
BIAS_PAD_ROW = BIAS_ROWS

# Offset clamp for the cell LUT: |dq|, |dr| are clamped to LUT_M before the
# lookup (model.py:625-641), giving a (2*LUT_M+1)^2 table.
LUT_M = BIAS_RING_MAX + 1
LUT_W = 2 * LUT_M + 1

PAD_KEY_MASK_VALUE = -3.0e4
