"""Featurizer and synthetic-position contracts (CPU)."""

from __future__ import annotations

import random

import numpy as np
import torch

from hexo_bot_b200 import constants as K
from hexo_bot_b200 import featurize as F
from hexo_bot_b200 import positions as P


def test_ply0_support():
    sup = F.build_support([], 8)
    assert (sup.num_nodes, sup.legal_count, sup.stone_count, sup.halo_count) == (7, 1, 0, 6)
    assert tuple(sup.coords[0]) == (0, 0)
    assert sup.dist.tolist() == [0] * 7


def test_one_stone_scale_anchor():
    # reference tests/test_shrimp_support.py:103-109
    sup = F.build_support([(0, 0)], 8)
    assert (sup.num_nodes, sup.legal_count, sup.stone_count, sup.halo_count) == (271, 216, 1, 54)
    sup4 = F.build_support([(0, 0)], 4)
    assert sup4.num_nodes == 91


def test_neighbor_table_convention():
    sup = F.build_support([(0, 0), (1, 0), (0, 1), (2, -1)], 4)
    for row, (q, r) in enumerate(sup.coords.tolist()):
        for k, (dq, dr) in enumerate(K.DIRECTIONS):
            assert sup.nbr[row, k] == sup.index.get((q + dq, r + dr), -1)


def test_disk_support_has_fixed_size_and_order():
    for seed in range(5):
        sup, feats, facts = P.disk_position(seed, 0, 30, 4)
        assert sup.num_nodes == 61 and feats.shape == (61, 15)
        assert sup.legal_count + sup.stone_count + sup.halo_count == 61
        assert np.all(feats[: sup.legal_count, K.F_LEGAL] == 1.0)
        stones = sup.coords[sup.legal_count: sup.legal_count + sup.stone_count]
        assert sorted(map(tuple, stones.tolist())) == sorted(facts.stones())


def test_random_play_rules():
    rng = random.Random(3)
    recs = P.play_random(rng, 40, None)
    assert recs[0][:2] == (0, 0) and recs[0][2] == 0 and recs[0][3] == 1
    for i, (q, r, owner, idx) in enumerate(recs):
        assert owner == F.record_player(i) and idx == i + 1
    cells = [(q, r) for q, r, _, _ in recs]
    assert len(set(cells)) == len(cells)
    for i in range(1, len(cells)):
        assert min(max(abs(cells[i][0] - a), abs(cells[i][1] - b), abs(cells[i][0] + cells[i][1] - a - b))
                   for a, b in cells[:i]) <= K.LEGAL_RADIUS


def test_positions_are_deterministic():
    a = P.disk_batch(4, 9, 20, 4)
    b = P.disk_batch(4, 9, 20, 4)
    for k in a:
        assert torch.equal(a[k], b[k])


def test_collate_padding_convention():
    rows = [P.support_position(1, i, 6, 4)[:2] for i in range(3)]
    batch = F.collate_rows(rows)
    npad = batch["feats"].shape[1]
    for g, (sup, _) in enumerate(rows):
        n = sup.num_nodes
        assert bool(batch["mask"][g, :n].all()) and not bool(batch["mask"][g, n:].any())
        assert bool((batch["nbr"][g, n:] == npad).all())
        assert float(batch["feats"][g, n:].abs().sum()) == 0.0
        assert int(batch["legal_counts"][g]) == sup.legal_count
