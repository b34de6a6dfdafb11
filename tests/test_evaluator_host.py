"""Host side of the serve path, without a GPU: the native plan_groups against
the restated reference planner (inference.py:201-223), the wire-payload
builder, and the evaluator's refusal of a non-CUDA device."""

from __future__ import annotations

import random

import numpy as np
import pytest
import torch

from hexo_bot_b200 import _lib
from hexo_bot_b200 import evaluator as E
from hexo_bot_b200 import payload as PL
from oracle import evaluator as OE


def _sorted_sizes(rng, n, lo, hi):
    return sorted((rng.randint(lo, hi) for _ in range(n)), reverse=True)


@pytest.mark.parametrize("seed", range(40))
def test_native_plan_groups_matches_reference_planner(seed):
    rng = random.Random(seed)
    lo, hi = rng.choice([(7, 70), (7, 400), (300, 2500), (1, 6000), (64, 64)])
    sizes = _sorted_sizes(rng, rng.randint(1, 300), lo, hi)
    assert E.plan_groups(sizes) == OE.plan_groups(sizes)


def test_plan_groups_edge_cases():
    for sizes in ([], [7], [64], [65], [128, 128, 64, 1], [2387] * 40, [5341, 7, 7], [10] * 700):
        assert E.plan_groups(sizes) == OE.plan_groups(sizes)
    groups = E.plan_groups([2387] * 40)
    assert all((e - s) * (p + 8) ** 2 <= E.PAIR_CEILING for s, e, p in groups)


def test_plan_groups_rejects_rows_out_of_size_order():
    with pytest.raises(_lib.NativeError, match="sorted"):
        E.plan_groups([64, 300])


def test_payload_builder_sorts_rows_and_keeps_the_wire_layout():
    payload, order = PL.seeded_payload(24, 3, 40, 4, request_moves_left=True)
    b, total = payload["shape"]
    off = np.asarray(payload["node_row_offsets"])
    sizes = off[1:] - off[:-1]
    assert b == 24 and off[-1] == total and off[0] == 0
    assert list(sizes) == sorted(sizes, reverse=True)
    assert len(payload["node_feats"]) == total * 15 * 2 and len(payload["nbr"]) == total * 12
    nbr = np.frombuffer(payload["nbr"], dtype=np.uint16).reshape(total, 6)
    for r in range(b):
        rows = nbr[off[r]:off[r + 1]]
        live = rows[rows != PL.NBR_SENTINEL]
        assert (live < sizes[r]).all()
    legal = np.frombuffer(payload["legal_counts"], dtype=np.int32)
    assert (legal >= 1).all() and (legal <= sizes).all()
    assert sorted(order) == list(range(24))


def test_evaluator_refuses_a_cpu_device():
    from hexo_bot_b200.model import ShrimpNet

    with pytest.raises(RuntimeError, match="not CUDA"):
        E.ShrimpEvaluator(ShrimpNet(channels=32, attention_heads=4, trunk_layout="CCA"), "cpu")


def test_oracle_evaluator_reply_layout():
    from hexo_bot_b200.model import ShrimpNet

    torch.manual_seed(0)
    sd = ShrimpNet(channels=32, attention_heads=4, trunk_layout="CCA").state_dict()
    payload, _ = PL.seeded_payload(6, 1, 20, 4, request_moves_left=True, request_logits=True)
    reply = OE.evaluate_payload(sd, payload, heads=4, layout="CCA")
    r = PL.parse_reply(reply, payload)
    assert r["values"].shape == (6,) and np.all(np.abs(r["values"]) <= 1)
    for p, lg in zip(r["priors"], r["priors_logits"]):
        assert abs(float(p.sum()) - 1.0) < 1e-5 and p.shape == lg.shape
    assert np.all((r["moves_left"] >= 0) & (r["moves_left"] <= 209))
