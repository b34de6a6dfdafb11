"""Pins the CPU oracle, the featurizer and the index-table math to outputs of
the reference implementation itself (fixtures from tests/golden/make_golden.py).
CPU only."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from hexo_bot_b200 import featurize as F
from hexo_bot_b200.geometry import cell_bias_lut, rel_bias_index
from hexo_bot_b200.model import ShrimpNet
from oracle import forward as O


def test_rel_bias_index_matches_reference():
    g = np.load(GOLDEN / "geometry.npz")
    mine = np.array([rel_bias_index(int(a), int(b)) for a, b in g["offsets"]])
    assert np.array_equal(mine, g["rows"])
    oracle_rows = np.array([O.rel_bias_row(int(a), int(b)) for a, b in g["offsets"][::7]])
    assert np.array_equal(oracle_rows, g["rows"][::7])


def test_cell_lut_matches_reference():
    g = np.load(GOLDEN / "geometry.npz")
    assert np.array_equal(cell_bias_lut().astype(np.int32), g["lut"])
    assert np.array_equal(O.cell_lut().astype(np.int32), g["lut"])


def test_featurizer_matches_reference():
    g = np.load(GOLDEN / "featurize.npz")
    ro, no = g["rec_offsets"], g["node_offsets"]
    for i in range(len(ro) - 1):
        records = [tuple(int(v) for v in r) for r in g["records"][ro[i]:ro[i + 1]]]
        facts = F.facts_from_records(records)
        sup = F.build_support(facts.stones(), 8)
        sl = slice(no[i], no[i + 1])
        assert np.array_equal(sup.coords, g["coords"][sl]), i
        assert np.array_equal(sup.nbr, g["nbr"][sl]), i
        assert np.array_equal(sup.dist, g["dist"][sl]), i
        assert [sup.legal_count, sup.stone_count, sup.halo_count] == g["counts"][i].tolist()
        assert np.array_equal(F.build_features(facts, sup), g["feats"][sl]), i


def test_index_tables_match_reference():
    t = torch.load(GOLDEN / "tables.pt", weights_only=False)
    batch = t["batch"]
    pair, key_live = O.build_pair(batch["coords"], batch["mask"])
    assert torch.equal(pair, t["pair"].long())
    assert torch.equal(key_live, t["key_pad"])
    assert torch.equal(O.build_pair_u8(batch["coords"], batch["mask"]), t["pair_u8"])
    assert torch.equal(O.gather_index(batch["nbr"]), t["gather_idx"].long())


@pytest.mark.parametrize("name", ["smoke", "main", "stress"])
def test_oracle_forward_matches_reference(name):
    rec = torch.load(GOLDEN / f"forward_{name}.pt", weights_only=False)
    cfg = rec["config"]
    kw = {k: cfg[k] for k in ("channels", "attention_heads", "trunk_layout")}
    torch.manual_seed(cfg["seed"])
    sd0 = ShrimpNet(**kw).state_dict()
    for mode in ("default", "derandomized"):
        sd = sd0 if mode == "default" else O.derandomize(sd0)
        assert O.state_checksum(sd) == rec[f"checksum_{mode}"], "seeded init differs from the reference"
        for (m, bname), case in rec["cases"].items():
            if m != mode:
                continue
            b = case["inputs"]
            out = O.forward_policy_value(sd, b["feats"], b["nbr"], b["mask"], b["coords"],
                                         heads=kw["attention_heads"], layout=kw["trunk_layout"],
                                         request_moves_left=True)
            for key in ("policy", "value", "moves_left"):
                diff = (out[key] - case[key]).abs().max().item()
                assert diff <= 1e-6, f"{name}/{mode}/{bname}/{key}: {diff}"


def test_decode_binned_value_properties():
    logits = torch.randn(16, 65, generator=torch.Generator().manual_seed(0)) * 3
    v = O.decode_binned_value(logits)
    assert v.shape == (16,) and bool((v.abs() <= 1).all())
    flat = O.decode_binned_value(torch.zeros(1, 65))
    assert abs(flat.item()) < 1e-6
