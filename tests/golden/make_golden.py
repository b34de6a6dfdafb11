"""Generate the golden fixtures that pin the oracle and the featurizer to the
reference implementation itself.

Run in a container that has the reference checkout (it is not needed anywhere
else; the fixtures are committed):

    python tests/golden/make_golden.py /path/to/hexo-bot

It imports the reference's own `shrimp` package (packages/shrimp/python) and
records, on seeded synthetic inputs:

- geometry.npz   rel_bias_index over offsets [-20, 20]^2 and the model's
                 35x35 clamped-offset LUT (model.py:625-641);
- featurize.npz  reference build_support / window_scan / build_features
                 outputs for seeded positions (support.py, features.py);
- tables.pt      reference _build_pair, _build_pair_u8 and gather_idx for a
                 padded batch (model.py:677-792, 860-863);
- forward_*.pt   reference forward_policy_value outputs (fp32, CPU) for the
                 smoke, main and stress architectures, default init and
                 derandomized, plus a per-tensor checksum of the weights.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

CONFIGS = {
    "smoke": dict(channels=32, attention_heads=4, trunk_layout="CCA", seed=0, disk=4, plies=30, batch=8,
                  support_batch=4),
    "main": dict(channels=128, attention_heads=8, trunk_layout="CCACCACCACCA", seed=0, disk=4, plies=60, batch=4,
                 support_batch=2),
    "stress": dict(channels=192, attention_heads=12, trunk_layout="CCACCACCACCA", seed=1, disk=8, plies=120,
                   batch=2, support_batch=0),
}


def main(ref_root: str) -> None:
    sys.path.insert(0, str(Path(ref_root) / "packages" / "shrimp" / "python"))
    from shrimp import features as rf
    from shrimp import geometry as rg
    from shrimp import support as rs
    from shrimp.model import ShrimpNet as RefNet

    from hexo_bot_b200 import featurize as mf
    from hexo_bot_b200 import positions as P
    from oracle import forward as O

    # ---- geometry ----
    offs = np.array([[dq, dr] for dq in range(-20, 21) for dr in range(-20, 21)], dtype=np.int32)
    rows = np.array([rg.rel_bias_index(int(a), int(b)) for a, b in offs], dtype=np.int32)
    net = RefNet(channels=32, attention_heads=4, trunk_layout="CCA")
    lut = net._cell_bias_lut.numpy().astype(np.int32)
    np.savez_compressed(HERE / "geometry.npz", offsets=offs, rows=rows, lut=lut)

    # ---- featurization (reference support radius 8 and the model radius 4) ----
    recs, coords, nbr, dist, feats, counts = [], [], [], [], [], []
    import random

    for i in range(24):
        rng = random.Random(1000 + i)
        records = P.play_random(rng, rng.randint(0, 40), None)
        recs.append(np.asarray(records, dtype=np.int32).reshape(-1, 4))
        facts_m = mf.facts_from_records(records)
        wr = rf.window_scan(tuple(facts_m.records), facts_m.current_player, facts_m.placements_made)
        facts = rf.PositionFacts(
            records=facts_m.records, current_player=facts_m.current_player, phase=facts_m.phase,
            first_stone=facts_m.first_stone, own_hot=wr[0], opp_hot=wr[1], own_win=wr[2], opp_win=wr[3],
        )
        sup = rs.build_support(facts.stones())
        coords.append(sup.coords)
        nbr.append(sup.nbr)
        dist.append(sup.dist)
        feats.append(rf.build_features(facts, sup))
        counts.append([sup.legal_count, sup.stone_count, sup.halo_count])

    np.savez_compressed(
        HERE / "featurize.npz",
        rec_offsets=np.cumsum([0] + [len(r) for r in recs]),
        records=np.concatenate(recs, 0) if recs else np.zeros((0, 4), np.int32),
        node_offsets=np.cumsum([0] + [len(c) for c in coords]),
        coords=np.concatenate(coords, 0),
        nbr=np.concatenate(nbr, 0),
        dist=np.concatenate(dist, 0),
        feats=np.concatenate(feats, 0),
        counts=np.asarray(counts, dtype=np.int32),
    )

    # ---- tables ----
    tb = P.support_batch(3, 7, 6, 4)
    with torch.no_grad():
        pair, key_pad = net._build_pair(tb["coords"], tb["mask"])
        pair_u8 = net._build_pair_u8(tb["coords"], tb["mask"])
    n = tb["feats"].shape[1]
    gidx = torch.cat([torch.arange(n).reshape(1, n, 1).expand(tb["nbr"].shape[0], -1, -1), tb["nbr"]], dim=2)
    torch.save({"batch": tb, "pair": pair.to(torch.int16), "key_pad": key_pad, "pair_u8": pair_u8,
                "gather_idx": gidx.to(torch.int32)}, HERE / "tables.pt")

    # ---- forward outputs ----
    for name, cfg in CONFIGS.items():
        kw = {k: cfg[k] for k in ("channels", "attention_heads", "trunk_layout")}
        batches = {"disk": P.disk_batch(cfg["batch"], cfg["seed"], cfg["plies"], cfg["disk"])}
        if cfg["support_batch"]:
            batches["support"] = P.support_batch(cfg["support_batch"], cfg["seed"] + 100, cfg["plies"] // 2,
                                                 cfg["disk"])
        torch.manual_seed(cfg["seed"])
        ref = RefNet(**kw).eval()
        sd0 = {k: v.clone() for k, v in ref.state_dict().items()}
        record = {"config": cfg, "cases": {}}
        for mode in ("default", "derandomized"):
            sd = sd0 if mode == "default" else O.derandomize(sd0)
            ref.load_state_dict(sd)
            record[f"checksum_{mode}"] = O.state_checksum(sd)
            for bname, batch in batches.items():
                with torch.no_grad():
                    out = ref.forward_policy_value(batch["feats"], batch["nbr"], batch["mask"], batch["coords"],
                                                   request_moves_left=True)
                record["cases"][(mode, bname)] = {
                    "inputs": batch,
                    "policy": out["policy"].clone(),
                    "value": out["value"].clone(),
                    "moves_left": out["moves_left"].clone(),
                }
        torch.save(record, HERE / f"forward_{name}.pt")
        print("wrote", name, flush=True)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py /path/to/hexo-bot")
    main(sys.argv[1])
