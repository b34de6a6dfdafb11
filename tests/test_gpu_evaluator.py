"""The serve path end to end on the GPU: ShrimpEvaluator on wire payloads of
seeded real-support positions (variable node counts, several forward groups)
against the oracle of the reference evaluator (CPU, fp32). Every call goes
through the C ABI (sb_plan_groups, sb_evaluate_payload).

Gates: decoded values max-abs <= 1e-2; raw policy logits (priors_logits)
max-abs <= 2e-2; legal-prefix prior argmax agreement >= 99.5 %, counted
tie-aware (our argmax's reference logit within 1e-3 of the reference maximum:
near-ties reorder under any rounding), and for the derandomized model exact
on every row whose reference top-2 logit gap exceeds 1e-3; moves-left
(decisions, 0..209) max-abs <= 2."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from hexo_bot_b200 import payload as PL
from hexo_bot_b200 import positions as P
from hexo_bot_b200.evaluator import ShrimpEvaluator
from hexo_bot_b200.model import ShrimpNet
from oracle import evaluator as OE
from oracle import forward as O

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")
MAIN = dict(channels=128, attention_heads=8, trunk_layout="CCACCACCACCA")
SMOKE = dict(channels=32, attention_heads=4, trunk_layout="CCA")


def model_sd(kw, seed, derandomized):
    torch.manual_seed(seed)
    m = ShrimpNet(**kw)
    sd = m.state_dict()
    if derandomized:
        sd = O.derandomize(sd)
        m.load_state_dict(sd)
    return m.to(DEV), {k: v.clone() for k, v in sd.items()}


def compare(got, want, payload, strict):
    g, w = PL.parse_reply(got, payload), PL.parse_reply(want, payload)
    assert set(got) == set(want)
    dv = float(np.abs(g["values"] - w["values"]).max())
    assert dv <= 1e-2, dv
    assert np.all(np.abs(g["values"]) <= 1.0)
    if "moves_left" in w:
        dml = float(np.abs(g["moves_left"] - w["moves_left"]).max())
        assert dml <= 2.0, dml
    exact = near = clear = clear_ok = 0
    dl = 0.0
    for i, (pg, pw) in enumerate(zip(g["priors"], w["priors"])):
        assert pg.shape == pw.shape
        assert abs(float(pg.sum()) - 1.0) < 1e-4
        a, b = int(pg.argmax()), int(pw.argmax())
        exact += a == b
        lw = w["priors_logits"][i] if "priors_logits" in w else np.log(np.maximum(pw, 1e-30))
        near += bool(lw[a] >= lw[b] - 1e-3)
        if strict and lw.shape[0] > 1:
            top2 = np.sort(lw)[-2:]
            if top2[1] - top2[0] > 1e-3:
                clear += 1
                clear_ok += a == b
        if "priors_logits" in w:
            dl = max(dl, float(np.abs(g["priors_logits"][i] - w["priors_logits"][i]).max()))
    n = len(g["priors"])
    assert dl <= 2e-2, dl
    assert near / n >= 0.995, near / n
    if strict:
        assert clear_ok == clear, (clear_ok, clear)
    return dv, dl, exact / n


@pytest.mark.parametrize("kw,seed", [(SMOKE, 0), (MAIN, 0)])
@pytest.mark.parametrize("derandomized", [False, True])
def test_evaluator_matches_reference_evaluator_on_real_supports(kw, seed, derandomized):
    model, sd = model_sd(kw, seed, derandomized)
    payload, _ = PL.seeded_payload(40, 5, 60, 4, request_moves_left=True, request_logits=True)
    ev = ShrimpEvaluator(model, DEV)
    got = ev.evaluate_payload(payload)
    want = OE.evaluate_payload(sd, payload, heads=kw["attention_heads"], layout=kw["trunk_layout"])
    dv, dl, agree = compare(got, want, payload, strict=derandomized)
    print(f"PARITY evaluator {kw['channels']} derandomized={derandomized}: value {dv:.2e}, logits {dl:.2e}, "
          f"argmax {agree:.4f}")


def test_evaluator_reply_without_optional_columns_and_async_split():
    model, sd = model_sd(MAIN, 1, True)
    ev = ShrimpEvaluator(model, DEV)
    p1, _ = PL.seeded_payload(12, 9, 30, 4)
    p2, _ = PL.seeded_payload(20, 10, 60, 4, request_logits=True)
    h1 = ev.submit_payload(p1)
    h2 = ev.submit_payload(p2)
    r2 = ev.result(h2)
    r1 = ev.result(h1)
    assert set(r1) == {"values_bytes", "priors_bytes"}
    assert set(r2) == {"values_bytes", "priors_bytes", "priors_logits_bytes"}
    assert r1 == ev.evaluate_payload(p1)
    for p, r in ((p1, r1), (p2, r2)):
        compare(r, OE.evaluate_payload(sd, p, heads=8, layout=MAIN["trunk_layout"]), p, strict=True)


def test_evaluator_agrees_with_the_module_forward():
    """The payload path (device unpack, per-position skips, fused reply) and
    the module's dense forward give the same logits for the same positions."""
    model, _ = model_sd(MAIN, 2, True)
    rows = [P.support_position(7, i, 60, 4)[:2] for i in range(16)]
    payload, order = PL.build_payload(rows, request_logits=True)
    rep = PL.parse_reply(ShrimpEvaluator(model, DEV).evaluate_payload(payload), payload)
    from hexo_bot_b200.featurize import collate_rows

    dense = collate_rows([rows[i] for i in order])
    out = model.forward_policy_value(*[dense[k].to(DEV) for k in ("feats", "nbr", "mask", "coords")])
    pol = out["policy"].cpu()
    for r in range(16):
        lc = int(dense["legal_counts"][r])
        assert float(np.abs(rep["priors_logits"][r] - pol[r, :lc].numpy()).max()) <= 2e-3
    vals = O.decode_binned_value(out["value"].cpu()).numpy()
    assert float(np.abs(rep["values"] - vals).max()) <= 1e-3


def test_evaluator_disk_positions_and_empty_board():
    """Disk-regime positions (every row 61 nodes: one group padded to 64) and
    the opening position (7 nodes, one legal cell)."""
    model, sd = model_sd(MAIN, 0, True)
    rows = [P.disk_position(0, i, 60, 4)[:2] for i in range(30)] + [P.support_position(0, 0, 0, 4)[:2]]
    payload, _ = PL.build_payload(rows, request_moves_left=True)
    got = ShrimpEvaluator(model, DEV).evaluate_payload(payload)
    compare(got, OE.evaluate_payload(sd, payload, heads=8, layout=MAIN["trunk_layout"]), payload, strict=True)


def test_evaluator_rejects_malformed_payloads():
    model, _ = model_sd(SMOKE, 0, False)
    ev = ShrimpEvaluator(model, DEV)
    payload, _ = PL.seeded_payload(4, 1, 10, 4)
    bad = dict(payload, abi=2)
    with pytest.raises(ValueError, match="ABI"):
        ev.evaluate_payload(bad)
    bad = dict(payload, node_row_offsets=payload["node_row_offsets"][:-1])
    with pytest.raises(ValueError, match="offsets"):
        ev.evaluate_payload(bad)
    bad = dict(payload, legal_counts=payload["legal_counts"][:-4])
    with pytest.raises(ValueError, match="legal_counts"):
        ev.evaluate_payload(bad)


def test_evaluator_groups_on_lanes_inside_a_cuda_graph():
    """The groups of a payload run on four stream lanes forked from and joined
    back into the caller's stream. The whole call captures into one CUDA graph
    whose replays give the eager reply bit for bit, also after the device
    reply was overwritten between replays."""
    model, _ = model_sd(MAIN, 3, True)
    payload, _ = PL.seeded_payload(40, 11, 60, 4, request_moves_left=True, request_logits=True)
    ev = ShrimpEvaluator(model, DEV)
    eager = ev.evaluate_payload(payload)
    req = ev.stage_payload(payload)
    assert req["ng"] > 4, req["ng"]  # every lane holds at least one group
    ev.launch(req)
    torch.cuda.synchronize()
    first = req["dev_out"].clone()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        ev.launch(req)
    for _ in range(2):
        req["dev_out"].fill_(float("nan"))
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(req["dev_out"], first)
    host = first.cpu().numpy()
    b, p = req["b"], req["n_priors"]
    assert host[:b].tobytes() == eager["values_bytes"]
    assert host[b:b + p].tobytes() == eager["priors_bytes"]
    assert int(host[-1:].view(np.int32)[0]) == 0
