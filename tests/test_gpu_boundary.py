"""The module called the way the reference's ShrimpEvaluator calls its model
(packages/shrimp/python/shrimp/inference.py:355-494, 914-997): an fp16 copy
with fp32 value / moves-left tops (SHRIMP_SERVE_HALF), fp16 autocast,
torch.compile(dynamic=True) around forward_policy_value, and CUDA-graph
capture per shape (_GraphCache: warm-up on a side stream, then capture into a
shared pool), including a capture that holds the very first call and a
load_state_dict between captures."""

from __future__ import annotations

import copy

import pytest
import torch

from hexo_bot_b200 import positions as P
from hexo_bot_b200.model import ShrimpNet
from oracle import forward as O

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")
MAIN = dict(channels=128, attention_heads=8, trunk_layout="CCACCACCACCA")
KEYS = ("feats", "nbr", "mask", "coords")


def model_and_sd(derandomized=True, seed=0):
    torch.manual_seed(seed)
    m = ShrimpNet(**MAIN)
    sd = m.state_dict()
    if derandomized:
        sd = O.derandomize(sd)
        m.load_state_dict(sd)
    return m.to(DEV).eval(), {k: v.clone() for k, v in sd.items()}


def inputs(batch, feats_dtype=torch.float16):
    d = [batch[k].to(DEV) for k in KEYS]
    d[0] = d[0].to(feats_dtype)
    return d


def close_to_oracle(out, sd, batch):
    ref = O.forward_policy_value(sd, batch["feats"], batch["nbr"], batch["mask"], batch["coords"],
                                 heads=MAIN["attention_heads"], layout=MAIN["trunk_layout"])
    mask = batch["mask"].bool()
    pol = ((out["policy"].float().cpu() - ref["policy"]).abs() * mask).max().item()
    dv = (O.decode_binned_value(out["value"].float().cpu()) - O.decode_binned_value(ref["value"])).abs().max().item()
    assert pol <= 2e-2 and dv <= 1e-2, (pol, dv)


def test_half_module_with_fp32_value_tops():
    model, _ = model_and_sd()
    half = copy.deepcopy(model).half().eval()
    for mod in (half.value_reduction, half.value_head, half.ml_reduction, half.moves_left_head):
        mod.float()
    batch = P.disk_batch(64, 3, 60, 4)
    out = half.forward_policy_value(*inputs(batch), request_moves_left=True)
    torch.cuda.synchronize()
    # the half module computes with its fp16-rounded weights
    sd_rounded = {k: v.float().cpu() for k, v in half.state_dict().items()}
    close_to_oracle(out, sd_rounded, batch)


def test_fp16_autocast_leaves_results_unchanged():
    model, _ = model_and_sd()
    batch = P.disk_batch(48, 4, 60, 4)
    ins = inputs(batch)
    base = model.forward_policy_value(*ins)
    with torch.autocast(device_type="cuda", dtype=torch.float16):
        auto = model.forward_policy_value(*ins)
    torch.cuda.synchronize()
    for k in base:
        assert torch.equal(base[k], auto[k]), k


def test_torch_compile_dynamic_runs_the_native_forward():
    model, _ = model_and_sd()
    fpv = torch.compile(model.forward_policy_value, dynamic=True)
    for b in (5, 33):
        ins = inputs(P.disk_batch(b, 6, 60, 4))
        got = fpv(*ins, request_moves_left=True)
        want = model.forward_policy_value(*ins, request_moves_left=True)
        torch.cuda.synchronize()
        for k in want:
            assert torch.equal(got[k], want[k]), k


def test_graph_capture_holding_the_first_call():
    """No warm-up: the capture records the weight packing too. The replay and
    an eager call made after the capture both give the eager results."""
    model, sd = model_and_sd()
    batch = P.disk_batch(40, 7, 60, 4)
    ins = inputs(batch)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        static_out = model.forward_policy_value(*ins)
    graph.replay()
    torch.cuda.synchronize()
    replayed = {k: v.clone() for k, v in static_out.items()}
    eager = model.forward_policy_value(*ins)
    torch.cuda.synchronize()
    for k in eager:
        assert torch.equal(replayed[k], eager[k]), k
    close_to_oracle(eager, sd, batch)


def _capture(model, bb, npad, pool):
    """The reference _GraphCache._capture: static inputs in the pad-row
    convention, three warm-up calls on a side stream, capture on the current
    stream into a shared pool."""
    static_in = [torch.zeros(bb, npad, 15, dtype=torch.float16, device=DEV),
                 torch.full((bb, npad, 6), npad, dtype=torch.int64, device=DEV),
                 torch.zeros(bb, npad, dtype=torch.bool, device=DEV),
                 torch.zeros(bb, npad, 2, dtype=torch.int64, device=DEV)]
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):
            with torch.autocast(device_type="cuda", dtype=torch.float16):
                model.forward_policy_value(*static_in)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, pool=pool):
        with torch.autocast(device_type="cuda", dtype=torch.float16):
            static_out = model.forward_policy_value(*static_in)
    return graph, static_in, static_out


def _replay(entry, batch):
    graph, static_in, static_out = entry
    g = batch["feats"].shape[0]
    for dst, src in zip(static_in, inputs(batch)):
        dst[:g].copy_(src)
    graph.replay()
    torch.cuda.synchronize()
    return {k: v[:g].clone() for k, v in static_out.items()}


def test_reference_graph_cache_flow_and_load_state_dict_between_captures():
    model, sd_a = model_and_sd(derandomized=False, seed=0)
    pool = torch.cuda.graph_pool_handle()
    batch = P.disk_batch(12, 8, 60, 4)
    g1 = _capture(model, 16, 61, pool)
    close_to_oracle(_replay(g1, batch), sd_a, batch)
    # new weights between captures (in-place copy into the same parameters)
    torch.manual_seed(5)
    sd_b = O.derandomize(ShrimpNet(**MAIN).state_dict(), seed=13)
    model.load_state_dict(sd_b)
    g2 = _capture(model, 20, 61, pool)
    close_to_oracle(_replay(g2, batch), sd_b, batch)
    # the graph captured before the load reads the re-packed weights
    close_to_oracle(_replay(g1, batch), sd_b, batch)
    close_to_oracle(model.forward_policy_value(*inputs(batch)), sd_b, batch)
