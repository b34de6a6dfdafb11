"""CPU oracle of the reference evaluator's serve path — TEST INFRASTRUCTURE ONLY.

Restates, over the CPU oracle forward (oracle/forward.py), what the
reference's ShrimpEvaluator does with one wire payload on its default
(CSR / Python pack) path:

- plan_groups            packages/shrimp/python/shrimp/inference.py:201-223
- submit_payload checks  inference.py:509-533
- _forward_group pack    inference.py:865-897 (pad feats 0, nbr sentinel ->
                          pad_to, mask False, coords 0)
- _run_forward           inference.py:914-997 (forward_policy_value per group)
- _decode_group          inference.py:998-1042 (binned value, moves-left,
                          legal-prefix softmax, flat gather of priors / logits)
- result                 inference.py:807-863 (reply bytes)

Only tests/ and bench.py's CPU leg use it; the product path never does.
"""

from __future__ import annotations

import numpy as np
import torch

from . import forward as F

QUANT_NODES = 64
WASTE_FRACTION = 0.18
PAIR_CEILING = 3.8e7
NBR_SENTINEL = 0xFFFF
MOVES_LEFT_CAP = 209
NUM_FEATURES = 15


def ceil_quant(n: int) -> int:
    return max(QUANT_NODES, -(-int(n) // QUANT_NODES) * QUANT_NODES)


def plan_groups(sizes) -> list[tuple[int, int, int]]:
    """inference.py:201-223, restated."""

    n = len(sizes)
    groups = []
    start = 0
    while start < n:
        pad_to = ceil_quant(int(sizes[start]))
        floor = pad_to - max(QUANT_NODES, int(WASTE_FRACTION * pad_to))
        end = start + 1
        while end < n:
            if (end - start + 1) * (pad_to + F.NUM_TOKENS) ** 2 > PAIR_CEILING:
                break
            if int(sizes[end]) < floor:
                break
            end += 1
        groups.append((start, end, pad_to))
        start = end
    return groups


def decode_moves_left(logits: torch.Tensor) -> torch.Tensor:
    """losses.py:54-61: binned expectation clamped to [-1, 1], mapped to [0, 209]."""

    return (F.decode_binned_value(logits) + 1.0) * 0.5 * MOVES_LEFT_CAP


def evaluate_payload(sd: dict, payload: dict, *, heads: int, layout: str) -> dict:
    """The reply dict the reference evaluator returns for `payload`, computed
    with the fp32 CPU oracle forward."""

    if int(payload["abi"]) != 1:
        raise ValueError(f"unsupported shrimp ABI {payload['abi']}")
    b, total = (int(x) for x in payload["shape"])
    offsets = np.asarray(payload["node_row_offsets"], dtype=np.int64)
    legal = np.frombuffer(payload["legal_counts"], dtype=np.int32)
    feats = np.frombuffer(payload["node_feats"], dtype=np.float16).astype(np.float32).reshape(total, NUM_FEATURES)
    qr = np.frombuffer(payload["node_qr"], dtype=np.int16).reshape(total, 2)
    nbr = np.frombuffer(payload["nbr"], dtype=np.uint16).reshape(total, 6)
    request_ml = bool(payload.get("request_moves_left", False))
    request_logits = bool(payload.get("request_logits", False))
    sizes = offsets[1:] - offsets[:-1]
    values, mls, priors, logits_out = [], [], [], []
    for start, end, pad_to in plan_groups(sizes):
        g = end - start
        np_feats = np.zeros((g, pad_to, NUM_FEATURES), dtype=np.float32)
        np_nbr = np.full((g, pad_to, 6), pad_to, dtype=np.int64)
        np_mask = np.zeros((g, pad_to), dtype=np.bool_)
        np_coords = np.zeros((g, pad_to, 2), dtype=np.int64)
        for k in range(g):
            row = start + k
            n = int(sizes[row])
            o = int(offsets[row])
            np_feats[k, :n] = feats[o:o + n]
            rn = nbr[o:o + n].astype(np.int64)
            np_nbr[k, :n] = np.where(rn == NBR_SENTINEL, pad_to, rn)
            np_mask[k, :n] = True
            np_coords[k, :n] = qr[o:o + n].astype(np.int64)
        with torch.no_grad():
            out = F.forward_policy_value(sd, torch.from_numpy(np_feats), torch.from_numpy(np_nbr),
                                         torch.from_numpy(np_mask), torch.from_numpy(np_coords), heads=heads,
                                         layout=layout, request_moves_left=request_ml)
        values.append(F.decode_binned_value(out["value"]))
        if request_ml:
            mls.append(decode_moves_left(out["moves_left"]))
        pol = out["policy"].float()
        for k in range(g):
            lc = int(legal[start + k])
            if lc:
                priors.append(torch.softmax(pol[k, :lc], dim=0))
                logits_out.append(pol[k, :lc])
    cat = lambda xs: (torch.cat(xs) if xs else torch.zeros(0)).numpy().astype(np.float32)  # noqa: E731
    reply = {"values_bytes": cat(values).tobytes(), "priors_bytes": cat(priors).tobytes()}
    if request_ml:
        reply["moves_left_bytes"] = cat(mls).tobytes()
    if request_logits:
        reply["priors_logits_bytes"] = cat(logits_out).tobytes()
    return reply
