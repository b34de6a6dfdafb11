"""The evaluator's wire payload (abi 1), built on the host from featurized rows.

The reference's Rust search featurizes every leaf state, sorts the rows by
node count (largest first, stable by request index) and concatenates them
into one CSR request dict (packages/shrimp/rust/src/payload.rs:53-158):

    abi                1
    shape              (B, total_nodes)
    node_feats         f16 bytes, (total_nodes, 15)
    node_qr            i16 bytes, (total_nodes, 2) axial coordinates
    node_row_offsets   list of B + 1 ints (first node of each row)
    nbr                u16 bytes, (total_nodes, 6) row-local, 0xFFFF = missing
    legal_counts       i32 bytes, (B,)
    request_moves_left bool
    request_logits     bool

The Rust crate cannot be built here, so this module restates that packing for
tests and benchmarks; `ShrimpEvaluator` consumes the dicts either side makes.
"""

from __future__ import annotations

import numpy as np

from . import constants as K
from . import positions

ABI_VERSION = 1
NBR_SENTINEL = 0xFFFF


def build_payload(rows, request_moves_left: bool = False, request_logits: bool = False):
    """(payload dict, order) from (Support, feats) rows in request order;
    `order[i]` is the request index of payload row i (rows sorted by node
    count, largest first, stable by request index, payload.rs:96-101)."""

    order = sorted(range(len(rows)), key=lambda i: (-rows[i][0].num_nodes, i))
    feats, qr, nbr, legal, offsets = [], [], [], [], [0]
    for i in order:
        sup, fr = rows[i]
        if sup.num_nodes > NBR_SENTINEL:
            raise ValueError(f"support of {sup.num_nodes} nodes exceeds the u16 neighbour wire limit")
        feats.append(np.asarray(fr, dtype=np.float32).astype(np.float16))
        qr.append(sup.coords.astype(np.int16))
        nbr.append(np.where(sup.nbr < 0, NBR_SENTINEL, sup.nbr).astype(np.uint16))
        legal.append(sup.legal_count)
        offsets.append(offsets[-1] + sup.num_nodes)
    total = offsets[-1]
    payload = {
        "abi": ABI_VERSION,
        "shape": (len(rows), total),
        "node_feats": np.concatenate(feats).reshape(total, K.NUM_FEATURES).tobytes() if rows else b"",
        "node_qr": np.concatenate(qr).reshape(total, 2).tobytes() if rows else b"",
        "node_row_offsets": offsets,
        "nbr": np.concatenate(nbr).reshape(total, 6).tobytes() if rows else b"",
        "legal_counts": np.asarray(legal, dtype=np.int32).tobytes(),
        "request_moves_left": bool(request_moves_left),
        "request_logits": bool(request_logits),
    }
    return payload, order


def seeded_payload(batch: int, seed: int, max_plies: int, radius: int, request_moves_left: bool = False,
                   request_logits: bool = False):
    """Payload of `batch` seeded positions on the reference support (variable
    node counts), plies ~ U{0..max_plies}."""

    rows = [positions.support_position(seed, i, max_plies, radius)[:2] for i in range(batch)]
    return build_payload(rows, request_moves_left, request_logits)


def parse_reply(reply: dict, payload: dict) -> dict:
    """The reply bytes as arrays: values (B,), priors per row (list of (L_b,)),
    moves_left (B,) and priors_logits (list) when present."""

    legal = np.frombuffer(payload["legal_counts"], dtype=np.int32)
    offs = np.concatenate([[0], np.cumsum(legal)]).astype(np.int64)
    pri = np.frombuffer(reply["priors_bytes"], dtype=np.float32)
    out = {"values": np.frombuffer(reply["values_bytes"], dtype=np.float32),
           "priors": [pri[offs[i]:offs[i + 1]] for i in range(len(legal))]}
    if "moves_left_bytes" in reply:
        out["moves_left"] = np.frombuffer(reply["moves_left_bytes"], dtype=np.float32)
    if "priors_logits_bytes" in reply:
        lg = np.frombuffer(reply["priors_logits_bytes"], dtype=np.float32)
        out["priors_logits"] = [lg[offs[i]:offs[i + 1]] for i in range(len(legal))]
    return out


__all__ = ["ABI_VERSION", "NBR_SENTINEL", "build_payload", "seeded_payload", "parse_reply"]
