"""ShrimpEvaluator: the serve entry the reference's Rust search calls, on B200.

Mirrors the reference evaluator's interface (packages/shrimp/python/shrimp/
inference.py:355-863): ``ShrimpEvaluator(model, device)``, ``__call__`` /
``evaluate_payload(payload) -> reply``, and the async split
``submit_payload(payload) -> handle`` (enqueue only) + ``result(handle) ->
reply`` (the one device-to-host synchronisation). Payload and reply follow the
wire ABI 1 (payload.rs:108-158 / inference.py:807-863): rows sorted by node
count, CSR over support nodes; reply ``values_bytes``, ``priors_bytes`` and,
on request, ``moves_left_bytes`` and ``priors_logits_bytes``.

What runs where:

- host: the payload's byte buffers are copied into one pinned staging buffer
  (no per-row pack loop) and the rows are grouped by `plan_groups` (the
  reference's padding-aware planner, run natively by ``sb_plan_groups``);
- device: one host-to-device copy of the staging buffer, then
  ``sb_evaluate_payload`` unpacks every group's rows from the CSR on the GPU,
  runs the forward with dead key / query tiles skipped per position, and the
  heads kernel writes the reply arrays (decoded value and moves-left, the
  legal-prefix priors and raw logits, flat in row order); one device-to-host
  copy of the reply.

There is no CPU path: a non-CUDA device raises.
"""

from __future__ import annotations

import ctypes as C
import os

import numpy as np
import torch

from . import _lib
from . import constants as K

# Grouping constants of the reference evaluator (inference.py:25-43).
QUANT_NODES = 64
WASTE_FRACTION = float(os.environ.get("SHRIMP_WASTE_FRACTION", 0) or 0.18)
PAIR_CEILING = float(os.environ.get("SHRIMP_PAIR_CEILING", 0) or 3.8e7)
NBR_SENTINEL = 0xFFFF


def _groups_from_offsets(offsets: np.ndarray) -> tuple[list, object]:
    b = int(offsets.shape[0]) - 1
    arr = (_lib.Group * max(b, 1))()
    n = C.c_int(0)
    off = np.ascontiguousarray(offsets, dtype=np.int64)
    _lib.check(_lib.lib().sb_plan_groups(off.ctypes.data, b, QUANT_NODES, WASTE_FRACTION, PAIR_CEILING, arr,
                                         C.byref(n)), "sb_plan_groups")
    return [(arr[i].start, arr[i].end, arr[i].pad_to) for i in range(n.value)], (arr, n.value)


def plan_groups(sizes) -> list[tuple[int, int, int]]:
    """(start, end, pad_to) groups over rows sorted by size, largest first
    (inference.py:201-223), planned by the native library."""

    sizes = np.asarray(sizes, dtype=np.int64)
    offsets = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)
    return _groups_from_offsets(offsets)[0]


def _align16(n: int) -> int:
    return (n + 15) // 16 * 16


class ShrimpEvaluator:
    """Batched leaf evaluation of a ShrimpNet over wire payloads."""

    def __init__(self, model, device: torch.device | str = "cuda") -> None:
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise RuntimeError(f"ShrimpEvaluator: device {self.device} is not CUDA; the B200 build has no CPU path")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.model = model.to(self.device).eval()
        self._workspace: torch.Tensor | None = None
        self._retired: list = []

    def __call__(self, payload: dict) -> dict:
        return self.evaluate_payload(payload)

    @torch.no_grad()
    def evaluate_payload(self, payload: dict) -> dict:
        """Synchronous serve: submit_payload followed by result."""

        return self.result(self.submit_payload(payload))

    def _workspace_bytes(self, nbytes: int) -> torch.Tensor:
        ws = self._workspace
        if ws is None or ws.numel() < nbytes:
            # a graph captured around `launch` keeps the old address: retire,
            # never free (growth by >= 1.5x bounds the retired bytes)
            if ws is not None:
                self._retired.append(ws)
            ws = torch.empty(max(nbytes, 1 if ws is None else int(ws.numel() * 1.5)), dtype=torch.uint8,
                             device=self.device)
            self._workspace = ws
        return ws

    @torch.no_grad()
    def stage_payload(self, payload: dict) -> dict:
        """Check the request, copy its buffers to the device (one pinned
        staging buffer, one H2D on the current stream), plan its groups and
        allocate its device reply. The returned request is what `launch`
        evaluates; it can be launched again (e.g. captured in a CUDA graph)."""

        if int(payload["abi"]) != 1:
            raise ValueError(f"unsupported shrimp ABI {payload['abi']}")
        b, total = (int(x) for x in payload["shape"])
        offsets = np.asarray(payload["node_row_offsets"], dtype=np.int64)
        if offsets.shape[0] != b + 1 or int(offsets[-1]) != total:
            raise ValueError("node_row_offsets inconsistent with shape")
        legal = np.frombuffer(payload["legal_counts"], dtype=np.int32)
        if legal.shape[0] != b:
            raise ValueError("legal_counts byte count mismatch")
        feats = np.frombuffer(payload["node_feats"], dtype=np.uint8)
        if feats.shape[0] != total * K.NUM_FEATURES * 2:
            raise ValueError("node_feats byte count mismatch")
        qr = np.frombuffer(payload["node_qr"], dtype=np.uint8)
        nbr = np.frombuffer(payload["nbr"], dtype=np.uint8)
        if qr.shape[0] != total * 4 or nbr.shape[0] != total * 12:
            raise ValueError("node_qr / nbr byte count mismatch")
        request_ml = bool(payload.get("request_moves_left", False))
        request_logits = bool(payload.get("request_logits", False))
        prior_offs = np.zeros(b, dtype=np.int64)
        if b > 1:
            np.cumsum(legal[:-1], out=prior_offs[1:])
        n_priors = int(legal.astype(np.int64).sum())

        # one pinned staging buffer: feats | qr | nbr | offsets | legal | prior offsets
        pieces = [feats, qr, nbr, offsets.view(np.uint8), legal.view(np.uint8), prior_offs.view(np.uint8)]
        starts, pos = [], 0
        for p in pieces:
            starts.append(pos)
            pos = _align16(pos + p.shape[0])
        staging = torch.empty(max(pos, 16), dtype=torch.uint8, pin_memory=True)
        host = staging.numpy()
        for p, o in zip(pieces, starts):
            host[o:o + p.shape[0]] = p
        dev_in = staging.to(self.device, non_blocking=True)
        base = dev_in.data_ptr()

        # reply: values | priors | moves_left | priors_logits (f32), then the status word
        n_out = b + n_priors + (b if request_ml else 0) + (n_priors if request_logits else 0)
        dev_out = torch.empty(n_out + 1, dtype=torch.float32, device=self.device)
        ptr = dev_out.data_ptr()
        reply = _lib.Reply(ptr, ptr + 4 * b, ptr + 4 * (b + n_priors) if request_ml else None,
                           ptr + 4 * (b + n_priors + (b if request_ml else 0)) if request_logits else None,
                           ptr + 4 * n_out)
        req = {"b": b, "n_priors": n_priors, "n_out": n_out, "request_ml": request_ml,
               "request_logits": request_logits, "reply": reply, "dev_out": dev_out,
               "keep": (staging, dev_in), "groups": None}
        if b > 0:
            groups, (garr, ng) = _groups_from_offsets(offsets)
            req["groups"] = groups
            req["garr"], req["ng"] = garr, ng
            req["payload"] = _lib.Payload(base + starts[0], _lib.DT_F16, base + starts[1], base + starts[2],
                                          base + starts[3], base + starts[4], base + starts[5], b)
            net = self.model.packed(self.device).net
            nbytes = C.c_size_t(0)
            _lib.check(_lib.lib().sb_evaluate_workspace_bytes(C.byref(net), garr, ng, C.byref(nbytes)),
                       "sb_evaluate_workspace_bytes")
            self._workspace_bytes(nbytes.value)
        return req

    def launch(self, req: dict) -> None:
        """Enqueue the staged request's forwards and reply on the current stream
        (clears its status word first)."""

        req["dev_out"][req["n_out"]:].zero_()
        if req["b"] == 0:
            return
        net = self.model.packed(self.device).net
        ws = self._workspace
        stream = torch.cuda.current_stream(self.device).cuda_stream
        _lib.check(_lib.lib().sb_evaluate_payload(C.byref(net), C.byref(req["payload"]), req["garr"], req["ng"],
                                                  C.byref(req["reply"]), ws.data_ptr(), ws.numel(), stream),
                   "sb_evaluate_payload")

    @torch.no_grad()
    def submit_payload(self, payload: dict) -> dict:
        """Parse the request and enqueue its forwards without synchronising;
        returns the handle `result` reads."""

        req = self.stage_payload(payload)
        self.launch(req)
        host_out = torch.empty(req["n_out"] + 1, dtype=torch.float32, pin_memory=True)
        host_out.copy_(req["dev_out"], non_blocking=True)
        done = torch.cuda.Event()
        done.record(torch.cuda.current_stream(self.device))
        return {"b": req["b"], "n_priors": req["n_priors"], "request_ml": req["request_ml"],
                "request_logits": req["request_logits"], "host_out": host_out, "event": done, "keep": req}

    @torch.no_grad()
    def result(self, handle: dict) -> dict:
        """Wait for the handle's forwards and return the reply bytes."""

        handle["event"].synchronize()
        out = handle["host_out"].numpy()
        b, p = handle["b"], handle["n_priors"]
        status = int(out[-1:].view(np.int32)[0])
        if status:
            raise RuntimeError(f"shrimp_b200 evaluate: device status {status:#x} (1 = bounded wait timed out, "
                               "2 = neighbour index out of range, 4 = row larger than its group)")
        reply = {"values_bytes": out[:b].tobytes(), "priors_bytes": out[b:b + p].tobytes()}
        o = b + p
        if handle["request_ml"]:
            reply["moves_left_bytes"] = out[o:o + b].tobytes()
            o += b
        if handle["request_logits"]:
            reply["priors_logits_bytes"] = out[o:o + p].tobytes()
        return reply


__all__ = ["ShrimpEvaluator", "plan_groups", "QUANT_NODES", "WASTE_FRACTION", "PAIR_CEILING"]
