"""Benchmark: Shrimp-main forward_policy_value, positions/s at global batch 4096.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl native|reference] [--config NAME]

Configs: main (default), stress (config 5), smoke (config 1),
and the two kernel microbenches attn_micro (config 2, sb_offset_attention) and
conv19_micro (config 3, sb_raytap_conv).

One process per GPU (torchrun for N > 1, NCCL). The global batch is split by
position across ranks (strong scaling: the config's batch in total); weights are
built on rank 0 and broadcast once over NCCL; there is no collective in the
timed steps. Each timed step is one full forward (or one kernel call) over the
rank's shard with its inputs resident in HBM; L2 is flushed between steps
(outside the timed window). Step times are CUDA events on the launching
stream; the reported time is the max over ranks. Rank 0 prints one JSON line.

`--impl reference` times the CPU restatement of the reference path (the oracle
port, fp32 torch on the host cores) on a bounded sample of the same workload;
the native line's `cpu_baseline` is that same measurement, run in a child
process with the same arguments.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from hexo_bot_b200 import microbench  # noqa: E402
from hexo_bot_b200.microbench import disk_cells  # noqa: E402

FORWARD_CONFIGS = {
    "main": dict(channels=128, attention_heads=8, trunk_layout="CCACCACCACCA", seed=0, disk=4, plies=60,
                 batch=4096, mflop=321.7, cpu_sample=256),
    "stress": dict(channels=192, attention_heads=12, trunk_layout="CCACCACCACCA", seed=1, disk=8, plies=120,
                   batch=1024, mflop=2599.3, cpu_sample=32),
    "smoke": dict(channels=32, attention_heads=4, trunk_layout="CCA", seed=0, disk=4, plies=30, batch=64,
                  mflop=6.5, cpu_sample=64),
}
MICRO_CONFIGS = {
    "attn_micro": dict(**microbench.ATTN_MICRO, cpu_sample=512),
    "conv19_micro": dict(**microbench.CONV19_MICRO, cpu_sample=256),
}
# The serve path on the reference support (variable node counts): wire
# payloads through ShrimpEvaluator (plan_groups, device unpack, fused reply).
SERVE_CONFIGS = {
    "serve": dict(channels=128, attention_heads=8, trunk_layout="CCACCACCACCA", seed=0, radius=4, plies=60,
                  batch=256, cpu_sample=16),
}
CONFIGS = {**FORWARD_CONFIGS, **MICRO_CONFIGS, **SERVE_CONFIGS}
METRIC = "Shrimp positions/sec at batch 4096 (1/2/4/8 B200); p50 latency at batch 256"
LATENCY_BATCHES = (1, 16, 64, 256, 1024)
# DRAM bytes (read + write) of one launch of the dominant kernel, from an ncu
# capture of that launch at the named (config, per-GPU batch); shapes that were
# not captured report null.
DOMINANT_TRAFFIC_BYTES: dict[tuple[str, int], int] = {
    ("main", 4096): 83_642_368,  # conv_grid_kernel, conv1 of the main forward: 66.2 MB read + 17.4 MB written
}


def load_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "tflops": d["bf16_tflops"], "tflops_sustained": d["bf16_tflops_sustained"],
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "tflops": 1590.0, "tflops_sustained": 1400.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while active."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": max(smax) if smax else None,
            "reasons": sorted(reasons),
            "samples": len(sm),
        }


# ---- inputs -----------------------------------------------------------------------


def make_batch(cfg: dict, count: int, start: int):
    from hexo_bot_b200 import positions

    return positions.disk_batch(count, cfg["seed"], cfg["plies"], cfg["disk"], start=start)


def micro_inputs(name: str, cfg: dict, count: int, start: int) -> dict:
    from hexo_bot_b200 import microbench

    if name == "attn_micro":
        return microbench.attention_inputs(cfg, count, start)
    return microbench.conv19_inputs(cfg, count, start)


def serve_payload(cfg: dict, count: int, start: int, request_moves_left: bool = True):
    """Wire payload of seeded reference-support positions [start, start+count)."""

    from hexo_bot_b200 import payload as PL
    from hexo_bot_b200 import positions

    rows = [positions.support_position(cfg["seed"], start + i, cfg["plies"], cfg["radius"])[:2]
            for i in range(count)]
    return PL.build_payload(rows, request_moves_left=request_moves_left)[0]


def serve_mflop(payload: dict, cfg: dict) -> float:
    """Algorithmic MFLOP of the payload's forwards over the real nodes only
    (padding is waste, not work): stem, 2 convs per ConvBlock, the policy conv,
    and per AttnBlock the q/k/v/out projections, the MLP and the attention core
    over S = nodes + 8 tokens."""

    import numpy as np

    c = cfg["channels"]
    lay = cfg["trunk_layout"]
    off = np.asarray(payload["node_row_offsets"], dtype=np.float64)
    n = off[1:] - off[:-1]
    s = n + 8
    conv = 2 * n * 7 * c * c
    flops = 2 * n * 7 * 16 * c + (2 * lay.count("C") + 1) * conv
    flops = flops + lay.count("A") * (2 * s * c * 4 * c + 2 * s * c * 4 * c + 4 * s * s * c)
    return float(flops.sum()) / 1e6


def bench_config(name: str, cfg: dict, world: int) -> dict:
    """The `config` object of the JSON line; the same for both arms."""

    base = {"global_batch": cfg["batch"], "parallelism": f"position-sharded x{world}",
            "l2": "flushed (256 MB write) between timed steps"}
    if name in SERVE_CONFIGS:
        return {"workload": "ShrimpEvaluator.evaluate_payload on reference supports (wire payload in, reply out)",
                **base, "channels": cfg["channels"], "heads": cfg["attention_heads"],
                "trunk_layout": cfg["trunk_layout"], "support_radius": cfg["radius"], "plies": f"0-{cfg['plies']}",
                "grouping": "plan_groups (quant 64, waste 0.18, pair ceiling 3.8e7)"}
    n = disk_cells(cfg["disk"])
    if name in FORWARD_CONFIGS:
        return {"workload": f"{name}-size ShrimpNet.forward_policy_value", **base,
                "channels": cfg["channels"], "heads": cfg["attention_heads"], "trunk_layout": cfg["trunk_layout"],
                "cells": n, "seq_len": n + 8, "weights": "NCCL-broadcast once", "cuda_graph": True}
    if name == "attn_micro":
        return {"workload": "biased-attention microbench (sb_offset_attention)", **base, "tokens": n,
                "heads": cfg["heads"], "head_dim": cfg["head_dim"],
                "table_rows": disk_cells(cfg["table_radius"]), "dtype_io": "bf16"}
    return {"workload": "19-tap ray conv microbench (sb_raytap_conv)", **base, "cells": n,
            "channels": cfg["channels"], "taps": 19, "dtype_io": "bf16"}


def data_note(name: str, cfg: dict) -> str:
    if name in SERVE_CONFIGS:
        return (f"synthetic: seeded uniform-random legal play, 0-{cfg['plies']} plies, reference support of radius "
                f"{cfg['radius']} (variable node counts), random-init weights (seed {cfg['seed']})")
    if name in FORWARD_CONFIGS:
        return (f"synthetic: seeded uniform-random legal play on the radius-{cfg['disk']} disk, "
                f"0-{cfg['plies']} plies, random-init weights (seed {cfg['seed']})")
    return f"synthetic: seeded N(0,1) activations and seeded tables/weights (seed {cfg['seed']})"


# ---- CPU reference (both arms) --------------------------------------------------


def cpu_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def time_reference_cpu(name: str, cfg: dict, steps: int, warmup: int) -> dict:
    """The oracle port of the reference path (fp32 torch on every host thread
    this process may use) on a fixed sample of the workload: `warmup` untimed
    calls, then `steps` timed calls. One function for the reference arm and for
    the native line's cpu_baseline, so both report the same measurement."""

    from oracle import forward as oracle

    threads = cpu_threads()
    torch.set_num_threads(threads)
    sample = min(cfg["cpu_sample"], cfg["batch"])
    if name in FORWARD_CONFIGS:
        from hexo_bot_b200.model import ShrimpNet

        kw = {k: cfg[k] for k in ("channels", "attention_heads", "trunk_layout")}
        torch.manual_seed(cfg["seed"])
        sd = ShrimpNet(**kw).state_dict()
        batch = make_batch(cfg, sample, 0)
        a = (batch["feats"], batch["nbr"], batch["mask"], batch["coords"])
        call = lambda: oracle.forward_policy_value(sd, *a, heads=kw["attention_heads"], layout=kw["trunk_layout"])
        what = f"{sample} positions per call, oracle forward_policy_value (fp32 torch CPU)"
    elif name in SERVE_CONFIGS:
        from hexo_bot_b200.model import ShrimpNet
        from oracle import evaluator as oracle_eval

        kw = {k: cfg[k] for k in ("channels", "attention_heads", "trunk_layout")}
        torch.manual_seed(cfg["seed"])
        sd = ShrimpNet(**kw).state_dict()
        payload = serve_payload(cfg, sample, 0)
        call = lambda: oracle_eval.evaluate_payload(sd, payload, heads=kw["attention_heads"],  # noqa: E731
                                                    layout=kw["trunk_layout"])
        what = (f"{sample} positions per call, oracle evaluate_payload (the reference evaluator's CPU path: "
                f"plan_groups, per-group pack, fp32 torch forward, decode)")
    elif name == "attn_micro":
        m = micro_inputs(name, cfg, sample, 0)
        q, k, v = (m[x].float() for x in ("q", "k", "v"))
        call = lambda: oracle.offset_bias_attention(q, k, v, m["table"], m["offset_map"], cfg["heads"]).bfloat16()
        what = f"{sample} positions per call, oracle offset_bias_attention (fp32 torch CPU, bf16 out)"
    else:
        m = micro_inputs(name, cfg, sample, 0)
        x = m["x"].float()
        call = lambda: oracle.raytap_conv(x, m["nbr"], m["weight"].float(), m["bias"]).bfloat16()
        what = f"{sample} positions per call, oracle raytap_conv (fp32 torch CPU, bf16 out)"
    with torch.no_grad():
        for _ in range(max(warmup, 1)):
            call()
        times = []
        for _ in range(steps):
            t0 = time.perf_counter()
            call()
            times.append(time.perf_counter() - t0)
    total = sum(times)
    return {"value": sample * steps / total, "sample": sample, "threads": threads, "ms_per_call": total / steps * 1e3,
            "median_ms": statistics.median(times) * 1e3, "what": what}


def reference_line(args, name: str, cfg: dict, r: dict) -> dict:
    value = round(r["value"], 2)
    return {
        "metric": METRIC, "value": value, "unit": "positions/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(r["ms_per_call"], 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": data_note(name, cfg), "config": bench_config(name, cfg, args.gpus),
        "impl": "reference",
        "cpu_baseline": {"value": value, "unit": "positions/s", "cores": r["threads"], "kind": "port",
                         "sample": f"{r['what']}; {r['threads']} threads; median call {r['median_ms']:.1f} ms"},
        "e2e": {"value": value, "unit": "positions/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def run_reference(args, name: str, cfg: dict):
    if int(os.environ.get("RANK", "0")) != 0:
        return
    r = time_reference_cpu(name, cfg, args.steps, args.warmup)
    print(json.dumps(reference_line(args, name, cfg, r)), flush=True)


def cpu_baseline(name: str, steps: int = 10, warmup: int = 3) -> dict | None:
    """The reference arm's measurement, run as a fresh child process (no CUDA
    context, no distributed environment) so it sees the host exactly as the
    `--impl reference` run does."""

    env = {k: v for k, v in os.environ.items()
           if k not in ("RANK", "LOCAL_RANK", "WORLD_SIZE", "LOCAL_WORLD_SIZE", "MASTER_ADDR", "MASTER_PORT",
                        "GROUP_RANK", "ROLE_RANK", "TORCHELASTIC_RUN_ID")}
    env["CUDA_VISIBLE_DEVICES"] = ""
    cmd = [sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--config", name, "--steps", str(steps),
           "--warmup", str(warmup)]
    proc = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=ROOT, timeout=900)
    lines = [l for l in proc.stdout.splitlines() if l.startswith("{")]
    if proc.returncode != 0 or not lines:
        return {"value": None, "error": proc.stderr[-400:]}
    d = json.loads(lines[-1])
    cb = dict(d["cpu_baseline"])
    cb["sample"] += f"; {steps} timed calls after {warmup} warm-up (bench.py --impl reference, child process)"
    return cb


# ---- GPU timing -------------------------------------------------------------------


def flush_l2(buf: torch.Tensor):
    buf.add_(1)


def time_steps(fn, steps: int, warmup: int, flush: torch.Tensor) -> list[float]:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    out = []
    for _ in range(steps):
        flush_l2(flush)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        e.synchronize()
        out.append(s.elapsed_time(e))
    return out


def max_over_ranks(ms: float, device, world: int) -> float:
    t = torch.tensor([ms], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def build_model(cfg: dict, device, world: int):
    from hexo_bot_b200.model import ShrimpNet
    from hexo_bot_b200.sharding import broadcast_weights

    kw = {k: cfg[k] for k in ("channels", "attention_heads", "trunk_layout")}
    torch.manual_seed(cfg["seed"])
    model = ShrimpNet(**kw).to(device)
    if world > 1:
        broadcast_weights(model, src=0)  # the one NCCL collective of the run
    model.packed(device)
    return model


def e2e_serving_loop(call, host_in: list, host_out: list, make_dev_out, device, steps: int, warmup: int) -> float:
    """ms per step of a serving loop through the public call with HOST buffers:
    the H2D of step s+1's inputs and the D2H of step s's outputs run on a copy
    stream while step s computes (two device input / output sets). Every step's
    copies are inside the timed region, one event pair around all steps."""

    dev_in = [[torch.empty_like(x, device=device) for x in host_in] for _ in range(2)]
    dev_out = [make_dev_out() for _ in range(2)]
    host_o = [[torch.empty_like(x).pin_memory() for x in host_out] for _ in range(2)]
    main_st = torch.cuda.current_stream()
    copy_st = torch.cuda.Stream()

    def run(k: int) -> float:
        h2d_ev = [torch.cuda.Event() for _ in range(2)]
        fwd_ev = [torch.cuda.Event() for _ in range(2)]
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(main_st)
        copy_st.wait_stream(main_st)

        def h2d(step: int):
            b = step % 2
            with torch.cuda.stream(copy_st):
                if step >= 2:
                    copy_st.wait_event(fwd_ev[b])  # the step that last read buffer b
                for d, h in zip(dev_in[b], host_in):
                    d.copy_(h, non_blocking=True)
                h2d_ev[b].record(copy_st)

        h2d(0)
        for step in range(k):
            b = step % 2
            if step + 1 < k:
                h2d(step + 1)
            main_st.wait_event(h2d_ev[b])
            call(dev_in[b], dev_out[b])
            fwd_ev[b].record(main_st)
            with torch.cuda.stream(copy_st):
                copy_st.wait_event(fwd_ev[b])
                for h, d in zip(host_o[b], dev_out[b]):
                    h.copy_(d, non_blocking=True)
        main_st.wait_stream(copy_st)
        end.record(main_st)
        end.synchronize()
        return start.elapsed_time(end) / k

    run(warmup)
    torch.cuda.synchronize()
    return run(steps)


# ---- forward bench ----------------------------------------------------------------


def run_forward(args, name, cfg, rank, world, local, device):
    from hexo_bot_b200.model import ShrimpNet
    from hexo_bot_b200.sharding import shard_range

    total = cfg["batch"]
    lo, hi = shard_range(total, rank, world)
    shard = hi - lo
    host = make_batch(cfg, shard, lo)
    model = build_model(cfg, device, world)
    npad = host["feats"].shape[1]
    dev_in = [host[k].to(device) for k in ("feats", "nbr", "mask", "coords")]
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=device)
    if args.kernel == "conv":
        r = conv_roofline(model, dev_in, name, cfg, shard, npad, device, flush, steps=args.steps, warmup=args.warmup)
        if rank == 0:
            print(json.dumps({"kernel_only": r}), flush=True)
        return
    out = {
        "policy": torch.empty(shard, npad, dtype=torch.float32, device=device),
        "value": torch.empty(shard, 65, dtype=torch.float32, device=device),
    }

    def fwd():
        model.forward_policy_value(*dev_in, out=out)

    # capture the whole forward once as a CUDA graph (serve mode)
    fwd()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fwd()

    sampler = ClockSampler(local) if rank == 0 else None
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    if sampler:
        sampler.start()
    times = time_steps(graph.replay, args.steps, args.warmup, flush)
    clocks = sampler.stop() if sampler else None
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms_max = max_over_ranks(statistics.mean(times), device, world)
    value = total / (ms_max / 1e3)

    # ---- end to end: pinned host inputs -> H2D -> forward -> D2H, every step ----
    feats_h = host["feats"].half().pin_memory()
    nbr_h = torch.where(host["nbr"] >= npad, torch.full_like(host["nbr"], 0xFFFF), host["nbr"]).to(
        torch.int32).to(torch.uint16).pin_memory()
    mask_h = host["mask"].pin_memory()
    coords_h = host["coords"].to(torch.int16).pin_memory()
    host_in = [feats_h, nbr_h, mask_h, coords_h]
    host_out = [torch.empty(shard, npad, dtype=torch.float32), torch.empty(shard, 65, dtype=torch.float32)]

    def e2e_call(d_in, d_out):
        model.forward_policy_value(*d_in, out={"policy": d_out[0], "value": d_out[1]})

    def e2e_out():
        return [torch.empty(shard, npad, dtype=torch.float32, device=device),
                torch.empty(shard, 65, dtype=torch.float32, device=device)]

    e2e_ms = max_over_ranks(e2e_serving_loop(e2e_call, host_in, host_out, e2e_out, device, args.steps, args.warmup),
                            device, world)
    e2e_value = total / (e2e_ms / 1e3)
    h2d = sum(x.numel() * x.element_size() for x in host_in)
    d2h = sum(x.numel() * x.element_size() for x in host_out)

    roofline = None
    if rank == 0:
        roofline = conv_roofline(model, dev_in, name, cfg, shard, npad, device, flush)
    extra = {}
    if rank == 0 and world == 1 and not args.no_latency and name == "main":
        extra["latency_p50_ms"] = latency_sweep(model, cfg, device)
    cpu = cpu_baseline(name) if rank == 0 and world == 1 and not args.no_cpu_baseline else None

    if rank == 0:
        peaks = load_peaks()
        tflops = cfg["mflop"] * 1e6 * total / (ms_max / 1e3) / 1e12 / world
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "positions/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f16",
            "data": data_note(name, cfg), "config": bench_config(name, cfg, world),
            "roofline": roofline,
            "model_roofline": {
                "bound": "tensor", "achieved": round(tflops, 2), "peak": peaks["tflops_sustained"],
                "unit": "TFLOP/s per GPU", "frac": round(tflops / peaks["tflops_sustained"], 4),
                "note": f"{cfg['mflop']} MFLOP/position algorithmic, vs sustained bf16 peak ({peaks['source']})",
            },
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_value, 1), "unit": "positions/s", "h2d_bytes_per_step": int(h2d),
                    "d2h_bytes_per_step": int(d2h),
                    "note": "public module call per step; H2D of the next step and D2H of this step on a "
                            "copy stream overlapping the forward; timed over all steps"},
            "gpu_launches": ShrimpNet.kernel_launches(
                cfg["trunk_layout"],
                grid=npad <= 81 and cfg["channels"] % 64 == 0 and cfg["channels"] <= 128 and shard >= 1024,
                channels=cfg["channels"])
            * args.steps,
            "clocks": clocks,
        }
        line.update(extra)
        print(json.dumps(line), flush=True)
    if world > 1:
        del graph
        dist.barrier()


def conv_roofline(model, dev_in, name, cfg, shard, npad, device, flush, steps=20, warmup=3) -> dict:
    """Time the trunk's 7-tap conv (conv + LN + ReLU epilogue, the kernel that
    carries ~70 % of the FLOPs) alone at the bench shape via the C ABI."""

    import ctypes as C

    from hexo_bot_b200 import _lib

    lib = _lib.lib()
    c = cfg["channels"]
    blk = model.conv_blocks[0]
    w = blk.conv1.weight.detach().float().contiguous()
    kpad = (7 * c + 63) // 64 * 64
    wp = torch.empty(c, kpad, dtype=torch.float16, device=device)
    st = torch.cuda.current_stream().cuda_stream
    _lib.check(lib.sb_pack_hex_conv_weight(w.data_ptr(), 7, c, c, c, wp.data_ptr(), st), "pack")
    x = torch.randn(shard, npad, c, device=device).half()
    gidx = torch.empty(shard, npad, 7, dtype=torch.int32, device=device)
    _lib.check(lib.sb_build_gather_index(dev_in[1].data_ptr(), _lib.DT_I64, shard, npad, gidx.data_ptr(), None, st),
               "gidx")
    mask = dev_in[2].to(torch.uint8)
    out = torch.empty(shard, npad, c, dtype=torch.float16, device=device)
    nb = C.c_size_t()
    lib.sb_hex_conv_workspace_bytes(shard, npad, C.byref(nb))
    plan = torch.empty(nb.value, dtype=torch.uint8, device=device)
    bias = blk.conv1.bias.detach().float().contiguous()
    lw = blk.ln1.weight.detach().float().contiguous()
    lb = blk.ln1.bias.detach().float().contiguous()
    kernel_stream = torch.cuda.current_stream()
    # the neighbour table's plan (gather rows, row mask, grid slots) is built
    # once, outside the timed region, as a trunk of convs over one table would
    lattice = C.c_int(0)
    _lib.check(lib.sb_hex_conv_plan(gidx.data_ptr(), mask.data_ptr(), shard, npad, plan.data_ptr(), nb.value,
                                    C.byref(lattice), kernel_stream.cuda_stream), "hex_conv_plan")
    kname = "conv_grid_kernel (7-tap conv on the hex grid" if lattice.value else "conv_ts_kernel (windowed 7-tap conv"

    def call():
        _lib.check(lib.sb_hex_conv_ln_planned(x.data_ptr(), plan.data_ptr(), nb.value, lattice.value, wp.data_ptr(),
                                              bias.data_ptr(), lw.data_ptr(), lb.data_ptr(), 1e-5, 1, shard, npad, c,
                                              c, out.data_ptr(), kernel_stream.cuda_stream), "conv")

    # one planned call = one launch of the conv kernel, timed by CUDA events on
    # the stream it is launched on
    times = time_steps(call, steps, warmup, flush)
    ms = statistics.mean(times)
    flops = 2.0 * shard * npad * 7 * c * c
    peaks = load_peaks()
    achieved = flops / (ms / 1e3) / 1e12
    return {
        "kernel": kname + " + LayerNorm/ReLU epilogue, the forward's first ConvBlock conv), one launch per "
                          "sb_hex_conv_ln_planned call",
        "bound": "tensor",
        "achieved": round(achieved, 2),
        "peak": peaks["tflops"],
        "unit": "TFLOP/s",
        "frac": round(achieved / peaks["tflops"], 4),
        "traffic": DOMINANT_TRAFFIC_BYTES.get((name, shard)),
        "algorithmic_flop_per_launch": flops,
        "ms_per_launch": round(ms, 4),
        "peak_source": f"bf16_tflops burst, {peaks['source']} (f16 runs at the same tensor rate)",
    }


def latency_sweep(model, cfg, device) -> dict:
    """p50 graph-replay latency of the full forward at MCTS-sized batches."""

    res = {}
    base = make_batch(cfg, max(LATENCY_BATCHES), 0)
    for b in LATENCY_BATCHES:
        ins = [base[k][:b].to(device) for k in ("feats", "nbr", "mask", "coords")]
        npad = ins[0].shape[1]
        out = {"policy": torch.empty(b, npad, device=device), "value": torch.empty(b, 65, device=device)}
        model.forward_policy_value(*ins, out=out)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            model.forward_policy_value(*ins, out=out)
        for _ in range(10):
            g.replay()
        torch.cuda.synchronize()
        ts = []
        for _ in range(200):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            g.replay()
            e.record()
            e.synchronize()
            ts.append(s.elapsed_time(e))
        res[str(b)] = round(statistics.median(ts), 4)
        del g
    return res


# ---- microbench lines -------------------------------------------------------------


def run_micro(args, name, cfg, rank, world, local, device):
    """One kernel call per step through the C ABI at the microbench shape."""

    from hexo_bot_b200 import _lib
    from hexo_bot_b200.sharding import shard_range

    lib = _lib.lib()
    total = cfg["batch"]
    lo, hi = shard_range(total, rank, world)
    shard = hi - lo
    m = micro_inputs(name, cfg, shard, lo)
    n = disk_cells(cfg["disk"])
    st = torch.cuda.current_stream()
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=device)
    peaks = load_peaks()
    if name == "attn_micro":
        h, d = cfg["heads"], cfg["head_dim"]
        table = m["table"].to(device)
        om = m["offset_map"].to(device)
        rows = table.shape[0]
        host_in = [m["q"].pin_memory(), m["k"].pin_memory(), m["v"].pin_memory()]
        dev = [x.to(device) for x in host_in]
        out = torch.empty_like(dev[0])

        def call(d_in, d_out):
            _lib.check(lib.sb_offset_attention(d_in[0].data_ptr(), d_in[1].data_ptr(), d_in[2].data_ptr(),
                                               table.data_ptr(), rows, om.data_ptr(), shard, n, h, d,
                                               d_out[0].data_ptr(), st.cuda_stream), "sb_offset_attention")

        launches = 1
        algo = 4 * shard * n * h * d * 2 + table.numel() * 4 + om.numel() * 4  # q, k, v read + out write
        bound, unit, peak = "hbm", "GB/s", peaks["hbm_gbs"]
        kname = "attn_kernel (OFFSET bias mode)"
    else:
        c = cfg["channels"]
        taps = m["nbr"].shape[1]
        nbr = m["nbr"].to(device)
        wp = m["weight"].t().contiguous().to(device)  # [Cout][taps*Cin], K-major
        bias = m["bias"].to(device)
        ws = torch.empty(shard * n * taps * 4 + 64, dtype=torch.uint8, device=device)
        host_in = [m["x"].pin_memory()]
        dev = [host_in[0].to(device)]
        out = torch.empty_like(dev[0])

        def call(d_in, d_out):
            _lib.check(lib.sb_raytap_conv(d_in[0].data_ptr(), nbr.data_ptr(), taps, wp.data_ptr(), bias.data_ptr(),
                                          shard, n, c, d_out[0].data_ptr(), ws.data_ptr(), ws.numel(),
                                          st.cuda_stream), "sb_raytap_conv")

        launches = 2
        algo = 2.0 * shard * n * taps * c * c
        bound, unit, peak = "tensor", "TFLOP/s", peaks["tflops"]
        kname = "conv_ts_kernel<bf16, heavy, 19 taps> (position-windowed ray-tap conv, bias + residual + ReLU epilogue)"

    sampler = ClockSampler(local) if rank == 0 else None
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    if sampler:
        sampler.start()
    times = time_steps(lambda: call(dev, [out]), args.steps, args.warmup, flush)
    clocks = sampler.stop() if sampler else None
    if world > 1:
        dist.barrier()
    ms_max = max_over_ranks(statistics.mean(times), device, world)
    value = total / (ms_max / 1e3)
    achieved = algo / (statistics.mean(times) / 1e3) / (1e9 if bound == "hbm" else 1e12)
    host_out = [torch.empty_like(host_in[0])]
    e2e_ms = max_over_ranks(
        e2e_serving_loop(call, host_in, host_out, lambda: [torch.empty_like(dev[0])], device, args.steps,
                         args.warmup), device, world)
    cpu = cpu_baseline(name) if rank == 0 and world == 1 and not args.no_cpu_baseline else None
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "positions/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": data_note(name, cfg), "config": bench_config(name, cfg, world),
            "roofline": {"kernel": kname, "bound": bound, "achieved": round(achieved, 2), "peak": peak, "unit": unit,
                         "frac": round(achieved / peak, 4), "traffic": None,
                         "algorithmic_per_launch": algo, "ms_per_launch": round(statistics.mean(times), 4),
                         "peak_source": peaks["source"]},
            "cpu_baseline": cpu,
            "e2e": {"value": round(total / (e2e_ms / 1e3), 1), "unit": "positions/s",
                    "h2d_bytes_per_step": int(sum(x.numel() * x.element_size() for x in host_in)),
                    "d2h_bytes_per_step": int(host_out[0].numel() * host_out[0].element_size())},
            "gpu_launches": launches * args.steps,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)


# ---- serve path -------------------------------------------------------------------


def run_serve(args, name, cfg, rank, world, local, device):
    """value: sb_evaluate_payload over the rank's payload already on the device
    (captured as one CUDA graph); e2e: ShrimpEvaluator.evaluate_payload with
    the wire payload in host memory and the reply bytes back, per step."""

    from hexo_bot_b200.evaluator import ShrimpEvaluator
    from hexo_bot_b200.model import ShrimpNet
    from hexo_bot_b200.sharding import shard_range

    total = cfg["batch"]
    lo, hi = shard_range(total, rank, world)
    payload = serve_payload(cfg, hi - lo, lo)
    model = build_model(cfg, device, world)
    ev = ShrimpEvaluator(model, device)
    ev.evaluate_payload(payload)  # warm-up: packs weights, sizes the workspace
    torch.cuda.synchronize()

    # device-resident variant of the same call: stage once, then time the
    # evaluate launch sequence alone (graph replay)
    import numpy as np

    req = ev.stage_payload(payload)
    groups = req["groups"]
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    offsets = np.asarray(payload["node_row_offsets"], dtype=np.int64)
    b = req["b"]

    def evaluate():
        ev.launch(req)

    evaluate()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        evaluate()
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=device)
    sampler = ClockSampler(local) if rank == 0 else None
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    if sampler:
        sampler.start()
    times = time_steps(graph.replay, args.steps, args.warmup, flush)
    clocks = sampler.stop() if sampler else None
    if world > 1:
        dist.barrier()
    ms_max = max_over_ranks(statistics.mean(times), device, world)
    value = total / (ms_max / 1e3)

    # end to end through the public call: payload bytes in, reply bytes out
    for _ in range(args.warmup):
        ev.evaluate_payload(payload)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    start_ev, end_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start_ev.record()
    for _ in range(args.steps):
        ev.evaluate_payload(payload)
    end_ev.record()
    end_ev.synchronize()
    e2e_ms = max_over_ranks(start_ev.elapsed_time(end_ev) / args.steps, device, world)
    h2d = req["keep"][0].numel()
    d2h = 4 * (req["n_out"] + 1)
    cpu = cpu_baseline(name) if rank == 0 and world == 1 and not args.no_cpu_baseline else None
    if rank == 0:
        peaks = load_peaks()
        mflop = serve_mflop(payload, cfg)
        tflops = mflop * 1e6 / (ms_max / 1e3) / 1e12
        sizes = offsets[1:] - offsets[:-1]
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "positions/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f16",
            "data": data_note(name, cfg), "config": bench_config(name, cfg, world),
            "roofline": None,
            "model_roofline": {"bound": "tensor", "achieved": round(tflops, 2), "peak": peaks["tflops_sustained"],
                               "unit": "TFLOP/s per GPU", "frac": round(tflops / peaks["tflops_sustained"], 4),
                               "note": f"{mflop / (hi - lo):.0f} MFLOP/position over real nodes (padding excluded)"},
            "cpu_baseline": cpu,
            "e2e": {"value": round(total / (e2e_ms / 1e3), 1), "unit": "positions/s", "h2d_bytes_per_step": int(h2d),
                    "d2h_bytes_per_step": int(d2h),
                    "note": "ShrimpEvaluator.evaluate_payload per step: host staging, plan_groups, one H2D, the "
                            "group forwards, one D2H and the reply bytes"},
            # per group the whole forward: prep_csr, tokens, stem, the trunk, policy conv, heads
            "gpu_launches": sum(ShrimpNet.kernel_launches(cfg["trunk_layout"], grid=False, channels=cfg["channels"],
                                                          pooled=ShrimpNet.pools_cells_apart(e - s, pad, sms))
                                for s, e, pad in groups) * args.steps,
            "groups": len(groups),
            "nodes": {"min": int(sizes.min()), "p50": int(np.median(sizes)), "max": int(sizes.max())},
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    del graph



def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["native", "reference"], default="native")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="main")
    ap.add_argument("--batch", type=int, default=None, help="override the global batch")
    ap.add_argument("--no-latency", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--kernel", choices=["conv"], default=None,
                    help="time only the dominant kernel at the bench shape (for profiling)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    name = args.config
    cfg = dict(CONFIGS[name])
    if args.batch:
        cfg["batch"] = args.batch

    if args.impl == "reference":
        run_reference(args, name, cfg)
        return

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    try:
        if name in FORWARD_CONFIGS:
            run_forward(args, name, cfg, rank, world, local, device)
        elif name in SERVE_CONFIGS:
            run_serve(args, name, cfg, rank, world, local, device)
        else:
            run_micro(args, name, cfg, rank, world, local, device)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
