"""Benchmark: Shrimp-main forward_policy_value, positions/s at global batch 4096.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl native|reference] [--config main|stress|...]

One process per GPU (torchrun for N > 1, NCCL). The global batch is split by
position across ranks (strong scaling: 4096 positions in total); weights are
built on rank 0 and broadcast once over NCCL; there is no collective in the
timed steps. Each timed step is one full forward over the rank's shard with its
inputs resident in HBM; L2 is flushed between steps (outside the timed
window). Step times are CUDA events on the launching stream; the reported time
is the max over ranks. Rank 0 prints one JSON line.

`--impl reference` times the CPU restatement of the reference forward on the
host cores instead (the reference is Python/PyTorch; no GPU is used).
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

CONFIGS = {
    "main": dict(channels=128, attention_heads=8, trunk_layout="CCACCACCACCA", seed=0, disk=4, plies=60,
                 batch=4096, mflop=321.7),
    "stress": dict(channels=192, attention_heads=12, trunk_layout="CCACCACCACCA", seed=1, disk=8, plies=120,
                   batch=1024, mflop=2599.3),
    "smoke": dict(channels=32, attention_heads=4, trunk_layout="CCA", seed=0, disk=4, plies=30, batch=64,
                  mflop=6.5),
}
METRIC = "Shrimp positions/sec at batch 4096 (1/2/4/8 B200); p50 latency at batch 256"
LATENCY_BATCHES = (1, 16, 64, 256, 1024)
# dram bytes (read + write) of one dominant-kernel launch at the bench shape,
# from the committed ncu capture (profiles/conv_ts_main.md); None until captured.
DOMINANT_TRAFFIC_BYTES = 94_057_984


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


def make_batch(cfg: dict, count: int, start: int):
    from hexo_bot_b200 import positions

    return positions.disk_batch(count, cfg["seed"], cfg["plies"], cfg["disk"], start=start)


def build_model(cfg: dict, device, rank: int, world: int):
    from hexo_bot_b200.model import ShrimpNet
    from hexo_bot_b200.sharding import broadcast_weights

    kw = {k: cfg[k] for k in ("channels", "attention_heads", "trunk_layout")}
    torch.manual_seed(cfg["seed"])
    model = ShrimpNet(**kw).to(device)
    if world > 1:
        broadcast_weights(model, src=0)  # the one NCCL collective of the run
    model.packed(device)
    return model


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


def cpu_baseline(cfg: dict, budget_s: float = 12.0) -> dict:
    """The CPU restatement of the reference forward (fp32, all host threads) on
    a bounded sample of the workload."""

    from oracle import forward as oracle
    from hexo_bot_b200.model import ShrimpNet

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    kw = {k: cfg[k] for k in ("channels", "attention_heads", "trunk_layout")}
    torch.manual_seed(cfg["seed"])
    sd = ShrimpNet(**kw).state_dict()
    sample = 256 if cfg["batch"] >= 256 else cfg["batch"]
    batch = make_batch(cfg, sample, 0)
    args = (batch["feats"], batch["nbr"], batch["mask"], batch["coords"])
    oracle.forward_policy_value(sd, *args, heads=kw["attention_heads"], layout=kw["trunk_layout"])
    times = []
    t_end = time.perf_counter() + budget_s
    while time.perf_counter() < t_end or len(times) < 3:
        t0 = time.perf_counter()
        oracle.forward_policy_value(sd, *args, heads=kw["attention_heads"], layout=kw["trunk_layout"])
        times.append(time.perf_counter() - t0)
        if len(times) >= 50:
            break
    med = statistics.median(times)
    return {
        "value": round(sample / med, 2),
        "unit": "positions/s",
        "cores": threads,
        "kind": "port",
        "sample": f"{sample} positions of the same workload per call, median of {len(times)} calls "
                  f"({med * 1e3:.0f} ms each), fp32 torch CPU",
    }


def run_reference(args, cfg):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    from oracle import forward as oracle
    from hexo_bot_b200.model import ShrimpNet

    kw = {k: cfg[k] for k in ("channels", "attention_heads", "trunk_layout")}
    torch.manual_seed(cfg["seed"])
    sd = ShrimpNet(**kw).state_dict()
    sample = 128 if cfg["batch"] >= 128 else cfg["batch"]
    batch = make_batch(cfg, sample, 0)
    a = (batch["feats"], batch["nbr"], batch["mask"], batch["coords"])
    call = lambda: oracle.forward_policy_value(sd, *a, heads=kw["attention_heads"], layout=kw["trunk_layout"])
    for _ in range(args.warmup):
        call()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        call()
        times.append(time.perf_counter() - t0)
    total = sum(times)
    value = sample * args.steps / total
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "positions/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(total / args.steps * 1e3, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": f"synthetic: seeded uniform-random legal play on the radius-{cfg['disk']} disk, "
                f"0-{cfg['plies']} plies, random-init weights (seed {cfg['seed']})",
        "config": {"workload": f"{args.config} forward_policy_value (CPU reference restatement)",
                   "global_batch": cfg["batch"], "sample_per_step": sample},
        "impl": "reference",
        "cpu_baseline": {"value": round(value, 2), "unit": "positions/s", "cores": threads, "kind": "port",
                         "sample": f"{sample} positions per step, fp32 torch CPU, {threads} threads"},
        "e2e": {"value": round(value, 2), "unit": "positions/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


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
    cfg = dict(CONFIGS[args.config])
    if args.batch:
        cfg["batch"] = args.batch

    if args.impl == "reference":
        run_reference(args, cfg)
        return

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)

    from hexo_bot_b200 import _lib
    from hexo_bot_b200.model import ShrimpNet

    total = cfg["batch"]
    from hexo_bot_b200.sharding import shard_range

    lo, hi = shard_range(total, rank, world)
    shard = hi - lo
    host = make_batch(cfg, shard, lo)
    model = build_model(cfg, device, rank, world)
    npad = host["feats"].shape[1]
    dev_in = [host[k].to(device) for k in ("feats", "nbr", "mask", "coords")]
    if args.kernel == "conv":
        flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=device)
        r = conv_roofline(model, dev_in, cfg, shard, npad, device, flush, steps=args.steps, warmup=args.warmup)
        if rank == 0:
            print(json.dumps({"kernel_only": r}), flush=True)
        return
    out = {
        "policy": torch.empty(shard, npad, dtype=torch.float32, device=device),
        "value": torch.empty(shard, 65, dtype=torch.float32, device=device),
    }
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=device)

    def fwd():
        model.forward_policy_value(*dev_in, out=out)

    # capture the whole forward once as a CUDA graph (serve mode)
    fwd()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fwd()
    step = graph.replay

    sampler = ClockSampler(local) if rank == 0 else None
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    if sampler:
        sampler.start()
    times = time_steps(step, args.steps, args.warmup, flush)
    clocks = sampler.stop() if sampler else None
    torch.cuda.synchronize()
    ms = statistics.mean(times)
    t = torch.tensor([ms], device=device, dtype=torch.float64)
    if world > 1:
        dist.barrier()
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    value = total / (ms_max / 1e3)

    # ---- end to end: pinned host inputs -> H2D -> forward -> D2H, every step ----
    # A serving loop: the copies of step s+1's inputs and of step s's outputs
    # run on a copy stream while the forward of step s runs (two device input
    # and output sets). Every step's H2D and D2H is inside the timed region,
    # which spans all K steps (one event pair around the loop, no L2 flush:
    # each step's inputs arrive from the host and the forward's working set,
    # ~1.3 GB at B=4096, is larger than L2).
    feats_h = host["feats"].half().pin_memory()
    nbr_h = torch.where(host["nbr"] >= npad, torch.full_like(host["nbr"], 0xFFFF), host["nbr"]).to(
        torch.int32).to(torch.uint16).pin_memory()
    mask_h = host["mask"].pin_memory()
    coords_h = host["coords"].to(torch.int16).pin_memory()
    host_in = (feats_h, nbr_h, mask_h, coords_h)
    e2e_in = [[torch.empty_like(x, device=device) for x in host_in] for _ in range(2)]
    e2e_out = [{"policy": torch.empty(shard, npad, dtype=torch.float32, device=device),
                "value": torch.empty(shard, 65, dtype=torch.float32, device=device)} for _ in range(2)]
    pol_h = [torch.empty(shard, npad, dtype=torch.float32).pin_memory() for _ in range(2)]
    val_h = [torch.empty(shard, 65, dtype=torch.float32).pin_memory() for _ in range(2)]
    main_st = torch.cuda.current_stream()
    copy_st = torch.cuda.Stream()

    def e2e_run(k: int) -> float:
        h2d_ev = [torch.cuda.Event() for _ in range(2)]
        fwd_ev = [torch.cuda.Event() for _ in range(2)]
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(main_st)
        copy_st.wait_stream(main_st)

        def h2d(step: int):
            b = step % 2
            with torch.cuda.stream(copy_st):
                if step >= 2:
                    copy_st.wait_event(fwd_ev[b])  # the forward that last read buffer b
                for d, h in zip(e2e_in[b], host_in):
                    d.copy_(h, non_blocking=True)
                h2d_ev[b].record(copy_st)

        h2d(0)
        for step in range(k):
            b = step % 2
            if step + 1 < k:
                h2d(step + 1)
            main_st.wait_event(h2d_ev[b])
            model.forward_policy_value(*e2e_in[b], out=e2e_out[b])
            fwd_ev[b].record(main_st)
            with torch.cuda.stream(copy_st):
                copy_st.wait_event(fwd_ev[b])
                pol_h[b].copy_(e2e_out[b]["policy"], non_blocking=True)
                val_h[b].copy_(e2e_out[b]["value"], non_blocking=True)
        main_st.wait_stream(copy_st)
        end.record(main_st)
        end.synchronize()
        return start.elapsed_time(end) / k

    e2e_run(args.warmup)
    torch.cuda.synchronize()
    t2 = torch.tensor([e2e_run(args.steps)], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t2, op=dist.ReduceOp.MAX)
    e2e_value = total / (float(t2.item()) / 1e3)
    h2d = sum(x.numel() * x.element_size() for x in host_in)
    d2h = pol_h[0].numel() * 4 + val_h[0].numel() * 4

    # ---- dominant kernel: the ConvBlock gather-GEMM at the bench shape ----
    roofline = None
    if rank == 0:
        roofline = conv_roofline(model, dev_in, cfg, shard, npad, device, flush)

    extra = {}
    if rank == 0 and world == 1 and not args.no_latency and args.config == "main":
        extra["latency_p50_ms"] = latency_sweep(model, cfg, device)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(cfg)

    if rank == 0:
        launches = ShrimpNet.kernel_launches(cfg["trunk_layout"]) * args.steps
        line = {
            "metric": METRIC,
            "value": round(value, 1),
            "unit": "positions/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_max, 4),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "f16",
            "data": f"synthetic: seeded uniform-random legal play on the radius-{cfg['disk']} disk, "
                    f"0-{cfg['plies']} plies, random-init weights (seed {cfg['seed']})",
            "config": {
                "workload": f"{args.config}-size ShrimpNet.forward_policy_value",
                "global_batch": total,
                "channels": cfg["channels"],
                "heads": cfg["attention_heads"],
                "trunk_layout": cfg["trunk_layout"],
                "cells": npad,
                "seq_len": npad + 8,
                "parallelism": f"position-sharded x{world}, weights NCCL-broadcast once",
                "l2": "flushed (256 MB write) between timed steps",
                "cuda_graph": True,
            },
            "roofline": roofline,
            "model_roofline": {
                "bound": "tensor",
                "achieved": round(cfg["mflop"] * 1e6 * total / (ms_max / 1e3) / 1e12 / world, 2),
                "peak": load_peaks()["tflops_sustained"],
                "unit": "TFLOP/s per GPU",
                "frac": round(cfg["mflop"] * 1e6 * total / (ms_max / 1e3) / 1e12 / world
                              / load_peaks()["tflops_sustained"], 4),
                "note": f"{cfg['mflop']} MFLOP/position algorithmic, vs sustained bf16 peak "
                        f"({load_peaks()['source']})",
            },
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_value, 1), "unit": "positions/s", "h2d_bytes_per_step": int(h2d),
                    "d2h_bytes_per_step": int(d2h),
                    "note": "public module call per step; H2D of the next step and D2H of this step on a "
                            "copy stream overlapping the forward; timed over all steps"},
            "gpu_launches": launches,
            "clocks": clocks,
        }
        line.update(extra)
        print(json.dumps(line), flush=True)
    if world > 1:
        del graph
        dist.barrier()
        dist.destroy_process_group()


def conv_roofline(model, dev_in, cfg, shard, npad, device, flush, steps=20, warmup=3) -> dict:
    """Time the trunk's gather-GEMM conv (conv + LN + ReLU epilogue, the kernel
    that carries ~70 % of the FLOPs) alone at the bench shape via the C ABI."""

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
    ws = torch.empty(nb.value, dtype=torch.uint8, device=device)
    bias = blk.conv1.bias.detach().float().contiguous()
    lw = blk.ln1.weight.detach().float().contiguous()
    lb = blk.ln1.bias.detach().float().contiguous()

    def call():
        _lib.check(lib.sb_hex_conv_ln(x.data_ptr(), gidx.data_ptr(), mask.data_ptr(), wp.data_ptr(), bias.data_ptr(),
                                      lw.data_ptr(), lb.data_ptr(), 1e-5, 1, shard, npad, c, c, out.data_ptr(),
                                      ws.data_ptr(), nb.value, torch.cuda.current_stream().cuda_stream), "conv")

    times = time_steps(call, steps, warmup, flush)
    ms = statistics.mean(times)
    flops = 2.0 * shard * npad * 7 * c * c
    peaks = load_peaks()
    achieved = flops / (ms / 1e3) / 1e12
    return {
        "kernel": "conv_ts_kernel (position-windowed 7-tap conv + LayerNorm/ReLU epilogue), timed via sb_hex_conv_ln",
        "bound": "tensor",
        "achieved": round(achieved, 2),
        "peak": peaks["tflops"],
        "unit": "TFLOP/s",
        "frac": round(achieved / peaks["tflops"], 4),
        "traffic": DOMINANT_TRAFFIC_BYTES,
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


if __name__ == "__main__":
    main()
