"""Multi-rank host logic on CPU (gloo, world_size 2): position shards, the
one-time weight broadcast, and that sharded results reassemble into the
single-process forward (the oracle stands in for the GPU forward here)."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from hexo_bot_b200.sharding import shard_range


def test_shard_range_covers_exactly():
    for total in (0, 1, 7, 64, 4096, 4097):
        for world in (1, 2, 3, 4, 8):
            spans = [shard_range(total, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            for (a, b), (c, d) in zip(spans, spans[1:]):
                assert b == c
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1


def test_shard_range_rejects_bad_rank():
    with pytest.raises(ValueError):
        shard_range(10, 2, 2)
    with pytest.raises(ValueError):
        shard_range(10, 0, 0)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from hexo_bot_b200.model import ShrimpNet
        from hexo_bot_b200.positions import disk_batch
        from hexo_bot_b200.sharding import broadcast_weights, shard_range
        from oracle import forward as O

        # rank 0 holds the seeded weights; the other rank starts from different ones
        torch.manual_seed(0 if rank == 0 else 1234)
        model = ShrimpNet(channels=32, attention_heads=4, trunk_layout="CCA")
        broadcast_weights(model, src=0)
        sd = {k: v.clone() for k, v in model.state_dict().items()}
        fp = O.state_checksum(sd)
        csum = torch.tensor([sum(a + b for a, b in fp.values())], dtype=torch.float64)
        sums = [torch.zeros(1, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(sums, csum)

        total = 10
        batch = disk_batch(total, seed=3, max_plies=20, disk_radius=4)
        lo, hi = shard_range(total, rank, world)
        args = [batch[k][lo:hi] for k in ("feats", "nbr", "mask", "coords")]
        out = O.forward_policy_value(sd, *args, heads=4, layout="CCA")
        # shards differ by at most one position: pad to the largest and gather
        n_max = total // world + (1 if total % world else 0)
        pol = torch.zeros(n_max, batch["feats"].shape[1])
        val = torch.zeros(n_max, 65)
        pol[: hi - lo] = out["policy"]
        val[: hi - lo] = out["value"]
        pols = [torch.zeros_like(pol) for _ in range(world)]
        vals = [torch.zeros_like(val) for _ in range(world)]
        dist.all_gather(pols, pol)
        dist.all_gather(vals, val)
        if rank == 0:
            spans = [shard_range(total, r, world) for r in range(world)]
            pol_all = torch.cat([p[: b - a] for p, (a, b) in zip(pols, spans)])
            val_all = torch.cat([v[: b - a] for v, (a, b) in zip(vals, spans)])
            full = O.forward_policy_value(
                sd, *[batch[k] for k in ("feats", "nbr", "mask", "coords")], heads=4, layout="CCA")
            q.put((
                [float(s) for s in sums],
                float((pol_all - full["policy"]).abs().max()),
                float((val_all - full["value"]).abs().max()),
            ))
    finally:
        dist.destroy_process_group()


def test_two_rank_shards_reassemble_the_full_forward():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    sums, dpol, dval = q.get(timeout=10)
    assert sums[0] == sums[1], "weights differ after the broadcast"
    # same arithmetic per position; CPU BLAS blocking may differ with the batch size
    assert dpol <= 1e-6 and dval <= 1e-6
