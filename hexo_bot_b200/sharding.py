"""Position sharding of a leaf batch across the GPUs of one node.

Every position of a batch is independent (LayerNorm and attention never mix
positions; the reference's row-independence test is
tests/test_shrimp_model.py:167-203), so N ranks split the batch into
contiguous position ranges and run the forward with no collective in the
steady state. The only exchange is one broadcast of the weights from rank 0
when the model is built (over NCCL on GPUs, gloo in the CPU tests).
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def shard_range(total: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous position range [lo, hi) of `rank`; shard sizes differ by at most one."""

    if world <= 0 or not 0 <= rank < world or total < 0:
        raise ValueError(f"bad shard request total={total} rank={rank} world={world}")
    base, extra = divmod(total, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def broadcast_weights(module: torch.nn.Module, src: int = 0, group=None) -> None:
    """Overwrite every parameter and persistent buffer of `module` with rank
    `src`'s values: one flattened broadcast per dtype, in place."""

    tensors = [p.data for p in module.parameters()]
    tensors += [b for name, b in module.named_buffers() if name in module.state_dict()]
    by_dtype: dict[torch.dtype, list[torch.Tensor]] = {}
    for t in tensors:
        by_dtype.setdefault(t.dtype, []).append(t)
    for dtype in sorted(by_dtype, key=str):
        group_ts = by_dtype[dtype]
        flat = torch.cat([t.reshape(-1) for t in group_ts])
        dist.broadcast(flat, src=src, group=group)
        off = 0
        for t in group_ts:
            n = t.numel()
            t.copy_(flat[off:off + n].view_as(t))
            off += n
