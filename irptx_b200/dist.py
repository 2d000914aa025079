"""One plan over several GPUs: one process per GPU (torch.distributed), each rank launching its
shard of the plan through irx_launch_shard.

How a plan splits is the library's (irx_plan_shard): contiguous unit ranges, element blocks of
a pointwise graph or a full reduction, rows of row reductions and row ops, 256-column blocks of
a matmul's C, (batch, head) pairs of attention. Only a full reduction exchanges anything: every
rank's shard writes a partial total, and one all-reduce (sum, max, min or product, the graph's
own fold) makes the whole result on every rank. The other families write disjoint parts of
their outputs, with no collective.

The reference has no counterpart: its runner launches one kernel on one GPU
(tests/gpurun.py:91-125)."""
from __future__ import annotations


def reduce_op(how: str):
    import torch.distributed as dist
    return {"sum": dist.ReduceOp.SUM, "max": dist.ReduceOp.MAX, "min": dist.ReduceOp.MIN,
            "prod": dist.ReduceOp.PRODUCT}[how]


def out_tensors(plan, args):
    """The args of ``args`` that are KIR outputs."""
    return [t for a, t in zip(plan.args, args) if a.kind == "out"]


def combine(plan, args, how: str, group=None):
    """All-reduce the outputs of ``args`` in place with the shards' combine rule (no-op for
    "none" or a single rank)."""
    import torch.distributed as dist
    if how == "none" or not dist.is_initialized() or dist.get_world_size(group) == 1:
        return
    for t in out_tensors(plan, args):
        dist.all_reduce(t, op=reduce_op(how), group=group)


def run_shard(plan, args, rank: int, world: int, group=None, stream=None):
    """Launch this rank's shard of ``plan`` over full-size ``args`` (device tensors), then
    combine the shards' partial results where the plan has any. Outputs outside this rank's
    shard are left as they were, except after a combine, which makes them whole on every rank."""
    plan.launch_shard(rank, world, args, stream)
    _, _, how = plan.shard(rank, world)
    combine(plan, args, how, group)
