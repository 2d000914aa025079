"""The multi-GPU host logic on CPU: world_size 2 over gloo.

Each rank asks the library for its shard of a plan (irx_plan_shard), computes that shard with
numpy in place of the kernel (the tests here have no GPU), and combines through
irptx_b200.dist.combine, the function the GPU path uses. Checked: the ranks' unit ranges tile
the plan exactly once, in order; a full reduction's partials combine into the whole total (sum,
mean); the families that write disjoint parts need no
collective and their parts assemble into the whole output."""
import os
import socket

import numpy as np
import pytest

WORLD = 2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, port, q):
    try:
        import datetime
        import torch
        import torch.distributed as dist
        import irptx_b200 as irx
        from irptx_b200 import dist as idist
        from irptx_b200 import kir_author as ka
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=WORLD,
                                timeout=datetime.timedelta(seconds=60))
        rng = np.random.default_rng(7)
        res = {}

        # full reductions: partials over element blocks, combined with the graph's fold
        n = 100003
        x = rng.standard_normal(n).astype(np.float32)
        # (a full maximum is not expressible: the KIR combines blocks with an atomic add, which
        # the reference allows for sums only, src/isel.c:1254-1260)
        for label, kir, fold, ref in [("sum", ka.reduce_all(n), np.sum, x.astype(np.float64).sum()),
                                      ("mean", ka.reduce_all(n, mean=True), None, x.astype(np.float64).mean())]:
            plan = irx.compile(kir)
            u0, u1, how = plan.shard(rank, WORLD)
            part = x[u0 * 8:min(u1 * 8, n)].astype(np.float64)
            if label == "mean":
                val = part.sum() / n                  # the shard's partial: its sum over the count
            else:
                val = fold(part)
            y = torch.tensor([val], dtype=torch.float64)
            outs = [torch.zeros(1)] * (len(plan.args) - 1) + [y]
            idist.combine(plan, outs, how)
            res[label] = (how, float(y.item()), float(ref))
            res[label + "_range"] = (u0, u1, plan.units())

        # disjoint families: each rank's range, no collective
        for label, kir in [("pointwise", ka.pointwise_relu_mul_affine(4099)), ("rows", ka.reduce_rows(1001, 64)),
                           ("rowop", ka.rmsnorm(77, 8192)), ("matmul", ka.matmul(256, 1000, 64)),
                           ("attention", ka.attention(3, 5, 128, 128))]:
            plan = irx.compile(kir)
            res[label] = plan.shard(rank, WORLD) + (plan.units(),)
        gathered = [None] * WORLD
        dist.all_gather_object(gathered, res)
        dist.destroy_process_group()
        q.put((rank, gathered))
    except Exception as exc:  # reported to the parent, which fails the test
        q.put((rank, repr(exc)))


@pytest.fixture(scope="module")
def ranks(irx):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    env = dict(os.environ)
    os.environ["CUDA_VISIBLE_DEVICES"] = ""
    try:
        procs = [ctx.Process(target=_rank_main, args=(r, port, q)) for r in range(WORLD)]
        for p in procs:
            p.start()
        out = dict(q.get(timeout=240) for _ in range(WORLD))
        for p in procs:
            p.join(timeout=60)
    finally:
        os.environ.clear()
        os.environ.update(env)
    for r, v in out.items():
        assert not isinstance(v, str), f"rank {r} failed: {v}"
    return out[0]


def test_full_reductions_combine(ranks):
    for rank_res in ranks:
        for label, tol in (("sum", 1e-9), ("mean", 1e-12)):
            how, got, want = rank_res[label]
            assert how == "sum"
            assert abs(got - want) <= tol * max(1.0, abs(want)), (label, got, want)


def test_ranges_tile_the_plan(ranks):
    for label in ("sum_range", "pointwise", "rows", "rowop", "matmul", "attention"):
        parts = [r[label] for r in ranks]
        units = parts[0][-1]
        assert parts[0][0] == 0 and parts[-1][1] == units
        for a, b in zip(parts, parts[1:]):
            assert a[1] == b[0]
        if label != "sum_range":
            assert all(p[2] == "none" for p in parts)


def test_single_shard_has_no_combine(irx):
    from irptx_b200 import kir_author as ka
    plan = irx.compile(ka.reduce_all(1000))
    assert plan.shard(0, 1) == (0, plan.units(), "none")
    with pytest.raises(irx.IrxError):
        plan.shard(2, 2)
