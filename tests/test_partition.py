"""The (batch x value-head group) partitioner and its one collective, on CPU ranks (gloo).

The per-rank work is the CPU oracle on the rank's shard (the CUDA kernels need a GPU); what is tested
here is the split, the all-reduce of the gate-parameter gradients against a single-process run, and
that a rank failing before the collective makes the others fail with an error instead of waiting.
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from quotebound_b200 import partition


def test_plans_cover_every_unit_once():
    for world in (1, 2, 4, 8):
        shards = partition.plan(B=8, Hk=16, Hv=64, world=world)
        seen = np.zeros((8, 64), int)
        for s in shards:
            seen[s.b0:s.b1, s.hv0:s.hv1] += 1
            assert (s.hv1 - s.hv0) == 4 * (s.hk1 - s.hk0)
        assert (seen == 1).all(), world
    # batch split first: whole head sets per GPU
    assert all(s.hk0 == 0 and s.hk1 == 16 for s in partition.plan(8, 16, 64, 8))
    assert partition.needs_allreduce(partition.plan(8, 16, 64, 2))
    # B < world: heads split too; B = 1 over 4 GPUs needs no collective at all
    sh = partition.plan(B=1, Hk=16, Hv=32, world=4)
    assert [(s.hk0, s.hk1) for s in sh] == [(0, 4), (4, 8), (8, 12), (12, 16)]
    assert not partition.needs_allreduce(sh)
    with pytest.raises(ValueError):
        partition.plan(B=3, Hk=16, Hv=32, world=2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gate_inputs(seed=0, B=4, T=33, Hk=4, Hv=8, Dk=32):
    gen = torch.Generator().manual_seed(seed)
    r = lambda *s: torch.randn(*s, generator=gen)
    return dict(q=r(B, T, Hk, Dk), k=r(B, T, Hk, Dk), a=r(B, T, Hv), b=r(B, T, Hv),
                A_log=torch.log(1 + 15 * torch.rand(Hv, generator=gen)), dt=0.5 * r(Hv),
                dqn=r(B, T, Hk, Dk), dkn=r(B, T, Hk, Dk), dg=r(B, T, Hv), dbeta=r(B, T, Hv))


def _shard_sums(x, s):
    from oracle import oracle
    sl = lambda t, h0, h1: t[s.b0:s.b1, :, h0:h1].numpy()
    out = oracle.gate_bwd(sl(x["q"], s.hk0, s.hk1), sl(x["k"], s.hk0, s.hk1), sl(x["a"], s.hv0, s.hv1),
                          sl(x["b"], s.hv0, s.hv1), x["A_log"][s.hv0:s.hv1].numpy(), x["dt"][s.hv0:s.hv1].numpy(),
                          sl(x["dqn"], s.hk0, s.hk1), sl(x["dkn"], s.hk0, s.hk1), sl(x["dg"], s.hv0, s.hv1),
                          sl(x["dbeta"], s.hv0, s.hv1))
    return torch.from_numpy(out[4]), torch.from_numpy(out[5])


def _worker(rank, world, port, B, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        x = _gate_inputs(B=B)
        shards = partition.plan(B=B, Hk=4, Hv=8, world=world)
        dA, ddt = _shard_sums(x, shards[rank])
        fa, fd = partition.reduce_gate_grads(dA, ddt, shards[rank], Hv=8)
        q.put((rank, fa.numpy(), fd.numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("B", [4, 1])
def test_allreduce_matches_single_process(B):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, B, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    x = _gate_inputs(B=B)
    full = partition.Shard(0, 0, B, 0, 4, 0, 8)
    wa, wd = _shard_sums(x, full)
    for _, fa, fd in got:
        np.testing.assert_allclose(fa, wa.numpy(), rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(fd, wd.numpy(), rtol=1e-5, atol=1e-6)


def _failing_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        # this rank dies between steps, before the collective, with nothing of its own in flight
        q.put((rank, "raised"))
        q.close()
        q.join_thread()  # the message is out before the process goes
        os._exit(3)
    try:
        buf = torch.ones(16)
        dist.all_reduce(buf)
        q.put((rank, "completed"))
    except Exception as e:  # the survivor learns of it as an error, within the group's timeout
        q.put((rank, "error: " + type(e).__name__))


def test_rank_failure_surfaces_as_error():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert res[1] == "raised"
    assert res[0].startswith("error"), res[0]
