"""Sharding rules and the pipeline handoff of ``fracture_b200.shards``, on CPU.

The multi-rank tests start 2 or 3 ``gloo`` ranks as spawned processes on 127.0.0.1 and run the
same code the GPU pipeline runs over NCCL: micro-batches flow stage 0 -> 1 -> ... with
asynchronous sends and receives posted ahead, and the last stage's results must equal the
stage functions applied in sequence on one process.
"""

import os
import socket
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from fracture_b200 import shards


def test_sequence_shard_partitions():
    for n, world in [(16, 1), (16, 2), (16, 8), (17, 4), (3, 4)]:
        got = [list(shards.sequence_shard(n, world, r)) for r in range(world)]
        assert sum(got, []) == list(range(n))
        assert max(map(len, got)) - min(map(len, got)) <= 1


def test_block_shard_is_block_aligned_and_complete():
    for n, world in [(65536, 1), (65536, 2), (65536, 8), (1000, 3), (17, 4), (5, 2)]:
        rs = [shards.block_shard(n, world, r) for r in range(world)]
        assert sum((list(r) for r in rs), []) == list(range(n))
        for r in rs:
            if len(r):
                assert r.start % shards.BLOCK_TOKENS == 0
                assert r.stop == n or r.stop % shards.BLOCK_TOKENS == 0


def test_stage_layers():
    assert [shards.stage_layers(80, 8, r) for r in range(8)] == [range(10 * s, 10 * s + 10) for s in range(8)]
    assert sum((list(shards.stage_layers(10, 3, r)) for r in range(3)), []) == list(range(10))
    with pytest.raises(ValueError):
        shards.stage_layers(10, 2, 2)


def test_stage_link_neighbours():
    assert (shards.StageLink(0, 4).prev, shards.StageLink(0, 4).next) == (None, 1)
    assert (shards.StageLink(3, 4).prev, shards.StageLink(3, 4).next) == (2, None)
    assert (shards.StageLink(0, 4, ring=True).prev, shards.StageLink(3, 4, ring=True).next) == (3, 0)
    assert shards.StageLink(0, 1, ring=True).next is None


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _stage_fn(rank):
    # layer stand-ins of stage `rank`: exact float arithmetic, different on each stage
    def fn(m, x):
        return x * (rank + 2) + (m + 1) * (rank + 1)
    return fn


def _worker(rank, world, port, n_micro, errq):
    try:
        os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        link = shards.StageLink(rank, world)
        outs = {}
        shape = (4, 3)
        fn = _stage_fn(rank)
        # stage outputs alternate between two buffers, as the GPU stages do
        obuf = [torch.empty(shape), torch.empty(shape)]

        def stage(m, x):
            obuf[m % 2].copy_(fn(m, x))
            return obuf[m % 2]

        shards.run_pipeline(n_micro, link,
                            first_input=lambda m: torch.full(shape, float(m)),
                            stage_fn=stage,
                            recv_buffers=[torch.empty(shape), torch.empty(shape)],
                            on_output=lambda m, y: outs.__setitem__(m, y.clone()))
        if rank == world - 1:
            for m in range(n_micro):
                x = torch.full(shape, float(m))
                for s in range(world):
                    x = _stage_fn(s)(m, x)
                assert torch.equal(outs[m], x), (m, outs[m], x)
            assert sorted(outs) == list(range(n_micro))
        # stages that work in place on the received buffer and send it on (three buffers)
        outs2 = {}

        def stage_inplace(m, x):
            if rank == 0:
                x = x.clone()
            x.mul_(rank + 2).add_((m + 1) * (rank + 1))
            return x

        shards.run_pipeline(n_micro, link,
                            first_input=lambda m: torch.full(shape, float(m)),
                            stage_fn=stage_inplace,
                            recv_buffers=[torch.empty(shape) for _ in range(3)],
                            on_output=lambda m, y: outs2.__setitem__(m, y.clone()))
        if rank == world - 1:
            assert all(torch.equal(outs2[m], outs[m]) for m in range(n_micro))
        # timing aggregate
        assert shards.max_over_ranks(float(rank) * 1.5) == (world - 1) * 1.5
        # ring: the last stage hands a tensor back to stage 0
        ring = shards.StageLink(rank, world, ring=True)
        t = torch.full((2,), float(rank))
        if rank == world - 1:
            ring.isend(t).wait()
        if rank == 0:
            got = torch.empty(2)
            ring.irecv(got).wait()
            assert torch.equal(got, torch.full((2,), float(world - 1)))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        errq.put(f"rank {rank}: {traceback.format_exc()}")
        raise


@pytest.mark.parametrize("world,n_micro", [(2, 5), (3, 4), (2, 1)])
def test_pipeline_handoff_gloo(world, n_micro):
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n_micro, errq)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
    errors = []
    while not errq.empty():
        errors.append(errq.get())
    assert not errors, "\n".join(errors)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
