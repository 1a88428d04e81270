"""Host logic of multi-GPU replicas on CPU (gloo, world size 2): round-robin partitioning,
each rank serving its share through its own continuous batcher (host-only stand-in backend),
max-over-ranks timing and gathering results on rank 0; the union must equal a single-process
run of the whole job."""
import asyncio
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tiny_infra_b200 import replicas
from tiny_infra_b200.scheduler import ContinuousBatcher

from test_scheduler_trace import _HostKV, _StandInBackend

CFG = {"max_batch_size": 2, "max_seq_len": 64, "block_size": 16, "head_dim": 8}
JOB = [([3 + i, 7, 11 * i % 97, 5], 3 + i % 4) for i in range(7)]


def _serve(world, rank):
    kv = _HostKV(CFG)
    sched = ContinuousBatcher(None, kv, eos_token_id=13, backend=_StandInBackend(kv, 97))

    async def main():
        loop = asyncio.create_task(sched.run_loop())
        out = await replicas.serve_partition(sched, JOB, world, rank, temperature=0.0)
        loop.cancel()
        return out

    return asyncio.run(main())


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        out = _serve(world, rank)
        t = replicas.max_over_ranks(1.5 + rank)
        gathered = replicas.gather_to_rank0(out)
        if rank == 0:
            merged = {}
            for part in gathered:
                merged.update(part)
            q.put((t, merged))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_partition_round_robin():
    assert replicas.partition(7, 2, 0) == [0, 2, 4, 6]
    assert replicas.partition(7, 2, 1) == [1, 3, 5]
    assert sorted(replicas.partition(10, 3, 0) + replicas.partition(10, 3, 1)
                  + replicas.partition(10, 3, 2)) == list(range(10))
    with pytest.raises(ValueError):
        replicas.partition(4, 2, 2)


def test_two_replicas_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    t, merged = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert t == 2.5                       # max over ranks of 1.5 + rank
    assert merged == _serve(1, 0)         # the union is the single-process job
    assert sorted(merged) == list(range(len(JOB)))
