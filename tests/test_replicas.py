"""Replica sharding host logic, with world_size-2 gloo process groups on the CPU.

Each rank runs the eager (unpatched) model on its block of sequences as a
stand-in for its GPU replica; the gathered batch must equal a single-process
forward of the whole batch.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tinker_b200.replicas import shard_bounds


def test_shard_bounds_cover_the_batch_in_order():
    for batch in (0, 1, 5, 64):
        for world in (1, 2, 3, 8):
            spans = [shard_bounds(batch, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == batch
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [e - s for s, e in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_bounds(4, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from bench_model import TINY, build_model, make_tokens
        from tinker_b200.replicas import gather_batch, local_shard
        torch.set_num_threads(1)
        model = build_model(TINY, seed=3)
        tokens = make_tokens(TINY, 5, 12, seed=4)
        with torch.inference_mode():
            out = model(local_shard(tokens))
        full = gather_batch(out, tokens.shape[0])
        if rank == 0:
            with torch.inference_mode():
                ref = model(tokens)
            q.put(bool(torch.allclose(full, ref, atol=1e-5, rtol=1e-5)) and full.shape == ref.shape)
    finally:
        dist.destroy_process_group()


def test_two_replicas_reproduce_the_full_batch():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    assert q.get(timeout=10) is True
