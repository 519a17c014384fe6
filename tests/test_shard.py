"""Multi-GPU host logic on the CPU: heads split over ranks and outputs gathered, with two `gloo` ranks
(the same calls run over NCCL in bench.py --gpus N)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from htrc_b200 import shard

N, D, HEADS = 96, 128, 4


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _head_output(h):
    # a per-head pattern that identifies the head in every element
    return torch.arange(N * D, dtype=torch.float32).reshape(N, D) * 1e-3 + 1000.0 * h


def _rank(rank, world, port, errors):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
        mine = shard.heads_of_rank(HEADS, rank, world)
        slots = [shard.gather_slot(_head_output(h)) for h in mine]
        full = shard.assemble(slots, HEADS)
        want = torch.stack([_head_output(h) for h in range(HEADS)])
        assert torch.equal(full, want)
        dist.destroy_process_group()
    except Exception as e:  # reported back to the parent
        errors.put(f"rank {rank}: {type(e).__name__}: {e}")


def test_heads_of_rank_partitions_the_layer():
    for world in (1, 2, 4, 8):
        got = [h for r in range(world) for h in shard.heads_of_rank(24, r, world)]
        assert got == list(range(24))
    with pytest.raises(ValueError):
        shard.heads_of_rank(24, 0, 5)
    with pytest.raises(ValueError):
        shard.heads_of_rank(24, 2, 2)


def test_gather_over_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    errors = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, errors)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    msgs = []
    while not errors.empty():
        msgs.append(errors.get())
    assert not alive, "a rank did not finish"
    assert not msgs, msgs
    assert all(p.exitcode == 0 for p in procs)
