"""Batch-shard bookkeeping on CPU ranks (gloo, world_size 2): shards cover the batch exactly,
and sharded processing + gather equals the single-process result bit for bit. The per-shard
compute is the CPU oracle on a tiny pi0.5 case (observations are independent)."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from flashact_b200.sharding import gather_actions, shard_range


def test_shard_range_covers_batch():
    for batch in range(0, 13):
        for world in range(1, 9):
            spans = [shard_range(batch, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == batch
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            sizes = [hi - lo for lo, hi in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


def _tiny_case():
    from oracle import pi05_oracle as O
    return O.make_case(seed=5, L=1, T=4, AD=8, Lp=6, B=5, num_steps=2)


def _run_shard(case, lo, hi):
    from oracle import pi05_oracle as O
    sub = O.Pi05Case(**{**case.__dict__})
    sub.B = hi - lo
    sub.k, sub.v, sub.noise = case.k[lo:hi], case.v[lo:hi], case.noise[lo:hi]
    sub.valid_len = case.valid_len[lo:hi]
    return O.denoise(sub)


def _worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.set_num_threads(1)
    case = _tiny_case()
    lo, hi = shard_range(case.B, world, rank)
    out = gather_actions(_run_shard(case, lo, hi), case.B)
    if rank == 0:
        q.put(out)
    dist.barrier()
    dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_sharded_equals_single_process():
    torch.set_num_threads(1)
    case = _tiny_case()
    ref = _run_shard(case, 0, case.B)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = q.get(timeout=240)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert torch.equal(out, ref)
