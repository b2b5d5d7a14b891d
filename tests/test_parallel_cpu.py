"""Multi-process plumbing on CPU: world-size-2 gloo ranks (one weight broadcast, root sharding,
max-over-ranks timing, result gather), and a rank that fails before the first collective."""
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import REPO


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, queue, fail_rank):
    sys.path.insert(0, REPO)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    import datetime
    from omoknuni_quantum_b200 import parallel
    from omoknuni_quantum_b200.resnet import ResNetSpec, init_state_dict
    from omoknuni_quantum_b200.roots import random_roots
    try:
        if rank == fail_rank:
            raise RuntimeError("injected failure before joining")
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=10))
        spec = ResNetSpec(num_blocks=1, filters=128, fc_value_hidden=16, fc_policy_hidden=16)
        sd = init_state_dict(spec, seed=100 + rank)       # ranks start with different weights
        calls = []
        real = dist.broadcast
        dist.broadcast = lambda *a, **k: (calls.append(1), real(*a, **k))[1]
        try:
            sd = parallel.broadcast_state_dict(sd, "cpu")
        finally:
            dist.broadcast = real
        src = init_state_dict(spec, seed=100)
        exact = all(torch.equal(sd[k], src[k]) and sd[k].dtype == src[k].dtype for k in src)
        digest = (float(sum(v.double().sum() for v in sd.values())), len(calls), exact)
        shard = parallel.shard_range(10, world, rank)
        roots = random_roots(5, 10)[shard.start:shard.stop]
        ms = parallel.max_over_ranks(10.0 * (rank + 1), "cpu")
        total = parallel.sum_over_ranks(len(shard), "cpu")
        g = parallel.gather_results(np.full((2,), rank, np.int32), "cpu")
        queue.put((rank, digest, list(shard), int(roots.sum()), ms, total,
                   None if g is None else g.tolist()))
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent, never hangs it
        queue.put((rank, "error", repr(e)))


def _run(world, fail_rank=-1, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, fail_rank)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=timeout) for _ in range(world)]
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return sorted(out, key=lambda x: x[0])


def test_two_rank_broadcast_shard_and_reduce():
    out = _run(2)
    (r0, d0, s0, _, ms0, tot0, g0), (r1, d1, s1, _, ms1, tot1, g1) = out
    assert d0 == d1                       # rank 1 received rank 0's weights
    assert d0[1] == 1 and d0[2]           # in one collective, bit-exact in every dtype
    assert s0 == [0, 1, 2, 3, 4] and s1 == [5, 6, 7, 8, 9]
    assert ms0 == ms1 == 20.0             # max over ranks
    assert tot0 == tot1 == 10
    assert g0 == [0, 0, 1, 1] and g1 is None


def test_failed_rank_is_reported_not_hung():
    out = _run(2, fail_rank=1, timeout=120)
    assert out[1][1] == "error" and "injected" in out[1][2]
    assert out[0][1] == "error"           # rank 0's rendezvous times out and raises


def test_shard_range_covers_everything():
    from omoknuni_quantum_b200.parallel import shard_range
    for total in (0, 1, 7, 256, 513):
        for ws in (1, 2, 3, 8):
            seen = []
            for r in range(ws):
                seen.extend(shard_range(total, ws, r))
            assert seen == list(range(total))
