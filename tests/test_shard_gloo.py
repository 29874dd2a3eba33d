"""Multi-rank host logic on CPU (gloo, world size 2): requests are sharded by
prompt length, each rank runs its own requests with no exchange, and the
gathered results equal one process serving everything."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from yanchor_b200 import shard


def _free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _requests(n=9, seed=3):
    """Varlen GDN requests (prompt lengths 5..70, H=2, HV=4, K=V=16)."""
    rng = np.random.default_rng(seed)
    reqs = []
    for _ in range(n):
        T = int(rng.integers(5, 71))
        q = rng.standard_normal((1, T, 2, 16)).astype(np.float32)
        k = rng.standard_normal((1, T, 2, 16)).astype(np.float32)
        v = rng.standard_normal((1, T, 4, 16)).astype(np.float32)
        g = np.log(1 / (1 + np.exp(-rng.standard_normal((1, T, 4))))).astype(np.float32)
        beta = (1 / (1 + np.exp(-rng.standard_normal((1, T, 4))))).astype(np.float32)
        reqs.append((q, k, v, g, beta))
    return reqs


def _serve(req):
    from oracle import gdn
    q, k, v, g, beta = req
    o, s = gdn.chunk_gated_delta_rule(q, k, v, g, beta, use_qk_l2norm=True)
    return o, s


def _worker(rank, world, port, out_path):
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port))
    import datetime
    import torch.distributed as dist
    dist.init_process_group('gloo', rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        reqs = _requests()
        owned = shard.shard_requests([r[0].shape[1] for r in reqs], world)[rank]
        local = [_serve(reqs[i]) for i in owned]          # no exchange while serving
        results = shard.gather_by_request(local, owned, len(reqs))
        slowest = shard.max_over_ranks(1.5 + rank)
        if rank == 0:
            np.savez(out_path, slowest=slowest, owned=np.array(owned),
                     **{f'o{i}': r[0] for i, r in enumerate(results)}, **{f's{i}': r[1] for i, r in enumerate(results)})
    finally:
        dist.destroy_process_group()


def test_sharded_serving_equals_one_process(tmp_path):
    out = str(tmp_path / 'gathered.npz')
    mp.spawn(_worker, args=(2, _free_port(), out), nprocs=2, join=True)
    got = np.load(out)
    assert float(got['slowest']) == 2.5
    for i, req in enumerate(_requests()):
        o, s = _serve(req)
        np.testing.assert_array_equal(got[f'o{i}'], o)
        np.testing.assert_array_equal(got[f's{i}'], s)


def test_shard_requests_balanced_and_complete():
    rng = np.random.default_rng(0)
    lengths = rng.integers(512, 16385, 512)           # the serving-sweep prompt lengths
    for world in (1, 2, 4, 8):
        owned = shard.shard_requests(lengths, world)
        flat = sorted(i for o in owned for i in o)
        assert flat == list(range(len(lengths)))
        loads = [int(lengths[o].sum()) for o in owned]
        assert max(loads) - min(loads) <= int(lengths.max())
        assert owned == shard.shard_requests(lengths, world)       # same answer on every rank
    assert shard.shard_requests([], 3) == [[], [], []]
    with pytest.raises(ValueError):
        shard.shard_requests([1, 2], 0)
