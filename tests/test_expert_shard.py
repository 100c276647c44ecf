"""Expert-parallel host logic on CPU.

* The sharded parameter layouts: every rank holds its own experts first ([0, shared_begin)) and the
  replicated parameters after, at the same offsets on every rank; the ranks' shards together cover
  every parameter exactly once and pack / unpack round-trips.
* The exchange of the expert-parallel step on two gloo ranks: the replicated range and the loss are
  summed, each rank's expert range is left alone, and the FP64 norm partials of the experts are
  summed, so that every rank sees the global gradient norm.
"""
import os
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from sejong_b200 import model as pm


def _config():
    return pm.with_(pm.small_hierarchy(), experts=pm.ExpertConfig(4, 2, 128))


@pytest.mark.parametrize("world", [1, 2, 4])
def test_shards_partition_the_parameters(world):
    c = _config()
    full = pm.FlatLayout(c)
    rng = np.random.default_rng(world)
    params = {n: rng.standard_normal(s).astype(np.float32) for n, s, _ in pm.reference_layout(c)}
    seen = {}
    shared = None
    for rank in range(world):
        lay = pm.FlatLayout(c, expert_shard=(rank, world))
        assert lay.shared_begin > 0 and lay.shared_begin % pm.ALIGN == 0
        for e in lay.entries.values():
            assert (".experts." in e.name) == (e.offset < lay.shared_begin), e.name
        offs = {n: e.offset - lay.shared_begin for n, e in lay.entries.items() if ".experts." not in n}
        assert shared is None or offs == shared  # the replicated range is laid out alike on every rank
        shared = offs
        assert lay.n_decay > lay.shared_begin
        out = lay.unpack(lay.pack(params))
        for n, v in out.items():
            np.testing.assert_array_equal(v, params[n])
            if ".experts." in n:
                assert n not in seen, n
                seen[n] = rank
    assert set(seen) == {n for n in params if ".experts." in n}
    assert full.shared_begin == 0


def test_shard_rejects_an_uneven_split():
    with pytest.raises(ValueError):
        pm.FlatLayout(_config(), expert_shard=(0, 3))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out_dir):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    from sejong_b200 import distributed
    _, _, _, group = distributed.init_from_env("gloo", timeout_s=20)
    sb = 64
    g = torch.arange(256, dtype=torch.float32) + 1000 * rank
    loss = torch.tensor([1.5 + rank], dtype=torch.float64)
    partials = torch.tensor([float(rank + 1), 2.0 * (rank + 1)], dtype=torch.float64)
    distributed.exchange(g[sb:], loss, group, partials)
    np.savez(os.path.join(out_dir, f"{rank}.npz"), g=g.numpy(), loss=loss.numpy(), partials=partials.numpy())
    torch.distributed.destroy_process_group()


def test_expert_parallel_exchange_on_two_gloo_ranks():
    world = 2
    with tempfile.TemporaryDirectory() as out:
        mp.spawn(_worker, args=(world, _port(), out), nprocs=world, join=True)
        res = [dict(np.load(os.path.join(out, f"{r}.npz"))) for r in range(world)]
    base = np.arange(256, dtype=np.float32)
    for r in range(world):
        g = res[r]["g"]
        np.testing.assert_array_equal(g[:64], base[:64] + 1000 * r)          # own experts untouched
        np.testing.assert_array_equal(g[64:], 2 * base[64:] + 1000)           # replicated range summed
        assert float(res[r]["loss"][0]) == 1.5 + 2.5
        np.testing.assert_array_equal(res[r]["partials"], [3.0, 6.0])
