"""Data-parallel exchange on CPU: two gloo ranks, the product's `sejong_b200.distributed` logic.

* Two ranks, each with its own batch and the product's per-rank seed scaling: the SUM-reduced
  flat gradient (product `FlatLayout`) and loss equal the single-process mean over both batches.
* A rank that dies before the exchange makes the surviving rank's collective fail with an error
  within the process-group timeout instead of hanging (failure detection on the host).
"""
import os
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

ROWS_SEQ = 64


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _config():
    from oracle import model as om
    return om.ModelConfig(width=64, layers=1, heads=1, kv_heads=1, ffn_width=64,
                          hierarchy=om.HierarchyConfig(8, 64, 1, 1, 64, 64, 1, 1, 64, 16))


def _batch(rank):
    from oracle.corpus import synthetic_corpus
    from oracle.rng import Rng
    from sejong_b200.distributed import rank_seed
    return synthetic_corpus(3, 20000).batch(Rng(rank_seed(123, rank)), 1, ROWS_SEQ)


def _worker(rank, world, port, out_dir, die_rank):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from oracle import model as om
    from sejong_b200 import distributed
    from sejong_b200 import model as pm
    _, _, _, group = distributed.init_from_env("gloo", timeout_s=5)
    c = _config()
    params = om.initialize(c)
    ids, tg = _batch(rank)
    # per-row seed 1/(rows*world): the oracle's mean-loss gradient times 1/world
    seed = distributed.ce_seed(ROWS_SEQ, world) * ROWS_SEQ
    loss, grads = om.loss_and_grads(params, c, ids, tg, ROWS_SEQ, scale=seed)
    pc = pm.ModelConfig(width=c.width, layers=c.layers, heads=c.heads, ffn_width=c.ffn_width,
                        kv_heads=c.kv_heads, hierarchy=pm.HierarchyConfig(**c.hierarchy.__dict__))
    lay = pm.FlatLayout(pc)
    g = torch.from_numpy(lay.pack({k: v.astype(np.float32) for k, v in grads.items()}))
    loss_sum = torch.tensor([loss / world], dtype=torch.float64)
    if rank == die_rank:
        os._exit(0)  # leaves between steps, with no collective in flight
    try:
        distributed.exchange(g, loss_sum, group)
        status = "ok"
    except Exception as e:  # the surviving rank must see an error, not hang
        status = f"error: {type(e).__name__}"
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), g=g.numpy(), loss=loss_sum.numpy(), status=status)
    try:
        dist.destroy_process_group()
    except Exception:
        pass


def test_two_rank_exchange_equals_single_process():
    from oracle import model as om
    from sejong_b200 import model as pm
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_worker, args=(2, _port(), d, -1), nprocs=2, start_method="spawn", join=True)
        r0 = np.load(os.path.join(d, "rank0.npz"))
        r1 = np.load(os.path.join(d, "rank1.npz"))
    assert str(r0["status"]) == "ok" and str(r1["status"]) == "ok"
    np.testing.assert_array_equal(r0["g"], r1["g"])
    c = _config()
    params = om.initialize(c)
    (i0, t0), (i1, t1) = _batch(0), _batch(1)
    ids, tg = np.concatenate([i0, i1]), np.concatenate([t0, t1])
    loss, grads = om.loss_and_grads(params, c, ids, tg, ROWS_SEQ)
    pc = pm.ModelConfig(width=c.width, layers=c.layers, heads=c.heads, ffn_width=c.ffn_width,
                        kv_heads=c.kv_heads, hierarchy=pm.HierarchyConfig(**c.hierarchy.__dict__))
    want = pm.FlatLayout(pc).pack({k: v.astype(np.float32) for k, v in grads.items()})
    np.testing.assert_allclose(r0["g"], want, rtol=1e-5, atol=1e-8)
    assert abs(float(r0["loss"][0]) - loss) < 1e-9


@pytest.mark.timeout(120)
def test_dead_rank_surfaces_as_error_not_hang():
    with tempfile.TemporaryDirectory() as d:
        ctx = mp.start_processes(_worker, args=(2, _port(), d, 1), nprocs=2, start_method="spawn", join=False)
        while not ctx.join(timeout=60):
            pass
        r0 = np.load(os.path.join(d, "rank0.npz"))
    assert str(r0["status"]).startswith("error"), str(r0["status"])


@pytest.mark.parametrize("name", ["config_c3", "config_c1", "small_hierarchy"])
def test_gradient_buckets_partition_the_flat_gradient(name):
    """The overlapped exchange's buckets cover every element of the flat gradient exactly once, never
    split a parameter, and list a stage's matrices only where the backward has finished them."""
    from sejong_b200 import model as pm
    from sejong_b200.train import gradient_buckets
    c = getattr(pm, name)()
    lay = pm.FlatLayout(c)
    buckets = gradient_buckets(lay, c)
    spans = sorted((b, e) for _, b, e in buckets)
    assert spans[0][0] == 0 and spans[-1][1] == lay.total
    assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    tags = {}
    for e in lay.entries.values():
        owner = [t for t, b, en in buckets if b <= e.offset < en]
        assert len(owner) == 1
        t = owner[0]
        b, en = next((b, en) for tt, b, en in buckets if tt == t and b <= e.offset < en)
        assert e.offset + e.size <= en, e.name
        tags[e.name] = t
    half = pm.global_stage(c).layers // 2
    for name_, t in tags.items():
        if name_.startswith("decoder.") and lay[name_].decay:
            assert t == "decoder"
        if name_.startswith("layers.") and lay[name_].decay:
            layer = int(name_.split(".")[1])
            assert t == ("global_half" if layer >= half else ("global" if c.hierarchy else None))
        if not lay[name_].decay:
            assert t is None  # norm vectors: at the end
