"""Data parallelism with the gradient exchange overlapping the backward pass (two GPUs).

Each of two ranks trains on its own rows; the flat gradient is all-reduced in buckets that start as
soon as the backward has finished them (the decoder blocks and heads, then each half of the global
blocks, then the rest; ByteTrainer.grad_buckets), on NCCL's stream while later phases of the backward
run.  The step -- eagerly, and replayed from the per-phase CUDA graphs -- must equal one device's
step on the two batches concatenated in rank order: loss, gradients, the FP64 gradient norm and the
AdamW update.  Bars: loss and norm 1e-6 / 1e-5 relative; gradients 1e-4 relative L2 (the two ranks'
weight-gradient sums meet in the all-reduce, one device's in one reduction), except `global_bos`: its
gradient is a GEMM of the batch-summed BOS gradient, which each rank rounds to bf16 (the GEMM operand)
over its own rows, so it carries one bf16 rounding of a partial sum, 5e-3 (measured 1.9e-3).  The two
ranks' weights after the update are bit-identical (they apply the same all-reduced gradient); against
one device they agree to 0.05 of the learning rate: AdamW's first step moves a weight by about
lr * g / (|g| + eps), so where |g| is near eps the step follows the gradient's last bits.
"""
import os
import socket
import tempfile

import numpy as np
import pytest
import torch

from oracle.corpus import synthetic_corpus
from oracle.rng import Rng

pytestmark = pytest.mark.gpu

BATCH, SEQ = 2, 1024


def _config():
    from sejong_b200 import model as pm
    return pm.small_hierarchy()


def _batches(ranks):
    ids, tg = synthetic_corpus(5, 400000).batch(Rng(77), BATCH * ranks, SEQ)
    return np.asarray(ids).reshape(ranks * BATCH, SEQ), np.asarray(tg).reshape(ranks * BATCH, SEQ)


def _trainer(batch, params, group=None, device=0):
    from sejong_b200.train import ByteTrainer, TrainConfig
    tc = TrainConfig(sequence=SEQ, batch=batch, warmup_steps=0, steps=100)
    return ByteTrainer(_config(), tc, device=device, params=params, process_group=group)


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out_dir):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    from sejong_b200 import distributed
    from sejong_b200.model import initialize
    _, _, _, group = distributed.init_from_env("nccl", timeout_s=60)
    params = initialize(_config())
    ids, tg = _batches(world)
    mine = slice(rank * BATCH, (rank + 1) * BATCH)
    out = {}
    for mode in ("eager", "graph"):
        tr = _trainer(BATCH, params, group=group, device=rank)
        assert tr.overlapped_exchange()
        tr.stage_batch(ids[mine], tg[mine])
        if mode == "eager":
            tr.forward_backward()
            torch.cuda.synchronize()
            out["grads"] = tr.gradients()
            tr.optimizer_step()
        else:
            tr.capture()
            tr.replay()
        torch.cuda.synchronize()
        out[f"{mode}_loss"] = tr.loss()
        out[f"{mode}_norm"] = float(tr.hyper[4])
        out[f"{mode}_err"] = tr.device_error()
        out[f"{mode}_w"] = tr.parameters()
        tr.release_graphs()
        tr.close()
        del tr
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"),
             **{k: v for k, v in out.items() if not isinstance(v, dict)},
             **{f"g/{k}": v for k, v in out["grads"].items()},
             **{f"we/{k}": v for k, v in out["eager_w"].items()},
             **{f"wg/{k}": v for k, v in out["graph_w"].items()})
    torch.distributed.destroy_process_group()


def _rel(a, b):
    nb = np.linalg.norm(b)
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / nb) if nb > 0 else float(np.abs(a).max())


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_ranks_with_overlapped_exchange_match_one_device():
    import torch.multiprocessing as mp
    from sejong_b200.model import initialize
    world = 2
    with tempfile.TemporaryDirectory() as out:
        mp.spawn(_worker, args=(world, _port(), out), nprocs=world, join=True)
        ranks = [dict(np.load(os.path.join(out, f"rank{r}.npz"))) for r in range(world)]
    params = initialize(_config())
    ids, tg = _batches(world)
    ref = _trainer(BATCH * world, params)
    ref.stage_batch(ids, tg)
    ref.forward_backward()
    torch.cuda.synchronize()
    ref_loss, ref_grads = ref.loss(), ref.gradients()
    ref.optimizer_step()
    torch.cuda.synchronize()
    ref_norm, ref_w = float(ref.hyper[4]), ref.parameters()
    from sejong_b200.train import TrainConfig
    lr = TrainConfig(sequence=SEQ, batch=BATCH).learning_rate
    worst_g, worst_w = 0.0, 0.0
    for r, res in enumerate(ranks):
        for mode in ("eager", "graph"):
            assert int(res[f"{mode}_err"]) == 0
            assert abs(float(res[f"{mode}_loss"]) - ref_loss) < 1e-6 * abs(ref_loss), (r, mode)
            assert abs(float(res[f"{mode}_norm"]) - ref_norm) < 1e-5 * ref_norm, (r, mode)
            for k, v in ref_w.items():
                worst_w = max(worst_w, float(np.abs(res[f"w{mode[0]}/{k}"] - v).max()))
                assert np.array_equal(res[f"w{mode[0]}/{k}"], ranks[0][f"w{mode[0]}/{k}"]), (r, mode, k)
        for k, g in ref_grads.items():
            e = _rel(res[f"g/{k}"], g)
            assert e < (5e-3 if k == "global_bos" else 1e-4), (r, k, e)
            worst_g = max(worst_g, e)
    print("worst gradient", worst_g, "worst weight", worst_w)
    assert worst_w < 0.05 * lr
