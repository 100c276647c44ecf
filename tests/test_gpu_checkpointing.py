"""Activation checkpointing of the global stage (Graph::checkpoint, crates/sejong-gpu/src/graph.rs:151-174
and 756-799; the global stage is the checkpointed one, crates/sejong-model/src/architecture.rs:32,307-311).

With TrainConfig.activation_checkpointing the global blocks keep only their inputs and share one set of
activation buffers, which the backward refills by running each block's forward again.  The step must
compute what the retained step computes: the same loss (the forward is the same arithmetic) and the
same gradients up to the order of the split-K / attention reductions (1e-5 relative L2, or the
variation of the retained step between two runs where that is larger), checked on
the reduced hierarchy, the C3 architecture at 1 x 1024 bytes and an MoE hierarchy.  At the C3 batch the
checkpointed trainer must hold at least (layers - 1) blocks' activations less, and the planner's
checkpoint branch (value_execution.rs:246-352) must admit a larger batch than the retain branch for the
same budget -- a batch that this build then allocates and steps."""
import numpy as np
import pytest
import torch

from oracle.corpus import synthetic_corpus
from oracle.rng import Rng

pytestmark = pytest.mark.gpu


def _rel(a, b):
    nb = np.linalg.norm(b)
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / nb) if nb > 0 else float(np.abs(a).max())


def _step(c, params, batch, seq, ckpt):
    from sejong_b200.train import ByteTrainer, TrainConfig
    ids, tg = synthetic_corpus(7, 1 << 18).batch(Rng(3), batch, seq)
    tr = ByteTrainer(c, TrainConfig(sequence=seq, batch=batch, activation_checkpointing=ckpt), device=0,
                     params=params)
    tr.stage_batch(ids, tg)
    tr.forward_backward()
    torch.cuda.synchronize()
    assert tr.device_error() == 0
    out = tr.loss(), tr.gradients()
    tr.close()
    return out


@pytest.mark.parametrize("name,batch,seq", [("small_hierarchy", 2, 512), ("config_c3", 1, 1024),
                                            ("small_moe", 1, 1024)])
def test_checkpointed_step_equals_retained(name, batch, seq):
    from sejong_b200 import model as pm
    if name == "small_moe":
        c = pm.small_hierarchy()
        c.experts = pm.ExpertConfig(4, 2, 128)
    else:
        c = getattr(pm, name)()
    params = pm.initialize(c)
    loss0, g0 = _step(c, params, batch, seq, False)
    loss1, g1 = _step(c, params, batch, seq, True)
    _, g2 = _step(c, params, batch, seq, False)
    assert loss0 == loss1
    diffs = sorted(((_rel(g1[k], g0[k]), k) for k in g0), reverse=True)
    again = max(_rel(g2[k], g0[k]) for k in g0)
    print(name, "worst gradient differences", diffs[:6], "retained run twice", again)
    # The retained step itself varies from run to run where an attention backward adds three or more
    # f32 partial sums with atomics (the C3 global stage at this size: dK / dV of the three query
    # heads of a group): a last-bit change can tip a bf16 rounding of dK, and dK = dS^T Q cancels
    # strongly.  The checkpointed step may differ from the retained one by no more than that.
    assert diffs[0][0] < max(1e-5, 4 * again)


def test_checkpointing_saves_memory_and_the_planner_branch_runs():
    from sejong_b200 import model as pm
    from sejong_b200 import planner
    from sejong_b200.train import ByteTrainer, TrainConfig
    c = pm.config_c3()
    used = {}
    for ckpt in (False, True):
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        before = torch.cuda.memory_allocated()
        tr = ByteTrainer(c, TrainConfig(sequence=4096, batch=8, activation_checkpointing=ckpt), device=0)
        used[ckpt] = torch.cuda.memory_allocated() - before
        tr.close()
        del tr
    glob = pm.global_stage(c)
    rows, d, f = 8 * 512, glob.width, glob.ffn
    per_block = rows * (2 * d * 2 + glob.qkv_width * 2 + d * 4 + 2 * f * 2 + f * 2)  # z1, z2, qkv, x1, gu, h
    print("allocated retained", used[False], "checkpointed", used[True], "per block", per_block)
    assert used[False] - used[True] >= (glob.layers - 1) * per_block
    # the planner's checkpoint branch (value_execution.rs:246-352 keeps every activation whenever one
    # request fits that way): a budget that retains no request but checkpoints some
    from sejong_b200.value import sequence_for
    prompts = [bytes(40)] * 512
    big = 1 << 50

    def need(mode):
        p1 = planner.plan(c, prompts, 4, 512, big, activation_checkpointing=mode, max_examples=1)
        return p1.fixed_bytes + p1.workspace_bytes

    budget = (need(True) + need(False)) // 2
    with pytest.raises(planner.CapacityError):
        planner.plan(c, prompts, 4, 512, budget, activation_checkpointing=False)
    p = planner.plan(c, prompts, 4, 512, budget)
    print("budget", budget, "retain needs", need(False), "checkpoint needs", need(True), "planned", p.batch,
          p.checkpointing)
    assert p.checkpointing and p.batch >= 1
    fits, used_ck = planner.fits_this_build(c, p.batch, sequence_for(c, prompts), 4, 0, activation_checkpointing=True)
    assert fits
    tr = ByteTrainer(c, TrainConfig(sequence=sequence_for(c, prompts), batch=p.batch, values=4,
                                    activation_checkpointing=True), device=0)
    from sejong_b200 import value as pv
    ids, sel = pv.request_batch(prompts[:p.batch], tr.tc.sequence)
    tr.stage_requests(ids, sel, np.zeros(p.batch, dtype=np.int32))
    tr.step()
    torch.cuda.synchronize()
    assert tr.device_error() == 0 and np.isfinite(tr.loss())
    tr.close()
