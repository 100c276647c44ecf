"""NativeValue step on the GPU against the FP64 restatement (oracle/value.py): the requests laid out
as forward_batch does, the body on the tcgen05 kernels, the SEP rows through the f32 value head,
the mean value cross entropy and every gradient (body, input projection, native embedding, head),
for the hierarchical and the dense body.  The GPU pads every request to one fixed sequence (a
multiple of the patch), the oracle to the batch's longest prompt + 2 as the reference does: the
results agree because nothing after a SEP row reaches it.  Bar: the value logits and every gradient
within 2e-2 relative L2, the loss within 1e-3.  The batch holds enough requests
(32, 16) for the loss to average the bf16 noise of single logits, as the byte loss does over its
rows."""
import numpy as np
import pytest
import torch

from oracle import model as om
from oracle import value as ov

pytestmark = pytest.mark.gpu


def _oracle_config(c):
    h = c.hierarchy
    return om.ModelConfig(width=c.width, layers=c.layers, heads=c.heads, ffn_width=c.ffn_width, kv_heads=c.kv_heads,
                          hierarchy=None if h is None else om.HierarchyConfig(**h.__dict__), seed=c.seed,
                          init_std=c.init_std)


def _prompts(n, seed):
    rng = np.random.default_rng(seed)
    return [bytes(rng.integers(32, 127, size=int(rng.integers(3, 70))).astype(np.uint8)) for _ in range(n)]


def _rel(a, b):
    nb = np.linalg.norm(b)
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / nb)


def _parity(c, values=6, batch=32, seed=3):
    from sejong_b200 import value as pv
    from sejong_b200.model import initialize
    from sejong_b200.train import ByteTrainer, TrainConfig
    prompts = _prompts(batch, seed)
    labels = np.arange(batch) % values
    params = initialize(c)
    params.update(pv.initialize_value(c, values))
    seq = pv.sequence_for(c, prompts)
    tr = ByteTrainer(c, TrainConfig(sequence=seq, batch=batch, values=values, warmup_steps=0), device=0,
                     params=params)
    ids, sel = pv.request_batch(prompts, seq)
    tr.stage_requests(ids, sel, labels)
    tr.forward_backward()
    torch.cuda.synchronize()
    assert tr.device_error() == 0
    loss, grads = tr.loss(), tr.gradients()
    logits = tr.vlogits.cpu().numpy()
    ref_logits = []
    ref_loss, ref = ov.loss_and_grads(params, _oracle_config(c), prompts, labels, cast="bf16", logits_out=ref_logits)
    print("loss", loss, ref_loss, "logits rel", _rel(logits, ref_logits[0]),
          "max abs", float(np.abs(logits - ref_logits[0]).max()))
    assert _rel(logits, ref_logits[0]) < 2e-2
    assert set(grads) == set(ref) - {"embedding", "output"}
    worst = {}
    for k, g in grads.items():
        if np.all(ref[k] == 0):
            assert float(np.abs(g).max()) < 1e-6, k
            continue
        worst[k] = _rel(g, ref[k])
    print("worst gradients", sorted(worst.items(), key=lambda kv: -kv[1])[:5])
    bad = {k: v for k, v in worst.items() if v > 2e-2}
    assert not bad, bad
    assert abs(loss - ref_loss) < 1e-3, (loss, ref_loss)
    tr.optimizer_step()
    torch.cuda.synchronize()
    assert tr.device_error() == 0
    return worst


def test_value_step_parity_hierarchical_body():
    from sejong_b200 import model as pm
    worst = _parity(pm.small_hierarchy())
    assert worst["input_projection"] < 2e-2 and worst["native_embedding"] < 2e-2


def test_value_step_parity_dense_body():
    from sejong_b200 import model as pm
    c = pm.with_(pm.config_c1(), layers=2)
    _parity(c, values=5, batch=16, seed=8)


def test_planner_sizes_the_batch_from_device_memory():
    """value_execution::prepare with the device's free memory (cudaMemGetInfo) and a workspace
    budget: the planned batch is positive, within the inventory, and this build's trainer (every
    activation retained) allocates at that batch without running out of memory."""
    from sejong_b200 import model as pm
    from sejong_b200 import planner
    from sejong_b200 import value as pv
    c = pm.small_hierarchy()
    prompts = _prompts(300, 5)
    free = planner.available_bytes(0)
    assert free > 0
    p = planner.plan(c, prompts, 6, len(prompts), free, memory_bytes=512 << 20)
    assert 1 <= p.batch <= len(prompts) and p.available <= free
    ok, used = planner.fits_this_build(c, p.batch, pv.sequence_for(c, prompts), 6, 0)
    print("planned batch", p.batch, "checkpointing", p.checkpointing, "reference bytes",
          p.fixed_bytes + p.workspace_bytes, "this build allocates", used)
    assert ok and used > 0
