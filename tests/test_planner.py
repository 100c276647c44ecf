"""The NativeValue batch planner (value_execution.rs:101-352) on CPU: the reference's own unit test
(checkpoint_replay_keeps_one_block_and_hierarchy_shortens_global_sequence, value_execution.rs:
354-380) ported, the power-of-two allocation rule, the binary search against a linear scan, the
retained-then-checkpointed mode order, resumed batches and the capacity error."""
import numpy as np
import pytest

from sejong_b200 import model as pm
from sejong_b200 import planner
from sejong_b200.param_vjp import VjpConfig


def _default():
    # sejong_core::ModelConfig::default() (crates/sejong-core/src/lib.rs:108-124)
    return pm.ModelConfig(width=512, layers=8, heads=8, ffn_width=1536)


def test_reference_unit_test_checkpoint_replay_and_hierarchy():
    c = _default()
    retained = planner.workspace_bytes(c, 1024, 16, 1, False)
    replay = planner.workspace_bytes(c, 1024, 16, 1, True)
    assert replay < retained
    assert planner.workspace_bytes(c, 1024, 16, 2, False) >= retained
    h = pm.HierarchyConfig(8, 128, 2, 2, 384, 128, 2, 2, 384, 128)
    c = pm.with_(c, hierarchy=h)
    patched = planner.workspace_bytes(c, 1024, 16, 1, False)
    c1 = pm.with_(c, hierarchy=pm.HierarchyConfig(1, 128, 2, 2, 384, 128, 2, 2, 384, 128))
    assert planner.workspace_bytes(c1, 1024, 16, 1, False) > patched


def test_allocation_is_a_power_of_two():
    assert planner.allocation(0, 4) == 1
    assert planner.allocation(1, 4) == 4
    assert planner.allocation(3, 4) == 16
    assert planner.allocation(4096, 2) == 8192
    assert planner.allocation(4097, 2) == 16384


def _plan_args():
    c = pm.with_(pm.small_hierarchy(), experts=pm.ExpertConfig(4, 2, 128))
    prompts = [b"x" * n for n in (5, 40, 77, 12)]
    return c, prompts


@pytest.mark.parametrize("policy", [None, VjpConfig()])
def test_binary_search_is_the_largest_fitting_batch(policy):
    c, prompts = _plan_args()
    seq = max(len(p) for p in prompts) + 2
    params = planner.value_parameters(c, 7)
    fixed = planner.fixed_bytes(c, 7)

    def need(b, ck):
        return fixed + planner.workspace_bytes(c, seq, 7, b, ck) + planner.factor_bytes(params, policy, b, seq, c)
    rng = np.random.default_rng(0)
    for avail in [need(1, False), need(37, False) + 5, need(500, False), need(1, True), need(3, True) - 1]:
        avail += int(rng.integers(0, 1000))
        try:
            p = planner.plan(c, prompts, 7, 1000, avail, policy=policy)
        except planner.CapacityError:
            assert need(1, True) > avail and need(1, False) > avail
            continue
        scan = [b for b in range(1, 1001) if need(b, p.checkpointing) <= avail]
        assert p.batch == max(scan)
        if p.checkpointing:  # retained mode was tried first and did not fit a single request
            assert need(1, False) > avail
        assert p.fixed_bytes == fixed and p.workspace_bytes == need(p.batch, p.checkpointing) - fixed


def test_memory_budget_caps_and_resume_checks():
    c, prompts = _plan_args()
    big = 1 << 40
    p = planner.plan(c, prompts, 7, 64, big)
    assert p.batch == 64 and not p.checkpointing  # every request fits: the cap is the inventory
    q = planner.plan(c, prompts, 7, 64, big, max_examples=10)
    assert q.batch == 10
    small = planner.plan(c, prompts, 7, 64, big, memory_bytes=p.workspace_bytes // 4)
    assert small.batch < 64 and small.available == small.fixed_bytes + p.workspace_bytes // 4
    r = planner.plan(c, prompts, 7, 64, big, saved=(5, True))
    assert (r.batch, r.checkpointing) == (5, True)
    with pytest.raises(ValueError):
        planner.plan(c, prompts, 7, 64, big, saved=(65, False))
    with pytest.raises(planner.CapacityError) as e:
        planner.plan(c, prompts, 7, 64, 1000)
    assert e.value.available == 1000 and e.value.required > 1000
