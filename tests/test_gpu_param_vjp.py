"""GPU parity of the parameter VJP (index draw, basis, prepare, materialise, and the whole training
step with compressed weight gradients) against the oracle, through the C ABI.

Bars: indices and the generator state bit-exact; the basis to 1e-3 of the FP64 CGS2 of the same
donor columns (f32 Gram-space arithmetic on bf16 inputs); left to 1e-4 and E to 1e-2 relative
(E is bf16); the step's loss within 1e-3 and every gradient within 2e-2 relative L2 of the FP64
oracle replaying the same draws.
"""
import numpy as np
import pytest
import torch

from oracle import model as om
from oracle import param_vjp as opv
from oracle.corpus import synthetic_corpus
from oracle.rng import MASK64, Rng

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def lib():
    from sejong_b200 import _lib
    lib = _lib.load()
    _lib.call("sj_device_init", 0)
    return lib


def call(name, *args):
    from sejong_b200 import _lib
    return _lib.call(name, *args)


def ptr(t, off=0):
    return t.data_ptr() + off * t.element_size()


def stream():
    return torch.cuda.current_stream().cuda_stream


def rel(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    nb = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / nb) if nb > 0 else float(np.linalg.norm(a))


def u64_tensor(value):
    return torch.from_numpy(np.array([value], dtype=np.uint64).view(np.int64)).to(DEV)


def u64_of(t):
    return int(t.cpu().numpy().view(np.uint64)[0])


GEN = torch.Generator().manual_seed(4321)


def randn(*shape):
    return torch.randn(*shape, generator=GEN, dtype=torch.float64)


@pytest.mark.parametrize("a,b,nb,s,r,group", [(256, 768, 8, 2, 16, 32), (768, 2048, 24, 6, 16, 32),
                                              (0, 300, 0, 0, 16, 32), (200, 0, 7, 2, 0, 32), (71, 23, 5, 2, 6, 16)])
def test_device_indices(a, b, nb, s, r, group):
    state = 0x0123456789ABCDEF ^ (a * 1000003 + b)
    rng = u64_tensor(state)
    i32 = torch.int32
    columns = torch.full((max(r, 1),), -7, dtype=i32, device=DEV)
    rows = torch.full((max(s * group, 1),), -7, dtype=i32, device=DEV)
    row_map = torch.full((max(a, 1),), -7, dtype=i32, device=DEV)
    call("sj_param_indices", ptr(rng), a, b, nb, s, r, group, ptr(columns), ptr(rows), ptr(row_map), stream())
    torch.cuda.synchronize()
    host = Rng(state)
    seed = host.next_u64()
    ref_cols, ref_rows, ref_map = opv.parameter_indices(seed, a, b, nb, s, r, group)
    assert u64_of(rng) == host.state
    assert columns[:r].cpu().tolist() == list(ref_cols)
    assert rows[:s * group].cpu().tolist() == list(ref_rows)
    assert row_map[:a].cpu().tolist() == list(ref_map)


@pytest.mark.parametrize("n,a,ldw,offset,interleave,cols", [
    (4096, 768, 2304, 0, 0, None),        # global query donor inside the fused qkv weight
    (2048, 256, 1536, 0, 16, None),       # local "up" donor of an interleaved gate/up weight
    (1000, 128, 384, 256, 0, [3, 9, 3, 100, 17, 0, 64, 5]),   # repeated column: one zero basis vector
])
def test_basis(n, a, ldw, offset, interleave, cols):
    width = ldw // 2 if interleave else ldw - offset
    r = 16 if cols is None else len(cols)
    if cols is None:
        cols = list(np.random.default_rng(n).choice(min(width, 768), r, replace=False))
    x = randn(n, a).to(torch.bfloat16)
    w = (0.05 * randn(a, ldw)).to(torch.bfloat16)
    xd, wd = x.to(DEV), w.to(DEV)
    columns = torch.tensor(cols, dtype=torch.int32, device=DEV)
    q = torch.empty(n, r, dtype=torch.float32, device=DEV)
    from sejong_b200 import _lib
    ws = torch.empty((_lib.load().sj_param_basis_workspace(n, a, r) + 7) // 8, dtype=torch.float64, device=DEV)
    eps = opv.basis_eps(n, r)
    call("sj_param_basis", ptr(xd), a, n, a, ptr(wd, offset), ldw, interleave, ptr(columns), r, eps, ptr(q), ptr(ws),
         stream())
    torch.cuda.synchronize()
    phys = [((c // 16) * 32 + 16 + c % 16) if interleave else offset + c for c in cols]
    y = x.double().numpy() @ w.double().numpy()[:, phys]
    ref = opv.basis_cgs2(y, eps)
    got = q.cpu().numpy()
    zero = np.all(ref == 0, axis=0)
    assert list(np.all(got == 0, axis=0)) == list(zero)
    assert float(np.max(np.abs(got - ref))) < 1e-3 * max(1.0, float(np.max(np.abs(ref))))
    # orthonormal where not cut off
    gram = got[:, ~zero].T.astype(np.float64) @ got[:, ~zero]
    assert float(np.max(np.abs(gram - np.eye(gram.shape[0])))) < 1e-4


@pytest.mark.parametrize("n,a,k,inverse", [(4096, 768, 192, 4.0), (2048, 256, 64, 4.0), (640, 80, 64, 3.5)])
def test_prepare(n, a, k, inverse):
    r = 16
    x = randn(n, a).to(torch.bfloat16)
    q = torch.linalg.qr(randn(n, r))[0].float().contiguous()
    rows = np.arange(k) + 32
    rows[rows >= a] = -1
    xd, qd = x.to(DEV), q.to(DEV)
    rows_d = torch.tensor(rows, dtype=torch.int32, device=DEV)
    left = torch.empty(a, r, dtype=torch.float32, device=DEV)
    e = torch.empty(r + k, n, dtype=torch.bfloat16, device=DEV)
    call("sj_param_prepare", ptr(xd), a, n, a, ptr(qd), r, ptr(rows_d), k, inverse, ptr(left), ptr(e), stream())
    torch.cuda.synchronize()
    ref_left, ref_e = opv.prepare_factors(x.double().numpy(), q.double().numpy(), rows, inverse)
    assert rel(left.cpu().numpy(), ref_left) < 1e-4
    got_e = e.float().cpu().numpy()
    assert rel(got_e[:r], ref_e[:r]) < 1e-2
    for pos in range(k):
        if rows[pos] < 0:
            assert np.all(got_e[r + pos] == 0)
    assert rel(got_e[r:], ref_e[r:]) < 1e-2


def test_materialize():
    a, b, r, k, ldc = 300, 520, 16, 64, 1024
    left = randn(a, r).float()
    coeff = randn(r + k, ldc).float()
    row_map = np.full(a, -1, dtype=np.int32)
    row_map[64:128] = np.arange(64)
    g0 = randn(a, ldc).float()
    ld, cd, gd = left.to(DEV), coeff.to(DEV), g0.clone().to(DEV)
    md = torch.tensor(row_map, device=DEV)
    call("sj_param_materialize", ptr(ld), ptr(cd, 8), ldc, ptr(md), a, b, r, ptr(gd, 8), ldc, 1, stream())
    torch.cuda.synchronize()
    ref = g0.double().numpy().copy()
    c64 = coeff.double().numpy()
    upd = left.double().numpy() @ c64[:r, 8:8 + b]
    sel = row_map >= 0
    upd[sel] += c64[r + row_map[sel], 8:8 + b]
    ref[:, 8:8 + b] += upd
    got = gd.cpu().numpy()
    assert float(np.max(np.abs(got - ref))) < 1e-4
    assert np.array_equal(got[:, :8], g0.numpy()[:, :8]) and np.array_equal(got[:, 8 + b:], g0.numpy()[:, 8 + b:])


def oracle_config(c):
    h = c.hierarchy
    oh = None if h is None else om.HierarchyConfig(**h.__dict__)
    return om.ModelConfig(width=c.width, layers=c.layers, heads=c.heads, ffn_width=c.ffn_width,
                          kv_heads=c.kv_heads, rope_theta=c.rope_theta, norm_epsilon=c.norm_epsilon,
                          hierarchy=oh, seed=c.seed, init_std=c.init_std, router_std=c.router_std)


@pytest.mark.parametrize("config_name,batch,seq", [("small_hierarchy", 1, 2048), ("config_c1", 2, 512),
                                                    ("config_c3", 2, 4096)])
def test_step_parity(config_name, batch, seq):
    """One training step with the parameter VJP and compact SGD against the FP64 oracle.  The C4 case is
    C3's architecture at 2 x 4096 bytes with fraction 0.25: 1,024 global rows >= 768 features, so the
    global QKV and gate/up gradients are factored too, with 24 of 768 feature rows' blocks (192 rows)
    selected, beside the local stages' 2 of 8 blocks (64 rows)."""
    from sejong_b200 import model as pm
    from sejong_b200.param_vjp import VjpConfig
    from sejong_b200.train import ByteTrainer, TrainConfig
    c = getattr(pm, config_name)()
    oc = oracle_config(c)
    params = pm.initialize(c)
    ids, targets = synthetic_corpus(5, 200000).batch(Rng(77), batch, seq)
    vcfg = VjpConfig()
    tc = TrainConfig(sequence=seq, batch=batch, optimizer="sgd", learning_rate=1e-2, warmup_steps=0, steps=100,
                     parameter_vjp=vcfg)
    tr = ByteTrainer(c, tc, device=0, params=params)
    assert tr.vjp.compressed, "the case must compress some weight gradients"
    if config_name == "config_c3":
        assert tr.vjp.groups["layers.0.z1"].k == 192 and tr.vjp.groups["encoder.0.z1"].k == 64
    tr.stage_batch(ids, targets)
    tr.forward_backward()
    torch.cuda.synchronize()
    assert tr.device_error() == 0
    grads = tr.gradients()
    ocfg = opv.VjpConfig(rank=vcfg.rank, residual_fraction=vcfg.residual_fraction, block_rows=vcfg.block_rows,
                         seed=vcfg.seed)
    orng = Rng(ocfg.seed)
    loss, ref_grads, info = opv.vjp_gradients(params, oc, ids, targets, seq, ocfg, orng, cast="bf16")
    # draws: generator state, token-basis columns and feature rows bit-exact
    assert tr.vjp_rng_state() == orng.state
    assert sorted(info["compressed"]) == sorted(tr.vjp.compressed)
    for key, cols in info["bases"].items():
        assert tr.vjp_columns[key].cpu().tolist() == list(cols), key
    for width, (rows, row_map) in info["selections"].items():
        assert tr.vjp_rows[width].cpu().tolist() == list(rows), width
        assert tr.vjp_map[width].cpu().tolist() == list(row_map), width
    assert abs(tr.loss() - loss) < 1e-3
    worst = {name: rel(grads[name], g) for name, g in ref_grads.items() if np.any(g != 0)}
    bad = {k: v for k, v in worst.items() if v > 2e-2}
    assert not bad, f"gradients beyond 2e-2: {bad}"
    # compact SGD on the GPU gradients against the FP64 update rule
    tr.optimizer_step()
    torch.cuda.synchronize()
    new = tr.parameters()
    otc = om.TrainConfig(sequence=seq, batch=batch, learning_rate=1e-2, warmup_steps=0, steps=100)
    ref_new, norm = opv.sgd_update(params, {k: v.astype(np.float64) for k, v in grads.items()}, otc, 0)
    assert abs(float(tr.hyper[4]) - norm) < 1e-5 * max(norm, 1.0)
    for k in params:
        assert float(np.max(np.abs(new[k] - ref_new[k]))) < 2e-6, k


def test_draws_advance_per_step():
    """An eager step and two graph replays make three passes' draws: the device generator ends
    where the oracle's does."""
    from sejong_b200 import model as pm
    from sejong_b200.param_vjp import VjpConfig
    from sejong_b200.train import ByteTrainer, TrainConfig
    c = pm.small_hierarchy()
    tc = TrainConfig(sequence=2048, batch=1, optimizer="sgd", learning_rate=1e-2, parameter_vjp=VjpConfig())
    tr = ByteTrainer(c, tc, device=0)
    ids, targets = synthetic_corpus(5, 200000).batch(Rng(3), 1, 2048)
    tr.stage_batch(ids, targets)
    tr.step()
    tr.capture()
    tr.replay()
    tr.replay()
    torch.cuda.synchronize()
    assert tr.device_error() == 0
    assert np.isfinite(tr.loss())
    host = Rng(tc.parameter_vjp.seed)
    for _ in range(3 * tr.vjp.draws):
        host.next_u64()
    assert tr.vjp_rng_state() == host.state & MASK64
    tr.release_graphs()


def test_adamw_with_parameter_vjp():
    """AdamW fed the parameter VJP's materialised gradient (GradientMaterializer,
    crates/sejong-gpu/src/parameter_vjp.rs:347-380; used by the NativeValue trainer, crates/sejong-train/
    src/memory.rs:1001-1010): the gradient equals the SGD route's for the same draws, and the update is
    the FP64 AdamW transition of that gradient."""
    from sejong_b200 import model as pm
    from sejong_b200.param_vjp import VjpConfig
    from sejong_b200.train import ByteTrainer, TrainConfig
    c = pm.small_hierarchy()
    params = pm.initialize(c)
    ids, targets = synthetic_corpus(5, 200000).batch(Rng(77), 1, 2048)
    out = {}
    for opt in ("sgd", "adamw"):
        tc = TrainConfig(sequence=2048, batch=1, optimizer=opt, learning_rate=1e-3, warmup_steps=0, steps=100,
                         parameter_vjp=VjpConfig())
        tr = ByteTrainer(c, tc, device=0, params=params)
        tr.stage_batch(ids, targets)
        tr.forward_backward()
        torch.cuda.synchronize()
        assert tr.device_error() == 0
        grads = tr.gradients()
        rng_state = tr.vjp_rng_state()
        tr.optimizer_step()
        torch.cuda.synchronize()
        out[opt] = (grads, rng_state, tr.parameters(), float(tr.hyper[4]))
        tr.close()
    g_sgd, rng_sgd, _, _ = out["sgd"]
    g_adam, rng_adam, new, norm_gpu = out["adamw"]
    assert rng_sgd == rng_adam
    # the two runs add their split-K f32 partials with reduce-adds in whatever order the SMs finish,
    # so the gradients agree to f32 rounding of those sums (measured up to 1.02e-5), not bit for bit
    for k in g_sgd:
        assert rel(g_adam[k], g_sgd[k]) < 1e-4, k
    otc = om.TrainConfig(sequence=2048, batch=1, learning_rate=1e-3, warmup_steps=0, steps=100)
    ref_new, norm = om.adam_update(params, {k: v.astype(np.float64) for k, v in g_adam.items()}, om.AdamState(), otc)
    assert abs(norm_gpu - norm) < 1e-5 * max(norm, 1.0)
    for k in params:
        assert float(np.max(np.abs(new[k] - ref_new[k]))) < 2e-6, k
