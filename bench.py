"""Benchmark: hierarchical byte-model training step (fwd + bwd + AdamW) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    (N > 1: launched by torch.distributed.run, one rank per GPU, NCCL)

Workload ("C3"): per GPU batch 8 x 4096 Zipf(1.1) bytes, patch 8;
local encoder/decoder d256 x 2 layers each (4 heads, window 128, SwiGLU 768); global d768 x 8
layers, HQ12/HK4, SwiGLU 2048; bf16 with f32 accumulation; AdamW.  Data-parallel: each rank
trains its own batch, gradients summed over NCCL (weak scaling).

Metric: bytes/s of the whole job (BASELINE metric "train ms/step & bytes/s", the unit of
crates/sejong-cli/src/benchmark.rs:325).  `value` times K graph replays with the K batches
already resident in HBM; `e2e` times the same K steps through the public API with each
step's bytes copied from pinned host memory and the loss read back.  Both are CUDA-event
times on the launching stream, barrier + synchronize on both sides, max over ranks.  The
per-step working set (several GB of activations) exceeds the 126 MB L2, so no flush runs.

`roofline` covers the dominant kernel family (timed live with CUDA events in an extra eager
step); `cpu_baseline` times the CPU restatement in oracle/ (PyTorch fp32, all host threads)
on a bounded sample of the same workload (rank 0, N = 1 only).
`--impl reference` times that CPU restatement alone (the reference itself has no CPU path and
its Rust/HIP host cannot be built here).
"""
import argparse
import ctypes
import json
import os
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "train_bytes_per_s"
WORKLOADS = {"c1": "C1 dense byte model, one training step in fp32: fwd+bwd+AdamW (BASELINE configs[0]), f32 CUDA-core "
                   "GEMMs and attention",
             "c3": "C3 hierarchical byte model, fwd+bwd+AdamW (BASELINE configs[2])",
             "c4": "C4 hierarchical byte model, fwd + input VJP + parameter VJP (rank 16, fraction 0.25) + "
                   "compact SGD lr 1e-2 (BASELINE configs[3])",
             "c5": "C5 byte MoE model, fwd+bwd+AdamW (BASELINE configs[4]) with expert capacity factor 1.25 and "
                   "load-balance loss weight 0.01: on one GPU all 8 experts of a layer are local; on N GPUs each "
                   "owns 8/N experts and routed rows move over NVLink peer memory (expert parallelism), the rest is "
                   "data parallel"}
MODELS = {"c1": "dense byte model: d256 x4, HQ4/HK2, SwiGLU 1024, eps 1e-6, RoPE 1e4",
          "c3": "hierarchical byte model: local d256 2+2 layers W128, global d768 x8 HQ12/HK4 SwiGLU2048",
          "c4": "hierarchical byte model: local d256 2+2 layers W128, global d768 x8 HQ12/HK4 SwiGLU2048",
          "c5": "byte MoE model: local d256 2+2 layers W128, global d1024 x12 HQ16/HK4, 8 SwiGLU experts of 2816 "
                "top-2 (router N(0,0.006))"}
SHAPES = {"c1": (8, 512), "c3": (8, 4096), "c4": (8, 4096), "c5": (4, 8192)}  # per-GPU batch x bytes
L2_NOTE = {"c1": "per-step working set of about 0.3 GB (f32 activations) > 126 MB L2; no flush"}
# the f32 step runs on the CUDA cores: 148 SMs x 128 FMA lanes x 2 FLOP x 1965 MHz (nominal)
FP32_SIMT_PEAK_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12
UNIT = "bytes/s"
CPU_SAMPLE_BATCH, CPU_SAMPLE_SEQ = 1, 1024
CPU_SAMPLES = {"c1": (8, 512)}  # C1 is small enough for the CPU to run the whole step
# DRAM bytes (read + write) of all GEMM launches of one C3 step, from the ncu launch list of
# `python bench.py --steps 1 --warmup 3 --no-cpu-baseline --no-kernel-timing` summarised in
# profiles/c3_step_launch_list.txt (ncu flushes caches between launches: an upper bound)
NCU_GEMM_DRAM_BYTES_PER_STEP = {"c3": 5.492e9}
NCU_TRAFFIC_SOURCE = ("ncu --metrics gpu__time_duration.sum,dram__bytes_read.sum,dram__bytes_write.sum launch list of "
                      "one C3 step (profiles/c3_step_launch_list.txt), summed over the GEMM launches; not measured in "
                      "this run")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=None, help="per-GPU batch (default: the config's)")
    ap.add_argument("--seq", type=int, default=None, help="bytes per row (default: the config's)")
    ap.add_argument("--config", choices=["c1", "c2", "c3", "c4", "c5"], default="c3",
                    help="c1: dense fp32 step (BASELINE configs[0]); c3: AdamW (configs[2]); "
                         "c4: parameter-VJP SGD (configs[3]); "
                         "c2: MiniLM encoder forward (configs[1]); c5: byte MoE (configs[4])")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-kernel-timing", action="store_true")
    ap.add_argument("--kernel-report", default=None, help="write per-call kernel timings (JSON) to this path")
    return ap.parse_args()


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return {"hbm": p["hbm_gbs"], "bf16": p["bf16_tflops"], "bf16_sustained": p["bf16_tflops_sustained"],
                "source": "measured"}
    except Exception:
        return {"hbm": 6650.0, "bf16": 1590.0, "bf16_sustained": 1400.0, "source": "fallback"}


# ---------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        sm = sorted(float(r[1]) for r in rows if r[1].replace(".", "").isdigit())
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": float(rows[0][2]) if rows else None,
                "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------- CPU restatement (oracle) timing
def cpu_step_rate(steps, warmup, threads=None, config="c3", sample=None):
    """bytes/s of the oracle's fp32 CPU training step on the bounded sample of C3 (AdamW) or C4
    (parameter-VJP SGD)."""
    import numpy as np
    import torch

    from oracle import model as omodel
    from oracle import param_vjp as opv
    from oracle.corpus import synthetic_corpus
    from oracle.rng import Rng
    if threads:
        torch.set_num_threads(threads)
    c = {"c1": omodel.config_c1, "c5": omodel.config_c5}.get(config, omodel.config_c3)()
    params = omodel.initialize(c)
    corp = synthetic_corpus(1000, 1 << 20)
    rng = Rng(123)
    state = omodel.AdamState()
    batch, seq = sample or CPU_SAMPLES.get(config, (CPU_SAMPLE_BATCH, CPU_SAMPLE_SEQ))
    tc = omodel.TrainConfig(sequence=seq, batch=batch, learning_rate=1e-2 if config == "c4" else 3e-4)
    vcfg = opv.VjpConfig()
    vrng = Rng(vcfg.seed)
    times = []
    for i in range(warmup + steps):
        ids, tg = corp.batch(rng, batch, seq)
        t0 = time.perf_counter()
        if config == "c4":
            _, grads, _ = opv.vjp_gradients(params, c, ids, tg, seq, vcfg, vrng)
            params, _ = opv.sgd_update(params, grads, tc, i)
        else:
            loss, grads = omodel.loss_and_grads(params, c, ids, tg, seq, dtype=torch.float32)
            params, _ = omodel.adam_update(params, grads, state, tc)
        params = {k: np.asarray(v, dtype=np.float32) for k, v in params.items()}
        if i >= warmup:
            times.append(time.perf_counter() - t0)
    sec = sum(times) / len(times)
    return batch * seq / sec, sec, torch.get_num_threads()


def cpu_sample_text(steps, config="c3", sample=None):
    b, t = sample or CPU_SAMPLES.get(config, (CPU_SAMPLE_BATCH, CPU_SAMPLE_SEQ))
    if config == "c1":
        whole = "the whole step" if (b, t) == (8, 512) else "a reduced batch"
        return f"C1, {whole} ({b} x {t} bytes), fp32 torch CPU fwd+bwd+AdamW, mean of {steps} steps"
    if config == "c4":
        return (f"C4 architecture, batch {b} x {t} bytes (vs 8 x 4096 on the GPU), "
                f"FP64 CPU fwd + input VJP + parameter VJP + compact SGD, mean of {steps} steps")
    if config == "c5":
        return (f"C5 architecture (8 experts, top-2), batch {b} x {t} bytes (vs 4 x 8192 "
                f"on the GPU), fp32 torch CPU fwd+bwd+AdamW, mean of {steps} steps")
    return (f"C3 architecture, batch {b} x {t} bytes (vs 8 x 4096 on the GPU), "
            f"fp32 torch CPU fwd+bwd+AdamW, mean of {steps} steps")


REFERENCE_ARM_BUDGET_S = 150.0


def reference_sample(steps, warmup, config):
    """The per-step CPU sample of the reference arm: the config's bounded sample, shrunk (bytes per
    row, or rows for C1) so that warmup + steps steps take about REFERENCE_ARM_BUDGET_S seconds on
    this host; one untimed calibration step decides."""
    b, t = CPU_SAMPLES.get(config, (CPU_SAMPLE_BATCH, CPU_SAMPLE_SEQ))
    _, sec, _ = cpu_step_rate(1, 0, config=config, sample=(b, t))
    scale = REFERENCE_ARM_BUDGET_S / max(sec * (steps + warmup), 1e-9)
    if scale >= 1.0:
        return b, t
    if config == "c1":
        return max(1, int(b * scale)), t
    return b, max(256, int(t * scale) // 256 * 256)


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    steps, warmup = max(1, args.steps), max(0, args.warmup)
    sample = reference_sample(steps, warmup, args.config)
    rate, sec, cores = cpu_step_rate(steps, warmup, config=args.config, sample=sample)
    line = {"metric": METRIC, "value": rate, "unit": UNIT, "n_gpus": args.gpus, "steps": steps, "warmup": warmup,
            "ms_per_step": sec * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic Zipf(1.1) bytes, random-init N(0,0.02) weights",
            "config": {"workload": WORKLOADS[args.config] + " (bounded CPU sample)",
                       "per_gpu_batch": sample[0], "seq_len": sample[1], "parallelism": "none"},
            "impl": "reference",
            "cpu_baseline": {"value": rate, "unit": UNIT, "cores": cores, "kind": "port",
                             "sample": cpu_sample_text(steps, args.config, sample)},
            "e2e": {"value": rate, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "the reference has no CPU execution path (Engine::new needs HIP) and its Rust host cannot "
                    "be built in this image; this arm times the CPU restatement of its step in oracle/"}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- GPU arm
def kernel_timing(trainer, report=None, replays=3):
    """Per-family kernel time and FLOPs of one step, measured in the regime of the headline: the step
    (forward, backward and update; no collective) is captured as a CUDA graph with an event node
    before and after every C-ABI call, and the graph is replayed `replays` times.  The event nodes
    cut the programmatic-launch overlap between neighbouring kernels, so each family's time is an
    upper bound of its share of the event-free graph; the sum over families is reported beside the
    headline step time."""
    import torch
    records = []
    original = trainer._call

    def timed(name, *a):
        s, e = torch.cuda.Event(enable_timing=True, external=True), torch.cuda.Event(enable_timing=True, external=True)
        stream = torch.cuda.current_stream()
        s.record(stream)
        original(name, *a)
        e.record(stream)
        flops = 2.0 * a[9] * a[10] * a[11] if name == "sj_gemm" else 0.0
        if name == "sj_sgemm":
            flops = 2.0 * a[8] * a[9] * a[10]
        if name == "sj_gemm_grouped":  # algorithmic rows: the routed ones, not the padded capacity
            routed = trainer.routed_rows()
            flops = 2.0 * a[10] * (a[11] * routed if a[17] == 1 else a[9] * routed)
        info = {"m": a[9], "n": a[10], "k": a[11], "epi": a[12], "a_t": a[2], "b_t": a[5]} if name == "sj_gemm" else {}
        records.append((name, s, e, flops, info))

    torch.cuda.synchronize()
    side = torch.cuda.Stream(trainer.dev)
    side.wait_stream(torch.cuda.current_stream(trainer.dev))
    graph = torch.cuda.CUDAGraph()
    trainer._call = timed
    try:
        with torch.cuda.stream(side):
            with torch.cuda.graph(graph, stream=side):
                trainer._local_forward_backward()
                trainer.optimizer_step()
    finally:
        trainer._call = original
    torch.cuda.current_stream(trainer.dev).wait_stream(side)
    torch.cuda.synchronize()
    graph.replay()  # warm
    torch.cuda.synchronize()
    per_call = [0.0] * len(records)
    for _ in range(replays):
        graph.replay()
        torch.cuda.synchronize()
        for i, (_, s, e, _, _) in enumerate(records):
            per_call[i] += s.elapsed_time(e) / replays
    graph.reset()
    fam = {}
    rows = []
    for (name, s, e, flops, info), ms in zip(records, per_call):
        f = fam.setdefault(name, {"ms": 0.0, "calls": 0, "flops": 0.0})
        f["ms"] += ms
        f["calls"] += 1
        f["flops"] += flops
        rows.append(dict(name=name, us=round(ms * 1e3, 2), tflops=round(flops / ms / 1e9, 1) if flops else None,
                         **info))
    if report:
        with open(report, "w") as fh:
            json.dump({"families": fam, "calls": rows}, fh, indent=1)
    return fam


def run_ours(args):
    import ctypes

    import numpy as np
    import torch
    import torch.distributed as dist

    from sejong_b200 import distributed
    from sejong_b200 import model as pm
    from sejong_b200.train import ByteTrainer, TrainConfig, corpus_batch, synthetic_corpus_tokens

    rank, world, local, pg = distributed.init_from_env("nccl", timeout_s=300)
    torch.cuda.set_device(local)
    cfg = {"c1": pm.config_c1, "c5": pm.config_c5}.get(args.config, pm.config_c3)()
    if args.batch is None:
        args.batch = SHAPES[args.config][0]
    if args.seq is None:
        args.seq = SHAPES[args.config][1]
    if args.config == "c4":
        from sejong_b200.param_vjp import VjpConfig
        tc = TrainConfig(sequence=args.seq, batch=args.batch, optimizer="sgd", learning_rate=1e-2, warmup_steps=0,
                         steps=10000, parameter_vjp=VjpConfig())
    elif args.config == "c5":
        # capacity factor 1.25 and load-balance loss weight 0.01 (this build's additions;
        # the reference keeps every routed row and has no auxiliary loss); the capacity counts each rank's rows
        tc = TrainConfig(sequence=args.seq, batch=args.batch, warmup_steps=0, steps=10000, moe_capacity_factor=1.25,
                         moe_aux_loss_weight=0.01)
    else:
        tc = TrainConfig(sequence=args.seq, batch=args.batch, warmup_steps=0, steps=10000)
    # C5 on several GPUs: the experts are sharded over the ranks (expert parallelism), the rest is
    # data parallel
    ep = args.config == "c5" and world > 1
    if args.config == "c1":
        from sejong_b200.train_f32 import F32Trainer
        trainer = F32Trainer(cfg, tc, device=local, process_group=pg)
    else:
        trainer = ByteTrainer(cfg, tc, device=local, process_group=pg, expert_parallel=ep)
    rows = tc.batch * tc.sequence
    total = args.warmup + args.steps
    toks = synthetic_corpus_tokens(distributed.rank_seed(1000, rank), 1 << 22)
    st = ctypes.c_uint64(distributed.rank_seed(123, rank))
    host_ids = torch.empty(total, rows, dtype=torch.int32).pin_memory()
    host_tg = torch.empty(total, rows, dtype=torch.int32).pin_memory()
    for i in range(total):
        x, y = corpus_batch(toks, st, tc.batch, tc.sequence)
        host_ids[i].copy_(torch.from_numpy(x))
        host_tg[i].copy_(torch.from_numpy(y))
    dev_ids = host_ids.to(trainer.dev)
    dev_tg = host_tg.to(trainer.dev)
    loss_host = torch.zeros(total, dtype=torch.float64).pin_memory()

    trainer.stage_batch(dev_ids[0], dev_tg[0])
    trainer.step()  # eager first step: sets kernel attributes, checks the path runs
    torch.cuda.synchronize()
    trainer.capture()
    stream = torch.cuda.current_stream()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=trainer.dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    clocks = ClockSampler(local)  # sampling starts before warm-up so it is running in the timed region
    clocks.start()
    for i in range(args.warmup):
        trainer.ids.copy_(host_ids[i], non_blocking=True)
        trainer.targets.copy_(host_tg[i], non_blocking=True)
        trainer.replay()
        loss_host[i].copy_(trainer.loss_sum[0], non_blocking=True)
    barrier()
    time.sleep(0.3)

    # device-resident inputs
    barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for i in range(args.warmup, total):
        trainer.ids.copy_(dev_ids[i])
        trainer.targets.copy_(dev_tg[i])
        trainer.replay()
    t1.record(stream)
    barrier()
    dev_ms = max_over_ranks(t0.elapsed_time(t1))
    # end to end through the public API: H2D of the step's bytes, D2H of its loss
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    e0.record(stream)
    for i in range(args.warmup, total):
        trainer.ids.copy_(host_ids[i], non_blocking=True)
        trainer.targets.copy_(host_tg[i], non_blocking=True)
        trainer.replay()
        loss_host[i].copy_(trainer.loss_sum[0], non_blocking=True)
    e1.record(stream)
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    clk = clocks.stop()
    assert trainer.device_error() == 0, "device error word set during the benchmark"
    losses = loss_host.numpy()
    assert np.all(np.isfinite(losses)), "non-finite loss"

    per_step_launches = sum(trainer.kernels_of(n, a) for n, a in _call_names(trainer))
    fam = {} if args.no_kernel_timing else kernel_timing(trainer, args.kernel_report if rank == 0 else None)
    if world > 1:
        trainer.release_graphs()
    trainer.close()

    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return
    K = args.steps
    ms = dev_ms / K
    global_bytes = rows * world
    value = global_bytes / (ms / 1e3)
    e2e_value = global_bytes / ((e2e_ms / K) / 1e3)
    pk = peaks()
    step_flops = trainer.step_flops()
    tensor_frac = step_flops / (ms / 1e3) / (pk["bf16_sustained"] * 1e12)
    roofline = None
    if fam and args.config == "c1":
        g = fam.get("sj_sgemm")
        if g and g["ms"] > 0:
            achieved = g["flops"] / (g["ms"] / 1e3) / 1e12
            tensor_frac = step_flops / (ms / 1e3) / (FP32_SIMT_PEAK_TFLOPS * 1e12)
            roofline = {"bound": "fp32 CUDA cores", "kernel": "sgemm_kernel (all f32 GEMMs of one step)",
                        "achieved": achieved, "peak": FP32_SIMT_PEAK_TFLOPS, "unit": "TFLOP/s",
                        "frac": achieved / FP32_SIMT_PEAK_TFLOPS,
                        "peak_source": "nominal fp32 FMA peak (148 SMs x 128 lanes x 2 x 1965 MHz); no measured fp32 "
                                       "peak in MEASURED_PEAKS.json",
                        "traffic": None, "launches": g["calls"], "ms_per_step": g["ms"]}
    elif fam:
        gs = [fam[k] for k in ("sj_gemm", "sj_gemm_grouped") if k in fam]
        g = {"ms": sum(x["ms"] for x in gs), "flops": sum(x["flops"] for x in gs), "calls": sum(x["calls"] for x in gs)}
        if g["ms"] > 0:
            achieved = g["flops"] / (g["ms"] / 1e3) / 1e12
            roofline = {"bound": "tensor", "kernel": "gemm_tcgen05 (all GEMMs of one step, grouped expert GEMMs included)",
                        "achieved": achieved, "peak": pk["bf16_sustained"], "unit": "TFLOP/s",
                        "frac": achieved / pk["bf16_sustained"], "peak_source": pk["source"] + " sustained bf16",
                        "traffic": NCU_GEMM_DRAM_BYTES_PER_STEP.get(args.config),
                        "traffic_unit": "bytes per step, all GEMM launches",
                        "traffic_source": NCU_TRAFFIC_SOURCE if args.config in NCU_GEMM_DRAM_BYTES_PER_STEP else None,
                        "timing": "graph replay of one step with an event node around every call (mean of 3)",
                        "launches": g["calls"], "ms_per_step": g["ms"]}
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": K, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32" if args.config == "c1" else "bf16",
        "data": "synthetic: Zipf(1.1) bytes from the reference Rng (seed 1000+rank); random-init N(0,0.02) weights",
        "config": {"workload": WORKLOADS[args.config],
                   "model": MODELS[args.config],
                   "global_batch": tc.batch * world, "per_gpu_batch": tc.batch, "seq_len": tc.sequence,
                   "parallelism": f"dp{world}" + (f"+ep{world}" if ep else ""),
                   "l2": L2_NOTE.get(args.config, "per-step working set of several GB > 126 MB L2; no flush")},
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": 2 * rows * 4, "d2h_bytes_per_step": 8},
        "gpu_launches": per_step_launches * K,
        "roofline": roofline,
        "tensor_frac_of_step": tensor_frac,
        "step_tflop": step_flops / 1e12,
        "loss_first_last": [float(losses[0]), float(losses[-1])],
    }
    if clk:
        line["clocks"] = clk
    if fam:
        line["kernel_ms_per_step"] = {k.replace("sj_", ""): round(v["ms"], 4) for k, v in sorted(fam.items())}
        line["kernel_ms_sum"] = round(sum(v["ms"] for v in fam.values()), 4)
    if world == 1 and not args.no_cpu_baseline:
        rate, _, cores = cpu_step_rate(2, 1, config=args.config)
        line["cpu_baseline"] = {"value": rate, "unit": UNIT, "cores": cores, "kind": "port",
                                "sample": cpu_sample_text(2, args.config)}
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def _call_names(trainer):
    """(name, arguments) of the C-ABI calls one step makes (recorded without launching anything)."""
    names = []
    original = trainer._call
    trainer._call = lambda name, *a: names.append((name, a))
    try:
        trainer.step()
    finally:
        trainer._call = original
    return names


# ---------------------------------------------------------------- C2: MiniLM encoder forward
C2_BATCH = 64
C2_CPU_SEQS = 64
C2_CPU_PASSES = 3
C2_METRIC, C2_UNIT = "encoder_tokens_per_s", "tokens/s"
C2_WORKLOAD = ("C2 MiniLM-L6-shaped BERT encoder forward (BASELINE configs[1]): batch 64, lengths uniform "
               "16..128, d384 x 6 layers, 12 heads, FFN 1536 GELU, post-LN")


def c2_cpu_rate(threads=None):
    """Valid tokens/s of the CPU restatement (oracle/bert.py, fp32 torch, per unpadded sequence as the
    reference runs it) on one C2 batch, mean of C2_CPU_PASSES passes."""
    import torch

    from oracle import bert as obert
    from sejong_b200 import bert
    if threads:
        torch.set_num_threads(threads)
    c = bert.MiniLMConfig()
    params = bert.initialize(c)
    seqs = bert.synthetic_batch(3000, C2_BATCH)[:C2_CPU_SEQS]
    obert.COMPUTE = torch.float32
    try:
        obert.hidden(params, seqs[0], c.layers, c.heads)  # warm-up
        t0 = time.perf_counter()
        for _ in range(C2_CPU_PASSES):
            for sq in seqs:
                obert.hidden(params, sq, c.layers, c.heads)
        sec = (time.perf_counter() - t0) / C2_CPU_PASSES
    finally:
        obert.COMPUTE = torch.float64
    tokens = sum(len(sq) for sq in seqs)
    return tokens / sec, sec, tokens, torch.get_num_threads()


def run_c2_reference(args):
    if int(os.environ.get("RANK", "0")) != 0:
        return
    rate, sec, tokens, cores = c2_cpu_rate()
    sample = (f"one C2 batch ({C2_CPU_SEQS} sequences, {tokens} tokens), fp32 torch CPU, one sequence at a time, "
              f"mean of {C2_CPU_PASSES} passes")
    line = {"metric": C2_METRIC, "value": rate, "unit": C2_UNIT, "n_gpus": args.gpus, "steps": 1, "warmup": 1,
            "ms_per_step": sec * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic ids per BASELINE C2, random-init N(0,0.02) weights",
            "config": {"workload": C2_WORKLOAD + " (bounded CPU sample)", "parallelism": "none"},
            "impl": "reference",
            "cpu_baseline": {"value": rate, "unit": C2_UNIT, "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": rate, "unit": C2_UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "the reference's BERT runs on HIP only; this arm times the CPU restatement in oracle/bert.py"}
    print(json.dumps(line), flush=True)


def run_c2(args):
    """MiniLM forward over batches of 64 packed sequences, one CUDA graph per batch; `value` with the
    batches resident in HBM, `e2e` with each batch's ids copied from pinned host memory and its hidden
    states [rows, 384] f32 read back; replicas on N GPUs (no collective)."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from sejong_b200 import bert, distributed
    rank, world, local, pg = distributed.init_from_env("nccl", timeout_s=300)
    torch.cuda.set_device(local)
    c = bert.MiniLMConfig()
    m = bert.MiniLM(c, device=local)
    total = args.warmup + args.steps
    cap = C2_BATCH * 128
    packed = [bert.pack(bert.synthetic_batch(distributed.rank_seed(3000, rank) + i, C2_BATCH)) for i in range(total)]
    rows = [len(ids) for ids, _ in packed]
    host_ids = torch.zeros(total, cap, dtype=torch.int32).pin_memory()
    host_cu = torch.zeros(total, C2_BATCH + 1, dtype=torch.int32).pin_memory()
    for i, (ids, cu) in enumerate(packed):
        host_ids[i, :len(ids)] = torch.from_numpy(ids)
        host_cu[i] = torch.from_numpy(cu)
    dev_ids, dev_cu = host_ids.to(m.dev), host_cu.to(m.dev)
    host_out = torch.empty(cap, c.hidden, dtype=torch.float32).pin_memory()
    m.reserve(cap)
    m.forward(dev_ids[0, :rows[0]], dev_cu[0])  # eager first pass: kernel attributes, checks the path runs
    torch.cuda.synchronize()
    s = torch.cuda.Stream(m.dev)
    s.wait_stream(torch.cuda.current_stream(m.dev))
    graphs = []
    launches0 = m.launches
    with torch.cuda.stream(s):
        for i in range(total):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                m.forward(dev_ids[i, :rows[i]], dev_cu[i], stream=s.cuda_stream)
            graphs.append(g)
    per_forward = (m.launches - launches0) // total
    torch.cuda.current_stream(m.dev).wait_stream(s)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=m.dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    clocks = ClockSampler(local)
    clocks.start()
    for i in range(args.warmup):
        graphs[i].replay()
    barrier()
    time.sleep(0.3)
    barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for i in range(args.warmup, total):
        graphs[i].replay()
    t1.record(stream)
    barrier()
    dev_ms = max_over_ranks(t0.elapsed_time(t1))
    h2d = d2h = 0
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    e0.record(stream)
    for i in range(args.warmup, total):
        dev_ids[i, :rows[i]].copy_(host_ids[i, :rows[i]], non_blocking=True)
        dev_cu[i].copy_(host_cu[i], non_blocking=True)
        graphs[i].replay()
        host_out[:rows[i]].copy_(m.x[:rows[i]], non_blocking=True)
        h2d += rows[i] * 4 + (C2_BATCH + 1) * 4
        d2h += rows[i] * c.hidden * 4
    e1.record(stream)
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    clk = clocks.stop()
    code = ctypes.c_int(0)
    from sejong_b200._lib import call
    call("sj_device_error", ctypes.byref(code), 0, None)
    assert code.value == 0, f"device error {code.value} during the benchmark"
    assert torch.isfinite(host_out[:rows[-1]]).all(), "non-finite hidden states"

    # GEMM family: one eager forward with CUDA events around each GEMM call
    gemm = {"ms": 0.0, "flops": 0.0, "calls": 0}
    original = m._call
    recs = []

    def timed(name, *a):
        if name != "sj_gemm_bias":
            return original(name, *a)
        e_s, e_e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e_s.record(stream)
        original(name, *a)
        e_e.record(stream)
        recs.append((e_s, e_e, 2.0 * a[9] * a[10] * a[11]))

    torch.cuda.synchronize()
    torch.cuda._sleep(100_000_000)
    m._call = timed
    try:
        m.forward(dev_ids[0, :rows[0]], dev_cu[0])
    finally:
        m._call = original
    torch.cuda.synchronize()
    for e_s, e_e, fl in recs:
        gemm["ms"] += e_s.elapsed_time(e_e)
        gemm["flops"] += fl
        gemm["calls"] += 1
    for g in graphs:
        g.reset()
    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return
    K = args.steps
    tokens = sum(rows[args.warmup:]) * world
    pk = peaks()
    flops = sum(m.flops(packed[i][1]) for i in range(args.warmup, total)) / K
    ms = dev_ms / K
    achieved = gemm["flops"] / (gemm["ms"] / 1e3) / 1e12
    line = {
        "metric": C2_METRIC, "value": tokens / (dev_ms / 1e3), "unit": C2_UNIT, "n_gpus": world, "steps": K,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic ids per BASELINE C2 (reference Rng, seed 3000+rank+step); random-init N(0,0.02) weights",
        "config": {"workload": C2_WORKLOAD, "global_batch": C2_BATCH * world, "per_gpu_batch": C2_BATCH,
                   "seq_len": 128, "mean_tokens_per_step": sum(rows[args.warmup:]) / K, "parallelism": f"replicas{world}",
                   "l2": "weights and activations of one forward fit in L2 across replays; no flush"},
        "e2e": {"value": tokens / (e2e_ms / 1e3), "unit": C2_UNIT, "h2d_bytes_per_step": h2d // K,
                "d2h_bytes_per_step": d2h // K},
        "gpu_launches": per_forward * K,
        "roofline": {"bound": "tensor", "kernel": "gemm_tcgen05 with bias epilogues (all GEMMs of one forward)",
                     "achieved": achieved, "peak": pk["bf16"], "unit": "TFLOP/s", "frac": achieved / pk["bf16"],
                     "peak_source": pk["source"] + " bf16 (burst)", "traffic": None, "launches": gemm["calls"],
                     "ms_per_step": gemm["ms"]},
        "tensor_frac_of_step": flops / (ms / 1e3) / (pk["bf16"] * 1e12),
        "step_tflop": flops / 1e12,
    }
    if clk:
        line["clocks"] = clk
    if world == 1 and not args.no_cpu_baseline:
        rate, _, ctoks, cores = c2_cpu_rate()
        line["cpu_baseline"] = {"value": rate, "unit": C2_UNIT, "cores": cores, "kind": "port",
                                "sample": f"one C2 batch ({C2_CPU_SEQS} sequences, {ctoks} tokens), fp32 torch CPU "
                                          f"restatement, one sequence at a time, mean of {C2_CPU_PASSES} passes"}
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def main():
    args = parse()
    if args.config == "c2":
        if args.impl == "reference":
            run_c2_reference(args)
        else:
            run_c2(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
