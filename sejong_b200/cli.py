"""Command line of this build: `python -m sejong_b200 <command>`, the reference's `sejong` binary for the
training step (crates/sejong-cli/src/main.rs:20-164 commands, 165-407 dispatch).

  train        Train from UTF-8 text files; resume with the saved optimizer and RNG
               (main.rs:319-333 -> sejong_train::train, crates/sejong-train/src/lib.rs:300-471 for AdamW,
               control_variate.rs:417-895 for the SGD / parameter-VJP route).  Writes config.json,
               metrics.jsonl (one JSON record at step 1, every log_every steps and at the last step),
               checkpoints/step-XXXXXXXX every checkpoint_every steps, model/ and execution.json.
  train-value  Train a NativeValue head and body over request states (main.rs:219-228 ->
               crates/sejong-train/src/memory.rs:799-1065): checkpoints/value-XXXXXXXX (original/,
               optimizer.safetensors, training.json) and model/.
  benchmark    Measure training, held-out bits per byte and cached decoding for explicit configurations
               (crates/sejong-cli/src/benchmark.rs:173-353): out/run-XXX/ and out/benchmark.json.
  init         Initialise a model and save its weights (main.rs:306-318).
  generate     Generate bytes with the KV cache (main.rs:334-390).
  inspect      Print a model artifact's configuration and provenance (main.rs:391-405).

Every step runs on the GPU through libsejong_b200.so (ByteTrainer); the host loop only draws batches,
reads the loss, gradient norm and learning rate back, and writes the records and artifacts.
"""
import argparse
import ctypes
import json
import os
import sys
import time

import numpy as np


def _eprint(*a):
    print(*a, file=sys.stderr, flush=True)


def _peak_mib(dev):
    import torch
    free, total = torch.cuda.mem_get_info(dev)
    return int((total - free) // 1048576)


class TrainingSummary:
    def __init__(self, steps, last_loss, model_directory):
        self.steps, self.last_loss, self.model_directory = steps, last_loss, model_directory


def _same_training(previous, current):
    """The resume check of lib.rs:339-352: the training configs agree except checkpoint_every and
    log_every."""
    a, b = dict(previous), dict(current)
    for f in ("checkpoint_every", "log_every"):
        a.pop(f, None)
        b.pop(f, None)
    return a == b


def train(cfg, corpus, output, resume=None, measure=False):
    """sejong_train::train_configured (lib.rs:309-471) / control_variate::train_configured
    (control_variate.rs:417-895) on ByteTrainer.  `corpus` is a sejong_b200.corpus.Corpus."""
    import torch

    from . import checkpoint
    from .config import device_of
    from .train import ByteTrainer
    if cfg.training.optimizer == "control_variate_sgd":
        return train_control_variate(cfg, corpus, output, resume, measure)
    complete_started = time.perf_counter()
    tc = cfg.training
    if os.path.exists(output):
        raise checkpoint.ArtifactError(f"training destination already exists: {output}")
    if corpus.count <= tc.sequence:
        raise checkpoint.ArtifactError("corpus is shorter than the training sequence")
    dev = device_of(cfg)
    trainer = ByteTrainer(cfg.model, tc, device=dev)
    rng = ctypes.c_uint64(int(tc.seed))
    if resume is not None:
        manifest = checkpoint.load_manifest(resume)
        if manifest["model"] != checkpoint.model_config_json(cfg.model, cfg.model_id, cfg.precision):
            raise checkpoint.ArtifactError("resume model configuration differs from checkpoint")
        if manifest.get("data_fingerprint") != corpus.fingerprint:
            raise checkpoint.ArtifactError("resume corpus differs from checkpoint")
        if manifest.get("training") is None:
            raise checkpoint.ArtifactError("checkpoint training configuration missing")
        if not _same_training(manifest["training"], checkpoint.train_config_json(tc)):
            raise checkpoint.ArtifactError("resume optimizer, schedule or batch settings differ from checkpoint")
        if manifest.get("rng_state") is None:
            raise checkpoint.ArtifactError("checkpoint RNG state missing")
        trainer.load_checkpoint(resume)
        rng.value = int(manifest["rng_state"])
    step = int(trainer.opt_state[0].item())
    if step >= tc.steps:
        raise checkpoint.ArtifactError("checkpoint already reached the configured training steps")
    os.makedirs(output)
    with open(os.path.join(output, "config.json"), "w") as fh:
        json.dump(cfg.to_json(), fh, indent=2)
    n_params = sum(int(np.prod(s)) for _, s, _ in checkpoint.reference_layout(cfg.model))
    _eprint(f"Sejong {cfg.model_id} | {n_params} parameters | {torch.cuda.get_device_name(trainer.dev)} | "
            f"{corpus.count} corpus tokens")
    acc = max(1, tc.accumulation)
    started = time.perf_counter()
    last_loss = 0.0
    vjp_stats = trainer.vjp_statistics() if trainer.vjp is not None else None
    torch.cuda.synchronize(trainer.dev)
    with open(os.path.join(output, "metrics.jsonl"), "w") as log:
        while step < tc.steps:
            t0 = time.perf_counter()
            for obs in range(acc):
                ids, tg = corpus.batch(rng, tc.batch, tc.sequence)
                trainer.stage_batch(ids, tg)
                trainer.forward_backward(first=obs == 0, last=obs == acc - 1)
            trainer.optimizer_step()
            torch.cuda.synchronize(trainer.dev)
            step_seconds = time.perf_counter() - t0
            if trainer.device_error():
                raise RuntimeError(f"device error {trainer.device_error()} in step {step + 1}")
            loss = trainer.loss()
            hyper = trainer.hyper.cpu().numpy()
            step += 1
            diagnostics = tc.gradient_diagnostics_every > 0 and step % tc.gradient_diagnostics_every == 0
            norm = float(trainer.opt_state[1].item()) if (tc.clip_enabled or diagnostics) else None
            if norm is not None and not np.isfinite(norm):
                raise RuntimeError("nonfinite clipping gradient")
            last_loss = loss
            if step == 1 or step % tc.log_every == 0 or step == tc.steps:
                observed = acc * tc.batch * tc.sequence
                record = {"step": step, "optimizer": tc.optimizer, "loss": loss}
                if tc.optimizer == "sgd":
                    record["loss_estimator"] = "weighted_control_mean"
                record.update({"gradient_norm": norm, "learning_rate": float(hyper[0]), "step_seconds": step_seconds,
                               "observed_bytes": observed, "elapsed_seconds": time.perf_counter() - started})
                if tc.optimizer == "sgd":
                    v = tc.parameter_vjp
                    record["parameter_vjp"] = None if v is None else {
                        "rank": v.rank, "residual_fraction": v.residual_fraction, "block_rows": v.block_rows,
                        "seed": v.seed}
                    record["parameter_vjp_statistics"] = vjp_stats or {
                        "compressed_matrices": 0, "dense_matrices": 0, "basis_groups": 0, "projection_groups": 0}
                    compressed = bool(vjp_stats and vjp_stats["compressed_matrices"])
                    record.update({"exact_bytes": None if compressed else observed, "backward_bytes": observed,
                                   "controls": acc, "basis_refreshed": False,
                                   "basis_source": "control_gradient_contrast" if acc > 1 else "control_gradient",
                                   "gradient_diagnostics": diagnostics})
                else:
                    record["exact_bytes"] = observed
                record["peak_gpu_mib"] = _peak_mib(trainer.dev)
                record["counters"] = {"launches": trainer.launches} if measure else None
                log.write(json.dumps(record) + "\n")
                log.flush()
                _eprint(json.dumps(record))
            if tc.checkpoint_every > 0 and step % tc.checkpoint_every == 0 and step < tc.steps:
                trainer.save_checkpoint(os.path.join(output, "checkpoints", f"step-{step:08d}"), corpus.fingerprint,
                                        rng.value, cfg.model_id, cfg.precision)
    model_dir = os.path.join(output, "model")
    trainer.save_checkpoint(model_dir, corpus.fingerprint, rng.value, cfg.model_id, cfg.precision)
    with open(os.path.join(output, "execution.json"), "w") as fh:
        json.dump({"elapsed_seconds": time.perf_counter() - complete_started, "metrics_collected": bool(measure),
                   "scope": "initialization_training_checkpoint_and_save", "launches": trainer.launches}, fh,
                  indent=2)
    trainer.close()
    return TrainingSummary(step, last_loss, model_dir)


def train_control_variate(cfg, corpus, output, resume=None, measure=False):
    """control_variate::train_configured (control_variate.rs:417-895) for optimizer
    "control_variate_sgd": per step `accumulation` corpus batches through ControlVariateTrainer, the
    reference's metrics.jsonl record, and checkpoints holding the flushed weights with the SGD and
    control-variate state (SgdState::tensors)."""
    import torch

    from . import checkpoint
    from .config import device_of
    from .control_variate import ControlVariateTrainer
    complete_started = time.perf_counter()
    tc = cfg.training
    if os.path.exists(output):
        raise checkpoint.ArtifactError(f"training destination already exists: {output}")
    if corpus.count <= tc.sequence:
        raise checkpoint.ArtifactError("corpus is shorter than the training sequence")
    dev = device_of(cfg)
    rng = ctypes.c_uint64(int(tc.seed))
    params, state, step = None, None, 0
    if resume is not None:
        manifest = checkpoint.load_manifest(resume)
        if manifest["model"] != checkpoint.model_config_json(cfg.model, cfg.model_id, cfg.precision):
            raise checkpoint.ArtifactError("resume model configuration differs from checkpoint")
        if manifest.get("data_fingerprint") != corpus.fingerprint:
            raise checkpoint.ArtifactError("resume corpus differs from checkpoint")
        if manifest.get("training") is None:
            raise checkpoint.ArtifactError("checkpoint training configuration missing")
        if not _same_training(manifest["training"], checkpoint.train_config_json(tc)):
            raise checkpoint.ArtifactError("resume SGD, predictor, schedule or batch settings differ from checkpoint")
        if manifest.get("rng_state") is None:
            raise checkpoint.ArtifactError("checkpoint corpus RNG state missing")
        _, params, manifest, state = checkpoint.load(resume, cfg.model.init_std)
        if state is None:
            raise checkpoint.ArtifactError("resume requires SGD optimizer state")
        rng.value = int(manifest["rng_state"])
        step = int(manifest["step"])
    trainer = ControlVariateTrainer(cfg.model, tc, tc.control_variate, device=dev, params=params)
    if state is not None:
        trainer.load_state_tensors(state)
        trainer.step_count = step
        trainer.tr.opt_state[0] = float(step)
    if step >= tc.steps:
        raise checkpoint.ArtifactError("checkpoint already reached configured training steps")
    os.makedirs(output)
    with open(os.path.join(output, "config.json"), "w") as fh:
        json.dump(cfg.to_json(), fh, indent=2)

    def save(directory):
        params_now, tensors = trainer.snapshot()
        checkpoint.save(directory, cfg.model, params_now, trainer.step_count, tensors,
                        checkpoint.train_config_json(tc), corpus.fingerprint, rng.value, model_id=cfg.model_id,
                        precision=cfg.precision)

    acc = tc.accumulation
    started = time.perf_counter()
    last_loss = 0.0
    with open(os.path.join(output, "metrics.jsonl"), "w") as log:
        while step < tc.steps:
            t0 = time.perf_counter()
            observations = [corpus.batch(rng, tc.batch, tc.sequence) for _ in range(acc)]
            m = trainer.step(observations)
            step_seconds = time.perf_counter() - t0
            if trainer.tr.device_error():
                raise RuntimeError(f"device error {trainer.tr.device_error()} in step {step + 1}")
            step = trainer.step_count
            last_loss = m["loss"]
            if step == 1 or step % tc.log_every == 0 or step == tc.steps:
                controls = m["controls"]
                backward = controls * tc.batch * tc.sequence
                diag = m["gradient_diagnostics"]
                record = {"step": step, "optimizer": tc.optimizer, "loss": m["loss"],
                          "loss_estimator": "weighted_control_mean", "gradient_norm": m["gradient_norm"],
                          "parameter_vjp": None,
                          "parameter_vjp_statistics": {"compressed_matrices": 0, "dense_matrices": 0,
                                                       "basis_groups": 0, "projection_groups": 0},
                          "learning_rate": m["learning_rate"], "step_seconds": step_seconds,
                          "elapsed_seconds": time.perf_counter() - started,
                          "observed_bytes": acc * tc.batch * tc.sequence, "exact_bytes": backward,
                          "backward_bytes": backward, "controls": controls,
                          "basis_refreshed": m["basis_refreshed"],
                          "basis_source": "control_gradient_contrast" if controls > 1 else "control_gradient",
                          "gradient_diagnostics": diag,
                          "diagnostic_seconds": m.get("diagnostic_seconds") if diag else None,
                          "predictor_mse": m.get("predictor_mse") if diag else None,
                          "control_gradient_dispersion": m.get("control_gradient_dispersion") if diag else None,
                          "control_residual_dispersion": m.get("control_residual_dispersion") if diag else None,
                          "residual_variance_ratio_diagnostic":
                              m.get("residual_variance_ratio_diagnostic") if diag else None,
                          "peak_gpu_mib": _peak_mib(trainer.tr.dev),
                          "counters": {"launches": trainer.tr.launches} if measure else None}
                log.write(json.dumps(record) + "\n")
                log.flush()
                _eprint(json.dumps(record))
            if tc.checkpoint_every > 0 and step % tc.checkpoint_every == 0 and step < tc.steps:
                save(os.path.join(output, "checkpoints", f"step-{step:08d}"))
    model_dir = os.path.join(output, "model")
    save(model_dir)
    with open(os.path.join(output, "execution.json"), "w") as fh:
        json.dump({"elapsed_seconds": time.perf_counter() - complete_started, "metrics_collected": bool(measure),
                   "scope": "initialization_training_checkpoint_and_save", "launches": trainer.tr.launches}, fh,
                  indent=2)
    trainer.close()
    torch.cuda.synchronize()
    return TrainingSummary(step, last_loss, model_dir)


# ------------------------------------------------------------------------------------------ train-value
VALUE_FORMAT = "sejong-native-value-v1"
PROGRESS_FORMAT = "sejong-local-training-v3"
VALUE_RECIPE = "native-value-resource-batch-explicit-policy-v1"


def _byte_value(x):
    """ByteValue's JSON forms (crates/sejong-core/src/native/bytes.rs): a string, or {"hex": "..."}."""
    if isinstance(x, str):
        return x.encode()
    if isinstance(x, dict) and set(x) == {"hex"}:
        return bytes.fromhex(x["hex"])
    raise ValueError(f"byte value must be a string or {{\"hex\": ...}}, got {x!r}")


def _byte_json(b):
    try:
        return b.decode()
    except UnicodeDecodeError:
        return {"hex": b.hex()}


def value_fingerprint(spec):
    """fingerprint (memory.rs:39-55): BLAKE3 of the compact JSON {"recipe", "specification"} with the
    resume path removed.  The specification is the spec as given; the reference serialises its parsed
    struct, so the digests agree when the spec spells out every field in the struct's order."""
    from .corpus import blake3_hex
    body = {k: v for k, v in spec.items() if k != "resume"}
    text = json.dumps({"recipe": VALUE_RECIPE, "specification": body}, separators=(",", ":"), ensure_ascii=False)
    return blake3_hex([text.encode()])


def _value_settings(spec, batch):
    """OptimizerPolicy::configuration (crates/sejong-core/src/native.rs:467-518) as a TrainConfig."""
    pol = spec.get("optimizer") or {}
    steps, lr, observations = int(spec["steps"]), float(spec["learning_rate"]), len(spec["requests"])
    if steps <= 0 or batch <= 0 or not np.isfinite(lr) or lr <= 0:
        raise ValueError("positive optimizer dimensions and learning rate required")

    def effective(examples):
        if examples <= 0:
            raise ValueError("optimizer memory horizon must be positive")
        h = float(-(-examples // batch))
        return min(float(np.float32((h - 1.0) / (h + 1.0))), float(np.nextafter(np.float32(1), np.float32(0))))

    beta1 = effective(pol.get("momentum_examples") or observations)
    beta2 = effective(pol.get("variance_examples") or steps * batch)
    clip = pol.get("clip_norm")
    return dict(steps=steps, learning_rate=lr, min_learning_rate=lr, warmup_steps=0, beta1=beta1, beta2=beta2,
                epsilon=float(pol.get("epsilon") or 0.0), weight_decay=float(pol.get("weight_decay", 0.0)),
                clip_enabled=clip is not None, clip_norm=float(clip or 0.0), loss_scale=1.0)


def _atomic_directory(path, write):
    import shutil
    parent = os.path.dirname(os.path.abspath(path))
    os.makedirs(parent, exist_ok=True)
    if os.path.exists(path):
        raise FileExistsError(f"output already exists: {path}")
    staging = os.path.join(parent, f".{os.path.basename(path)}.{os.getpid()}.tmp")
    os.mkdir(staging)
    try:
        write(staging)
        os.rename(staging, path)
    except BaseException:
        shutil.rmtree(staging, ignore_errors=True)
        raise


def _value_signature(params, metadata):
    """This build's seal of a trained NativeValue: BLAKE3 over the metadata JSON and every tensor's
    name, shape and f32 bytes (the reference computes its own signature the same way in spirit,
    value.rs:160-215; the digests are not meant to agree)."""
    from .corpus import blake3_hex
    parts = [json.dumps(metadata, sort_keys=True).encode()]
    for name in sorted(params):
        a = np.ascontiguousarray(params[name], dtype=np.float32)
        parts += [name.encode(), json.dumps(list(a.shape)).encode(), a.tobytes()]
    return blake3_hex(parts)


def _write_value(directory, cfg_model, model_id, precision, params, metadata, values):
    """NativeValue::write (value.rs:199-216): body/ (a model artifact), native.safetensors
    (embedding [259, d], value [d, n], bias [1, n]) and value.json."""
    from . import checkpoint
    from .model import reference_layout
    body_names = {n for n, _, _ in reference_layout(cfg_model)}
    body = {n: params[n] for n in body_names if n in params}
    # the value body has no byte embedding / head of its own: the reference's Model still stores them
    for n, shape, _ in reference_layout(cfg_model):
        if n not in body:
            body[n] = np.zeros(shape, dtype=np.float32)
    checkpoint.save(os.path.join(directory, "body"), cfg_model, body, metadata["steps"], model_id=model_id,
                    precision=precision)
    checkpoint.write_safetensors(os.path.join(directory, "native.safetensors"),
                                 {"embedding": params["native_embedding"], "value": params["native_value"],
                                  "bias": np.asarray(params["native_bias"], np.float32).reshape(1, values)})
    with open(os.path.join(directory, "value.json"), "w") as fh:
        json.dump(metadata, fh, indent=2)


def _read_value(directory, cfg_model):
    from . import checkpoint
    with open(os.path.join(directory, "value.json")) as fh:
        metadata = json.load(fh)
    if metadata.get("format") != VALUE_FORMAT:
        raise checkpoint.ArtifactError("native value format mismatch")
    _, body, _, _ = checkpoint.load(os.path.join(directory, "body"), cfg_model.init_std)
    native = checkpoint.read_safetensors(os.path.join(directory, "native.safetensors"))
    n = len(metadata["values"])
    d = cfg_model.width
    want = {"embedding": (259, d), "value": (d, n), "bias": (1, n)}
    if set(native) != set(want) or any(tuple(native[k].shape) != s for k, s in want.items()):
        raise checkpoint.ArtifactError("native value tensor contract mismatch")
    params = dict(body)
    params["native_embedding"] = native["embedding"]
    params["native_value"] = native["value"]
    params["native_bias"] = native["bias"].reshape(n)
    return params, metadata


def train_value(spec, out, resume=None, device=0):
    """train_value (memory.rs:799-1065) on ByteTrainer in NativeValue mode: AdamW or SGD, either with
    exact gradients or with the parameter VJP; the batch from the planner over the device's
    free memory; checkpoints/value-XXXXXXXX/ {original/, optimizer.safetensors, training.json} every
    checkpoint_every steps and at the end; model/ (sealed) last."""
    import torch

    from . import checkpoint, planner
    from . import value as pv
    from .config import model_from_table
    from .param_vjp import VjpConfig
    from .train import ByteTrainer, TrainConfig
    kind = spec.get("optimizer_kind", "adamw")
    if kind not in ("adamw", "sgd"):
        raise ValueError("native value optimizer requires adamw or sgd")
    pol = spec.get("optimizer") or {}
    if kind == "sgd" and any(pol.get(k) is not None for k in ("momentum_examples", "variance_examples", "epsilon")):
        raise ValueError("native SGD uses weight_decay and clip_norm; moment options require adamw")
    requests = [_byte_value(x) for x in spec["requests"]]
    prompts = [_byte_value(x) for x in spec["prompts"]]
    values = [_byte_value(x) for x in spec["values"]]
    labels = [int(x) for x in spec["labels"]]
    for name, xs in (("requests", requests), ("values", values)):
        if not xs or len(set(xs)) != len(xs) or any(len(x) == 0 for x in xs):
            raise ValueError(f"native {name} requires unique nonempty byte entries")
    if len(labels) != len(requests) or any(not 0 <= l < len(values) for l in labels) or len(prompts) != len(requests):
        raise ValueError("native value labels invalid")
    model_table = dict(spec["model"])
    c, model_id, precision = model_from_table(model_table)
    vjp = None
    if spec.get("parameter_vjp") is not None:
        p = spec["parameter_vjp"]
        # with AdamW the factored gradient is materialised into the dense gradient buffer before the
        # update (GradientMaterializer, crates/sejong-gpu/src/parameter_vjp.rs:347-380); with SGD it is
        # applied the same way and the update is the compact one
        vjp = VjpConfig(rank=int(p.get("rank", 16)), residual_fraction=float(p.get("residual_fraction", 0.25)),
                        block_rows=int(p.get("block_rows", 32)), seed=int(p.get("seed", 124)))
    source = value_fingerprint(spec)
    if os.path.exists(out):
        raise FileExistsError(f"output already exists: {out}")
    saved = None
    if resume is not None:
        with open(os.path.join(resume, "training.json")) as fh:
            saved = json.load(fh)
        if saved.get("format") != PROGRESS_FORMAT or saved.get("source") != source:
            raise checkpoint.ArtifactError("native value checkpoint source mismatch")
        if saved.get("phase") != "value":
            raise checkpoint.ArtifactError("native value checkpoint phase mismatch")
    torch.cuda.set_device(device)
    batch_policy = spec.get("batch") or {}
    plan = planner.plan(c, prompts, len(values), len(requests), planner.available_bytes(device),
                        memory_bytes=batch_policy.get("memory_bytes"), max_examples=batch_policy.get("max_examples"),
                        activation_checkpointing=spec.get("activation_checkpointing"),
                        saved=None if saved is None else (int(saved["batch_size"]),
                                                          bool(saved.get("activation_checkpointing", True))))
    batch = plan.batch
    settings = _value_settings(spec, batch)
    seq = pv.sequence_for(c, prompts)
    tc = TrainConfig(sequence=seq, batch=batch, optimizer=kind, values=len(values), parameter_vjp=vjp,
                     activation_checkpointing=plan.checkpointing, **settings)
    metadata = {"format": VALUE_FORMAT, "requests": [_byte_json(x) for x in requests],
                "prompts": [_byte_json(x) for x in prompts], "values": [_byte_json(x) for x in values],
                "model": checkpoint.model_config_json(c, model_id, precision), "steps": 0, "source_hash": source,
                "loss": 0.0}
    params = None
    if resume is not None:
        params, meta = _read_value(os.path.join(resume, "original"), c)
        if meta.get("source_hash") != source:
            raise checkpoint.ArtifactError("native value checkpoint source mismatch")
        metadata.update(steps=meta["steps"], loss=meta["loss"])
    trainer = ByteTrainer(c, tc, device=device, params=params)
    rng = pv.sampler(c.seed)
    start = 0
    if saved is not None:
        start = int(saved["step"])
        rng.value = int(saved["rng"])
        if kind == "adamw":
            opt = checkpoint.read_safetensors(os.path.join(resume, "optimizer.safetensors"))
            for prefix, buf in (("m", trainer.m), ("v", trainer.v)):
                named = {k[len(prefix) + 1:]: v for k, v in opt.items() if k.startswith(prefix + ".")}
                buf.copy_(torch.from_numpy(trainer.layout.pack(named)).to(trainer.dev))
            trainer.opt_state[0] = float(saved["optimizer_step"])
        else:
            if int(saved["optimizer_step"]) != start:
                raise checkpoint.ArtifactError("native SGD checkpoint step mismatch")
            trainer.opt_state[0] = float(start)
        if vjp is not None:
            if saved.get("parameter_rng") is None:
                raise checkpoint.ArtifactError("native value checkpoint parameter RNG missing")
            trainer.vjp_rng.copy_(torch.from_numpy(np.array([int(saved["parameter_rng"])], dtype=np.uint64)
                                                   .view(np.int64)).to(trainer.dev))
    if start > tc.steps:
        raise checkpoint.ArtifactError("native value checkpoint step exceeds target")
    os.makedirs(out)
    _eprint(json.dumps({"native_execution": {"optimizer": kind, "batch": batch,
                                             "activation_checkpointing": plan.checkpointing,
                                             "gradient_and_cast_bytes": plan.fixed_bytes,
                                             "activation_and_factor_bytes": plan.workspace_bytes}}))
    every = int(spec.get("checkpoint_every", 0))
    for step in range(start, tc.steps):
        idx = pv.sample_requests(rng, batch, len(requests))
        ids, sel = pv.request_batch([prompts[i] for i in idx], seq)
        trainer.stage_requests(ids, sel, np.array([labels[i] for i in idx], dtype=np.int32))
        trainer.forward_backward()
        trainer.optimizer_step()
        torch.cuda.synchronize(trainer.dev)
        if trainer.device_error():
            raise RuntimeError(f"device error {trainer.device_error()} in native step {step + 1}")
        value = trainer.loss()
        metadata["steps"] = step + 1
        metadata["loss"] = value
        if step == start or (every > 0 and (step + 1) % every == 0) or step + 1 == tc.steps:
            _eprint(f"{model_id} native {step + 1} loss {value:.6f}")
            if vjp is not None:
                _eprint(json.dumps({"step": step + 1, "parameter_vjp_statistics": trainer.vjp_statistics()}))
        if (every > 0 and (step + 1) % every == 0) or step + 1 == tc.steps:
            params_now = trainer.parameters()
            progress = {"format": PROGRESS_FORMAT, "phase": "value", "step": step + 1,
                        "optimizer_step": int(trainer.opt_state[0].item()), "rng": int(rng.value), "source": source,
                        "guard": None, "batch_size": batch, "activation_checkpointing": plan.checkpointing}
            if vjp is not None:
                progress["parameter_rng"] = trainer.vjp_rng_state()

            def write(d, params_now=params_now, progress=progress):
                _write_value(os.path.join(d, "original"), c, model_id, precision, params_now, dict(metadata),
                             len(values))
                if kind == "adamw":
                    opt = {}
                    for prefix, buf in (("m", trainer.m), ("v", trainer.v)):
                        for name, v in trainer.layout.unpack(buf.cpu().numpy()).items():
                            opt[f"{prefix}.{name}"] = v
                    checkpoint.write_safetensors(os.path.join(d, "optimizer.safetensors"), opt)
                with open(os.path.join(d, "training.json"), "w") as fh:
                    json.dump(progress, fh, indent=2)

            _atomic_directory(os.path.join(out, "checkpoints", f"value-{step + 1:08d}"), write)
    final = trainer.parameters()
    seal = _value_signature(final, metadata)

    def write_model(d):
        _write_value(d, c, model_id, precision, final, dict(metadata), len(values))
        with open(os.path.join(d, "signature"), "w") as fh:
            fh.write(seal)

    _atomic_directory(os.path.join(out, "model"), write_model)
    trainer.close()
    return metadata


# ------------------------------------------------------------------------------------------ benchmark
def _distribution(values):
    """distribution (benchmark.rs:99-110)."""
    if not values:
        return None
    o = sorted(values)
    n = len(o)
    return {"samples": n, "mean": sum(values) / n, "median": (o[(n - 1) // 2] + o[n // 2]) / 2.0, "minimum": o[0],
            "maximum": o[-1]}


def evaluate(trainer, corpus, cfg, batches):
    """evaluate (benchmark.rs:71-97): mean held-out cross entropy in bits per byte token over
    `batches` batches drawn from Rng(training.seed)."""
    import torch
    tc = cfg.training
    rng = ctypes.c_uint64(int(tc.seed))
    total = 0.0
    for _ in range(batches):
        ids, tg = corpus.batch(rng, tc.batch, tc.sequence)
        trainer.stage_batch(ids, tg)
        loss = trainer.evaluate()
        torch.cuda.synchronize(trainer.dev)
        if not np.isfinite(loss):
            raise RuntimeError("evaluation produced nonfinite loss")
        total += loss
    return total / batches / np.log(2.0)


def cached_measurement(params, cfg, corpus, decode, device):
    """cached_measurement (benchmark.rs:112-168): prefill of the held-out prefix, then teacher-forced
    byte-by-byte decoding, timed on the second of two passes; the last logits against a fresh prefill
    of the whole input."""
    import torch

    from .generate import Generator
    tc = cfg.training
    rng = ctypes.c_uint64(int(tc.seed))
    ids, _ = corpus.batch(rng, 1, tc.sequence)
    ids = [int(x) for x in ids]
    prefix = len(ids) - decode
    gen = Generator(cfg.model, params=params, device=device, context=tc.sequence)
    full = gen.forward_cached(ids).cpu().numpy().astype(np.float64)
    prefill_seconds, decode_seconds, last = 0.0, [], None
    for attempt in range(2):
        gen.reset()
        torch.cuda.synchronize(gen.dev)
        t0 = time.perf_counter()
        gen.forward_cached(ids[:prefix])
        torch.cuda.synchronize(gen.dev)
        if attempt == 1:
            prefill_seconds = time.perf_counter() - t0
        for tok in ids[prefix:]:
            t0 = time.perf_counter()
            out = gen.forward_cached([tok])
            torch.cuda.synchronize(gen.dev)
            if attempt == 1:
                decode_seconds.append(time.perf_counter() - t0)
            last = out
    last = last.cpu().numpy().astype(np.float64)
    if not np.all(np.isfinite(last)):
        raise RuntimeError("cached inference produced nonfinite logits")
    return {"prefill_tokens": prefix, "decode_tokens": decode, "prefill_seconds": prefill_seconds,
            "decode_seconds_per_token": _distribution(decode_seconds),
            "decode_tokens_per_second": decode / sum(decode_seconds),
            "cached_vs_full_last_logits_max_abs_error": float(np.abs(last - full).max()),
            "measurement": "same held-out input, one cache warmup, synchronized teacher-forced decoding"}


def benchmark(config_paths, data, validation, out, warmup_steps, measure_steps, evaluation_batches, decode_bytes):
    """benchmark::run (benchmark.rs:170-353)."""
    import torch

    from . import checkpoint
    from . import config as cfgmod
    from .corpus import Corpus
    from .model import initialize
    from .train import ByteTrainer
    if measure_steps <= 0 or evaluation_batches <= 0 or decode_bytes <= 0:
        raise ValueError("measurement steps, evaluation batches and decode bytes must be positive")
    if not config_paths:
        raise ValueError("benchmark requires at least one configuration")
    if os.path.exists(out):
        raise FileExistsError("benchmark destination already exists")
    steps = warmup_steps + measure_steps
    val = Corpus.open(validation)
    train_corpus = Corpus.open(data)
    if val.fingerprint == train_corpus.fingerprint:
        raise ValueError("benchmark requires distinct training and validation corpora")
    configs = []
    for path in config_paths:
        cfg = cfgmod.load(path)
        if decode_bytes >= cfg.training.sequence:
            raise ValueError("decode bytes must be smaller than the training sequence")
        if cfg.training.sequence >= val.count:
            raise ValueError("validation corpus must exceed the sequence length")
        cfg.training.steps = steps
        cfg.training.log_every = 1
        configs.append(cfg)
    os.makedirs(out)
    reports = []
    for index, cfg in enumerate(configs):
        dest = os.path.join(out, f"run-{index:03d}")
        dev = cfgmod.device_of(cfg)
        init_params = initialize(cfg.model)
        tr = ByteTrainer(cfg.model, cfg.training, device=dev, params=init_params)
        initial_bpb = evaluate(tr, val, cfg, evaluation_batches)
        tr.close()
        del tr
        n_params = sum(int(np.prod(s)) for _, s, _ in checkpoint.reference_layout(cfg.model))
        device_name = torch.cuda.get_device_name(dev)
        wall = time.perf_counter()
        summary = train(cfg, train_corpus, dest, measure=True)
        complete = time.perf_counter() - wall
        with open(os.path.join(dest, "execution.json")) as fh:
            execution = json.load(fh)
        with open(os.path.join(dest, "metrics.jsonl")) as fh:
            records = [json.loads(line) for line in fh if line.strip()]
        measured = [r for r in records if r["step"] > warmup_steps]
        if len(measured) != measure_steps:
            raise RuntimeError("training metrics must contain every measured step")
        times = [r["step_seconds"] for r in measured]
        observed = sum(r["observed_bytes"] for r in measured)
        exact = sum(r["exact_bytes"] for r in measured) if all(r.get("exact_bytes") is not None
                                                              for r in measured) else None
        backward = sum(r.get("backward_bytes", r.get("exact_bytes")) or 0 for r in measured)
        _, params, _, _ = checkpoint.load(summary.model_directory, cfg.model.init_std)
        tr = ByteTrainer(cfg.model, cfg.training, device=dev, params=params)
        final_bpb = evaluate(tr, val, cfg, evaluation_batches)
        tr.close()
        del tr
        inference = cached_measurement(params, cfg, val, decode_bytes, dev) if cfg.model.experts is None else None
        report = {"config_path": str(config_paths[index]), "config": cfg.to_json(), "device": device_name,
                  "model_parameters": n_params, "training_fingerprint": train_corpus.fingerprint,
                  "validation_fingerprint": val.fingerprint, "evaluation_batches": evaluation_batches,
                  "initial_validation_bits_per_byte_token": initial_bpb,
                  "final_validation_bits_per_byte_token": final_bpb, "warmup_steps": warmup_steps,
                  "measured_steps": measure_steps, "training_step_seconds": _distribution(times),
                  "steps_without_compilation_seconds": _distribution(times), "observed_bytes": observed,
                  "exact_bytes": exact, "backward_bytes": backward,
                  "observed_bytes_per_second": observed / sum(times),
                  "exact_bytes_per_second": None if exact is None else exact / sum(times),
                  "backward_bytes_per_second": backward / sum(times),
                  "complete_training_seconds_including_initialization_and_save": complete,
                  "complete_execution": execution, "build_profile": "release",
                  "flops_scope": "executed GEMM and attention arithmetic of libsejong_b200.so, FMA=2; pointwise and "
                                 "transfers included in wall time",
                  "measured_step_records": measured, "inference": inference,
                  "loss_unit": "cross entropy / ln(2), byte vocabulary with document EOS",
                  "precision_unit_roundoff": 2.0 ** -8}
        with open(os.path.join(dest, "benchmark.json"), "w") as fh:
            json.dump(report, fh, indent=2)
        reports.append(report)
        tmp = os.path.join(out, "benchmark.json.tmp")
        with open(tmp, "w") as fh:
            json.dump({"format": "sejong-measured-benchmark-v1", "training_data": str(data),
                       "validation_data": str(validation), "runs": reports}, fh, indent=2)
            fh.flush()
            os.fsync(fh.fileno())
        os.replace(tmp, os.path.join(out, "benchmark.json"))
    print(os.path.join(out, "benchmark.json"))
    return reports


# ------------------------------------------------------------------------------------------ small commands
def init(cfg, out):
    """Init (main.rs:306-318): initialise the model (reference initialisation) and save it."""
    from . import checkpoint
    from .model import initialize
    params = initialize(cfg.model)
    checkpoint.save(out, cfg.model, params, 0, model_id=cfg.model_id, precision=cfg.precision)
    n = sum(int(np.prod(v.shape)) for v in params.values())
    print(f"{n} parameters saved to {out}")


def inspect(model):
    """Inspect (main.rs:391-405): the manifest of a model artifact."""
    from . import checkpoint
    print(json.dumps(checkpoint.load_manifest(model), indent=2))


def generate(model, prompt, max_bytes, temperature, top_k, top_p, seed, raw=False, device=0):
    """Generate (main.rs:334-390): sample bytes after `prompt` with the KV cache."""
    from . import checkpoint
    from .generate import Generator, Sampling
    config, params, _, _ = checkpoint.load(model)
    gen = Generator(config, params=params, device=device)
    text, _ = gen.generate(prompt.encode(), Sampling(temperature=temperature, top_k=top_k, top_p=top_p, seed=seed,
                                                    max_bytes=max_bytes))
    if raw:
        sys.stdout.buffer.write(text)
        sys.stdout.flush()
    else:
        print(text.decode(errors="replace"))


def main(argv=None):
    ap = argparse.ArgumentParser(prog="python -m sejong_b200", description="Sejong byte-model training on B200")
    sub = ap.add_subparsers(dest="command", required=True)
    p = sub.add_parser("train", help="train from UTF-8 text files; resume with the saved optimizer and RNG")
    p.add_argument("--config", required=True)
    p.add_argument("--data", required=True)
    p.add_argument("--out", required=True)
    p.add_argument("--resume", default=None)
    p = sub.add_parser("train-value", help="train a native value head over request states")
    p.add_argument("--spec", required=True)
    p.add_argument("--out", required=True)
    p.add_argument("--resume", default=None)
    p.add_argument("--device", type=int, default=0)
    p = sub.add_parser("benchmark", help="measure training, held-out loss and cached inference")
    p.add_argument("--config", action="append", required=True)
    p.add_argument("--data", required=True)
    p.add_argument("--validation", required=True)
    p.add_argument("--out", required=True)
    p.add_argument("--warmup-steps", type=int, required=True)
    p.add_argument("--measure-steps", type=int, required=True)
    p.add_argument("--evaluation-batches", type=int, required=True)
    p.add_argument("--decode-bytes", type=int, required=True)
    p = sub.add_parser("init", help="initialise a model and save its weights")
    p.add_argument("--config", required=True)
    p.add_argument("--out", required=True)
    p = sub.add_parser("inspect", help="display a model's configuration and provenance")
    p.add_argument("--model", required=True)
    p = sub.add_parser("generate", help="generate bytes with the KV cache")
    p.add_argument("--model", required=True)
    p.add_argument("--prompt", default="")
    p.add_argument("--max-bytes", type=int, default=512)
    p.add_argument("--temperature", type=float, default=0.8)
    p.add_argument("--top-k", type=int, default=0)
    p.add_argument("--top-p", type=float, default=0.95)
    p.add_argument("--seed", type=int, default=42)
    p.add_argument("--raw", action="store_true")
    a = ap.parse_args(argv)
    from . import config as cfgmod
    if a.command == "train":
        from .corpus import Corpus
        s = train(cfgmod.load(a.config), Corpus.open(a.data), a.out, a.resume)
        print(f"{s.steps} updates | loss {s.last_loss:.6f} | {s.model_directory}")
    elif a.command == "train-value":
        with open(a.spec) as fh:
            spec = json.load(fh)
        resume = a.resume or spec.get("resume")
        train_value(spec, a.out, resume, device=a.device)
        print(os.path.join(a.out, "model"))
    elif a.command == "benchmark":
        benchmark(a.config, a.data, a.validation, a.out, a.warmup_steps, a.measure_steps, a.evaluation_batches,
                  a.decode_bytes)
    elif a.command == "init":
        init(cfgmod.load(a.config), a.out)
    elif a.command == "inspect":
        inspect(a.model)
    elif a.command == "generate":
        generate(a.model, a.prompt, a.max_bytes, a.temperature, a.top_k, a.top_p, a.seed, a.raw)
    return 0
