"""Model artifacts in the reference's layout: a directory holding `manifest.json`,
`weights.safetensors` and, for a training checkpoint, `optimizer.safetensors`.

Restates:
* `Model::save` (crates/sejong-model/src/lib.rs:395-442): the directory must not exist; files are
  written into a staging directory `.<name>.<pid>.tmp` beside it, which is renamed into place
  (and removed when anything fails);
* `save_tensors` / `load_tensors` (lib.rs:457-538): F32 (or F64) tensors under the reference's
  parameter names; loading rejects other dtypes and non-finite values;
* `Model::load` (lib.rs:134-170): tensor count and every shape must match the configuration;
* `Manifest` (crates/sejong-core/src/lib.rs:547-577): format 1, file names local basenames;
* `save_training` (crates/sejong-train/src/lib.rs:472-491) and `Adam::tensors`
  (lib.rs:239-246): the training config, data fingerprint and the data generator's state word in
  the manifest; AdamW moments as `m.<name>` / `v.<name>`.

The safetensors container is written here (no dependency): an 8-byte little-endian header length,
a compact JSON header listing the tensors in the order the safetensors serializer uses (wider
dtypes first, then by name) with `[begin, end)` byte offsets, padded with spaces to a multiple of
8 bytes, then the little-endian data.  Files are byte-identical to those of the reference's
serializer for the same tensors.
"""
import json
import os
import shutil
import struct
from dataclasses import asdict

import numpy as np

from .model import ExpertConfig, HierarchyConfig, ModelConfig, reference_layout

FORMAT = 1
WEIGHTS = "weights.safetensors"
OPTIMIZER = "optimizer.safetensors"
MANIFEST = "manifest.json"

_DTYPES = {"F64": np.dtype("<f8"), "F32": np.dtype("<f4")}
_DTYPE_RANK = {"F64": 1, "F32": 0}   # serializer order: wider dtype first


class ArtifactError(ValueError):
    """A malformed or mismatching artifact (the reference's Error::Message)."""


# ---------------------------------------------------------------------------------- safetensors
def write_safetensors(path, tensors, metadata=None):
    """Write {name: f32 or f64 array} to `path` (safetensors format)."""
    items = []
    for name, value in tensors.items():
        arr = np.asarray(value)
        if arr.dtype == np.float64:
            tag = "F64"
        elif arr.dtype == np.float32:
            tag = "F32"
        else:
            raise ArtifactError(f"tensor {name}: dtype {arr.dtype} is not f32 or f64")
        items.append((name, tag, np.ascontiguousarray(arr, dtype=_DTYPES[tag])))
    items.sort(key=lambda it: (-_DTYPE_RANK[it[1]], it[0]))
    header = {}
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    offset = 0
    for name, tag, arr in items:
        header[name] = {"dtype": tag, "shape": list(arr.shape), "data_offsets": [offset, offset + arr.nbytes]}
        offset += arr.nbytes
    text = json.dumps(header, separators=(",", ":")).encode()
    text += b" " * (-len(text) % 8)
    with open(path, "wb") as fh:
        fh.write(struct.pack("<Q", len(text)))
        fh.write(text)
        for _, _, arr in items:
            fh.write(arr.tobytes())


def read_safetensors(path):
    """{name: array} from a safetensors file; only F32 and F64 tensors are accepted."""
    with open(path, "rb") as fh:
        raw = fh.read()
    if len(raw) < 8:
        raise ArtifactError(f"{path}: truncated header")
    n = struct.unpack("<Q", raw[:8])[0]
    if 8 + n > len(raw):
        raise ArtifactError(f"{path}: header length {n} beyond the file")
    header = json.loads(raw[8:8 + n])
    data = memoryview(raw)[8 + n:]
    out = {}
    for name, info in header.items():
        if name == "__metadata__":
            continue
        tag = info["dtype"]
        if tag not in _DTYPES:
            raise ArtifactError(f"tensor {name} requires F32 storage")
        begin, end = info["data_offsets"]
        shape = tuple(int(s) for s in info["shape"])
        count = int(np.prod(shape)) if shape else 1
        if not (0 <= begin <= end <= len(data)) or end - begin != count * _DTYPES[tag].itemsize:
            raise ArtifactError(f"tensor {name}: data offsets do not match its shape")
        arr = np.frombuffer(data[begin:end], dtype=_DTYPES[tag]).reshape(shape).copy()
        if not np.all(np.isfinite(arr)):
            raise ArtifactError(f"tensor {name} contains nonfinite values")
        out[name] = arr
    return out


# ---------------------------------------------------------------------------------- configs
def model_config_json(c, model_id="sejong", precision="f16"):
    """ModelConfig as the reference serialises it (crates/sejong-core/src/lib.rs:60-106).  The
    `precision` field names the reference's compute dtype; this build computes in bf16 whatever
    it says."""
    out = {"id": model_id, "width": c.width, "layers": c.layers, "heads": c.heads, "ffn_width": c.ffn_width,
           "context": c.context, "rope_theta": float(c.rope_theta), "norm_epsilon": float(c.norm_epsilon),
           "precision": precision, "seed": int(c.seed)}
    if c.hierarchy is not None:
        h = asdict(c.hierarchy)
        h["checkpoint_encoder"] = False
        h["checkpoint_decoder"] = False
        out["hierarchy"] = h
    if c.kv_heads is not None:
        out["kv_heads"] = c.kv_heads
    if c.experts is not None:
        out["experts"] = asdict(c.experts)
    return out


def model_config_from_json(m, init_std=0.0):
    """ModelConfig from a manifest's `model` object (reference defaults for absent fields)."""
    h = m.get("hierarchy")
    e = m.get("experts")
    hier = None
    if h is not None:
        hier = HierarchyConfig(h["patch_size"], h["encoder_width"], h["encoder_layers"], h["encoder_heads"],
                               h["encoder_ffn_width"], h["decoder_width"], h["decoder_layers"], h["decoder_heads"],
                               h["decoder_ffn_width"], h["local_window"])
    return ModelConfig(width=m.get("width", 512), layers=m.get("layers", 8), heads=m.get("heads", 8),
                       ffn_width=m.get("ffn_width", 1536), kv_heads=m.get("kv_heads"), context=m.get("context", 2048),
                       rope_theta=m.get("rope_theta", 10000.0), norm_epsilon=m.get("norm_epsilon", 1.1920929e-07),
                       hierarchy=hier, experts=None if e is None else ExpertConfig(e["count"], e["top_k"], e["ffn_width"]),
                       seed=m.get("seed", 42), init_std=init_std)


def train_config_json(tc):
    """TrainConfig as the reference serialises it (crates/sejong-core/src/lib.rs:308-362); fields this
    build does not use keep the reference defaults."""
    cv = getattr(tc, "control_variate", None)
    out = {"optimizer": tc.optimizer, "control_variate": None if cv is None else {
        "controls": int(cv.controls), "rank": int(cv.rank), "sampling": str(cv.sampling), "strata": int(cv.strata),
        "basis_refresh": int(cv.basis_refresh), "predictor_learning_rate": float(cv.predictor_learning_rate)}}
    if tc.parameter_vjp is not None:
        v = tc.parameter_vjp
        out["parameter_vjp"] = {"rank": v.rank, "residual_fraction": float(v.residual_fraction),
                                "block_rows": v.block_rows, "seed": int(v.seed)}
    out.update({"gradient_diagnostics_every": 0, "activation_checkpointing": False, "steps": tc.steps,
                "sequence": tc.sequence, "batch": tc.batch, "accumulation": int(getattr(tc, "accumulation", 1)),
                "learning_rate": float(tc.learning_rate), "min_learning_rate": float(tc.min_learning_rate),
                "warmup_steps": tc.warmup_steps, "beta1": float(tc.beta1), "beta2": float(tc.beta2),
                "epsilon": float(tc.epsilon), "weight_decay": float(tc.weight_decay),
                "clip_norm": float(tc.clip_norm), "clip_enabled": bool(tc.clip_enabled),
                "loss_scale": float(tc.loss_scale), "checkpoint_every": int(getattr(tc, "checkpoint_every", 500)),
                "log_every": int(getattr(tc, "log_every", 10)), "seed": int(tc.seed)})
    if getattr(tc, "moe_capacity_factor", 0.0) or getattr(tc, "moe_aux_loss_weight", 0.0):
        # this build's MoE additions; absent (and so reference-compatible) when they are off
        out["moe_capacity_factor"] = float(tc.moe_capacity_factor)
        out["moe_aux_loss_weight"] = float(tc.moe_aux_loss_weight)
    out["gradient_diagnostics_every"] = int(getattr(tc, "gradient_diagnostics_every", 0))
    out["activation_checkpointing"] = bool(getattr(tc, "activation_checkpointing", False))
    return out


# ---------------------------------------------------------------------------------- SGD state
SGD_SAMPLING_MIX = 0x38B87C4D9F0A1265   # SgdState::new (control_variate.rs:66-74)
SGD_BASIS_MIX = 0xA41239C507EF68BD


def rng_words(state):
    """rng_tensor (control_variate.rs:42-47): a generator state as four 16-bit words, in f32."""
    state = int(state) & (2**64 - 1)
    return np.array([(state >> (16 * i)) & 0xFFFF for i in range(4)], dtype=np.float32)


def rng_from_words(words, key):
    """read_rng (control_variate.rs:49-64)."""
    w = np.asarray(words)
    if w.shape != (4,):
        raise ArtifactError("RNG state requires four 16-bit words")
    value = 0
    for i, x in enumerate(w.tolist()):
        if not (np.isfinite(x) and 0.0 <= x <= 65535.0 and float(x).is_integer()):
            raise ArtifactError(f"invalid optimizer RNG word in {key}")
        value |= int(x) << (16 * i)
    return value


def sgd_state_tensors(seed, parameter_rng=None):
    """SgdState::tensors for the plain SGD route: sgd.version = [1], the sampling and basis generators
    (never advanced by plain SGD, so still at their seeds) and, with the parameter VJP, its generator."""
    out = {"sgd.version": np.array([1.0], dtype=np.float32),
           "sgd.sampling_rng": rng_words(int(seed) ^ SGD_SAMPLING_MIX),
           "sgd.basis_rng": rng_words(int(seed) ^ SGD_BASIS_MIX)}
    if parameter_rng is not None:
        out["sgd.parameter_rng"] = rng_words(parameter_rng)
    return out


def read_sgd_state(tensors, parameter_vjp):
    """Checks of SgdState::load (control_variate.rs:122-195) for the plain SGD route; returns the
    generator states by key."""
    version = tensors.get("sgd.version")
    if version is None:
        raise ArtifactError("SGD state version missing")
    if np.shape(version) != (1,) or float(np.asarray(version)[0]) != 1.0:
        raise ArtifactError("unsupported SGD state version")
    keys = ["sgd.sampling_rng", "sgd.basis_rng"] + (["sgd.parameter_rng"] if parameter_vjp else [])
    out = {}
    for k in keys:
        if k not in tensors:
            raise ArtifactError(f"missing optimizer state {k}")
        out[k] = rng_from_words(tensors[k], k)
    if len(tensors) != 1 + len(keys):
        raise ArtifactError("SGD checkpoint tensor count differs from its configuration")
    return out


# ---------------------------------------------------------------------------------- artifacts
def _check_basename(name):
    if not name or os.path.basename(name) != name or name in (".", ".."):
        raise ArtifactError("artifact file names must be local basenames")


def save(directory, config, params, step, optimizer=None, training=None, data_fingerprint=None,
         rng_state=None, model_id="sejong", precision="f16"):
    """Write an artifact directory atomically.

    params: {reference name: f32 array} for every tensor of the configuration's layout;
    optimizer: optional {"m.<name>" / "v.<name>": f32 array}; training: a train_config_json dict."""
    directory = os.path.abspath(directory)
    if os.path.exists(directory):
        raise ArtifactError(f"artifact destination already exists: {directory}")
    expected = reference_layout(config)
    if set(params) != {n for n, _, _ in expected}:
        raise ArtifactError("parameters differ from the configuration's layout")
    for name, shape, _ in expected:
        if tuple(np.shape(params[name])) != tuple(shape):
            raise ArtifactError(f"tensor {name} shape differs from configuration")
    parent = os.path.dirname(directory)
    os.makedirs(parent, exist_ok=True)
    staging = os.path.join(parent, f".{os.path.basename(directory)}.{os.getpid()}.tmp")
    os.mkdir(staging)
    try:
        manifest = {"format": FORMAT, "model": model_config_json(config, model_id, precision), "step": int(step),
                    "weights": WEIGHTS, "optimizer": None, "training": training,
                    "data_fingerprint": data_fingerprint, "rng_state": None if rng_state is None else int(rng_state)}
        write_safetensors(os.path.join(staging, WEIGHTS), {n: np.asarray(params[n], np.float32) for n in params})
        if optimizer is not None:
            manifest["optimizer"] = OPTIMIZER
            write_safetensors(os.path.join(staging, OPTIMIZER), optimizer)
        with open(os.path.join(staging, MANIFEST), "w") as fh:
            json.dump(manifest, fh, indent=2)
        os.rename(staging, directory)
    except BaseException:
        shutil.rmtree(staging, ignore_errors=True)
        raise
    return manifest


def load_manifest(directory):
    with open(os.path.join(directory, MANIFEST)) as fh:
        m = json.load(fh)
    if m.get("format") != FORMAT:
        raise ArtifactError(f"unsupported artifact format {m.get('format')}")
    _check_basename(m["weights"])
    if m.get("optimizer") is not None:
        _check_basename(m["optimizer"])
    return m


def load(directory, init_std=0.0):
    """(config, {name: f32 array}, manifest, optimizer tensors or None) of an artifact directory."""
    m = load_manifest(directory)
    config = model_config_from_json(m["model"], init_std)
    tensors = read_safetensors(os.path.join(directory, m["weights"]))
    expected = reference_layout(config)
    if len(tensors) != len(expected):
        raise ArtifactError("model tensor count differs from configuration")
    params = {}
    for name, shape, _ in expected:
        if name not in tensors:
            raise ArtifactError(f"missing tensor {name}")
        v = tensors[name]
        if tuple(v.shape) != tuple(shape) or v.dtype != np.float32:
            raise ArtifactError(f"tensor {name} shape or dtype differs from configuration")
        params[name] = v
    optimizer = None
    if m.get("optimizer") is not None:
        optimizer = read_safetensors(os.path.join(directory, m["optimizer"]))
    return config, params, m, optimizer
