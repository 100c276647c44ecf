"""NativeValue: the byte model as a categorical value predictor over request prompts.

Restates the host side of `NativeValue` (crates/sejong-model/src/native/value.rs) and of its
training loop `train_value` (crates/sejong-train/src/memory.rs:799-1065) on top of the byte-model
step (`ByteTrainer` with `TrainConfig.values` > 0):

  * `initialize_value`: the 259-row native embedding and the f32 value head drawn from
    Rng(seed ^ 0x76616c7565), each element normal() / sqrt(width), bias 0 (value.rs:39-76);
  * `request_batch`: a batch of prompts laid out as forward_batch does (value.rs:117-137): per
    request BOS (257), the prompt bytes, SEP (258), then PAD (256) to the sequence length; the SEP
    row of each request is the one the head reads;
  * `sample_requests`: the requests of each step, Rng(seed ^ 0x6e6174697665).index(requests)
    (memory.rs:948-956).

The reference pads each batch to its own longest prompt + 2.  Here every step uses one sequence
length (the trainer's buffers and captured graph have fixed shapes), at least the longest prompt
of the inventory + 2 and, for the hierarchical body, a multiple of the patch size.  Every layer is
causal and the global stage sees a patch only from the next patch on, so the rows after a SEP row
change neither its hidden state nor, their loss gradient being zero, any gradient: the extra
padding changes the cost of a step, not its result.
"""
import ctypes

import numpy as np

from . import _lib
from ._lib import call
from .model import NATIVE_BOS, NATIVE_PAD, NATIVE_SEP, value_layout

VALUE_SEED = 0x76616C7565     # "value"
SAMPLE_SEED = 0x6E6174697665  # "native"


def initialize_value(c, values, lib=None):
    """native_embedding [259, width], native_value [width, values] (normal / sqrt(width)), native_bias 0."""
    lib = lib or _lib.load()
    state = ctypes.c_uint64((int(c.seed) ^ VALUE_SEED) & (2**64 - 1))
    scale = np.float32(np.sqrt(np.float32(c.width)))
    out = {}
    for name, shape, _ in value_layout(c, values):
        if name == "native_bias":
            out[name] = np.zeros(shape, dtype=np.float32)
            continue
        buf = np.empty(int(np.prod(shape)), dtype=np.float32)
        call("sj_rng_normal_fill", ctypes.byref(state), buf.ctypes.data, buf.size, 1.0)
        out[name] = (buf / scale).astype(np.float32).reshape(shape)
    return out


def request_batch(prompts, sequence=None):
    """(ids int32 [batch, sequence], sel int32 [batch]) for a list of prompts (bytes or str).

    sel[b] = b * sequence + len(prompt b) + 1, the flat index of request b's SEP row."""
    raw = [p.encode() if isinstance(p, str) else bytes(p) for p in prompts]
    need = max(len(p) for p in raw) + 2
    sequence = need if sequence is None else int(sequence)
    if sequence < need:
        raise ValueError(f"sequence {sequence} shorter than the longest prompt + 2 ({need})")
    ids = np.full((len(raw), sequence), NATIVE_PAD, dtype=np.int32)
    sel = np.empty(len(raw), dtype=np.int32)
    for b, p in enumerate(raw):
        ids[b, 0] = NATIVE_BOS
        ids[b, 1:1 + len(p)] = np.frombuffer(p, dtype=np.uint8)
        ids[b, 1 + len(p)] = NATIVE_SEP
        sel[b] = b * sequence + 1 + len(p)
    return ids, sel


def sample_requests(state, batch, requests):
    """`batch` request indices drawn with Rng::index from the generator state (a ctypes.c_uint64,
    advanced in place); start from `sampler(seed)`."""
    lib = _lib.load()
    return np.array([lib.sj_rng_index(ctypes.byref(state), requests) for _ in range(batch)], dtype=np.int64)


def sampler(seed):
    return ctypes.c_uint64((int(seed) ^ SAMPLE_SEED) & (2**64 - 1))


def sequence_for(config, prompts):
    """The fixed sequence length the trainer uses for an inventory of prompts: longest + 2, rounded up
    to a multiple of the patch size (hierarchical body) and of 8."""
    need = max(len(p.encode() if isinstance(p, str) else p) for p in prompts) + 2
    unit = 8
    if config.hierarchy is not None:
        unit = int(np.lcm(unit, config.hierarchy.patch_size))
    return -(-need // unit) * unit
