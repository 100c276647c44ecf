"""Memory-budgeted batch planner of the NativeValue trainer, sized from cudaMemGetInfo.

Restates `value_execution::prepare` (crates/sejong-train/src/value_execution.rs:101-352) and the
allocation accounting it relies on (`allocation` / `workspace_sum`, crates/sejong-train/src/
memory.rs:59-75; `Engine::allocation_bytes`, crates/sejong-gpu/src/lib.rs:234-239: every tensor is a
power-of-two allocation) as exact integer arithmetic, so that for the same available memory the
plan -- batch and activation checkpointing -- is the reference's:

  * fixed bytes: every trained parameter's f32 gradient allocation, two of the largest for
    temporaries, and the compute-precision cast of every body parameter and of the native
    embedding;
  * workspace bytes (workspace_bytes): per activation a forward allocation and an f32 adjoint,
    block by block (9 width-sized, 3 kv-sized, LSE / delta, the FFN or the expert routing and
    expert tensors), retained per layer, or with checkpointing one output per layer plus one
    replayed block; three of the largest f32 activations as reduction scratch; ids and labels;
  * factor bytes (factor_bytes): the parameter VJP's bases, prepared inputs and coefficients;
  * the largest batch (binary search in [1, cap]) whose total fits, retained first, else with
    checkpointing; an error naming required and available bytes when even batch 1 does not fit.

`available` is the device's free memory (`sj_mem_info`, i.e. cudaMemGetInfo), optionally capped
by a memory budget as BatchPolicy.memory_bytes does.  This build's own step keeps every activation
(no recomputation), so `fits_this_build` checks the planned batch against the bytes the B200
trainer itself allocates for it.
"""
import ctypes
from dataclasses import dataclass
from typing import Optional

import numpy as np

from .model import HierarchyConfig, ModelConfig, reference_layout, value_layout

F32, I32 = 4, 4


class CapacityError(RuntimeError):
    """sejong_core::Error::Capacity: an operation needs more device memory than is available."""

    def __init__(self, operation, required, available):
        super().__init__(f"{operation}: {required} bytes required, {available} available")
        self.operation, self.required, self.available = operation, int(required), int(available)


def allocation(elements, dtype_bytes):
    """Engine::allocation_bytes of a tensor: the next power of two of its byte size (at least 1)."""
    b = max(int(elements) * int(dtype_bytes), 1)
    return 1 << (b - 1).bit_length()


def workspace_sum(terms):
    return sum(int(c) * int(s) for c, s in terms)


def floats(elements):
    return allocation(elements, F32)


def pair(elements, forward_bytes):
    """A forward value and its f32 adjoint, each its own allocation."""
    return allocation(elements, forward_bytes) + floats(elements)


class Activations:
    """value_execution.rs:24-100."""

    def __init__(self, precision_bytes):
        self.precision = precision_bytes
        self.retained = 0
        self.replay = 0
        self.largest = 0

    def value(self, elements):
        self.value_as(elements, self.precision)

    def value_as(self, elements, forward_bytes):
        self.retained += pair(elements, forward_bytes)
        self.largest = max(self.largest, floats(elements))

    def stage(self, rows, width, layers, heads, kv_heads, ffn, experts=None, checkpoint=False):
        kv = width // heads * kv_heads
        block = workspace_sum([(9, pair(rows * width, self.precision)), (3, pair(rows * kv, self.precision)),
                               (1, pair(rows * heads, F32))])
        largest = floats(rows * max(width, experts.ffn_width if experts is not None else ffn))
        if experts is not None:
            routes = rows * experts.top_k

            def expert_tensor(columns):  # the per-expert power-of-two bound: 2x the packed bytes
                return 2 * routes * columns * (self.precision + F32)
            block = workspace_sum([(1, block), (1, pair(rows * experts.count, self.precision)),
                                   (1, pair(routes, F32)), (1, allocation(routes, I32)),
                                   (2, allocation(experts.count * routes, I32)), (1, allocation(experts.count, I32)),
                                   (2, expert_tensor(width)), (3, expert_tensor(experts.ffn_width))])
            largest = max(largest, floats(rows * experts.ffn_width))
        else:
            block += 3 * pair(rows * ffn, self.precision)
        if checkpoint:
            self.retained += layers * pair(rows * width, self.precision)
            self.replay = max(self.replay, block)
        else:
            self.retained += layers * block
        self.largest = max(self.largest, largest)


def workspace_bytes(c: ModelConfig, sequence, values, batch, checkpointing, precision_bytes=2,
                    checkpoint_encoder=False, checkpoint_decoder=False):
    """value_execution.rs:101-178."""
    rows = batch * sequence
    a = Activations(precision_bytes)
    a.value(rows * c.width)                                     # native byte embedding
    h: Optional[HierarchyConfig] = c.hierarchy
    if h is not None:
        globals_ = batch * -(-sequence // h.patch_size)
        a.value(rows * h.encoder_width)                         # input projection
        a.stage(rows, h.encoder_width, h.encoder_layers, h.encoder_heads, h.encoder_heads, h.encoder_ffn_width,
                None, checkpointing and checkpoint_encoder)
        a.value(rows * h.encoder_width)                         # encoder norm
        a.value(globals_ * h.encoder_width)                     # patch pool
        a.value(globals_ * c.width)                             # encoder-to-global
        global_rows = globals_
    else:
        global_rows = rows
    a.stage(global_rows, c.width, c.layers, c.heads, c.kv_heads or c.heads, c.ffn_width, c.experts, checkpointing)
    if h is not None:
        a.value(global_rows * c.width)                          # global norm
        a.value(global_rows * h.decoder_width)                  # global-to-decoder
        a.value(h.decoder_width)                                # global BOS projection
        a.value(rows * h.decoder_width)                         # patch broadcast
        a.value(rows * h.decoder_width)                         # encoder-to-decoder
        a.value(rows * h.decoder_width)                         # decoder input add
        a.stage(rows, h.decoder_width, h.decoder_layers, h.decoder_heads, h.decoder_heads, h.decoder_ffn_width,
                None, checkpointing and checkpoint_decoder)
        a.value(rows * h.decoder_width)                         # decoder norm
        a.value(rows * c.width)                                 # output projection
    a.value(rows * c.width)                                     # final norm
    a.value(batch * c.width)                                    # selected request states
    a.value_as(batch * c.width, F32)                            # FP32 selection cast
    a.value_as(batch * values, F32)                             # value projection
    a.value_as(batch * values, F32)                             # bias add
    a.value_as(batch, F32)                                      # cross-entropy losses
    return workspace_sum([(1, a.retained), (1, a.replay), (3, a.largest), (1, allocation(rows, I32)),
                          (2, allocation(batch, I32))])


def factor_bytes(parameters, policy, batch, sequence, c: ModelConfig):
    """value_execution.rs:180-238: parameters = [(name, shape)] of the trained parameters."""
    if policy is None:
        return 0
    from .param_vjp import budget
    groups = {}
    for name, shape in parameters:
        if "." not in name:
            continue
        prefix, suffix = name.rsplit(".", 1)
        if suffix in ("query", "key", "value"):
            groups.setdefault((prefix, False), []).append(shape)
        elif suffix in ("gate", "up"):
            groups.setdefault((prefix, True), []).append(shape)
    h = c.hierarchy
    global_rows = batch * (sequence if h is None else -(-sequence // h.patch_size))
    retained = scratch = 0
    for (prefix, _), members in sorted(groups.items()):
        rows = batch * sequence if prefix.startswith(("encoder.", "decoder.")) else global_rows
        a = members[0][0]
        if rows < a or len(members) <= 1:
            continue
        donor = max(s[1] for s in members)
        rank, blocks, selected = budget(policy, rows, a, donor)
        if selected == blocks:
            continue
        k = selected * policy.block_rows
        retained += (floats(a * rank) + floats((rank + k) * rows) + floats(rows * rank) + allocation(a, I32)
                     + allocation(k, I32) + allocation(rank, I32))
        for s in members:
            retained += floats((rank + k) * s[1])
        scratch = max(scratch, allocation(donor + blocks, I32))
    return retained + scratch


def value_parameters(c: ModelConfig, values):
    """NativeValue::parameters (value.rs:84-106): the body without embedding / output, then the
    native embedding, value head and bias, as (name, shape)."""
    body = [(n, s) for n, s, _ in reference_layout(c) if n not in ("embedding", "output")]
    return body + [(n, s) for n, s, _ in value_layout(c, values)]


def fixed_bytes(c: ModelConfig, values, precision_bytes=2):
    """value_execution.rs:249-277: gradients of the trained parameters (+ 2x the largest) and the
    compute-precision casts of every body parameter and of the native embedding."""
    params = value_parameters(c, values)
    sizes = [floats(int(np.prod(s))) for _, s in params]
    fixed = sum(sizes) + 2 * max(sizes)
    if precision_bytes != F32:
        fixed += sum(allocation(int(np.prod(s)), precision_bytes) for _, s, _ in reference_layout(c))
        fixed += allocation(259 * c.width, precision_bytes)
    return fixed


@dataclass
class Plan:
    batch: int
    checkpointing: bool
    workspace_bytes: int
    fixed_bytes: int
    available: int


def plan(c: ModelConfig, prompts, values, requests, available, memory_bytes=None, max_examples=None,
         activation_checkpointing=None, policy=None, saved=None, precision_bytes=2):
    """value_execution::prepare (value_execution.rs:240-352) for `available` free bytes.

    prompts: the request prompts (their longest + 2 is the sequence); requests: how many requests
    the inventory holds; saved: (batch, checkpointing) of a resumed run.  Raises CapacityError."""
    sequence = max(len(p) for p in prompts) + 2
    fixed = fixed_bytes(c, values, precision_bytes)
    if memory_bytes is not None:
        available = min(fixed + int(memory_bytes), available)
    cap = min(max_examples if max_examples is not None else requests, requests)
    params = value_parameters(c, values)

    def required(batch, checkpoint):
        return (fixed + workspace_bytes(c, sequence, values, batch, checkpoint, precision_bytes)
                + factor_bytes(params, policy, batch, sequence, c))

    if saved is not None:
        batch, checkpoint = saved
        if not 0 < batch <= cap:
            raise ValueError("saved native batch exceeds requested batch limit")
        need = required(batch, checkpoint)
        if need > available:
            raise CapacityError("native resumed batch", need, available)
        return Plan(batch, checkpoint, need - fixed, fixed, available)
    modes = [False, True] if activation_checkpointing is None else [bool(activation_checkpointing)]
    for checkpoint in modes:
        if cap == 0 or required(1, checkpoint) > available:
            continue
        low, high = 1, cap
        while low < high:
            middle = low + -(-(high - low) // 2)
            if required(middle, checkpoint) <= available:
                low = middle
            else:
                high = middle - 1
        need = required(low, checkpoint)
        return Plan(low, checkpoint, need - fixed, fixed, available)
    checkpoint = True if activation_checkpointing is None else bool(activation_checkpointing)
    raise CapacityError("native training workspace", required(1, checkpoint), available)


def available_bytes(device=None):
    """Free device memory from cudaMemGetInfo (sj_mem_info) on the current or given CUDA device."""
    import torch

    from ._lib import call
    if device is not None:
        torch.cuda.set_device(device)
    free, total = ctypes.c_size_t(0), ctypes.c_size_t(0)
    call("sj_mem_info", ctypes.byref(free), ctypes.byref(total))
    return int(free.value)


def fits_this_build(c: ModelConfig, batch, sequence, values, device=None, activation_checkpointing=False):
    """Whether this build's trainer fits `batch` requests of `sequence` bytes in free memory, with every
    activation retained or with the global stage checkpointed: allocates the trainer, reports (fits,
    bytes allocated), frees it."""
    import torch

    from .train import ByteTrainer, TrainConfig
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else device)
    torch.cuda.synchronize(dev)
    before = torch.cuda.memory_allocated(dev)
    try:
        tr = ByteTrainer(c, TrainConfig(sequence=sequence, batch=batch, values=values,
                                        activation_checkpointing=activation_checkpointing), device=dev.index)
    except torch.cuda.OutOfMemoryError:
        return False, None
    used = torch.cuda.memory_allocated(dev) - before
    del tr
    torch.cuda.empty_cache()
    return True, used
