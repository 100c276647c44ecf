"""Parameter VJP planning: which weight gradients are compressed and when the index draws happen.

Host-side restatement of crates/sejong-gpu/src/parameter_vjp.rs (the integer tile-cost model,
lines 9-13 and 85-130) and of the tape's group decision (crates/sejong-gpu/src/graph.rs:915-1005):

* Matmul nodes that share one input X with rows >= features form a group.  The donor is the
  member with the widest output; on ties the LAST such member (Rust `max_by_key`).
* Members are pruned by `selects_compression(n, a, b, donor, uses)` with the current member count
  until the set is stable; a group with at least one member left is prepared once per backward
  pass, when its first member is visited in reverse creation order.
* The basis is shared per (rows, rank) and the feature selection per width (graph.rs:974-990); a
  preparation that needs either draws one `rng.next_u64()` (parameter_vjp.rs:190).

Everything here depends on shapes only, so the plan is fixed for a model and batch shape and the
step's device work (sejong_b200/train.py) is a static schedule that never reads back to the host.
"""
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import numpy as np

from .model import HEAD_DIM, global_stage, local_stage

BM, BN, BK = 16, 32, 32
F32_EPS = 2.0 ** -23


@dataclass
class VjpConfig:
    """sejong_core::ParameterVjpConfig (crates/sejong-core/src/lib.rs:444-466)."""
    rank: int = 16
    residual_fraction: float = 0.25
    block_rows: int = 32
    seed: int = 7


def _ceil_div(a, b):
    return -(-a // b)


def _next_pow2(n):
    return 1 if n <= 1 else 1 << (n - 1).bit_length()


def issued_gemm(m, n, k):
    """FLOPs the reference's tiled GEMM issues for an m x n x k product (padded to its tiles)."""
    return 2 * (_ceil_div(m, BM) * BM) * (_ceil_div(n, BN) * BN) * (_ceil_div(k, BK) * BK)


def budget(cfg, n, a, donor):
    """(rank, feature blocks, selected blocks) of a preparation (parameter_vjp.rs:85-96)."""
    rank = min(cfg.rank, n, a, donor)
    blocks = _ceil_div(a, cfg.block_rows)
    selected = max(min(int(np.ceil(blocks * cfg.residual_fraction)), blocks), 1)
    return rank, blocks, selected


def selects_compression(cfg, n, a, b, donor, uses):
    """The cost comparison of parameter_vjp.rs:97-130: compressed work (shared QR and preparation
    amortised over `uses` members, plus each member's coefficient and factor GEMMs) against the
    dense X^T dY GEMMs."""
    if n < a or uses <= 1:
        return False
    rank, blocks, selected = budget(cfg, n, a, donor)
    if selected == blocks:
        return False
    k = selected * cfg.block_rows
    padded = _ceil_div(n, BM) * BM
    last = max(rank - 1, 0)
    full, tail = last // BN, last % BN
    tiles = BN * full * (full + 1) // 2 + tail * (full + 1)
    streaming = 2 * (4 * padded * BN + padded) * tiles + 5 * padded * rank
    resident = 8 * _next_pow2(n) * _next_pow2(rank) * rank + 5 * _next_pow2(n) * rank
    shared = max(streaming, resident) + issued_gemm(a, rank, n) + issued_gemm(k, n, rank)
    own = issued_gemm(rank + k, b, n) + issued_gemm(a, b, rank)
    return own * uses + shared < issued_gemm(a, b, n) * uses


def group_active(cfg, n, width, member_widths, donor_width):
    """Indices of the members that stay compressed (graph.rs:944-965)."""
    active = set(range(len(member_widths)))
    while active:
        count = len(active)
        active = {i for i in active if selects_compression(cfg, n, width, member_widths[i], donor_width, count)}
        if len(active) == count:
            break
    return active


def donor_index(member_widths):
    """Rust Iterator::max_by_key: the last member of maximal output width."""
    best = 0
    for i, w in enumerate(member_widths):
        if w >= member_widths[best]:
            best = i
    return best


def basis_eps(rows, rank):
    """Small-norm cutoff gamma(rows (4 rank + 1)) of parameter_vjp.rs:226-235, as an f32."""
    operations = rows * (4.0 * rank + 1.0)
    roundoff = operations * (F32_EPS / 2.0)
    tol = roundoff / (1.0 - roundoff) if roundoff < 1.0 else np.inf
    return float(np.float32(min(tol, np.finfo(np.float32).max)))


@dataclass
class Node:
    """One Matmul node of the model's forward, in creation order."""
    name: str        # reference parameter name
    input: str       # key of the input tensor (nodes with the same key share X)
    rows: int
    features: int
    width: int


def matmul_nodes(c, batch, seq):
    """The Matmul nodes of one forward in creation order (crates/sejong-model/src/architecture.rs:
    201-393; the order the tape records them)."""
    nodes = []

    def stage(s, rows):
        for i in range(s.layers):
            p = f"{s.prefix}.{i}"
            d = s.width
            nodes.extend([Node(f"{p}.query", f"{p}.z1", rows, d, s.heads * HEAD_DIM),
                          Node(f"{p}.key", f"{p}.z1", rows, d, s.kv_heads * HEAD_DIM),
                          Node(f"{p}.value", f"{p}.z1", rows, d, s.kv_heads * HEAD_DIM),
                          Node(f"{p}.attention_output", f"{p}.o", rows, s.heads * HEAD_DIM, d),
                          Node(f"{p}.gate", f"{p}.z2", rows, d, s.ffn),
                          Node(f"{p}.up", f"{p}.z2", rows, d, s.ffn),
                          Node(f"{p}.down", f"{p}.h", rows, s.ffn, d)])

    n = batch * seq
    h = c.hierarchy
    if h is None:
        stage(global_stage(c), n)
        top = c.width
    else:
        patches = -(-seq // h.patch_size)
        np_ = batch * patches
        stage(local_stage(c, True), n)
        nodes.append(Node("encoder_to_global", "pooled", np_, h.encoder_width, c.width))
        stage(global_stage(c), np_)
        nodes.append(Node("global_to_decoder", "zG", np_, c.width, h.decoder_width))
        nodes.append(Node("global_to_decoder", "global_bos", 1, c.width, h.decoder_width))
        nodes.append(Node("encoder_to_decoder", "zE", n, h.encoder_width, h.decoder_width))
        stage(local_stage(c, False), n)
        nodes.append(Node("output_projection", "zD", n, h.decoder_width, c.width))
        top = c.width
    nodes.append(Node("output", "hf", n, top, 257))
    return nodes


@dataclass
class GroupPlan:
    """One compressed group and what its preparation does."""
    input: str
    rows: int
    features: int
    members: List[Node]
    donor: int                       # index into members
    active: List[int]                # indices of compressed members
    rank: int
    blocks: int
    selected: int
    block_rows: int
    draw: bool = False               # one next_u64 of the device Rng
    new_basis: bool = False          # computes the basis shared by every group with these rows
    new_selection: bool = False      # draws the rows shared by every group of this width
    order: int = 0                   # preparation order within the backward pass

    @property
    def k(self):
        """Selected feature rows (selected blocks x block_rows, padded rows included)."""
        return self.selected * self.block_rows

    @property
    def basis_key(self) -> Tuple[int, int]:
        return (self.rows, self.rank)

    @property
    def inverse(self):
        """NB / S in f32 (the INVERSE argument, parameter_vjp.rs:282)."""
        return float(np.float32(self.blocks) / np.float32(self.selected))


@dataclass
class VjpPlan:
    cfg: VjpConfig
    groups: Dict[str, GroupPlan] = field(default_factory=dict)   # by input key, active groups only
    prepare_order: List[str] = field(default_factory=list)
    compressed: List[str] = field(default_factory=list)           # reference names, visit order

    @property
    def draws(self):
        return sum(1 for k in self.prepare_order if self.groups[k].draw)


def plan(c, batch, seq, cfg=None):
    """The group decisions and preparation schedule of one backward pass."""
    cfg = cfg or VjpConfig()
    nodes = matmul_nodes(c, batch, seq)
    members: Dict[str, List[int]] = {}
    for idx, node in enumerate(nodes):
        if node.rows >= node.features:
            members.setdefault(node.input, []).append(idx)
    out = VjpPlan(cfg)
    visited = set()
    bases, selections = set(), set()
    active_nodes = set()
    for idx in reversed(range(len(nodes))):
        node = nodes[idx]
        key = node.input
        if key in members and key not in visited:
            visited.add(key)
            mem = [nodes[i] for i in members[key]]
            widths = [m.width for m in mem]
            donor = donor_index(widths)
            active = group_active(cfg, node.rows, node.features, widths, widths[donor])
            if active:
                rank, blocks, selected = budget(cfg, node.rows, node.features, widths[donor])
                g = GroupPlan(key, node.rows, node.features, mem, donor, sorted(active), rank, blocks, selected,
                              cfg.block_rows)
                g.new_basis = g.basis_key not in bases
                g.new_selection = node.features not in selections
                g.draw = g.new_basis or g.new_selection
                bases.add(g.basis_key)
                selections.add(node.features)
                g.order = len(out.prepare_order)
                out.groups[key] = g
                out.prepare_order.append(key)
                active_nodes.update(members[key][i] for i in active)
        if idx in active_nodes:
            out.compressed.append(node.name)
    return out
