"""CPU oracle for the Sejong byte-Transformer training step.

TEST INFRASTRUCTURE ONLY.  Nothing in the product package (`sejong_b200`) may
import, link or execute anything under `oracle/`.  The only callers are the
tests under `tests/`, `__graft_entry__.smoke()` (as the checker of one small
CUDA invocation) and the `cpu_baseline` / `--impl reference` legs of
`bench.py`.

Contents
--------
rng.py     SplitMix64 `Rng` (crates/sejong-core/src/lib.rs:591-623), vectorised.
corpus.py  Byte corpus and `Corpus::batch` (crates/sejong-train/src/lib.rs:17-109),
           synthetic Zipf(1.1) documents.
ops.py     FP64 restatement of every reference kernel on the path
           (python/sejong_kernels/ops/{kernels,hierarchy,projection}.py).
model.py   Dense / hierarchical byte model (crates/sejong-model/src/architecture.rs),
           AdamW (crates/sejong-train/src/lib.rs:199-238, kernels.py:194-203),
           LR schedule (crates/sejong-core/src/lib.rs:422-433).

Parity pinning: `tests/golden/make_golden.py` runs the reference's own Triton
kernels (python/sejong_kernels/ops/*.py, unmodified) in Triton's CPU
interpreter on small seeded inputs and stores their outputs as fixtures;
`tests/test_oracle_pins.py` checks every function in `ops.py` against them.
"""
