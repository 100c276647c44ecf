"""Restatement of the runtime's sampling rule (crates/sejong-runtime/src/lib.rs:44-78) on the
test-side Rng (oracle/rng.py): test infrastructure, the checker of sejong_b200.generate.sample.

Rank the logits in descending order (a stable sort: equal logits keep their index order); at
temperature 0 return the first; else keep the top_k first (if top_k > 0), weight each by
exp((v - max) / T) in f32, keep the shortest prefix whose cumulative share reaches top_p, and
return the first index whose running weight reaches uniform() * total."""
import numpy as np


def sample(logits, temperature, top_k, top_p, rng):
    x = np.asarray(logits, dtype=np.float32)
    ranked = sorted(range(len(x)), key=lambda i: -float(x[i]))  # Python's sort is stable
    if temperature == 0:
        return ranked[0]
    if top_k > 0:
        ranked = ranked[:min(top_k, len(ranked))]
    m = x[ranked[0]]
    vals = [np.float32(np.exp(np.float32((x[i] - m) / np.float32(temperature)))) for i in ranked]
    total = np.float32(0)
    for v in vals:
        total = np.float32(total + v)
    cum = np.float32(0)
    keep = len(vals)
    for i, v in enumerate(vals):
        cum = np.float32(cum + v / total)
        if cum >= np.float32(top_p):
            keep = i + 1
            break
    ranked, vals = ranked[:keep], vals[:keep]
    total = np.float32(0)
    for v in vals:
        total = np.float32(total + v)
    threshold = np.float32(np.float32(rng.uniform()) * total)
    acc = np.float32(0)
    for i, v in zip(ranked, vals):
        acc = np.float32(acc + v)
        if acc >= threshold:
            return i
    return ranked[-1]
