"""Byte corpus and batch sampling restated from crates/sejong-train/src/lib.rs:17-109.

Layout (lib.rs:24-58): documents are joined as EOS + bytes for each document,
with one final EOS; `tokens` counts all of them.  `token(i)` (lib.rs:59-71)
returns EOS at a document start and at the very end, else the byte.
`batch` (lib.rs:72-88) draws `start = rng.index(tokens - sequence)` per row and
takes inputs token(start+i) and targets token(start+i+1).

Synthetic documents: bytes i.i.d. Zipf(s) on 0..255 with p_k proportional to
(k+1)^-s, drawn by inverse CDF from `Rng.uniform` (one draw per byte); byte =
the smallest k with cdf[k] >= u (cdf accumulated in float64, u is the f32 draw
widened to float64).
"""
import numpy as np

from .rng import Rng

EOS = 256
VOCAB = 257


def zipf_cdf(s=1.1):
    p = (np.arange(256, dtype=np.float64) + 1.0) ** (-float(s))
    return np.cumsum(p / p.sum())


def zipf_bytes(seed, count, s=1.1):
    u = Rng(seed).bulk_uniform(count).astype(np.float64)
    k = np.searchsorted(zipf_cdf(s), u, side="left")
    return np.minimum(k, 255).astype(np.uint8)


class Corpus:
    def __init__(self, documents):
        self.documents = [np.asarray(d, dtype=np.uint8) for d in documents if len(d) > 0]
        self.ends = []
        tokens = 0
        for d in self.documents:
            tokens += len(d) + 1
            self.ends.append(tokens)
        assert tokens > 1, "corpus contains no text"
        self.tokens = tokens + 1
        self.ends = np.asarray(self.ends, dtype=np.int64)

    def token_array(self):
        """All tokens in order (EOS, doc0 bytes, EOS, doc1 bytes, ..., EOS)."""
        out = np.empty(self.tokens, dtype=np.int32)
        pos = 0
        for d in self.documents:
            out[pos] = EOS
            out[pos + 1: pos + 1 + len(d)] = d
            pos += len(d) + 1
        out[pos] = EOS
        return out

    def token(self, index):
        if index == self.tokens - 1:
            return EOS
        doc = int(np.searchsorted(self.ends, index, side="right"))
        start = 0 if doc == 0 else int(self.ends[doc - 1])
        local = index - start
        return EOS if local == 0 else int(self.documents[doc][local - 1])

    def batch(self, rng, batch, sequence):
        toks = self.token_array()
        inputs = np.empty(batch * sequence, dtype=np.int32)
        targets = np.empty(batch * sequence, dtype=np.int32)
        for b in range(batch):
            start = rng.index(self.tokens - sequence)
            inputs[b * sequence:(b + 1) * sequence] = toks[start:start + sequence]
            targets[b * sequence:(b + 1) * sequence] = toks[start + 1:start + sequence + 1]
        return inputs, targets


def synthetic_corpus(seed, length, s=1.1):
    """One synthetic document of `length` Zipf bytes."""
    return Corpus([zipf_bytes(seed, length, s)])
