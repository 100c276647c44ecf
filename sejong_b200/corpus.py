"""Byte corpora from UTF-8 text files: `Corpus::open` / `token` / `batch`
(crates/sejong-train/src/lib.rs:17-109).

A corpus is a file, or a directory searched recursively for `*.txt` files, sorted by path component
as the reference sorts `PathBuf`s.  Empty files are skipped.  The token stream is EOS + bytes of each
document in turn, and one final EOS (lib.rs:59-71); it is held as int32 so that `sj_corpus_batch`
draws batches from it with the reference `Rng`.  The fingerprint is BLAKE3 over the domain string
and, per document, its length (u64 little endian) and bytes (lib.rs:34-48), computed by the
library's `sj_blake3`; checkpoints carry it and a resume checks it.
"""
import ctypes
import os
from pathlib import Path

import numpy as np

from ._lib import call
from .model import EOS

DOMAIN = b"Sejong byte corpus v1: EOS + document bytes + EOS"


class CorpusError(ValueError):
    """A corpus the reference would refuse (missing path, no text)."""


def blake3_hex(parts):
    """BLAKE3 (32 bytes, hex) of the concatenation of `parts` (bytes-like objects)."""
    bufs = [np.frombuffer(p, dtype=np.uint8) if len(p) else np.zeros(1, np.uint8) for p in parts]
    ptrs = (ctypes.c_void_p * max(1, len(parts)))(*[b.ctypes.data for b in bufs])
    lens = (ctypes.c_uint64 * max(1, len(parts)))(*[len(p) for p in parts])
    out = (ctypes.c_uint8 * 32)()
    call("sj_blake3", ctypes.cast(ptrs, ctypes.c_void_p), ctypes.cast(lens, ctypes.c_void_p), len(parts),
         ctypes.cast(out, ctypes.c_void_p))
    return bytes(out).hex()


def collect_text(path):
    """collect_text (lib.rs:89-109): the file itself, or every *.txt below a directory."""
    p = Path(path)
    if p.is_file():
        return [p]
    if p.is_dir():
        out = []
        for root, dirs, files in os.walk(p):
            for f in files:
                if f.endswith(".txt"):
                    out.append(Path(root) / f)
        return out
    raise CorpusError(f"corpus path does not exist: {p}")


class Corpus:
    """A byte corpus: `tokens` (int32 stream), `count` (= the reference's `tokens` field) and
    `fingerprint`."""

    def __init__(self, documents):
        docs = [bytes(d) for d in documents if len(d)]
        if not docs:
            raise CorpusError("corpus contains no text")
        parts = [DOMAIN]
        for d in docs:
            parts.append(len(d).to_bytes(8, "little"))
            parts.append(d)
        self.fingerprint = blake3_hex(parts)
        total = sum(len(d) + 1 for d in docs) + 1
        toks = np.empty(total, dtype=np.int32)
        at = 0
        for d in docs:
            toks[at] = EOS
            toks[at + 1:at + 1 + len(d)] = np.frombuffer(d, dtype=np.uint8)
            at += len(d) + 1
        toks[at] = EOS
        self.tokens = toks
        self.count = total

    @classmethod
    def open(cls, path):
        files = sorted(collect_text(path), key=lambda f: f.parts)
        if not files:
            raise CorpusError("corpus requires at least one text file")
        return cls([f.read_bytes() for f in files])

    def batch(self, rng_state, batch, sequence):
        """Corpus::batch (lib.rs:72-88): `rng_state` is a ctypes.c_uint64 holding the Rng state."""
        if self.count <= sequence:
            raise CorpusError("corpus is shorter than the training sequence")
        inputs = np.empty(batch * sequence, dtype=np.int32)
        targets = np.empty(batch * sequence, dtype=np.int32)
        call("sj_corpus_batch", self.tokens.ctypes.data, self.tokens.size, ctypes.byref(rng_state), batch, sequence,
             inputs.ctypes.data, targets.ctypes.data)
        return inputs, targets
