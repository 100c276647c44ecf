"""Corpus::open (crates/sejong-train/src/lib.rs:17-109) and its BLAKE3 fingerprint.

`sj_blake3` (the library's streaming BLAKE3) is checked against the published digests of the empty
string and "abc" and against an independent restatement here that builds the hash tree recursively
(the left subtree holds the largest power-of-two number of chunks below the total), for lengths
around every block, chunk and tree boundary and for input split into uneven parts.
"""
import ctypes

import numpy as np
import pytest

from sejong_b200 import corpus as sc
from sejong_b200.model import EOS

IV = [0x6A09E667, 0xBB67AE85, 0x3C6EF372, 0xA54FF53A, 0x510E527F, 0x9B05688C, 0x1F83D9AB, 0x5BE0CD19]
PERM = [2, 6, 3, 10, 7, 0, 4, 13, 1, 11, 12, 5, 9, 14, 15, 8]
M32 = 0xFFFFFFFF


def _g(s, a, b, c, d, x, y):
    s[a] = (s[a] + s[b] + x) & M32
    s[d] = ((s[d] ^ s[a]) >> 16 | (s[d] ^ s[a]) << 16) & M32
    s[c] = (s[c] + s[d]) & M32
    s[b] = ((s[b] ^ s[c]) >> 12 | (s[b] ^ s[c]) << 20) & M32
    s[a] = (s[a] + s[b] + y) & M32
    s[d] = ((s[d] ^ s[a]) >> 8 | (s[d] ^ s[a]) << 24) & M32
    s[c] = (s[c] + s[d]) & M32
    s[b] = ((s[b] ^ s[c]) >> 7 | (s[b] ^ s[c]) << 25) & M32


def _compress(cv, block, counter, blen, flags):
    m = [int.from_bytes(block[4 * i:4 * i + 4], "little") for i in range(16)]
    s = list(cv) + IV[:4] + [counter & M32, counter >> 32, blen, flags]
    for r in range(7):
        for i, (a, b, c, d) in enumerate(((0, 4, 8, 12), (1, 5, 9, 13), (2, 6, 10, 14), (3, 7, 11, 15),
                                          (0, 5, 10, 15), (1, 6, 11, 12), (2, 7, 8, 13), (3, 4, 9, 14))):
            _g(s, a, b, c, d, m[2 * i], m[2 * i + 1])
        m = [m[p] for p in PERM]
    return [s[i] ^ s[i + 8] for i in range(8)] + [s[i + 8] ^ cv[i] for i in range(8)]


def _chunk_node(data, index):
    """(cv, block, counter, block_len, flags) of the final compression of one chunk."""
    blocks = [data[i:i + 64] for i in range(0, len(data), 64)] or [b""]
    cv = IV
    for j, blk in enumerate(blocks[:-1]):
        cv = _compress(cv, blk, index, 64, 1 if j == 0 else 0)[:8]
    last = blocks[-1]
    return cv, last.ljust(64, b"\0"), index, len(last), (1 if len(blocks) == 1 else 0) | 2


def _words(w):
    return b"".join(x.to_bytes(4, "little") for x in w)


def _node(data, first_chunk):
    chunks = max(1, (len(data) + 1023) // 1024)
    if chunks == 1:
        return _chunk_node(data, first_chunk)
    left_chunks = 1 << ((chunks - 1).bit_length() - 1)
    left, right = data[:left_chunks * 1024], data[left_chunks * 1024:]
    lcv = _compress(*_node(left, first_chunk))[:8]
    rcv = _compress(*_node(right, first_chunk + left_chunks))[:8]
    return IV, _words(lcv) + _words(rcv), 0, 64, 4


def blake3_restated(data):
    cv, block, _, blen, flags = _node(data, 0)
    return _words(_compress(cv, block, 0, blen, flags | 8)[:8]).hex()


def test_published_digests():
    assert sc.blake3_hex([b""]) == "af1349b9f5f9a1a6a0404dea36dcc9499bcb25c9adc112b7cc9a93cae41f3262"
    assert sc.blake3_hex([]) == "af1349b9f5f9a1a6a0404dea36dcc9499bcb25c9adc112b7cc9a93cae41f3262"
    assert sc.blake3_hex([b"abc"]) == "6437b3ac38465133ffb63b75273a8db548c558465d79db03fd359c6cd5bd9d85"
    assert blake3_restated(b"") == "af1349b9f5f9a1a6a0404dea36dcc9499bcb25c9adc112b7cc9a93cae41f3262"
    assert blake3_restated(b"abc") == "6437b3ac38465133ffb63b75273a8db548c558465d79db03fd359c6cd5bd9d85"


@pytest.mark.parametrize("n", [1, 63, 64, 65, 1023, 1024, 1025, 2048, 2049, 3072, 3073, 4096, 5121, 8193])
def test_library_matches_restatement(n):
    data = bytes((i * 7 + 3) % 251 for i in range(n))
    assert sc.blake3_hex([data]) == blake3_restated(data)
    cuts = sorted({0, n // 3, n // 3 + 1, (2 * n) // 3, n})
    parts = [data[a:b] for a, b in zip(cuts, cuts[1:])]
    assert sc.blake3_hex(parts) == blake3_restated(data)


def test_corpus_layout_and_fingerprint(tmp_path):
    (tmp_path / "b").mkdir()
    (tmp_path / "b" / "two.txt").write_bytes(b"xyz")
    (tmp_path / "a.txt").write_bytes(b"hello")
    (tmp_path / "empty.txt").write_bytes(b"")
    (tmp_path / "skip.md").write_bytes(b"not text")
    c = sc.Corpus.open(tmp_path)
    # component order: "a.txt" < "b" < "empty.txt"; the empty file and the .md file are skipped
    want = [EOS, *b"hello", EOS, *b"xyz", EOS]
    assert c.tokens.tolist() == want and c.count == len(want)
    raw = sc.DOMAIN + (5).to_bytes(8, "little") + b"hello" + (3).to_bytes(8, "little") + b"xyz"
    assert c.fingerprint == blake3_restated(raw)
    st = ctypes.c_uint64(7)
    ids, tg = c.batch(st, 2, 4)
    assert ids.shape == (8,) and np.array_equal(ids.reshape(2, 4)[:, 1:], tg.reshape(2, 4)[:, :-1])


def test_corpus_errors(tmp_path):
    with pytest.raises(sc.CorpusError):
        sc.Corpus.open(tmp_path / "missing")
    (tmp_path / "e.txt").write_bytes(b"")
    with pytest.raises(sc.CorpusError):
        sc.Corpus.open(tmp_path)
