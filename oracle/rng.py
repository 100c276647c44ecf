"""SplitMix64 generator restated from crates/sejong-core/src/lib.rs:591-623.

`Rng.next_u64` follows lib.rs:599-605, `uniform` lib.rs:606-608, `index`
lib.rs:609-618 (Lemire-free rejection with threshold = (-n) mod n), `normal`
lib.rs:619-621 (Box-Muller on two consecutive uniforms, f32 arithmetic).

Because SplitMix64's state advances by a constant, the i-th output depends only
on seed + (i+1)*GAMMA, so bulk draws are vectorised with numpy uint64
arithmetic (wrapping multiply) and stay bit-identical to the sequential form.
"""
import numpy as np

GAMMA = np.uint64(0x9E3779B97F4A7C15)
M1 = np.uint64(0xBF58476D1CE4E5B9)
M2 = np.uint64(0x94D049BB133111EB)
MASK64 = (1 << 64) - 1


def _mix(z):
    z = np.asarray(z, dtype=np.uint64)
    with np.errstate(over="ignore"):
        z = (z ^ (z >> np.uint64(30))) * M1
        z = (z ^ (z >> np.uint64(27))) * M2
    return z ^ (z >> np.uint64(31))


class Rng:
    """Sequential SplitMix64 with the reference's derived draws."""

    def __init__(self, seed):
        self.state = int(seed) & MASK64

    def clone(self):
        r = Rng(0)
        r.state = self.state
        return r

    def next_u64(self):
        self.state = (self.state + int(GAMMA)) & MASK64
        z = self.state
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & MASK64
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & MASK64
        return z ^ (z >> 31)

    def bulk_u64(self, count):
        """The next `count` outputs of next_u64, vectorised."""
        steps = np.arange(1, count + 1, dtype=np.uint64)
        with np.errstate(over="ignore"):
            states = np.uint64(self.state) + steps * GAMMA
        self.state = (self.state + count * int(GAMMA)) & MASK64
        return _mix(states)

    def uniform(self):
        return np.float32(((self.next_u64() >> 40) + 0.5) / 16777216.0)

    def bulk_uniform(self, count):
        x = self.bulk_u64(count)
        return (((x >> np.uint64(40)).astype(np.float64) + 0.5) / 16777216.0).astype(np.float32)

    def index(self, size):
        n = int(size)
        threshold = ((-n) & MASK64) % n
        while True:
            x = self.next_u64()
            if x >= threshold:
                return x % n

    def normal(self):
        a = self.uniform()
        b = self.uniform()
        return _box_muller(np.array([a]), np.array([b]))[0]

    def bulk_normal(self, count):
        u = self.bulk_uniform(2 * count).reshape(count, 2)
        return _box_muller(u[:, 0], u[:, 1])


def _box_muller(a, b):
    a = np.asarray(a, dtype=np.float32)
    b = np.asarray(b, dtype=np.float32)
    tau = np.float32(2.0 * np.pi)
    return (np.sqrt(np.float32(-2.0) * np.log(a)) * np.cos(tau * b)).astype(np.float32)
