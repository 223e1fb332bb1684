"""Pure-Python restatement of the reference's token-shard DataLoader
(TEST INFRASTRUCTURE ONLY: tests use it to check libllmk's loader).

Follows utils/dataloader.cpp and utils/rand.h of the reference:

- shard format (dataloader.cpp:84-115): 256 int32 header words, [0] = 20240520,
  [1] = 1, [2] = token count n, then n uint16 tokens; file size must be
  1024 + 2n; samples per shard = (2n - 2) // (world*B*T*2);
- shard list (dataloader.cpp:26-40): the path itself if it is a file, else the
  directory's regular files in directory-iteration order (os.scandir gives the
  same order as std::filesystem::directory_iterator: both walk readdir);
- shuffling (dataloader.cpp:42-48, 176-216; rand.h:11-19): std::mt19937
  seeded 42 + world; Reset permutes the shard order, every opened shard
  (Reset, Advance) draws a fresh sample order; a permutation is Fisher-Yates
  from the back, j = uniform_int_distribution<int>{0, i}(rng);
- sample i of rank r is B*T+1 tokens from byte 1024 + i*world*B*T*2 + r*B*T*2
  (dataloader.cpp:147-156); inputs = tokens[:-1], targets = tokens[1:];
- NextBatch (dataloader.h:80-87) advances to the next shard when the open one
  is exhausted, and resets after the last shard (dataloader.cpp:160-172).

The engine is MT19937 as published by Matsumoto and Nishimura (1998) with its
init_genrand seeding, which is what std::mt19937(seed) specifies. The bounded
draw is the one GCC's libstdc++ uses for a 32-bit engine: Lemire's multiply
and reject method ("Fast Random Integer Generation in an Interval", 2019).
The test suite pins this restatement against the reference's own loader
compiled from its sources.
"""
from __future__ import annotations

import os

import numpy as np

MAGIC, VERSION, HEADER_INTS = 20240520, 1, 256


class MT19937:
    N, M = 624, 397

    def __init__(self, seed: int):
        mt = [0] * self.N
        mt[0] = seed & 0xFFFFFFFF
        for i in range(1, self.N):
            mt[i] = (1812433253 * (mt[i - 1] ^ (mt[i - 1] >> 30)) + i) & 0xFFFFFFFF
        self.mt, self.idx = mt, self.N

    def _twist(self):
        mt = self.mt
        for i in range(self.N):
            y = (mt[i] & 0x80000000) | (mt[(i + 1) % self.N] & 0x7FFFFFFF)
            mt[i] = mt[(i + self.M) % self.N] ^ (y >> 1) ^ (0x9908B0DF if y & 1 else 0)
        self.idx = 0

    def __call__(self) -> int:
        if self.idx >= self.N:
            self._twist()
        y = self.mt[self.idx]
        self.idx += 1
        y ^= y >> 11
        y ^= (y << 7) & 0x9D2C5680
        y ^= (y << 15) & 0xEFC60000
        y ^= y >> 18
        return y & 0xFFFFFFFF


def uniform_int(rng: MT19937, lo: int, hi: int) -> int:
    """Uniform integer in [lo, hi] from 32-bit draws (Lemire's method)."""
    rng_range = hi - lo + 1
    product = rng() * rng_range
    low = product & 0xFFFFFFFF
    if low < rng_range:
        threshold = (-rng_range & 0xFFFFFFFF) % rng_range
        while low < threshold:
            product = rng() * rng_range
            low = product & 0xFFFFFFFF
    return lo + (product >> 32)


def permute(v: list, rng: MT19937) -> None:
    for i in range(len(v) - 1, 0, -1):
        j = uniform_int(rng, 0, i)
        v[i], v[j] = v[j], v[i]


def write_shard(path: str, tokens) -> None:
    """A shard file in the format the loader reads (the reference's data
    preprocessing writes the same layout)."""
    t = np.ascontiguousarray(tokens, dtype=np.uint16)
    header = np.zeros(HEADER_INTS, dtype=np.int32)
    header[:3] = [MAGIC, VERSION, t.size]
    with open(path, "wb") as f:
        f.write(header.tobytes())
        f.write(t.tobytes())


class DataLoader:
    def __init__(self, path: str, B: int, T: int, rank: int, world: int, shuffle: bool):
        self.B, self.T, self.rank, self.world, self.shuffle = B, T, rank, world, shuffle
        if os.path.isfile(path):
            self.shards = [path]
        else:
            self.shards = [e.path for e in os.scandir(path) if e.is_file()]
        if not self.shards:
            raise ValueError("no shards")
        self.rng = MT19937(42 + world) if shuffle else None
        self.shard_order = list(range(len(self.shards)))
        self.sample_order: list[int] = []
        self.num_tokens = 0
        for i in range(len(self.shards)):
            n = self._open(i)
            if n < world * B * T + 1:
                raise ValueError("shard too small")
            self.num_tokens += n
        self.reset()

    def _open(self, i: int) -> int:
        k = self.shard_order[i] if self.shuffle else i
        raw = open(self.shards[k], "rb").read()
        header = np.frombuffer(raw[:HEADER_INTS * 4], dtype=np.int32)
        if header[0] != MAGIC or header[1] != VERSION:
            raise ValueError("bad header")
        n = int(header[2])
        if n <= 0 or len(raw) != HEADER_INTS * 4 + 2 * n:
            raise ValueError("bad size")
        self.tokens = np.frombuffer(raw[HEADER_INTS * 4:], dtype=np.uint16)
        self.shard_samples = (2 * n - 2) // (self.world * self.B * self.T * 2)
        return n

    def _order_samples(self):
        self.sample_order = list(range(self.shard_samples))
        permute(self.sample_order, self.rng)

    def reset(self):
        self.shard_idx, self.sample_idx = 0, 0
        if self.shuffle:
            permute(self.shard_order, self.rng)
        self._open(0)
        if self.shuffle:
            self._order_samples()

    def _advance(self):
        if self.shard_idx == len(self.shards) - 1:
            self.reset()
            return
        self.shard_idx += 1
        self.sample_idx = 0
        self._open(self.shard_idx)
        if self.shuffle:
            self._order_samples()

    def resume(self, shard_idx: int, sample_idx: int):
        self.shard_idx, self.sample_idx = shard_idx, sample_idx
        self._open(shard_idx)

    def next_batch(self):
        if self.sample_idx >= self.shard_samples:
            self._advance()
        idx = self.sample_order[self.sample_idx] if self.shuffle else self.sample_idx
        bt = self.B * self.T
        start = idx * self.world * bt + self.rank * bt
        buf = self.tokens[start:start + bt + 1].astype(np.int32)
        self.sample_idx += 1
        return buf[:-1].reshape(self.B, self.T), buf[1:].reshape(self.B, self.T)
