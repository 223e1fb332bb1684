"""Token-shard loader (include/llmk_data.h) against the restatement in
oracle/dataloader.py, which is itself pinned to the reference's DataLoader
compiled from utils/dataloader.cpp (oracle/_ref/libref.so).

Covers what the reference's loader does with its inputs: rank striding of the
samples, the shard size checks, shard advance and reset after the last shard,
the mt19937 shuffles of shard and sample order (seeded 42 + world), and
Resume. All on CPU: the loader is host code."""
import os

import numpy as np
import pytest

import oracle as O
from oracle import dataloader as D


def make_shards(d, sizes, seed=0, vocab=50257):
    rng = np.random.default_rng(seed)
    os.makedirs(d, exist_ok=True)
    for i, n in enumerate(sizes):
        D.write_shard(os.path.join(d, f"shard_{i:02d}.bin"), rng.integers(0, vocab, n))
    return d


CASES = [
    # (shard sizes, B, T, world, shuffle)
    ([4097], 2, 64, 1, False),
    ([4097], 2, 64, 1, True),
    ([3001, 5000, 2600], 2, 32, 2, False),
    ([3001, 5000, 2600, 7777, 4100], 1, 48, 3, True),
    ([2049, 2049], 4, 16, 4, True),
    ([1025], 1, 1024, 1, False),  # exactly one sample per shard
]


def _sequence(make, n):
    ld = make()
    return [tuple(a.copy() for a in ld.next_batch()) for _ in range(n)]


class RefLoader:
    def __init__(self, path, B, T, rank, world, shuffle):
        self.B, self.T = B, T
        self.h = O.ref().ref_loader_create(path.encode(), B, T, rank, world, int(shuffle))
        self.num_tokens = O.ref().ref_loader_num_tokens(self.h)

    def next_batch(self):
        a = np.empty((self.B, self.T), np.int32)
        b = np.empty((self.B, self.T), np.int32)
        O.ref().ref_loader_next(self.h, a.reshape(-1), b.reshape(-1))
        return a, b

    def resume(self, shard, sample):
        O.ref().ref_loader_resume(self.h, shard, sample)

    def __del__(self):
        if getattr(self, "h", None):
            O.ref().ref_loader_destroy(self.h)


def test_mt19937_known_answer():
    # std::mt19937 default seed 5489: the 10000th output is 4123659995 (C++ standard, [rand.predef])
    g = D.MT19937(5489)
    for _ in range(9999):
        g()
    assert g() == 4123659995


@pytest.mark.skipif(not O.ref_available(), reason="reference library not built")
@pytest.mark.parametrize("case", range(len(CASES)))
def test_oracle_matches_reference_loader(tmp_path, case):
    sizes, B, T, world, shuffle = CASES[case]
    d = make_shards(str(tmp_path / "s"), sizes, seed=case)
    for rank in range(world):
        nsteps = 3 * sum(((2 * n - 2) // (world * B * T * 2)) for n in sizes) + 2
        ref = _sequence(lambda: RefLoader(d, B, T, rank, world, shuffle), nsteps)
        orc = _sequence(lambda: D.DataLoader(d, B, T, rank, world, shuffle), nsteps)
        for (ri, rt), (oi, ot) in zip(ref, orc):
            assert np.array_equal(ri, oi) and np.array_equal(rt, ot)


@pytest.mark.parametrize("case", range(len(CASES)))
def test_loader_matches_oracle(tmp_path, llmk_lib, case):
    import llmk
    sizes, B, T, world, shuffle = CASES[case]
    d = make_shards(str(tmp_path / "s"), sizes, seed=100 + case)
    for rank in range(world):
        # three passes over every shard: covers advance and the reset (re-shuffle) after the last shard
        nsteps = 3 * sum(((2 * n - 2) // (world * B * T * 2)) for n in sizes) + 2
        ours = llmk.DataLoader(d, B, T, rank, world, shuffle)
        assert ours.num_tokens == sum(sizes)
        orc = D.DataLoader(d, B, T, rank, world, shuffle)
        for _ in range(nsteps):
            oi, ot = orc.next_batch()
            li, lt = ours.next_batch()
            assert np.array_equal(li, oi) and np.array_equal(lt, ot)
            assert ours.position() == (orc.shard_idx, orc.sample_idx)


def test_ranks_tile_the_shard(tmp_path, llmk_lib):
    """Without shuffling, the ranks' batches of one step are consecutive
    B*T windows of the shard and targets are inputs shifted by one."""
    import llmk
    B, T, world = 2, 32, 4
    d = make_shards(str(tmp_path / "s"), [world * B * T * 3 + 1])
    toks = np.fromfile(os.path.join(d, "shard_00.bin"), dtype=np.uint16)[512:].astype(np.int32)
    loaders = [llmk.DataLoader(d, B, T, r, world) for r in range(world)]
    for step in range(3):
        for r, ld in enumerate(loaders):
            i, t = ld.next_batch()
            s = (step * world + r) * B * T
            assert np.array_equal(i.reshape(-1), toks[s:s + B * T])
            assert np.array_equal(t.reshape(-1), toks[s + 1:s + B * T + 1])


def test_resume_continues_the_sequence(tmp_path, llmk_lib):
    import llmk
    d = make_shards(str(tmp_path / "s"), [3001, 5000, 2600])
    a = llmk.DataLoader(d, 2, 32, 0, 1)
    seq = [tuple(x.copy() for x in a.next_batch()) for _ in range(70)]
    b = llmk.DataLoader(d, 2, 32, 0, 1)
    for _ in range(40):
        b.next_batch()
    pos = b.position()
    c = llmk.DataLoader(d, 2, 32, 0, 1)
    c.resume(*pos)
    for k in range(40, 70):
        i, t = c.next_batch()
        assert np.array_equal(i, seq[k][0]) and np.array_equal(t, seq[k][1])


@pytest.mark.skipif(not O.ref_available(), reason="reference library not built")
def test_resume_matches_reference(tmp_path, llmk_lib):
    import llmk
    d = make_shards(str(tmp_path / "s"), [3001, 5000, 2600])
    ours, ref = llmk.DataLoader(d, 2, 32, 1, 2), RefLoader(d, 2, 32, 1, 2, False)
    ours.resume(1, 3)
    ref.resume(1, 3)
    for _ in range(12):
        li, lt = ours.next_batch()
        ri, rt = ref.next_batch()
        assert np.array_equal(li, ri) and np.array_equal(lt, rt)


def test_single_file_path_and_reset(tmp_path, llmk_lib):
    import llmk
    d = make_shards(str(tmp_path / "s"), [4097])
    f = os.path.join(d, "shard_00.bin")
    ld = llmk.DataLoader(f, 2, 64)
    first = [x.copy() for x in ld.next_batch()]
    for _ in range(5):
        ld.next_batch()
    ld.reset()
    assert ld.position() == (0, 0)
    i, t = ld.next_batch()
    assert np.array_equal(i, first[0]) and np.array_equal(t, first[1])


def test_bad_shards_fail_cleanly(tmp_path, llmk_lib):
    import llmk
    d = str(tmp_path)
    bad_magic = os.path.join(d, "magic.bin")
    h = np.zeros(256, np.int32)
    h[:3] = [12345, 1, 100]
    with open(bad_magic, "wb") as f:
        f.write(h.tobytes() + np.zeros(100, np.uint16).tobytes())
    with pytest.raises(llmk.LlmkError, match="bad magic"):
        llmk.DataLoader(bad_magic, 1, 8)
    bad_version = os.path.join(d, "version.bin")
    h[:3] = [20240520, 2, 100]
    with open(bad_version, "wb") as f:
        f.write(h.tobytes() + np.zeros(100, np.uint16).tobytes())
    with pytest.raises(llmk.LlmkError, match="bad version"):
        llmk.DataLoader(bad_version, 1, 8)
    short = os.path.join(d, "short.bin")
    h[:3] = [20240520, 1, 100]
    with open(short, "wb") as f:
        f.write(h.tobytes() + np.zeros(99, np.uint16).tobytes())
    with pytest.raises(llmk.LlmkError, match="file size"):
        llmk.DataLoader(short, 1, 8)
    small = os.path.join(d, "small.bin")
    D.write_shard(small, np.arange(64))
    with pytest.raises(llmk.LlmkError, match="fewer than"):
        llmk.DataLoader(small, 1, 64)  # needs B*T+1 = 65 tokens
    with pytest.raises(llmk.LlmkError, match="no shard"):
        llmk.DataLoader(os.path.join(d, "missing"), 1, 8)
    with pytest.raises(llmk.LlmkError, match="bad arguments"):
        llmk.DataLoader(small, 1, 8, rank=2, world=2)
