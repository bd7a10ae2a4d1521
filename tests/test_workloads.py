"""Host-side layout and sharding logic (nibble_b200/workloads.py), no GPU."""
import numpy as np
import pytest

from nibble_b200 import workloads as W


def test_page_tables_cover_every_position_once():
    lens = [1, 16, 17, 0, 300]
    for seed in (None, 3):
        table, n = W.make_page_tables(lens, 16, shuffle_seed=seed)
        assert n == sum(W.pages_for(x) for x in lens)
        used = table[table >= 0]
        assert sorted(used.tolist()) == list(range(n)), "every page used exactly once"
        for r, L in enumerate(lens):
            assert (table[r, :W.pages_for(L)] >= 0).all() and (table[r, W.pages_for(L):] == -1).all()
    t1, _ = W.make_page_tables(lens, shuffle_seed=3)
    t2, _ = W.make_page_tables(lens, shuffle_seed=3)
    assert np.array_equal(t1, t2), "seeded shuffles are reproducible"
    with pytest.raises(ValueError):
        W.make_page_tables([100], 16, stride=2)


def test_even_shard_partitions():
    for n in (0, 1, 7, 64):
        for world in (1, 2, 3, 8):
            parts = [W.even_shard(n, world, r) for r in range(world)]
            flat = [i for p in parts for i in p]
            assert flat == list(range(n))
            sizes = [len(p) for p in parts]
            assert max(sizes) - min(sizes) <= 1


def test_lpt_balances_ragged_lengths():
    lens = W.ragged_lengths(256, 1, 8192, seed=5)
    for world in (2, 4, 8):
        parts = W.lpt_partition(lens, world)
        flat = sorted(i for p in parts for i in p)
        assert flat == list(range(256))
        loads = [lens[p].sum() for p in parts]
        # LPT bound: max load <= average + largest item
        assert max(loads) <= lens.sum() / world + lens.max()
        assert max(loads) / (lens.sum() / world) < 1.02  # many small items: near perfect
    assert W.lpt_partition([5, 1], 4)[2:] == [[], []]


def test_kv_split_is_contiguous_and_page_aligned():
    for length in (1, 15, 16, 131073):
        for world in (1, 2, 4, 8):
            chunks = W.kv_split(length, world)
            assert chunks[0][0] == 0 and chunks[-1][1] == length
            for (a, b), (c, d) in zip(chunks, chunks[1:]):
                assert b == c or (a == b == c == d) or b == length
            for a, b in chunks:
                assert (a % 16 == 0 or a == length) and a <= b
    sizes = [b - a for a, b in W.kv_split(131073, 8)]
    assert max(sizes) - min(sizes) <= 2 * 16  # page granularity


def test_ragged_lengths_seeded():
    a = W.ragged_lengths(10, 1, 8192, 7)
    assert np.array_equal(a, W.ragged_lengths(10, 1, 8192, 7)) and a.min() >= 1 and a.max() <= 8192
