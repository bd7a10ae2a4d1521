"""Host-side layout and sharding logic for the paged attention path (no GPU needed).

* page tables: which pool pages hold which positions of which (sequence, layer) row;
* sequence sharding across ranks: even split (batched decode, prefill) and longest-processing-time (LPT)
  bin packing by KV length (ragged decode);
* contiguous KV-sequence splits across ranks for one long context (each rank attends its chunk, then the
  (O, lse) partials are all-gathered and merged).

The reference has none of this (one flat fp32 cache per layer, one process: src/model/transformer.cpp:74-90);
these are the B200 build's own data layout decisions.
"""
from __future__ import annotations

import heapq

import numpy as np


def pages_for(length: int, page_size: int = 16) -> int:
    return (int(length) + page_size - 1) // page_size


def make_page_tables(lens, page_size: int = 16, shuffle_seed: int | None = None, stride: int | None = None,
                     first_page: int = 0):
    """Page tables for rows of the given KV lengths. Returns (table [rows, stride] int32, n_pages).

    Pages are numbered first_page.. in row order, or randomly permuted across all rows with shuffle_seed (the
    "pages shuffled in a shared pool" layout). Unused table slots are -1."""
    lens = np.asarray(lens, dtype=np.int64)
    counts = np.array([pages_for(x, page_size) for x in lens], dtype=np.int64)
    total = int(counts.sum())
    width = int(stride if stride is not None else max(1, counts.max(initial=1)))
    if (counts > width).any():
        raise ValueError("stride smaller than a row's page count")
    ids = np.arange(total, dtype=np.int64) + first_page
    if shuffle_seed is not None:
        ids = np.random.default_rng(shuffle_seed).permutation(ids)
    table = np.full((len(lens), width), -1, dtype=np.int32)
    off = 0
    for r, c in enumerate(counts):
        table[r, :c] = ids[off:off + c]
        off += c
    return table, total


def even_shard(n_units: int, world: int, rank: int) -> range:
    """Contiguous block of unit indices for `rank` (sizes differ by at most one)."""
    base, extra = divmod(n_units, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def lpt_partition(weights, n_parts: int) -> list[list[int]]:
    """Longest-processing-time greedy: items in decreasing weight go to the currently lightest part.
    Deterministic (ties broken by index). Returns item indices per part, each list in increasing order."""
    w = np.asarray(weights, dtype=np.float64)
    order = sorted(range(len(w)), key=lambda i: (-w[i], i))
    heap = [(0.0, p) for p in range(n_parts)]
    parts: list[list[int]] = [[] for _ in range(n_parts)]
    for i in order:
        load, p = heapq.heappop(heap)
        parts[p].append(i)
        heapq.heappush(heap, (load + w[i], p))
    return [sorted(p) for p in parts]


def kv_split(length: int, world: int, page_size: int = 16) -> list[tuple[int, int]]:
    """Splits positions [0, length) into `world` contiguous page-aligned chunks [start, end) of near-equal size
    (the last may be shorter; a chunk may be empty when length is small)."""
    n_pages = pages_for(length, page_size)
    out = []
    for r in range(world):
        blk = even_shard(n_pages, world, r)
        start = min(length, blk.start * page_size)
        end = min(length, blk.stop * page_size)
        out.append((start, end))
    return out


def ragged_lengths(n: int, lo: int, hi: int, seed: int) -> np.ndarray:
    """Context lengths drawn uniformly in [lo, hi] from a seed (the ragged paged-decode workload)."""
    return np.random.default_rng(seed).integers(lo, hi + 1, size=n, dtype=np.int64)
