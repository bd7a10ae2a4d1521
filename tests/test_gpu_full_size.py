"""Parity at the benchmark configurations' full sizes: the exact bench steps of configs 2, 3 and 5 (same shapes, page layouts and
seeds as bench.py), checked on sampled rows against the CPU oracle.

The oracle cannot redo a whole step in seconds, so each test runs the full-size step on the GPU and recomputes a
seeded sample of rows on the CPU from the operands the kernels saw: the roped query (as written by the append) and
the row's keys/values gathered out of the pool on the GPU. Tolerances are the ones the small-shape tests use:
decode max relative error per head <= 1e-4 (fp32 accumulation over the fp16 cache); prefill max abs <= 1e-2 and
per-head cosine >= 0.9999 against the exact-operand fp32 result (only P's rounding to bf16 separates them).
"""
import numpy as np
import pytest

import bench
import oracle
from helpers import max_rel_err_per_head, min_cosine_per_head
from nibble_b200.workloads import lpt_partition, make_page_tables, ragged_lengths, pages_for

pytestmark = pytest.mark.gpu
D, PAGE = 64, 16


def _gather(kv, table_row, length, n_kv, bf16=False):
    """Keys and values [length, n_kv, 64] of one row as fp32, gathered from the pool on the GPU."""
    import torch
    n = pages_for(length, PAGE)
    pages = torch.from_numpy(np.ascontiguousarray(table_row[:n]).astype(np.int64)).cuda()
    blk = kv.tensor()[pages]  # [n, 2, n_kv, 16, 64] int16
    bits = blk.cpu().numpy().view(np.uint16)
    widen = oracle.bf16_bits_to_f32 if bf16 else oracle.fp16_bits_to_f32
    k = widen(bits[:, 0].transpose(0, 2, 1, 3).reshape(n * PAGE, n_kv, D)[:length])
    v = widen(bits[:, 1].transpose(0, 2, 1, 3).reshape(n * PAGE, n_kv, D)[:length])
    return k, v


def _decode_check(ctx, kv, q, out, table, lens, rows, H, KV):
    import torch
    torch.cuda.synchronize()
    for r in rows:
        k, v = _gather(kv, table[r], int(lens[r]), KV)
        qr = q[r].cpu().numpy()
        ref = oracle.attention(qr[None], k, v, 1, int(lens[r]) - 1, H, KV, D)[0]
        err = max_rel_err_per_head(out[r].cpu().numpy(), ref)
        assert err <= 1e-4, f"row {r} (len {lens[r]}): rel err {err}"


def test_config2_batched_decode_full_size():
    """Config 2: 64 sequences x 16 layers = 1024 rows of 4097 fp16 keys, interleaved RoPE theta 5e5."""
    import torch
    import nibble_b200 as nb
    rows, length = bench.SEQ2 * bench.LAYERS2, bench.CTX2 + 1
    ctx = nb.Context(0)
    table, n_pages = make_page_tables([length] * rows, 16, shuffle_seed=100)
    kv = ctx.kv_pool(n_pages, bench.KV2)
    bench.fill_normal_(kv.tensor().view(torch.float16), seed=1000)
    rng = np.random.default_rng(0)
    q_in = torch.from_numpy(rng.standard_normal((rows, bench.H2, D)).astype(np.float32)).cuda()
    k_in = torch.from_numpy(rng.standard_normal((rows, bench.KV2, D)).astype(np.float32)).cuda()
    v_in = torch.from_numpy(rng.standard_normal((rows, bench.KV2, D)).astype(np.float32)).cuda()
    q, out = torch.empty_like(q_in), torch.full_like(q_in, float("nan"))
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    lens = np.full(rows, length, np.int32)
    t_table = d(table)
    ctx.rope_kv_append(kv, q_in, k_in, v_in, q, d(np.arange(rows, dtype=np.int32)),
                       d(np.full(rows, length - 1, np.int32)), t_table, bench.H2, nb.RopeSpec(5e5, False))
    ctx.attn_decode(kv, q, t_table, d(lens), length, out)
    ctx.check()
    sample = [0, 1, 333, 511, 512, 777, rows - 1] + list(np.random.default_rng(2).integers(0, rows, 3))
    _decode_check(ctx, kv, q, out, table, lens, sample, bench.H2, bench.KV2)
    assert torch.isfinite(out).all()
    kv.close()
    ctx.close()


def test_config5_ragged_decode_full_size():
    """Config 5: Qwen heads (14 / 2, NeoX theta 1e6), 256 sequences with lengths U[1, 8192] (seed 5) x 24 layers,
    pages shuffled in one pool."""
    import torch
    import nibble_b200 as nb
    ctx_lens = ragged_lengths(bench.SEQ5, 1, bench.MAXLEN5, seed=5)
    mine = lpt_partition(ctx_lens + 1, 1)[0]
    my_ctx = np.repeat(ctx_lens[mine], bench.LAYERS5)
    lens = (my_ctx + 1).astype(np.int32)
    rows = len(lens)
    ctx = nb.Context(0)
    table, n_pages = make_page_tables(lens, 16, shuffle_seed=500)
    kv = ctx.kv_pool(n_pages, bench.KV5)
    bench.fill_normal_(kv.tensor().view(torch.float16), seed=5000)
    rng = np.random.default_rng(0)
    q_in = torch.from_numpy(rng.standard_normal((rows, bench.H5, D)).astype(np.float32)).cuda()
    k_in = torch.from_numpy(rng.standard_normal((rows, bench.KV5, D)).astype(np.float32)).cuda()
    v_in = torch.from_numpy(rng.standard_normal((rows, bench.KV5, D)).astype(np.float32)).cuda()
    q, out = torch.empty_like(q_in), torch.full_like(q_in, float("nan"))
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    t_table = d(table)
    ctx.rope_kv_append(kv, q_in, k_in, v_in, q, d(np.arange(rows, dtype=np.int32)), d(my_ctx.astype(np.int32)),
                       t_table, bench.H5, nb.RopeSpec(1e6, True))
    ctx.attn_decode(kv, q, t_table, d(lens), int(lens.max()), out)
    ctx.check()
    sample = [int(np.argmin(lens)), int(np.argmax(lens)), 0, rows - 1] + list(np.random.default_rng(3).integers(0, rows, 4))
    _decode_check(ctx, kv, q, out, table, lens, sample, bench.H5, bench.KV5)
    assert torch.isfinite(out).all()
    kv.close()
    ctx.close()


def test_config3_prefill_full_size():
    """Config 3: TinyLlama heads (32 / 4, interleaved theta 1e4), 8 sequences x 2048 bf16 tokens x 22 layers
    = 176 items; sampled rows of three items against the exact-operand fp32 attention."""
    import torch
    import nibble_b200 as nb
    items, T, H, KV = bench.SEQ3 * bench.LAYERS3, bench.T3, bench.H3, bench.KV3
    ctx = nb.Context(0)
    table, n_pages = make_page_tables([T] * items, 16, shuffle_seed=200)
    kv = ctx.kv_pool(n_pages, KV, dtype=nb.BF16)
    n_tok = items * T
    q_in = torch.empty((n_tok, H, D), device="cuda", dtype=torch.bfloat16)
    k_in = torch.empty((n_tok, KV, D), device="cuda", dtype=torch.bfloat16)
    v_in = torch.empty((n_tok, KV, D), device="cuda", dtype=torch.bfloat16)
    for i, t in enumerate((q_in, k_in, v_in)):
        bench.fill_normal_(t, seed=3000 + i)
    q = torch.empty_like(q_in)
    out = torch.full((n_tok, H, D), float("nan"), device="cuda", dtype=torch.bfloat16)
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    t_table = d(table)
    ctx.rope_kv_append(kv, q_in, k_in, v_in, q, d(np.repeat(np.arange(items, dtype=np.int32), T)),
                       d(np.tile(np.arange(T, dtype=np.int32), items)), t_table, H, nb.RopeSpec(1e4, False))
    ctx.attn_prefill(kv, q, d(np.arange(items, dtype=np.int32) * T), d(np.full(items, T, np.int32)),
                     d(np.zeros(items, np.int32)), t_table, T, out)
    ctx.check()
    torch.cuda.synchronize()
    rows_in_item = [0, 1, 63, 64, 127, 128, 129, 511, 1000, 1535, 2046, 2047]
    for it in (0, items // 2, items - 1):
        k, v = _gather(kv, table[it], T, KV, bf16=True)
        for t in rows_in_item:
            g = it * T + t
            qr = q[g].float().cpu().numpy()
            ref = oracle.attention(qr[None], k[:t + 1], v[:t + 1], 1, t, H, KV, D)[0]
            got = out[g].float().cpu().numpy()
            assert np.isfinite(got).all()
            assert np.abs(got - ref).max() <= 1e-2, f"item {it} row {t}"
            assert min_cosine_per_head(got[None], ref[None]) >= 0.9999, f"item {it} row {t}"
    kv.close()
    ctx.close()
