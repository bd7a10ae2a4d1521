"""nbl_attn_decode_static -- the decode entry point that allocates no device memory -- against the ordinary
nbl_attn_decode and the CPU oracle, through the C ABI.

Some callers cannot allocate device memory once they are running: an engine that hands all of a GPU's memory to
its own pool at start-up, or a decode loop that cannot absorb cudaMalloc's device-wide synchronisation. For them
the library keeps the split-K partials in a fixed 8 MiB device array instead of growing context scratch. These
tests check that its results equal the ordinary entry point's on two calls in a row (the array is shared and
keeps old contents, so the second call must not be affected by the first), and that a request that does not fit
is refused with an error instead of running. This file is collected last on purpose, and it builds its own
context so it also passes when run alone.
"""

import numpy as np
import pytest

import oracle
from helpers import max_rel_err_per_head
from nibble_b200.workloads import make_page_tables

pytestmark = pytest.mark.gpu
D = 64


def _static_decode(ctx, kv, q, table, lens, max_len, out, lse, n_splits):
    from nibble_b200 import _abi
    _abi.check(_abi.lib.nbl_attn_decode_static(ctx.handle, kv.handle, q.data_ptr(), table.data_ptr(),
                                               table.shape[-1], lens.data_ptr(), max_len, q.shape[0], q.shape[1],
                                               out.data_ptr(), lse.data_ptr(), n_splits))


@pytest.fixture(scope="module")
def setup():
    import torch
    import nibble_b200 as nb
    ctx = nb.Context(0)
    H, KV = 32, 8
    lens = [4097, 1, 700, 131, 2048, 16]  # few rows: the library splits each row, so the partials are used
    table, n_pages = make_page_tables(lens, 16, shuffle_seed=3)
    kv = ctx.kv_pool(n_pages, KV)
    g = torch.Generator(device="cuda").manual_seed(5)
    pool = kv.tensor().view(torch.float16)
    pool.copy_(torch.randn(pool.shape, generator=g, device="cuda").half())
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    yield ctx, kv, d(table), d(np.array(lens, np.int32)), max(lens), H, table, lens
    kv.close()
    ctx.close()


@pytest.mark.parametrize("n_splits", [0, 5])
def test_static_decode_matches_regular_on_two_calls_in_a_row(setup, n_splits):
    import torch
    ctx, kv, table, lens, max_len, H, np_table, np_lens = setup
    rows = lens.shape[0]
    qs = [torch.randn((rows, H, D), device="cuda", generator=torch.Generator(device="cuda").manual_seed(s))
          for s in (11, 12)]
    got = []
    for q in qs:  # two calls of the static entry point back to back, different queries
        out = torch.full((rows, H, D), float("nan"), device="cuda")
        lse = torch.full((rows, H), float("nan"), device="cuda")
        _static_decode(ctx, kv, q, table, lens, max_len, out, lse, n_splits)
        got.append((out, lse))
    ctx.check()
    for q, (out, lse) in zip(qs, got):
        ref = torch.empty_like(out)
        ref_lse = torch.empty_like(lse)
        ctx.attn_decode(kv, q, table, lens, max_len, ref, ref_lse, n_splits=n_splits)
        ctx.check()
        torch.cuda.synchronize()
        assert max_rel_err_per_head(out.cpu().numpy(), ref.cpu().numpy()) <= 1e-4
        np.testing.assert_allclose(lse.cpu().numpy(), ref_lse.cpu().numpy(), rtol=0, atol=2e-5)
    # and against the CPU oracle (nibble's scalar attention restated) on the same fp16 pages
    bits = kv.tensor().cpu().numpy().view(np.uint16)
    KV = kv.n_kv_heads
    for q, (out, _) in zip(qs, got):
        qn, on = q.cpu().numpy(), out.cpu().numpy()
        for r, L in enumerate(np_lens):
            k, v = oracle.gather_pages(bits, np_table[r], L, KV, D, 16)
            want = oracle.attention(qn[r][None], k, v, 1, L - 1, H, KV, D)[0]
            assert max_rel_err_per_head(on[r], want) <= 1e-4, f"row {r} (length {L})"


def test_static_decode_refuses_partials_larger_than_its_array(setup):
    import torch
    import nibble_b200 as nb
    ctx, kv, table, lens, max_len, H, _, _ = setup
    rows = 128  # 16 splits requested -> 10 splits of 2 pages: 10 x 128 rows x 32 heads x 65 floats = 10.6 MB > 8 MiB
    big_table = torch.zeros((rows, table.shape[-1]), dtype=torch.int32, device="cuda")
    big_lens = torch.full((rows,), 300, dtype=torch.int32, device="cuda")
    q = torch.zeros((rows, H, D), device="cuda")
    out = torch.zeros_like(q)
    lse = torch.zeros((rows, H), device="cuda")
    with pytest.raises(nb.NibbleError) as e:
        _static_decode(ctx, kv, q, big_table, big_lens, 300, out, lse, 16)
    assert e.value.status == nb._abi.NBL_E_INVALID and "static" in str(e.value)
    _static_decode(ctx, kv, q, big_table, big_lens, 300, out, lse, 0)  # the library-chosen count fits
    ctx.check()


def test_static_decode_allocates_no_device_memory():
    """Free device memory (cudaMemGetInfo) is the same before the entry point's first call on a fresh context and
    after two calls: one on the first 8 rows with the library's own split count (37 splits: the rows are split to
    fill one wave of CTAs, merged through the static counters), one on all rows with an explicit count whose
    partials fill most of the array. The context, pool and every tensor exist before the first reading."""
    import torch
    import nibble_b200 as nb
    ctx = nb.Context(0)
    H, KV = 8, 1
    rows = 544  # 7 splits x 544 rows x 8 heads x 65 floats = 7.9 MB of the 8 MiB array
    few = 8  # library plan: 8 units on 148 SMs x 2 CTAs -> 37 splits
    lens = [8192] * rows
    table, n_pages = make_page_tables(lens, 16, shuffle_seed=9)
    kv = ctx.kv_pool(n_pages, KV)
    g = torch.Generator(device="cuda").manual_seed(7)
    pool = kv.tensor().view(torch.float16)
    pool.copy_(torch.randn(pool.shape, generator=g, device="cuda").half())
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    t_table, t_lens = d(table), d(np.array(lens, np.int32))
    q = torch.randn((rows, H, D), device="cuda", generator=g)
    outs = [torch.full((rows, H, D), float("nan"), device="cuda") for _ in range(2)]
    lses = [torch.full((rows, H), float("nan"), device="cuda") for _ in range(2)]
    ref, ref_lse = torch.empty_like(q), torch.empty((rows, H), device="cuda")
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    _static_decode(ctx, kv, q[:few], t_table[:few], t_lens[:few], 8192, outs[0][:few], lses[0][:few], 0)
    _static_decode(ctx, kv, q, t_table, t_lens, 8192, outs[1], lses[1], 7)  # 7.9 MB of the 8 MiB array
    ctx.check()
    torch.cuda.synchronize()
    free1 = torch.cuda.mem_get_info()[0]
    assert free1 == free0, f"free device memory changed by {free0 - free1} bytes"
    ctx.attn_decode(kv, q, t_table, t_lens, 8192, ref, ref_lse)  # the ordinary entry point, after the reading
    ctx.check()
    torch.cuda.synchronize()
    for out, lse, n in zip(outs, lses, (few, rows)):
        assert max_rel_err_per_head(out[:n].cpu().numpy(), ref[:n].cpu().numpy()) <= 1e-4
        np.testing.assert_allclose(lse[:n].cpu().numpy(), ref_lse[:n].cpu().numpy(), rtol=0, atol=2e-5)
    kv.close()
    ctx.close()


def test_static_decode_long_rows_with_the_library_split_count():
    """Sixteen 65,537-token rows of 8 query heads over one KV head: the library splits every row 18 ways (16 units
    fill one wave of CTAs), and the last split of each row merges all 18 through the static arrival counters. Two
    calls in a row (the counters must be back at zero after each launch) match the ordinary entry point."""
    import torch
    import nibble_b200 as nb
    ctx = nb.Context(0)
    H, KV, rows, L = 8, 1, 16, 65537
    table, n_pages = make_page_tables([L] * rows, 16, shuffle_seed=15)
    kv = ctx.kv_pool(n_pages, KV)
    g = torch.Generator(device="cuda").manual_seed(16)
    pool = kv.tensor().view(torch.float16)
    pool.copy_(torch.randn(pool.shape, generator=g, device="cuda").half())
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    t_table, t_lens = d(table), d(np.full(rows, L, np.int32))
    ref, ref_lse = torch.empty((rows, H, D), device="cuda"), torch.empty((rows, H), device="cuda")
    for seed in (17, 18):
        q = torch.randn((rows, H, D), device="cuda", generator=torch.Generator(device="cuda").manual_seed(seed))
        out = torch.full((rows, H, D), float("nan"), device="cuda")
        lse = torch.full((rows, H), float("nan"), device="cuda")
        _static_decode(ctx, kv, q, t_table, t_lens, L, out, lse, 0)
        ctx.attn_decode(kv, q, t_table, t_lens, L, ref, ref_lse)
        ctx.check()
        torch.cuda.synchronize()
        assert max_rel_err_per_head(out.cpu().numpy(), ref.cpu().numpy()) <= 1e-4
        np.testing.assert_allclose(lse.cpu().numpy(), ref_lse.cpu().numpy(), rtol=0, atol=2e-5)
    kv.close()
    ctx.close()


def test_static_decode_many_rows_with_the_library_split_count():
    """2100 rows of 8 query heads over one KV head: the library runs one split per row (no partials), and the
    static entry point's results match the ordinary entry point's, on two calls in a row."""
    import torch
    import nibble_b200 as nb
    ctx = nb.Context(0)
    H, KV, rows, L = 8, 1, 2100, 1024
    table, n_pages = make_page_tables([L] * rows, 16, shuffle_seed=11)
    kv = ctx.kv_pool(n_pages, KV)
    g = torch.Generator(device="cuda").manual_seed(12)
    pool = kv.tensor().view(torch.float16)
    pool.copy_(torch.randn(pool.shape, generator=g, device="cuda").half())
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    t_table, t_lens = d(table), d(np.full(rows, L, np.int32))
    ref, ref_lse = torch.empty((rows, H, D), device="cuda"), torch.empty((rows, H), device="cuda")
    for seed in (13, 14):
        q = torch.randn((rows, H, D), device="cuda", generator=torch.Generator(device="cuda").manual_seed(seed))
        out = torch.full((rows, H, D), float("nan"), device="cuda")
        lse = torch.full((rows, H), float("nan"), device="cuda")
        _static_decode(ctx, kv, q, t_table, t_lens, L, out, lse, 0)
        ctx.attn_decode(kv, q, t_table, t_lens, L, ref, ref_lse)
        ctx.check()
        torch.cuda.synchronize()
        assert max_rel_err_per_head(out.cpu().numpy(), ref.cpu().numpy()) <= 1e-4
        np.testing.assert_allclose(lse.cpu().numpy(), ref_lse.cpu().numpy(), rtol=0, atol=2e-5)
    kv.close()
    ctx.close()
