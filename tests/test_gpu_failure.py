"""Device-side failure detection, exercised without a fault: a bounded wait that runs out.

Every completion wait in the TMA / tensor-core kernels (mbarrier phases of copies and MMAs) is bounded in wall-clock
time. When one runs out, the kernel sets a timeout bit in the context's error word and returns instead of spinning,
and nbl_ctx_check reports NBL_E_DEVICE -- the device-side form of nibble's failure reporting (nibble::Error,
include/nibble/error.h:8-13). nbl_selftest_bounded_wait runs that same wait routine against an mbarrier nothing ever
arrives on, with a 1 ms limit: nothing faults, traps or hangs. The test checks the error is reported, that the check
clears it, and that the same context then computes a correct decode.
"""
import time

import numpy as np
import pytest

import oracle
from helpers import max_rel_err_per_head
from nibble_b200.workloads import make_page_tables

pytestmark = pytest.mark.gpu
D = 64


def test_bounded_wait_runs_out_and_context_recovers():
    import torch
    import nibble_b200 as nb
    from nibble_b200 import _abi
    ctx = nb.Context(0)
    try:
        t0 = time.perf_counter()
        _abi.check(_abi.lib.nbl_selftest_bounded_wait(ctx.handle, 1_000_000))  # 1 ms limit
        with pytest.raises(nb.NibbleError) as e:
            ctx.check()
        elapsed = time.perf_counter() - t0
        assert e.value.status == _abi.NBL_E_DEVICE
        assert "bounded wait" in str(e.value)
        assert elapsed < 5.0, f"the wait was meant to give up after 1 ms; the kernel took {elapsed:.1f} s"
        ctx.check()  # the flag was cleared by the failed check

        # the same context now runs a decode normally (the sticky timeout bit would make every wait give up)
        H, KV = 32, 8
        lens = [1, 700, 4097]
        table, n_pages = make_page_tables(lens, 16, shuffle_seed=4)
        kv = ctx.kv_pool(n_pages, KV)
        g = torch.Generator(device="cuda").manual_seed(8)
        pool = kv.tensor().view(torch.float16)
        pool.copy_(torch.randn(pool.shape, generator=g, device="cuda").half())
        q = np.random.default_rng(3).standard_normal((len(lens), H, D)).astype(np.float32)
        out = torch.full((len(lens), H, D), float("nan"), device="cuda")
        d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
        ctx.attn_decode(kv, d(q), d(table), d(np.array(lens, np.int32)), max(lens), out)
        ctx.check()
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        bits = kv.tensor().cpu().numpy().view(np.uint16)
        for r, L in enumerate(lens):
            k, v = oracle.gather_pages(bits, table[r], L, KV, D, 16)
            ref = oracle.attention(q[r][None], k, v, 1, L - 1, H, KV, D)[0]
            assert max_rel_err_per_head(got[r], ref) <= 1e-4
        kv.close()
    finally:
        ctx.close()


def test_bounded_wait_selftest_rejects_bad_limits():
    import nibble_b200 as nb
    from nibble_b200 import _abi
    ctx = nb.Context(0)
    try:
        assert _abi.lib.nbl_selftest_bounded_wait(ctx.handle, 0) == _abi.NBL_E_INVALID
        assert _abi.lib.nbl_selftest_bounded_wait(ctx.handle, 2_000_000_000) == _abi.NBL_E_INVALID
        ctx.check()
    finally:
        ctx.close()
