"""The config-4 exchange on real GPUs: two ranks (one process per GPU, NCCL) split one long KV sequence into
contiguous chunks, each attends its chunk with nbl_attn_decode (lse out), one NCCL all-gather moves the packed
(O, lse) partials, and nbl_lse_merge gives both ranks the full-context result; the exchange over peer memory
(nbl_lse_exchange_peers: stores into the other rank's symmetric-memory buffer, flags, merge) must give the same
bits on five steps in a row, and so must the decode with that exchange fused into it (nbl_attn_decode_peers). Checked against the CPU oracle on
the whole sequence (max relative error per head <= 1e-4), and the two ranks' merged outputs must be identical.

Needs two GPUs (skipped otherwise). NVLS is off (NCCL_NVLS_ENABLE=0) and the process group has a short timeout,
so a failing rank ends the test with an error instead of a hang.
"""
import os
import socket
import traceback

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
H, KV, D, PAGE = 32, 8, 64, 16
LENGTH, ROWS = 20000, 3


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _inputs():
    """The same full-sequence K/V (fp16 bits, [rows, length, KV, D]) and q on every rank, from one seed."""
    rng = np.random.default_rng(123)
    kv_f = rng.standard_normal((2, ROWS, LENGTH, KV, D)).astype(np.float32)
    import oracle
    bits = oracle.f32_to_fp16_bits(kv_f)
    q = rng.standard_normal((ROWS, H, D)).astype(np.float32)
    return bits, q


def _worker(rank, world, port, outdir):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        import nibble_b200 as nb
        from nibble_b200 import dist as ndist
        from nibble_b200.workloads import kv_split, make_page_tables
        bits, q = _inputs()
        a, b = kv_split(LENGTH, world)[rank]
        my_len = b - a
        ctx = nb.Context(rank)
        table, n_pages = make_page_tables([my_len] * ROWS, PAGE, shuffle_seed=10 + rank)
        kv = ctx.kv_pool(max(1, n_pages), KV)
        # scatter this rank's chunk into its pages: pool[page][0|1][kvh][slot][d]
        pool = np.zeros((max(1, n_pages), 2, KV, PAGE, D), np.uint16)
        for r in range(ROWS):
            for t in range(my_len):
                page, slot = table[r, t // PAGE], t % PAGE
                pool[page, 0, :, slot, :] = bits[0, r, a + t]
                pool[page, 1, :, slot, :] = bits[1, r, a + t]
        kv.tensor().copy_(torch.from_numpy(pool.view(np.int16)).cuda())
        d = lambda x: torch.from_numpy(np.ascontiguousarray(x)).cuda()  # noqa: E731
        out = torch.empty((ROWS, H, D), device="cuda")
        lse = torch.empty((ROWS, H), device="cuda")
        ctx.attn_decode(kv, d(q), d(table), d(np.full(ROWS, my_len, np.int32)), max(1, my_len), out, lse)
        g = ndist.all_gather_partials(ndist.pack_partials(out, lse))
        po, pl = ndist.unpack_partials(g, ROWS, H, D)
        merged = torch.empty((ROWS * H, D), device="cuda")
        ctx.lse_merge(po, pl, merged)
        # the same gathered buffer merged in place (nbl_lse_merge_packed) gives the same bits
        merged_packed = torch.empty_like(merged)
        ctx.lse_merge_packed(g, 2, ROWS * H, D, merged_packed)
        ctx.check()
        assert torch.equal(merged, merged_packed)
        # the exchange over peer memory (stores into the other rank's buffer + flags, nbl_lse_exchange_peers) gives
        # the same bits, call after call (the buffers alternate halves by step; flags count the steps)
        px = ndist.PeerExchange(ctx, ROWS * H, D)
        send = ndist.pack_partials(out, lse)
        for step in range(5):
            merged_peer = torch.full_like(merged, float("nan"))
            px.exchange(send, merged_peer)
            ctx.check()
            assert torch.equal(merged, merged_peer), f"peer exchange differs at step {step}"
        # the decode with the exchange fused in (nbl_attn_decode_peers): the decode kernel stores every finished row
        # into both ranks' buffers and raises the flags itself; the same bits, call after call, interleaved with the
        # unfused exchange (both advance the same step count)
        for step in range(5):
            merged_fused = torch.full((ROWS, H, D), float("nan"), device="cuda")
            px.decode_exchange(kv, d(q), d(table), d(np.full(ROWS, my_len, np.int32)), max(1, my_len), merged_fused)
            ctx.check()
            assert torch.equal(merged.view(ROWS, H, D), merged_fused), f"fused decode + exchange differs at step {step}"
            if step == 2:
                px.exchange(send, merged_peer)
        px.close()
        np.save(os.path.join(outdir, f"merged{rank}.npy"), merged.cpu().numpy())
        dist.barrier()
        kv.close()
        ctx.close()
        dist.destroy_process_group()
    except Exception:
        with open(os.path.join(outdir, f"error{rank}.txt"), "w") as f:
            f.write(traceback.format_exc())
        raise


def test_kv_split_decode_over_two_gpus_matches_full_attention(tmp_path):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    mp.start_processes(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, start_method="spawn", join=True)
    import oracle
    from helpers import max_rel_err_per_head
    m0 = np.load(tmp_path / "merged0.npy").reshape(ROWS, H, D)
    m1 = np.load(tmp_path / "merged1.npy").reshape(ROWS, H, D)
    assert np.array_equal(m0, m1), "ranks disagree on the merged result"
    bits, q = _inputs()
    for r in range(ROWS):
        k = oracle.fp16_bits_to_f32(bits[0, r])
        v = oracle.fp16_bits_to_f32(bits[1, r])
        ref = oracle.attention(q[r][None], k, v, 1, LENGTH - 1, H, KV, D)[0]
        err = max_rel_err_per_head(m0[r], ref)
        assert err <= 1e-4, f"row {r}: rel err {err}"
