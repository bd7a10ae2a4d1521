"""The multi-rank protocols on CPU ranks (torch.distributed gloo, world size 2), no GPU:

* long-context decode split along the KV sequence: each rank attends its contiguous chunk (here with the CPU
  oracle standing in for the kernel), packs (O, lse), one all-gather, LSE merge -> equals full attention;
* sequence sharding: the shards of all ranks cover every row exactly once (even split and LPT).
* failure on the host: a rank that raises before the collective makes the others' collective fail with an
  error inside a short process-group timeout instead of hanging.
"""
import math
import os
import socket
import traceback

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

H, KV, D = 8, 2, 16


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _chunk_partial(q, k, v, a, b):
    """(O, lse) of one KV chunk [a, b) in double, per head (the decode kernel's partial form)."""
    g = H // KV
    if b <= a:
        return np.zeros((H, D)), np.full(H, -np.inf)
    kk = np.repeat(k[a:b].astype(np.float64), g, axis=1)
    vv = np.repeat(v[a:b].astype(np.float64), g, axis=1)
    s = np.einsum("hd,jhd->hj", q.astype(np.float64), kk) / math.sqrt(D)
    m = s.max(1)
    p = np.exp(s - m[:, None])
    return np.einsum("hj,jhd->hd", p, vv) / p.sum(1)[:, None], m + np.log(p.sum(1))


def _worker(rank, world, port, mode, errfile):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        import datetime
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
        import oracle
        from nibble_b200 import dist as ndist
        from nibble_b200 import workloads as W
        if mode == "kv_split":
            rng = np.random.default_rng(0)  # same inputs on every rank
            length, rows = 1000, 3
            q = rng.standard_normal((rows, H, D)).astype(np.float32)
            k = rng.standard_normal((rows, length, KV, D)).astype(np.float32)
            v = rng.standard_normal((rows, length, KV, D)).astype(np.float32)
            a, b = W.kv_split(length, world)[rank]
            o = np.zeros((rows, H, D), np.float32)
            lse = np.zeros((rows, H), np.float32)
            for r in range(rows):
                o[r], lse[r] = _chunk_partial(q[r], k[r], v[r], a, b)
            packed = ndist.pack_partials(torch.from_numpy(o), torch.from_numpy(lse))
            gathered = ndist.all_gather_partials(packed)
            part_o, part_lse = ndist.unpack_partials(gathered, rows, H, D)
            out, _ = oracle.lse_merge(part_o.numpy(), part_lse.numpy())
            for r in range(rows):
                full = oracle.attention(q[r][None], k[r], v[r], 1, length - 1, H, KV, D)[0]
                assert np.abs(out.reshape(rows, H, D)[r] - full).max() <= 2e-6
        elif mode == "shards":
            lens = W.ragged_lengths(64, 1, 8192, seed=1)
            mine = torch.tensor(sorted(W.lpt_partition(lens, world)[rank]) + [-1] * 64)[:64]
            even = torch.tensor(list(W.even_shard(64, world, rank)) + [-1] * 64)[:64]
            got = [torch.empty(64, dtype=torch.int64) for _ in range(world)]
            dist.all_gather(got, mine)
            ids = sorted(int(x) for t in got for x in t if x >= 0)
            assert ids == list(range(64))
            dist.all_gather(got, even)
            ids = sorted(int(x) for t in got for x in t if x >= 0)
            assert ids == list(range(64))
        elif mode == "rank_fails":
            if rank == 1:
                raise SystemExit(0)  # leaves before the collective, between steps
            try:
                dist.all_reduce(torch.ones(4))
            except Exception:
                return  # the survivor sees an error, not a hang
            raise AssertionError("collective with a departed rank completed")
        dist.destroy_process_group()
    except SystemExit:
        raise
    except Exception:
        with open(errfile, "a") as f:
            f.write(f"rank {rank}: {traceback.format_exc()}\n")
        raise


@pytest.mark.parametrize("mode", ["kv_split", "shards"])
def test_two_ranks(tmp_path, mode):
    errfile = str(tmp_path / "err.txt")
    mp.start_processes(_worker, args=(2, _free_port(), mode, errfile), nprocs=2, join=True, start_method="spawn")
    assert not os.path.exists(errfile), open(errfile).read()


def test_departed_rank_fails_collective_quickly(tmp_path):
    errfile = str(tmp_path / "err.txt")
    ctx = mp.start_processes(_worker, args=(2, _free_port(), "rank_fails", errfile), nprocs=2, join=False,
                             start_method="spawn")
    import time
    t0 = time.time()
    while not ctx.join(timeout=60):
        assert time.time() - t0 < 60, "collective hung"
    assert not os.path.exists(errfile), open(errfile).read()
