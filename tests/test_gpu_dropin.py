"""GPU parity of the drop-in Backend operations (fp32 device buffers, the reference's own layouts) through the
C ABI: nbl_rope, nbl_add_bias, nbl_attention, nbl_alloc/free/read/write, against the committed golden fixtures
(nibble's own outputs) and the C oracle.

Tolerances: RoPE bit-identical (same double-precision angles, uncontracted float rotation); attention max
relative error per head <= 1e-4 against the fp32 CPU result (the decode tolerance of the attention path), and max abs error
<= 2e-5 * max(1, q scale).
"""
import glob
import os

import numpy as np
import pytest

import oracle
from helpers import max_rel_err_per_head

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")


def dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    import torch
    torch.cuda.synchronize()
    return t.cpu().numpy()


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLD, "rope_*.npz"))),
                         ids=lambda p: os.path.basename(p)[5:-4])
def test_rope_bit_identical_to_reference(nbl_ctx, path):
    import nibble_b200 as nb
    f = np.load(path)
    n, H, D, pos0, neox = (int(x) for x in f["meta"])
    ff = tuple(float(x) for x in f["ff"]) if f["ff"].size else None
    x = dev(f["x"])
    nbl_ctx.rope(x, n, H, D, pos0, nb.RopeSpec(float(f["base"]), bool(neox), ff))
    got = host(x)
    assert np.array_equal(got.view(np.uint32), f["out"].view(np.uint32))


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLD, "attention_*.npz"))),
                         ids=lambda p: os.path.basename(p)[10:-4])
def test_attention_matches_reference(nbl_ctx, path):
    import torch
    f = np.load(path)
    n, pos0, H, KV, D = (int(x) for x in f["meta"])
    q, k, v = dev(f["q"]), dev(f["k"]), dev(f["v"])
    out = torch.full((n, H, D), float("nan"), device="cuda")
    nbl_ctx.attention(q, k, v, out, n, pos0, H, KV, D)
    got = host(out)
    ref = f["out_scalar"]
    qscale = max(1.0, float(np.abs(f["q"]).max()) / 4.0)
    assert max_rel_err_per_head(got, ref) <= 1e-4
    assert np.abs(got - ref).max() <= 2e-5 * qscale


def test_add_bias(nbl_ctx):
    rng = np.random.default_rng(3)
    x = rng.standard_normal((5, 96)).astype(np.float32)
    b = rng.standard_normal(96).astype(np.float32)
    xd = dev(x)
    nbl_ctx.add_bias(xd, dev(b), 96, 5)
    assert np.array_equal(host(xd), oracle.add_bias(x, b, 5).reshape(5, 96))


def test_backend_memory_contract(nbl_ctx):
    import nibble_b200 as nb
    p = nbl_ctx.alloc(1000)
    buf = np.full(1000, 7.0, np.float32)
    nbl_ctx.read(buf, p, 1000)
    assert np.all(buf == 0.0), "alloc returns zeroed memory (backend.h:46)"
    src = np.arange(1000, dtype=np.float32)
    nbl_ctx.write(p, src, 1000)
    nbl_ctx.read(buf, p, 1000)
    assert np.array_equal(buf, src)
    nbl_ctx.free(p)
    nbl_ctx.free(None)          # no-op
    nbl_ctx.free(0x1234560)     # not ours: ignored, like CpuBackend::free
    with pytest.raises(nb.NibbleError) as e:
        nbl_ctx.alloc(-1)
    assert e.value.status == 1 and "negative" in str(e.value)
    assert nbl_ctx.alloc(0) != 0  # zero-size blocks are valid, distinct allocations


def test_attention_rejects_bad_geometry(nbl_ctx):
    import torch
    import nibble_b200 as nb
    q = torch.zeros(6 * 16, device="cuda")
    with pytest.raises(nb.NibbleError):
        nbl_ctx.attention(q, q, q, q, 1, 0, 6, 4, 16)  # 6 heads not a multiple of 4 KV heads
    with pytest.raises(nb.NibbleError):
        nbl_ctx.attention(q, q, q, q, 1, -1, 6, 2, 16)


def test_config1_qwen_prefill_then_decode_every_step(nbl_ctx):
    """Benchmark config 1: Qwen2.5-0.5B attention shape, one layer, fp32 on the reference's own layout. Prefill
    128 tokens, then 128 single-token decode steps; every step is checked against nibble's scalar attention
    (through the oracle, which tests/test_oracle.py pins bit-exactly to it). The op sequence is the
    Transformer's: K/V rows written into the cache at pos0, rope(q), rope(k cache rows), attention."""
    import torch
    import nibble_b200 as nb
    H, KV, D = 14, 2, 64
    rope = nb.RopeSpec(1e6, True)
    rng = np.random.default_rng(1234)
    q_all = rng.standard_normal((256, H, D)).astype(np.float32)
    k_all = rng.standard_normal((256, KV, D)).astype(np.float32)
    v_all = rng.standard_normal((256, KV, D)).astype(np.float32)
    kc = torch.zeros((256, KV, D), device="cuda")
    vc = torch.zeros((256, KV, D), device="cuda")
    out = torch.zeros((128, H, D), device="cuda")
    # CPU side, in the reference's order
    k_ref = np.zeros_like(k_all)
    v_ref = np.zeros_like(v_all)
    worst = 0.0

    def step(pos0, n):
        nonlocal worst
        qd = dev(q_all[pos0:pos0 + n])
        kc[pos0:pos0 + n] = dev(k_all[pos0:pos0 + n])
        vc[pos0:pos0 + n] = dev(v_all[pos0:pos0 + n])
        nbl_ctx.rope(qd, n, H, D, pos0, rope)
        nbl_ctx.rope(kc[pos0:pos0 + n], n, KV, D, pos0, rope)
        o = out[:n]
        nbl_ctx.attention(qd, kc, vc, o, n, pos0, H, KV, D)
        q_r = oracle.rope(q_all[pos0:pos0 + n], H, D, pos0, 1e6, True)
        k_ref[pos0:pos0 + n] = oracle.rope(k_all[pos0:pos0 + n], KV, D, pos0, 1e6, True).reshape(n, KV, D)
        v_ref[pos0:pos0 + n] = v_all[pos0:pos0 + n]
        ref = oracle.attention(q_r, k_ref[:pos0 + n], v_ref[:pos0 + n], n, pos0, H, KV, D)
        got = host(o)
        assert np.array_equal(host(qd).view(np.uint32), q_r.reshape(n, H, D).view(np.uint32))
        err = max_rel_err_per_head(got, ref)
        worst = max(worst, err)
        assert err <= 1e-4, f"pos0={pos0} n={n}: rel err {err}"

    step(0, 128)
    for t in range(128, 256):
        step(t, 1)
    assert worst <= 1e-4


@pytest.mark.parametrize("n,pos0,H,KV,D", [(1, 999, 8, 2, 256), (3, 500, 4, 4, 160), (2, 2000, 32, 4, 64),
                                           (40, 0, 2, 1, 130), (1, 0, 4, 2, 64), (5, 31, 6, 3, 96)])
def test_attention_wide_heads_and_long_context(nbl_ctx, n, pos0, H, KV, D):
    """head_dim above 128 (the 4-warp configuration), contexts spanning many 32-key chunks per warp, a single key,
    and keys that end inside a warp's first chunk; against the C oracle (nibble's scalar attention)."""
    import torch
    rng = np.random.default_rng(n * 7 + pos0 + D)
    L = pos0 + n
    q = rng.standard_normal((n, H, D)).astype(np.float32)
    k = rng.standard_normal((L, KV, D)).astype(np.float32)
    v = rng.standard_normal((L, KV, D)).astype(np.float32)
    out = torch.full((n, H, D), float("nan"), device="cuda")
    nbl_ctx.attention(dev(q), dev(k), dev(v), out, n, pos0, H, KV, D)
    ref = oracle.attention(q, k, v, n, pos0, H, KV, D)
    assert max_rel_err_per_head(host(out), ref) <= 1e-4


@pytest.mark.parametrize("n,pos0,H,KV,D", [(16, 0, 8, 2, 64), (100, 37, 4, 1, 128), (300, 500, 14, 2, 64),
                                           (65, 3, 6, 3, 128), (64, 0, 32, 4, 64)])
def test_attention_query_tiles(nbl_ctx, n, pos0, H, KV, D):
    """Prefill chunks of 16 rows or more with head_dim 64 or 128 run 64-query tiles: a partial last tile, keys
    before the chunk (pos0 > 0), GQA ratios 4, 7, 2 and 8; against the C oracle (nibble's scalar attention)."""
    import torch
    rng = np.random.default_rng(n + pos0 + D + H)
    L = pos0 + n
    q = rng.standard_normal((n, H, D)).astype(np.float32)
    k = rng.standard_normal((L, KV, D)).astype(np.float32)
    v = rng.standard_normal((L, KV, D)).astype(np.float32)
    out = torch.full((n, H, D), float("nan"), device="cuda")
    nbl_ctx.attention(dev(q), dev(k), dev(v), out, n, pos0, H, KV, D)
    ref = oracle.attention(q, k, v, n, pos0, H, KV, D)
    assert max_rel_err_per_head(host(out), ref) <= 1e-4
