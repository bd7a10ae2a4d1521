"""GPU parity of the paged K/V path through the C ABI: fused bias->RoPE->append, split-K flash-decode, LSE merge
and the tcgen05 prefill, against the C oracle (pinned bit-exactly to nibble's scalar code by test_oracle.py).

Tolerances (those of the attention path):
  * append: bit-identical (q_out fp32 = cpu::rope(q + bq); pool K = fp16/bf16 RNE of cpu::rope(k + bk)).
  * decode (fp32 accumulate over the fp16 cache): max relative error per head <= 1e-4 against the fp32 CPU
    result on the same fp16 values widened.
  * prefill (bf16 tensor cores): max abs error <= 2e-2 and per-head cosine >= 0.9999 against the fp32 CPU
    result on the bf16 inputs widened (RoPE in fp32, as nibble runs it).
"""
import math

import numpy as np
import pytest

import oracle
from helpers import max_rel_err_per_head, min_cosine_per_head
from nibble_b200.workloads import make_page_tables

pytestmark = pytest.mark.gpu
D = 64


def dev(a, dtype=None):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t if dtype is None else t.to(dtype)


def host(t):
    import torch
    torch.cuda.synchronize()
    return t.cpu().numpy()


def pool_bits(kv):
    import torch
    torch.cuda.synchronize()
    return kv.tensor().cpu().numpy().view(np.uint16)


def fill_random(kv, seed):
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    dt = torch.float16 if kv.dtype == 1 else torch.bfloat16
    t = kv.tensor().view(dt)
    t.copy_(torch.randn(t.shape, generator=g, device="cuda", dtype=torch.float32).to(dt))


def ref_lse(q, k, v_unused, H, KV):
    """ln sum_j exp(q.k_j / 8) per head, in double."""
    g = H // KV
    kk = np.repeat(k.astype(np.float64), g, axis=1)  # [len, H, D]
    s = np.einsum("hd,jhd->hj", q.astype(np.float64), kk) / math.sqrt(D)
    m = s.max(1)
    return m + np.log(np.exp(s - m[:, None]).sum(1))


# ---------------------------------------------------------------- fused bias + RoPE + append
@pytest.mark.parametrize("cfg", ["qwen_neox_bias_f16", "llama_interleaved_factors_f16", "tinyllama_bf16_in_bf16"])
def test_rope_kv_append_bit_exact(nbl_ctx, cfg):
    import torch
    import nibble_b200 as nb
    if cfg == "qwen_neox_bias_f16":
        H, KV, base, neox, ff, bias, pool_dt, in_dt = 14, 2, 1e6, True, None, True, nb.F16, torch.float32
    elif cfg == "llama_interleaved_factors_f16":
        H, KV, base, neox, bias, pool_dt, in_dt = 32, 8, 5e5, False, False, nb.F16, torch.float32
        ff = tuple(float(x) for x in np.linspace(1.0, 8.0, D // 2, dtype=np.float32))
    else:
        H, KV, base, neox, ff, bias, pool_dt, in_dt = 32, 4, 1e4, False, None, False, nb.BF16, torch.bfloat16
    rng = np.random.default_rng(hash(cfg) % 2 ** 32)
    lens = [40, 17, 300]
    table, n_pages = make_page_tables(lens, 16, shuffle_seed=5)
    kv = nbl_ctx.kv_pool(n_pages + 2, KV, dtype=pool_dt)
    rows = np.concatenate([np.full(L, r) for r, L in enumerate(lens)]).astype(np.int32)
    pos = np.concatenate([np.arange(L) for L in lens]).astype(np.int32)
    perm = rng.permutation(len(rows))  # tokens in any order
    rows, pos = rows[perm], pos[perm]
    n = len(rows)
    q_in = rng.standard_normal((n, H, D)).astype(np.float32)
    k_in = rng.standard_normal((n, KV, D)).astype(np.float32)
    v_in = rng.standard_normal((n, KV, D)).astype(np.float32)
    bq = rng.standard_normal(H * D).astype(np.float32) if bias else None
    bk = rng.standard_normal(KV * D).astype(np.float32) if bias else None
    bv = rng.standard_normal(KV * D).astype(np.float32) if bias else None
    qd, kd, vd = dev(q_in, in_dt), dev(k_in, in_dt), dev(v_in, in_dt)
    q_out = torch.empty((n, H, D), device="cuda", dtype=torch.float32)
    nbl_ctx.rope_kv_append(kv, qd, kd, vd, q_out, dev(rows), dev(pos), dev(table), H,
                           nb.RopeSpec(base, neox, ff), bq=None if bq is None else dev(bq),
                           bk=None if bk is None else dev(bk), bv=None if bv is None else dev(bv))
    nbl_ctx.check()
    # what the GPU saw as input (bf16 inputs are widened exactly)
    q_w, k_w, v_w = (host(t.float()) for t in (qd, kd, vd))
    ffa = None if ff is None else np.array(ff, np.float32)
    got_q = host(q_out)
    pool = pool_bits(kv)
    narrow = oracle.f32_to_fp16_bits if pool_dt == nb.F16 else oracle.f32_to_bf16_bits
    for i in range(n):
        qi = q_w[i] if bq is None else oracle.add_bias(q_w[i], bq, 1).reshape(H, D)
        ki = k_w[i] if bk is None else oracle.add_bias(k_w[i], bk, 1).reshape(KV, D)
        vi = v_w[i] if bv is None else oracle.add_bias(v_w[i], bv, 1).reshape(KV, D)
        q_ref = oracle.rope(qi, H, D, int(pos[i]), base, neox, ffa).reshape(H, D)
        k_ref = oracle.rope(ki, KV, D, int(pos[i]), base, neox, ffa).reshape(KV, D)
        assert np.array_equal(got_q[i].view(np.uint32), q_ref.view(np.uint32)), f"q token {i}"
        page, slot = table[rows[i], pos[i] // 16], pos[i] % 16
        assert np.array_equal(pool[page, 0, :, slot, :], narrow(k_ref)), f"k token {i}"
        assert np.array_equal(pool[page, 1, :, slot, :], narrow(vi)), f"v token {i}"


@pytest.mark.parametrize("neox,offset", [(False, 0), (True, 0), (False, 4), (False, 1), (True, 2), (True, 3)])
def test_rope_kv_append_vector_and_scalar_paths(nbl_ctx, neox, offset):
    """The 8-element vector path (16-byte-aligned rows) and the per-pair path (q/k/v that start off a 16-byte
    boundary: `offset` shifts them by that many fp32 elements, 4 staying aligned) give the reference's bits, with
    bias on every stream."""
    import torch
    import nibble_b200 as nb
    H, KV, base, hd = 6, 2, 1e4, D
    rng = np.random.default_rng(offset + (7 if neox else 0))
    lens = [33, 5]
    table, n_pages = make_page_tables(lens, 16, shuffle_seed=2)
    kv = nbl_ctx.kv_pool(n_pages, KV, dtype=nb.BF16)
    rows = np.concatenate([np.full(L, r) for r, L in enumerate(lens)]).astype(np.int32)
    pos = np.concatenate([np.arange(L) for L in lens]).astype(np.int32)
    n = len(rows)

    def shifted(a):  # a device copy of `a` whose data pointer sits `offset` fp32 elements into its buffer
        flat = torch.zeros(a.size + offset, device="cuda", dtype=torch.float32)
        flat[offset:] = torch.from_numpy(a.ravel()).cuda()
        return flat[offset:].view(a.shape)

    q_in = rng.standard_normal((n, H, hd)).astype(np.float32)
    k_in = rng.standard_normal((n, KV, hd)).astype(np.float32)
    v_in = rng.standard_normal((n, KV, hd)).astype(np.float32)
    bq, bk, bv = (rng.standard_normal(w * hd).astype(np.float32) for w in (H, KV, KV))
    q_out = torch.empty((n, H, hd), device="cuda", dtype=torch.float32)
    nbl_ctx.rope_kv_append(kv, shifted(q_in), shifted(k_in), shifted(v_in), q_out, dev(rows), dev(pos), dev(table),
                           H, nb.RopeSpec(base, neox), bq=dev(bq), bk=dev(bk), bv=dev(bv))
    nbl_ctx.check()
    got_q = host(q_out)
    pool = pool_bits(kv)
    for i in range(n):
        qi = oracle.add_bias(q_in[i], bq, 1).reshape(H, hd)
        ki = oracle.add_bias(k_in[i], bk, 1).reshape(KV, hd)
        vi = oracle.add_bias(v_in[i], bv, 1).reshape(KV, hd)
        q_ref = oracle.rope(qi, H, hd, int(pos[i]), base, neox).reshape(H, hd)
        k_ref = oracle.rope(ki, KV, hd, int(pos[i]), base, neox).reshape(KV, hd)
        assert np.array_equal(got_q[i].view(np.uint32), q_ref.view(np.uint32)), f"q token {i}"
        page, slot = table[rows[i], pos[i] // 16], pos[i] % 16
        assert np.array_equal(pool[page, 0, :, slot, :], oracle.f32_to_bf16_bits(k_ref)), f"k token {i}"
        assert np.array_equal(pool[page, 1, :, slot, :], oracle.f32_to_bf16_bits(vi)), f"v token {i}"


# ---------------------------------------------------------------- decode
DECODE_LENS = [1, 15, 16, 17, 33, 100, 257, 1000, 2049]


@pytest.mark.parametrize("H,KV", [(14, 2), (32, 8), (32, 4), (8, 8), (6, 2), (7, 1)])
@pytest.mark.parametrize("n_splits", [1, 0, 3])
def test_decode_matches_oracle(nbl_ctx, H, KV, n_splits):
    import torch
    lens = DECODE_LENS
    table, n_pages = make_page_tables(lens, 16, shuffle_seed=H * 31 + KV)
    kv = nbl_ctx.kv_pool(n_pages + 1, KV)
    fill_random(kv, seed=H + KV)
    rng = np.random.default_rng(H * 7 + KV)
    q = rng.standard_normal((len(lens), H, D)).astype(np.float32)
    out = torch.full((len(lens), H, D), float("nan"), device="cuda")
    lse = torch.full((len(lens), H), float("nan"), device="cuda")
    nbl_ctx.attn_decode(kv, dev(q), dev(table), dev(np.array(lens, np.int32)), max(lens), out, lse,
                        n_splits=n_splits)
    nbl_ctx.check()
    got, got_lse = host(out), host(lse)
    pool = pool_bits(kv)
    for r, L in enumerate(lens):
        k, v = oracle.gather_pages(pool, table[r], L, KV, D, 16)
        ref = oracle.attention(q[r][None], k, v, 1, L - 1, H, KV, D)[0]
        err = max_rel_err_per_head(got[r], ref)
        assert err <= 1e-4, f"row {r} len {L}: rel err {err}"
        np.testing.assert_allclose(got_lse[r], ref_lse(q[r], k, v, H, KV), rtol=0, atol=2e-5)


@pytest.mark.parametrize("n_chunks,bias", [(3, False), (0, True), (1, False)])
def test_decode_step_host_matches_separate_calls(nbl_ctx, n_chunks, bias):
    """nbl_decode_step_host (host q/k/v in, host out; uploads, append + decode and downloads overlapped over row
    chunks) equals nbl_write + nbl_rope_kv_append + nbl_attn_decode + nbl_read on the same data, and the oracle."""
    import torch
    import nibble_b200 as nb
    H, KV = 32, 8
    rng = np.random.default_rng(n_chunks * 3 + int(bias))
    lens = [int(x) for x in rng.integers(1, 3000, size=37)] + [1, 4097]  # counting the new token
    rows = len(lens)
    table, n_pages = make_page_tables(lens, 16, shuffle_seed=21)
    kv = nbl_ctx.kv_pool(n_pages, KV)
    fill_random(kv, seed=22)
    q_in = torch.from_numpy(rng.standard_normal((rows, H, D)).astype(np.float32)).pin_memory()
    k_in = torch.from_numpy(rng.standard_normal((rows, KV, D)).astype(np.float32)).pin_memory()
    v_in = torch.from_numpy(rng.standard_normal((rows, KV, D)).astype(np.float32)).pin_memory()
    bq, bk, bv = ((dev(rng.standard_normal(w * D).astype(np.float32)) if bias else None) for w in (H, KV, KV))
    out_h = torch.full((rows, H, D), float("nan")).pin_memory()
    t_table, t_lens = dev(table), dev(np.array(lens, np.int32))
    spec = nb.RopeSpec(5e5, False)
    nbl_ctx.decode_step_host(kv, q_in, k_in, v_in, t_table, t_lens, max(lens), spec, out_h, bq=bq, bk=bk, bv=bv,
                             n_chunks=n_chunks)
    nbl_ctx.check()
    got = out_h.numpy().copy()
    # the same step as separate calls (the append rewrites the same bits at the same slots)
    q = torch.empty((rows, H, D), device="cuda")
    out = torch.empty((rows, H, D), device="cuda")
    nbl_ctx.rope_kv_append(kv, q_in.cuda(), k_in.cuda(), v_in.cuda(), q, dev(np.arange(rows, dtype=np.int32)),
                           dev(np.array(lens, np.int32) - 1), t_table, H, spec, bq=bq, bk=bk, bv=bv)
    nbl_ctx.attn_decode(kv, q, t_table, t_lens, max(lens), out)
    nbl_ctx.check()
    ref_sep = host(out)
    np.testing.assert_allclose(got, ref_sep, rtol=1e-5, atol=1e-6)
    pool = pool_bits(kv)
    qr = host(q)
    for r in (0, rows - 2, rows - 1):
        k, v = oracle.gather_pages(pool, table[r], lens[r], KV, D, 16)
        ref = oracle.attention(qr[r][None], k, v, 1, lens[r] - 1, H, KV, D)[0]
        assert max_rel_err_per_head(got[r], ref) <= 1e-4


def test_decode_empty_row_and_long_context(nbl_ctx):
    """A zero-length row yields out = 0, lse = -inf; a 131073-token row (config 4's length) takes the split-K
    path with the automatic split count and still matches."""
    import torch
    H, KV = 32, 8
    lens = [0, 131073, 5]
    table, n_pages = make_page_tables(lens, 16, shuffle_seed=9)
    kv = nbl_ctx.kv_pool(n_pages, KV)
    fill_random(kv, seed=11)
    rng = np.random.default_rng(4)
    q = rng.standard_normal((3, H, D)).astype(np.float32)
    out = torch.full((3, H, D), float("nan"), device="cuda")
    lse = torch.zeros((3, H), device="cuda")
    nbl_ctx.attn_decode(kv, dev(q), dev(table), dev(np.array(lens, np.int32)), max(lens), out, lse)
    nbl_ctx.check()
    got, got_lse = host(out), host(lse)
    assert np.all(got[0] == 0.0) and np.all(np.isneginf(got_lse[0]))
    pool = pool_bits(kv)
    for r in (1, 2):
        k, v = oracle.gather_pages(pool, table[r], lens[r], KV, D, 16)
        ref = oracle.attention(q[r][None], k, v, 1, lens[r] - 1, H, KV, D)[0]
        assert max_rel_err_per_head(got[r], ref) <= 1e-4


def test_decode_bad_page_id_sets_device_flag(nbl_ctx):
    """An out-of-range page id is skipped and reported by nbl_ctx_check as NBL_E_DEVICE; the context stays
    usable and the next call is correct."""
    import torch
    import nibble_b200 as nb
    H, KV = 8, 2
    lens = [40]
    table, n_pages = make_page_tables(lens, 16)
    kv = nbl_ctx.kv_pool(n_pages, KV)
    fill_random(kv, seed=2)
    bad = table.copy()
    bad[0, 1] = n_pages + 1000
    q = dev(np.ones((1, H, D), np.float32))
    out = torch.zeros((1, H, D), device="cuda")
    nbl_ctx.attn_decode(kv, q, dev(bad), dev(np.array(lens, np.int32)), 40, out)
    with pytest.raises(nb.NibbleError) as e:
        nbl_ctx.check()
    assert e.value.status == nb._abi.NBL_E_DEVICE and "page id" in str(e.value)
    nbl_ctx.attn_decode(kv, q, dev(table), dev(np.array(lens, np.int32)), 40, out)
    nbl_ctx.check()
    pool = pool_bits(kv)
    k, v = oracle.gather_pages(pool, table[0], 40, KV, D, 16)
    ref = oracle.attention(np.ones((1, H, D), np.float32), k, v, 1, 39, H, KV, D)[0]
    assert max_rel_err_per_head(host(out)[0], ref) <= 1e-4


def test_decode_rejects_bad_arguments(nbl_ctx):
    import torch
    import nibble_b200 as nb
    kv = nbl_ctx.kv_pool(4, 2)
    q = torch.zeros((1, 6, D), device="cuda")
    t = dev(np.zeros((1, 4), np.int32))
    ln = dev(np.ones(1, np.int32))
    with pytest.raises(nb.NibbleError):   # 6 heads over 2 KV heads is fine, 5 is not a multiple
        nbl_ctx.attn_decode(kv, torch.zeros((1, 5, D), device="cuda"), t, ln, 1, q)
    with pytest.raises(nb.NibbleError):   # max_seq_len beyond the page table
        nbl_ctx.attn_decode(kv, q, t, ln, 65, q)
    bf = nbl_ctx.kv_pool(4, 2, dtype=nb.BF16)
    with pytest.raises(nb.NibbleError):   # decode reads fp16 pools
        nbl_ctx.attn_decode(bf, q, t, ln, 1, q)


def test_lse_merge_matches_oracle(nbl_ctx):
    import torch
    rng = np.random.default_rng(8)
    P, rows = 5, 77
    po = rng.standard_normal((P, rows, D)).astype(np.float32)
    pl = (rng.standard_normal((P, rows)) * 3).astype(np.float32)
    pl[2, :10] = -np.inf
    pl[:, 20] = -np.inf  # a row with no keys anywhere
    out = torch.zeros((rows, D), device="cuda")
    lse = torch.zeros(rows, device="cuda")
    nbl_ctx.lse_merge(dev(po), dev(pl), out, lse)
    ref_o, ref_l = oracle.lse_merge(po, pl)
    np.testing.assert_allclose(host(out), ref_o, rtol=0, atol=2e-6)
    got_l = host(lse)
    assert np.isneginf(got_l[20]) and np.all(host(out)[20] == 0)
    fin = np.isfinite(ref_l)
    np.testing.assert_allclose(got_l[fin], ref_l[fin], rtol=0, atol=2e-6)


def test_lse_merge_packed_matches_lse_merge(nbl_ctx):
    """The packed layout of one all-gather ([parts][rows*D outputs | rows lse]) merged in place equals
    nbl_lse_merge on the same partials, including parts with lse = -inf (empty chunks)."""
    import torch
    from nibble_b200 import dist as ndist
    rng = np.random.default_rng(8)
    parts, rows = 5, 37
    o = torch.from_numpy(rng.standard_normal((parts, rows, D)).astype(np.float32)).cuda()
    lse_np = rng.standard_normal((parts, rows)).astype(np.float32) * 4
    lse_np[1, :] = -np.inf
    lse_np[3, 5] = -np.inf
    lse = torch.from_numpy(lse_np).cuda()
    packed = torch.cat([o.reshape(parts, -1), lse], dim=1).contiguous()
    a = torch.empty((rows, D), device="cuda")
    b = torch.empty((rows, D), device="cuda")
    la, lb = torch.empty(rows, device="cuda"), torch.empty(rows, device="cuda")
    nbl_ctx.lse_merge(o, lse, a, la)
    nbl_ctx.lse_merge_packed(packed, parts, rows, D, b, lb)
    nbl_ctx.check()
    assert torch.equal(a, b) and torch.equal(la, lb)
    send, ov, lv = ndist.partials_buffer(3, 2, D)
    assert ov.shape == (3, 2, D) and lv.shape == (3, 2) and send.numel() == 3 * 2 * (D + 1)


# ---------------------------------------------------------------- prefill (tcgen05)
PREFILL_ITEMS = [(1, 0), (37, 0), (128, 0), (129, 0), (300, 0), (64, 200), (200, 57)]  # (q_len, pos0)


def _prefill_case(nbl_ctx, H, KV, pool_dtype, items, base, neox, seed):
    """Appends every item's tokens 0..pos0+q_len-1 with rope_kv_append (bf16/fp16 inputs), then runs the
    prefill over each item's last q_len rows. Returns GPU out, the reference-path oracle result, and the
    oracle on the exact operands the tensor cores saw."""
    import torch
    import nibble_b200 as nb
    tdt = torch.bfloat16 if pool_dtype == nb.BF16 else torch.float16
    narrow_bits = oracle.f32_to_bf16_bits if pool_dtype == nb.BF16 else oracle.f32_to_fp16_bits
    widen_bits = oracle.bf16_bits_to_f32 if pool_dtype == nb.BF16 else oracle.fp16_bits_to_f32
    kv_lens = [q + p for q, p in items]
    table, n_pages = make_page_tables(kv_lens, 16, shuffle_seed=seed)
    kv = nbl_ctx.kv_pool(n_pages + 1, KV, dtype=pool_dtype)
    rng = np.random.default_rng(seed)
    tot = sum(kv_lens)
    q_in = widen_bits(narrow_bits(rng.standard_normal((tot, H, D)).astype(np.float32)))
    k_in = widen_bits(narrow_bits(rng.standard_normal((tot, KV, D)).astype(np.float32)))
    v_in = widen_bits(narrow_bits(rng.standard_normal((tot, KV, D)).astype(np.float32)))
    rows = np.concatenate([np.full(L, r) for r, L in enumerate(kv_lens)]).astype(np.int32)
    pos = np.concatenate([np.arange(L) for L in kv_lens]).astype(np.int32)
    q_out = torch.empty((tot, H, D), device="cuda", dtype=tdt)
    spec = nb.RopeSpec(base, neox)
    nbl_ctx.rope_kv_append(kv, dev(q_in, tdt), dev(k_in, tdt), dev(v_in, tdt), q_out, dev(rows), dev(pos),
                           dev(table), H, spec)
    starts = np.cumsum([0] + kv_lens[:-1]).astype(np.int32)
    q_start = (starts + np.array([p for _, p in items])).astype(np.int32)
    q_len = np.array([q for q, _ in items], np.int32)
    pos0 = np.array([p for _, p in items], np.int32)
    out = torch.full((tot, H, D), float("nan"), device="cuda")
    nbl_ctx.attn_prefill(kv, q_out, dev(q_start), dev(q_len), dev(pos0), dev(table), int(q_len.max()), out)
    nbl_ctx.check()
    got = host(out)
    qk_bits = host(q_out.view(torch.int16)).view(np.uint16)
    pool = pool_bits(kv)
    results = []
    for i, (ql, p0) in enumerate(items):
        if ql == 0:
            continue
        L = ql + p0
        s = starts[i]
        # reference path: bf16 inputs widened, RoPE in fp32, attention in fp32 (nibble's order)
        q_r = oracle.rope(q_in[s + p0:s + L], H, D, p0, base, neox).reshape(ql, H, D)
        k_r = oracle.rope(k_in[s:s + L], KV, D, 0, base, neox).reshape(L, KV, D)
        ref = oracle.attention(q_r, k_r, v_in[s:s + L], ql, p0, H, KV, D)
        # the operands the tensor cores saw (roped, narrowed)
        k_g, v_g = oracle.gather_pages(pool, table[i], L, KV, D, 16, bf16=pool_dtype == nb.BF16)
        q_g = widen_bits(qk_bits[s + p0:s + L])
        ref_g = oracle.attention(q_g, k_g, v_g, ql, p0, H, KV, D)
        results.append((got[s + p0:s + L], ref, ref_g))
    return results


@pytest.mark.parametrize("H,KV,dt", [(32, 4, "bf16"), (14, 2, "bf16"), (32, 8, "f16"), (8, 8, "bf16")])
def test_prefill_matches_oracle(nbl_ctx, H, KV, dt):
    import nibble_b200 as nb
    pool_dtype = nb.BF16 if dt == "bf16" else nb.F16
    for got, ref, ref_g in _prefill_case(nbl_ctx, H, KV, pool_dtype, PREFILL_ITEMS, 1e4, False, seed=H + KV):
        assert np.isfinite(got).all()
        assert np.abs(got - ref).max() <= 2e-2
        assert min_cosine_per_head(got, ref) >= 0.9999
        assert np.abs(got - ref_g).max() <= 1e-2  # only P's rounding to 16 bits separates these


def test_prefill_many_works_per_cta(nbl_ctx):
    """More works than the persistent grid holds (each CTA walks several, through both Q buffers and across the
    K/V ring), with an odd group (Qwen's 14 / 2: the last head pair of a KV group has one head), empty items and
    items that continue a cached prefix."""
    import nibble_b200 as nb
    rng = np.random.default_rng(5)
    items = [(0, 0), (0, 40)] + [(int(q), int(p)) for q, p in zip(rng.integers(1, 300, 38), rng.integers(0, 200, 38))]
    cases = _prefill_case(nbl_ctx, 14, 2, nb.BF16, items, 1e6, True, seed=31)
    assert len(cases) == 38
    for got, ref, ref_g in cases:
        assert np.isfinite(got).all()
        assert np.abs(got - ref).max() <= 2e-2
        assert min_cosine_per_head(got, ref) >= 0.9999
        assert np.abs(got - ref_g).max() <= 1e-2


def test_prefill_tinyllama_full_tile_rows(nbl_ctx):
    """Config 3's head layout (32 Q / 4 KV heads, theta 1e4) on a 2048-token item: 16 query tiles, causal."""
    import nibble_b200 as nb
    for got, ref, ref_g in _prefill_case(nbl_ctx, 32, 4, nb.BF16, [(2048, 0)], 1e4, False, seed=77):
        assert np.abs(got - ref).max() <= 2e-2
        assert min_cosine_per_head(got, ref) >= 0.9999
