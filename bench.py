#!/usr/bin/env python
"""Benchmark of the B200 attention path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

Workloads (the benchmark configurations 1-5, synthetic seeded inputs of their shapes; no dataset is involved):
  decode_batched  config 2 (the headline): Llama-3.2-1B attention (32 Q / 8 KV heads, head_dim 64, interleaved
                  RoPE theta 5e5); per GPU 64 sequences x 16 layers = 1024 independent rows, each a 4096-token
                  fp16 paged cache plus one new token. A step = fused bias/RoPE/append of the 1024 new tokens +
                  split-K flash-decode of all rows. Metric: decode attention HBM GB/s = algorithmic bytes / time,
                  algorithmic bytes = fp16 K/V read (rows x 4097 x 8 x 64 x 2 x 2) + q, out, new-token traffic.
  prefill         config 3: TinyLlama-1.1B attention (32 Q / 4 KV heads, theta 1e4), 8 sequences x 2048 bf16
                  tokens x 22 layers = 176 items; a step = fused RoPE/append of all tokens + tcgen05 causal prefill.
                  Metric: TFLOP/s with causal FLOPs 4 * H * D * sum(keys attended).
  decode_long / decode_ragged   configs 4 and 5 (extra legs of the default run).
  model_gemv      the weight matmuls of one decode token of a TinyLlama-1.1B-shaped F16 model (the rest of the
                  Backend on the GPU; bounds a whole-model decode step). Metric: weight bytes / time (HBM GB/s).
  model_gemv_q4_0 the same with Q4_0 weights (nibble's quantized matmul, bit-identical to its CPU kernels).
  model_qgemm     the weight matmuls of a 512-token prefill of the Q4_0 model on the tcgen05 kind::i8 path.
                  Metric: tokens/s of the matmul part.
  model_fgemm     the same for the F16 model on the tcgen05 kind::f16 path (activations split into two fp16 terms).
With N > 1 (torchrun, one rank per GPU, NCCL) the benchmark configurations' fixed total work is split over the ranks
("strong" scaling): config 2's 64 sequences and config 3's 176 (sequence, layer) items evenly by sequence with no
collective, config 5's sequences by LPT on KV length, config 4's one KV sequence in contiguous chunks whose (O, lse)
partials one NCCL all-gather moves before the LSE merge (--exchange peer: every rank stores its partials straight
into the other ranks' memory over NVLink instead, nbl_lse_exchange_peers; --exchange fused: the decode kernel stores
them there itself, nbl_attn_decode_peers). --scaling weak gives every rank the whole configuration
instead (a labelled extra). value = all ranks' work / max-over-ranks device time. Every run checks sampled rows of
its own results (config 2), and the merged long-context result (config 4) on rank 0, against a float64 attention
computed on the GPU from the same fp16 cache; a mismatch fails the run.

--impl reference times nibble's own CPU attention (CpuBackend::attention with its AVX2/AVX-VNNI tier on a
ThreadPool of all host threads, compiled from the reference sources into oracle/_ref) on a bounded sample of the
same workload, in the same metric.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

H2, KV2, D, CTX2, SEQ2, LAYERS2 = 32, 8, 64, 4096, 64, 16         # config 2
H3, KV3, T3, SEQ3, LAYERS3 = 32, 4, 2048, 8, 22                     # config 3


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), float(p.get("bf16_tflops_sustained", p["bf16_tflops"])), "measured"
    except Exception:
        return 6650.0, 1590.0, 1400.0, "fallback"


# Per-launch DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) of the dominant kernels at this bench's full
# sizes, from one ncu capture each on a smaller case of the same kernel, scaled by the units processed (traffic grows
# in proportion):
#   decode_kernel, config 2: `ncu --set full --clock-control none -k regex:decode_kernel -s 3 -c 1 python bench.py
#     --seqs 8 --steps 1 --warmup 3 --no-prefill --no-extra --no-e2e --cpu-seconds 0` -> 1.0834 GB for 128 rows
#     (1.079154 GB read + 4.28 MB written), x 8 for the 1024-row launch;
#   prefill_kernel, config 3: `ncu --set full --clock-control none -k regex:prefill_kernel -s 3 -c 1 python bench.py
#     --workload prefill --prefill-seqs 1 --steps 1 --warmup 3` -> 371.3 MB for 22 items, x 8 for 176 items.
TRAFFIC_DECODE_CFG2 = 8667488000
TRAFFIC_PREFILL_CFG3 = 2970780000


class ClockSampler:
    """nvidia-smi clock/throttle sampling (200 ms) in the background; keeps timestamped samples."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.samples = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(self.device)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except OSError:
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                self.samples.append((time.time(), parts))

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self, t0, t1):
        win = [s for t, s in self.samples if t0 - 0.25 <= t <= t1 + 0.25] or [s for _, s in self.samples[-3:]]
        if not win:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no nvidia-smi samples"], "samples": 0}
        sm = [float(s[1]) for s in win if s[1].replace(".", "", 1).isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in win for i in range(4) if s[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": float(win[0][2]) if win else None,
                "reasons": reasons, "samples": len(win)}


# ---------------------------------------------------------------- distributed plumbing
def dist_setup(gpus):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != gpus:
        raise SystemExit(f"--gpus {gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x, world):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def fill_normal_(t, seed):
    """Fills a 16-bit tensor with N(0,1) values rounded to its dtype, in chunks (bounded temporaries)."""
    import torch
    g = torch.Generator(device=t.device).manual_seed(seed)
    flat = t.view(-1)
    step = 1 << 27
    for i in range(0, flat.numel(), step):
        n = min(step, flat.numel() - i)
        flat[i:i + n].copy_(torch.randn(n, generator=g, device=t.device, dtype=torch.float32).to(flat.dtype))


def gather_row_kv(kv, table_row, length, n_kv):
    """K, V [length, n_kv, 64] of one row of a paged fp16 pool, as device tensors (pages gathered in order)."""
    import torch
    pool = kv.tensor().view(torch.float16).view(-1, 2, n_kv, 16, D)
    npg = (length + 15) // 16
    idx = torch.as_tensor(np.asarray(table_row[:npg], np.int64), device=pool.device)
    pages = pool.index_select(0, idx)  # [npg, 2, KV, 16, D]
    k = pages[:, 0].permute(0, 2, 1, 3).reshape(npg * 16, n_kv, D)[:length]
    v = pages[:, 1].permute(0, 2, 1, 3).reshape(npg * 16, n_kv, D)[:length]
    return k, v


def attention_f64(q, k, v):
    """Single-query causal attention in float64 on the GPU: q [H, D], k/v [L, KVH, D] -> [H, D] (the parity check
    of the bench runs; the tests hold the kernels against the C oracle)."""
    import torch
    H, kvh = q.shape[0], k.shape[1]
    g = H // kvh
    kk = k.double().repeat_interleave(g, dim=1)  # [L, H, D]
    vv = v.double().repeat_interleave(g, dim=1)
    s = torch.einsum("hd,lhd->hl", q.double(), kk) / math.sqrt(q.shape[1])
    p = torch.softmax(s, dim=1)
    return torch.einsum("hl,lhd->hd", p, vv)


def rel_err_per_head(got, ref):
    """max over heads of max|got - ref| / max|ref| (the decode tolerance metric), got/ref [H, D]."""
    import torch
    g, r = got.double(), ref.double()
    return float(((g - r).abs().amax(1) / r.abs().amax(1).clamp_min(1e-30)).max())


def fail_together(bad, world, what):
    """Every rank learns whether any rank's parity check failed, and all exit non-zero together."""
    if world > 1:
        import torch
        import torch.distributed as dist
        t = torch.tensor([1.0 if bad else 0.0], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        bad = t.item() > 0
    if bad:
        raise SystemExit(f"parity check failed: {what}")


# ---------------------------------------------------------------- config 2: batched decode
def decode_batched(args, world, rank, local):
    import torch
    import nibble_b200 as nb
    from nibble_b200.workloads import make_page_tables
    total_seqs = args.seqs or SEQ2
    if args.scaling == "weak":
        seqs = total_seqs
    else:
        if total_seqs % world:
            raise SystemExit(f"config 2: {total_seqs} sequences do not split evenly over {world} GPUs")
        seqs = total_seqs // world
    rows = seqs * LAYERS2
    length = CTX2 + 1
    ctx = nb.Context(local)
    table, n_pages = make_page_tables([length] * rows, 16, shuffle_seed=100 + rank)
    kv = ctx.kv_pool(n_pages, KV2)
    fill_normal_(kv.tensor().view(torch.float16), seed=1000 + rank)
    rng = np.random.default_rng(rank)
    q_in_h = torch.from_numpy(rng.standard_normal((rows, H2, D)).astype(np.float32)).pin_memory()
    k_in_h = torch.from_numpy(rng.standard_normal((rows, KV2, D)).astype(np.float32)).pin_memory()
    v_in_h = torch.from_numpy(rng.standard_normal((rows, KV2, D)).astype(np.float32)).pin_memory()
    out_h = torch.empty((rows, H2, D), dtype=torch.float32).pin_memory()
    q_in, k_in, v_in = (t.cuda() for t in (q_in_h, k_in_h, v_in_h))
    q = torch.empty((rows, H2, D), device="cuda")
    out = torch.empty((rows, H2, D), device="cuda")
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    t_table = d(table)
    lens = d(np.full(rows, length, np.int32))
    tok_row = d(np.arange(rows, dtype=np.int32))
    tok_pos = d(np.full(rows, CTX2, np.int32))
    spec = nb.RopeSpec(5e5, False)
    st = torch.cuda.current_stream()

    def step(ev=None):
        ctx.rope_kv_append(kv, q_in, k_in, v_in, q, tok_row, tok_pos, t_table, H2, spec)
        if ev:
            ev[0].record(st)
        ctx.attn_decode(kv, q, t_table, lens, length, out)
        if ev:
            ev[1].record(st)

    kv_bytes = rows * length * KV2 * D * 2 * 2
    qo_bytes = 2 * rows * H2 * D * 4
    append_bytes = rows * (H2 + 2 * KV2) * D * 4 + rows * H2 * D * 4 + rows * 2 * KV2 * D * 2
    step_bytes = kv_bytes + qo_bytes + append_bytes
    for _ in range(args.warmup):
        step()
    ctx.check()
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    barrier(world)
    torch.cuda.synchronize()
    t_wall0 = time.time()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for i in range(args.steps):
        step(kev[i])
    e1.record(st)
    torch.cuda.synchronize()
    barrier(world)
    t_wall1 = time.time()
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, world)
    kern_ms = statistics.mean(a.elapsed_time(b) for a, b in kev)
    ctx.check()
    # parity of sampled rows of this rank's results: the last step's roped queries and outputs against a float64
    # attention over the same fp16 pages (4097 keys, the appended token included)
    worst = 0.0
    for r in sorted({0, rows // 3, rows // 2, rows - 1}):
        k, v = gather_row_kv(kv, table[r], length, KV2)
        worst = max(worst, rel_err_per_head(out[r], attention_f64(q[r], k, v)))
    fail_together(worst > 1e-4, world, f"config 2 rows: relative error {worst:.3e} > 1e-4")
    worst = max_over_ranks(worst, world)
    e2e_ms = None
    if not args.no_e2e:
        # e2e through the C ABI: pinned host inputs -> nbl_write, kernels, nbl_read of the outputs, every step
        for _ in range(max(1, args.warmup // 2)):
            e2e_step(ctx, kv, q_in_h, k_in_h, v_in_h, out_h, t_table, lens, length, spec)
        barrier(world)
        torch.cuda.synchronize()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(st)
        for _ in range(args.steps):
            e2e_step(ctx, kv, q_in_h, k_in_h, v_in_h, out_h, t_table, lens, length, spec)
        f1.record(st)
        torch.cuda.synchronize()
        e2e_ms = max_over_ranks(f0.elapsed_time(f1) / args.steps, world)
    sampler.stop()
    hbm, _, _, src = peaks()
    decode_bytes = kv_bytes + qo_bytes
    achieved = decode_bytes / (kern_ms * 1e-3) / 1e9
    traffic = TRAFFIC_DECODE_CFG2 * rows / (SEQ2 * LAYERS2)
    res = {
        "metric": "decode attn HBM GB/s", "value": world * step_bytes / (ms * 1e-3) / 1e9, "unit": "GB/s",
        "ms_per_step": ms, "dtype": "fp16 KV, fp32 accumulate", "scaling": args.scaling,
        "parity": {"check": "4 sampled rows per GPU vs float64 attention on the same fp16 pages",
                   "max_rel_err_per_head": worst, "tolerance": 1e-4},
        "config": {"workload": "config 2: Llama-3.2-1B batched decode", "heads": f"{H2}q/{KV2}kv", "head_dim": D,
                   "sequences_total": seqs * world, "sequences_per_gpu": seqs, "layers": LAYERS2, "kv_tokens": length,
                   "page_size": 16,
                   "kv_bytes_per_step_per_gpu": kv_bytes, "algorithmic_bytes_per_step_per_gpu": step_bytes,
                   "l2": f"inputs ({kv_bytes / 1e9:.2f} GB/GPU) larger than L2; no flush needed",
                   "parallelism": f"sequence-sharded x{world}"},
        "e2e": None if e2e_ms is None else {
            "value": world * step_bytes / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": e2e_ms,
            "h2d_bytes_per_step": int(q_in_h.numel() * 4 + k_in_h.numel() * 4 + v_in_h.numel() * 4),
            "d2h_bytes_per_step": int(out_h.numel() * 4),
            "path": "nbl_decode_step_host: pinned host q/k/v -> append + decode -> pinned host out, copies overlapped "
                    "with compute over row chunks"},
        "roofline": {"kernel": "decode_kernel", "bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                     "frac": achieved / hbm, "peak_source": f"{src} (MEASURED_PEAKS.json hbm_gbs)" if src == "measured" else "fallback 6650 GB/s",
                     "frac_of_nominal_8000": achieved / 8000.0, "kernel_ms": kern_ms,
                     "algorithmic_bytes_per_launch": decode_bytes, "traffic": traffic},
        "gpu_launches_per_step": 2,
        "clocks": sampler.summary(t_wall0, t_wall1),
    }
    kv.close()
    ctx.close()
    return res


def e2e_step(ctx, kv, q_in_h, k_in_h, v_in_h, out_h, t_table, lens, length, spec):
    """One config-2 step through the public host-buffer entry point: pinned host q/k/v in, pinned host out; the
    library overlaps the uploads and downloads with the append + decode of other row chunks."""
    ctx.decode_step_host(kv, q_in_h, k_in_h, v_in_h, t_table, lens, length, spec, out_h)


# ---------------------------------------------------------------- config 3: prefill
def prefill(args, world, rank, local, steps=None, warmup=None):
    import torch
    import nibble_b200 as nb
    from nibble_b200.workloads import make_page_tables
    steps = steps or args.steps
    warmup = warmup or args.warmup
    seqs = args.prefill_seqs or SEQ3
    total_items = seqs * LAYERS3  # (sequence, layer) units
    if args.scaling == "weak":
        items = total_items
    else:
        if total_items % world:
            raise SystemExit(f"config 3: {total_items} items do not split evenly over {world} GPUs")
        items = total_items // world
    ctx = nb.Context(local)
    table, n_pages = make_page_tables([T3] * items, 16, shuffle_seed=200 + rank)
    kv = ctx.kv_pool(n_pages, KV3, dtype=nb.BF16)
    n_tok = items * T3
    q_in = torch.empty((n_tok, H3, D), device="cuda", dtype=torch.bfloat16)
    k_in = torch.empty((n_tok, KV3, D), device="cuda", dtype=torch.bfloat16)
    v_in = torch.empty((n_tok, KV3, D), device="cuda", dtype=torch.bfloat16)
    for i, t in enumerate((q_in, k_in, v_in)):
        fill_normal_(t, seed=3000 + 10 * rank + i)
    q = torch.empty_like(q_in)
    out = torch.empty((n_tok, H3, D), device="cuda", dtype=torch.bfloat16)
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    t_table = d(table)
    tok_row = d(np.repeat(np.arange(items, dtype=np.int32), T3))
    tok_pos = d(np.tile(np.arange(T3, dtype=np.int32), items))
    q_start = d(np.arange(items, dtype=np.int32) * T3)
    q_len = d(np.full(items, T3, np.int32))
    pos0 = d(np.zeros(items, np.int32))
    spec = nb.RopeSpec(1e4, False)
    st = torch.cuda.current_stream()

    def step(ev=None):
        ctx.rope_kv_append(kv, q_in, k_in, v_in, q, tok_row, tok_pos, t_table, H3, spec)
        if ev:
            ev[0].record(st)
        ctx.attn_prefill(kv, q, q_start, q_len, pos0, t_table, T3, out)
        if ev:
            ev[1].record(st)

    for _ in range(warmup):
        step()
    ctx.check()
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for i in range(steps):
        step(kev[i])
    e1.record(st)
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1) / steps, world)
    kern_ms = statistics.mean(a.elapsed_time(b) for a, b in kev)
    ctx.check()
    flops = 4.0 * H3 * D * items * (T3 * (T3 + 1) / 2)
    _, bf16, bf16_sus, src = peaks()
    ach = flops / (kern_ms * 1e-3) / 1e12
    res = {
        "metric": "prefill attn TFLOP/s", "value": world * flops / (ms * 1e-3) / 1e12, "unit": "TFLOP/s",
        "ms_per_step": ms, "kernel_ms": kern_ms, "dtype": "bf16 operands, fp32 accumulate", "scaling": args.scaling,
        "config": {"workload": "config 3: TinyLlama-1.1B causal prefill", "heads": f"{H3}q/{KV3}kv", "head_dim": D,
                   "items_total": items * world, "items_per_gpu": items, "tokens": T3, "layers": LAYERS3,
                   "flops_per_step_per_gpu": flops},
        "roofline": {"kernel": "prefill_kernel", "bound": "tensor", "achieved": ach, "peak": bf16, "unit": "TFLOP/s",
                     "frac": ach / bf16, "peak_source": f"{src} bf16_tflops (burst)", "frac_of_sustained": ach / bf16_sus,
                     "frac_of_nominal_2250": ach / 2250.0, "traffic": TRAFFIC_PREFILL_CFG3 * items / (SEQ3 * LAYERS3)},
    }
    kv.close()
    ctx.close()
    return res


# ---------------------------------------------------------------- config 4: one long context, KV split over ranks
H4, KV4, LEN4, LAYERS4 = 32, 8, 131072, 16


def decode_long(args, world, rank, local, steps, warmup):
    """Config 4: one sequence with a 131072-token fp16 cache + 1 new token, 16 layers (16 independent rows). The
    KV sequence is split into contiguous page-aligned chunks over the ranks; each rank attends its chunk with the
    split-K decode (lse out), then one NCCL all-gather of the packed (O, lse) partials of all 16 layers and the
    LSE merge give every rank the full result. Strong scaling: the total work is fixed."""
    import torch
    import nibble_b200 as nb
    from nibble_b200 import dist as ndist
    from nibble_b200.workloads import kv_split, make_page_tables
    length = LEN4 + 1
    a, b = kv_split(length, world)[rank]
    my_len = b - a
    rows = LAYERS4
    ctx = nb.Context(local)
    table, n_pages = make_page_tables([my_len] * rows, 16, shuffle_seed=400 + rank)
    kv = ctx.kv_pool(max(1, n_pages), KV4)
    fill_normal_(kv.tensor().view(torch.float16), seed=4000 + rank)
    rng = np.random.default_rng(7)  # the query is the same on every rank
    q = torch.from_numpy(rng.standard_normal((rows, H4, D)).astype(np.float32)).cuda()
    # the decode writes (O, lse) straight into the all-gather send buffer; the merge reads the gathered buffer
    send, out, lse = ndist.partials_buffer(rows, H4, D)
    recv = torch.empty((world, send.numel()), device="cuda")
    merged = torch.empty((rows * H4, D), device="cuda")
    d = lambda x: torch.from_numpy(np.ascontiguousarray(x)).cuda()  # noqa: E731
    t_table, lens = d(table), d(np.full(rows, my_len, np.int32))
    main = torch.cuda.current_stream()

    px = ndist.PeerExchange(ctx, rows * H4, D) if world > 1 and args.exchange in ("peer", "fused") else None
    fused = px is not None and args.exchange == "fused"

    def decode():
        ctx.attn_decode(kv, q, t_table, lens, max(1, my_len), out, lse)

    def exchange():
        if px is not None:  # partials stored straight into the peers' memory, merged once every flag is up
            px.exchange(send, merged)
        else:
            import torch.distributed as dist
            dist.all_gather_into_tensor(recv, send)
            ctx.lse_merge_packed(recv, world, rows * H4, D, merged)

    def step():
        if fused:  # the decode kernel stores its finished rows into every rank's buffer; then the merge
            px.decode_exchange(kv, q, t_table, lens, max(1, my_len), merged.view(rows, H4, D))
            return
        decode()
        if world > 1:
            exchange()

    for _ in range(warmup):
        step()
    ctx.check()
    # kernel time of the decode alone (the roofline), events around each launch
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for a0, b0 in kev:
        a0.record(main)
        decode()
        b0.record(main)
    torch.cuda.synchronize()
    kern_ms = statistics.mean(x.elapsed_time(y) for x, y in kev)
    # the step (decode + all-gather + merge) captured once as a CUDA graph and replayed: at a few tens of
    # microseconds of work per rank, launching it op by op from Python would be the bottleneck
    side = torch.cuda.Stream()
    side.wait_stream(main)
    with torch.cuda.stream(side):
        ctx.set_stream(side.cuda_stream)
        step()
        side.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        ctx.set_stream(torch.cuda.current_stream().cuda_stream)
        step()
    ctx.set_stream(main.cuda_stream)
    for _ in range(warmup):
        graph.replay()
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(main)
    for i in range(steps):
        graph.replay()
    e1.record(main)
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1) / steps, world)
    ctx.check()
    # the exchange on its own (peer stores + flags + merge, or the NCCL all-gather + merge), timed with events; fused
    # into the decode it has no launch of its own, so its part is the step minus the decode alone
    ex_ms = 0.0
    if world > 1 and not fused:
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        barrier(world)
        for x0, x1 in ev:
            x0.record(main)
            exchange()
            x1.record(main)
        torch.cuda.synchronize()
        ex_ms = max_over_ranks(statistics.mean(a.elapsed_time(b) for a, b in ev), world)
    kern_max_ms = max_over_ranks(kern_ms, world)
    if fused:
        ex_ms = max(0.0, ms - kern_max_ms)
    del graph  # released before the process group is destroyed
    # parity: layer 0's merged result on rank 0 against a float64 attention over the whole 131073-token cache, whose
    # chunks the ranks send to rank 0 (an all-gather of each rank's layer-0 K/V, outside the timed region)
    k0, v0 = gather_row_kv(kv, table[0], my_len, KV4)
    chunk = max(b_ - a_ for a_, b_ in kv_split(length, world))
    mine = torch.zeros((2, chunk, KV4, D), dtype=torch.float16, device="cuda")
    mine[0, :my_len], mine[1, :my_len] = k0, v0
    if world > 1:
        import torch.distributed as dist
        every = torch.empty((world,) + tuple(mine.shape), dtype=torch.float16, device="cuda")
        dist.all_gather_into_tensor(every, mine)
    else:
        every = mine[None]
    err = 0.0
    if rank == 0:
        spans = kv_split(length, world)
        kf = torch.cat([every[r, 0, :b_ - a_] for r, (a_, b_) in enumerate(spans)])
        vf = torch.cat([every[r, 1, :b_ - a_] for r, (a_, b_) in enumerate(spans)])
        got = (merged if world > 1 else out.view(rows * H4, D))[:H4]
        err = rel_err_per_head(got, attention_f64(q[0], kf, vf))
    fail_together(err > 1e-4, world, f"config 4 merged layer 0: relative error {err:.3e} > 1e-4")
    del every, mine
    if px is not None:
        px.close()
    total_kv = rows * length * KV4 * D * 2 * 2
    my_kv = rows * my_len * KV4 * D * 2 * 2
    hbm, _, _, src = peaks()
    ach = (my_kv + 2 * rows * H4 * D * 4) / (kern_ms * 1e-3) / 1e9
    parts = {"decode": kern_max_ms, "exchange": ex_ms}
    res = {"metric": "decode attn HBM GB/s", "value": total_kv / (ms * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": ms,
           "scaling": "strong",
           "step_ms_breakdown": {**parts, "graph_step": ms, "decode_share": kern_max_ms / ms,
                                 "exchange_kind": ("decode kernel storing into the peers' memory + flags + merge "
                                                   "(nbl_attn_decode_peers; exchange = step - decode)" if fused else
                                                   "peer stores over NVLink + flags + merge (nbl_lse_exchange_peers)"
                                                   if px is not None else "NCCL all-gather + nbl_lse_merge_packed"),
                                 "limiter": "decode (HBM)" if kern_max_ms >= 0.5 * ms else "exchange"},
           "parity": {"check": "layer 0 merged over all ranks' chunks vs float64 attention on rank 0",
                      "max_rel_err_per_head": err, "tolerance": 1e-4},
           "config": {"workload": "config 4: long-context decode, KV split over ranks", "kv_tokens": length,
                      "layers": LAYERS4, "heads": f"{H4}q/{KV4}kv", "kv_tokens_this_rank": my_len,
                      "exchange": ("packed (O, lse) of all layers stored into every peer's memory, flags, LSE merge"
                                   if px is not None else "one NCCL all-gather of packed (O, lse) for all layers + "
                                   "LSE merge") + ", the step replayed as one CUDA graph" if world > 1 else
                                  "none (one GPU; CUDA graph)"},
           "roofline": {"kernel": "decode_kernel (+ lse_merge)", "bound": "hbm", "achieved": ach, "peak": hbm,
                        "unit": "GB/s", "frac": ach / hbm, "peak_source": src, "kernel_ms": kern_ms}}
    kv.close()
    ctx.close()
    return res


# ---------------------------------------------------------------- the model's weight matmuls at decode
E6, FF6, Q6, KV6, LAYERS6, VOCAB6 = 2048, 5632, 2048, 256, 22, 32000   # TinyLlama-1.1B


Q4_0_CODE, Q4_0_BLOCK = 3, 18  # nbl_dtype NBL_Q4_0; GGUF bytes per 32-element block


def tinyllama_weights(ctx, rng, wtype, with_output=True):
    """Random (synthetic) TinyLlama-1.1B weight matrices in nibble's order per layer (Q, K, V, O, gate, up, down)
    plus the output projection: F16 values ~ N(0, 0.02), or Q4_0 blocks of random 4-bit values with fp16 scale
    0.01. Returns (weights, shapes, device bytes read by one pass over them)."""
    shapes = []
    for _ in range(LAYERS6):
        shapes += [(Q6, E6), (KV6, E6), (KV6, E6), (E6, Q6), (FF6, E6), (FF6, E6), (E6, FF6)]
    if with_output:
        shapes.append((VOCAB6, E6))
    if wtype == "F16":
        pool = (rng.standard_normal(VOCAB6 * E6, dtype=np.float32) * 0.02).astype(np.float16)
        weights = [ctx.weight(pool[: r * c].reshape(r, c)) for r, c in shapes]
        return weights, shapes, sum(r * c * 2 for r, c in shapes)
    nbk = VOCAB6 * E6 // 32
    pool = rng.integers(0, 256, size=(nbk, Q4_0_BLOCK), dtype=np.uint8)
    pool[:, :2] = np.frombuffer(np.float16(0.01).tobytes(), np.uint8)
    weights = [ctx.weight(pool[: r * c // 32].reshape(r, c // 32 * Q4_0_BLOCK), Q4_0_CODE, c) for r, c in shapes]
    return weights, shapes, sum(r * c // 32 * Q4_0_BLOCK for r, c in shapes)


def model_gemv(args, world, rank, local, steps, warmup, wtype="F16"):
    """The weight matmuls of one decode token of a TinyLlama-1.1B-shaped model through nbl_matmul (n = 1): per
    layer Q, K, V, O, gate, up and down projections, then the output projection -- Q/K/V and gate/up as one
    multi-weight call each (the Transformer's matmul_multi), 89 calls, replayed as one CUDA graph. F16 weights
    (2.07 GB) run the weight-streaming GEMV; Q4_0 weights (0.58 GB) run nibble's quantized matmul (activations
    quantized to Q8_0, block dots summed in the reference's order: one quantize and one GEMV launch per call).
    This is what bounds a decode step of the whole Transformer on CudaBackend. Metric: weight bytes / step time
    (HBM GB/s); tokens/s = 1 / step time. Weights are random (synthetic)."""
    import torch
    import nibble_b200 as nb
    ctx = nb.Context(local)
    rng = np.random.default_rng(60 + rank)
    weights, shapes, wbytes = tinyllama_weights(ctx, rng, wtype)
    x = {c: torch.randn(c, device="cuda") for c in (E6, FF6)}
    y = {w: torch.empty(w, device="cuda") for w in (Q6, KV6, E6, FF6, VOCAB6)}
    y["v"], y["u"] = torch.empty(KV6, device="cuda"), torch.empty(FF6, device="cuda")
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())

    def step():  # as the Transformer calls them: matmul_multi for Q/K/V and for gate/up, matmul for O and down
        for layer in range(LAYERS6):
            wq, wk, wv, wo, wg, wu, wd = weights[7 * layer:7 * layer + 7]
            ctx.matmul_multi([wq, wk, wv], x[E6], [y[Q6], y[KV6], y["v"]], 1)
            ctx.matmul(wo, x[E6], y[E6], 1)
            ctx.matmul_multi([wg, wu], x[E6], [y[FF6], y["u"]], 1)
            ctx.matmul(wd, x[FF6], y[E6], 1)
        ctx.matmul(weights[-1], x[E6], y[VOCAB6], 1)

    with torch.cuda.stream(side):
        ctx.set_stream(side.cuda_stream)
        step()
        side.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        ctx.set_stream(torch.cuda.current_stream().cuda_stream)
        step()
    main = torch.cuda.current_stream()
    ctx.set_stream(main.cuda_stream)
    for _ in range(warmup):
        graph.replay()
    ctx.check()
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(main)
    for _ in range(steps):
        graph.replay()
    e1.record(main)
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1) / steps, world)
    ctx.check()
    del graph
    for w in weights:
        w.close()
    ctx.close()
    hbm, _, _, src = peaks()
    ach = wbytes / (ms * 1e-3) / 1e9
    calls = 4 * LAYERS6 + 1
    return {"metric": "model decode weight-matmul HBM GB/s", "value": world * ach, "unit": "GB/s", "ms_per_step": ms,
            "tokens_per_s_per_gpu": 1e3 / ms, "scaling": "weak",
            "gpu_launches_per_step": calls if wtype == "F16" else 2 * calls,
            "config": {"workload": f"TinyLlama-1.1B decode-step weight matmuls ({wtype} weights, n = 1)",
                       "launches_per_step": calls if wtype == "F16" else 2 * calls, "weight_bytes": wbytes,
                       "l2": f"weights ({wbytes / 1e9:.2f} GB) larger than L2; no flush needed"},
            "roofline": {"kernel": "gemv_kernel" if wtype == "F16" else "quantize_rows_kernel + gemv_q_kernel",
                         "bound": "hbm", "achieved": ach, "peak": hbm, "unit": "GB/s", "frac": ach / hbm,
                         "peak_source": src}}


def model_qgemm(args, world, rank, local, steps, warmup, n=512, wtype="Q4_0"):
    """The weight matmuls of one 512-token prefill of a TinyLlama-1.1B-shaped model through nbl_matmul (the
    tensor-core paths for more than 8 activation rows): per layer Q/K/V and gate/up as matmul_multi, O and down as
    matmul -- 88 calls (the output projection runs on the last row only), replayed as one CUDA graph.
    Q4_0: each call quantizes its activation rows to Q8_0 and runs qgemm_kernel: one tcgen05 kind::i8 MMA per
    32-element block into TMEM, the reference's per-block float terms added in block order by the epilogue warps;
    the kernel's rate is given as int8 TOPS and as block terms per second against the epilogue's issue bound.
    F16: each call scales each activation row by a power of two, splits it into two fp16 terms and runs
    fgemm_kernel on the F16 weights as they are (tcgen05 kind::f16, two MMAs per K-step, fp32 accuracy); the rate is
    useful TFLOP/s against the peak for two MMAs per step (half the measured dense bf16 rate). Metric: activation
    rows (tokens) per second of the matmul part."""
    import torch
    import nibble_b200 as nb
    ctx = nb.Context(local)
    rng = np.random.default_rng(70 + rank)
    weights, shapes, wbytes = tinyllama_weights(ctx, rng, wtype, with_output=False)
    x = {c: torch.randn(n, c, device="cuda") for c in (E6, FF6)}
    y = {w: torch.empty(n, w, device="cuda") for w in (Q6, KV6, E6, FF6)}
    y["v"], y["u"] = torch.empty(n, KV6, device="cuda"), torch.empty(n, FF6, device="cuda")
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())

    def step():
        for layer in range(LAYERS6):
            wq, wk, wv, wo, wg, wu, wd = weights[7 * layer:7 * layer + 7]
            ctx.matmul_multi([wq, wk, wv], x[E6], [y[Q6], y[KV6], y["v"]], n)
            ctx.matmul(wo, x[E6], y[E6], n)
            ctx.matmul_multi([wg, wu], x[E6], [y[FF6], y["u"]], n)
            ctx.matmul(wd, x[FF6], y[E6], n)

    with torch.cuda.stream(side):  # the first pass makes the int8 operands and the activation scratch
        ctx.set_stream(side.cuda_stream)
        step()
        side.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        ctx.set_stream(torch.cuda.current_stream().cuda_stream)
        step()
    main = torch.cuda.current_stream()
    ctx.set_stream(main.cuda_stream)
    for _ in range(warmup):
        graph.replay()
    ctx.check()
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(main)
    for _ in range(steps):
        graph.replay()
    e1.record(main)
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1) / steps, world)
    ctx.check()
    del graph
    for w in weights:
        w.close()
    ctx.close()
    macs = n * sum(r * c for r, c in shapes)
    res = {"metric": "model prefill weight-matmul tokens/s", "value": world * n / (ms * 1e-3), "unit": "tokens/s",
           "ms_per_step": ms, "scaling": "weak", "gpu_launches_per_step": 8 * LAYERS6,
           "config": {"workload": f"TinyLlama-1.1B {n}-token prefill weight matmuls ({wtype} weights)",
                      "calls_per_step": 4 * LAYERS6, "launches_per_step": 8 * LAYERS6, "weight_bytes": wbytes,
                      "l2": "activations and each weight matrix are re-read from L2 by the tiles sharing them"}}
    if wtype == "F16":
        _, bf16, _, src = peaks()
        tflops = 2 * macs / (ms * 1e-3) / 1e12
        res["roofline"] = {"kernel": "fgemm_kernel<2, BN>", "bound": "tensor (kind::f16, 2 MMAs per K-step)",
                           "achieved": tflops, "peak": bf16 / 2, "unit": "TFLOP/s (useful)", "frac": tflops / (bf16 / 2),
                           "peak_source": f"{src} dense bf16 / 2: two fp16 MMAs per K-step"}
        return res
    terms = macs // 32
    clock = gpu_clock_mhz(local)
    issue_bound = 148 * 128 / 4 * clock * 1e6  # 4 FP32-pipe issue slots per output and block, 128 lanes per SM
    res["int8_tops"] = 2 * macs / (ms * 1e-3) / 1e12
    res["roofline"] = {"kernel": "qgemm_kernel", "bound": "issue (fp32 epilogue)", "achieved": terms / (ms * 1e-3),
                       "peak": issue_bound, "unit": "block terms/s", "frac": terms / (ms * 1e-3) / issue_bound,
                       "peak_source": f"148 SMs x 32 terms/clk at the SM clock sampled ({clock:.0f} MHz)"}
    return res


def gpu_clock_mhz(local):
    """Current SM clock of this GPU from nvidia-smi (MHz); 1965 if it cannot be read."""
    try:
        out = subprocess.run(["nvidia-smi", "-i", str(local), "--query-gpu=clocks.sm", "--format=csv,noheader,nounits"],
                             capture_output=True, text=True, timeout=10).stdout.strip()
        return float(out.splitlines()[0])
    except Exception:
        return 1965.0


# ---------------------------------------------------------------- config 5: ragged paged decode, LPT-balanced
H5, KV5, SEQ5, LAYERS5, MAXLEN5 = 14, 2, 256, 24, 8192


def decode_ragged(args, world, rank, local, steps, warmup):
    """Config 5: Qwen2.5-0.5B heads, 256 sequences with seeded lengths U[1, 8192], 24 layers, 16-token fp16 pages
    shuffled in one shared pool; one new token per sequence (appended, then attended). Sequences are bin-packed
    over ranks by KV length (LPT). Strong scaling: the total work is fixed."""
    import torch
    import nibble_b200 as nb
    from nibble_b200.workloads import lpt_partition, make_page_tables, ragged_lengths
    ctx_lens = ragged_lengths(SEQ5, 1, MAXLEN5, seed=5)
    mine = lpt_partition(ctx_lens + 1, world)[rank]
    my_ctx = np.repeat(ctx_lens[mine], LAYERS5)  # rows = (sequence, layer), sequence-major
    lens_after = (my_ctx + 1).astype(np.int32)
    rows = len(lens_after)
    ctx = nb.Context(local)
    table, n_pages = make_page_tables(lens_after, 16, shuffle_seed=500 + rank)
    kv = ctx.kv_pool(n_pages, KV5)
    fill_normal_(kv.tensor().view(torch.float16), seed=5000 + rank)
    rng = np.random.default_rng(rank)
    q_in = torch.from_numpy(rng.standard_normal((rows, H5, D)).astype(np.float32)).cuda()
    k_in = torch.from_numpy(rng.standard_normal((rows, KV5, D)).astype(np.float32)).cuda()
    v_in = torch.from_numpy(rng.standard_normal((rows, KV5, D)).astype(np.float32)).cuda()
    q = torch.empty_like(q_in)
    out = torch.empty_like(q_in)
    d = lambda x: torch.from_numpy(np.ascontiguousarray(x)).cuda()  # noqa: E731
    t_table, t_lens = d(table), d(lens_after)
    tok_row, tok_pos = d(np.arange(rows, dtype=np.int32)), d(my_ctx.astype(np.int32))
    spec = nb.RopeSpec(1e6, True)
    st = torch.cuda.current_stream()
    max_len = int(lens_after.max())

    def step(ev=None):
        ctx.rope_kv_append(kv, q_in, k_in, v_in, q, tok_row, tok_pos, t_table, H5, spec)
        if ev:
            ev[0].record(st)
        ctx.attn_decode(kv, q, t_table, t_lens, max_len, out)
        if ev:
            ev[1].record(st)

    for _ in range(warmup):
        step()
    ctx.check()
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for i in range(steps):
        step(kev[i])
    e1.record(st)
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1) / steps, world)
    kern_ms = statistics.mean(x.elapsed_time(y) for x, y in kev)
    ctx.check()
    total_kv = int((ctx_lens + 1).sum()) * LAYERS5 * KV5 * D * 2 * 2
    my_kv = int(lens_after.sum()) * KV5 * D * 2 * 2
    hbm, _, _, src = peaks()
    ach = (my_kv + 2 * rows * H5 * D * 4) / (kern_ms * 1e-3) / 1e9
    res = {"metric": "decode attn HBM GB/s", "value": total_kv / (ms * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": ms,
           "scaling": "strong",
           "config": {"workload": "config 5: ragged paged decode (Qwen2.5-0.5B heads)", "sequences": SEQ5,
                      "layers": LAYERS5, "ctx_lengths": "U[1, 8192] seed 5", "kv_bytes_total": total_kv,
                      "sequences_this_rank": len(mine), "balance": "LPT by KV length"},
           "roofline": {"kernel": "decode_kernel", "bound": "hbm", "achieved": ach, "peak": hbm, "unit": "GB/s",
                        "frac": ach / hbm, "peak_source": src, "kernel_ms": kern_ms}}
    kv.close()
    ctx.close()
    return res


# ---------------------------------------------------------------- CPU baseline: nibble's own CpuBackend
def cpu_baseline(seconds=10.0, n_bufs=48):
    """CpuBackend::attention (AVX2/AVX-VNNI tier, ThreadPool of all host threads) on config-2 rows: one call per
    (sequence, layer) with q [1, 32, 64] and the row's 4097-token cache widened to fp32 [4097, 8, 64]. Enough
    distinct caches to exceed the CPU caches; runs for about `seconds`."""
    import oracle
    threads = os.cpu_count() or 1
    be = oracle.RefBackend(threads)
    length = CTX2 + 1
    be.reserve(length, H2, 1, H2 * D)
    rng = np.random.default_rng(0)
    bufs = []
    for _ in range(n_bufs):
        k = rng.standard_normal((length, KV2, D)).astype(np.float16).astype(np.float32)
        v = rng.standard_normal((length, KV2, D)).astype(np.float16).astype(np.float32)
        bufs.append((k, v))
    q = rng.standard_normal((1, H2, D)).astype(np.float32)
    out = np.empty((1, H2, D), np.float32)
    for k, v in bufs[:4]:
        be.attention_into(q, k, v, out, 1, CTX2, H2, KV2, D)
    calls = 0
    t0 = time.perf_counter()
    while True:
        k, v = bufs[calls % n_bufs]
        be.attention_into(q, k, v, out, 1, CTX2, H2, KV2, D)
        calls += 1
        el = time.perf_counter() - t0
        if el >= seconds and calls >= 8:
            break
    row_bytes = length * KV2 * D * 2 * 2 + 2 * H2 * D * 4  # the GPU metric's algorithmic bytes for one row
    return {"value": calls * row_bytes / el / 1e9, "unit": "GB/s", "cores": be.threads, "kind": "reference",
            "sample": f"{calls} CpuBackend::attention calls (config-2 rows, ctx 4097, fp32 K/V widened from fp16) "
                      f"in {el:.1f} s on {be.threads} threads; kernels tier {oracle.ref_kernels_name()}",
            "ms_per_row": 1e3 * el / calls}


def reference_arm(args):
    """--impl reference: nibble's own CPU attention on config 2, each step a bounded sample of 32 rows."""
    import oracle
    threads = os.cpu_count() or 1
    be = oracle.RefBackend(threads)
    length = CTX2 + 1
    rows_per_step = 32
    rng = np.random.default_rng(0)
    bufs = [(rng.standard_normal((length, KV2, D)).astype(np.float16).astype(np.float32),
             rng.standard_normal((length, KV2, D)).astype(np.float16).astype(np.float32)) for _ in range(rows_per_step)]
    q = rng.standard_normal((1, H2, D)).astype(np.float32)
    out = np.empty((1, H2, D), np.float32)

    def step():
        for k, v in bufs:
            be.attention_into(q, k, v, out, 1, CTX2, H2, KV2, D)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    el = time.perf_counter() - t0
    row_bytes = length * KV2 * D * 2 * 2 + 2 * H2 * D * 4
    val = rows_per_step * args.steps * row_bytes / el / 1e9
    sample = (f"{rows_per_step} config-2 rows per step (1/32 of the per-GPU 1024-row step), CpuBackend::attention "
              f"on {be.threads} threads, tier {oracle.ref_kernels_name()}")
    return {"impl": "reference", "metric": "decode attn HBM GB/s", "value": val, "unit": "GB/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * el / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic (seeded N(0,1), fp16-rounded)",
            "config": {"workload": "config 2: Llama-3.2-1B batched decode", "rows_per_step": rows_per_step,
                       "kv_tokens": length},
            "cpu_baseline": {"value": val, "unit": "GB/s", "cores": be.threads, "kind": "reference", "sample": sample},
            "e2e": {"value": val, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["decode_batched", "prefill", "decode_long", "decode_ragged", "model_gemv",
                                           "model_gemv_q4_0", "model_qgemm", "model_fgemm"],
                    default="decode_batched")
    ap.add_argument("--no-prefill", action="store_true", help="skip the config-3 prefill leg of the default run")
    ap.add_argument("--no-extra", action="store_true", help="skip the config-4/5 legs of the default run")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end (host buffers) leg")
    ap.add_argument("--seqs", type=int, default=0, help="config-2 sequences per GPU (default 64; smaller for profiling)")
    ap.add_argument("--prefill-seqs", type=int, default=0, help="config-3 sequences per GPU (default 8)")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU-baseline sample length (0 skips it)")
    ap.add_argument("--exchange", choices=["peer", "nccl", "fused"], default="nccl",
                    help="config 4 at N > 1: an NCCL all-gather (default; measured faster at 8 GPUs), the partials "
                         "stored straight into the peers' memory by a push kernel, or by the decode kernel itself")
    ap.add_argument("--scaling", choices=["strong", "weak"], default="strong",
                    help="strong: the configuration's total work split over the GPUs (default); weak: every GPU runs "
                         "all of it")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    if args.impl == "reference":
        if int(os.environ.get("RANK", "0")) != 0:
            return
        print(json.dumps(reference_arm(args)), flush=True)
        return

    world, rank, local = dist_setup(args.gpus)
    legs = max(3, args.steps // 5)
    if args.workload == "prefill":
        res = prefill(args, world, rank, local)
    elif args.workload == "decode_long":
        res = decode_long(args, world, rank, local, args.steps, args.warmup)
    elif args.workload == "decode_ragged":
        res = decode_ragged(args, world, rank, local, args.steps, args.warmup)
    elif args.workload == "model_gemv":
        res = model_gemv(args, world, rank, local, args.steps, args.warmup)
    elif args.workload == "model_gemv_q4_0":
        res = model_gemv(args, world, rank, local, args.steps, args.warmup, wtype="Q4_0")
    elif args.workload == "model_qgemm":
        res = model_qgemm(args, world, rank, local, args.steps, args.warmup)
    elif args.workload == "model_fgemm":
        res = model_qgemm(args, world, rank, local, args.steps, args.warmup, wtype="F16")
    else:
        res = decode_batched(args, world, rank, local)
        if not args.no_prefill:
            res["prefill"] = prefill(args, world, rank, local, steps=legs, warmup=3)
        if not args.no_extra:
            res["decode_long"] = decode_long(args, world, rank, local, legs, 3)
            res["decode_ragged"] = decode_ragged(args, world, rank, local, legs, 3)
            res["model_decode_gemv"] = model_gemv(args, world, rank, local, legs, 3)
            res["model_decode_gemv_q4_0"] = model_gemv(args, world, rank, local, legs, 3, wtype="Q4_0")
            res["model_prefill_qgemm_q4_0"] = model_qgemm(args, world, rank, local, legs, 3)
            res["model_prefill_fgemm_f16"] = model_qgemm(args, world, rank, local, legs, 3, wtype="F16")
    res.setdefault("scaling", args.scaling)
    res.update({"n_gpus": world, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
                "vs_baseline": None, "data": "synthetic (seeded N(0,1))"})
    res["gpu_launches"] = res.pop("gpu_launches_per_step", 2) * args.steps
    if rank == 0 and world == 1 and args.cpu_seconds > 0 and args.workload == "decode_batched":
        res["cpu_baseline"] = cpu_baseline(args.cpu_seconds)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
