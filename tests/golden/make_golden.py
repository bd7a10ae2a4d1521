"""Generates tests/golden/*.npz from nibble's own code (oracle/_ref/libnibble_ref.so, compiled from the reference
sources by oracle/Makefile). Run where the reference tree exists:

    python tests/golden/make_golden.py

Each fixture stores the seeded inputs and the reference's outputs:
  attention_<name>.npz : q, k, v, n, pos0, H, KV, D -> out_scalar (cpu::attention_heads, ref_ops.cpp:188) and
                         out_backend (CpuBackend::attention with the AVX2/AVX-VNNI tier, cpu_backend.cpp:272)
  rope_<name>.npz      : x, n, H, D, pos0, base, neox, ff -> out (cpu::rope, ref_ops.cpp:166)
  softmax.npz          : x -> out (cpu::softmax_inplace, ref_ops.cpp:66)
  fp16.npz             : every fp16 bit pattern -> fp32 (src/fp16.h:18), and a float sample -> fp16 (fp16.h:46)

The attention shapes are the reference's own test cases (tests/test_ops.cpp:200-201,
tests/test_cpu_backend.cpp:66) plus small cases shaped like the benchmark models (Qwen2.5 / Llama-3.2 / TinyLlama head layouts).
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import oracle  # noqa: E402

ATTN_CASES = {
    # name: (n, pos0, H, KV, D, qscale, seed)
    "ops_1_0_2_1_8": (1, 0, 2, 1, 8, 1.0, 5),
    "ops_7_3_6_2_16": (7, 3, 6, 2, 16, 1.0, 6),
    "ops_4_300_4_2_64": (4, 300, 4, 2, 64, 1.0, 7),
    "ops_3_40_2_2_13": (3, 40, 2, 2, 13, 1.0, 8),
    "ops_2_20_4_1_128": (2, 20, 4, 1, 128, 1.0, 9),
    "ops_5_60_4_2_64_q30": (5, 60, 4, 2, 64, 30.0, 10),
    "backend_7_3_6_2_16": (7, 3, 6, 2, 16, 1.0, 2),
    "qwen_prefill_16": (16, 0, 14, 2, 64, 1.0, 11),
    "qwen_decode_pos200": (1, 200, 14, 2, 64, 1.0, 12),
    "llama_decode_pos255": (1, 255, 32, 8, 64, 1.0, 13),
    "tinyllama_prefill_24_pos9": (24, 9, 32, 4, 64, 1.0, 14),
}

ROPE_CASES = {
    # name: (n, H, D, pos0, base, neox, with_factors, seed)
    "qwen_neox": (3, 14, 64, 0, 1e6, True, False, 21),
    "qwen_neox_far": (2, 2, 64, 131070, 1e6, True, False, 22),
    "llama_interleaved": (3, 8, 64, 4093, 5e5, False, False, 23),
    "llama_factors": (2, 4, 64, 77, 5e5, False, True, 24),
    "tinyllama": (4, 4, 64, 2044, 1e4, False, False, 25),
    "odd_small": (1, 1, 4, 1, 1e4, False, False, 26),
}


def main() -> None:
    if not oracle.have_ref():
        sys.exit("oracle/_ref/libnibble_ref.so is not built (needs the reference tree): make -C oracle ref")
    be = oracle.RefBackend(4)
    for name, (n, pos0, H, KV, D, qs, seed) in ATTN_CASES.items():
        rng = np.random.default_rng(seed)
        ctx = pos0 + n
        q = (rng.standard_normal((n, H, D)) * qs).astype(np.float32)
        k = rng.standard_normal((ctx, KV, D)).astype(np.float32)
        v = rng.standard_normal((ctx, KV, D)).astype(np.float32)
        out_s = oracle.ref_attention_scalar(q, k, v, n, pos0, H, KV, D)
        out_b = be.attention(q, k, v, n, pos0, H, KV, D)
        np.savez_compressed(os.path.join(HERE, f"attention_{name}.npz"), q=q, k=k, v=v,
                            meta=np.array([n, pos0, H, KV, D], np.int64), out_scalar=out_s, out_backend=out_b)
    for name, (n, H, D, pos0, base, neox, with_ff, seed) in ROPE_CASES.items():
        rng = np.random.default_rng(seed)
        x = rng.standard_normal((n, H, D)).astype(np.float32)
        ff = (1.0 + rng.random(D // 2)).astype(np.float32) if with_ff else np.zeros(0, np.float32)
        out = oracle.ref_rope(x, H, D, pos0, base, neox, ff if with_ff else None)
        np.savez_compressed(os.path.join(HERE, f"rope_{name}.npz"), x=x, ff=ff, out=out,
                            meta=np.array([n, H, D, pos0, int(neox)], np.int64), base=np.float32(base))
    rng = np.random.default_rng(31)
    x = np.concatenate([rng.standard_normal(37).astype(np.float32) * 20, np.array([1000, 1000, -1000], np.float32)])
    np.savez_compressed(os.path.join(HERE, "softmax.npz"), x=x, out=oracle.ref_softmax(x))
    widened = oracle.ref_fp16_bits_to_f32(np.arange(65536, dtype=np.uint16))
    sample = np.concatenate([rng.standard_normal(4000).astype(np.float32) * np.float32(1000),
                             np.array([65504, 65520, 1e-8, -6e-8, 3e-5, np.inf, -np.inf, 0.0, -0.0], np.float32)])
    narrowed = oracle.ref_f32_to_fp16_bits(sample)
    np.savez_compressed(os.path.join(HERE, "fp16.npz"), widened=widened, sample=sample, narrowed=narrowed)
    print("kernels tier:", oracle.ref_kernels_name())
    print("wrote", len(ATTN_CASES) + len(ROPE_CASES) + 2, "fixtures to", HERE)


if __name__ == "__main__":
    main()
