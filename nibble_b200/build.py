"""Builds libnibble_cuda.so (the C ABI + sm_100a kernels) in-tree with nvcc.

    python -m nibble_b200.build [--force] [--verbose]

The library is compiled for sm_100a only (`-gencode arch=compute_100a,code=sm_100a`); nvcc cross-compiles it
without a GPU. A stamp file keyed on the sources' contents and the flags skips rebuilding unchanged code.
"""
from __future__ import annotations

import argparse
import hashlib
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libnibble_cuda.so")
STAMP = LIB + ".stamp"
SOURCES = ["api.cu", "rope.cu", "attn_f32.cu", "decode.cu", "decode_static.cu", "prefill.cu", "model_ops.cu", "quant_ops.cu", "quant_gemm.cu", "quant_blocks.cu", "f32_gemm.cu", "selftest.cu", "backend_route.cu"]
HEADERS = ["qkv_epilogue.cuh", "nbl_device.cuh", "nbl_internal.h", "nbl_errors.h", "model_ops.h", "quant_common.cuh"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-I" + os.path.join(ROOT, "include")]
# Per-file additions: quant_gemm.cu must keep every multiply and add separately rounded (the reference's
# arithmetic), so nothing in it may be contracted into a fused multiply-add.
FILE_FLAGS = {"quant_gemm.cu": ["-fmad=false"], "quant_blocks.cu": ["-fmad=false"]}


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libnibble_cuda.so")


def _digest(extra: list[str]) -> str:
    h = hashlib.sha256()
    for name in SOURCES + HEADERS:
        with open(os.path.join(CSRC, name), "rb") as f:
            h.update(name.encode() + b"\0" + f.read())
    with open(os.path.join(ROOT, "include", "nibble_cuda.h"), "rb") as f:
        h.update(f.read())
    # the flags name the repository's absolute path (-I): leave it out, so a tree copied elsewhere (the GPU box's
    # snapshot) keeps the stamp of the library it ships with
    h.update(" ".join(ARCH + FLAGS + extra).replace(ROOT, "<root>").encode())
    h.update(repr(sorted(FILE_FLAGS.items())).encode())
    return h.hexdigest()


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> str:
    """Compiles the library if its sources changed; returns the .so path."""
    extra = list(extra or [])
    digest = _digest(extra)
    if not force and os.path.exists(LIB) and os.path.exists(STAMP):
        with open(STAMP) as f:
            if f.read().strip() == digest:
                return LIB
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    objs = []
    cc = nvcc()
    procs = []
    for name in SOURCES:
        obj = os.path.join(objdir, name.replace(".cu", ".o"))
        cmd = [cc, *ARCH, *FLAGS, *FILE_FLAGS.get(name, []), *extra, "-c", os.path.join(CSRC, name), "-o", obj]
        if verbose:
            cmd += ["-Xptxas", "-v"]
            print(" ".join(cmd), file=sys.stderr)
        procs.append((name, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
        objs.append(obj)
    failed = []
    for name, p in procs:
        out, _ = p.communicate()
        if verbose or p.returncode:
            sys.stderr.write(out)
        if p.returncode:
            failed.append(name)
    if failed:
        raise RuntimeError(f"nvcc failed for {', '.join(failed)}")
    tmp = LIB + ".tmp"
    subprocess.run([cc, *ARCH, "-shared", "-o", tmp, *objs, "-lcudart_static", "-lrt", "-ldl", "-lpthread"],
                   check=True)
    os.replace(tmp, LIB)
    with open(STAMP, "w") as f:
        f.write(digest)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose))


if __name__ == "__main__":
    main()
