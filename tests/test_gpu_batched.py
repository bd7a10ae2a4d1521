"""Many sequences over one model (row (f)4): the batched decoder (nibble_b200/csrc/host/batched_decoder.cpp) runs N
sequences' decode steps as one forward pass over paged fp16 KV pools; every sequence's logits must match nibble's
own single-sequence Transformer on CpuBackend fed the same tokens (tests/cpp/test_batched.cpp states the scenario
and the tolerance). The binary is oracle/_ref/nbl_batched_check, built with the reference tree present
(oracle/Makefile, target batched-check); it travels to the GPU box with the rest of oracle/_ref."""
import os
import subprocess

import pytest

import oracle


def test_batched_check_is_built_where_the_reference_is():
    if not os.path.isdir(os.path.join(oracle.REF_TREE, "src")):
        pytest.skip("reference tree not present here (the binary is built where it is)")
    oracle.build()
    assert os.path.exists(oracle.BATCHED_CHECK)
    assert os.path.exists(oracle.BATCHED_BENCH)


@pytest.mark.gpu
def test_batched_sequences_match_single_sequence_transformer():
    assert os.path.exists(oracle.BATCHED_CHECK), "oracle/_ref/nbl_batched_check missing: run build() where the reference is"
    r = subprocess.run([oracle.BATCHED_CHECK], capture_output=True, text=True, timeout=900)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "all passed" in r.stdout
