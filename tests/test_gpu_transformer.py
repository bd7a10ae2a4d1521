"""nibble's own Transformer forward pass (src/model/transformer.cpp, compiled unchanged from the reference tree)
run over nibble's CpuBackend and over this repository's CudaBackend on the same random models; the logits of a
chunked prefill, of decode steps and of a continuation must agree (tests/cpp/test_transformer.cpp states the
models and the tolerance). The binary is oracle/_ref/nbl_model_check, built with the reference tree present
(oracle/Makefile, target model-check); it travels to the GPU box with the rest of oracle/_ref."""
import os
import subprocess

import pytest

import oracle


def test_model_check_is_built_where_the_reference_is():
    if not os.path.isdir(os.path.join(oracle.REF_TREE, "src")):
        pytest.skip("reference tree not present here (the binary is built where it is)")
    oracle.build()
    assert os.path.exists(oracle.MODEL_CHECK)


@pytest.mark.gpu
def test_transformer_runs_on_cuda_backend_like_cpu_backend():
    assert os.path.exists(oracle.MODEL_CHECK), "oracle/_ref/nbl_model_check missing: run build() where the reference is"
    r = subprocess.run([oracle.MODEL_CHECK], capture_output=True, text=True, timeout=600)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "all passed" in r.stdout
