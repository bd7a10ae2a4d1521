"""The C ABI library without a GPU: it builds for sm_100a, loads, exports every entry point include/nibble_cuda.h
declares (and nothing the Python binding lacks), and rejects bad arguments on the host before touching CUDA."""
import ctypes as C
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "nibble_cuda.h")


def declared():
    with open(HEADER) as f:
        text = f.read()
    return sorted(set(re.findall(r"NBL_API\s+[\w\*\s]+?\b(nbl_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    from nibble_b200 import _abi
    names = declared()
    assert len(names) >= 20
    out = subprocess.run(["nm", "-D", "--defined-only", _abi.LIB_PATH], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\sT\s(nbl_\w+)", out))
    missing = [n for n in names if n not in exported]
    assert not missing, f"declared but not exported: {missing}"
    extra = sorted(exported - set(names))
    assert not extra, f"exported but not declared in the header: {extra}"
    assert set(_abi.SIGNATURES) == set(names), "the Python binding covers exactly the header's entry points"


def test_build_targets_sm100a_only():
    from nibble_b200 import build
    assert build.ARCH == ["-gencode", "arch=compute_100a,code=sm_100a"]


def test_abi_version_matches_header():
    from nibble_b200 import _abi
    with open(HEADER) as f:
        v = int(re.search(r"#define NBL_ABI_VERSION (\d+)", f.read()).group(1))
    assert _abi.lib.nbl_abi_version() == v


def test_host_side_argument_checks_need_no_gpu():
    from nibble_b200 import _abi
    p = C.c_void_p()
    assert _abi.lib.nbl_alloc(None, 10, C.byref(p)) == _abi.NBL_E_INVALID
    assert "NULL" in _abi.last_error()
    assert _abi.lib.nbl_kv_create(None, None, C.byref(p)) == _abi.NBL_E_INVALID
    assert _abi.lib.nbl_rope(None, None, 1, 1, 2, 0, None) == _abi.NBL_E_INVALID
    assert _abi.lib.nbl_ctx_destroy(None) == _abi.NBL_OK  # destroying nothing is a no-op
    # nbl_last_error truncates into small buffers and reports the full length
    full = _abi.lib.nbl_last_error(None, 0)
    buf = C.create_string_buffer(4)
    assert _abi.lib.nbl_last_error(buf, 4) == full and len(buf.value) == 3


def test_ctx_create_without_gpu_reports_cuda_error():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from nibble_b200 import _abi
    h = C.c_void_p()
    st = _abi.lib.nbl_ctx_create(0, C.byref(h))
    assert st in (_abi.NBL_E_CUDA, _abi.NBL_E_INVALID) and not h.value
    assert _abi.last_error()


def test_python_wrapper_raises_nibble_error():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    import nibble_b200 as nb
    with pytest.raises(nb.NibbleError):
        nb.Context(0, use_torch_stream=False)


def test_dtype_codes_match_header():
    """The Python binding's element-type codes are the header's nbl_dtype values, and the quantized ones map to
    nibble's DType ids the oracle uses (src/tensor.h:21-31) in the same order the CudaBackend maps them."""
    from nibble_b200 import _abi
    import oracle
    with open(HEADER) as f:
        text = f.read()
    enum = dict((k, int(v)) for k, v in re.findall(r"\bNBL_(F32|F16|BF16|Q\d_[0-9K])\s*=\s*(\d+)", text))
    assert set(enum) == {"F32", "F16", "BF16", "Q4_0", "Q5_0", "Q8_0", "Q5_1", "Q4_K", "Q5_K", "Q6_K"}
    for name, code in enum.items():
        assert getattr(_abi, name) == code, name
    with open(os.path.join(ROOT, "nibble_b200", "csrc", "host", "cuda_backend.cpp")) as f:
        mapped = dict(re.findall(r"case DType::(\w+): dt = NBL_(\w+);", f.read()))
    assert mapped == {n: n for n in ("F32", "F16", "Q4_0", "Q5_0", "Q8_0", "Q5_1", "Q4_K", "Q5_K", "Q6_K")}
    for name in ("Q4_0", "Q5_0", "Q5_1", "Q8_0", "Q4_K", "Q5_K", "Q6_K"):
        assert getattr(oracle, name) in oracle.BLOCK_BYTES
