"""CPU-only checks of the C-ABI library: it loads, exports every entry point
include/ipuc.h declares, and its host-side argument validation (the
validate_kernel_run rules, crates/ipu-codegen/src/kernel.rs:1384-1435) rejects
bad calls before any CUDA call is made."""
import ctypes
import os
import re

import pytest

import ipuc

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    text = open(os.path.join(ROOT, "include", "ipuc.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ipuc_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_header_symbol():
    L = ipuc.lib()
    names = header_functions()
    assert len(names) >= 20
    for name in names:
        assert hasattr(L, name), name


def test_bindings_cover_header():
    assert set(header_functions()) <= set(ipuc.SIGNATURES) | {"ipuc_version"}


def test_status_strings():
    L = ipuc.lib()
    assert L.ipuc_status_string(0) == b"IPUC_OK"
    assert L.ipuc_status_string(6) == b"IPUC_ERR_DEVICE_TIMEOUT"
    assert b"sm_100a" in L.ipuc_version()


@pytest.mark.parametrize("fn,args,status,text", [
    ("ipuc_gelu_f16", (None, None, 3, None), ipuc.ERR_INVALID_ARGUMENT, "even"),
    ("ipuc_reduce_sum", (None, None, None, 0, 8, 0, None), ipuc.ERR_INVALID_ARGUMENT, "two partials"),
    ("ipuc_reduce_sum", (None, None, None, 1, 12, 0, None), ipuc.ERR_INVALID_ARGUMENT, "multiple of 8"),
    ("ipuc_fill_zero", (None, 12, None), ipuc.ERR_INVALID_ARGUMENT, "multiple of 8"),
    ("ipuc_rearrange_f16", (None, None, 1, 4, 4, 0, 3, 16, 64, 16, None), ipuc.ERR_INVALID_ARGUMENT, "even"),
    ("ipuc_rearrange_f16", (None, None, 1, 4, 4, 5, 4, 16, 64, 16, None), ipuc.ERR_INVALID_ARGUMENT, "target_order"),
    ("ipuc_rearrange_f16", (None, None, 1, 8, 4, 0, 4, 16, 64, 16, None), ipuc.ERR_INVALID_ARGUMENT, "exceeds"),
    ("ipuc_unpack_f16", (None, None, 2, 1, 4, 4, 4, 16, None), ipuc.ERR_INVALID_ARGUMENT, "source_order"),
    ("ipuc_gemm_f16", (None, None, None, 4, 4, 0, 8, 8, 8, 0, None), ipuc.ERR_INVALID_ARGUMENT, "k must"),
    ("ipuc_gemm_f16", (None, None, None, 4, 4, 8, 8, 8, 8, 1 << 7, None), ipuc.ERR_INVALID_ARGUMENT, "flag"),
    ("ipuc_attention_softmax_f16", (None, None, 4, 10, 24, 64, None), ipuc.ERR_INVALID_ARGUMENT, "multiple of 16"),
    ("ipuc_attention_merge_f16", (None, None, None, 4, 64, 65, 1, 1, None), ipuc.ERR_INVALID_ARGUMENT, "state"),
])
def test_validation_rejects_before_launch(fn, args, status, text):
    L = ipuc.lib()
    st = getattr(L, fn)(*args)
    assert st == status
    assert text in L.ipuc_last_error_string().decode()


def test_ipuc_error_carries_status():
    with pytest.raises(ipuc.IpucError) as e:
        ipuc.call("ipuc_gelu_f16", None, None, 5, None)
    assert e.value.status == ipuc.ERR_INVALID_ARGUMENT
