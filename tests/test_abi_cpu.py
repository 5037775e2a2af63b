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


FAKE = 1 << 20   # a 256-byte aligned address that validation rejects the call before touching


@pytest.mark.parametrize("args,status,text", [
    ((FAKE, FAKE, FAKE, 64, 64, 64, 64, 64, 64, ipuc.GEMM_OUT_F32, FAKE, 1 << 30, None), ipuc.ERR_INVALID_ARGUMENT,
     "only IPUC_GEMM_ACCUMULATE"),
    ((FAKE, FAKE, FAKE, 64, 64, 62, 62, 64, 64, 0, FAKE, 1 << 30, None), ipuc.ERR_ALIGNMENT, "multiples of 4"),
    ((FAKE, FAKE, FAKE, 64, 64, 64, 64, 64, 64, ipuc.GEMM_F32_SPLIT_TF32, None, 0, None), ipuc.ERR_INVALID_ARGUMENT,
     "workspace smaller"),
    ((FAKE, FAKE, FAKE, 64, 64, 64, 64, 64, 64, 0, FAKE, 16, None), ipuc.ERR_INVALID_ARGUMENT, "workspace smaller"),
])
def test_gemm_f32_validation(args, status, text):
    L = ipuc.lib()
    assert L.ipuc_gemm_f32(*args) == status
    assert text in L.ipuc_last_error_string().decode()


def test_gemm_f32_workspace_covers_both_splits():
    for m, n, k in [(1, 4, 4), (300, 260, 100), (4096, 4096, 4096), (2200, 4104, 1000)]:
        kp = (k + 7) // 8 * 8
        r = lambda x: (x + 255) // 256 * 256
        # planes, exponents/maxima/tiny counts/fix-up flags, fix-up bitmap
        f16 = 2 * r(m * kp * 2) + 2 * r(n * kp * 2) + 3 * r(m * 4) + 3 * r(n * 4) + r(m * ((n + 31) // 32) * 4)
        tf32 = 2 * r(m * k * 4) + 2 * r(k * n * 4)
        assert ipuc.gemm_f32_workspace_bytes(m, n, k) == max(f16, tf32)


def test_graph_library_exports_every_ipug_symbol():
    text = re.sub(r"/\*.*?\*/", "", open(os.path.join(ROOT, "include", "ipug.h")).read(), flags=re.S)
    names = sorted(set(re.findall(r"\b(ipug_[a-z0-9_]+)\s*\(", text)))
    assert len(names) >= 15
    L = ipuc.lib()
    for name in names:
        assert hasattr(L, name), name


def test_ipuc_error_carries_status():
    with pytest.raises(ipuc.IpucError) as e:
        ipuc.call("ipuc_gelu_f16", None, None, 5, None)
    assert e.value.status == ipuc.ERR_INVALID_ARGUMENT


def test_peer_all_reduce_argument_checks():
    """ipuc_peer_all_reduce_f16 rejects bad pointer tables, worlds, ranks,
    element counts and alignment before touching the device."""
    L = ipuc.lib()
    arr = ctypes.c_void_p * 2
    good = arr(0x1000, 0x2000)
    sig = arr(0x3000, 0x4000)
    assert L.ipuc_peer_signal_bytes() > 0 and L.ipuc_peer_signal_bytes() % 16 == 0
    cases = [
        ((None, good, sig, 0, 2, 1024), 1, "null pointer table"),
        ((good, good, sig, 0, 1, 1024), 1, "world"),
        ((good, good, sig, 0, 9, 1024), 1, "world"),
        ((good, good, sig, 2, 2, 1024), 1, "rank"),
        ((good, good, sig, 0, 2, 1000), 1, "multiple of 8 * world"),
        ((good, arr(0x2000, None), sig, 0, 2, 1024), 1, "null buffer"),
        ((arr(0x1001, 0x2000), good, sig, 0, 2, 1024), 3, "16-byte aligned"),
    ]
    for args, code, text in cases:
        st = L.ipuc_peer_all_reduce_f16(*args, None)
        assert st == code, (args, st)
        assert text in L.ipuc_last_error_string().decode()
    assert L.ipuc_peer_all_reduce_f16(good, good, sig, 0, 2, 0, None) == 0  # nothing to do


def test_ipc_argument_checks():
    L = ipuc.lib()
    off = ctypes.c_uint64(0)
    buf = ctypes.create_string_buffer(64)
    assert L.ipuc_ipc_handle(None, buf, 64, ctypes.byref(off)) == 1
    assert L.ipuc_ipc_handle(ctypes.c_void_p(0x1000), buf, 32, ctypes.byref(off)) == 1
    p = ctypes.c_void_p()
    assert L.ipuc_ipc_open(None, 0, ctypes.byref(p)) == 1
    assert L.ipuc_ipc_close(None) == 1


def test_session_peer_reduce_rejects_null_session():
    from ipuc.graph import glib
    assert glib().ipug_session_peer_reduce(None, 1, None) == 1
    assert "null session" in ipuc.lib().ipuc_last_error_string().decode()
