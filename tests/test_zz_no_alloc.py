"""The allocation-free FP32 GEMM entry point (ipuc_gemm_f32_noalloc).

It exists for callers that cannot allocate device memory when they issue the
GEMM (plug-ins whose host framework owns the device allocator, host callbacks,
fixed-budget real-time paths): its f16 split planes live in a fixed 64 MiB device array inside
libipuc.so.  These tests call it through the C ABI and check it against the
workspace entry point ipuc_gemm_f32 on two calls in a row (the second with new
inputs, so leftover scratch contents would show), within the FP32 GEMM
tolerance rel-L2 <= 1e-5, plus the size limit.  This file is named to be
collected last."""
import ctypes

import numpy as np
import pytest
import torch

import ipuc

pytestmark = pytest.mark.gpu


def _noalloc(c, a, b, m, n, k, flags=0):
    return ipuc.lib().ipuc_gemm_f32_noalloc(c.data_ptr(), a.data_ptr(), b.data_ptr(), m, n, k, k,
                                            k if flags & ipuc.GEMM_B_TRANSPOSED else n, n, flags,
                                            torch.cuda.current_stream().cuda_stream)


def _with_workspace(m, n, k, a, b, flags=0):
    c = torch.empty((m, n), dtype=torch.float32, device="cuda")
    ws = torch.empty(ipuc.gemm_f32_workspace_bytes(m, n, k), dtype=torch.uint8, device="cuda")
    ipuc.gemm_f32(c, a, b, m, n, k, ws, flags)
    return c


def _rel_l2(x, y):
    x, y = x.double(), y.double()
    return float((x - y).norm() / y.norm())


@pytest.mark.parametrize("m,n,k,flags", [(1024, 768, 512, 0), (300, 260, 100, ipuc.GEMM_B_TRANSPOSED),
                                         (2048, 2048, 2048, 0), (2864, 2864, 2864, 0),
                                         (2048, 2048, 2048, ipuc.GEMM_F32_SPLIT_TF32)])
def test_noalloc_matches_workspace_entry_twice(m, n, k, flags):
    g = torch.Generator(device="cuda")
    for call in range(2):
        g.manual_seed(1000 * call + m + k)
        a = torch.rand((m, k), generator=g, device="cuda") * 2 - 1
        b = torch.rand((n, k) if flags & ipuc.GEMM_B_TRANSPOSED else (k, n), generator=g, device="cuda") * 2 - 1
        want = _with_workspace(m, n, k, a, b, flags)
        got = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
        assert _noalloc(got, a, b, m, n, k, flags) == ipuc.OK, ipuc.lib().ipuc_last_error_string()
        torch.cuda.synchronize()
        assert torch.isfinite(got).all()
        assert _rel_l2(got, want) <= 1e-5
        ref = a.double() @ (b.double().t() if flags & ipuc.GEMM_B_TRANSPOSED else b.double())
        assert _rel_l2(got, ref) <= 1e-5
    ipuc.device_status()


def test_noalloc_accumulate_flag():
    m, n, k = 256, 512, 384
    a = torch.rand((m, k), device="cuda") - 0.5
    b = torch.rand((k, n), device="cuda") - 0.5
    c0 = torch.rand((m, n), device="cuda")
    got = c0.clone()
    assert _noalloc(got, a, b, m, n, k, ipuc.GEMM_ACCUMULATE) == ipuc.OK
    want = c0.clone()
    ws = torch.empty(ipuc.gemm_f32_workspace_bytes(m, n, k), dtype=torch.uint8, device="cuda")
    ipuc.gemm_f32(want, a, b, m, n, k, ws, ipuc.GEMM_ACCUMULATE)
    torch.cuda.synchronize()
    assert _rel_l2(got, want) <= 1e-5


def test_noalloc_rejects_shapes_beyond_the_array():
    m = n = k = 4096  # needs 256 MiB of split planes
    x = torch.zeros(16, dtype=torch.float32, device="cuda")
    st = ipuc.lib().ipuc_gemm_f32_noalloc(x.data_ptr(), x.data_ptr(), x.data_ptr(), m, n, k, k, n, n, 0,
                                          torch.cuda.current_stream().cuda_stream)
    assert st == ipuc.ERR_INVALID_ARGUMENT
    assert b"64 MiB" in ipuc.lib().ipuc_last_error_string()
