"""Parity of the three-pass TF32 FP32 GEMM (gemm_f32_64_amp replacement)
against the oracle's f32 SGEMM (diagnostic.rs:581-654).  BASELINE tolerance:
rel-L2 <= 1e-5."""
import numpy as np
import pytest
import torch

import ipuc
import oracle
from conftest import seeded_uniform
from gpu_util import dev_f32, host_f32

pytestmark = pytest.mark.gpu


def rel_l2(a, b):
    return float(np.linalg.norm(a.astype(np.float64) - b) / np.linalg.norm(b))


def run(m, n, k, flags=0, c0=None, seed=0):
    bt = bool(flags & ipuc.GEMM_B_TRANSPOSED)
    a = seeded_uniform(seed, (m, k))
    b = seeded_uniform(seed + 1, (n, k) if bt else (k, n))
    ref = oracle.gemm(a.astype(np.float64), b.astype(np.float64), False, bt)
    c = dev_f32(c0) if c0 is not None else torch.empty((m, n), dtype=torch.float32, device="cuda")
    if c0 is not None:
        ref = ref + c0
    ws = torch.empty(max(1, ipuc.gemm_f32_workspace_bytes(m, n, k)), dtype=torch.uint8, device="cuda")
    ipuc.gemm_f32(c, dev_f32(a), dev_f32(b), m, n, k, ws, flags)
    return host_f32(c), ref, a, b


@pytest.mark.parametrize("m,n,k", [(256, 256, 256), (128, 512, 64), (300, 260, 100), (1, 4, 4), (1024, 1024, 1024),
                                   (4096, 4096, 4096)])
@pytest.mark.parametrize("bt", [False, True])
def test_gemm_f32_rel_l2(m, n, k, bt):
    got, ref, a, b = run(m, n, k, ipuc.GEMM_B_TRANSPOSED if bt else 0, seed=m + k)
    assert rel_l2(got, ref) <= 1e-5
    if m * n * k <= 1 << 27:
        # also against the f32 BLAS evaluator itself
        blas = oracle.gemm(a, b, False, bt)
        assert rel_l2(got, blas.astype(np.float64)) <= 1e-5


def test_gemm_f32_accumulate():
    c0 = seeded_uniform(9, (200, 136))
    got, ref, _, _ = run(200, 136, 520, ipuc.GEMM_ACCUMULATE, c0=c0, seed=4)
    assert rel_l2(got, ref) <= 1e-5


@pytest.mark.parametrize("bt", [False, True])
def test_gemm_f32_pair_path_ragged(bt):
    """At least a wave of 256x256 tiles takes the CTA-pair kernel: ragged rows
    (2200 = 8.6 pair tiles), a column tail (4104 = 16 * 256 + 8) and a K tail
    (200 = 6.25 blocks of 32)."""
    got, ref, _, _ = run(2200, 4104, 200, ipuc.GEMM_B_TRANSPOSED if bt else 0, seed=31)
    assert rel_l2(got, ref) <= 1e-5


def test_gemm_f32_pair_path_accumulate():
    c0 = seeded_uniform(12, (2048, 2560))
    got, ref, _, _ = run(2048, 2560, 1000, ipuc.GEMM_ACCUMULATE, c0=c0, seed=13)
    assert rel_l2(got, ref) <= 1e-5


def test_gemm_f32_workspace_checked():
    a = torch.zeros((64, 64), device="cuda")
    small = torch.empty(16, dtype=torch.uint8, device="cuda")
    with pytest.raises(ipuc.IpucError) as e:
        ipuc.gemm_f32(a, a, a, 64, 64, 64, small)
    assert e.value.status == ipuc.ERR_INVALID_ARGUMENT
