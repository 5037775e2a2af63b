"""Parity of the FP32 GEMM (gemm_f32_64_amp replacement): the default scaled
three-pass f16 split and the three-pass TF32 split (IPUC_GEMM_F32_SPLIT_TF32)
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


SPLITS = [0, ipuc.GEMM_F32_SPLIT_TF32]   # default scaled 3xF16, and 3xTF32


@pytest.mark.parametrize("m,n,k", [(256, 256, 256), (128, 512, 64), (300, 260, 100), (1, 4, 4), (1024, 1024, 1024),
                                   (4096, 4096, 4096)])
@pytest.mark.parametrize("bt", [False, True])
@pytest.mark.parametrize("split", SPLITS)
def test_gemm_f32_rel_l2(m, n, k, bt, split):
    got, ref, a, b = run(m, n, k, (ipuc.GEMM_B_TRANSPOSED if bt else 0) | split, seed=m + k)
    assert rel_l2(got, ref) <= 1e-5
    if m * n * k <= 1 << 27:
        # also against the f32 BLAS evaluator itself
        blas = oracle.gemm(a, b, False, bt)
        assert rel_l2(got, blas.astype(np.float64)) <= 1e-5


@pytest.mark.parametrize("split", SPLITS)
def test_gemm_f32_accumulate(split):
    c0 = seeded_uniform(9, (200, 136))
    got, ref, _, _ = run(200, 136, 520, ipuc.GEMM_ACCUMULATE | split, c0=c0, seed=4)
    assert rel_l2(got, ref) <= 1e-5


@pytest.mark.parametrize("bt", [False, True])
@pytest.mark.parametrize("split", SPLITS)
def test_gemm_f32_pair_path_ragged(bt, split):
    """At least a wave of 256x256 tiles takes the CTA-pair kernel: ragged rows
    (2200 = 8.6 pair tiles), a column tail (4104 = 16 * 256 + 8) and a K tail
    (200 = 6.25 blocks of 32)."""
    got, ref, _, _ = run(2200, 4104, 200, (ipuc.GEMM_B_TRANSPOSED if bt else 0) | split, seed=31)
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


@pytest.mark.parametrize("bt", [False, True])
def test_gemm_f32_row_and_column_scales(bt):
    """The f16 split scales every row of A and column of B by its own power of
    two, so rows and columns spread over 1e-36 .. 1e35 keep fp32 accuracy
    relative to their own size: C_ij / (sA_i sB_j) against fp64 within rel-L2
    1e-5 (scales chosen so that C itself stays inside the fp32 range; the
    combined exponent still leaves the single-multiply range, which takes the
    two-step unscale).  All-zero rows and columns give exact zeros."""
    m, n, k = 384, 520, 300
    rng = np.random.default_rng(41)
    sa = 10.0 ** rng.uniform(-28, 27, m)
    sb = 10.0 ** rng.uniform(-8, 8, n)
    a0 = seeded_uniform(42, (m, k)).astype(np.float64)
    b0 = seeded_uniform(43, (k, n)).astype(np.float64)
    a0[5] = 0.0
    b0[:, 7] = 0.0
    a = (a0 * sa[:, None]).astype(np.float32)
    b = (b0 * sb[None, :]).astype(np.float32)
    ref = a.astype(np.float64) @ b.astype(np.float64)
    bd = np.ascontiguousarray(b.T) if bt else b
    c = torch.empty((m, n), dtype=torch.float32, device="cuda")
    ws = torch.empty(ipuc.gemm_f32_workspace_bytes(m, n, k), dtype=torch.uint8, device="cuda")
    ipuc.gemm_f32(c, dev_f32(a), dev_f32(bd), m, n, k, ws, ipuc.GEMM_B_TRANSPOSED if bt else 0)
    got = host_f32(c).astype(np.float64)
    assert np.isfinite(got).all()
    scale = sa[:, None] * sb[None, :]
    assert rel_l2(got / scale, ref / scale) <= 1e-5
    assert (got[5] == 0).all() and (got[:, 7] == 0).all()


def test_gemm_f32_tiny_and_huge_magnitudes():
    """Rows near the fp32 limits (subnormal and 1e38 maxima) stay accurate
    relative to their own maximum."""
    m, n, k = 256, 256, 128
    a0 = seeded_uniform(51, (m, k)).astype(np.float64)
    b = seeded_uniform(52, (k, n))
    a0[0] *= 1e-40                       # subnormal fp32 row
    a0[1] *= 1e-36
    a0[2] *= 1e37 / np.abs(a0[2]).max()  # largest element 1e37 (C stays below the fp32 limit)
    a = a0.astype(np.float32)
    ref = a.astype(np.float64) @ b.astype(np.float64)
    c = torch.empty((m, n), dtype=torch.float32, device="cuda")
    ws = torch.empty(ipuc.gemm_f32_workspace_bytes(m, n, k), dtype=torch.uint8, device="cuda")
    ipuc.gemm_f32(c, dev_f32(a), dev_f32(b), m, n, k, ws)
    got = host_f32(c).astype(np.float64)
    for r in range(m):
        s = np.abs(a[r]).astype(np.float64).max() * np.abs(b).max()
        tol = 1e-5 if r != 0 else 1e-3   # a subnormal row carries fewer than 24 bits itself
        assert np.abs(got[r] - ref[r]).max() <= tol * s * np.sqrt(k), r


@pytest.mark.parametrize("bt", [False, True])
@pytest.mark.parametrize("split", SPLITS)
def test_gemm_f32_split_k_tail(bt, split):
    """153 pair tiles on 74 CTA pairs leave a last wave of 5 tiles, which runs as
    two K halves per tile added into C by atomics: the last tile column is 8
    wide (4104 = 16 * 256 + 8) and the last tile row ragged (2200 rows)."""
    got, ref, _, _ = run(2200, 4104, 1000, (ipuc.GEMM_B_TRANSPOSED if bt else 0) | split, seed=37)
    assert rel_l2(got, ref) <= 1e-5
    again, _, _, _ = run(2200, 4104, 1000, (ipuc.GEMM_B_TRANSPOSED if bt else 0) | split, seed=37)
    assert np.array_equal(got, again)   # two atomic adds onto zero do not depend on their order


def _elementwise_ok(got, a, b, bt, c0=None, rtol=1e-5, atol_rel=1e-6):
    """|err_ij| <= rtol |ref_ij| + atol_rel (|A| |B|)_ij against fp64."""
    a64, b64 = a.astype(np.float64), (b.T if bt else b).astype(np.float64)
    ref = a64 @ b64 + (0 if c0 is None else c0)
    scale = np.abs(a64) @ np.abs(b64) + (0 if c0 is None else np.abs(c0))
    err = np.abs(got.astype(np.float64) - ref)
    bad = err > rtol * np.abs(ref) + atol_rel * scale
    return not bad.any(), f"{bad.sum()} elements off; worst {np.max(err / np.maximum(np.abs(ref), 1e-300)):.3g} rel"


def _wide_rows(m, k, seed):
    """Rows mixing 1.0 (in columns `big`) with values near 1e-8."""
    rng = np.random.default_rng(seed)
    a = (rng.uniform(-1, 1, (m, k)) * 1e-8).astype(np.float32)
    big = rng.choice(k, max(1, k // 16), replace=False)
    a[:, big] = 1.0
    return a, big


@pytest.mark.parametrize("m,n,k", [(256, 384, 512), (2304, 2048, 1024)])
@pytest.mark.parametrize("bt", [False, True])
def test_gemm_f32_wide_dynamic_range_rows(m, n, k, bt):
    """Each row of A holds 1.0 and values near 1e-8; B is zero where A is 1.0,
    so every C element is made of the tiny values alone.  The scaled split
    alone loses ~10 bits here; the fix-up must give an fp32 result."""
    a, big = _wide_rows(m, k, seed=m + k)
    b = seeded_uniform(7, (k, n))
    b[big, :] = 0.0
    bb = np.ascontiguousarray(b.T) if bt else b
    c = torch.empty((m, n), dtype=torch.float32, device="cuda")
    ws = torch.empty(ipuc.gemm_f32_workspace_bytes(m, n, k), dtype=torch.uint8, device="cuda")
    ipuc.gemm_f32(c, dev_f32(a), dev_f32(bb), m, n, k, ws, ipuc.GEMM_B_TRANSPOSED if bt else 0)
    got = host_f32(c)
    ok, msg = _elementwise_ok(got, a, bb, bt)
    assert ok, msg
    ref = a.astype(np.float64) @ b.astype(np.float64)
    assert rel_l2(got, ref) <= 1e-5


@pytest.mark.parametrize("bt", [False, True])
def test_gemm_f32_wide_dynamic_range_columns(bt):
    """The same with the wide range along B's columns, A zero where B is big,
    and IPUC_GEMM_ACCUMULATE onto a random C."""
    m, n, k = 640, 520, 768
    bcols, big = _wide_rows(n, k, seed=3)          # [n, k]: column j of B is row j here
    b = np.ascontiguousarray(bcols.T)              # [k, n]
    a = seeded_uniform(8, (m, k))
    a[:, big] = 0.0
    c0 = seeded_uniform(9, (m, n))
    bb = bcols if bt else b
    c = dev_f32(c0)
    ws = torch.empty(ipuc.gemm_f32_workspace_bytes(m, n, k), dtype=torch.uint8, device="cuda")
    ipuc.gemm_f32(c, dev_f32(a), dev_f32(bb), m, n, k, ws,
                  ipuc.GEMM_ACCUMULATE | (ipuc.GEMM_B_TRANSPOSED if bt else 0))
    ok, msg = _elementwise_ok(host_f32(c), a, bb, bt, c0=c0.astype(np.float64))
    assert ok, msg


@pytest.mark.parametrize("bt", [False, True])
def test_gemm_f32_non_finite_inputs(bt):
    """inf, -inf and NaN inputs give the IEEE pattern of the evaluator's SGEMM
    (oracle.gemm) element by element; everything else keeps the tolerance."""
    m, n, k = 2304, 2048, 520       # a CTA-pair shape with a K tail
    a = seeded_uniform(21, (m, k))
    b = seeded_uniform(22, (k, n))
    a[5, 7] = np.inf
    a[300, 11] = -np.inf
    a[301, 11] = np.inf
    a[301, 12] = -np.inf            # +inf and -inf in one row: NaN wherever both meet finite nonzero B
    a[1000, 100] = np.nan
    b[11, 40] = 0.0                 # inf * 0 in column 40 for rows 300 and 301
    b[200, 77] = np.inf
    b[201, 1500] = np.nan
    bb = np.ascontiguousarray(b.T) if bt else b
    c = torch.empty((m, n), dtype=torch.float32, device="cuda")
    ws = torch.empty(ipuc.gemm_f32_workspace_bytes(m, n, k), dtype=torch.uint8, device="cuda")
    ipuc.gemm_f32(c, dev_f32(a), dev_f32(bb), m, n, k, ws, ipuc.GEMM_B_TRANSPOSED if bt else 0)
    got = host_f32(c)
    with np.errstate(invalid="ignore", over="ignore"):
        ref = oracle.gemm(a, b)
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    assert np.array_equal(np.isposinf(got), np.isposinf(ref))
    assert np.array_equal(np.isneginf(got), np.isneginf(ref))
    fin = np.isfinite(ref)
    assert fin.sum() > 0.99 * m * n
    # elements outside the rows and columns that hold a non-finite input
    r64 = np.where(np.isfinite(a), a, 0).astype(np.float64) @ np.where(np.isfinite(b), b, 0).astype(np.float64)
    keep = fin & np.isfinite(a).all(1)[:, None] & np.isfinite(b).all(0)[None, :]
    assert rel_l2(got[keep], r64[keep]) <= 1e-5
