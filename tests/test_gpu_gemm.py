"""Parity of the tcgen05 FP16 GEMM (gemm_f16_amp replacement) against the
oracle: the reference's known-answer fixtures bit-exactly, random cases within
the BASELINE FP16 tolerance (max|err| <= 2e-2*max|ref|, rel-L2 <= 5e-3)."""
import os

import numpy as np
import pytest
import torch

import ipuc
import oracle
from conftest import f16_close, seeded_normal
from gpu_util import dev_f32, dev_u16, empty_u16, f16_of, host_f32, host_u16

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def test_gemm_smoke_golden_bits():
    """gemm-smoke (main.rs:1060-1119, 2077-2136): exact f16 bits."""
    g = np.load(os.path.join(GOLDEN, "gemm_smoke.npz"))
    tiles, batch, _ = g["a"].shape
    out = empty_u16(tiles * batch * 64)
    ipuc.gemm_f16_batched(out, dev_u16(g["a"]), dev_u16(g["b"]), tiles, batch, 64, 64)
    assert np.array_equal(host_u16(out).reshape(g["c"].shape), g["c"])


def test_gemm_allones_golden():
    g = np.load(os.path.join(GOLDEN, "gemm_allones.npz"))
    m, k, n = (int(x) for x in g["shape"])
    a = torch.full((m, k), 1.0, dtype=torch.float16, device="cuda")
    b = torch.full((k, n), 0.25, dtype=torch.float16, device="cuda")
    c = torch.empty((m, n), dtype=torch.float16, device="cuda")
    ipuc.gemm_f16(c, a, b, m, n, k)
    torch.cuda.synchronize()
    assert (c.float() - float(g["expected"][0])).abs().max().item() <= float(g["atol"][0])


def run_case(m, n, k, flags=0, seed=0, with_c=False):
    bt = bool(flags & ipuc.GEMM_B_TRANSPOSED)
    a = oracle.f16_bits(seeded_normal(seed, (m, k), 0.1))
    b = oracle.f16_bits(seeded_normal(seed + 1, (n, k) if bt else (k, n), 0.1))
    af, bf = f16_of(a), f16_of(b)
    ref = oracle.gemm(af, bf, False, bt)
    out_f32 = bool(flags & ipuc.GEMM_OUT_F32)
    c0 = seeded_normal(seed + 2, (m, n)) if with_c else None
    if with_c:
        c0 = c0 if out_f32 else oracle.quantize_f16(c0)
        ref = ref + c0
    if not out_f32:
        ref = oracle.quantize_f16(ref)
    if flags & ipuc.GEMM_EPILOGUE_GELU:
        ref = oracle.gelu(ref)
        if not out_f32:
            ref = oracle.quantize_f16(ref)
    if out_f32:
        c = dev_f32(c0) if with_c else torch.empty((m, n), dtype=torch.float32, device="cuda")
    else:
        c = dev_u16(oracle.f16_bits(c0)) if with_c else empty_u16(m * n)
    ipuc.gemm_f16(c, dev_u16(a), dev_u16(b), m, n, k, flags=flags)
    got = host_f32(c) if out_f32 else f16_of(host_u16(c))
    return got.reshape(m, n), ref


@pytest.mark.parametrize("m,n,k", [(256, 256, 256), (128, 256, 64), (512, 1024, 512), (300, 200, 136),
                                   (1, 8, 8), (1000, 520, 1032), (2048, 2048, 4096)])
@pytest.mark.parametrize("bt", [False, True])
def test_gemm_random(m, n, k, bt):
    got, ref = run_case(m, n, k, ipuc.GEMM_B_TRANSPOSED if bt else 0, seed=m + n + k)
    ok, msg = f16_close(got, ref)
    assert ok, msg


@pytest.mark.parametrize("flags,with_c", [
    (ipuc.GEMM_ACCUMULATE, True), (ipuc.GEMM_OUT_F32, False), (ipuc.GEMM_OUT_F32 | ipuc.GEMM_ACCUMULATE, True),
    (ipuc.GEMM_EPILOGUE_GELU, False), (ipuc.GEMM_EPILOGUE_GELU | ipuc.GEMM_ACCUMULATE, True),
    (ipuc.GEMM_EPILOGUE_GELU | ipuc.GEMM_B_TRANSPOSED, False),
])
def test_gemm_epilogues(flags, with_c):
    got, ref = run_case(384, 640, 320, flags, seed=flags, with_c=with_c)
    if flags & ipuc.GEMM_OUT_F32:
        l2 = np.linalg.norm(got - ref) / np.linalg.norm(ref)
        assert l2 <= 1e-5, l2
    else:
        ok, msg = f16_close(got, ref)
        assert ok, msg


@pytest.mark.parametrize("m,n,k,flags,ld_pad", [
    (384, 640, 320, 0, 0), (300, 520, 256, ipuc.GEMM_EPILOGUE_GELU, 8), (2048, 2048, 1024, 0, 0),
    (384, 640, 320, ipuc.GEMM_OUT_F32, 4), (1000, 136, 72, ipuc.GEMM_B_TRANSPOSED, 16)])
def test_gemm_addend_epilogue(m, n, k, flags, ld_pad):
    """ipuc_gemm_f16_addend: C = epilogue(A.B + D) with D a separate tensor (the
    fused residual add), read at its own leading dimension; C is not read."""
    bt = bool(flags & ipuc.GEMM_B_TRANSPOSED)
    out_f32 = bool(flags & ipuc.GEMM_OUT_F32)
    a = oracle.f16_bits(seeded_normal(m, (m, k), 0.1))
    b = oracle.f16_bits(seeded_normal(n, (n, k) if bt else (k, n), 0.1))
    ld = n + ld_pad
    d = seeded_normal(k, (m, ld))
    d = d if out_f32 else oracle.quantize_f16(d)
    ref = oracle.gemm(f16_of(a), f16_of(b), False, bt) + d[:, :n]
    if not out_f32:
        ref = oracle.quantize_f16(ref)
    if flags & ipuc.GEMM_EPILOGUE_GELU:
        ref = oracle.quantize_f16(oracle.gelu(ref))
    if out_f32:
        c, dd = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda"), dev_f32(d)
    else:
        c, dd = empty_u16(m * n), dev_u16(oracle.f16_bits(d))
    ipuc.gemm_f16_addend(c, dev_u16(a), dev_u16(b), m, n, k, dd, ld_addend=ld, flags=flags)
    got = (host_f32(c) if out_f32 else f16_of(host_u16(c))).reshape(m, n)
    if out_f32:
        assert np.linalg.norm(got - ref) / np.linalg.norm(ref) <= 1e-5
    else:
        ok, msg = f16_close(got, ref)
        assert ok, msg


def test_gemm_splitk_partials_reduce():
    """Config-3 lowering shape: split-K into 4 f32 partials (GEMM with
    OUT_F32 on K slices), combined by reduce_add, then GELU."""
    m, n, k, parts = 256, 512, 1024, 4
    a = oracle.f16_bits(seeded_normal(7, (m, k)))
    b = oracle.f16_bits(seeded_normal(8, (k, n), 1 / 32))
    ad, bd = dev_u16(a), dev_u16(b)
    partials = torch.empty((parts, m, n), dtype=torch.float32, device="cuda")
    ks = k // parts
    for p in range(parts):
        ipuc.call("ipuc_gemm_f16", partials[p].data_ptr(), ad.data_ptr() + p * ks * 2, bd.data_ptr() + p * ks * n * 2,
                  m, n, ks, k, n, n, ipuc.GEMM_OUT_F32, torch.cuda.current_stream().cuda_stream)
    summed = empty_u16(m * n)
    ipuc.reduce_sum(summed, partials[0], partials[1:], parts - 1, m * n, ipuc.F32)
    out = empty_u16(m * n)
    ipuc.gelu_f16(out, summed)
    ref = oracle.quantize_f16(oracle.gelu(oracle.quantize_f16(oracle.gemm(f16_of(a), f16_of(b)))))
    ok, msg = f16_close(f16_of(host_u16(out)).reshape(m, n), ref)
    assert ok, msg


def test_gemm_batched_random():
    batch, m, n, k = 3, 200, 96, 128
    a = oracle.f16_bits(seeded_normal(1, (batch, m, k)))
    b = oracle.f16_bits(seeded_normal(2, (batch, k, n)))
    out = empty_u16(batch * m * n)
    ipuc.gemm_f16_batched(out, dev_u16(a), dev_u16(b), batch, m, n, k)
    ref = oracle.quantize_f16(oracle.gemm(f16_of(a), f16_of(b)))
    ok, msg = f16_close(f16_of(host_u16(out)).reshape(batch, m, n), ref)
    assert ok, msg


def test_gemm_device_status_clean():
    ipuc.device_status()


@pytest.mark.parametrize("m,n,k", [(256, 256, 256), (128, 192, 64), (1024, 2048, 512), (304, 200, 136),
                                   (2048, 2048, 1024)])
@pytest.mark.parametrize("bt", [False, True])
def test_gemm_a_transposed(m, n, k, bt):
    """GemmOptions::transpose_left: A stored [k x m], read M-major by the
    tensor cores (single-CTA and CTA-pair kernels, with either B layout)."""
    at = oracle.f16_bits(seeded_normal(m + 1, (k, m), 0.1))
    b = oracle.f16_bits(seeded_normal(n + 2, (n, k) if bt else (k, n), 0.1))
    ref = oracle.quantize_f16(oracle.gemm(f16_of(at), f16_of(b), True, bt))
    c = empty_u16(m * n)
    flags = ipuc.GEMM_A_TRANSPOSED | (ipuc.GEMM_B_TRANSPOSED if bt else 0)
    ipuc.gemm_f16(c, dev_u16(at), dev_u16(b), m, n, k, flags=flags)
    ok, msg = f16_close(f16_of(host_u16(c)).reshape(m, n), ref)
    assert ok, msg


def test_gemm_a_transposed_batched_gelu():
    batch, m, n, k = 3, 384, 256, 192
    at = oracle.f16_bits(seeded_normal(5, (batch, k, m), 0.1))
    b = oracle.f16_bits(seeded_normal(6, (batch, k, n), 0.1))
    ref = oracle.quantize_f16(oracle.gelu(oracle.quantize_f16(oracle.gemm(f16_of(at), f16_of(b), True, False))))
    c = empty_u16(batch * m * n)
    ipuc.gemm_f16_batched(c, dev_u16(at), dev_u16(b), batch, m, n, k,
                          flags=ipuc.GEMM_A_TRANSPOSED | ipuc.GEMM_EPILOGUE_GELU)
    ok, msg = f16_close(f16_of(host_u16(c)).reshape(batch, m, n), ref)
    assert ok, msg


@pytest.mark.parametrize("flags,with_c", [(0, False), (ipuc.GEMM_EPILOGUE_GELU, False), (ipuc.GEMM_OUT_F32, False),
                                          (ipuc.GEMM_ACCUMULATE, True), (ipuc.GEMM_B_TRANSPOSED, False)])
def test_gemm_partial_last_wave(flags, with_c):
    """80 pair tiles (2048 x 2560) on the persistent CTA-pair kernel: a full
    wave of 74 pair slots and a partial one, with every epilogue."""
    got, ref = run_case(2048, 2560, 1024, flags, seed=77 + flags, with_c=with_c)
    ok, msg = f16_close(got, ref)
    assert ok, msg


def test_gemm_partial_last_wave_with_addend():
    """gemm_f16_addend (C = A.B + D, D separate) on the same shape, twice in a
    row."""
    m, n, k = 2048, 2560, 1024
    a = oracle.f16_bits(seeded_normal(91, (m, k), 0.1))
    b = oracle.f16_bits(seeded_normal(92, (k, n), 0.1))
    d = oracle.f16_bits(seeded_normal(93, (m, n)))
    ref = oracle.quantize_f16(oracle.gemm(f16_of(a), f16_of(b)) + f16_of(d))
    for _ in range(2):
        c = empty_u16(m * n)
        ipuc.gemm_f16_addend(c, dev_u16(a), dev_u16(b), m, n, k, dev_u16(d))
        ok, msg = f16_close(f16_of(host_u16(c)).reshape(m, n), ref)
        assert ok, msg
    ipuc.device_status()


@pytest.mark.parametrize("shared", ["a", "b"])
@pytest.mark.parametrize("at", [False, True])
def test_gemm_batched_shared_operand(shared, at):
    """ipuc_gemm_f16_batched with a zero stride: one operand shared by every
    batch entry (K-major A with shared B takes the one-GEMM path; the others
    run per entry)."""
    batch, m, n, k = 3, 256, 192, 128
    a_shape = (k, m) if at else (m, k)
    a = oracle.f16_bits(seeded_normal(61, (1 if shared == "a" else batch,) + a_shape, 0.1))
    b = oracle.f16_bits(seeded_normal(62, (1 if shared == "b" else batch, k, n), 0.1))
    af = np.broadcast_to(f16_of(a), (batch,) + a_shape)
    bf = np.broadcast_to(f16_of(b), (batch, k, n))
    ref = oracle.quantize_f16(oracle.gemm(af, bf, at, False))
    c = empty_u16(batch * m * n)
    flags = ipuc.GEMM_A_TRANSPOSED if at else 0
    ad, bd = dev_u16(a), dev_u16(b)
    ipuc.call("ipuc_gemm_f16_batched", c.data_ptr(), ad.data_ptr(), bd.data_ptr(), batch, m, n, k,
              m if at else k, n, n, 0 if shared == "a" else m * k, 0 if shared == "b" else k * n, m * n, flags,
              torch.cuda.current_stream().cuda_stream)
    ok, msg = f16_close(f16_of(host_u16(c)).reshape(batch, m, n), ref)
    assert ok, msg
