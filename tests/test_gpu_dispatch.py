"""ipuc_launch on the GPU: every TileKernelSpec kind routed through the
spec-driven entry gives the oracle's result (and the typed entry's bits)."""
import numpy as np
import pytest
import torch

import ipuc
import oracle
from conftest import f16_close, seeded_normal, seeded_uniform
from gpu_util import dev_f32, dev_u16, empty_u16, f16_of, host_f32, host_u16

pytestmark = pytest.mark.gpu
T = ipuc.TileKernelSpec


def h(t, shape):
    return ipuc.tensor(t, shape, ipuc.F16)


def f(t, shape):
    return ipuc.tensor(t, shape, ipuc.F32)


def test_fill_zero():
    out = empty_u16(96)
    ipuc.launch(T.fill_zero(), h(out, [96]), [], [96 * 2 // 8 // 6, 96 * 2 // 8 % 6])
    assert (host_u16(out) == 0).all()


@pytest.mark.parametrize("mode,b_transposed,gelu", [("initialize", False, False), ("accumulate", False, False),
                                                    ("initialize", True, True)])
def test_gemm_f16(mode, b_transposed, gelu):
    m, n, k = 192, 160, 256
    a = oracle.f16_bits(seeded_normal(1, (m, k), 0.1))
    b = oracle.f16_bits(seeded_normal(2, (k, n), 0.1))
    c0 = oracle.f16_bits(seeded_normal(3, (m, n), 0.5))
    b_dev = np.ascontiguousarray(b.T) if b_transposed else b
    out = dev_u16(c0)
    ipuc.launch(T.gemm(mode=mode, b_transposed=b_transposed, epilogue_gelu=gelu), h(out, [m, n]),
                [h(dev_u16(a), [m, k]), h(dev_u16(b_dev), [n, k] if b_transposed else [k, n])])
    want = oracle.gemm(f16_of(a), f16_of(b))
    if mode == "accumulate":
        want = want + f16_of(c0)
    want = f16_of(oracle.f16_bits(want))
    if gelu:
        want = f16_of(oracle.gelu_f16_bits(oracle.f16_bits(want)))
    ok, msg = f16_close(f16_of(host_u16(out)).reshape(m, n), want)
    assert ok, msg


def test_gemm_f16_batched_out_f32():
    bt, m, n, k = 3, 64, 48, 32
    a = oracle.f16_bits(seeded_normal(4, (bt, m, k), 0.2))
    b = oracle.f16_bits(seeded_normal(5, (bt, k, n), 0.2))
    out = torch.empty(bt * m * n, dtype=torch.float32, device="cuda")
    ipuc.launch(T.gemm(), f(out, [bt, m, n]), [h(dev_u16(a), [bt, m, k]), h(dev_u16(b), [bt, k, n])])
    got = host_f32(out).reshape(bt, m, n)
    for i in range(bt):
        want = oracle.gemm(f16_of(a[i]), f16_of(b[i]))
        assert np.abs(got[i] - want).max() <= 1e-3 * max(1.0, np.abs(want).max())


def test_gemm_f32_with_workspace():
    m, n, k = 128, 96, 64
    a = seeded_uniform(6, (m, k))
    b = seeded_uniform(7, (k, n))
    ws = torch.empty(ipuc.gemm_f32_workspace_bytes(m, n, k), dtype=torch.uint8, device="cuda")
    out = torch.empty(m * n, dtype=torch.float32, device="cuda")
    ipuc.launch(T.gemm(multiply=ipuc.F32), f(out, [m, n]), [f(dev_f32(a), [m, k]), f(dev_f32(b), [k, n])],
                workspace=ws)
    want = a.astype(np.float64) @ b.astype(np.float64)
    got = host_f32(out).reshape(m, n)
    assert np.linalg.norm(got - want) / np.linalg.norm(want) <= 1e-5


def test_gemm_f32_workspace_too_small():
    m = n = k = 64
    out = torch.empty(m * n, dtype=torch.float32, device="cuda")
    a = torch.zeros(m * k, dtype=torch.float32, device="cuda")
    with pytest.raises(ipuc.IpucError) as e:
        ipuc.launch(T.gemm(multiply=ipuc.F32), f(out, [m, n]), [f(a, [m, k]), f(a, [k, n])],
                    workspace=torch.empty(16, dtype=torch.uint8, device="cuda"))
    assert e.value.status == ipuc.ERR_INVALID_ARGUMENT


def test_gelu_matches_typed_entry():
    n = 4096
    x = dev_u16(oracle.f16_bits(seeded_normal(8, n, 2.0)))
    a, b = empty_u16(n), empty_u16(n)
    ipuc.launch(T.gelu(), h(a, [n]), [h(x, [n])], [n])
    ipuc.gelu_f16(b, x)
    assert (host_u16(a) == host_u16(b)).all()


@pytest.mark.parametrize("prec", [ipuc.F16, ipuc.F32])
def test_reduction_sum(prec):
    partials, n = 4, 8 * 1000
    init = seeded_normal(9, n)
    remote = seeded_normal(10, (partials - 1) * n)
    if prec == ipuc.F16:
        init, remote = f16_of(oracle.f16_bits(init)), f16_of(oracle.f16_bits(remote))
        di, dr = dev_u16(oracle.f16_bits(init)), dev_u16(oracle.f16_bits(remote))
        ti, tr = h(di, [n]), h(dr, [(partials - 1) * n])
    else:
        di, dr = dev_f32(init), dev_f32(remote)
        ti, tr = f(di, [n]), f(dr, [(partials - 1) * n])
    out = empty_u16(n)
    ipuc.launch(T.reduction_sum(partials), h(out, [n]), [ti, tr], [partials - 1, n])
    want = oracle.reduce_sum(init, remote.reshape(partials - 1, n))
    ok, msg = f16_close(f16_of(host_u16(out)), f16_of(want))
    assert ok, msg


def test_add_broadcast_bit_exact():
    n, period = 64 * 48, 48
    left = oracle.f16_bits(seeded_normal(11, n))
    right = oracle.f16_bits(seeded_normal(12, period))
    out = empty_u16(n)
    ipuc.launch(T.add(), h(out, [64, 48]), [h(dev_u16(left), [64, 48]), h(dev_u16(right), [48])], [n, 0, period])
    assert (host_u16(out) == oracle.add_f16(left, right, n, 0, period)).all()


@pytest.mark.parametrize("out_prec", [ipuc.F16, ipuc.F32])
def test_flash_attention(out_prec):
    M, S, D = 3, 200, 64
    q, k, v = (oracle.f16_bits(seeded_normal(20 + i, (M, S, D))) for i in range(3))
    if out_prec == ipuc.F16:
        out = empty_u16(M * S * D)
        o = h(out, [M, S, D])
    else:
        out = torch.empty(M * S * D, dtype=torch.float32, device="cuda")
        o = f(out, [M, S, D])
    ipuc.launch(T.flash_attention(), o, [h(dev_u16(x), [M, S, D]) for x in (q, k, v)])
    got = f16_of(host_u16(out)) if out_prec == ipuc.F16 else host_f32(out)
    want = oracle.attention(f16_of(q), f16_of(k), f16_of(v), threads=4)
    ok, msg = f16_close(got.reshape(M, S, D), want)
    assert ok, msg


def test_attention_stage_chain_matches_typed_entries():
    """Softmax then merge through ipuc_launch, the merge reading the row state
    that follows the weights in the softmax output (low.rs:2405-2465)."""
    rows, kbc, hd, V, Vp = 48, 64, 64, 64, 80
    scores = oracle.f16_bits(seeded_normal(30, kbc * rows, 2.0))
    block = oracle.f16_bits(seeded_normal(31, (V // 16) * rows * 16))
    weights = torch.zeros(rows * kbc + 4 * rows, dtype=torch.int16, device="cuda")
    ipuc.launch(T.attention_softmax(hd, 50, kbc), h(weights, [rows * kbc + 4 * rows]),
                [h(dev_u16(scores), [kbc // 16, rows, 16])])
    w_ref, state_ref = oracle.attention_softmax(scores, rows, 50, kbc, hd)
    w = host_u16(weights)
    assert (w[:rows * kbc] == w_ref).all()
    assert np.array_equal(w[rows * kbc:].view(np.float32), state_ref)
    acc = torch.zeros(rows * Vp, dtype=torch.float32, device="cuda")
    ipuc.launch(T.attention_merge(V, Vp, kbc, True, True), f(acc, [rows, Vp]),
                [h(dev_u16(block), [V // 16, rows, 16]), h(weights, [rows * kbc + 4 * rows])], [1, 1])
    want = oracle.attention_merge(np.zeros(rows * Vp, np.float32), block, state_ref, rows, V, Vp, True, True)
    got = host_f32(acc)
    assert np.allclose(got.reshape(rows, Vp)[:, :V], want.reshape(rows, Vp)[:, :V], rtol=1e-5, atol=1e-6)


def test_cast_round_trip():
    n = 1000
    x = seeded_normal(40, n)
    src = dev_f32(x)
    half = empty_u16(n)
    ipuc.launch(T.cast(ipuc.F32, ipuc.F16), h(half, [n]), [f(src, [n])], [n])
    assert (host_u16(half) == oracle.f16_bits(x)).all()
    back = torch.empty(n, dtype=torch.float32, device="cuda")
    ipuc.launch(T.cast(ipuc.F16, ipuc.F32), f(back, [n]), [h(half, [n])], [n])
    assert np.array_equal(host_f32(back), f16_of(oracle.f16_bits(x)))


@pytest.mark.parametrize("target,order", [(0, ipuc.AMP_LEFT), (1, ipuc.AMP_TRANSPOSED_RIGHT),
                                          (2, ipuc.BLOCK_MAJOR)])
def test_rearrange_row_major_to_target(target, order):
    mats, R, C = 2, 70, 40
    Rp, Cp = 128, 48
    src = oracle.f16_bits(seeded_normal(50 + target, mats * R * C))
    out = empty_u16(mats * Rp * Cp)
    spec = T.rearrange(ipuc.ROW_MAJOR, (order, 64, 16) if order == ipuc.BLOCK_MAJOR else order)
    ipuc.launch(spec, h(out, [mats, Rp, Cp]), [h(dev_u16(src), [mats, R, C])], [R, Rp, target, C, Cp])
    assert (host_u16(out) == oracle.rearrange_f16(src, mats, R, Rp, target, C, Cp)).all()


@pytest.mark.parametrize("source", [0, 1])
def test_unpack_to_row_major(source):
    mats, R, C, Rp, Cp = 2, 50, 30, 64, 32
    src = oracle.f16_bits(seeded_normal(60 + source, mats * Rp * Cp))
    out = empty_u16(mats * Rp * Cp)
    order = ipuc.AMP_OUTPUT if source == 0 else ipuc.AMP_TRANSPOSED_LEFT
    ipuc.launch(T.rearrange(order, ipuc.ROW_MAJOR), h(out, [mats, Rp, Cp]), [h(dev_u16(src), [mats, Rp, Cp])],
                [mats, R, Rp, C, Cp])
    assert (host_u16(out) == oracle.unpack_f16(src, source, mats, R, Rp, C, Cp)).all()


def test_generic_rearrange_matches_typed_entry():
    mats, R, C = 2, 128, 64
    src = dev_u16(oracle.f16_bits(seeded_normal(70, mats * R * C)))
    a, b = empty_u16(mats * R * C), empty_u16(mats * R * C)
    ipuc.launch(T.rearrange(ipuc.AMP_LEFT, ipuc.AMP_OUTPUT), h(a, [mats, R, C]), [h(src, [mats, R, C])])
    ipuc.convert_order_f16(b, ipuc.AMP_OUTPUT, src, ipuc.AMP_LEFT, mats, R, C)
    assert (host_u16(a) == host_u16(b)).all()
