"""Bit-exact parity of the layout kernels (rearrange / unpack / general order
conversion / SplitHeads) against the oracle's restatement of
device/rearrange_f16.cpp, device/unpack_amp_f16.cpp and storage.rs."""
import numpy as np
import pytest

import ipuc
import oracle
from gpu_util import dev_u16, empty_u16, host_u16

pytestmark = pytest.mark.gpu


def bits(seed, n):
    return np.random.default_rng(seed).integers(0, 0x7C00, n, dtype=np.uint16)


@pytest.mark.parametrize("target,matrices,R,Rp,C,Cp,rb,cb", [
    (0, 1, 64, 64, 64, 64, 64, 16), (0, 3, 17, 20, 30, 32, 64, 16), (0, 1, 1, 1, 2, 16, 64, 16),
    (0, 2, 129, 130, 250, 256, 64, 16),
    (1, 1, 64, 64, 16, 16, 64, 16), (1, 2, 50, 64, 14, 16, 64, 16), (1, 1, 128, 128, 72, 80, 64, 16),
    (2, 1, 64, 64, 64, 64, 64, 16), (2, 2, 60, 64, 60, 64, 64, 16), (2, 1, 100, 128, 32, 32, 64, 32),
    (2, 1, 256, 256, 128, 128, 128, 64),
])
def test_rearrange_bit_exact(target, matrices, R, Rp, C, Cp, rb, cb):
    src = bits(target * 100 + R, matrices * R * C)
    want = oracle.rearrange_f16(src, matrices, R, Rp, target, C, Cp, rb, cb)
    out = empty_u16(matrices * Rp * Cp)
    ipuc.rearrange_f16(out, dev_u16(src), matrices, R, Rp, target, C, Cp, rb, cb)
    assert np.array_equal(host_u16(out), want)


@pytest.mark.parametrize("matrices,R,C", [(1, 64, 64), (3, 192, 320), (1, 4096, 4096), (2, 1024, 1088)])
def test_rearrange_block_major_tma_path(matrices, R, C):
    """Row-major -> BlockMajor{64,16} over whole 64x64 tiles takes the TMA +
    ldmatrix.trans/stmatrix kernel (4096 x 4096: every CTA wraps its 8-stage
    ring several times); bit-exact against storage.rs's index map."""
    src = bits(R * 3 + C, matrices * R * C)
    want = oracle.rearrange_f16(src, matrices, R, R, 2, C, C, 64, 16)
    out = empty_u16(matrices * R * C)
    ipuc.rearrange_f16(out, dev_u16(src), matrices, R, R, 2, C, C, 64, 16)
    assert np.array_equal(host_u16(out), want)


@pytest.mark.parametrize("order,matrices,R,Rp,C,Cp", [
    (0, 1, 64, 64, 64, 64), (0, 2, 7, 9, 30, 32), (0, 1, 100, 100, 17, 48), (0, 2, 1000, 1024, 3999, 4096),
    (1, 1, 64, 64, 64, 64), (1, 3, 30, 32, 20, 22), (1, 1, 128, 128, 1, 2),
])
def test_unpack_bit_exact(order, matrices, R, Rp, C, Cp):
    src = bits(order * 7 + R, matrices * Rp * Cp)
    want = oracle.unpack_f16(src, order, matrices, R, Rp, C, Cp)
    out = empty_u16(matrices * Rp * Cp)
    ipuc.unpack_f16(out, dev_u16(src), order, matrices, R, Rp, C, Cp)
    assert np.array_equal(host_u16(out), want)


ORDERS = [oracle.ROW_MAJOR, oracle.AMP_LEFT, oracle.AMP_TRANSPOSED_LEFT, oracle.AMP_TRANSPOSED_RIGHT,
          oracle.AMP_OUTPUT, oracle.AMP_TRANSPOSED_OUTPUT, oracle.BLOCK_MAJOR, oracle.BLOCK_MAJOR_TRANSPOSED]


def pack(logical, order, rows, cols, rb, cb):
    out = np.zeros(rows * cols, np.uint16)
    for r in range(rows):
        for c in range(cols):
            out[oracle.layout_index(order, rows, cols, r, c, rb, cb)] = logical[r, c]
    return out


@pytest.mark.parametrize("frm", ORDERS)
@pytest.mark.parametrize("to", ORDERS)
def test_convert_order_every_pair(frm, to):
    rows, cols, rb, cb = 64, 64, 32, 16
    logical = bits(frm * 8 + to, rows * cols).reshape(rows, cols)
    src = pack(logical, frm, rows, cols, rb, cb)
    want = pack(logical, to, rows, cols, rb, cb)
    out = empty_u16(rows * cols)
    ipuc.convert_order_f16(out, to, dev_u16(src), frm, 1, rows, cols, rb, cb)
    assert np.array_equal(host_u16(out), want)


@pytest.mark.parametrize("b,r,h,c", [(2, 33, 4, 16), (1, 7, 3, 5), (4, 128, 32, 128)])
def test_split_heads_bit_exact(b, r, h, c):
    x = bits(b * r + h, b * r * h * c).reshape(b, r, h * c)
    want = oracle.split_heads(x, h)
    out = empty_u16(x.size)
    ipuc.split_heads_f16(out, dev_u16(x), b, r, h, c)
    assert np.array_equal(host_u16(out), want.ravel())


@pytest.mark.parametrize("b,r,h,c", [(2, 33, 4, 16), (1, 7, 3, 5)])
def test_merge_heads_inverts_split_heads(b, r, h, c):
    x = bits(b * r * h + c, b * r * h * c).reshape(b, r, h * c)
    split = empty_u16(x.size)
    ipuc.split_heads_f16(split, dev_u16(x), b, r, h, c)
    back = empty_u16(x.size)
    ipuc.merge_heads_f16(back, split, b, r, h, c)
    assert np.array_equal(host_u16(back), x.ravel())
