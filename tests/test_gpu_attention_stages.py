"""Parity of the staged attention kernels (softmax, merge) against the
oracle's restatement of device/attention_softmax_f16.cpp and
device/attention_stages_f16.S."""
import numpy as np
import pytest
import torch

import ipuc
import oracle
from conftest import seeded_normal
from gpu_util import dev_f32, dev_u16, empty_u16, host_f32, host_u16

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("Q,keys,KB,D", [(16, 64, 64, 64), (33, 50, 64, 72), (128, 128, 128, 128), (1, 1, 16, 8)])
def test_softmax_stage(Q, keys, KB, D):
    scores = oracle.f16_bits(seeded_normal(Q + keys, (KB // 16, Q, 16), 4.0))
    w_want, state_want = oracle.attention_softmax(scores, Q, keys, KB, D)
    nbytes_half = Q * KB + 4 * Q  # weights + 2*Q f32 state
    out = empty_u16(nbytes_half)
    ipuc.attention_softmax_f16(out, dev_u16(scores), Q, keys, KB, D)
    got = host_u16(out)
    w = got[: Q * KB]
    state = got[Q * KB:].view(np.float32)
    dw = np.abs(w.view(np.float16).astype(np.float32) - w_want.view(np.float16).astype(np.float32))
    assert dw.max() <= 1e-3
    assert (w == w_want).mean() > 0.99
    assert np.allclose(state[:Q], state_want[:Q], rtol=0, atol=0)
    assert np.allclose(state[Q:], state_want[Q:], rtol=1e-5)


@pytest.mark.parametrize("initial,final", [(1, 0), (0, 0), (0, 1), (1, 1)])
def test_merge_stage(initial, final):
    Q, V, Vp = 40, 72, 80
    rng = np.random.default_rng(initial * 2 + final)
    acc = rng.standard_normal((Q, Vp)).astype(np.float32)
    acc[:, V] = rng.standard_normal(Q)          # running max
    acc[:, V + 1] = rng.uniform(1, 5, Q)        # running denominator
    block = oracle.f16_bits(seeded_normal(9, ((V + 15) // 16, Q, 16)))
    state = np.concatenate([rng.standard_normal(Q), rng.uniform(1, 5, Q)]).astype(np.float32)
    want = oracle.attention_merge(acc, block, state, Q, V, Vp, initial, final)
    a = dev_f32(acc)
    ipuc.attention_merge_f16(a, dev_u16(block), dev_f32(state), Q, V, Vp, initial, final)
    got = host_f32(a)
    assert np.allclose(got[:, : V + 2], want[:, : V + 2], rtol=2e-6, atol=1e-6)
    assert np.array_equal(got[:, V + 2:], acc[:, V + 2:])
