"""Generates the known-answer fixtures in tests/golden/ from the constructions
in the reference's own hardware tests (crates/ipu-tests/src/main.rs).  Expected
outputs come from the closed-form answers those tests check, not from the
oracle, so the fixtures pin the oracle and the CUDA kernels alike.

    python tests/golden/make_golden.py      # rewrites the .npz files
"""
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def gemm_right_value(inner, column):
    """main.rs:2132-2135: B pattern over {-1, -0.5, 0, 0.5, 1} as f16 bits."""
    values = np.array([0xBC00, 0xB800, 0x0000, 0x3800, 0x3C00], dtype=np.uint16)
    return values[(inner * 3 + column) % 5]


def gemm_smoke(tiles=4, batch=32):
    """gemm-smoke (main.rs:1060-1104 inputs, :2077-2131 check): per logical tile
    t, A[b, i] = 1 where i == (7b + t) % 64 else 0; B[i, c] =
    gemm_right_value(i, 64t + c); expected C[b, c] = gemm_right_value(sel, 64t + c)
    bit-exactly."""
    a = np.zeros((tiles, batch, 64), dtype=np.uint16)
    b = np.zeros((tiles, 64, 64), dtype=np.uint16)
    c = np.zeros((tiles, batch, 64), dtype=np.uint16)
    inner = np.arange(64)[:, None]
    for t in range(tiles):
        cols = 64 * t + np.arange(64)[None, :]
        b[t] = gemm_right_value(inner, cols)
        for bi in range(batch):
            sel = (bi * 7 + t) % 64
            a[t, bi, sel] = 0x3C00
            c[t, bi] = gemm_right_value(sel, 64 * t + np.arange(64))
    return dict(a=a, b=b, c=c)


def gemm_allones(rows=1024, inner=64, columns=64):
    """gemm-benchmark (main.rs:1591-1592 inputs 0x3c00 / 0x3400, :1774-1800
    check): every output equals 0.25 * inner within 0.002*|e| + 0.01."""
    return dict(shape=np.array([rows, inner, columns]), expected=np.array([0.25 * inner], dtype=np.float32),
                atol=np.array([0.25 * inner * 0.002 + 0.01], dtype=np.float32))


def projected_attention(heads=16, tokens=729, head_dim=72):
    """siglip-attention-benchmark (main.rs:1199-1299): input all 1.0, Q/K/V
    weights all f16(1/model_width); every output equals
    f16(1/width) * width within 0.02 (main.rs:1286, :1297-1299)."""
    width = heads * head_dim
    w = np.float16(1.0 / width)
    expected = np.float32(w) * np.float32(width)
    return dict(shape=np.array([heads, tokens, head_dim]), weight_bits=np.array([w.view(np.uint16)]),
                expected=np.array([expected], dtype=np.float32), atol=np.array([0.02], dtype=np.float32))


def attention_smoke():
    """attention-smoke (main.rs:1305-1505): 4 heads, 17 queries, 19 keys, head
    dim 72, inputs ~ N(0, 0.25^2) in f16; tolerance max 0.012, rms 0.003.
    The reference's generator (SplitMix64 + StandardNormal) is not
    reproducible here, so inputs come from numpy's PCG64 with these seeds."""
    rng = np.random.default_rng(0x6174746E5F71)
    q = (rng.standard_normal((4, 17, 72)) * 0.25).astype(np.float16)
    k = (rng.standard_normal((4, 19, 72)) * 0.25).astype(np.float16)
    v = (rng.standard_normal((4, 19, 72)) * 0.25).astype(np.float16)
    return dict(q=q.view(np.uint16), k=k.view(np.uint16), v=v.view(np.uint16),
                max_err=np.array([0.012], dtype=np.float32), rms_err=np.array([0.003], dtype=np.float32))


def main():
    np.savez_compressed(os.path.join(HERE, "gemm_smoke.npz"), **gemm_smoke())
    np.savez_compressed(os.path.join(HERE, "gemm_allones.npz"), **gemm_allones())
    np.savez_compressed(os.path.join(HERE, "projected_attention.npz"), **projected_attention())
    np.savez_compressed(os.path.join(HERE, "attention_smoke.npz"), **attention_smoke())


if __name__ == "__main__":
    main()
