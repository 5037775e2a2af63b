"""Pins the CPU oracle (oracle/) against the known-answer checks of the
reference's own tests.  Each test names the reference test it restates."""
import os

import numpy as np
import pytest

import oracle
from conftest import seeded_normal

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def test_half_conversion_matches_ieee_rne():
    """half 2.7.1 f32->f16 is IEEE round-to-nearest-even (main.rs:2040-2046);
    numpy float16 implements the same rounding."""
    rng = np.random.default_rng(1)
    x = np.concatenate([rng.standard_normal(20000).astype(np.float32) * s for s in (1e-6, 1e-3, 1, 100, 7e4)])
    x = np.concatenate([x, np.array([0.0, -0.0, 65504, 65520, 1e-8, 6.1e-5, np.inf, -np.inf], dtype=np.float32)])
    with np.errstate(over="ignore"):
        want = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(oracle.f16_bits(x), want)


def test_blas_gemm_matches_scalar_reference():
    """randomized_blas_gemm_matches_scalar_reference (diagnostic.rs:855-907):
    256 random shapes, both transposes, |blas - scalar| <= 2e-5."""
    rng = np.random.default_rng(0x424C415347454D4D)
    for _ in range(256):
        rows, inner, cols = rng.integers(1, 17), rng.integers(1, 25), rng.integers(1, 17)
        ta, tb = bool(rng.integers(2)), bool(rng.integers(2))
        a = (rng.random((inner, rows) if ta else (rows, inner)) - 0.5).astype(np.float32)
        b = (rng.random((cols, inner) if tb else (inner, cols)) - 0.5).astype(np.float32)
        blas = oracle.gemm(a, b, ta, tb)
        scalar = oracle.gemm_scalar(a, b, ta, tb)
        assert np.abs(blas - scalar).max() <= 2e-5


def test_gemm_smoke_exact_bits():
    """gemm-smoke (main.rs:1060-1119, 2077-2136): one-hot A x patterned B gives
    exact f16 bits."""
    g = np.load(os.path.join(GOLDEN, "gemm_smoke.npz"))
    a = g["a"].view(np.float16).astype(np.float32)
    b = g["b"].view(np.float16).astype(np.float32)
    c = oracle.f16_bits(oracle.gemm(a, b))
    assert np.array_equal(c, g["c"])


def test_gemm_allones_benchmark_value():
    """gemm-benchmark check (main.rs:1774-1800): ones x 0.25 -> 0.25*K."""
    g = np.load(os.path.join(GOLDEN, "gemm_allones.npz"))
    m, k, n = g["shape"]
    c = oracle.quantize_f16(oracle.gemm(np.ones((m, k), np.float32), np.full((k, n), 0.25, np.float32)))
    assert np.abs(c - g["expected"][0]).max() <= g["atol"][0]


def test_projected_attention_expected_value():
    """siglip-attention-benchmark (main.rs:1199-1299): ones input, constant
    f16(1/width) projections -> every attention output = f16(1/w)*w +- 0.02."""
    g = np.load(os.path.join(GOLDEN, "projected_attention.npz"))
    heads, tokens, d = (int(x) for x in g["shape"])
    tokens = 64  # the expectation is independent of the token count; keep the scalar loop fast
    width = heads * d
    w = np.full((width, width), np.float32(g["weight_bits"].view(np.float16)[0]))
    x = np.ones((tokens, width), np.float32)
    proj = oracle.quantize_f16(oracle.gemm(x, w))  # Q = K = V, f16 op results
    qkv = oracle.split_heads(oracle.f16_bits(proj)[None], heads).view(np.float16).astype(np.float32)
    out = oracle.attention(qkv, qkv, qkv)
    assert np.abs(out - g["expected"][0]).max() <= g["atol"][0]


def test_attention_smoke_online_vs_evaluator():
    """attention-smoke (main.rs:1305-1505): the online (flash) vertex against the
    exact softmax, max err 0.012, rms 0.003."""
    g = np.load(os.path.join(GOLDEN, "attention_smoke.npz"))
    q, k, v = (g[n].view(np.float16).astype(np.float32) for n in ("q", "k", "v"))
    ref = oracle.attention(q, k, v)
    online = oracle.flash_attention_online(g["q"], g["k"], g["v"])
    err = np.abs(online - ref)
    assert err.max() <= g["max_err"][0] and np.sqrt((err ** 2).mean()) <= g["rms_err"][0]


def test_mlp_chain_rounds_between_stages():
    """mlp-smoke reference (main.rs:1996-2033): GEMM-GELU-GEMM-GELU with f16
    rounding of every op result; the evaluator's quantise rule gives the same."""
    x = oracle.quantize_f16(seeded_normal(10, (16, 64), 0.5))
    w0 = oracle.quantize_f16(seeded_normal(11, (64, 64), 0.125))
    w1 = oracle.quantize_f16(seeded_normal(12, (64, 64), 0.125))
    h = oracle.quantize_f16(oracle.gelu(oracle.quantize_f16(oracle.gemm(x, w0))))
    out = oracle.quantize_f16(oracle.gelu(oracle.quantize_f16(oracle.gemm(h, w1))))
    # scalar restatement of mlp_smoke_reference
    ref = np.zeros_like(out)
    for r in range(16):
        hidden = [float(oracle.lib().oracle_gelu(np.float32(np.float16(np.dot(x[r], w0[:, c])))))
                  for c in range(64)]
        hidden = np.array(hidden, np.float32).astype(np.float16).astype(np.float32)
        for c in range(64):
            s = np.float32(np.dot(hidden, w1[:, c]))
            ref[r, c] = np.float16(oracle.lib().oracle_gelu(np.float32(np.float16(s))))
    assert np.abs(out - ref).max() <= 2e-3


def test_gelu_matches_formula():
    """gelu_reference (main.rs:1985-1987) in the C oracle vs numpy."""
    x = np.linspace(-8, 8, 4001, dtype=np.float32)
    c = np.array([oracle.lib().oracle_gelu(float(v)) for v in x], np.float32)
    assert np.abs(c - oracle.gelu(x)).max() <= 1e-6


LAYOUT_CASES = [
    (oracle.AMP_LEFT, 19, 64), (oracle.AMP_LEFT, 64, 48), (oracle.AMP_TRANSPOSED_LEFT, 32, 20),
    (oracle.AMP_TRANSPOSED_RIGHT, 64, 32), (oracle.AMP_OUTPUT, 7, 64), (oracle.AMP_TRANSPOSED_OUTPUT, 48, 9),
    (oracle.BLOCK_MAJOR, 64, 64), (oracle.BLOCK_MAJOR_TRANSPOSED, 32, 128),
]


@pytest.mark.parametrize("order,rows,cols", LAYOUT_CASES)
def test_layout_maps_are_bijections(order, rows, cols):
    """randomized_amp_mappings_are_bijections_and_views_preserve_element_count
    (storage.rs:822) and the coordinate inverses (storage.rs:656-782)."""
    n = rows * cols
    seen = np.zeros(n, bool)
    for r in range(rows):
        for c in range(cols):
            i = oracle.layout_index(order, rows, cols, r, c)
            assert 0 <= i < n and not seen[i]
            seen[i] = True
            assert oracle.layout_coordinates(order, rows, cols, i) == (r, c)
    assert seen.all()


def test_output_to_left_reorder_permutation():
    """randomized_gelu_reorder_preserves_logical_coordinates (diagnostic.rs:910-946):
    word permutation [0,4,1,5,2,6,3,7] maps AMP-Output words onto AMP-Left words."""
    rng = np.random.default_rng(0x47454C555245)
    for _ in range(20):
        rows, cols = int(rng.integers(1, 65)), int(rng.integers(1, 9)) * 16
        words = rows * cols // 2
        perm = [0, 4, 1, 5, 2, 6, 3, 7]
        for worker in range(6):
            base = worker * 8
            while base + 8 <= words:
                for sw, dw in enumerate(perm):
                    for lane in range(2):
                        s = oracle.layout_coordinates(oracle.AMP_OUTPUT, rows, cols, (base + sw) * 2 + lane)
                        d = oracle.layout_coordinates(oracle.AMP_LEFT, rows, cols, (base + dw) * 2 + lane)
                        assert s == d
                base += 48


@pytest.mark.parametrize("target,order,R,Rp,C,Cp", [
    (0, oracle.AMP_LEFT, 17, 20, 30, 32), (0, oracle.AMP_LEFT, 64, 64, 64, 64),
    (1, oracle.AMP_TRANSPOSED_RIGHT, 50, 64, 14, 16), (2, oracle.BLOCK_MAJOR, 64, 64, 60, 64),
    (2, oracle.BLOCK_MAJOR, 100, 128, 32, 32),
])
def test_rearrange_restatement_matches_storage_maps(target, order, R, Rp, C, Cp):
    """The device rearrange codelets (rearrange_f16.cpp) agree with the
    storage.rs index maps: every logical element lands at its index, padding is 0."""
    src = np.arange(2 * R * C, dtype=np.uint16) + 1
    dst = oracle.rearrange_f16(src, 2, R, Rp, target, C, Cp)
    for m in range(2):
        for r in range(Rp):
            for c in range(Cp):
                i = m * Rp * Cp + oracle.layout_index(order, Rp, Cp, r, c)
                want = src[m * R * C + r * C + c] if (r < R and c < C) else 0
                assert dst[i] == want


@pytest.mark.parametrize("source_order,order", [(0, oracle.AMP_OUTPUT), (1, oracle.AMP_TRANSPOSED_LEFT)])
def test_unpack_restatement_inverts_packing(source_order, order):
    """unpack_amp_f16.cpp reverses the AMP-Output / TransposedLeft packing."""
    R, Rp, C, Cp = 30, 32, 40, 48
    packed = np.zeros(Rp * Cp, np.uint16)
    for r in range(Rp):
        for c in range(Cp):
            packed[oracle.layout_index(order, Rp, Cp, r, c)] = r * Cp + c + 1
    out = oracle.unpack_f16(packed, source_order, 1, R, Rp, C, Cp).reshape(Rp, Cp)
    want = (np.arange(Rp)[:, None] * Cp + np.arange(Cp)[None, :] + 1).astype(np.uint16)
    want[R:, :] = 0
    want[:, C:] = 0
    assert np.array_equal(out, want)


def test_staged_softmax_merge_equals_attention():
    """Materialized/staged flash path (low.rs:2385-2470: QK^T -> softmax ->
    PV -> merge per 64-key block) restated with the stage oracles reproduces
    the evaluator's attention within the attention-smoke tolerance."""
    rng = np.random.default_rng(5)
    Q, D, S = 24, 64, 150
    q = (rng.standard_normal((Q, D)) * 0.25).astype(np.float16).astype(np.float32)
    k = (rng.standard_normal((S, D)) * 0.25).astype(np.float16).astype(np.float32)
    v = (rng.standard_normal((S, D)) * 0.25).astype(np.float16).astype(np.float32)
    ref = oracle.attention(q[None], k[None], v[None])[0]
    KB, Vp = 64, D + 16
    acc = np.zeros((Q, Vp), np.float32)
    nblocks = (S + KB - 1) // KB
    for blk in range(nblocks):
        keys = min(KB, S - blk * KB)
        kk = np.zeros((KB, D), np.float32)
        kk[:keys] = k[blk * KB: blk * KB + keys]
        scores = oracle.f16_bits(q @ kk.T)  # QK^T op result rounded to f16
        panels = scores.reshape(Q, KB // 16, 16).transpose(1, 0, 2).copy()
        w, state = oracle.attention_softmax(panels, Q, keys, KB, D)
        wl = w.view(np.float16).astype(np.float32).reshape(KB // 16, Q, 16).transpose(1, 0, 2).reshape(Q, KB)
        vv = np.zeros((KB, D), np.float32)
        vv[:keys] = v[blk * KB: blk * KB + keys]
        pv = oracle.f16_bits(wl @ vv)
        pv_panels = pv.reshape(Q, D // 16, 16).transpose(1, 0, 2).copy()
        acc = oracle.attention_merge(acc, pv_panels, state, Q, D, Vp, blk == 0, blk == nblocks - 1)
    out = acc[:, :D]
    err = np.abs(out - ref)
    assert err.max() <= 0.012 and np.sqrt((err ** 2).mean()) <= 0.003


# ---- explicit index values of the storage orders (f16), computed by hand from
# the closed forms of crates/ipu-codegen/src/storage.rs, so that a wrong but
# bijective map in the oracle (and so in the bit-exact GPU tests) is caught.

# AMP-Left (storage.rs:315-325): (c / 16) * rows * 16 + r * 16 + c % 16.
# rows 4, cols 32.
AMP_LEFT_KAT = [((0, 0), 0), ((0, 15), 15), ((1, 0), 16), ((3, 15), 63), ((0, 16), 64), ((2, 20), 100),
                ((3, 31), 127)]
# AMP-Output (storage.rs:329-340): pair p = (c % 16) / 2 lands at pair
# (p % 4) * 2 + p / 4, i.e. logical columns 0..15 sit at physical columns
# 0 1 4 5 8 9 12 13 2 3 6 7 10 11 14 15.  rows 2, cols 32.
AMP_OUTPUT_COLUMN = [0, 1, 4, 5, 8, 9, 12, 13, 2, 3, 6, 7, 10, 11, 14, 15]
AMP_OUTPUT_KAT = [((0, 2), 4), ((0, 8), 2), ((1, 8), 18), ((1, 13), 27), ((0, 16), 32), ((1, 27), 55),
                  ((1, 31), 63)]
# AMP-TransposedRight (storage.rs:326, 344-371, right_matrix_index on the
# transposed extents): panel (r / 16) * (cols / 16) + c / 16, then
# (r % 16) * 16 + c % 16 inside the 256-element panel.  rows 32, cols 32.
AMP_TRANSPOSED_RIGHT_KAT = [((0, 0), 0), ((0, 1), 1), ((1, 0), 16), ((5, 20), 340), ((20, 3), 579),
                            ((31, 31), 1023)]
# BlockMajor{64, 16} (storage.rs:372-426): panel
# (r / 64) * (cols / 16) * 4 + (c / 16) * 4 + (r % 64) / 16, then
# (c % 16) * 16 + r % 16 inside the 256-element micro-block.  rows 128, cols 32.
BLOCK_MAJOR_KAT = [((0, 0), 0), ((1, 0), 1), ((0, 1), 16), ((16, 0), 256), ((0, 16), 1024), ((70, 17), 3094),
                   ((127, 31), 4095)]
# BlockMajor transposed {64, 16}: the same map on the transposed matrix
# (rows 32, cols 128: element (r, c) takes the index of (c, r) above).
BLOCK_MAJOR_T_KAT = [((17, 70), 3094), ((31, 127), 4095), ((1, 0), 16), ((0, 1), 1)]


@pytest.mark.parametrize("order,rows,cols,table", [
    (oracle.AMP_LEFT, 4, 32, AMP_LEFT_KAT),
    (oracle.AMP_OUTPUT, 2, 32, AMP_OUTPUT_KAT),
    (oracle.AMP_TRANSPOSED_RIGHT, 32, 32, AMP_TRANSPOSED_RIGHT_KAT),
    (oracle.BLOCK_MAJOR, 128, 32, BLOCK_MAJOR_KAT),
    (oracle.BLOCK_MAJOR_TRANSPOSED, 32, 128, BLOCK_MAJOR_T_KAT),
])
def test_layout_index_known_values(order, rows, cols, table):
    for (r, c), want in table:
        assert oracle.layout_index(order, rows, cols, r, c) == want, (r, c)


def test_amp_output_pair_swizzle_row():
    """Every column of one 16-column micro-panel (storage.rs:333-336)."""
    got = [oracle.layout_index(oracle.AMP_OUTPUT, 1, 16, 0, c) for c in range(16)]
    assert got == AMP_OUTPUT_COLUMN


@pytest.mark.parametrize("rows,cols,cb", [(256, 96, 16), (128, 256, 64), (512, 64, 32)])
def test_block_major_span_offsets(rows, cols, cb):
    """The span offset assertion of the block-major view test
    (storage.rs:1034-1045): a view starting at row `inner` (a multiple of 64)
    and column `column` (a multiple of the column block) starts at byte
    ((inner / 64) * column_blocks + column / column_block) * 64 * column_block * 2."""
    for inner in range(0, rows, 64):
        for column in range(0, cols, cb):
            want = ((inner // 64) * (cols // cb) + column // cb) * 64 * cb * 2
            assert oracle.layout_index(oracle.BLOCK_MAJOR, rows, cols, inner, column, 64, cb) * 2 == want
