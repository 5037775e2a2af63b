"""Spec-driven dispatch on CPU: ipuc_query_abi reproduces the reference's
tile_kernel_abi table (crates/ipu-codegen/src/kernel.rs:1215-1382) and
ipuc_launch applies validate_kernel_run (kernel.rs:1384-1435) before any
device work, so every case here runs without a GPU."""
import ctypes

import pytest

import ipuc

T = ipuc.TileKernelSpec
FAKE = 0x10000  # never dereferenced: every case below fails validation first


def fake(shape, precision=ipuc.F16):
    dims = (ctypes.c_int64 * 4)(*(list(shape) + [0] * (4 - len(shape))))
    return ipuc.Tensor(FAKE, precision, len(shape), dims)


# (spec, output precision) -> (input count, scalar names) as kernel.rs lists them.
ABI_TABLE = [
    ("fill_zero", T.fill_zero(), ipuc.F16, 0, ["words_per_worker", "remainder_workers"]),       # :1224-1229
    ("gemm f16", T.gemm(), ipuc.F16, 2, []),                                                     # :1230-1250
    ("gemm f32", T.gemm(multiply=ipuc.F32), ipuc.F32, 2, []),
    ("gelu", T.gelu(), ipuc.F16, 1, ["element_count"]),                                          # :1251-1263
    ("reduction_sum", T.reduction_sum(4), ipuc.F16, 2, ["num_partials", "element_count"]),       # :1264-1274
    ("add", T.add(), ipuc.F16, 2, ["element_count", "left_broadcast_stride", "right_broadcast_stride"]),  # :1275-1287
    ("flash_attention", T.flash_attention(), ipuc.F32, 3, []),                                   # :1288-1300
    ("attention_softmax", T.attention_softmax(64, 50, 64), ipuc.F16, 1, []),                     # :1301-1306
    ("attention_merge", T.attention_merge(64, 80, 64, True, False), ipuc.F32, 2,
     ["initial_block", "final_block"]),                                                          # :1307-1312
    ("cast", T.cast(ipuc.F16, ipuc.F32), ipuc.F32, 1, ["element_count"]),                        # :1313-1318
    ("unpack", T.rearrange(ipuc.AMP_OUTPUT, ipuc.ROW_MAJOR), ipuc.F16, 1,
     ["matrices", "logical_rows", "physical_rows", "logical_columns", "physical_columns"]),      # :1319-1339
    ("rearrange", T.rearrange(ipuc.ROW_MAJOR, (ipuc.BLOCK_MAJOR, 64, 16)), ipuc.F16, 1,
     ["logical_rows", "physical_rows", "target_order", "logical_columns", "physical_columns"]),  # :1340-1364
    ("generic rearrange", T.rearrange(ipuc.AMP_LEFT, ipuc.AMP_OUTPUT), ipuc.F16, 1, []),         # :1365-1370
]


@pytest.mark.parametrize("name,spec,prec,n_in,scalars", ABI_TABLE, ids=[r[0] for r in ABI_TABLE])
def test_abi_matches_reference_table(name, spec, prec, n_in, scalars):
    abi = ipuc.query_abi(spec, prec)
    assert abi["input_count"] == n_in
    assert abi["scalar_names"] == scalars
    assert abi["availability"] == ipuc.AVAILABILITY_IMPLEMENTED
    assert abi["symbol"].startswith("ipuc_")


def test_reference_symbols():
    assert ipuc.query_abi(T.fill_zero())["reference_symbol"] == "ipu_stack_fill_zero_u64"
    assert ipuc.query_abi(T.reduction_sum(2))["reference_symbol"] == "ipu_stack_reduce_sum_f16"
    assert ipuc.query_abi(T.gelu())["reference_symbol"] == "ipu_stack_gelu_tanh_approx_f16"
    assert ipuc.query_abi(T.gemm(mode="accumulate"))["reference_symbol"] == "ipu_stack_gemm_f16_accumulate"
    assert ipuc.query_abi(T.cast(ipuc.F32, ipuc.F16))["reference_symbol"] == "ipu_stack_cast_f32_f16"
    assert ipuc.query_abi(T.cast(ipuc.F16, ipuc.F16))["reference_symbol"] == "ipu_stack_cast_identity"


def test_requirement_mismatch_and_availability():
    # Interleaved weights need F16 multiply (kernel.rs:1240-1242).
    with pytest.raises(ipuc.IpucError) as e:
        ipuc.query_abi(T.gemm(multiply=ipuc.F32, interleaved_weights=True), ipuc.F32)
    assert e.value.status == ipuc.ERR_INVALID_ARGUMENT
    assert "requirements do not match" in e.value.message
    # ReductionSum output must be F16 (kernel.rs:1265-1267).
    with pytest.raises(ipuc.IpucError):
        ipuc.query_abi(T.reduction_sum(2), ipuc.F32)
    # GELU with a non-f16 output: the reference's unsupported symbol, Required.
    abi = ipuc.query_abi(T.gelu(), ipuc.F32)
    assert abi["availability"] == ipuc.AVAILABILITY_REQUIRED
    assert abi["reference_symbol"] == "ipu_stack_unsupported_gelu"
    # Causal attention is rejected (operator.rs:997).
    assert ipuc.query_abi(T.flash_attention(causal=True), ipuc.F16)["availability"] == ipuc.AVAILABILITY_REQUIRED


def launch_error(spec, out, inputs=(), scalars=()):
    with pytest.raises(ipuc.IpucError) as e:
        ipuc.launch(spec, out, inputs, scalars)
    return e.value


def test_pointer_arity():
    err = launch_error(T.gelu(), fake([8]), [], [8])
    assert err.status == ipuc.ERR_INVALID_ARGUMENT
    assert err.message == "kernel run has 0 pointer operands, ABI requires 1"
    err = launch_error(T.gemm(), fake([4, 4]), [fake([4, 8])], [])
    assert err.message == "kernel run has 1 pointer operands, ABI requires 2"


def test_scalar_arity_and_values():
    err = launch_error(T.gelu(), fake([8]), [fake([8])], [])
    assert "scalar arguments, ABI requires 1" in err.message
    err = launch_error(T.gelu(), fake([8]), [fake([8])], [6])
    assert err.message == "scalar element_count is 6, the run implies 8"
    err = launch_error(T.attention_merge(64, 80, 64, True, False), fake([4, 80], ipuc.F32),
                       [fake([5, 16, 4, 16]), fake([4 * 64 + 16])], [0, 0])
    assert "initial_block" in err.message


def test_count_divisibility_messages():
    # GELU count even (kernel.rs:1400-1413).
    err = launch_error(T.gelu(), fake([7]), [fake([7])], [7])
    assert err.message == "kernel ipu_stack_gelu_tanh_approx_f16 requires an element count divisible by 2, got 7"
    # ReductionSum: partials >= 2 and count % 8 (kernel.rs:1414-1423).
    err = launch_error(T.reduction_sum(3), fake([12]), [fake([12]), fake([24])], [2, 12])
    assert err.message == "kernel ipu_stack_reduce_sum_f16 requires an element count divisible by 8, got 12"
    err = launch_error(T.reduction_sum(1), fake([16]), [fake([16]), fake([0])], [0, 16])
    assert "divisible by 8" in err.message
    # FillZero bytes % 8 (kernel.rs:1425-1434): 5 f16 = 10 bytes.
    err = launch_error(T.fill_zero(), fake([5]), [], [0, 1])
    assert err.message == "kernel ipu_stack_fill_zero_u64 requires an element count divisible by 8, got 10"
    # words_per_worker / remainder_workers must describe the output (kernel.rs:1172-1173).
    err = launch_error(T.fill_zero(), fake([64]), [], [3, 0])
    assert err.message == "scalar words_per_worker is 3, the run implies 2"


def test_unsupported_is_reported_not_launched():
    err = launch_error(T.flash_attention(causal=True), fake([1, 4, 64]),
                       [fake([1, 4, 64]), fake([1, 4, 64]), fake([1, 4, 64])])
    assert err.status == ipuc.ERR_UNSUPPORTED
    assert "no device implementation" in err.message
    err = launch_error(T.add(), fake([8], ipuc.F32), [fake([8], ipuc.F32), fake([8], ipuc.F32)], [8, 0, 0])
    assert err.status == ipuc.ERR_UNSUPPORTED


def test_shape_checks():
    err = launch_error(T.gemm(), fake([4, 4]), [fake([4, 8]), fake([16, 4])])
    assert "do not chain" in err.message
    err = launch_error(T.flash_attention(), fake([2, 8, 64]), [fake([2, 8, 64]), fake([2, 9, 64]), fake([2, 8, 64])])
    assert "Q[M,Sq,D]" in err.message
    err = launch_error(T.rearrange(ipuc.ROW_MAJOR, ipuc.AMP_LEFT), fake([64, 16]), [fake([4, 16])], [4, 64, 1, 16, 16])
    assert err.message == "scalar target_order is 1, the run implies 0"
