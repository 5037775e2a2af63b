// Spec-driven dispatch (include/ipuc.h: ipuc_query_abi, ipuc_launch).
//
// The reference plans every tile-kernel call from a TileKernelSpec
// (crates/ipu-codegen/src/operator.rs:57-96): tile_kernel_abi
// (crates/ipu-codegen/src/kernel.rs:1215-1382) gives the symbol family, its
// availability, the pointer-operand count and the named u32 scalars, and
// validate_kernel_run (kernel.rs:1384-1435) checks a run before it is
// materialised.  Here the same spec and scalar vector select one of the typed
// ipuc_* entry points for a GPU shard; checks and error texts follow the
// reference's KernelAbiError (kernel.rs:140-160) so a caller sees the same
// failures for the same runs.  Where the reference has no device kernel
// (Add, Cast, general Rearrange: KernelAvailability::Required) the B200
// library does, and reports IMPLEMENTED.
#include <cuda_runtime.h>

#include <cstdio>
#include <string>

#include "../../include/ipuc.h"

namespace ipuc {
void set_error(const std::string &msg);
ipuc_status fail(ipuc_status st, const std::string &msg);
}  // namespace ipuc

namespace {

using ipuc::fail;

ipuc_status requirement_mismatch() {
  return fail(IPUC_ERR_INVALID_ARGUMENT, "kernel requirements do not match the tile-kernel family");
}

void set_scalars(ipuc_kernel_abi *abi, std::initializer_list<const char *> names) {
  abi->scalar_count = 0;
  for (const char *n : names) abi->scalar_names[abi->scalar_count++] = n;
}

bool is_precision(ipuc_precision p) { return p == IPUC_F16 || p == IPUC_F32; }

bool is_unpack_source(ipuc_order o) {
  return o == IPUC_ORDER_AMP_OUTPUT || o == IPUC_ORDER_AMP_TRANSPOSED_LEFT;
}

// RearrangeTarget::codelet_index (kernel.rs:99-121): AMP-Left 0,
// AMP-TransposedRight 1, BlockMajor 2; -1 when the order has no specialised
// rearrange codelet.
int rearrange_target(ipuc_order o) {
  switch (o) {
    case IPUC_ORDER_AMP_LEFT: return 0;
    case IPUC_ORDER_AMP_TRANSPOSED_RIGHT: return 1;
    case IPUC_ORDER_BLOCK_MAJOR: return 2;
    default: return -1;
  }
}

ipuc_status query(const ipuc_kernel_spec &spec, ipuc_precision out, ipuc_kernel_abi *abi) {
  *abi = ipuc_kernel_abi{};
  abi->availability = IPUC_AVAILABILITY_IMPLEMENTED;
  if (!is_precision(out)) return requirement_mismatch();
  switch (spec.kind) {
    case IPUC_KERNEL_FILL_ZERO:
      abi->symbol = "ipuc_fill_zero";
      abi->reference_symbol = "ipu_stack_fill_zero_u64";
      abi->input_count = 0;
      set_scalars(abi, {"words_per_worker", "remainder_workers"});
      return IPUC_OK;
    case IPUC_KERNEL_GEMM: {
      const auto &g = spec.gemm;
      if (!is_precision(g.multiply) || g.mode > 1) return requirement_mismatch();
      if (g.interleaved_weights && g.multiply != IPUC_F16) return requirement_mismatch();
      const bool acc = g.mode == 1;
      if (g.multiply == IPUC_F16) {
        abi->symbol = "ipuc_gemm_f16";
        abi->reference_symbol = acc ? "ipu_stack_gemm_f16_accumulate" : "ipu_stack_gemm_f16_init";
      } else {
        abi->symbol = "ipuc_gemm_f32";
        abi->reference_symbol = acc ? "ipu_stack_gemm_f32_accumulate" : "ipu_stack_gemm_f32_init";
        // f32 operands accumulate into an f32 result only.
        if (out != IPUC_F32 || g.epilogue_gelu) abi->availability = IPUC_AVAILABILITY_REQUIRED;
      }
      abi->input_count = 2;
      set_scalars(abi, {});
      return IPUC_OK;
    }
    case IPUC_KERNEL_GELU:
      // gelu_symbol (kernel.rs:1437-1452): f16 in and out, else unsupported.
      abi->symbol = "ipuc_gelu_f16";
      abi->reference_symbol = "ipu_stack_gelu_tanh_approx_f16";
      if (out != IPUC_F16) {
        abi->reference_symbol = "ipu_stack_unsupported_gelu";
        abi->availability = IPUC_AVAILABILITY_REQUIRED;
      }
      abi->input_count = 1;
      set_scalars(abi, {"element_count"});
      return IPUC_OK;
    case IPUC_KERNEL_REDUCTION_SUM:
      if (out != IPUC_F16) return requirement_mismatch();
      abi->symbol = "ipuc_reduce_sum";
      abi->reference_symbol = "ipu_stack_reduce_sum_f16";
      abi->input_count = 2;
      set_scalars(abi, {"num_partials", "element_count"});
      return IPUC_OK;
    case IPUC_KERNEL_ADD:
      abi->symbol = "ipuc_add_f16";
      abi->reference_symbol = out == IPUC_F16 ? "ipu_stack_add_f16" : "ipu_stack_add_f32";
      if (out != IPUC_F16) abi->availability = IPUC_AVAILABILITY_REQUIRED;
      abi->input_count = 2;
      set_scalars(abi, {"element_count", "left_broadcast_stride", "right_broadcast_stride"});
      return IPUC_OK;
    case IPUC_KERNEL_FLASH_ATTENTION:
      abi->symbol = "ipuc_flash_attention_f16";
      abi->reference_symbol = "flash_attention_online_f16";
      if (spec.flash_attention.causal) abi->availability = IPUC_AVAILABILITY_REQUIRED;
      abi->input_count = 3;
      set_scalars(abi, {});
      return IPUC_OK;
    case IPUC_KERNEL_ATTENTION_SOFTMAX:
      abi->symbol = "ipuc_attention_softmax_f16";
      abi->reference_symbol = "attention_softmax_f16";
      abi->input_count = 1;
      set_scalars(abi, {});
      return IPUC_OK;
    case IPUC_KERNEL_ATTENTION_MERGE:
      abi->symbol = "ipuc_attention_merge_f16";
      abi->reference_symbol = "attention_merge_f16";
      abi->input_count = 2;
      set_scalars(abi, {"initial_block", "final_block"});
      return IPUC_OK;
    case IPUC_KERNEL_CAST: {
      const auto &c = spec.cast;
      if (!is_precision(c.from) || !is_precision(c.to)) return requirement_mismatch();
      abi->symbol = "ipuc_cast";
      abi->reference_symbol = c.from == c.to ? "ipu_stack_cast_identity"
                              : c.from == IPUC_F16 ? "ipu_stack_cast_f16_f32"
                                                   : "ipu_stack_cast_f32_f16";
      abi->input_count = 1;
      set_scalars(abi, {"element_count"});
      return IPUC_OK;
    }
    case IPUC_KERNEL_REARRANGE: {
      const auto &r = spec.rearrange;
      abi->input_count = 1;
      if (out == IPUC_F16 && is_unpack_source(r.from.order) && r.to.order == IPUC_ORDER_ROW_MAJOR) {
        abi->symbol = "ipuc_unpack_f16";
        abi->reference_symbol = "unpack_amp_f16";
        set_scalars(abi, {"matrices", "logical_rows", "physical_rows", "logical_columns", "physical_columns"});
      } else if (out == IPUC_F16 && r.from.order == IPUC_ORDER_ROW_MAJOR && rearrange_target(r.to.order) >= 0) {
        abi->symbol = "ipuc_rearrange_f16";
        abi->reference_symbol = "rearrange_f16";
        set_scalars(abi, {"logical_rows", "physical_rows", "target_order", "logical_columns", "physical_columns"});
      } else {
        abi->symbol = "ipuc_convert_order_f16";
        abi->reference_symbol = "ipu_stack_rearrange";
        if (out != IPUC_F16) abi->availability = IPUC_AVAILABILITY_REQUIRED;
        set_scalars(abi, {});
      }
      return IPUC_OK;
    }
  }
  return requirement_mismatch();
}

int64_t numel(const ipuc_tensor &t) {
  int64_t n = 1;
  for (int i = 0; i < t.rank; ++i) n *= t.dims[i];
  return n;
}

uint64_t bytes_of(const ipuc_tensor &t) { return (uint64_t)numel(t) * (t.precision == IPUC_F32 ? 4u : 2u); }

bool valid_tensor(const ipuc_tensor &t) {
  if (t.rank < 1 || t.rank > 4 || !is_precision(t.precision)) return false;
  for (int i = 0; i < t.rank; ++i)
    if (t.dims[i] < 0) return false;
  return true;
}

ipuc_status count_error(const char *symbol, uint64_t count, uint32_t divisor) {
  char buf[192];
  std::snprintf(buf, sizeof buf, "kernel %s requires an element count divisible by %u, got %llu", symbol, divisor,
                (unsigned long long)count);
  return fail(IPUC_ERR_INVALID_ARGUMENT, buf);
}

ipuc_status scalar_error(const char *name, uint64_t expected, uint32_t got) {
  char buf[192];
  std::snprintf(buf, sizeof buf, "scalar %s is %u, the run implies %llu", name, got, (unsigned long long)expected);
  return fail(IPUC_ERR_INVALID_ARGUMENT, buf);
}

// Matrix view of a rank-2/3 tensor: [matrices, rows, cols].
void matrix_dims(const ipuc_tensor &t, int64_t &matrices, int64_t &rows, int64_t &cols) {
  cols = t.dims[t.rank - 1];
  rows = t.rank >= 2 ? t.dims[t.rank - 2] : 1;
  matrices = 1;
  for (int i = 0; i + 2 < t.rank; ++i) matrices *= t.dims[i];
}

ipuc_status launch(const ipuc_kernel_spec &spec, const ipuc_tensor &out, const ipuc_tensor *in, int32_t n_in,
                   const uint32_t *sc, int32_t n_sc, void *workspace, uint64_t workspace_bytes, ipuc_stream stream) {
  if (!valid_tensor(out)) return fail(IPUC_ERR_INVALID_ARGUMENT, "output tensor: rank 1..4, non-negative dims");
  ipuc_kernel_abi abi;
  ipuc_status st = query(spec, out.precision, &abi);
  if (st != IPUC_OK) return st;
  if (n_in != abi.input_count) {
    char buf[128];
    std::snprintf(buf, sizeof buf, "kernel run has %d pointer operands, ABI requires %d", n_in, abi.input_count);
    return fail(IPUC_ERR_INVALID_ARGUMENT, buf);
  }
  if (n_sc != abi.scalar_count) {
    char buf[128];
    std::snprintf(buf, sizeof buf, "kernel run has %d scalar arguments, ABI requires %d", n_sc, abi.scalar_count);
    return fail(IPUC_ERR_INVALID_ARGUMENT, buf);
  }
  for (int i = 0; i < n_in; ++i) {
    if (!valid_tensor(in[i])) {
      char buf[96];
      std::snprintf(buf, sizeof buf, "input tensor %d: rank 1..4, non-negative dims", i);
      return fail(IPUC_ERR_INVALID_ARGUMENT, buf);
    }
  }
  if (abi.availability == IPUC_AVAILABILITY_REQUIRED)
    return fail(IPUC_ERR_UNSUPPORTED, std::string("kernel ") + abi.reference_symbol + " has no device implementation");
  const int64_t count = numel(out);

  switch (spec.kind) {
    case IPUC_KERNEL_FILL_ZERO: {
      const uint64_t bytes = bytes_of(out);
      if (bytes % 8) return count_error(abi.reference_symbol, bytes, 8);
      // words_per_worker / remainder_workers split the u64 words over the
      // IPU's six workers (kernel.rs:1172-1173); one GPU launch covers all.
      const uint64_t words = bytes / 8;
      if (sc[0] != words / 6) return scalar_error("words_per_worker", words / 6, sc[0]);
      if (sc[1] != words % 6) return scalar_error("remainder_workers", words % 6, sc[1]);
      return ipuc_fill_zero(out.data, bytes, stream);
    }
    case IPUC_KERNEL_GEMM: {
      const auto &g = spec.gemm;
      const ipuc_tensor &A = in[0], &B = in[1];
      if (A.precision != g.multiply || B.precision != g.multiply)
        return fail(IPUC_ERR_INVALID_ARGUMENT, "gemm: operand precision differs from the spec's multiply precision");
      const int rank = out.rank;
      if (rank < 2 || rank > 3 || A.rank != rank || B.rank != rank)
        return fail(IPUC_ERR_INVALID_ARGUMENT, "gemm: operands must be matrices [m,k] [k,n] -> [m,n] (or batched)");
      const int64_t batch = rank == 3 ? out.dims[0] : 1;
      if (rank == 3 && (A.dims[0] != batch || B.dims[0] != batch))
        return fail(IPUC_ERR_INVALID_ARGUMENT, "gemm: batch extents differ");
      const int64_t m = A.dims[rank - 2], k = A.dims[rank - 1];
      const int64_t n = g.b_transposed ? B.dims[rank - 2] : B.dims[rank - 1];
      const int64_t kb = g.b_transposed ? B.dims[rank - 1] : B.dims[rank - 2];
      if (kb != k || out.dims[rank - 2] != m || out.dims[rank - 1] != n)
        return fail(IPUC_ERR_INVALID_ARGUMENT, "gemm: operand shapes do not chain");
      uint32_t flags = (g.mode == 1 ? (uint32_t)IPUC_GEMM_ACCUMULATE : 0u) |
                       (g.b_transposed ? (uint32_t)IPUC_GEMM_B_TRANSPOSED : 0u) |
                       (g.epilogue_gelu ? (uint32_t)IPUC_GEMM_EPILOGUE_GELU : 0u);
      const int64_t ldb = g.b_transposed ? k : n;
      if (g.multiply == IPUC_F16) {
        if (out.precision == IPUC_F32) flags |= IPUC_GEMM_OUT_F32;
        if (rank == 3)
          return ipuc_gemm_f16_batched(out.data, A.data, B.data, batch, m, n, k, k, ldb, n, m * k, n * k, m * n,
                                       flags, stream);
        return ipuc_gemm_f16(out.data, A.data, B.data, m, n, k, k, ldb, n, flags, stream);
      }
      if (rank == 3) return fail(IPUC_ERR_UNSUPPORTED, "gemm: batched f32 GEMM is not supported");
      return ipuc_gemm_f32(static_cast<float *>(out.data), static_cast<const float *>(A.data),
                           static_cast<const float *>(B.data), m, n, k, k, ldb, n, flags, workspace, workspace_bytes,
                           stream);
    }
    case IPUC_KERNEL_GELU: {
      if (in[0].precision != IPUC_F16 || numel(in[0]) != count)
        return fail(IPUC_ERR_INVALID_ARGUMENT, "gelu: input must be f16 with the output's element count");
      if (count % 2) return count_error(abi.reference_symbol, (uint64_t)count, 2);
      if (sc[0] != (uint64_t)count) return scalar_error("element_count", (uint64_t)count, sc[0]);
      return ipuc_gelu_f16(out.data, in[0].data, (uint64_t)count, stream);
    }
    case IPUC_KERNEL_REDUCTION_SUM: {
      const uint32_t partials = spec.reduction_sum.partials;
      if (partials < 2 || count % 8) return count_error(abi.reference_symbol, (uint64_t)count, 8);
      if (sc[0] != partials - 1) return scalar_error("num_partials", partials - 1, sc[0]);
      if (sc[1] != (uint64_t)count) return scalar_error("element_count", (uint64_t)count, sc[1]);
      if (in[0].precision != in[1].precision || numel(in[0]) != count ||
          numel(in[1]) != (int64_t)(partials - 1) * count)
        return fail(IPUC_ERR_INVALID_ARGUMENT,
                    "reduce_sum: inputs are initial[count] and remote[(partials-1) * count] of one precision");
      return ipuc_reduce_sum(out.data, in[0].data, in[1].data, partials - 1, (uint64_t)count, in[0].precision,
                             stream);
    }
    case IPUC_KERNEL_ADD: {
      if (in[0].precision != IPUC_F16 || in[1].precision != IPUC_F16)
        return fail(IPUC_ERR_INVALID_ARGUMENT, "add: f16 operands");
      if (sc[0] != (uint64_t)count) return scalar_error("element_count", (uint64_t)count, sc[0]);
      const uint64_t lp = sc[1], rp = sc[2];
      if ((uint64_t)numel(in[0]) != (lp ? lp : (uint64_t)count) ||
          (uint64_t)numel(in[1]) != (rp ? rp : (uint64_t)count))
        return fail(IPUC_ERR_INVALID_ARGUMENT, "add: operand sizes disagree with the broadcast strides");
      return ipuc_add_f16(out.data, in[0].data, in[1].data, (uint64_t)count, lp, rp, stream);
    }
    case IPUC_KERNEL_FLASH_ATTENTION: {
      const ipuc_tensor &Q = in[0], &K = in[1], &V = in[2];
      if (Q.precision != IPUC_F16 || K.precision != IPUC_F16 || V.precision != IPUC_F16)
        return fail(IPUC_ERR_INVALID_ARGUMENT, "flash_attention: f16 query, key and value");
      int64_t mq, sq, d, mk, sk, dk, mv, sv, dv, mo, so, dout;
      matrix_dims(Q, mq, sq, d);
      matrix_dims(K, mk, sk, dk);
      matrix_dims(V, mv, sv, dv);
      matrix_dims(out, mo, so, dout);
      if (mk != mq || mv != mq || mo != mq || dk != d || sv != sk || so != sq || dout != dv)
        return fail(IPUC_ERR_INVALID_ARGUMENT, "flash_attention: Q[M,Sq,D] K[M,Sk,D] V[M,Sk,Dv] -> O[M,Sq,Dv]");
      if (dv != d) return fail(IPUC_ERR_UNSUPPORTED, "flash_attention: value width must equal the query width");
      return ipuc_flash_attention_f16(out.data, out.precision, Q.data, K.data, V.data, mq, sq, sk, d,
                                      spec.flash_attention.scale, stream);
    }
    case IPUC_KERNEL_ATTENTION_SOFTMAX: {
      const auto &a = spec.attention_softmax;
      if (in[0].precision != IPUC_F16 || out.precision != IPUC_F16)
        return fail(IPUC_ERR_INVALID_ARGUMENT, "attention_softmax: f16 scores and weights");
      if (a.padded_key_columns == 0 || numel(in[0]) % a.padded_key_columns)
        return fail(IPUC_ERR_INVALID_ARGUMENT, "attention_softmax: scores are [padded_key_columns/16][rows][16]");
      const int64_t rows = numel(in[0]) / a.padded_key_columns;
      // weights (rows x padded_key_columns f16) followed by 2*rows f32 state.
      if (count < rows * (int64_t)a.padded_key_columns + 4 * rows)
        return fail(IPUC_ERR_INVALID_ARGUMENT, "attention_softmax: output too small for weights and row state");
      return ipuc_attention_softmax_f16(out.data, in[0].data, rows, a.key_columns, a.padded_key_columns,
                                        a.head_dimension, stream);
    }
    case IPUC_KERNEL_ATTENTION_MERGE: {
      const auto &a = spec.attention_merge;
      if (sc[0] != a.initial) return scalar_error("initial_block", a.initial, sc[0]);
      if (sc[1] != a.final_block) return scalar_error("final_block", a.final_block, sc[1]);
      if (out.precision != IPUC_F32 || in[0].precision != IPUC_F16 || in[1].precision != IPUC_F16)
        return fail(IPUC_ERR_INVALID_ARGUMENT, "attention_merge: f32 accumulator, f16 block and weights");
      if (a.padded_value_dimension == 0 || count % a.padded_value_dimension)
        return fail(IPUC_ERR_INVALID_ARGUMENT, "attention_merge: accumulator is [rows][padded_value_dimension]");
      const int64_t rows = count / a.padded_value_dimension;
      const int64_t weights = rows * (int64_t)a.key_block_columns;
      if (numel(in[1]) < weights + 4 * rows)
        return fail(IPUC_ERR_INVALID_ARGUMENT, "attention_merge: weights buffer lacks the softmax row state");
      const float *state = reinterpret_cast<const float *>(static_cast<const uint16_t *>(in[1].data) + weights);
      return ipuc_attention_merge_f16(static_cast<float *>(out.data), in[0].data, state, rows, a.value_dimension,
                                      a.padded_value_dimension, (int)a.initial, (int)a.final_block, stream);
    }
    case IPUC_KERNEL_CAST: {
      if (in[0].precision != spec.cast.from || out.precision != spec.cast.to || numel(in[0]) != count)
        return fail(IPUC_ERR_INVALID_ARGUMENT, "cast: operand precisions or counts differ from the spec");
      if (sc[0] != (uint64_t)count) return scalar_error("element_count", (uint64_t)count, sc[0]);
      return ipuc_cast(out.data, spec.cast.to, in[0].data, spec.cast.from, (uint64_t)count, stream);
    }
    case IPUC_KERNEL_REARRANGE: {
      const auto &r = spec.rearrange;
      if (in[0].precision != IPUC_F16) return fail(IPUC_ERR_INVALID_ARGUMENT, "rearrange: f16 operands");
      if (is_unpack_source(r.from.order) && r.to.order == IPUC_ORDER_ROW_MAJOR) {
        const int64_t matrices = sc[0], lr = sc[1], pr = sc[2], lc = sc[3], pc = sc[4];
        if (count != matrices * pr * pc || numel(in[0]) != matrices * pr * pc)
          return fail(IPUC_ERR_INVALID_ARGUMENT, "unpack: tensors disagree with matrices x physical extents");
        return ipuc_unpack_f16(out.data, in[0].data, r.from.order == IPUC_ORDER_AMP_OUTPUT ? 0 : 1, matrices, lr,
                               pr, lc, pc, stream);
      }
      const int target = rearrange_target(r.to.order);
      if (r.from.order == IPUC_ORDER_ROW_MAJOR && target >= 0) {
        const int64_t lr = sc[0], pr = sc[1], lc = sc[3], pc = sc[4];
        if (sc[2] != (uint32_t)target) return scalar_error("target_order", (uint64_t)target, sc[2]);
        if (lr <= 0 || lc <= 0 || numel(in[0]) % (lr * lc))
          return fail(IPUC_ERR_INVALID_ARGUMENT, "rearrange: input is matrices x logical_rows x logical_columns");
        const int64_t matrices = numel(in[0]) / (lr * lc);
        if (count != matrices * pr * pc)
          return fail(IPUC_ERR_INVALID_ARGUMENT, "rearrange: output is matrices x physical extents");
        const int64_t rb = target == 2 ? r.to.row_block : 64, cb = target == 2 ? r.to.column_block : 16;
        return ipuc_rearrange_f16(out.data, in[0].data, matrices, lr, pr, target, lc, pc, rb, cb, stream);
      }
      int64_t matrices, rows, cols;
      matrix_dims(out, matrices, rows, cols);
      if (numel(in[0]) != count) return fail(IPUC_ERR_INVALID_ARGUMENT, "rearrange: element counts differ");
      const bool from_bm = r.from.order == IPUC_ORDER_BLOCK_MAJOR || r.from.order == IPUC_ORDER_BLOCK_MAJOR_TRANSPOSED;
      const bool to_bm = r.to.order == IPUC_ORDER_BLOCK_MAJOR || r.to.order == IPUC_ORDER_BLOCK_MAJOR_TRANSPOSED;
      if (from_bm && to_bm && (r.from.row_block != r.to.row_block || r.from.column_block != r.to.column_block))
        return fail(IPUC_ERR_UNSUPPORTED, "rearrange: block-major to block-major with different blocks");
      const int64_t rb = to_bm ? r.to.row_block : from_bm ? r.from.row_block : 64;
      const int64_t cb = to_bm ? r.to.column_block : from_bm ? r.from.column_block : 16;
      return ipuc_convert_order_f16(out.data, r.to.order, in[0].data, r.from.order, matrices, rows, cols, rb, cb,
                                    stream);
    }
  }
  return requirement_mismatch();
}

}  // namespace

extern "C" ipuc_status ipuc_query_abi(const ipuc_kernel_spec *spec, ipuc_precision output_precision,
                                      ipuc_kernel_abi *abi) {
  if (!spec || !abi) return fail(IPUC_ERR_INVALID_ARGUMENT, "query_abi: null pointer");
  return query(*spec, output_precision, abi);
}

extern "C" ipuc_status ipuc_launch(const ipuc_kernel_spec *spec, const ipuc_tensor *output, const ipuc_tensor *inputs,
                                   int32_t input_count, const uint32_t *scalars, int32_t scalar_count,
                                   void *workspace, uint64_t workspace_bytes, ipuc_stream stream) {
  if (!spec || !output) return fail(IPUC_ERR_INVALID_ARGUMENT, "launch: null spec or output");
  if (input_count < 0 || (input_count > 0 && !inputs) || scalar_count < 0 || (scalar_count > 0 && !scalars))
    return fail(IPUC_ERR_INVALID_ARGUMENT, "launch: bad operand or scalar array");
  return launch(*spec, *output, inputs, input_count, scalars, scalar_count, workspace, workspace_bytes, stream);
}
