/*
 * ipuc.h — C ABI of the B200 operator-catalog backend (libipuc.so).
 *
 * One extern "C" entry per reference TileKernelSpec family
 * (crates/ipu-codegen/src/operator.rs:57-96).  Each entry replaces the
 * supervisor-ABI tile kernel the reference's ipu-codegen calls per tile
 * (crates/ipu-codegen/src/kernel.rs:1215-1382: m2 output, m3.. inputs, then
 * scalars), with device pointers in place of tile SRAM addresses and one GPU
 * shard in place of one tile's work list.
 *
 * Conventions
 *  - Every pointer is a device pointer owned by the caller.  The library never
 *    allocates device memory on these paths (reference: kernels never
 *    allocate; crates/ipu-codegen/src/operator.rs:533-537 for aliasing).
 *  - Calls are stream-ordered on `stream` (a cudaStream_t; NULL = legacy
 *    default stream) and return before the kernel finishes.
 *  - Arguments are validated on the host before any launch, mirroring
 *    validate_kernel_run (kernel.rs:1384-1435).  On failure nothing is
 *    launched, an ipuc_status error is returned and
 *    ipuc_last_error_string() describes it (thread-local).
 *  - f16 = IEEE binary16, f32 = IEEE binary32.  "row-major" matrices are dense
 *    with the stated leading dimension in elements.
 */
#ifndef IPUC_H
#define IPUC_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *ipuc_stream; /* == cudaStream_t */

/* Host-side Result<_, KernelAbiError | KernelMaterializationError>
 * (kernel.rs:140-176) becomes a status code. */
typedef enum {
  IPUC_OK = 0,
  IPUC_ERR_INVALID_ARGUMENT = 1, /* shape/arity/count checks (KernelAbiError::*) */
  IPUC_ERR_UNSUPPORTED = 2,      /* KernelAvailability::Required / unsupported geometry */
  IPUC_ERR_ALIGNMENT = 3,        /* pointer or leading-dimension alignment */
  IPUC_ERR_CUDA = 4,             /* a CUDA runtime/driver call failed */
  IPUC_ERR_NCCL = 5,             /* a collective failed */
  IPUC_ERR_DEVICE_TIMEOUT = 6    /* a bounded device wait gave up (error word set) */
} ipuc_status;

/* Precision (operator.rs Precision, F16/F32 only). */
typedef enum { IPUC_F16 = 0, IPUC_F32 = 1 } ipuc_precision;

/* ElementOrder (crates/ipu-codegen/src/layout.rs:7-45). */
typedef enum {
  IPUC_ORDER_ROW_MAJOR = 0,
  IPUC_ORDER_AMP_LEFT = 1,
  IPUC_ORDER_AMP_TRANSPOSED_LEFT = 2,
  IPUC_ORDER_AMP_TRANSPOSED_RIGHT = 3,
  IPUC_ORDER_AMP_OUTPUT = 4,
  IPUC_ORDER_AMP_TRANSPOSED_OUTPUT = 5,
  IPUC_ORDER_BLOCK_MAJOR = 6,           /* BlockMajorOrder::Matrix{row_block, column_block} */
  IPUC_ORDER_BLOCK_MAJOR_TRANSPOSED = 7 /* BlockMajorOrder::TransposedMatrix{..} */
} ipuc_order;

/* Library / device information ------------------------------------------ */
const char *ipuc_version(void);
const char *ipuc_status_string(ipuc_status status);
/* Thread-local description of the last error returned on this thread. */
const char *ipuc_last_error_string(void);
/* Reads and clears the device error word set by bounded waits inside kernels
 * on the current device (synchronises `stream`).  Reference: the device
 * "fails" only by host-side timeout (device/static_runtime.S:487-488). */
ipuc_status ipuc_device_status(ipuc_stream stream);

/* Exercises the bounded-wait failure path on the device: a kernel waits on an
 * mbarrier that is never signalled, gives up after limit_ns (<= 10 s), sets
 * the device error word and exits.  A following ipuc_device_status() returns
 * IPUC_ERR_DEVICE_TIMEOUT.  Nothing faults or traps. */
ipuc_status ipuc_selftest_bounded_wait(uint64_t limit_ns, ipuc_stream stream);

/* FillZero: device/static_runtime.S:269-316, ABI kernel.rs:1224-1229.
 * bytes % 8 == 0 (validate_kernel_run, kernel.rs:1425-1434). */
ipuc_status ipuc_fill_zero(void *out, uint64_t bytes, ipuc_stream stream);

/* Gemm ------------------------------------------------------------------- */
/* Replaces ipu_stack_gemm_f16_{init,accumulate}_* (device/gemm_f16_amp.S:
 * 186-440; spec TileKernelSpec::Gemm, operator.rs:59-66; expansion
 * lower_blocked_gemm, low.rs:3465-3560).
 *   C[m x n] = epilogue(A[m x k] . B[k x n] (+ C if IPUC_GEMM_ACCUMULATE))
 * A row-major (lda >= k).  B row-major [k x n] (ldb >= n), or with
 * IPUC_GEMM_B_TRANSPOSED stored as [n x k] (ldb >= k).  C row-major (ldc >= n),
 * f16, or f32 with IPUC_GEMM_OUT_F32 (split-K partials).  fp32 accumulation
 * over the whole k in tensor memory.  Requirements: 16-byte aligned
 * pointers; k, lda and ldb multiples of 8 elements (16-byte TMA rows).  Any
 * m, n >= 0 (tails are masked); stores are vectorised when ldc % 8 == 0.
 * Epilogue order: acc (+C) -> round to C's precision -> GELU -> store.
 * mode Accumulate == IPUC_GEMM_ACCUMULATE (GemmKernelMode, operator.rs:98-102). */
enum {
  IPUC_GEMM_ACCUMULATE = 1u << 0,
  IPUC_GEMM_B_TRANSPOSED = 1u << 1,
  IPUC_GEMM_OUT_F32 = 1u << 2,
  IPUC_GEMM_EPILOGUE_GELU = 1u << 3,
  /* ipuc_gemm_f32 only: the classic three-pass TF32 split (hi = tf32(x),
   * lo = tf32(x - hi), kind::tf32 MMAs) instead of the default scaled f16
   * split; same accuracy class, about 0.6x the throughput. */
  IPUC_GEMM_F32_SPLIT_TF32 = 1u << 4,
  /* ipuc_gemm_f16: A stored transposed, as [k x m] (lda >= m, m a multiple
   * of 8): GemmOptions::transpose_left (graph.rs:126-129).  The tensor cores
   * read it M-major straight from memory (no transpose copy). */
  IPUC_GEMM_A_TRANSPOSED = 1u << 5
};
ipuc_status ipuc_gemm_f16(void *c, const void *a, const void *b, int64_t m, int64_t n, int64_t k,
                          int64_t lda, int64_t ldb, int64_t ldc, uint32_t flags,
                          ipuc_stream stream);

/* GEMM with an epilogue addend (the graph's Gemm -> Add, the residual add):
 *   C[m x n] = epilogue(A . B + D)
 * with D [m x n] at leading dimension ld_addend, of C's precision (f16, or f32
 * with IPUC_GEMM_OUT_F32); D may equal C.  Epilogue order: acc + D -> round
 * to C's precision -> GELU (with IPUC_GEMM_EPILOGUE_GELU) -> store.  Otherwise
 * as ipuc_gemm_f16 (IPUC_GEMM_ACCUMULATE is implied). */
ipuc_status ipuc_gemm_f16_addend(void *c, const void *a, const void *b, int64_t m, int64_t n, int64_t k,
                                 int64_t lda, int64_t ldb, int64_t ldc, uint32_t flags, const void *addend,
                                 int64_t ld_addend, ipuc_stream stream);

/* Batched form: `batch` independent GEMMs at the given element strides
 * (batched-gemm-smoke, crates/ipu-tests/src/main.rs:201-220).  A stride of 0
 * for A or B shares that operand across the batch (numpy broadcasting of a
 * batch dimension); C's stride must be nonzero. */
ipuc_status ipuc_gemm_f16_batched(void *c, const void *a, const void *b, int64_t batch,
                                  int64_t m, int64_t n, int64_t k, int64_t lda, int64_t ldb,
                                  int64_t ldc, int64_t stride_a, int64_t stride_b,
                                  int64_t stride_c, uint32_t flags, ipuc_stream stream);

/* Replaces ipu_stack_gemm_f32_{init,accumulate}_* (device/gemm_f32_64_amp.S:
 * 129-385).  f32 in, f32 out, C (+)= A.B on the tensor cores with a
 * three-pass f16 split (each row of A and column of B scaled by a power of
 * two, then x = hi + lo in f16; hi.hi + hi.lo + lo.hi in fp32).  Elements
 * more than 2^17 below their row's or column's largest magnitude keep fewer
 * bits in that split; every C element whose value those elements (or an
 * inf/NaN input) could have moved beyond 2^-23 of itself is recomputed with
 * fp32 FMAs instead, so results hold an fp32 tolerance element by element
 * for any input, and non-finite inputs give the IEEE result per element.
 * (The IPUC_GEMM_F32_SPLIT_TF32 split keeps 22 bits per element by itself,
 * but an inf/NaN input there turns its whole row/column of C NaN.)
 * workspace: caller-provided device scratch of ipuc_gemm_f32_workspace_bytes()
 * bytes (the hi/lo split operands), 256-byte aligned.  Requirements:
 * 16-byte aligned pointers; k, n, lda and ldb multiples of 4 elements.
 * Flags: IPUC_GEMM_ACCUMULATE, IPUC_GEMM_B_TRANSPOSED and
 * IPUC_GEMM_F32_SPLIT_TF32 (the unscaled 3xTF32 split instead). */
uint64_t ipuc_gemm_f32_workspace_bytes(int64_t m, int64_t n, int64_t k);
ipuc_status ipuc_gemm_f32(float *c, const float *a, const float *b, int64_t m, int64_t n, int64_t k,
                          int64_t lda, int64_t ldb, int64_t ldc, uint32_t flags, void *workspace,
                          uint64_t workspace_bytes, ipuc_stream stream);

/* Allocation-free FP32 GEMM.  No counterpart in the reference: its tile
 * kernels never need scratch, while ipuc_gemm_f32 above takes a caller-provided
 * workspace for the f16 hi/lo split planes.  This entry point is for callers
 * that cannot allocate device memory when they issue the GEMM (a plug-in whose
 * host framework owns the device allocator and forbids library allocations, a
 * host callback, or a real-time path whose memory budget is fixed up front):
 * the split planes live in a fixed 64 MiB file-scope device array of
 * libipuc.so instead.  Arguments, flags and results are exactly those
 * of ipuc_gemm_f32 without the workspace pair.
 *  - Limit: 4 * (m + n) * kp + 12 * (m + n) + 4 * m * ceil(n / 32) bytes
 *    (kp = k rounded up to 8, each of the eleven arrays rounded up to 256
 *    bytes) <= 64 MiB (e.g. m = n = k = 2864); with
 *    IPUC_GEMM_F32_SPLIT_TF32, 8 * (m + n) * k bytes
 *    (e.g. m = n = k = 2048); larger
 *    shapes return IPUC_ERR_INVALID_ARGUMENT and launch nothing.
 *  - Allocates nothing: no cudaMalloc/cudaFree and no allocating library call.
 *    The array exists on every GPU that loads the library, until process exit.
 *  - The first call on each device resolves the array's device address with
 *    cudaGetSymbolAddress (with that device current); make that first call
 *    before any stream capture on the device.  The address is cached with the
 *    context it was resolved in: after cudaDeviceReset, or when the caller
 *    makes another context current on the device, the next call resolves it
 *    again (so that call, too, belongs before any capture).
 *  - Every call shares the one array: calls that overlap on the GPU (two
 *    streams, or concurrent host threads) race.  Nothing in it needs clearing
 *    between calls. */
ipuc_status ipuc_gemm_f32_noalloc(float *c, const float *a, const float *b, int64_t m, int64_t n, int64_t k,
                                  int64_t lda, int64_t ldb, int64_t ldc, uint32_t flags, ipuc_stream stream);

/* Gelu: ipu_stack_gelu_tanh_approx_f16 (device/gelu_f16.S:7-148; ABI
 * kernel.rs:1251-1263; element_count even, kernel.rs:1400-1413).
 * out may equal in. */
ipuc_status ipuc_gelu_f16(void *out, const void *in, uint64_t element_count, ipuc_stream stream);

/* ReductionSum: ipu_stack_reduce_sum_f16 (device/reduce_add_f16.S:7-72; ABI
 * kernel.rs:1264-1274, scalars num_partials = partials - 1 and element_count;
 * partials >= 2 and element_count % 8 == 0, kernel.rs:1414-1423).
 *   out = initial + sum_{p < num_partials} remote[p * element_count + i]
 * in_precision F16 (the reference's kernel) or F32 (split-K fp32 partials);
 * out is f16.  fp32 accumulation, one rounding. */
ipuc_status ipuc_reduce_sum(void *out, const void *initial, const void *remote, uint32_t num_partials,
                            uint64_t element_count, ipuc_precision in_precision, ipuc_stream stream);

/* Add (kernel.rs:1275-1287, KernelAvailability::Required in the reference):
 * out[i] = left[i % lp] + right[i % rp] with lp/rp = 0 meaning no broadcast
 * (scalars element_count, left_broadcast_stride, right_broadcast_stride). */
ipuc_status ipuc_add_f16(void *out, const void *left, const void *right, uint64_t element_count,
                         uint64_t left_broadcast_stride, uint64_t right_broadcast_stride,
                         ipuc_stream stream);

/* Cast (kernel.rs:1313-1318, Required in the reference): f16 <-> f32. */
ipuc_status ipuc_cast(void *out, ipuc_precision to, const void *in, ipuc_precision from,
                      uint64_t element_count, ipuc_stream stream);

/* FlashAttention: flash_attention_online_f16 (device/flash_attention_online_f16.
 * cpp:61-143; ABI kernel.rs:1288-1300; shape key kernel.rs:125-132).
 * Exact non-causal softmax(Q K^T * scale) V per stream:
 *   Q [matrices][query_rows][head_dim], K [matrices][key_rows][head_dim],
 *   V [matrices][key_rows][head_dim] f16 row-major; out [matrices][query_rows]
 *   [head_dim] in out_precision (F32 = the reference vertex; F16 = BASELINE).
 * scale <= 0 selects 1/sqrt(head_dim) (AttentionScale::InverseSqrtQueryWidth).
 * fp32 running max/denominator.  head_dim % 8 == 0 and head_dim <= 128
 * (smaller head dims are zero-padded to 128 inside the kernel); larger head
 * dims return IPUC_ERR_UNSUPPORTED.  Any query/key row counts >= 1. */
ipuc_status ipuc_flash_attention_f16(void *out, ipuc_precision out_precision, const void *q,
                                     const void *k, const void *v, int64_t matrices,
                                     int64_t query_rows, int64_t key_rows, int64_t head_dim,
                                     float scale, ipuc_stream stream);

/* The same attention with SplitHeads and its inverse folded into the memory
 * access (graph.rs:336-343; the copy-free strided form):
 *   Q [batch][query_rows][heads * head_dim], K and V [batch][key_rows][heads *
 *   head_dim], out [batch][query_rows][heads * head_dim]; stream (b, h) reads
 *   columns [h * head_dim, (h + 1) * head_dim) of its batch entry's rows.
 * Equals merge_heads(attention(split_heads(q), split_heads(k), split_heads(v)))
 * with no split or merge copies.  Same limits as ipuc_flash_attention_f16;
 * heads * head_dim is the row length. */
ipuc_status ipuc_flash_attention_heads_f16(void *out, ipuc_precision out_precision, const void *q,
                                           const void *k, const void *v, int64_t batch, int64_t heads,
                                           int64_t query_rows, int64_t key_rows, int64_t head_dim,
                                           float scale, ipuc_stream stream);

/* AttentionSoftmax (device/attention_softmax_f16.cpp:63-139, asm variant
 * device/attention_stages_f16.S:54-695): one key block per call.
 *   scores  f16 panels [key_block_columns/16][query_rows][16]
 *   weights f16 in the same order = exp(s*scale - max*scale), padding keys
 *           (>= key_rows) 0, followed in memory by query_rows f32 scaled maxima
 *           and query_rows f32 denominators (attention_softmax_f16.cpp:89-91).
 * scale = 1/sqrt(head_dimension).  key_block_columns % 16 == 0. */
ipuc_status ipuc_attention_softmax_f16(void *weights, const void *scores, int64_t query_rows,
                                       int64_t key_rows, int64_t key_block_columns,
                                       int64_t head_dimension, ipuc_stream stream);

/* AttentionMerge (device/attention_stages_f16.S:698-855).
 *   acc   f32 rows of padded_value_dimension; row r's {max, denominator} are
 *         stored at acc[r][value_dimension], acc[r][value_dimension+1]
 *         (so padded_value_dimension >= value_dimension + 2).
 *   block f16 PV panels [ceil(value_dimension/16)][query_rows][16].
 *   state the softmax stage's f32 maxima[query_rows] then denominators[query_rows].
 * initial: acc = block; final: acc *= 1/denominator. */
ipuc_status ipuc_attention_merge_f16(float *acc, const void *block, const float *state,
                                     int64_t query_rows, int64_t value_dimension,
                                     int64_t padded_value_dimension, int initial, int final_block,
                                     ipuc_stream stream);

/* Rearrange row-major -> {AMP-Left (0), AMP-TransposedRight (1), BlockMajor
 * (2)} f16, bit-exact with zero padding (device/rearrange_f16.cpp:36-155,
 * device/rearrange_amp_left_f16.S:42-140, device/rearrange_transposed_right_f16.S
 * :15-60, device/rearrange_block_major_f16.S:21-116; scalars kernel.rs:1149-1193
 * logical/physical rows/columns and target_order; selection kernel.rs:363-498).
 * src: `matrices` row-major [logical_rows x logical_columns]; dst: `matrices`
 * physical [physical_rows x physical_columns].  row_block/column_block apply to
 * BlockMajor; AMP-TransposedRight uses column_block rows per panel (16 in the
 * reference).  logical_columns even; physical_columns % 16 == 0. */
ipuc_status ipuc_rearrange_f16(void *dst, const void *src, int64_t matrices, int64_t logical_rows,
                               int64_t physical_rows, int32_t target_order,
                               int64_t logical_columns, int64_t physical_columns,
                               int64_t row_block, int64_t column_block, ipuc_stream stream);

/* Unpack AMP-Output (source_order 0) / AMP-TransposedLeft (1) -> row-major f16
 * (device/unpack_amp_f16.cpp:40-81; build kernel.rs:321-362).  dst is
 * `matrices` row-major [physical_rows x physical_columns], zero outside the
 * logical region. */
ipuc_status ipuc_unpack_f16(void *dst, const void *src, int32_t source_order, int64_t matrices,
                            int64_t logical_rows, int64_t physical_rows, int64_t logical_columns,
                            int64_t physical_columns, ipuc_stream stream);

/* General element-order conversion (kernel.rs:1365-1370, "ipu_stack_rearrange",
 * Required in the reference): any ipuc_order -> any ipuc_order for `matrices`
 * [rows x columns] f16 matrices (both physical extents equal), bit-exact. */
ipuc_status ipuc_convert_order_f16(void *dst, ipuc_order to, const void *src, ipuc_order from,
                                   int64_t matrices, int64_t rows, int64_t columns,
                                   int64_t row_block, int64_t column_block, ipuc_stream stream);

/* SplitHeads (graph.rs:336-343; evaluator diagnostic.rs:685-709):
 * [batch, rows, heads*channels] -> [batch*heads, rows, channels], f16. */
ipuc_status ipuc_split_heads_f16(void *out, const void *in, int64_t batch, int64_t rows,
                                 int64_t heads, int64_t channels, ipuc_stream stream);

/* MergeHeads: [batch*heads, rows, channels] -> [batch, rows, heads*channels],
 * the inverse of SplitHeads.  The reference graph has no such operator; it is
 * what an attention block's output projection needs after per-head attention. */
ipuc_status ipuc_merge_heads_f16(void *out, const void *in, int64_t batch, int64_t rows, int64_t heads,
                                 int64_t channels, ipuc_stream stream);

/* ---- Spec-driven dispatch ---------------------------------------------------
 * The reference selects a tile kernel from a TileKernelSpec (operator.rs:57-96),
 * derives its ABI with tile_kernel_abi (kernel.rs:1215-1382: symbol,
 * availability, pointer inputs, named u32 scalars) and checks each run with
 * validate_kernel_run (kernel.rs:1384-1435) before the call is materialised
 * (KernelBuildPlan::call, kernel.rs:713-806).  ipuc_query_abi and ipuc_launch
 * are that pair for one GPU shard: the spec and the scalar vector a reference
 * call site builds are passed unchanged, operands are device tensors, and the
 * call is routed to the typed entry point above. */

/* TileKernelSpec discriminant (operator.rs:57-96). */
typedef enum {
  IPUC_KERNEL_FILL_ZERO = 0,
  IPUC_KERNEL_GEMM = 1,
  IPUC_KERNEL_GELU = 2,
  IPUC_KERNEL_REDUCTION_SUM = 3,
  IPUC_KERNEL_ADD = 4,
  IPUC_KERNEL_FLASH_ATTENTION = 5,
  IPUC_KERNEL_ATTENTION_SOFTMAX = 6,
  IPUC_KERNEL_ATTENTION_MERGE = 7,
  IPUC_KERNEL_CAST = 8,
  IPUC_KERNEL_REARRANGE = 9
} ipuc_kernel_kind;

/* Layout {order} with the BlockMajorOrder block geometry (layout.rs:7-45). */
typedef struct {
  ipuc_order order;
  uint32_t row_block;    /* BLOCK_MAJOR[_TRANSPOSED]; 0 elsewhere */
  uint32_t column_block;
} ipuc_layout;

/* One TileKernelSpec.  Only the member of `kind` is read. */
typedef struct {
  ipuc_kernel_kind kind;
  struct {                     /* Gemm (operator.rs:59-66) */
    ipuc_precision multiply;   /* F16 or F32 (F8F143 has no B200 path) */
    ipuc_precision accumulate; /* AccumulationPrecision: F32 on B200 */
    uint32_t mode;             /* GemmKernelMode: 0 Initialize, 1 Accumulate */
    uint32_t interleaved_weights; /* GemmWeightLoad::Interleaved (requires F16) */
    uint32_t inner_block;      /* IPU K-block / output panel width: planning */
    uint32_t output_columns;   /*   parameters, accepted and not used on B200 */
    uint32_t b_transposed;     /* B200: right operand stored [n x k] */
    uint32_t epilogue_gelu;    /* B200: fused GELU epilogue (graph lowering) */
  } gemm;
  struct { uint16_t partials; } reduction_sum; /* ReductionSum (>= 2) */
  struct {                                      /* FlashAttention */
    uint32_t causal;                            /* rejected, as operator.rs:997 */
    float scale;                                /* <= 0: 1/sqrt(query width) */
    ipuc_precision accumulate;
  } flash_attention;
  struct { uint32_t head_dimension, key_columns, padded_key_columns; } attention_softmax;
  struct {
    uint32_t value_dimension, padded_value_dimension, key_block_columns;
    uint32_t initial, final_block;
  } attention_merge;
  struct { ipuc_precision from, to; } cast;
  struct { ipuc_layout from, to; } rearrange;
} ipuc_kernel_spec;

/* A single-view operand (KernelOperand with one view): a dense row-major
 * device tensor of up to 4 dims. */
typedef struct {
  void *data;
  ipuc_precision precision;
  int32_t rank;
  int64_t dims[4];
} ipuc_tensor;

/* KernelAvailability: IMPLEMENTED has a B200 kernel; REQUIRED names a call
 * the reference plans but nothing executes (ipuc_launch returns
 * IPUC_ERR_UNSUPPORTED). */
typedef enum { IPUC_AVAILABILITY_IMPLEMENTED = 0, IPUC_AVAILABILITY_REQUIRED = 1 } ipuc_availability;

typedef struct {
  const char *symbol;           /* the ipuc_* entry the call routes to */
  const char *reference_symbol; /* the reference tile-kernel family it replaces */
  ipuc_availability availability;
  int32_t input_count;          /* pointer operands after the output (m3..) */
  int32_t scalar_count;
  const char *scalar_names[8];  /* kernel.rs:1149-1193 names, in call order */
} ipuc_kernel_abi;

/* tile_kernel_abi for one spec and the output precision
 * (KernelRequirements::output.format.precision).  Pure host logic: touches
 * no device.  IPUC_ERR_INVALID_ARGUMENT = KernelAbiError::RequirementMismatch. */
ipuc_status ipuc_query_abi(const ipuc_kernel_spec *spec, ipuc_precision output_precision, ipuc_kernel_abi *abi);

/* validate_kernel_run + the call.  `scalars` are the u32 values in the ABI's
 * scalar order, as the reference derives them from the run; they must agree
 * with the tensors.  Operand roles per kind:
 *   FILL_ZERO      out; scalars words_per_worker, remainder_workers (bytes/8 = 6w + r)
 *   GEMM           out C[m,n] (or [b,m,n]); in A[m,k], B[k,n] ([n,k] if b_transposed);
 *                  F32 multiply needs `workspace` of ipuc_gemm_f32_workspace_bytes
 *   GELU           out, in (f16); scalars element_count (even)
 *   REDUCTION_SUM  out f16; in initial[count], remote[(partials-1) * count] (f16 or f32);
 *                  scalars num_partials (= partials - 1), element_count (% 8 == 0)
 *   ADD            out, left, right (f16); scalars element_count, left/right broadcast stride
 *   FLASH_ATTENTION out[M,Sq,D] (f16 or f32); in Q[M,Sq,D], K[M,Sk,D], V[M,Sk,D] f16
 *   ATTENTION_SOFTMAX out weights (+ f32 state); in scores [padded_key_columns/16][rows][16]
 *   ATTENTION_MERGE out acc f32 [rows][padded_value_dimension]; in PV block, softmax
 *                  weights buffer (state after key_block_columns * rows f16);
 *                  scalars initial_block, final_block (must match the spec)
 *   CAST           out, in; scalars element_count
 *   REARRANGE      row-major -> AMP-Left/AMP-TransposedRight/BlockMajor: scalars
 *                  logical_rows, physical_rows, target_order, logical_columns,
 *                  physical_columns; AMP-Output/AMP-TransposedLeft -> row-major:
 *                  matrices, logical_rows, physical_rows, logical_columns,
 *                  physical_columns; any other pair: no scalars, [matrices, rows, cols].
 * Errors mirror KernelAbiError: PointerArity / scalar arity and the count
 * divisibility checks -> IPUC_ERR_INVALID_ARGUMENT with the reference's
 * message; REQUIRED availability -> IPUC_ERR_UNSUPPORTED.  Nothing is
 * launched when a check fails. */
ipuc_status ipuc_launch(const ipuc_kernel_spec *spec, const ipuc_tensor *output, const ipuc_tensor *inputs,
                        int32_t input_count, const uint32_t *scalars, int32_t scalar_count, void *workspace,
                        uint64_t workspace_bytes, ipuc_stream stream);

/* ---- Peer-memory all-reduce (multi-GPU sum after a row-split GEMM) ----
 * The sharded session's all-reduce (transformer block out-proj / MLP-down,
 * Megatron split) done by this library's kernel over NVLink peer memory in
 * place of ncclAllReduce.  Its arithmetic is the reference's partial-sum
 * kernel ipu_stack_reduce_sum_f16 (device/reduce_add_f16.S:31-72, ABI
 * crates/ipu-codegen/src/kernel.rs:1264-1274) with the partials held by
 * other GPUs: out = sum over ranks in rank order, in f32, rounded once to f16,
 * identical bits on every rank.
 *
 * Buffers are shared between the ranks' processes through CUDA IPC:
 * ipuc_ipc_handle exports any device pointer of this process (64-byte handle
 * plus the pointer's offset inside its allocation), ipuc_ipc_open maps a
 * peer's handle into this process, ipuc_ipc_close unmaps it.  Each rank owns
 * one signal area of ipuc_peer_signal_bytes() bytes, zero-filled before any
 * rank's first call (and re-created after a timed-out call). */
uint64_t ipuc_peer_signal_bytes(void);
ipuc_status ipuc_ipc_handle(const void *device_ptr, void *handle_out, uint64_t size, uint64_t *offset);
ipuc_status ipuc_ipc_open(const void *handle, uint64_t offset, void **device_ptr);
ipuc_status ipuc_ipc_close(void *device_ptr);
/* inputs[q], outputs[q], signals[q]: this process's mapping of rank q's input,
 * output and signal area (its own at q == rank).  Every rank calls with the
 * same world and element_count (a multiple of 8 * world, 2 <= world <= 8);
 * buffers 16-byte aligned; input and output may be the same buffer.  All
 * ranks' launches must be able to run at the same time (one launch per GPU,
 * never two ranks on one GPU).  Waits on peers are bounded (2 s): on expiry
 * the kernel sets the device error word (ipuc_device_status ->
 * IPUC_ERR_DEVICE_TIMEOUT) and returns. */
ipuc_status ipuc_peer_all_reduce_f16(void *const *inputs, void *const *outputs, void *const *signals, int32_t rank,
                                     int32_t world, uint64_t element_count, ipuc_stream stream);

#ifdef __cplusplus
}
#endif
#endif /* IPUC_H */
