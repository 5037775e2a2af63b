/*
 * ipug.h — ComputeGraph lowering and device session on top of ipuc.h.
 *
 * Mirrors the reference's graph API (crates/ipu-codegen/src/graph.rs:209-515:
 * ComputeGraph::{host_input, parameter, gemm[_with_options], gelu, add,
 * split_heads, flash_attention[_with_options], set_outputs}) and its runtime
 * (crates/ipu-runtime/src/lib.rs:12-48: open, load, run, read back), with the
 * per-tile lowering (crates/ipu-codegen/src/low.rs:443, lower_operator
 * low.rs:1673-1709) replaced by a per-GPU lowering onto ipuc_* kernels:
 *   Gemm (+ a single-consumer Gelu)      -> ipuc_gemm_f16 with EPILOGUE_GELU
 *   Gemm (+ a single-consumer Add of a same-shaped value)
 *                                        -> copy of the addend + ipuc_gemm_f16 ACCUMULATE
 *   Gelu                                 -> ipuc_gelu_f16
 *   Add (same shape, or a trailing-suffix broadcast) -> ipuc_add_f16
 *   SplitHeads / MergeHeads              -> ipuc_split_heads_f16 / ipuc_merge_heads_f16
 *   FlashAttention (non-causal)          -> ipuc_flash_attention_f16
 * Every value is stored as f16 in its own device buffer (the evaluator's
 * per-op-result quantisation, crates/ipu-tests/src/diagnostic.rs:454-460).
 * Unsupported graph features (transpose_left, causal attention — rejected by
 * the reference too, operator.rs:997 — general broadcasting, Repeat) make
 * ipug_session_open fail with IPUC_ERR_UNSUPPORTED.
 */
#ifndef IPUG_H
#define IPUG_H

#include <stddef.h>
#include <stdint.h>

#include "ipuc.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct ipug_graph ipug_graph;
typedef struct ipug_session ipug_session;

/* Graph construction.  Value ids are >= 0; a negative return is an error
 * (ipuc_last_error_string() describes it, GraphError in graph.rs:1-40). */
ipug_graph *ipug_graph_create(void);
void ipug_graph_destroy(ipug_graph *g);
int32_t ipug_host_input(ipug_graph *g, const char *name, const uint32_t *dims, int32_t rank);
int32_t ipug_parameter(ipug_graph *g, const char *name, const uint32_t *dims, int32_t rank);
int32_t ipug_gemm(ipug_graph *g, int32_t left, int32_t right, int32_t transpose_left, int32_t transpose_right);
int32_t ipug_gelu(ipug_graph *g, int32_t input);
int32_t ipug_add(ipug_graph *g, int32_t left, int32_t right);
int32_t ipug_split_heads(ipug_graph *g, int32_t input, uint32_t heads);
/* Inverse of SplitHeads ([b*h, r, c] -> [b, r, h*c]); not in the reference's
 * graph API, needed to feed per-head attention into an output projection. */
int32_t ipug_merge_heads(ipug_graph *g, int32_t input, uint32_t heads);
/* scale <= 0: AttentionScale::InverseSqrtQueryWidth. */
int32_t ipug_flash_attention(ipug_graph *g, int32_t query, int32_t key, int32_t value, int32_t causal, float scale);
ipuc_status ipug_set_outputs(ipug_graph *g, const int32_t *values, int32_t count);
/* Shape of a value: returns its rank (<= 8 dims written), or -1. */
int32_t ipug_value_shape(const ipug_graph *g, int32_t value, uint32_t *dims);

/* The lowering ipug_session_open would perform (one line per step, as
 * ipug_session_plan), computed on the host without a device or allocation.
 * IPUC_ERR_INVALID_ARGUMENT if buf is too small (*needed = bytes required);
 * lowering errors (IPUC_ERR_UNSUPPORTED) as ipug_session_open reports them. */
ipuc_status ipug_graph_plan(const ipug_graph *g, char *buf, uint64_t size, uint64_t *needed);

/* Session: lower the graph for `device`, allocate every value's buffer. */
ipug_session *ipug_session_open(const ipug_graph *g, int32_t device, ipuc_status *status);
void ipug_session_close(ipug_session *s);
/* Copy f16 host data into an input/parameter (or any) value; bytes must equal
 * the value's element count * 2.  Stream-ordered on `stream`. */
ipuc_status ipug_session_write(ipug_session *s, int32_t value, const void *host, uint64_t bytes, ipuc_stream stream);
ipuc_status ipug_session_read(ipug_session *s, int32_t value, void *host, uint64_t bytes, ipuc_stream stream);
/* Device pointer of a value's buffer (for callers that keep data on the GPU). */
void *ipug_session_device_ptr(ipug_session *s, int32_t value);
ipuc_status ipug_session_run(ipug_session *s, ipuc_stream stream);
/* Run once with a CUDA event pair around every lowered step and write a JSON
 * report (one record per step: op ids, kernel, ms, FLOP or bytes) into buf —
 * the event-timed counterpart of the reference's cycle ProfileReport
 * (crates/ipu-package/src/lib.rs:193-265).  Returns IPUC_ERR_INVALID_ARGUMENT
 * if buf is too small (the required size is written to *needed). */
ipuc_status ipug_session_profile(ipug_session *s, ipuc_stream stream, char *buf, uint64_t size, uint64_t *needed);
/* Human-readable lowered plan (one line per step). */
const char *ipug_session_plan(const ipug_session *s);

#ifdef __cplusplus
}
#endif
#endif /* IPUG_H */
