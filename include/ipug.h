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
 *                                        -> ipuc_gemm_f16_addend (the epilogue adds the
 *                                           other operand; batched GEMMs copy it and
 *                                           accumulate)
 *   Gelu                                 -> ipuc_gelu_f16
 *   Add (same shape, or a trailing-suffix broadcast) -> ipuc_add_f16
 *   SplitHeads / MergeHeads              -> ipuc_split_heads_f16 / ipuc_merge_heads_f16
 *   FlashAttention (non-causal)          -> ipuc_flash_attention_f16
 * Every value is stored as f16 in its own device buffer (the evaluator's
 * per-op-result quantisation, crates/ipu-tests/src/diagnostic.rs:454-460).
 *   Gemm with transpose_left               -> IPUC_GEMM_A_TRANSPOSED (M-major A)
 *   Repeat                               -> unrolled, one body copy per iteration
 * Unsupported graph features (causal attention — rejected by the reference
 * too, operator.rs:997 — and broadcasting other than a trailing suffix) make
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

/* ---- Repeat regions (graph.rs:294-313, 382-473) ----
 * A value sequence names same-shaped values (e.g. per-layer weights); a Repeat
 * runs its body `count` times with carried values (threaded from one
 * iteration's yields to the next iteration's arguments), invariants, and one
 * entry of each iterated sequence per iteration.  ipug_repeat_begin writes
 * the body's argument value ids (carried, then invariants, then iterated) to
 * `arguments`; operations added until ipug_repeat_end form the body and may
 * use only those arguments and the body's own results.  ipug_repeat_end takes
 * one yield per carried value (same shape) and writes the Repeat's result ids
 * to `results`; it returns the number of results, or -1 (the body is then
 * discarded).  Errors follow GraphError's texts. */
int32_t ipug_value_sequence(ipug_graph *g, const char *name, const int32_t *values, int32_t count);
ipuc_status ipug_repeat_begin(ipug_graph *g, uint32_t count, const int32_t *carried, int32_t carried_count,
                              const int32_t *invariants, int32_t invariant_count, const int32_t *sequences,
                              int32_t sequence_count, int32_t *arguments);
int32_t ipug_repeat_end(ipug_graph *g, const int32_t *yields, int32_t yield_count, int32_t *results);

/* ---- Sessions ----
 * A session lowers the graph for one GPU and allocates every value's buffer.
 * With world > 1 it is one rank of a sharded session over `world` GPUs (one
 * process or thread per GPU, each opening its own rank with the same graph
 * and the same NCCL unique id): every rank derives its shard of the work from
 * the graph (column-split GEMMs -> head-local attention -> row-split GEMMs,
 * with an NCCL all-reduce where a row split's partial sums meet a consumer
 * that needs the whole value, an all-gather where a column split does), and
 * the session owns the NCCL communicator.  fuse = 0 keeps a buffer for every
 * operation result (no epilogue or attention fusion), for per-op diagnostics. */
typedef struct ipug_session_options {
  int32_t device;
  int32_t rank, world;   /* world 1: a single-GPU session */
  const void *nccl_id;   /* world > 1: 128-byte ncclUniqueId from ipug_nccl_unique_id on one rank */
  int32_t fuse;          /* 1: fused lowering (default); 0: every value kept */
} ipug_session_options;

ipug_session *ipug_session_open_ex(const ipug_graph *g, const ipug_session_options *options, ipuc_status *status);
/* A new NCCL unique id (ncclGetUniqueId) into out[0..128). */
ipuc_status ipug_nccl_unique_id(void *out, uint64_t size);
/* The plan ipug_session_open_ex would run with `options`, without a device
 * (as ipug_graph_plan; a sharded plan starts with "# rank r of w"). */
ipuc_status ipug_graph_plan_ex(const ipug_graph *g, const ipug_session_options *options, char *buf, uint64_t size,
                               uint64_t *needed);
/* Rank `rank`'s shard of the graph as JSON, without a device: values (local
 * shape, state replicated/columns/heads/partial, parameter slice), operations
 * (including the inserted all_reduce / all_gather_columns) and outputs. */
ipuc_status ipug_graph_shard_json(const ipug_graph *g, int32_t rank, int32_t world, char *buf, uint64_t size,
                                  uint64_t *needed);

/* Session: lower the graph for `device`, allocate every value's buffer
 * (ipug_session_open_ex with world 1 and fuse 1). */
ipug_session *ipug_session_open(const ipug_graph *g, int32_t device, ipuc_status *status);
void ipug_session_close(ipug_session *s);
/* Copy f16 data (host or device memory) into an input/parameter (or any)
 * value; bytes must equal the value's element count * 2.  In a sharded
 * session a parameter the rank holds a slice of takes the whole parameter
 * (the rank copies its columns or rows) or exactly its slice's bytes.
 * Stream-ordered on `stream`.  Values inside a Repeat body are not
 * addressable (the Repeat's results are). */
ipuc_status ipug_session_write(ipug_session *s, int32_t value, const void *host, uint64_t bytes, ipuc_stream stream);
ipuc_status ipug_session_read(ipug_session *s, int32_t value, void *host, uint64_t bytes, ipuc_stream stream);
/* Device pointer of a value's buffer (for callers that keep data on the GPU). */
void *ipug_session_device_ptr(ipug_session *s, int32_t value);
ipuc_status ipug_session_run(ipug_session *s, ipuc_stream stream);
/* Collective over the session's ranks (every rank calls it, after open and
 * before the next run): run the session's all-reduce steps with this
 * library's peer-memory kernel (ipuc_peer_all_reduce_f16) instead of
 * ncclAllReduce.  The ranks exchange CUDA IPC handles of the all-reduce
 * buffers and of a signal area over the session's NCCL communicator.  An
 * all-reduce whose element count is not a multiple of 8 * world, or a world
 * above 8, stays on NCCL.  `enable` 0 goes back to NCCL (the mappings stay
 * until close).  A world-1 session has no all-reduce: a no-op. */
ipuc_status ipug_session_peer_reduce(ipug_session *s, int32_t enable, ipuc_stream stream);

/* ---- Per-op diagnostic (build_diagnostic_package, crates/ipu-codegen/src/
 * package.rs:543; service_checkpoint, crates/ipu-tests/src/diagnostic.rs:
 * 92-199) ----
 * After a run, compare each listed value's buffer with caller-supplied f32
 * reference values (e.g. the host evaluator's): one report per value.  A
 * value fused into its consumer (open the session with fuse = 0 to keep
 * every value), inside a Repeat body, or held as a shard on this rank is
 * reported with available = 0. */
typedef struct ipug_value_report {
  int32_t value;
  int32_t producer;      /* graph operation id of the step that wrote it (-1: an input) */
  int32_t available;
  uint64_t elements;
  uint64_t nonfinite;    /* non-finite device elements (left out of the errors) */
  double max_abs_err, max_abs_ref, rel_l2;
} ipug_value_report;
ipuc_status ipug_session_diagnose(ipug_session *s, const int32_t *values, const float *const *reference,
                                  int32_t count, ipug_value_report *reports, ipuc_stream stream);
/* Run once with a CUDA event pair around every lowered step and write a JSON
 * report (one record per step: op ids, kernel, ms, FLOP or bytes) into buf —
 * the event-timed counterpart of the reference's cycle ProfileReport
 * (crates/ipu-package/src/lib.rs:193-265).  Returns IPUC_ERR_INVALID_ARGUMENT
 * if buf is too small (the required size is written to *needed). */
ipuc_status ipug_session_profile(ipug_session *s, ipuc_stream stream, char *buf, uint64_t size, uint64_t *needed);
/* ---- Profile reports in the reference's Cap'n Proto format ----
 * The message is a `Profile` of schemas/profile.capnp (schema version 5,
 * written by ProfileReport::write, crates/ipu-package/src/lib.rs:198-222):
 * clockHz, and per tile (here: per GPU) a list of CycleSamples, each a Step of
 * schemas/profile_common.capnp with a start and end cycle.  The bytes are the
 * standard single-segment stream framing (capnp::serialize::write_message), so
 * the reference's ProfileReport::read and `ipu-profile query` read them. */
typedef enum ipug_step_kind {
  IPUG_STEP_EXCHANGE = 0,
  IPUG_STEP_COMPUTE = 1,
  IPUG_STEP_SYNCHRONIZATION = 2,
  IPUG_STEP_IDLE = 3
} ipug_step_kind;

typedef struct ipug_exchange_activity {
  uint32_t kind; /* 0 send, 1 receive, 2 partnerBusy (ExchangeActivityKind) */
  uint32_t start_cycle, end_cycle;
} ipug_exchange_activity;

typedef struct ipug_profile_sample {
  uint32_t local_index, phase, epoch;
  uint32_t kind;                 /* ipug_step_kind */
  const char *operation;         /* "operation.<index>" in the reference; NULL = "" */
  const char *kernel;            /* NULL = "" */
  const char *const *metadata;   /* metadata_count (name, value) pairs: 2*count strings */
  uint32_t metadata_count;
  const ipug_exchange_activity *activities;
  uint32_t activity_count;
  uint32_t exchange_event_cycles;
  uint32_t start_cycle, end_cycle;
} ipug_profile_sample;

typedef struct ipug_profile_tile {
  uint32_t physical_tile;
  const ipug_profile_sample *samples;
  uint64_t sample_count;
} ipug_profile_tile;

/* Encode a Profile message.  IPUC_ERR_INVALID_ARGUMENT if buf is too small
 * (the required size is written to *needed) or a kind is out of range. */
ipuc_status ipug_profile_encode(uint64_t clock_hz, const ipug_profile_tile *tiles, uint64_t tile_count, void *buf,
                                uint64_t size, uint64_t *needed);
/* Run the session once with a CUDA event around every lowered step and write
 * the timings as a one-tile Profile message (physical tile = `physical_tile`,
 * normally the GPU's rank): clockHz 1e9, so a cycle is one nanosecond from the
 * first event; one Compute step per lowered step, operation "operation.<id>"
 * of its first graph operation, kernel = the step's kernel, metadata
 * "operations" (all fused op ids), "flop"/"tflops" or "bytes"/"gbs", "device".
 * Cycle counts are u32 in the schema: they saturate at 2^32 - 1 ns (4.29 s). */
ipuc_status ipug_session_profile_capnp(ipug_session *s, ipuc_stream stream, uint32_t physical_tile, void *buf,
                                       uint64_t size, uint64_t *needed);

/* Human-readable lowered plan (one line per step). */
const char *ipug_session_plan(const ipug_session *s);

#ifdef __cplusplus
}
#endif
#endif /* IPUG_H */
