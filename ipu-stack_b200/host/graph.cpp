// ComputeGraph builder, per-GPU lowering onto the ipuc_* kernels, and the
// device session (include/ipug.h).
//
// Graph semantics follow crates/ipu-codegen/src/graph.rs (value ids in
// construction order, shape inference graph.rs:661-760, numpy broadcasting
// graph.rs:762-788).  The lowering replaces lower_to_tiles / lower_operator
// (crates/ipu-codegen/src/low.rs:443,1673-1709): instead of per-tile kernel
// runs and exchange phases it emits one stream-ordered kernel call per GPU for
// each operator, fusing a Gemm into its single Gelu or Add consumer through the
// GEMM epilogue.  The session mirrors ipu-runtime (crates/ipu-runtime/src/
// lib.rs:12-48): open a device, upload inputs/weights, run, read back.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <memory>
#include <sstream>
#include <string>
#include <vector>

#include "../../include/ipug.h"

namespace ipuc {
void set_error(const std::string &msg);
ipuc_status fail(ipuc_status st, const std::string &msg);
}  // namespace ipuc

namespace {

enum class OpKind { Gemm, Gelu, Add, SplitHeads, MergeHeads, FlashAttention };

struct Op {
  OpKind kind;
  std::vector<int32_t> inputs;
  int32_t result;
  bool transpose_left = false, transpose_right = false;
  uint32_t heads = 0;
  bool causal = false;
  float scale = 0.0f;
};

struct Value {
  std::vector<uint32_t> shape;
  int kind;  // 0 host input, 1 parameter, 2 op result
  std::string name;
  int32_t producer = -1;  // op index
};

uint64_t numel(const std::vector<uint32_t> &s) {
  uint64_t n = 1;
  for (uint32_t d : s) n *= d;
  return n;
}

std::string shape_str(const std::vector<uint32_t> &s) {
  std::ostringstream o;
  o << "[";
  for (size_t i = 0; i < s.size(); ++i) o << (i ? "," : "") << s[i];
  o << "]";
  return o.str();
}

// graph.rs:762-788
bool broadcast(const std::vector<uint32_t> &l, const std::vector<uint32_t> &r, std::vector<uint32_t> &out) {
  const size_t rank = std::max(l.size(), r.size());
  out.assign(rank, 1);
  for (size_t i = 0; i < rank; ++i) {
    const uint32_t a = i + l.size() >= rank ? l[i + l.size() - rank] : 1;
    const uint32_t b = i + r.size() >= rank ? r[i + r.size() - rank] : 1;
    if (a != b && a != 1 && b != 1) return false;
    out[i] = std::max(a, b);
  }
  return true;
}

}  // namespace

struct ipug_graph {
  std::vector<Value> values;
  std::vector<Op> ops;
  std::vector<int32_t> outputs;

  bool valid(int32_t v) const { return v >= 0 && v < (int32_t)values.size(); }

  int32_t add_value(std::vector<uint32_t> shape, int kind, std::string name, int32_t producer) {
    values.push_back(Value{std::move(shape), kind, std::move(name), producer});
    return (int32_t)values.size() - 1;
  }

  int32_t add_op(Op op, std::vector<uint32_t> shape) {
    for (int32_t v : op.inputs)
      if (!valid(v)) {
        ipuc::set_error("unknown value " + std::to_string(v));
        return -1;
      }
    op.result = add_value(std::move(shape), 2, "", (int32_t)ops.size());
    ops.push_back(op);
    return op.result;
  }
};

namespace {

enum class StepKind { Gemm, Gelu, Add, SplitHeads, MergeHeads, Attention, AttentionHeads, Copy };

struct Step {
  StepKind kind;
  std::vector<int32_t> op_ids;
  // value ids
  int32_t out = -1, in0 = -1, in1 = -1, in2 = -1;
  int32_t addend = -1;  // Gemm: value the epilogue adds (the fused Add's other operand)
  // gemm
  int64_t batch = 1, m = 0, n = 0, k = 0;
  uint32_t flags = 0;
  // add
  uint64_t count = 0, right_period = 0;
  // split heads
  int64_t b = 0, rows = 0, heads = 0, channels = 0;
  // attention
  int64_t streams = 0, sq = 0, sk = 0, d = 0;
  float scale = 0.0f;
  double flop = 0.0, bytes = 0.0;
  std::string label;
};

}  // namespace

struct ipug_session {
  const ipug_graph *graph = nullptr;
  int device = 0;
  std::vector<void *> buffers;  // per value; nullptr = fused away
  std::vector<Step> steps;
  std::string plan;
  ~ipug_session() {
    bool any = false;
    for (void *p : buffers) any = any || p != nullptr;
    if (!any) return;  // a plan-only lowering holds no device memory
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(device);
    for (void *p : buffers)
      if (p) cudaFree(p);
    cudaSetDevice(prev);
  }
};

namespace {

// allocate = false lowers without touching a device (ipug_graph_plan).
ipuc_status lower(const ipug_graph &g, ipug_session &s, bool allocate = true) {
  const size_t nv = g.values.size();
  std::vector<std::vector<int32_t>> consumers(nv);
  for (size_t i = 0; i < g.ops.size(); ++i)
    for (int32_t v : g.ops[i].inputs) consumers[v].push_back((int32_t)i);
  std::vector<bool> is_output(nv, false);
  for (int32_t v : g.outputs) is_output[v] = true;
  std::vector<bool> fused_into_next(g.ops.size(), false);  // gemm handled by its consumer
  std::vector<int32_t> fused_gemm(g.ops.size(), -1);        // consumer op -> gemm op
  for (size_t i = 0; i < g.ops.size(); ++i) {
    const Op &op = g.ops[i];
    if (op.kind != OpKind::Gemm) continue;
    const int32_t r = op.result;
    if (is_output[r] || consumers[r].size() != 1) continue;
    const int32_t c = consumers[r][0];
    const Op &co = g.ops[c];
    if (fused_gemm[c] >= 0) continue;  // Add(Gemm, Gemm): the second GEMM keeps its own step and buffer
    if (co.kind == OpKind::Gelu) {
      fused_into_next[i] = true;
      fused_gemm[c] = (int32_t)i;
    } else if (co.kind == OpKind::Add && co.inputs[0] != co.inputs[1]) {
      const int32_t other = co.inputs[0] == r ? co.inputs[1] : co.inputs[0];
      if (g.values[other].shape == g.values[r].shape) {
        fused_into_next[i] = true;
        fused_gemm[c] = (int32_t)i;
      }
    }
  }

  // SplitHeads(q), SplitHeads(k), SplitHeads(v) -> FlashAttention -> MergeHeads,
  // with every intermediate used once and not an output, lowers to one
  // attention call on the unsplit [b, rows, heads * c] values (4-D tensor maps
  // stand in for the split and merge copies).  fused_attention[merge op] =
  // attention op; the split and attention ops emit no step.
  std::vector<int32_t> fused_attention(g.ops.size(), -1);
  auto single_use = [&](int32_t v) { return !is_output[v] && consumers[v].size() == 1; };
  for (size_t i = 0; i < g.ops.size(); ++i) {
    const Op &at = g.ops[i];
    if (at.kind != OpKind::FlashAttention || at.causal || !single_use(at.result)) continue;
    const Op &mg = g.ops[consumers[at.result][0]];
    if (mg.kind != OpKind::MergeHeads) continue;
    bool ok = true;
    for (int32_t in : at.inputs) {
      const Value &val = g.values[in];
      if (val.kind != 2 || !single_use(in)) { ok = false; break; }
      const Op &sp = g.ops[val.producer];
      ok = ok && sp.kind == OpKind::SplitHeads && sp.heads == mg.heads && g.values[sp.inputs[0]].shape.size() == 3;
    }
    if (!ok) continue;
    fused_attention[consumers[at.result][0]] = (int32_t)i;
    fused_into_next[i] = true;
    for (int32_t in : at.inputs) fused_into_next[g.values[in].producer] = true;
  }

  auto gemm_step = [&](const Op &op, Step &st) -> ipuc_status {
    const auto &L = g.values[op.inputs[0]].shape, &R = g.values[op.inputs[1]].shape;
    if (op.transpose_left) return ipuc::fail(IPUC_ERR_UNSUPPORTED, "lowering: Gemm transpose_left is not supported");
    const uint32_t m = L[L.size() - 2], k = L[L.size() - 1];
    const uint32_t n = op.transpose_right ? R[R.size() - 2] : R[R.size() - 1];
    const std::vector<uint32_t> lb(L.begin(), L.end() - 2), rb(R.begin(), R.end() - 2);
    if (rb.empty() || numel(rb) == 1) {
      st.batch = 1;
      st.m = (int64_t)numel(lb) * m;  // flatten the left batch into rows
    } else if (lb == rb) {
      st.batch = (int64_t)numel(lb);
      st.m = m;
    } else {
      return ipuc::fail(IPUC_ERR_UNSUPPORTED, "lowering: Gemm batch broadcasting other than a 2-D right operand");
    }
    st.n = n;
    st.k = k;
    st.flags |= op.transpose_right ? IPUC_GEMM_B_TRANSPOSED : 0u;
    st.in0 = op.inputs[0];
    st.in1 = op.inputs[1];
    st.flop = 2.0 * (double)st.batch * (double)st.m * (double)n * (double)k;
    return IPUC_OK;
  };

  std::ostringstream plan;
  for (size_t i = 0; i < g.ops.size(); ++i) {
    const Op &op = g.ops[i];
    if (fused_into_next[i]) continue;
    Step st;
    st.op_ids.push_back((int32_t)i);
    st.out = op.result;
    ipuc_status rc = IPUC_OK;
    switch (op.kind) {
      case OpKind::Gemm:
        st.kind = StepKind::Gemm;
        rc = gemm_step(op, st);
        st.label = "gemm_f16";
        break;
      case OpKind::Gelu:
        if (fused_gemm[i] >= 0) {
          const Op &gm = g.ops[fused_gemm[i]];
          st.kind = StepKind::Gemm;
          st.op_ids.insert(st.op_ids.begin(), fused_gemm[i]);
          rc = gemm_step(gm, st);
          st.flags |= IPUC_GEMM_EPILOGUE_GELU;
          st.label = "gemm_f16+gelu";
        } else {
          st.kind = StepKind::Gelu;
          st.in0 = op.inputs[0];
          st.count = numel(g.values[op.result].shape);
          st.bytes = 4.0 * st.count;
          st.label = "gelu_f16";
        }
        break;
      case OpKind::Add:
        if (fused_gemm[i] >= 0) {
          const Op &gm = g.ops[fused_gemm[i]];
          const int32_t other = op.inputs[0] == gm.result ? op.inputs[1] : op.inputs[0];
          st.kind = StepKind::Gemm;
          st.op_ids.insert(st.op_ids.begin(), fused_gemm[i]);
          rc = gemm_step(gm, st);
          st.flags |= IPUC_GEMM_ACCUMULATE;
          st.label = "gemm_f16+add";
          if (st.batch == 1) {
            st.addend = other;  // the GEMM epilogue reads it: no copy
          } else {
            // Batched: copy the addend into the output, then accumulate onto it.
            Step cp;
            cp.kind = StepKind::Copy;
            cp.op_ids.push_back((int32_t)i);
            cp.in0 = other;
            cp.out = op.result;
            cp.count = numel(g.values[op.result].shape);
            cp.bytes = 4.0 * cp.count;
            cp.label = "copy(addend)";
            s.steps.push_back(cp);
          }
        } else {
          st.kind = StepKind::Add;
          const auto &a = g.values[op.inputs[0]].shape, &b = g.values[op.inputs[1]].shape;
          const auto &o = g.values[op.result].shape;
          st.count = numel(o);
          auto is_suffix = [](const std::vector<uint32_t> &small, const std::vector<uint32_t> &big) {
            if (small.size() > big.size()) return false;
            std::vector<uint32_t> sq = small;
            while (!sq.empty() && sq.front() == 1) sq.erase(sq.begin());
            return std::equal(sq.rbegin(), sq.rend(), big.rbegin());
          };
          if (a == o && b == o) {
            st.in0 = op.inputs[0];
            st.in1 = op.inputs[1];
          } else if (a == o && is_suffix(b, o)) {
            st.in0 = op.inputs[0];
            st.in1 = op.inputs[1];
            st.right_period = numel(b);
          } else if (b == o && is_suffix(a, o)) {
            st.in0 = op.inputs[1];
            st.in1 = op.inputs[0];
            st.right_period = numel(a);
          } else {
            rc = ipuc::fail(IPUC_ERR_UNSUPPORTED, "lowering: Add broadcast other than a trailing suffix");
          }
          st.bytes = 6.0 * st.count;
          st.label = "add_f16";
        }
        break;
      case OpKind::SplitHeads: {
        st.kind = StepKind::SplitHeads;
        const auto &x = g.values[op.inputs[0]].shape;
        st.in0 = op.inputs[0];
        st.b = x[0];
        st.rows = x[1];
        st.heads = op.heads;
        st.channels = x[2] / op.heads;
        st.bytes = 4.0 * numel(x);
        st.label = "split_heads_f16";
        break;
      }
      case OpKind::MergeHeads: {
        if (fused_attention[i] >= 0) {
          // Attention on the unsplit projections, written in merged layout.
          const Op &at = g.ops[fused_attention[i]];
          const Op &sq = g.ops[g.values[at.inputs[0]].producer], &sk = g.ops[g.values[at.inputs[1]].producer],
                   &sv = g.ops[g.values[at.inputs[2]].producer];
          const auto &qx = g.values[sq.inputs[0]].shape, &kx = g.values[sk.inputs[0]].shape,
                     &vx = g.values[sv.inputs[0]].shape;
          if (qx[0] != kx[0] || kx != vx || qx[2] != kx[2]) {
            rc = ipuc::fail(IPUC_ERR_UNSUPPORTED, "lowering: attention needs equal batch and width for q, k and v");
            break;
          }
          st.kind = StepKind::AttentionHeads;
          st.op_ids = {g.values[at.inputs[0]].producer, g.values[at.inputs[1]].producer,
                       g.values[at.inputs[2]].producer, fused_attention[i], (int32_t)i};
          st.in0 = sq.inputs[0];
          st.in1 = sk.inputs[0];
          st.in2 = sv.inputs[0];
          st.b = qx[0];
          st.heads = op.heads;
          st.sq = qx[1];
          st.sk = kx[1];
          st.d = qx[2] / op.heads;
          st.streams = st.b * st.heads;
          st.scale = at.scale;
          st.flop = 4.0 * st.streams * st.sq * st.sk * st.d;
          st.label = "flash_attention_heads_f16";
          break;
        }
        st.kind = StepKind::MergeHeads;
        const auto &x = g.values[op.inputs[0]].shape;
        st.in0 = op.inputs[0];
        st.b = x[0] / op.heads;
        st.rows = x[1];
        st.heads = op.heads;
        st.channels = x[2];
        st.bytes = 4.0 * numel(x);
        st.label = "merge_heads_f16";
        break;
      }
      case OpKind::FlashAttention: {
        st.kind = StepKind::Attention;
        if (op.causal) {
          rc = ipuc::fail(IPUC_ERR_UNSUPPORTED, "lowering: causal attention is not supported (operator.rs:997)");
          break;
        }
        const auto &q = g.values[op.inputs[0]].shape, &k = g.values[op.inputs[1]].shape,
                   &v = g.values[op.inputs[2]].shape;
        const std::vector<uint32_t> qb(q.begin(), q.end() - 2), kb(k.begin(), k.end() - 2), vb(v.begin(), v.end() - 2);
        if (qb != kb || qb != vb || v.back() != q.back()) {
          rc = ipuc::fail(IPUC_ERR_UNSUPPORTED,
                          "lowering: attention needs equal batch dims and value width == query width");
          break;
        }
        st.in0 = op.inputs[0];
        st.in1 = op.inputs[1];
        st.in2 = op.inputs[2];
        st.streams = (int64_t)numel(qb);
        st.sq = q[q.size() - 2];
        st.sk = k[k.size() - 2];
        st.d = q.back();
        st.scale = op.scale;
        st.flop = 4.0 * st.streams * st.sq * st.sk * st.d;
        st.label = "flash_attention_f16";
        break;
      }
    }
    if (rc != IPUC_OK) return rc;
    s.steps.push_back(st);
  }
  for (const Step &st : s.steps) {
    plan << st.label << " ops=";
    for (size_t j = 0; j < st.op_ids.size(); ++j) plan << (j ? "," : "") << st.op_ids[j];
    plan << " out=v" << st.out << shape_str(g.values[st.out].shape) << "\n";
  }
  s.plan = plan.str();
  // Buffers: every value except the results of ops fused into a consumer.
  s.buffers.assign(nv, nullptr);
  if (!allocate) return IPUC_OK;
  for (size_t v = 0; v < nv; ++v) {
    const Value &val = g.values[v];
    if (val.kind == 2 && fused_into_next[val.producer]) continue;
    const uint64_t bytes = std::max<uint64_t>(numel(val.shape) * 2, 16);
    const cudaError_t e = cudaMalloc(&s.buffers[v], bytes);
    if (e != cudaSuccess) return ipuc::fail(IPUC_ERR_CUDA, std::string("session: cudaMalloc: ") + cudaGetErrorString(e));
  }
  return IPUC_OK;
}

ipuc_status run_step(ipug_session &s, const Step &st, cudaStream_t stream) {
  auto P = [&](int32_t v) { return s.buffers[v]; };
  switch (st.kind) {
    case StepKind::Gemm: {
      const int64_t lda = st.k, ldb = (st.flags & IPUC_GEMM_B_TRANSPOSED) ? st.k : st.n, ldc = st.n;
      if (st.batch == 1 && st.addend >= 0)
        return ipuc_gemm_f16_addend(P(st.out), P(st.in0), P(st.in1), st.m, st.n, st.k, lda, ldb, ldc, st.flags,
                                    P(st.addend), st.n, stream);
      if (st.batch == 1)
        return ipuc_gemm_f16(P(st.out), P(st.in0), P(st.in1), st.m, st.n, st.k, lda, ldb, ldc, st.flags, stream);
      return ipuc_gemm_f16_batched(P(st.out), P(st.in0), P(st.in1), st.batch, st.m, st.n, st.k, lda, ldb, ldc,
                                   st.m * st.k, st.n * st.k, st.m * st.n, st.flags, stream);
    }
    case StepKind::Gelu:
      return ipuc_gelu_f16(P(st.out), P(st.in0), st.count, stream);
    case StepKind::Add:
      return ipuc_add_f16(P(st.out), P(st.in0), P(st.in1), st.count, 0, st.right_period, stream);
    case StepKind::SplitHeads:
      return ipuc_split_heads_f16(P(st.out), P(st.in0), st.b, st.rows, st.heads, st.channels, stream);
    case StepKind::MergeHeads:
      return ipuc_merge_heads_f16(P(st.out), P(st.in0), st.b, st.rows, st.heads, st.channels, stream);
    case StepKind::Attention:
      return ipuc_flash_attention_f16(P(st.out), IPUC_F16, P(st.in0), P(st.in1), P(st.in2), st.streams, st.sq, st.sk,
                                      st.d, st.scale, stream);
    case StepKind::AttentionHeads:
      return ipuc_flash_attention_heads_f16(P(st.out), IPUC_F16, P(st.in0), P(st.in1), P(st.in2), st.b, st.heads,
                                            st.sq, st.sk, st.d, st.scale, stream);
    case StepKind::Copy: {
      const cudaError_t e = cudaMemcpyAsync(P(st.out), P(st.in0), st.count * 2, cudaMemcpyDeviceToDevice, stream);
      if (e != cudaSuccess) return ipuc::fail(IPUC_ERR_CUDA, std::string("session copy: ") + cudaGetErrorString(e));
      return IPUC_OK;
    }
  }
  return IPUC_OK;
}

struct DeviceGuard {
  int prev = 0;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    cudaSetDevice(dev);
  }
  ~DeviceGuard() { cudaSetDevice(prev); }
};

int32_t checked(ipug_graph *g, Op op, bool ok, const std::string &why, std::vector<uint32_t> shape) {
  if (!g) {
    ipuc::set_error("null graph");
    return -1;
  }
  for (int32_t v : op.inputs)
    if (!g->valid(v)) {
      ipuc::set_error("unknown value " + std::to_string(v));
      return -1;
    }
  if (!ok) {
    ipuc::set_error("invalid shape: " + why);
    return -1;
  }
  return g->add_op(op, std::move(shape));
}

}  // namespace

extern "C" {

ipug_graph *ipug_graph_create(void) { return new ipug_graph(); }
void ipug_graph_destroy(ipug_graph *g) { delete g; }

static int32_t add_input(ipug_graph *g, const char *name, const uint32_t *dims, int32_t rank, int kind) {
  if (!g || !name || !*name) {
    ipuc::set_error("input needs a graph and a nonempty name");
    return -1;
  }
  if (rank < 0 || rank > 8 || (rank > 0 && !dims)) {
    ipuc::set_error("input rank must be in [0, 8]");
    return -1;
  }
  std::vector<uint32_t> shape(dims, dims + rank);
  for (uint32_t d : shape)
    if (d == 0) {
      ipuc::set_error("input dimensions must be positive");
      return -1;
    }
  return g->add_value(shape, kind, name, -1);
}

int32_t ipug_host_input(ipug_graph *g, const char *name, const uint32_t *dims, int32_t rank) {
  return add_input(g, name, dims, rank, 0);
}
int32_t ipug_parameter(ipug_graph *g, const char *name, const uint32_t *dims, int32_t rank) {
  return add_input(g, name, dims, rank, 1);
}

int32_t ipug_gemm(ipug_graph *g, int32_t left, int32_t right, int32_t transpose_left, int32_t transpose_right) {
  Op op{OpKind::Gemm, {left, right}, -1};
  op.transpose_left = transpose_left != 0;
  op.transpose_right = transpose_right != 0;
  if (!g || !g->valid(left) || !g->valid(right)) return checked(g, op, false, "unknown value", {});
  const auto &L = g->values[left].shape, &R = g->values[right].shape;  // graph.rs:671-690
  if (L.size() < 2 || R.size() < 2) return checked(g, op, false, "GEMM inputs must have rank at least two", {});
  const uint32_t lr = L[L.size() - 2 + (op.transpose_left ? 1 : 0)], li = L[L.size() - 1 - (op.transpose_left ? 1 : 0)];
  const uint32_t ri = R[R.size() - 2 + (op.transpose_right ? 1 : 0)], rc = R[R.size() - 1 - (op.transpose_right ? 1 : 0)];
  if (li != ri) return checked(g, op, false, "GEMM inner dimensions do not match", {});
  std::vector<uint32_t> out;
  if (!broadcast(std::vector<uint32_t>(L.begin(), L.end() - 2), std::vector<uint32_t>(R.begin(), R.end() - 2), out))
    return checked(g, op, false, "GEMM batch dimensions cannot be broadcast", {});
  out.push_back(lr);
  out.push_back(rc);
  return checked(g, op, true, "", out);
}

int32_t ipug_gelu(ipug_graph *g, int32_t input) {
  Op op{OpKind::Gelu, {input}, -1};
  if (!g || !g->valid(input)) return checked(g, op, false, "unknown value", {});
  return checked(g, op, true, "", g->values[input].shape);
}

int32_t ipug_add(ipug_graph *g, int32_t left, int32_t right) {
  Op op{OpKind::Add, {left, right}, -1};
  if (!g || !g->valid(left) || !g->valid(right)) return checked(g, op, false, "unknown value", {});
  std::vector<uint32_t> out;
  const bool ok = broadcast(g->values[left].shape, g->values[right].shape, out);
  return checked(g, op, ok, "Add shapes cannot be broadcast", out);
}

int32_t ipug_split_heads(ipug_graph *g, int32_t input, uint32_t heads) {
  Op op{OpKind::SplitHeads, {input}, -1};
  op.heads = heads;
  if (!g || !g->valid(input)) return checked(g, op, false, "unknown value", {});
  const auto &x = g->values[input].shape;  // graph.rs:704-727
  if (x.size() != 3 || heads == 0)
    return checked(g, op, false, "split_heads requires nonzero heads and [batch, rows, channels] input", {});
  if (x[2] % heads) return checked(g, op, false, "split_heads channels must be divisible by heads", {});
  return checked(g, op, true, "", {x[0] * heads, x[1], x[2] / heads});
}

int32_t ipug_merge_heads(ipug_graph *g, int32_t input, uint32_t heads) {
  Op op{OpKind::MergeHeads, {input}, -1};
  op.heads = heads;
  if (!g || !g->valid(input)) return checked(g, op, false, "unknown value", {});
  const auto &x = g->values[input].shape;
  if (x.size() != 3 || heads == 0 || x[0] % heads)
    return checked(g, op, false, "merge_heads requires [batch*heads, rows, channels] input with heads dividing dim 0", {});
  return checked(g, op, true, "", {x[0] / heads, x[1], x[2] * heads});
}

int32_t ipug_flash_attention(ipug_graph *g, int32_t query, int32_t key, int32_t value, int32_t causal, float scale) {
  Op op{OpKind::FlashAttention, {query, key, value}, -1};
  op.causal = causal != 0;
  op.scale = scale;
  if (!g || !g->valid(query) || !g->valid(key) || !g->valid(value)) return checked(g, op, false, "unknown value", {});
  const auto &q = g->values[query].shape, &k = g->values[key].shape, &v = g->values[value].shape;  // graph.rs:728-758
  if (q.size() < 2 || k.size() < 2 || v.size() < 2)
    return checked(g, op, false, "FlashAttention inputs must have rank at least two", {});
  if (q.back() != k.back() || k[k.size() - 2] != v[v.size() - 2])
    return checked(g, op, false, "FlashAttention head or sequence dimensions do not match", {});
  if (scale > 0.0f && !std::isfinite(scale)) return checked(g, op, false, "attention scale must be finite and positive", {});
  std::vector<uint32_t> kvb, out;
  if (!broadcast(std::vector<uint32_t>(k.begin(), k.end() - 2), std::vector<uint32_t>(v.begin(), v.end() - 2), kvb) ||
      !broadcast(std::vector<uint32_t>(q.begin(), q.end() - 2), kvb, out))
    return checked(g, op, false, "FlashAttention batch dimensions cannot be broadcast", {});
  out.push_back(q[q.size() - 2]);
  out.push_back(v.back());
  return checked(g, op, true, "", out);
}

ipuc_status ipug_set_outputs(ipug_graph *g, const int32_t *values, int32_t count) {
  if (!g || count < 0 || (count > 0 && !values)) return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, "set_outputs: bad arguments");
  for (int32_t i = 0; i < count; ++i)
    if (!g->valid(values[i])) return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, "set_outputs: unknown value");
  g->outputs.assign(values, values + count);
  return IPUC_OK;
}

int32_t ipug_value_shape(const ipug_graph *g, int32_t value, uint32_t *dims) {
  if (!g || !g->valid(value)) return -1;
  const auto &s = g->values[value].shape;
  if (dims)
    for (size_t i = 0; i < s.size() && i < 8; ++i) dims[i] = s[i];
  return (int32_t)s.size();
}

ipug_session *ipug_session_open(const ipug_graph *g, int32_t device, ipuc_status *status) {
  auto set = [&](ipuc_status st) {
    if (status) *status = st;
  };
  if (!g) {
    set(ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, "session_open: null graph"));
    return nullptr;
  }
  DeviceGuard guard(device);
  std::unique_ptr<ipug_session> s(new ipug_session());
  s->graph = g;
  s->device = device;
  const ipuc_status st = lower(*g, *s);
  set(st);
  if (st != IPUC_OK) return nullptr;
  return s.release();
}

void ipug_session_close(ipug_session *s) { delete s; }

ipuc_status ipug_graph_plan(const ipug_graph *g, char *buf, uint64_t size, uint64_t *needed) {
  if (!g) return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, "graph_plan: null graph");
  ipug_session s;
  s.graph = g;
  const ipuc_status st = lower(*g, s, false);
  if (st != IPUC_OK) return st;
  if (needed) *needed = s.plan.size() + 1;
  if (!buf || size < s.plan.size() + 1)
    return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, "graph_plan: buffer too small");
  std::memcpy(buf, s.plan.c_str(), s.plan.size() + 1);
  return IPUC_OK;
}

static ipuc_status check_value(ipug_session *s, int32_t value, uint64_t bytes) {
  if (!s || !s->graph->valid(value)) return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, "session: unknown value");
  if (!s->buffers[value])
    return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, "session: value was fused into its consumer and has no buffer");
  if (bytes != numel(s->graph->values[value].shape) * 2)
    return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, "session: byte count must be element count * 2 (f16)");
  return IPUC_OK;
}

ipuc_status ipug_session_write(ipug_session *s, int32_t value, const void *host, uint64_t bytes, ipuc_stream stream) {
  const ipuc_status st = check_value(s, value, bytes);
  if (st != IPUC_OK) return st;
  DeviceGuard guard(s->device);
  const cudaError_t e = cudaMemcpyAsync(s->buffers[value], host, bytes, cudaMemcpyHostToDevice, stream);
  if (e != cudaSuccess) return ipuc::fail(IPUC_ERR_CUDA, std::string("session_write: ") + cudaGetErrorString(e));
  return IPUC_OK;
}

ipuc_status ipug_session_read(ipug_session *s, int32_t value, void *host, uint64_t bytes, ipuc_stream stream) {
  const ipuc_status st = check_value(s, value, bytes);
  if (st != IPUC_OK) return st;
  DeviceGuard guard(s->device);
  cudaError_t e = cudaMemcpyAsync(host, s->buffers[value], bytes, cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return ipuc::fail(IPUC_ERR_CUDA, std::string("session_read: ") + cudaGetErrorString(e));
  return IPUC_OK;
}

void *ipug_session_device_ptr(ipug_session *s, int32_t value) {
  if (!s || !s->graph->valid(value)) return nullptr;
  return s->buffers[value];
}

ipuc_status ipug_session_run(ipug_session *s, ipuc_stream stream) {
  if (!s) return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, "session_run: null session");
  DeviceGuard guard(s->device);
  for (const Step &st : s->steps) {
    const ipuc_status rc = run_step(*s, st, stream);
    if (rc != IPUC_OK) return rc;
  }
  return IPUC_OK;
}

}  // extern "C"

// Run every lowered step once with a CUDA event on each boundary; t[i] is the
// time of boundary i in ms after boundary 0 (t.size() == steps + 1).
static ipuc_status time_steps(ipug_session *s, ipuc_stream stream, std::vector<double> &t, const char *who) {
  DeviceGuard guard(s->device);
  std::vector<cudaEvent_t> ev(s->steps.size() + 1, nullptr);
  ipuc_status rc = IPUC_OK;
  for (auto &e : ev)
    if (rc == IPUC_OK && cudaEventCreate(&e) != cudaSuccess) rc = ipuc::fail(IPUC_ERR_CUDA, std::string(who) + ": cudaEventCreate");
  if (rc == IPUC_OK) {
    cudaEventRecord(ev[0], stream);
    for (size_t i = 0; i < s->steps.size() && rc == IPUC_OK; ++i) {
      rc = run_step(*s, s->steps[i], stream);
      cudaEventRecord(ev[i + 1], stream);
    }
  }
  if (rc == IPUC_OK && cudaEventSynchronize(ev.back()) != cudaSuccess)
    rc = ipuc::fail(IPUC_ERR_CUDA, std::string(who) + ": event synchronize failed");
  if (rc == IPUC_OK) {
    t.assign(ev.size(), 0.0);
    for (size_t i = 1; i < ev.size(); ++i) {
      float ms = 0.0f;
      cudaEventElapsedTime(&ms, ev[0], ev[i]);
      t[i] = ms;
    }
  }
  for (auto &e : ev)
    if (e) cudaEventDestroy(e);
  return rc;
}

extern "C" {

ipuc_status ipug_session_profile(ipug_session *s, ipuc_stream stream, char *buf, uint64_t size, uint64_t *needed) {
  if (!s) return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, "session_profile: null session");
  std::vector<double> t;
  const ipuc_status rc = time_steps(s, stream, t, "session_profile");
  if (rc != IPUC_OK) return rc;
  std::ostringstream o;
  o << "{\"device\": " << s->device << ", \"steps\": [";
  for (size_t i = 0; i < s->steps.size(); ++i) {
    const double ms = t[i + 1] - t[i];
    const Step &st = s->steps[i];
    o << (i ? ", " : "") << "{\"step\": " << i << ", \"kernel\": \"" << st.label << "\", \"ops\": [";
    for (size_t j = 0; j < st.op_ids.size(); ++j) o << (j ? ", " : "") << st.op_ids[j];
    o << "], \"ms\": " << ms;
    if (st.flop > 0) o << ", \"flop\": " << st.flop << ", \"tflops\": " << st.flop / (ms * 1e-3) / 1e12;
    if (st.bytes > 0) o << ", \"bytes\": " << st.bytes << ", \"gbs\": " << st.bytes / (ms * 1e-3) / 1e9;
    o << "}";
  }
  o << "], \"total_ms\": " << t.back() << "}";
  const std::string js = o.str();
  if (needed) *needed = js.size() + 1;
  if (!buf || size < js.size() + 1) return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, "session_profile: buffer too small");
  std::memcpy(buf, js.c_str(), js.size() + 1);
  return IPUC_OK;
}

ipuc_status ipug_session_profile_capnp(ipug_session *s, ipuc_stream stream, uint32_t physical_tile, void *buf,
                                       uint64_t size, uint64_t *needed) {
  if (!s) return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, "session_profile_capnp: null session");
  std::vector<double> t;
  const ipuc_status rc = time_steps(s, stream, t, "session_profile_capnp");
  if (rc != IPUC_OK) return rc;
  const size_t n = s->steps.size();
  // Strings the samples point at; reserved so the pointers stay put.
  std::vector<std::string> text;
  text.reserve(n * 16);
  std::vector<std::vector<const char *>> meta(n);
  std::vector<ipug_profile_sample> samples(n);
  auto keep = [&text](std::string v) { text.push_back(std::move(v)); return text.back().c_str(); };
  auto num = [](double v) { std::ostringstream o; o << v; return o.str(); };
  auto cycles = [](double ms) {  // 1 cycle = 1 ns at clockHz 1e9
    const double c = std::llround(ms * 1e6);
    return static_cast<uint32_t>(c < 0 ? 0 : (c > 4294967295.0 ? 4294967295.0 : c));
  };
  for (size_t i = 0; i < n; ++i) {
    const Step &st = s->steps[i];
    const double ms = t[i + 1] - t[i];
    std::string ops;
    for (size_t j = 0; j < st.op_ids.size(); ++j) ops += (j ? "," : "") + std::to_string(st.op_ids[j]);
    auto &m = meta[i];
    m = {keep("operations"), keep(ops), keep("device"), keep(std::to_string(s->device))};
    if (st.flop > 0) {
      m.insert(m.end(), {keep("flop"), keep(num(st.flop)), keep("tflops"), keep(num(st.flop / (ms * 1e-3) / 1e12))});
    }
    if (st.bytes > 0) {
      m.insert(m.end(), {keep("bytes"), keep(num(st.bytes)), keep("gbs"), keep(num(st.bytes / (ms * 1e-3) / 1e9))});
    }
    ipug_profile_sample &sm = samples[i];
    std::memset(&sm, 0, sizeof sm);
    sm.local_index = static_cast<uint32_t>(i);
    sm.phase = static_cast<uint32_t>(i);
    sm.kind = IPUG_STEP_COMPUTE;
    sm.operation = keep("operation." + std::to_string(st.op_ids.empty() ? -1 : st.op_ids.front()));
    sm.kernel = keep(st.label);
    sm.metadata = m.data();
    sm.metadata_count = static_cast<uint32_t>(m.size() / 2);
    sm.start_cycle = cycles(t[i]);
    sm.end_cycle = cycles(t[i + 1]);
  }
  const ipug_profile_tile tile = {physical_tile, samples.data(), n};
  return ipug_profile_encode(1000000000ull, &tile, 1, buf, size, needed);
}

const char *ipug_session_plan(const ipug_session *s) { return s ? s->plan.c_str() : ""; }

}  // extern "C"
