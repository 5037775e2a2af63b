// ComputeGraph builder, per-GPU shard lowering onto the ipuc_* kernels, and
// the device session (include/ipug.h).
//
// Graph semantics follow crates/ipu-codegen/src/graph.rs (value ids in
// construction order, shape inference graph.rs:661-760, numpy broadcasting
// graph.rs:762-788, value sequences graph.rs:294-313 and structured Repeat
// regions graph.rs:382-473).  The lowering replaces lower_to_tiles /
// lower_operator (crates/ipu-codegen/src/low.rs:443,1673-1709) in four passes:
//
//   flatten   Repeat regions are unrolled into straight-line operations, one
//             copy of the body per iteration (carried values threaded through,
//             iterated sequences indexed), as the evaluator runs them
//             (crates/ipu-tests/src/diagnostic.rs:467-520).
//   shard     for a world of N GPUs each rank derives its own shard of the
//             work from the graph: a GEMM of a replicated activation by a
//             weight whose result only feeds column-local consumers (GELU,
//             SplitHeads -> FlashAttention -> MergeHeads) splits the weight by
//             columns; a GEMM of such a column-split activation by a weight
//             splits the weight by rows and yields a partial sum; partial sums
//             add, and a replicated operand of such an add is added by rank 0
//             alone.  Where a consumer needs the whole value, an NCCL
//             all-reduce (partial sums) or all-gather (column shards) is
//             inserted.  Everything else is computed replicated.  With N = 1
//             this pass is the identity.
//   lower     one stream-ordered ipuc_* call (or collective) per operation,
//             fusing a GEMM into a single GELU or Add consumer through the GEMM
//             epilogue, and SplitHeads x3 -> FlashAttention -> MergeHeads into
//             one strided-heads attention call.
//   session   per-value device buffers, host/device I/O by graph value id,
//             run, event-timed profiles and the per-op diagnostic, mirroring
//             ipu-runtime (crates/ipu-runtime/src/lib.rs:12-48).
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <functional>
#include <map>
#include <memory>
#include <mutex>
#include <sstream>
#include <string>
#include <vector>

#include "../../include/ipug.h"

namespace ipuc {
void set_error(const std::string &msg);
ipuc_status fail(ipuc_status st, const std::string &msg);
ipuc_status cuda_fail(cudaError_t err, const char *what);
}  // namespace ipuc

namespace {

enum class OpKind { Gemm, Gelu, Add, SplitHeads, MergeHeads, FlashAttention, Repeat, AllReduce, AllGatherColumns };

struct Op;
struct RepeatInfo {
  uint32_t count = 0;
  int32_t carried = 0, invariants = 0;
  std::vector<int32_t> sequences;  // iterated value sequences
  std::vector<int32_t> arguments;  // carried, invariants, iterated
  std::vector<Op> body;
  std::vector<int32_t> yields;
};

struct Op {
  Op() = default;
  Op(OpKind k, std::vector<int32_t> in, std::vector<int32_t> res) : kind(k), inputs(std::move(in)), results(std::move(res)) {}
  OpKind kind = OpKind::Gemm;
  std::vector<int32_t> inputs;
  std::vector<int32_t> results;
  int32_t id = -1;  // operation id in construction order (body operations included)
  bool transpose_left = false, transpose_right = false;
  uint32_t heads = 0;
  bool causal = false;
  float scale = 0.0f;
  std::shared_ptr<RepeatInfo> repeat;
  int32_t result() const { return results.empty() ? -1 : results[0]; }
};

struct Value {
  std::vector<uint32_t> shape;
  int kind;  // 0 host input, 1 parameter, 2 op result, 3 region argument
  std::string name;
};

struct Sequence {
  std::string name;
  std::vector<int32_t> values;
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

// A Repeat body under construction (RegionBuilder, graph.rs:516-600): its
// operations and the values visible inside it (its arguments and the results
// of its own operations).
struct Frame {
  std::shared_ptr<RepeatInfo> info;
  std::vector<int32_t> inputs;  // carried + invariant operands of the Repeat
  std::vector<bool> visible;    // by value id
};

}  // namespace

struct ipug_graph {
  std::vector<Value> values;
  std::vector<Op> ops;  // top level
  std::vector<int32_t> outputs;
  std::vector<Sequence> sequences;
  std::unique_ptr<Frame> frame;  // open Repeat body, if any
  int32_t next_op = 0;

  bool valid(int32_t v) const { return v >= 0 && v < (int32_t)values.size(); }
  // A value an operation may use here: top-level values outside a region;
  // the region's arguments and its own results inside one.
  bool usable(int32_t v) const {
    if (!valid(v)) return false;
    if (frame) return v < (int32_t)frame->visible.size() && frame->visible[v];
    return values[v].kind != 3 && !body_value(v);
  }
  std::vector<bool> body_values;  // by value id: defined inside a region
  bool body_value(int32_t v) const { return v < (int32_t)body_values.size() && body_values[v]; }

  int32_t add_value(std::vector<uint32_t> shape, int kind, std::string name) {
    values.push_back(Value{std::move(shape), kind, std::move(name)});
    const int32_t id = (int32_t)values.size() - 1;
    body_values.resize(values.size(), false);
    if (frame) {
      body_values[id] = true;
      frame->visible.resize(values.size(), false);
      frame->visible[id] = true;
    }
    return id;
  }

  int32_t add_op(Op op, std::vector<uint32_t> shape) {
    for (int32_t v : op.inputs)
      if (!usable(v)) {
        ipuc::set_error("value " + std::to_string(v) + " is not available in this operation list");
        return -1;
      }
    op.results = {add_value(std::move(shape), 2, "")};
    op.id = next_op++;
    (frame ? frame->info->body : ops).push_back(op);
    return op.results[0];
  }
};

namespace {

// ---------------------------------------------------------------------------
// flatten: straight-line operations over "flat" values
// ---------------------------------------------------------------------------

enum class Shard { None, Columns, Rows };

struct FlatValue {
  std::vector<uint32_t> shape;
  int kind = 2;              // 0 host input, 1 parameter, 2 op result
  int32_t producer = -1;     // flat op index
  int32_t graph_value = -1;  // the graph value (top level; -1 inside unrolled bodies)
  // shard pass: how a parameter is sliced on this rank
  Shard slice = Shard::None;
  uint32_t slice0 = 0, slice1 = 0;  // [columns or rows) of the full parameter
  std::vector<uint32_t> full_shape;
};

struct FlatOp {
  OpKind kind;
  std::vector<int32_t> inputs;
  int32_t result = -1;
  int32_t graph_op = -1;  // operation id
  int32_t iteration = -1; // Repeat iteration (-1 at top level)
  bool transpose_left = false, transpose_right = false;
  uint32_t heads = 0;
  bool causal = false;
  float scale = 0.0f;
};

struct FlatGraph {
  std::vector<FlatValue> values;
  std::vector<FlatOp> ops;
  std::vector<int32_t> outputs;
  std::vector<int32_t> of_graph;  // graph value id -> flat value id (-1: none)
  int32_t add_value(std::vector<uint32_t> shape, int kind, int32_t producer, int32_t graph_value) {
    FlatValue v;
    v.shape = std::move(shape);
    v.full_shape = v.shape;
    v.kind = kind;
    v.producer = producer;
    v.graph_value = graph_value;
    values.push_back(v);
    return (int32_t)values.size() - 1;
  }
};

void flatten_ops(const ipug_graph &g, const std::vector<Op> &ops, std::vector<int32_t> &map, FlatGraph &f,
                 int32_t iteration, bool top) {
  for (const Op &op : ops) {
    if (op.kind == OpKind::Repeat) {
      const RepeatInfo &r = *op.repeat;
      std::vector<int32_t> carried, invariant;
      for (int32_t i = 0; i < r.carried; ++i) carried.push_back(map[op.inputs[i]]);
      for (int32_t i = 0; i < r.invariants; ++i) invariant.push_back(map[op.inputs[r.carried + i]]);
      for (uint32_t it = 0; it < r.count; ++it) {
        std::vector<int32_t> local = map;
        size_t a = 0;
        for (int32_t c : carried) local[r.arguments[a++]] = c;
        for (int32_t c : invariant) local[r.arguments[a++]] = c;
        for (int32_t sq : r.sequences) local[r.arguments[a++]] = map[g.sequences[sq].values[it]];
        flatten_ops(g, r.body, local, f, (int32_t)it, false);
        for (size_t y = 0; y < r.yields.size(); ++y) carried[y] = local[r.yields[y]];
      }
      for (size_t i = 0; i < op.results.size(); ++i) {
        map[op.results[i]] = carried[i];  // the last iteration's yields, no copy
        if (top && f.values[carried[i]].graph_value < 0) f.values[carried[i]].graph_value = op.results[i];
      }
      continue;
    }
    FlatOp fo;
    fo.kind = op.kind;
    for (int32_t v : op.inputs) fo.inputs.push_back(map[v]);
    fo.graph_op = op.id;
    fo.iteration = iteration;
    fo.transpose_left = op.transpose_left;
    fo.transpose_right = op.transpose_right;
    fo.heads = op.heads;
    fo.causal = op.causal;
    fo.scale = op.scale;
    const int32_t res = op.result();
    fo.result = f.add_value(g.values[res].shape, 2, (int32_t)f.ops.size(), top ? res : -1);
    map[res] = fo.result;
    f.ops.push_back(fo);
  }
}

FlatGraph flatten(const ipug_graph &g) {
  FlatGraph f;
  std::vector<int32_t> map(g.values.size(), -1);
  for (size_t v = 0; v < g.values.size(); ++v)
    if ((g.values[v].kind == 0 || g.values[v].kind == 1) && !g.body_value((int32_t)v))
      map[v] = f.add_value(g.values[v].shape, g.values[v].kind, -1, (int32_t)v);
  flatten_ops(g, g.ops, map, f, -1, true);
  for (int32_t o : g.outputs) f.outputs.push_back(map[o]);
  f.of_graph = map;
  for (size_t v = 0; v < g.values.size(); ++v)
    if (g.body_value((int32_t)v) || g.values[v].kind == 3) f.of_graph[v] = -1;
  return f;
}

// ---------------------------------------------------------------------------
// shard: this rank's part of the flat graph
// ---------------------------------------------------------------------------

enum class State { R, C, H, P };  // replicated, column shard, head shard, partial sum

struct ShardResult {
  FlatGraph local;
  std::vector<int32_t> local_of;   // flat value -> local value (-1: not materialised here)
  std::vector<State> state;        // by local value
};

ShardResult shard(const FlatGraph &f, int rank, int world) {
  ShardResult out;
  const size_t nv = f.values.size(), no = f.ops.size();
  std::vector<std::vector<int32_t>> consumers(nv);
  for (size_t i = 0; i < no; ++i)
    for (int32_t v : f.ops[i].inputs) consumers[v].push_back((int32_t)i);
  std::vector<bool> is_output(nv, false);
  for (int32_t v : f.outputs) is_output[v] = true;
  // A parameter matrix: [k, n], or with leading unit dimensions ([1, k, n]).
  auto is_param2d = [&](int32_t v) {
    const auto &s = f.values[v].shape;
    if (f.values[v].kind != 1 || s.size() < 2) return false;
    for (size_t i = 0; i + 2 < s.size(); ++i)
      if (s[i] != 1) return false;
    return true;
  };

  // Candidates for a column split: GEMMs of a 2-D parameter (no transposes)
  // whose column count divides by the world size.
  std::vector<bool> colpar(no, false);
  if (world > 1)
    for (size_t i = 0; i < no; ++i) {
      const FlatOp &op = f.ops[i];
      colpar[i] = op.kind == OpKind::Gemm && !op.transpose_left && !op.transpose_right && is_param2d(op.inputs[1]) &&
                  f.values[op.inputs[1]].shape.back() % world == 0;
    }
  // Column-sharded values under the current candidate set.
  std::vector<bool> cval(nv, false), hval(nv, false);
  auto recompute_states = [&]() {
    std::fill(cval.begin(), cval.end(), false);
    std::fill(hval.begin(), hval.end(), false);
    for (size_t i = 0; i < no; ++i) {
      const FlatOp &op = f.ops[i];
      bool c = false, h = false;
      switch (op.kind) {
        case OpKind::Gemm: c = colpar[i]; break;
        case OpKind::Gelu: c = cval[op.inputs[0]]; break;
        case OpKind::SplitHeads: h = cval[op.inputs[0]] && op.heads % world == 0; break;
        case OpKind::FlashAttention:
          h = !op.causal && hval[op.inputs[0]] && hval[op.inputs[1]] && hval[op.inputs[2]];
          break;
        case OpKind::MergeHeads: c = hval[op.inputs[0]]; break;
        default: break;
      }
      cval[op.result] = c;
      hval[op.result] = h;
    }
  };
  // Every use of a parameter must agree on how it is sliced.
  auto param_uses_ok = [&](int32_t p, bool rows) {
    for (int32_t c : consumers[p]) {
      const FlatOp &u = f.ops[c];
      if (u.kind != OpKind::Gemm || u.inputs[1] != p || u.inputs[0] == p) return false;
      if (rows ? !cval[u.inputs[0]] : !colpar[c]) return false;
    }
    return !is_output[p];
  };
  // A column-sharded value is fine if every consumer can work on its shard.
  std::vector<int> memo;
  std::function<bool(int32_t)> c_ok, h_ok;
  c_ok = [&](int32_t v) -> bool {
    if (is_output[v] || consumers[v].empty()) return false;
    for (int32_t ci : consumers[v]) {
      const FlatOp &c = f.ops[ci];
      switch (c.kind) {
        case OpKind::Gelu:
          if (!c_ok(c.result)) return false;
          break;
        case OpKind::Gemm:  // row split of the weight: a partial sum
          if (c.inputs[0] != v || c.inputs[1] == v || c.transpose_left || c.transpose_right ||
              !is_param2d(c.inputs[1]) || !param_uses_ok(c.inputs[1], true))
            return false;
          break;
        case OpKind::SplitHeads:
          if (c.heads % world || !h_ok(c.result)) return false;
          break;
        default:
          return false;
      }
    }
    return true;
  };
  h_ok = [&](int32_t v) -> bool {
    if (is_output[v] || consumers[v].empty()) return false;
    for (int32_t ci : consumers[v]) {
      const FlatOp &c = f.ops[ci];
      if (c.kind != OpKind::FlashAttention || c.causal) return false;
      for (int32_t in : c.inputs)
        if (!hval[in]) return false;
      if (is_output[c.result] || consumers[c.result].empty()) return false;
      for (int32_t mi : consumers[c.result]) {
        const FlatOp &m = f.ops[mi];
        if (m.kind != OpKind::MergeHeads || m.heads != f.ops[f.values[v].producer].heads || !c_ok(m.result))
          return false;
      }
    }
    return true;
  };
  for (bool changed = world > 1; changed;) {
    changed = false;
    recompute_states();
    for (size_t i = 0; i < no; ++i)
      // a GEMM of a column-split activation is the row split of the pair, not a new column split
      if (colpar[i] && (cval[f.ops[i].inputs[0]] || !c_ok(f.ops[i].result) ||
                        !param_uses_ok(f.ops[i].inputs[1], false))) {
        colpar[i] = false;  // in program order, one at a time: later states depend on it
        changed = true;
        break;
      }
  }
  recompute_states();

  // Emit this rank's graph.
  FlatGraph &L = out.local;
  out.local_of.assign(nv, -1);
  std::vector<State> &st = out.state;
  std::vector<int32_t> as_replicated(nv, -1);  // flat value -> local value holding it whole
  auto add_local = [&](std::vector<uint32_t> shape, int kind, State s, int32_t graph_value) {
    const int32_t id = L.add_value(std::move(shape), kind, -1, graph_value);
    st.push_back(s);
    return id;
  };
  auto emit = [&](FlatOp op, std::vector<uint32_t> shape, State s, int32_t graph_value) {
    op.result = add_local(std::move(shape), 2, s, graph_value);
    L.values[op.result].producer = (int32_t)L.ops.size();
    L.ops.push_back(op);
    return op.result;
  };
  // The whole value of flat value v on this rank (inserting a collective).
  auto whole = [&](int32_t v) -> int32_t {
    const int32_t lv = out.local_of[v];
    if (st[lv] == State::R) return lv;
    if (as_replicated[v] >= 0) return as_replicated[v];
    FlatOp c;
    c.inputs = {lv};
    c.graph_op = f.values[v].producer >= 0 ? f.ops[f.values[v].producer].graph_op : -1;
    if (st[lv] == State::P) {
      c.kind = OpKind::AllReduce;
    } else if (st[lv] == State::C) {
      c.kind = OpKind::AllGatherColumns;
    } else {
      return -1;  // head shards are never needed whole (h_ok)
    }
    L.values[lv].graph_value = -1;  // the graph value is the whole one
    return as_replicated[v] = emit(c, f.values[v].shape, State::R, f.values[v].graph_value);
  };
  const uint32_t w = (uint32_t)world, r = (uint32_t)rank;
  for (size_t v = 0; v < nv; ++v) {
    const FlatValue &fv = f.values[v];
    if (fv.kind == 2) continue;
    bool cols = false, rows = false;
    if (world > 1 && fv.kind == 1 && !consumers[v].empty() && is_param2d((int32_t)v)) {
      cols = param_uses_ok((int32_t)v, false);
      rows = !cols && param_uses_ok((int32_t)v, true) && fv.shape[fv.shape.size() - 2] % w == 0;
    }
    std::vector<uint32_t> shape = fv.shape;
    const int32_t lv = add_local(shape, fv.kind, State::R, fv.graph_value);
    FlatValue &x = L.values[lv];
    x.full_shape = fv.shape;
    if (cols) {
      const uint32_t part = fv.shape.back() / w;
      x.slice = Shard::Columns;
      x.slice0 = r * part;
      x.slice1 = (r + 1) * part;
      x.shape.back() = part;
      st[lv] = State::C;
    } else if (rows) {
      const uint32_t part = fv.shape[fv.shape.size() - 2] / w;
      x.slice = Shard::Rows;
      x.slice0 = r * part;
      x.slice1 = (r + 1) * part;
      x.shape[x.shape.size() - 2] = part;
      st[lv] = State::C;  // sliced, not whole
    }
    out.local_of[v] = lv;
  }
  for (size_t i = 0; i < no; ++i) {
    const FlatOp &op = f.ops[i];
    const FlatValue &res = f.values[op.result];
    FlatOp lo = op;
    std::vector<uint32_t> shape = res.shape;
    State s = State::R;
    auto in_state = [&](int k) { return st[out.local_of[op.inputs[k]]]; };
    auto local = [&](int k) { return out.local_of[op.inputs[k]]; };
    bool whole_inputs = true;
    int32_t alias = -1;  // result aliases an input (rank-0-only add on another rank)
    switch (op.kind) {
      case OpKind::Gemm:
        if (colpar[i]) {
          lo.inputs = {whole(op.inputs[0]), local(1)};
          shape.back() /= w;
          s = State::C;
          whole_inputs = false;
        } else if (world > 1 && cval[op.inputs[0]] && L.values[local(1)].slice == Shard::Rows) {
          lo.inputs = {local(0), local(1)};
          s = State::P;
          whole_inputs = false;
        }
        break;
      case OpKind::Gelu:
        if (in_state(0) == State::C) {
          lo.inputs = {local(0)};
          shape = L.values[local(0)].shape;
          s = State::C;
          whole_inputs = false;
        }
        break;
      case OpKind::SplitHeads:
        if (in_state(0) == State::C && hval[op.result]) {
          lo.inputs = {local(0)};
          shape[0] /= w;
          s = State::H;
          whole_inputs = false;
        }
        break;
      case OpKind::FlashAttention:
        if (in_state(0) == State::H && in_state(1) == State::H && in_state(2) == State::H) {
          lo.inputs = {local(0), local(1), local(2)};
          shape = L.values[local(0)].shape;
          shape.back() = L.values[local(2)].shape.back();
          s = State::H;
          whole_inputs = false;
        }
        break;
      case OpKind::MergeHeads:
        if (in_state(0) == State::H) {
          lo.inputs = {local(0)};
          shape.back() /= w;
          s = State::C;
          whole_inputs = false;
        }
        break;
      case OpKind::Add: {
        const State a = in_state(0), b = in_state(1);
        const auto &sa = f.values[op.inputs[0]].shape, &sb = f.values[op.inputs[1]].shape;
        if (a == State::P && b == State::P) {
          lo.inputs = {local(0), local(1)};
          s = State::P;
          whole_inputs = false;
        } else if ((a == State::P || b == State::P) && sa == sb) {
          // partial + whole: rank 0 adds the whole operand, the others pass
          // their partial sum on unchanged
          const int k = a == State::P ? 0 : 1;
          s = State::P;
          whole_inputs = false;
          if (rank == 0) lo.inputs = {local(k), whole(op.inputs[1 - k])};
          else alias = local(k);
        } else if (a == State::C && b == State::C && L.values[local(0)].shape == L.values[local(1)].shape &&
                   sa == sb) {
          lo.inputs = {local(0), local(1)};
          shape = L.values[local(0)].shape;
          s = State::C;
          whole_inputs = false;
        }
        break;
      }
      default:
        break;
    }
    if (whole_inputs) {
      lo.inputs.clear();
      for (int32_t in : op.inputs) lo.inputs.push_back(whole(in));
    }
    if (alias >= 0) {
      out.local_of[op.result] = alias;
      continue;
    }
    out.local_of[op.result] = emit(lo, shape, s, s == State::R ? res.graph_value : -1);
  }
  for (int32_t o : f.outputs) L.outputs.push_back(whole(o));
  // graph value ids of sharded values point at nothing whole on this rank
  L.of_graph.assign(f.of_graph.size(), -1);
  for (size_t gv = 0; gv < f.of_graph.size(); ++gv) {
    const int32_t fv = f.of_graph[gv];
    if (fv < 0) continue;
    const int32_t lv = as_replicated[fv] >= 0 ? as_replicated[fv] : out.local_of[fv];
    L.of_graph[gv] = lv;
  }
  return out;
}

// ---------------------------------------------------------------------------
// lower: steps over buffer slots
// ---------------------------------------------------------------------------

enum class StepKind { Gemm, Gelu, Add, SplitHeads, MergeHeads, Attention, AttentionHeads, Copy, AllReduce, AllGather };

struct Step {
  StepKind kind;
  std::vector<int32_t> op_ids;  // graph operation ids
  int32_t iteration = -1;
  int32_t out = -1, in0 = -1, in1 = -1, in2 = -1, tmp = -1;  // local value ids
  int32_t addend = -1;  // Gemm: value the epilogue adds (the fused Add's other operand)
  int64_t batch = 1, m = 0, n = 0, k = 0;
  uint32_t flags = 0;
  uint64_t count = 0, right_period = 0;
  int64_t b = 0, rows = 0, heads = 0, channels = 0;
  int64_t streams = 0, sq = 0, sk = 0, d = 0;
  float scale = 0.0f;
  double flop = 0.0, bytes = 0.0;
  std::string label;
};

struct Lowered {
  std::vector<Step> steps;
  std::vector<bool> has_buffer;  // by local value
  std::vector<uint64_t> extra_bytes;  // by local value: scratch beyond the value (all-gather staging)
  std::string plan;
};

ipuc_status lower(const FlatGraph &g, int rank, int world, bool fuse, Lowered &out) {
  const size_t nv = g.values.size();
  std::vector<std::vector<int32_t>> consumers(nv);
  for (size_t i = 0; i < g.ops.size(); ++i)
    for (int32_t v : g.ops[i].inputs) consumers[v].push_back((int32_t)i);
  std::vector<bool> is_output(nv, false);
  for (int32_t v : g.outputs) is_output[v] = true;
  std::vector<bool> fused_into_next(g.ops.size(), false);  // handled by a consumer's step
  std::vector<int32_t> fused_gemm(g.ops.size(), -1);        // consumer op -> gemm op
  for (size_t i = 0; fuse && i < g.ops.size(); ++i) {
    const FlatOp &op = g.ops[i];
    if (op.kind != OpKind::Gemm) continue;
    const int32_t r = op.result;
    if (is_output[r] || consumers[r].size() != 1) continue;
    const int32_t c = consumers[r][0];
    const FlatOp &co = g.ops[c];
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
  // every intermediate used once and not an output, lowers to one attention
  // call on the unsplit [b, rows, heads * c] values.
  std::vector<int32_t> fused_attention(g.ops.size(), -1);
  auto single_use = [&](int32_t v) { return !is_output[v] && consumers[v].size() == 1; };
  for (size_t i = 0; fuse && i < g.ops.size(); ++i) {
    const FlatOp &at = g.ops[i];
    if (at.kind != OpKind::FlashAttention || at.causal || !single_use(at.result)) continue;
    const FlatOp &mg = g.ops[consumers[at.result][0]];
    if (mg.kind != OpKind::MergeHeads) continue;
    bool ok = true;
    for (int32_t in : at.inputs) {
      const FlatValue &val = g.values[in];
      if (val.kind != 2 || !single_use(in)) {
        ok = false;
        break;
      }
      const FlatOp &sp = g.ops[val.producer];
      ok = ok && sp.kind == OpKind::SplitHeads && sp.heads == mg.heads && g.values[sp.inputs[0]].shape.size() == 3;
    }
    if (!ok) continue;
    fused_attention[consumers[at.result][0]] = (int32_t)i;
    fused_into_next[i] = true;
    for (int32_t in : at.inputs) fused_into_next[g.values[in].producer] = true;
  }

  auto gemm_step = [&](const FlatOp &op, Step &st) -> ipuc_status {
    const auto &L = g.values[op.inputs[0]].shape, &R = g.values[op.inputs[1]].shape;
    const uint32_t m = op.transpose_left ? L[L.size() - 1] : L[L.size() - 2];
    const uint32_t k = op.transpose_left ? L[L.size() - 2] : L[L.size() - 1];
    const uint32_t n = op.transpose_right ? R[R.size() - 2] : R[R.size() - 1];
    const std::vector<uint32_t> lb(L.begin(), L.end() - 2), rb(R.begin(), R.end() - 2);
    if (rb.empty() || numel(rb) == 1) {
      if (op.transpose_left && numel(lb) > 1) {
        // [batch, k, m] left operand with a shared right: batched GEMMs
        st.batch = (int64_t)numel(lb);
        st.m = m;
      } else {
        st.batch = 1;
        st.m = (int64_t)numel(lb) * m;  // flatten the left batch into rows
      }
    } else if (lb == rb) {
      st.batch = (int64_t)numel(lb);
      st.m = m;
    } else {
      return ipuc::fail(IPUC_ERR_UNSUPPORTED, "lowering: Gemm batch broadcasting other than a 2-D right operand");
    }
    st.n = n;
    st.k = k;
    st.flags |= op.transpose_right ? (uint32_t)IPUC_GEMM_B_TRANSPOSED : 0u;
    st.flags |= op.transpose_left ? (uint32_t)IPUC_GEMM_A_TRANSPOSED : 0u;
    st.in0 = op.inputs[0];
    st.in1 = op.inputs[1];
    st.flop = 2.0 * (double)st.batch * (double)st.m * (double)n * (double)k;
    return IPUC_OK;
  };

  out.steps.clear();
  out.extra_bytes.assign(nv, 0);
  for (size_t i = 0; i < g.ops.size(); ++i) {
    const FlatOp &op = g.ops[i];
    if (fused_into_next[i]) continue;
    Step st;
    st.op_ids.push_back(op.graph_op);
    st.iteration = op.iteration;
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
          const FlatOp &gm = g.ops[fused_gemm[i]];
          st.kind = StepKind::Gemm;
          st.op_ids.insert(st.op_ids.begin(), gm.graph_op);
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
          const FlatOp &gm = g.ops[fused_gemm[i]];
          const int32_t other = op.inputs[0] == gm.result ? op.inputs[1] : op.inputs[0];
          st.kind = StepKind::Gemm;
          st.op_ids.insert(st.op_ids.begin(), gm.graph_op);
          rc = gemm_step(gm, st);
          st.flags |= IPUC_GEMM_ACCUMULATE;
          st.label = "gemm_f16+add";
          if (st.batch == 1) {
            st.addend = other;  // the GEMM epilogue reads it: no copy
          } else {
            // Batched: copy the addend into the output, then accumulate onto it.
            Step cp;
            cp.kind = StepKind::Copy;
            cp.op_ids.push_back(op.graph_op);
            cp.iteration = op.iteration;
            cp.in0 = other;
            cp.out = op.result;
            cp.count = numel(g.values[op.result].shape);
            cp.bytes = 4.0 * cp.count;
            cp.label = "copy(addend)";
            out.steps.push_back(cp);
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
        st.heads = (int64_t)x[2] / (int64_t)(g.values[op.result].shape[2]);
        st.channels = g.values[op.result].shape[2];
        st.bytes = 4.0 * numel(x);
        st.label = "split_heads_f16";
        break;
      }
      case OpKind::MergeHeads: {
        const int64_t heads_here = (int64_t)g.values[op.result].shape[2] / (int64_t)g.values[op.inputs[0]].shape[2];
        if (fused_attention[i] >= 0) {
          const FlatOp &at = g.ops[fused_attention[i]];
          const FlatOp &sq = g.ops[g.values[at.inputs[0]].producer], &sk = g.ops[g.values[at.inputs[1]].producer],
                       &sv = g.ops[g.values[at.inputs[2]].producer];
          const auto &qx = g.values[sq.inputs[0]].shape, &kx = g.values[sk.inputs[0]].shape,
                     &vx = g.values[sv.inputs[0]].shape;
          if (qx[0] != kx[0] || kx != vx || qx[2] != kx[2]) {
            rc = ipuc::fail(IPUC_ERR_UNSUPPORTED, "lowering: attention needs equal batch and width for q, k and v");
            break;
          }
          st.kind = StepKind::AttentionHeads;
          st.op_ids = {sq.graph_op, sk.graph_op, sv.graph_op, at.graph_op, op.graph_op};
          st.in0 = sq.inputs[0];
          st.in1 = sk.inputs[0];
          st.in2 = sv.inputs[0];
          st.b = qx[0];
          st.heads = heads_here;
          st.sq = qx[1];
          st.sk = kx[1];
          st.d = qx[2] / heads_here;
          st.streams = st.b * st.heads;
          st.scale = at.scale;
          st.flop = 4.0 * st.streams * st.sq * st.sk * st.d;
          st.label = "flash_attention_heads_f16";
          break;
        }
        st.kind = StepKind::MergeHeads;
        const auto &x = g.values[op.inputs[0]].shape;
        st.in0 = op.inputs[0];
        st.heads = heads_here;
        st.b = x[0] / heads_here;
        st.rows = x[1];
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
      case OpKind::AllReduce:
        st.kind = StepKind::AllReduce;
        st.in0 = op.inputs[0];
        st.count = numel(g.values[op.result].shape);
        st.bytes = 2.0 * st.count;
        st.label = "nccl_all_reduce";
        break;
      case OpKind::AllGatherColumns: {
        st.kind = StepKind::AllGather;
        st.in0 = op.inputs[0];
        const auto &x = g.values[op.inputs[0]].shape;
        st.channels = x.back();
        st.rows = (int64_t)(numel(x) / x.back());
        st.heads = world;
        st.count = numel(x);
        st.bytes = 2.0 * st.count * world;
        out.extra_bytes[op.result] = st.count * 2 * (uint64_t)world;  // gathered [world, rows, columns/world]
        st.label = "nccl_all_gather+merge";
        break;
      }
      case OpKind::Repeat:
        rc = ipuc::fail(IPUC_ERR_UNSUPPORTED, "lowering: nested Repeat");
        break;
    }
    if (rc != IPUC_OK) return rc;
    out.steps.push_back(st);
  }
  std::ostringstream plan;
  for (const Step &st : out.steps) {
    plan << st.label << " ops=";
    for (size_t j = 0; j < st.op_ids.size(); ++j) plan << (j ? "," : "") << st.op_ids[j];
    plan << " out=";
    const int32_t gv = g.values[st.out].graph_value;
    if (gv >= 0) plan << "v" << gv;
    else plan << "l" << st.out;
    plan << shape_str(g.values[st.out].shape);
    if (st.iteration >= 0) plan << " iter=" << st.iteration;
    plan << "\n";
  }
  if (world > 1) {
    std::ostringstream head;
    head << "# rank " << rank << " of " << world << "\n";
    out.plan = head.str() + plan.str();
  } else {
    out.plan = plan.str();
  }
  // Buffers: every value except the results of operations fused into a consumer.
  out.has_buffer.assign(nv, false);
  for (size_t v = 0; v < nv; ++v) {
    const FlatValue &val = g.values[v];
    out.has_buffer[v] = !(val.kind == 2 && fused_into_next[val.producer]);
  }
  return IPUC_OK;
}

// ---------------------------------------------------------------------------
// NCCL, resolved at run time (only sharded sessions need it)
// ---------------------------------------------------------------------------

struct Nccl {
  decltype(&ncclGetUniqueId) get_unique_id = nullptr;
  decltype(&ncclCommInitRank) comm_init_rank = nullptr;
  decltype(&ncclCommDestroy) comm_destroy = nullptr;
  decltype(&ncclAllReduce) all_reduce = nullptr;
  decltype(&ncclAllGather) all_gather = nullptr;
  decltype(&ncclGetErrorString) error_string = nullptr;
  bool ok = false;
};

const Nccl &nccl() {
  static Nccl n;
  static std::once_flag once;
  std::call_once(once, [] {
    // The NCCL already in the process (e.g. torch's) first, else the system one.
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    n.get_unique_id = reinterpret_cast<decltype(n.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    n.comm_init_rank = reinterpret_cast<decltype(n.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    n.comm_destroy = reinterpret_cast<decltype(n.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    n.all_reduce = reinterpret_cast<decltype(n.all_reduce)>(dlsym(h, "ncclAllReduce"));
    n.all_gather = reinterpret_cast<decltype(n.all_gather)>(dlsym(h, "ncclAllGather"));
    n.error_string = reinterpret_cast<decltype(n.error_string)>(dlsym(h, "ncclGetErrorString"));
    n.ok = n.get_unique_id && n.comm_init_rank && n.comm_destroy && n.all_reduce && n.all_gather && n.error_string;
  });
  return n;
}

ipuc_status nccl_fail(ncclResult_t r, const char *what) {
  const Nccl &n = nccl();
  return ipuc::fail(IPUC_ERR_NCCL, std::string(what) + ": " + (n.error_string ? n.error_string(r) : "nccl error"));
}

struct DeviceGuard {
  int prev = 0;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    cudaSetDevice(dev);
  }
  ~DeviceGuard() { cudaSetDevice(prev); }
};

}  // namespace

struct ipug_session {
  const ipug_graph *graph = nullptr;
  int device = 0, rank = 0, world = 1;
  FlatGraph local;            // this rank's graph
  std::vector<State> state;   // by local value
  Lowered lowered;
  std::vector<void *> buffers;  // by local value; nullptr = fused away
  std::vector<void *> extra;    // by local value: all-gather staging
  ncclComm_t comm = nullptr;
  // Peer-memory all-reduce (ipug_session_peer_reduce): this process's mapping
  // of every rank's buffer, by local value, and of every rank's signal area.
  bool peer = false, peer_mapped = false;
  void *signal = nullptr;
  std::vector<void *> peer_signal;
  std::map<int32_t, std::vector<void *>> peer_buffers;
  std::vector<void *> peer_opened;  // mappings of other ranks' memory, closed at exit
  ~ipug_session() {
    bool any = comm != nullptr;
    for (void *p : buffers) any = any || p != nullptr;
    if (!any) return;  // a plan-only lowering holds no device memory
    DeviceGuard guard(device);
    for (void *p : buffers)
      if (p) cudaFree(p);
    for (void *p : extra)
      if (p) cudaFree(p);
    for (void *p : peer_opened) ipuc_ipc_close(p);
    if (signal) cudaFree(signal);
    if (comm) nccl().comm_destroy(comm);
  }
};

namespace {

ipuc_status build(const ipug_graph &g, const ipug_session_options &o, ipug_session &s) {
  if (g.frame) return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, "session: a Repeat body is still open");
  if (o.world < 1 || o.rank < 0 || o.rank >= o.world)
    return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, "session: rank must lie in [0, world)");
  s.graph = &g;
  s.device = o.device;
  s.rank = o.rank;
  s.world = o.world;
  const FlatGraph flat = flatten(g);
  ShardResult sr = shard(flat, o.rank, o.world);
  s.local = std::move(sr.local);
  s.state = std::move(sr.state);
  return lower(s.local, o.rank, o.world, o.fuse != 0, s.lowered);
}

ipuc_status allocate(ipug_session &s) {
  const size_t nv = s.local.values.size();
  s.buffers.assign(nv, nullptr);
  s.extra.assign(nv, nullptr);
  for (size_t v = 0; v < nv; ++v) {
    if (!s.lowered.has_buffer[v]) continue;
    const uint64_t bytes = std::max<uint64_t>(numel(s.local.values[v].shape) * 2, 16);
    cudaError_t e = cudaMalloc(&s.buffers[v], bytes);
    if (e == cudaSuccess && s.lowered.extra_bytes[v]) e = cudaMalloc(&s.extra[v], s.lowered.extra_bytes[v]);
    if (e != cudaSuccess) return ipuc::fail(IPUC_ERR_CUDA, std::string("session: cudaMalloc: ") + cudaGetErrorString(e));
  }
  return IPUC_OK;
}

ipuc_status run_step(ipug_session &s, const Step &st, cudaStream_t stream) {
  auto P = [&](int32_t v) { return s.buffers[v]; };
  switch (st.kind) {
    case StepKind::Gemm: {
      const bool at = (st.flags & IPUC_GEMM_A_TRANSPOSED) != 0;
      const int64_t lda = at ? st.m : st.k, ldb = (st.flags & IPUC_GEMM_B_TRANSPOSED) ? st.k : st.n, ldc = st.n;
      const uint64_t rb = numel(s.local.values[st.in1].shape);
      const int64_t sb = (st.batch > 1 && rb > (uint64_t)(st.n * st.k)) ? st.n * st.k : 0;  // shared right: stride 0
      if (st.batch == 1 && st.addend >= 0)
        return ipuc_gemm_f16_addend(P(st.out), P(st.in0), P(st.in1), st.m, st.n, st.k, lda, ldb, ldc, st.flags,
                                    P(st.addend), st.n, stream);
      if (st.batch == 1)
        return ipuc_gemm_f16(P(st.out), P(st.in0), P(st.in1), st.m, st.n, st.k, lda, ldb, ldc, st.flags, stream);
      return ipuc_gemm_f16_batched(P(st.out), P(st.in0), P(st.in1), st.batch, st.m, st.n, st.k, lda, ldb, ldc,
                                   st.m * st.k, sb, st.m * st.n, st.flags, stream);
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
    case StepKind::AllReduce: {
      if (s.peer) {
        const auto in = s.peer_buffers.find(st.in0), out = s.peer_buffers.find(st.out);
        if (in != s.peer_buffers.end() && out != s.peer_buffers.end())
          return ipuc_peer_all_reduce_f16(in->second.data(), out->second.data(), s.peer_signal.data(), s.rank,
                                          s.world, st.count, stream);
      }
      const ncclResult_t r = nccl().all_reduce(P(st.in0), P(st.out), st.count, ncclFloat16, ncclSum, s.comm, stream);
      return r == ncclSuccess ? IPUC_OK : nccl_fail(r, "session all-reduce");
    }
    case StepKind::AllGather: {
      const ncclResult_t r = nccl().all_gather(P(st.in0), s.extra[st.out], st.count, ncclFloat16, s.comm, stream);
      if (r != ncclSuccess) return nccl_fail(r, "session all-gather");
      // [world, rows, columns/world] -> [rows, columns]
      return ipuc_merge_heads_f16(P(st.out), s.extra[st.out], 1, st.rows, st.heads, st.channels, stream);
    }
  }
  return IPUC_OK;
}

int32_t checked(ipug_graph *g, Op op, bool ok, const std::string &why, std::vector<uint32_t> shape) {
  if (!g) {
    ipuc::set_error("null graph");
    return -1;
  }
  for (int32_t v : op.inputs)
    if (!g->usable(v)) {
      ipuc::set_error("value " + std::to_string(v) + " is not available in this operation list");
      return -1;
    }
  if (!ok) {
    ipuc::set_error("operation has invalid shapes: " + why);
    return -1;
  }
  return g->add_op(op, std::move(shape));
}

ipug_session_options default_options(int32_t device) {
  ipug_session_options o;
  std::memset(&o, 0, sizeof o);
  o.device = device;
  o.rank = 0;
  o.world = 1;
  o.fuse = 1;
  return o;
}

}  // namespace

extern "C" {

ipug_graph *ipug_graph_create(void) { return new ipug_graph(); }
void ipug_graph_destroy(ipug_graph *g) { delete g; }

static int32_t add_input(ipug_graph *g, const char *name, const uint32_t *dims, int32_t rank, int kind) {
  if (!g || !name || !*name) {
    ipuc::set_error("graph name must not be empty");
    return -1;
  }
  if (g->frame) {
    ipuc::set_error("inputs cannot be added inside a Repeat body");
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
  return g->add_value(shape, kind, name);
}

int32_t ipug_host_input(ipug_graph *g, const char *name, const uint32_t *dims, int32_t rank) {
  return add_input(g, name, dims, rank, 0);
}
int32_t ipug_parameter(ipug_graph *g, const char *name, const uint32_t *dims, int32_t rank) {
  return add_input(g, name, dims, rank, 1);
}

int32_t ipug_gemm(ipug_graph *g, int32_t left, int32_t right, int32_t transpose_left, int32_t transpose_right) {
  Op op{OpKind::Gemm, {left, right}, {}};
  op.transpose_left = transpose_left != 0;
  op.transpose_right = transpose_right != 0;
  if (!g || !g->usable(left) || !g->usable(right)) return checked(g, op, false, "unknown value", {});
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
  Op op{OpKind::Gelu, {input}, {}};
  if (!g || !g->usable(input)) return checked(g, op, false, "unknown value", {});
  return checked(g, op, true, "", g->values[input].shape);
}

int32_t ipug_add(ipug_graph *g, int32_t left, int32_t right) {
  Op op{OpKind::Add, {left, right}, {}};
  if (!g || !g->usable(left) || !g->usable(right)) return checked(g, op, false, "unknown value", {});
  std::vector<uint32_t> out;
  const bool ok = broadcast(g->values[left].shape, g->values[right].shape, out);
  return checked(g, op, ok, "Add shapes cannot be broadcast", out);
}

int32_t ipug_split_heads(ipug_graph *g, int32_t input, uint32_t heads) {
  Op op{OpKind::SplitHeads, {input}, {}};
  op.heads = heads;
  if (!g || !g->usable(input)) return checked(g, op, false, "unknown value", {});
  const auto &x = g->values[input].shape;  // graph.rs:704-727
  if (x.size() != 3 || heads == 0)
    return checked(g, op, false, "split_heads requires nonzero heads and [batch, rows, channels] input", {});
  if (x[2] % heads) return checked(g, op, false, "split_heads channels must be divisible by heads", {});
  return checked(g, op, true, "", {x[0] * heads, x[1], x[2] / heads});
}

int32_t ipug_merge_heads(ipug_graph *g, int32_t input, uint32_t heads) {
  Op op{OpKind::MergeHeads, {input}, {}};
  op.heads = heads;
  if (!g || !g->usable(input)) return checked(g, op, false, "unknown value", {});
  const auto &x = g->values[input].shape;
  if (x.size() != 3 || heads == 0 || x[0] % heads)
    return checked(g, op, false, "merge_heads requires [batch*heads, rows, channels] input with heads dividing dim 0", {});
  return checked(g, op, true, "", {x[0] / heads, x[1], x[2] * heads});
}

int32_t ipug_flash_attention(ipug_graph *g, int32_t query, int32_t key, int32_t value, int32_t causal, float scale) {
  Op op{OpKind::FlashAttention, {query, key, value}, {}};
  op.causal = causal != 0;
  op.scale = scale;
  if (!g || !g->usable(query) || !g->usable(key) || !g->usable(value)) return checked(g, op, false, "unknown value", {});
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

int32_t ipug_value_sequence(ipug_graph *g, const char *name, const int32_t *values, int32_t count) {
  if (!g || !name || !*name) {
    ipuc::set_error("graph name must not be empty");
    return -1;
  }
  if (g->frame) {
    ipuc::set_error("value sequences cannot be created inside a Repeat body");
    return -1;
  }
  if (count < 0 || (count > 0 && !values)) {
    ipuc::set_error("value_sequence: bad arguments");
    return -1;
  }
  for (int32_t i = 0; i < count; ++i)
    if (!g->usable(values[i])) {
      ipuc::set_error("value " + std::to_string(values[i]) + " is not available in this operation list");
      return -1;
    }
  for (int32_t i = 1; i < count; ++i)  // graph.rs:302-308
    if (g->values[values[i]].shape != g->values[values[0]].shape) {
      ipuc::set_error("value sequence entry " + std::to_string(i) + " has a different shape from its first entry");
      return -1;
    }
  g->sequences.push_back(Sequence{name, std::vector<int32_t>(values, values + count)});
  return (int32_t)g->sequences.size() - 1;
}

ipuc_status ipug_repeat_begin(ipug_graph *g, uint32_t count, const int32_t *carried, int32_t carried_count,
                              const int32_t *invariants, int32_t invariant_count, const int32_t *sequences,
                              int32_t sequence_count, int32_t *arguments) {
  if (!g) return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, "repeat: null graph");
  if (g->frame) return ipuc::fail(IPUC_ERR_UNSUPPORTED, "repeat: nested Repeat bodies are not supported");
  if (count == 0) return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, "repeat count must be nonzero");
  if (carried_count < 0 || invariant_count < 0 || sequence_count < 0 || (carried_count && !carried) ||
      (invariant_count && !invariants) || (sequence_count && !sequences) || !arguments)
    return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, "repeat: bad arguments");
  std::vector<int32_t> ins;
  for (int32_t i = 0; i < carried_count; ++i) ins.push_back(carried[i]);
  for (int32_t i = 0; i < invariant_count; ++i) ins.push_back(invariants[i]);
  for (int32_t v : ins)
    if (!g->usable(v))
      return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT,
                        "value " + std::to_string(v) + " is not available in this operation list");
  for (int32_t i = 0; i < sequence_count; ++i) {
    const int32_t sq = sequences[i];
    if (sq < 0 || sq >= (int32_t)g->sequences.size())
      return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, "value sequence " + std::to_string(sq) + " does not exist");
    if (g->sequences[sq].values.size() < count)  // graph.rs:404-409
      return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT,
                        "value sequence " + std::to_string(sq) + " has " +
                            std::to_string(g->sequences[sq].values.size()) + " entries for " + std::to_string(count) +
                            " iterations");
  }
  auto info = std::make_shared<RepeatInfo>();
  info->count = count;
  info->carried = carried_count;
  info->invariants = invariant_count;
  info->sequences.assign(sequences, sequences + sequence_count);
  std::vector<std::vector<uint32_t>> shapes;
  for (int32_t v : ins) shapes.push_back(g->values[v].shape);
  for (int32_t sq : info->sequences) shapes.push_back(g->values[g->sequences[sq].values[0]].shape);
  std::unique_ptr<Frame> fr(new Frame());
  fr->info = info;
  fr->inputs = ins;
  g->frame = std::move(fr);
  g->frame->visible.assign(g->values.size(), false);
  for (size_t a = 0; a < shapes.size(); ++a) {
    const int32_t id = g->add_value(shapes[a], 3, "");
    info->arguments.push_back(id);
    arguments[a] = id;
  }
  return IPUC_OK;
}

int32_t ipug_repeat_end(ipug_graph *g, const int32_t *yields, int32_t yield_count, int32_t *results) {
  if (!g || !g->frame) {
    ipuc::set_error("repeat_end: no Repeat body is open");
    return -1;
  }
  std::unique_ptr<Frame> fr = std::move(g->frame);  // the body closes whatever happens next
  RepeatInfo &info = *fr->info;
  if (yield_count != info.carried) {
    ipuc::set_error("repeat body yielded " + std::to_string(yield_count) + " values for " +
                    std::to_string(info.carried) + " carried values");
    return -1;
  }
  if (yield_count && (!yields || !results)) {
    ipuc::set_error("repeat_end: bad arguments");
    return -1;
  }
  for (int32_t i = 0; i < yield_count; ++i) {
    const int32_t y = yields[i];
    if (!g->valid(y) || y >= (int32_t)fr->visible.size() || !fr->visible[y]) {
      ipuc::set_error("value " + std::to_string(y) + " is not available in this operation list");
      return -1;
    }
    if (g->values[y].shape != g->values[fr->inputs[i]].shape) {
      ipuc::set_error("repeat yield " + std::to_string(i) + " does not have the shape of carried value " +
                      std::to_string(i));
      return -1;
    }
    info.yields.push_back(y);
  }
  Op op{OpKind::Repeat, fr->inputs, {}};
  op.repeat = fr->info;
  op.id = g->next_op++;
  for (int32_t i = 0; i < yield_count; ++i) {
    op.results.push_back(g->add_value(g->values[fr->inputs[i]].shape, 2, ""));
    results[i] = op.results.back();
  }
  g->ops.push_back(op);
  return yield_count;
}

ipuc_status ipug_set_outputs(ipug_graph *g, const int32_t *values, int32_t count) {
  if (!g || count < 0 || (count > 0 && !values)) return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, "set_outputs: bad arguments");
  if (g->frame) return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, "set_outputs: a Repeat body is still open");
  for (int32_t i = 0; i < count; ++i)
    if (!g->usable(values[i]))
      return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT,
                        "value " + std::to_string(values[i]) + " is not available in this operation list");
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

ipuc_status ipug_nccl_unique_id(void *out, uint64_t size) {
  if (!out || size < sizeof(ncclUniqueId))
    return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, "nccl_unique_id: needs a 128-byte buffer");
  const Nccl &n = nccl();
  if (!n.ok) return ipuc::fail(IPUC_ERR_NCCL, "nccl_unique_id: libnccl.so.2 could not be loaded");
  ncclUniqueId id;
  const ncclResult_t r = n.get_unique_id(&id);
  if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
  std::memcpy(out, &id, sizeof id);
  return IPUC_OK;
}

ipug_session *ipug_session_open_ex(const ipug_graph *g, const ipug_session_options *options, ipuc_status *status) {
  auto set = [&](ipuc_status st) {
    if (status) *status = st;
  };
  if (!g || !options) {
    set(ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, "session_open: null graph or options"));
    return nullptr;
  }
  if (options->world > 1 && !options->nccl_id) {
    set(ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, "session_open: a sharded session needs the NCCL unique id"));
    return nullptr;
  }
  DeviceGuard guard(options->device);
  std::unique_ptr<ipug_session> s(new ipug_session());
  ipuc_status st = build(*g, *options, *s);
  if (st == IPUC_OK && options->world > 1) {
    const Nccl &n = nccl();
    if (!n.ok) {
      st = ipuc::fail(IPUC_ERR_NCCL, "session_open: libnccl.so.2 could not be loaded");
    } else {
      ncclUniqueId id;
      std::memcpy(&id, options->nccl_id, sizeof id);
      const ncclResult_t r = n.comm_init_rank(&s->comm, options->world, id, options->rank);
      if (r != ncclSuccess) {
        s->comm = nullptr;
        st = nccl_fail(r, "ncclCommInitRank");
      }
    }
  }
  if (st == IPUC_OK) st = allocate(*s);
  set(st);
  if (st != IPUC_OK) return nullptr;
  return s.release();
}

ipug_session *ipug_session_open(const ipug_graph *g, int32_t device, ipuc_status *status) {
  const ipug_session_options o = default_options(device);
  return ipug_session_open_ex(g, &o, status);
}

void ipug_session_close(ipug_session *s) { delete s; }

ipuc_status ipug_graph_plan_ex(const ipug_graph *g, const ipug_session_options *options, char *buf, uint64_t size,
                               uint64_t *needed) {
  if (!g || !options) return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, "graph_plan: null graph or options");
  ipug_session s;
  const ipuc_status st = build(*g, *options, s);
  if (st != IPUC_OK) return st;
  const std::string &plan = s.lowered.plan;
  if (needed) *needed = plan.size() + 1;
  if (!buf || size < plan.size() + 1) return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, "graph_plan: buffer too small");
  std::memcpy(buf, plan.c_str(), plan.size() + 1);
  return IPUC_OK;
}

ipuc_status ipug_graph_plan(const ipug_graph *g, char *buf, uint64_t size, uint64_t *needed) {
  const ipug_session_options o = default_options(0);
  return ipug_graph_plan_ex(g, &o, buf, size, needed);
}

ipuc_status ipug_graph_shard_json(const ipug_graph *g, int32_t rank, int32_t world, char *buf, uint64_t size,
                                  uint64_t *needed) {
  if (!g) return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, "graph_shard_json: null graph");
  if (g->frame) return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, "graph_shard_json: a Repeat body is still open");
  if (world < 1 || rank < 0 || rank >= world)
    return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, "graph_shard_json: rank must lie in [0, world)");
  const ShardResult sr = shard(flatten(*g), rank, world);
  const FlatGraph &L = sr.local;
  static const char *kinds[] = {"gemm", "gelu", "add", "split_heads", "merge_heads", "flash_attention", "repeat",
                                "all_reduce", "all_gather_columns"};
  static const char *states[] = {"replicated", "columns", "heads", "partial"};
  std::ostringstream o;
  o << "{\"rank\": " << rank << ", \"world\": " << world << ", \"values\": [";
  for (size_t v = 0; v < L.values.size(); ++v) {
    const FlatValue &x = L.values[v];
    o << (v ? ", " : "") << "{\"id\": " << v << ", \"shape\": [";
    for (size_t i = 0; i < x.shape.size(); ++i) o << (i ? ", " : "") << x.shape[i];
    o << "], \"kind\": " << x.kind << ", \"graph_value\": " << x.graph_value << ", \"state\": \""
      << states[(int)sr.state[v]] << "\"";
    if (x.slice != Shard::None)
      o << ", \"slice\": \"" << (x.slice == Shard::Columns ? "columns" : "rows") << "\", \"range\": [" << x.slice0
        << ", " << x.slice1 << "]";
    o << "}";
  }
  o << "], \"ops\": [";
  for (size_t i = 0; i < L.ops.size(); ++i) {
    const FlatOp &op = L.ops[i];
    o << (i ? ", " : "") << "{\"kind\": \"" << kinds[(int)op.kind] << "\", \"inputs\": [";
    for (size_t j = 0; j < op.inputs.size(); ++j) o << (j ? ", " : "") << op.inputs[j];
    o << "], \"result\": " << op.result << ", \"op\": " << op.graph_op << ", \"iteration\": " << op.iteration
      << ", \"transpose_left\": " << (op.transpose_left ? "true" : "false")
      << ", \"transpose_right\": " << (op.transpose_right ? "true" : "false") << ", \"heads\": " << op.heads
      << ", \"causal\": " << (op.causal ? "true" : "false") << ", \"scale\": " << op.scale << "}";
  }
  o << "], \"outputs\": [";
  for (size_t i = 0; i < L.outputs.size(); ++i) o << (i ? ", " : "") << L.outputs[i];
  o << "]}";
  const std::string js = o.str();
  if (needed) *needed = js.size() + 1;
  if (!buf || size < js.size() + 1) return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, "graph_shard_json: buffer too small");
  std::memcpy(buf, js.c_str(), js.size() + 1);
  return IPUC_OK;
}

// The local value holding graph value `value`, and the bytes of its whole
// (graph) shape and of what this rank holds.
static ipuc_status locate(ipug_session *s, int32_t value, int32_t &lv, uint64_t &whole, uint64_t &here) {
  if (!s || !s->graph->valid(value)) return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, "session: unknown value");
  if (value >= (int32_t)s->local.of_graph.size() || s->local.of_graph[value] < 0)
    return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT,
                      "session: value lives inside a Repeat body (or is sharded away on this rank)");
  lv = s->local.of_graph[value];
  if (!s->buffers[lv])
    return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, "session: value was fused into its consumer and has no buffer");
  whole = numel(s->graph->values[value].shape) * 2;
  here = numel(s->local.values[lv].shape) * 2;
  return IPUC_OK;
}

ipuc_status ipug_session_write(ipug_session *s, int32_t value, const void *src, uint64_t bytes, ipuc_stream stream) {
  int32_t lv = -1;
  uint64_t whole = 0, here = 0;
  ipuc_status st = locate(s, value, lv, whole, here);
  if (st != IPUC_OK) return st;
  const FlatValue &x = s->local.values[lv];
  DeviceGuard guard(s->device);
  cudaError_t e = cudaSuccess;
  if (bytes == whole && x.slice == Shard::Columns) {
    // this rank's columns of a row-major [rows, columns] parameter
    const size_t pitch = (size_t)x.full_shape.back() * 2, width = (size_t)(x.slice1 - x.slice0) * 2;
    e = cudaMemcpy2DAsync(s->buffers[lv], width, static_cast<const uint8_t *>(src) + (size_t)x.slice0 * 2, pitch,
                          width, numel(x.full_shape) / x.full_shape.back(), cudaMemcpyDefault, stream);
  } else if (bytes == whole && x.slice == Shard::Rows) {
    const size_t row = (size_t)x.full_shape.back() * 2;
    e = cudaMemcpyAsync(s->buffers[lv], static_cast<const uint8_t *>(src) + (size_t)x.slice0 * row, here,
                        cudaMemcpyDefault, stream);
  } else if (bytes == here) {
    e = cudaMemcpyAsync(s->buffers[lv], src, bytes, cudaMemcpyDefault, stream);
  } else {
    return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, "session: byte count must be element count * 2 (f16)");
  }
  if (e != cudaSuccess) return ipuc::fail(IPUC_ERR_CUDA, std::string("session_write: ") + cudaGetErrorString(e));
  return IPUC_OK;
}

ipuc_status ipug_session_read(ipug_session *s, int32_t value, void *dst, uint64_t bytes, ipuc_stream stream) {
  int32_t lv = -1;
  uint64_t whole = 0, here = 0;
  ipuc_status st = locate(s, value, lv, whole, here);
  if (st != IPUC_OK) return st;
  if (bytes != here)
    return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT,
                      here == whole ? "session: byte count must be element count * 2 (f16)"
                                    : "session: this rank holds a shard of the value: read its shard's bytes");
  DeviceGuard guard(s->device);
  cudaError_t e = cudaMemcpyAsync(dst, s->buffers[lv], bytes, cudaMemcpyDefault, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return ipuc::fail(IPUC_ERR_CUDA, std::string("session_read: ") + cudaGetErrorString(e));
  return IPUC_OK;
}

void *ipug_session_device_ptr(ipug_session *s, int32_t value) {
  int32_t lv = -1;
  uint64_t whole = 0, here = 0;
  if (locate(s, value, lv, whole, here) != IPUC_OK) return nullptr;
  return s->buffers[lv];
}

ipuc_status ipug_session_run(ipug_session *s, ipuc_stream stream) {
  if (!s) return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, "session_run: null session");
  DeviceGuard guard(s->device);
  for (const Step &st : s->lowered.steps) {
    const ipuc_status rc = run_step(*s, st, stream);
    if (rc != IPUC_OK) return rc;
  }
  return IPUC_OK;
}

namespace {
// One exchanged entry: a CUDA IPC handle and the pointer's offset inside its allocation.
constexpr uint64_t kIpcEntry = 72;

ipuc_status exchange_peer_maps(ipug_session &s, cudaStream_t stream) {
  std::vector<int32_t> values;
  for (const Step &st : s.lowered.steps) {
    if (st.kind != StepKind::AllReduce || st.count % (8ull * (uint64_t)s.world) != 0) continue;
    for (int32_t v : {st.in0, st.out})
      if (std::find(values.begin(), values.end(), v) == values.end()) values.push_back(v);
  }
  const uint64_t sig_bytes = ipuc_peer_signal_bytes();
  cudaError_t me = cudaMalloc(&s.signal, sig_bytes);
  if (me == cudaSuccess) me = cudaMemsetAsync(s.signal, 0, sig_bytes, stream);
  if (me != cudaSuccess) return ipuc::cuda_fail(me, "session peer-reduce signal area");
  const uint64_t entries = values.size() + 1, blob = entries * kIpcEntry;
  std::vector<uint8_t> mine(blob), all(blob * (uint64_t)s.world);
  for (uint64_t e = 0; e < entries; ++e) {
    void *p = e == 0 ? s.signal : s.buffers[values[e - 1]];
    uint64_t offset = 0;
    if (ipuc_status st = ipuc_ipc_handle(p, mine.data() + e * kIpcEntry, 64, &offset)) return st;
    std::memcpy(mine.data() + e * kIpcEntry + 64, &offset, 8);
  }
  void *send = nullptr, *recv = nullptr;
  cudaError_t ce = cudaMalloc(&send, blob);
  if (ce == cudaSuccess) ce = cudaMalloc(&recv, blob * (uint64_t)s.world);
  ncclResult_t nr = ncclSuccess;
  if (ce == cudaSuccess) ce = cudaMemcpyAsync(send, mine.data(), blob, cudaMemcpyHostToDevice, stream);
  // The gather also orders every rank's signal-area memset before any peer's first flag.
  if (ce == cudaSuccess) nr = nccl().all_gather(send, recv, blob, ncclUint8, s.comm, stream);
  if (ce == cudaSuccess && nr == ncclSuccess)
    ce = cudaMemcpyAsync(all.data(), recv, all.size(), cudaMemcpyDeviceToHost, stream);
  if (ce == cudaSuccess && nr == ncclSuccess) ce = cudaStreamSynchronize(stream);
  if (send) cudaFree(send);
  if (recv) cudaFree(recv);
  if (nr != ncclSuccess) return nccl_fail(nr, "session peer-reduce handle exchange");
  if (ce != cudaSuccess) return ipuc::cuda_fail(ce, "session peer-reduce handle exchange");
  s.peer_signal.assign(s.world, nullptr);
  for (int32_t v : values) s.peer_buffers[v].assign(s.world, nullptr);
  for (int32_t q = 0; q < s.world; ++q) {
    for (uint64_t e = 0; e < entries; ++e) {
      void *local = e == 0 ? s.signal : s.buffers[values[e - 1]];
      void *mapped = local;
      if (q != s.rank) {
        const uint8_t *entry = all.data() + (uint64_t)q * blob + e * kIpcEntry;
        uint64_t offset = 0;
        std::memcpy(&offset, entry + 64, 8);
        if (ipuc_status st = ipuc_ipc_open(entry, offset, &mapped)) return st;
        s.peer_opened.push_back(mapped);
      }
      if (e == 0) s.peer_signal[q] = mapped;
      else s.peer_buffers[values[e - 1]][q] = mapped;
    }
  }
  return IPUC_OK;
}
}  // namespace

ipuc_status ipug_session_peer_reduce(ipug_session *s, int32_t enable, ipuc_stream stream) {
  if (!s) return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, "session_peer_reduce: null session");
  if (s->world == 1 || s->world > 8 || s->buffers.empty()) {
    s->peer = false;
    return IPUC_OK;
  }
  if (!enable) {
    s->peer = false;
    return IPUC_OK;
  }
  if (!s->comm) return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, "session_peer_reduce: no communicator");
  DeviceGuard guard(s->device);
  if (!s->peer_mapped) {
    if (s->signal)
      return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT,
                        "session_peer_reduce: an earlier handle exchange failed; re-open the session");
    const ipuc_status st = exchange_peer_maps(*s, stream);
    if (st != IPUC_OK) return st;
    s->peer_mapped = true;
  }
  s->peer = true;
  return IPUC_OK;
}

ipuc_status ipug_session_diagnose(ipug_session *s, const int32_t *values, const float *const *reference,
                                  int32_t count, ipug_value_report *reports, ipuc_stream stream) {
  if (!s || count < 0 || (count > 0 && (!values || !reference || !reports)))
    return ipuc::fail(IPUC_ERR_INVALID_ARGUMENT, "session_diagnose: bad arguments");
  DeviceGuard guard(s->device);
  std::vector<uint16_t> host;
  for (int32_t i = 0; i < count; ++i) {
    ipug_value_report &r = reports[i];
    std::memset(&r, 0, sizeof r);
    r.value = values[i];
    int32_t lv = -1;
    uint64_t whole = 0, here = 0;
    if (!s->graph->valid(values[i]) || !reference[i] || locate(s, values[i], lv, whole, here) != IPUC_OK ||
        here != whole)
      continue;  // fused away, inside a Repeat body, or sharded on this rank: not available
    const uint64_t n = whole / 2;
    host.resize(n);
    cudaError_t e = cudaMemcpyAsync(host.data(), s->buffers[lv], whole, cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) return ipuc::fail(IPUC_ERR_CUDA, std::string("session_diagnose: ") + cudaGetErrorString(e));
    double err2 = 0.0, ref2 = 0.0, max_err = 0.0, max_ref = 0.0;
    uint64_t nonfinite = 0;
    for (uint64_t j = 0; j < n; ++j) {
      // f16 -> f64 (IEEE binary16)
      const uint16_t h = host[j];
      const int ex = (h >> 10) & 0x1f, man = h & 0x3ff;
      double x = ex == 0 ? std::ldexp((double)man, -24)
                         : (ex == 31 ? (man ? NAN : INFINITY) : std::ldexp((double)(man | 0x400), ex - 25));
      if (h & 0x8000) x = -x;
      const double ref = reference[i][j];
      if (!std::isfinite(x)) {
        ++nonfinite;
        continue;
      }
      const double d = x - ref;
      err2 += d * d;
      ref2 += ref * ref;
      max_err = std::max(max_err, std::fabs(d));
      max_ref = std::max(max_ref, std::fabs(ref));
    }
    r.available = 1;
    r.elements = n;
    r.nonfinite = nonfinite;
    r.max_abs_err = max_err;
    r.max_abs_ref = max_ref;
    r.rel_l2 = ref2 > 0 ? std::sqrt(err2 / ref2) : std::sqrt(err2);
    r.producer = -1;
    for (const Step &st : s->lowered.steps)
      if (st.out == lv) r.producer = st.op_ids.back();
  }
  return IPUC_OK;
}

}  // extern "C"

// Run every lowered step once with a CUDA event on each boundary; t[i] is the
// time of boundary i in ms after boundary 0 (t.size() == steps + 1).
static ipuc_status time_steps(ipug_session *s, ipuc_stream stream, std::vector<double> &t, const char *who) {
  DeviceGuard guard(s->device);
  const auto &steps = s->lowered.steps;
  std::vector<cudaEvent_t> ev(steps.size() + 1, nullptr);
  ipuc_status rc = IPUC_OK;
  for (auto &e : ev)
    if (rc == IPUC_OK && cudaEventCreate(&e) != cudaSuccess) rc = ipuc::fail(IPUC_ERR_CUDA, std::string(who) + ": cudaEventCreate");
  if (rc == IPUC_OK) {
    cudaEventRecord(ev[0], stream);
    for (size_t i = 0; i < steps.size() && rc == IPUC_OK; ++i) {
      rc = run_step(*s, steps[i], stream);
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
  const auto &steps = s->lowered.steps;
  std::ostringstream o;
  o << "{\"device\": " << s->device << ", \"rank\": " << s->rank << ", \"world\": " << s->world << ", \"steps\": [";
  for (size_t i = 0; i < steps.size(); ++i) {
    const double ms = t[i + 1] - t[i];
    const Step &st = steps[i];
    o << (i ? ", " : "") << "{\"step\": " << i << ", \"kernel\": \"" << st.label << "\", \"ops\": [";
    for (size_t j = 0; j < st.op_ids.size(); ++j) o << (j ? ", " : "") << st.op_ids[j];
    o << "], \"ms\": " << ms;
    if (st.iteration >= 0) o << ", \"iteration\": " << st.iteration;
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
  const auto &steps = s->lowered.steps;
  const size_t n = steps.size();
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
    const Step &st = steps[i];
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
    sm.kind = (st.kind == StepKind::AllReduce || st.kind == StepKind::AllGather) ? IPUG_STEP_EXCHANGE
                                                                                : IPUG_STEP_COMPUTE;
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

const char *ipug_session_plan(const ipug_session *s) { return s ? s->lowered.plan.c_str() : ""; }

}  // extern "C"
