// graph.cu -- host-side tracer for elementwise programs: record a DAG,
// differentiate it in reverse mode, fuse it into op-tapes, run it.
//
// The reference records Primitive applications in a thread-local TraceContext
// (src/trace/tracer.rs:22-165) as IRNodes (src/trace/ir.rs:8-386), groups
// consecutive elementwise nodes (find_fusible_groups, src/trace/fusion.rs:97-294),
// emits one shader per group (generate_fused_shader :296-346) and runs it
// (Interpreter::eval_fused_op src/trace/interpreter.rs:177-221,
// JitFunction::call src/trace/jit.rs:44-107).  Reverse mode is VJPEngine
// (src/trace/grad.rs:450-837) over the transpose rules of
// src/trace/transpose_rules.rs.  Here:
//
//   * jx_graph records nodes {input, const, unary, binary, select_gt} over
//     equal-length f32 vectors; identical nodes are shared (structural CSE),
//     so ids are in topological order by construction.
//   * jx_graph_vjp appends the adjoint nodes of the given outputs with respect
//     to the given nodes, one rule per op, contributions summed in the order
//     reverse traversal reaches them.  The rules follow transpose_rules.rs
//     (tanh 1-t^2 :136-154, exp :157-169, log x^-1 :171-178, sqrt (2 s)^-1
//     :180-199, reciprocal -(x^2)^-1 :201-212, square 2x :214-225, add/sub
//     :237-277, mul :279-307) in the same operation order, with three
//     corrections where the reference's rule is not the derivative: the
//     divisor of a/b gets -(a/b)/b (the reference has -a*ct, :310-346),
//     the base of a^b gets b*a^(b-1) (the reference has b, :348-400), and
//     abs gets sign(x) as a select pair.  relu, gelu and sigmoid, untraced in
//     the reference, get their derivatives (select, jx gelu_grad, s(1-s)).
//   * jx_graph_compile lowers the nodes the outputs need into op-tapes.  The
//     outputs go in groups of up to four whose dependency cones fit one tape
//     together (4 inputs, 4 outputs, 15 live registers -- one is left for the
//     tape's own power-of-two division rewrite -- 64 constants, 128
//     instructions); each tape recomputes what it needs from the program
//     inputs, since an elementwise value is cheaper to recompute than to
//     round-trip through HBM.  An output whose cone alone exceeds a tape is
//     split along its topological order into consecutive tapes, the values
//     crossing them in scratch buffers.  Program outputs go straight to the
//     caller's buffers.  Registers are assigned by a linear scan; constants
//     are loaded where first used.
#include <string.h>

#include <algorithm>
#include <map>
#include <set>
#include <tuple>
#include <vector>

#include "jx_common.cuh"

namespace {

enum Kind { K_INPUT = 0, K_CONST = 1, K_UN = 2, K_BIN = 3, K_SEL = 4 };

struct GNode {
  int kind, op, a, b;
  float value;  // K_CONST
  int input;    // K_INPUT: program input index
};

}  // namespace

struct jx_graph {
  std::vector<GNode> nodes;
  int n_inputs = 0;
  std::map<std::tuple<int, int, int, int, uint32_t>, int> cse;
};

struct jx_program {
  struct TapeRun {
    jx_tape* tape = nullptr;
    std::vector<int> in_vals;   // node ids read (graph inputs or earlier values)
    std::vector<int> out_vals;  // node ids written, one per store slot
  };
  std::vector<TapeRun> tapes;
  std::vector<int> input_nodes;  // graph input index -> node id (-1 when unused)
  std::vector<int> outputs;      // program output index -> node id
  std::vector<int> scratch_vals; // node ids kept in scratch buffers
  int n_inputs = 0;
};

namespace {

int add_node(jx_graph* g, int kind, int op, int a, int b, float value, int* out) {
  uint32_t vbits = 0;
  memcpy(&vbits, &value, 4);
  const auto key = std::make_tuple(kind, op, a, b, kind == K_CONST ? vbits : 0u);
  if (kind != K_INPUT) {
    auto it = g->cse.find(key);
    if (it != g->cse.end()) {
      *out = it->second;
      return JX_OK;
    }
  }
  GNode n{kind, op, a, b, value, -1};
  if (kind == K_INPUT) n.input = g->n_inputs++;
  g->nodes.push_back(n);
  const int id = (int)g->nodes.size() - 1;
  if (kind != K_INPUT) g->cse.emplace(key, id);
  *out = id;
  return JX_OK;
}

bool valid(const jx_graph* g, int id) { return id >= 0 && id < (int)g->nodes.size(); }

// Node builders used by the VJP rules (status ignored: operands are valid by construction).
struct B {
  jx_graph* g;
  int c(float v) { int r; add_node(g, K_CONST, 0, -1, -1, v, &r); return r; }
  int un(int op, int x) { int r; add_node(g, K_UN, op, x, -1, 0.f, &r); return r; }
  int bin(int op, int x, int y) { int r; add_node(g, K_BIN, op, x, y, 0.f, &r); return r; }
  int sel(int x, int y) { int r; add_node(g, K_SEL, 0, x, y, 0.f, &r); return r; }
  int add(int x, int y) { return bin(JX_BIN_ADD, x, y); }
  int sub(int x, int y) { return bin(JX_BIN_SUB, x, y); }
  int mul(int x, int y) { return bin(JX_BIN_MUL, x, y); }
  int div(int x, int y) { return bin(JX_BIN_DIV, x, y); }
  int neg(int x) { return un(JX_UN_NEG, x); }
  int recip(int x) { return un(JX_UN_RECIP, x); }
};

// ---- lowering ------------------------------------------------------------
struct Range {
  std::vector<int> ins, outs, consts;  // tape inputs (sorted), outputs (slot order), constants
  int instr = 0, regs = 0;
};

// Tape requirements of compute nodes order[s..e] (inclusive).
Range analyse(const jx_graph* g, const std::vector<int>& order, int s, int e, const std::vector<int>& last_use,
              const std::vector<char>& is_out, const std::vector<int>& pos, std::vector<int> extra_outs) {
  Range r;
  std::set<int> ins, consts;
  std::set<int> inrange;
  for (int i = s; i <= e; ++i) inrange.insert(order[i]);
  auto operand = [&](int v) {
    if (v < 0) return;
    const GNode& n = g->nodes[v];
    if (n.kind == K_CONST) consts.insert(v);
    else if (!inrange.count(v)) ins.insert(v);
  };
  for (int i = s; i <= e; ++i) {
    const GNode& n = g->nodes[order[i]];
    operand(n.a);
    if (n.kind != K_UN) operand(n.b);
  }
  // values that program outputs need from this tape, or that later tapes read
  std::vector<int> outs;
  for (int i = s; i <= e; ++i) {
    const int v = order[i];
    if (is_out[v] || last_use[v] > e) outs.push_back(v);
  }
  for (int v : extra_outs) {  // program outputs that are inputs/constants (stored by the last tape)
    const GNode& n = g->nodes[v];
    if (n.kind == K_CONST) consts.insert(v);
    else ins.insert(v);
    outs.push_back(v);
  }
  r.ins.assign(ins.begin(), ins.end());
  r.consts.assign(consts.begin(), consts.end());
  r.outs = outs;
  // linear scan: inputs occupy registers from the start, constants from their
  // first use, computed values from their definition; each is freed after its
  // last use inside the range (outputs are stored right after definition)
  std::map<int, int> last_in;  // value -> last position in [s, e] it is read
  for (int i = s; i <= e; ++i) {
    const GNode& n = g->nodes[order[i]];
    if (n.a >= 0) last_in[n.a] = i;
    if (n.kind != K_UN && n.b >= 0) last_in[n.b] = i;
  }
  int live = (int)r.ins.size(), peak = live;
  std::set<int> loaded;
  for (int v : extra_outs)
    if (g->nodes[v].kind == K_CONST) { ++live; peak = std::max(peak, live); --live; }
  for (int i = s; i <= e; ++i) {
    const GNode& n = g->nodes[order[i]];
    for (int opnd : {n.a, n.kind != K_UN ? n.b : -1}) {
      if (opnd >= 0 && g->nodes[opnd].kind == K_CONST && !loaded.count(opnd)) {
        loaded.insert(opnd);
        ++live;
      }
    }
    ++live;  // the result (its register may equal a freed operand's, counted after frees below)
    peak = std::max(peak, live);
    for (int opnd : {n.a, n.kind != K_UN ? n.b : -1}) {
      if (opnd < 0) continue;
      auto it = last_in.find(opnd);
      if (it != last_in.end() && it->second == i) {
        --live;
        if (g->nodes[opnd].kind == K_CONST) loaded.erase(opnd);
        last_in.erase(it);
      }
    }
    const int v = order[i];
    if (!last_in.count(v)) --live;  // not read again in the range: stored (if needed) and freed at once
    (void)pos;
  }
  r.regs = peak;
  r.instr = (e - s + 1) + (int)r.consts.size() + (int)r.outs.size();
  return r;
}

bool fits(const Range& r) {
  return (int)r.ins.size() <= JX_TAPE_MAX_IO && (int)r.outs.size() <= JX_TAPE_MAX_IO &&
         r.regs <= JX_TAPE_MAX_REGS - 1 && (int)r.consts.size() <= JX_TAPE_MAX_CONSTS &&
         r.instr + 8 <= JX_TAPE_MAX_INSTR;  // slack for constant reloads
}

// Emit one tape for the range; returns JX_OK and fills the TapeRun.
int emit(const jx_graph* g, const std::vector<int>& order, int s, int e, const Range& r,
         jx_program::TapeRun* tr) {
  std::vector<int32_t> code;
  std::vector<float> consts;
  std::map<int, int> reg_of;                 // value -> register
  std::vector<int> free_regs;
  for (int i = JX_TAPE_MAX_REGS - 2; i >= (int)r.ins.size(); --i) free_regs.push_back(i);  // keep reg 15 spare
  for (size_t i = 0; i < r.ins.size(); ++i) reg_of[r.ins[i]] = (int)i;
  std::map<int, int> const_slot;
  for (size_t i = 0; i < r.consts.size(); ++i) {
    const_slot[r.consts[i]] = (int)i;
    consts.push_back(g->nodes[r.consts[i]].value);
  }
  std::map<int, std::vector<int>> out_slots;  // value -> store slots
  for (size_t i = 0; i < r.outs.size(); ++i) out_slots[r.outs[i]].push_back((int)i);
  std::map<int, int> last_in;
  for (int i = s; i <= e; ++i) {
    const GNode& n = g->nodes[order[i]];
    if (n.a >= 0) last_in[n.a] = i;
    if (n.kind != K_UN && n.b >= 0) last_in[n.b] = i;
  }
  auto take = [&](int* reg) -> int {
    if (free_regs.empty()) return jx::fail(JX_EINTERNAL, "graph: register allocation overflow");
    *reg = free_regs.back();
    free_regs.pop_back();
    return JX_OK;
  };
  auto instr = [&](int op, int dst, int s0, int s1) {
    code.push_back(op);
    code.push_back(dst);
    code.push_back(s0);
    code.push_back(s1);
  };
  auto store_all = [&](int v, int reg) {
    auto it = out_slots.find(v);
    if (it == out_slots.end()) return;
    for (int slot : it->second) instr(JX_OP_STORE, slot, reg, 0);
    out_slots.erase(it);
  };
  // program outputs that are tape inputs or constants
  for (auto& kv : std::map<int, std::vector<int>>(out_slots)) {
    const int v = kv.first;
    if (g->nodes[v].kind == K_CONST) {
      int reg;
      int rc = take(&reg);
      if (rc) return rc;
      instr(JX_OP_CONST, reg, const_slot[v], 0);
      store_all(v, reg);
      free_regs.push_back(reg);
    } else if (reg_of.count(v) && (g->nodes[v].kind == K_INPUT || std::find(order.begin() + s, order.begin() + e + 1, v) ==
                                                                      order.begin() + e + 1)) {
      store_all(v, reg_of[v]);
    }
  }
  // inputs never read inside the range can be released
  for (int v : r.ins)
    if (!last_in.count(v)) free_regs.push_back(reg_of[v]);
  for (int i = s; i <= e; ++i) {
    const int v = order[i];
    const GNode& n = g->nodes[v];
    auto ld = [&](int opnd) -> int {
      if (g->nodes[opnd].kind == K_CONST && !reg_of.count(opnd)) {
        int reg;
        int rc = take(&reg);
        if (rc) return -1;
        instr(JX_OP_CONST, reg, const_slot[opnd], 0);
        reg_of[opnd] = reg;
      }
      return reg_of[opnd];
    };
    const int ra = ld(n.a);
    const int rb = n.kind != K_UN ? ld(n.b) : 0;
    if (ra < 0 || rb < 0) return jx::fail(JX_EINTERNAL, "graph: register allocation overflow");
    // free operands whose last use is here (before allocating the result, so it may reuse one)
    for (int opnd : {n.a, n.kind != K_UN ? n.b : -1}) {
      if (opnd < 0) continue;
      auto it = last_in.find(opnd);
      if (it != last_in.end() && it->second == i) {
        free_regs.push_back(reg_of[opnd]);
        reg_of.erase(opnd);
        last_in.erase(it);
      }
    }
    int rd;
    int rc = take(&rd);
    if (rc) return rc;
    if (n.kind == K_UN) instr(JX_OP_UNARY + n.op, rd, ra, 0);
    else if (n.kind == K_BIN) instr(JX_OP_BINARY + n.op, rd, ra, rb);
    else instr(JX_OP_SELECT_GT, rd, ra, rb);
    store_all(v, rd);
    if (last_in.count(v)) reg_of[v] = rd;
    else free_regs.push_back(rd);
  }
  if (!out_slots.empty()) return jx::fail(JX_EINTERNAL, "graph: an output of a tape was not stored");
  const int n_instr = (int)code.size() / 4;
  jx_tape* t = nullptr;
  int rc = jx_tape_create(code.data(), n_instr, consts.empty() ? nullptr : consts.data(), (int)consts.size(),
                          (int)r.ins.size(), (int)r.outs.size(), &t);
  if (rc) return rc;
  tr->tape = t;
  tr->in_vals = r.ins;
  tr->out_vals = r.outs;
  return JX_OK;
}

}  // namespace

extern "C" {

int jx_graph_create(jx_graph** out) {
  JX_TRACE("jx_graph_create");
  JX_REQUIRE(out, "jx_graph_create: NULL");
  *out = new jx_graph();
  return JX_OK;
}

int jx_graph_destroy(jx_graph* g) {
  JX_TRACE("jx_graph_destroy");
  delete g;
  return JX_OK;
}

int jx_graph_input(jx_graph* g, int* node) {
  JX_TRACE("jx_graph_input");
  JX_REQUIRE(g && node, "jx_graph_input: NULL");
  return add_node(g, K_INPUT, 0, -1, -1, 0.f, node);
}

int jx_graph_const(jx_graph* g, float value, int* node) {
  JX_TRACE("jx_graph_const");
  JX_REQUIRE(g && node, "jx_graph_const: NULL");
  return add_node(g, K_CONST, 0, -1, -1, value, node);
}

int jx_graph_unary(jx_graph* g, int op, int x, int* node) {
  JX_TRACE("jx_graph_unary");
  JX_REQUIRE(g && node, "jx_graph_unary: NULL");
  JX_REQUIRE(op >= JX_UN_NEG && op <= JX_UN_LOG2, "jx_graph_unary: unknown op %d", op);
  JX_REQUIRE(valid(g, x), "jx_graph_unary: operand %d is not a node of this graph", x);
  return add_node(g, K_UN, op, x, -1, 0.f, node);
}

int jx_graph_binary(jx_graph* g, int op, int x, int y, int* node) {
  JX_TRACE("jx_graph_binary");
  JX_REQUIRE(g && node, "jx_graph_binary: NULL");
  JX_REQUIRE(op >= JX_BIN_ADD && op <= JX_BIN_MAX, "jx_graph_binary: unknown op %d", op);
  JX_REQUIRE(valid(g, x) && valid(g, y), "jx_graph_binary: operand is not a node of this graph");
  return add_node(g, K_BIN, op, x, y, 0.f, node);
}

int jx_graph_select_gt(jx_graph* g, int x, int y, int* node) {
  JX_TRACE("jx_graph_select_gt");
  JX_REQUIRE(g && node, "jx_graph_select_gt: NULL");
  JX_REQUIRE(valid(g, x) && valid(g, y), "jx_graph_select_gt: operand is not a node of this graph");
  return add_node(g, K_SEL, 0, x, y, 0.f, node);
}

int jx_graph_size(const jx_graph* g, int* n_nodes, int* n_inputs) {
  JX_TRACE("jx_graph_size");
  JX_REQUIRE(g, "jx_graph_size: NULL");
  if (n_nodes) *n_nodes = (int)g->nodes.size();
  if (n_inputs) *n_inputs = g->n_inputs;
  return JX_OK;
}

int jx_graph_vjp(jx_graph* g, int n_out, const int* outs, const int* cts, int n_wrt, const int* wrt, int* grads) {
  JX_TRACE("jx_graph_vjp");
  JX_REQUIRE(g && n_out >= 1 && outs && cts && n_wrt >= 1 && wrt && grads, "jx_graph_vjp: bad arguments");
  for (int i = 0; i < n_out; ++i)
    JX_REQUIRE(valid(g, outs[i]) && valid(g, cts[i]), "jx_graph_vjp: output or cotangent is not a node");
  for (int i = 0; i < n_wrt; ++i) JX_REQUIRE(valid(g, wrt[i]), "jx_graph_vjp: wrt %d is not a node", i);
  const int n0 = (int)g->nodes.size();
  // nodes that depend on some wrt node (only they receive cotangents)
  std::vector<char> dep(n0, 0);
  for (int i = 0; i < n_wrt; ++i) dep[wrt[i]] = 1;
  for (int v = 0; v < n0; ++v) {
    const GNode& n = g->nodes[v];
    if (n.a >= 0 && dep[n.a]) dep[v] = 1;
    if (n.kind != K_UN && n.b >= 0 && dep[n.b]) dep[v] = 1;
  }
  std::vector<int> adj(n0, -1);
  B b{g};
  auto acc = [&](int u, int contrib) {
    if (u < 0 || !dep[u]) return;
    adj[u] = adj[u] < 0 ? contrib : b.add(adj[u], contrib);
  };
  for (int i = 0; i < n_out; ++i) acc(outs[i], cts[i]);
  for (int v = n0 - 1; v >= 0; --v) {
    const int gv = adj[v];
    if (gv < 0) continue;
    const GNode n = g->nodes[v];  // copy: builders may grow the vector
    const int x = n.a, y = n.b;
    if (n.kind == K_UN) {
      switch (n.op) {
        case JX_UN_NEG: acc(x, b.neg(gv)); break;
        case JX_UN_ABS: acc(x, b.sub(b.sel(x, gv), b.sel(b.neg(x), gv))); break;
        case JX_UN_SIN: acc(x, b.mul(gv, b.un(JX_UN_COS, x))); break;
        case JX_UN_COS: acc(x, b.mul(gv, b.neg(b.un(JX_UN_SIN, x)))); break;
        case JX_UN_TANH: acc(x, b.mul(gv, b.sub(b.c(1.0f), b.mul(v, v)))); break;
        case JX_UN_EXP: acc(x, b.mul(gv, v)); break;
        case JX_UN_LOG: acc(x, b.mul(gv, b.recip(x))); break;
        case JX_UN_SQRT: acc(x, b.mul(gv, b.recip(b.mul(b.c(2.0f), v)))); break;
        case JX_UN_RECIP: acc(x, b.mul(gv, b.neg(b.recip(b.mul(x, x))))); break;
        case JX_UN_SQUARE: acc(x, b.mul(gv, b.mul(b.c(2.0f), x))); break;
        case JX_UN_RELU: acc(x, b.sel(x, gv)); break;
        case JX_UN_GELU: acc(x, b.mul(gv, b.un(JX_UN_GELU_GRAD, x))); break;
        case JX_UN_SIGMOID: acc(x, b.mul(gv, b.mul(v, b.sub(b.c(1.0f), v)))); break;
        // transpose_tan (:123-134): sec^2 = (cos x * cos x)^-1
        case JX_UN_TAN: { const int cx = b.un(JX_UN_COS, x); acc(x, b.mul(gv, b.recip(b.mul(cx, cx)))); break; }
        // transpose_sign (:227-229) and the rounding family: zero almost everywhere
        case JX_UN_SIGN: case JX_UN_CEIL: case JX_UN_FLOOR: case JX_UN_ROUND: case JX_UN_TRUNC:
          acc(x, b.c(0.0f));
          break;
        case JX_UN_SINH: acc(x, b.mul(gv, b.un(JX_UN_COSH, x))); break;
        case JX_UN_COSH: acc(x, b.mul(gv, b.un(JX_UN_SINH, x))); break;
        case JX_UN_ASIN: acc(x, b.mul(gv, b.recip(b.un(JX_UN_SQRT, b.sub(b.c(1.0f), b.mul(x, x)))))); break;
        case JX_UN_ACOS: acc(x, b.neg(b.mul(gv, b.recip(b.un(JX_UN_SQRT, b.sub(b.c(1.0f), b.mul(x, x))))))); break;
        case JX_UN_ATAN: acc(x, b.mul(gv, b.recip(b.add(b.c(1.0f), b.mul(x, x))))); break;
        case JX_UN_ASINH: acc(x, b.mul(gv, b.recip(b.un(JX_UN_SQRT, b.add(b.mul(x, x), b.c(1.0f)))))); break;
        case JX_UN_ACOSH: acc(x, b.mul(gv, b.recip(b.un(JX_UN_SQRT, b.sub(b.mul(x, x), b.c(1.0f)))))); break;
        case JX_UN_ATANH: acc(x, b.mul(gv, b.recip(b.sub(b.c(1.0f), b.mul(x, x))))); break;
        case JX_UN_EXPM1: acc(x, b.mul(gv, b.add(v, b.c(1.0f)))); break;
        case JX_UN_LOG1P: acc(x, b.mul(gv, b.recip(b.add(b.c(1.0f), x)))); break;
        case JX_UN_CBRT: acc(x, b.mul(gv, b.recip(b.mul(b.c(3.0f), b.mul(v, v))))); break;
        case JX_UN_LOG2: acc(x, b.mul(gv, b.recip(b.mul(x, b.c(0.693147180559945309f))))); break;
        default:
          return jx::fail(JX_EUNSUPPORTED, "jx_graph_vjp: no derivative for unary op %d", n.op);
      }
    } else if (n.kind == K_BIN) {
      switch (n.op) {
        case JX_BIN_ADD: acc(x, gv); acc(y, gv); break;
        case JX_BIN_SUB: acc(x, gv); acc(y, b.neg(gv)); break;
        case JX_BIN_MUL: acc(x, b.mul(gv, y)); acc(y, b.mul(gv, x)); break;
        case JX_BIN_DIV: acc(x, b.mul(gv, b.recip(y))); acc(y, b.neg(b.mul(gv, b.div(v, y)))); break;
        case JX_BIN_POW:
          acc(x, b.mul(gv, b.mul(y, b.bin(JX_BIN_POW, x, b.sub(y, b.c(1.0f))))));
          acc(y, b.mul(gv, b.mul(v, b.un(JX_UN_LOG, x))));
          break;
        case JX_BIN_MAX: {  // ties go to the second operand
          const int m = b.sel(b.sub(x, y), gv);
          acc(x, m);
          acc(y, b.sub(gv, m));
          break;
        }
        case JX_BIN_MIN: {
          const int m = b.sel(b.sub(y, x), gv);
          acc(x, m);
          acc(y, b.sub(gv, m));
          break;
        }
        default:
          return jx::fail(JX_EUNSUPPORTED, "jx_graph_vjp: no derivative for binary op %d", n.op);
      }
    } else if (n.kind == K_SEL) {
      acc(y, b.sel(x, gv));  // the mask operand gets no cotangent
    }
  }
  for (int i = 0; i < n_wrt; ++i) grads[i] = adj[wrt[i]] >= 0 ? adj[wrt[i]] : b.c(0.0f);
  return JX_OK;
}

int jx_graph_compile(const jx_graph* g, int n_out, const int* outs, jx_program** out) {
  JX_TRACE("jx_graph_compile");
  JX_REQUIRE(g && out && n_out >= 1 && outs, "jx_graph_compile: bad arguments");
  for (int i = 0; i < n_out; ++i) JX_REQUIRE(valid(g, outs[i]), "jx_graph_compile: output %d is not a node", i);
  const int n = (int)g->nodes.size();
  std::vector<int> couts, passthrough;  // distinct computed outputs; outputs that are inputs or constants
  for (int i = 0; i < n_out; ++i) {
    std::vector<int>& dstv = g->nodes[outs[i]].kind >= K_UN ? couts : passthrough;
    if (std::find(dstv.begin(), dstv.end(), outs[i]) == dstv.end()) dstv.push_back(outs[i]);
  }
  // compute nodes a set of roots needs, in topological (id) order
  auto cone = [&](const std::vector<int>& roots) {
    std::vector<char> in(n, 0);
    for (int r : roots) in[r] = 1;
    for (int v = n - 1; v >= 0; --v) {
      if (!in[v]) continue;
      const GNode& nd = g->nodes[v];
      if (nd.a >= 0) in[nd.a] = 1;
      if (nd.kind != K_UN && nd.b >= 0) in[nd.b] = 1;
    }
    std::vector<int> ord;
    for (int v = 0; v < n; ++v)
      if (in[v] && g->nodes[v].kind >= K_UN) ord.push_back(v);
    return ord;
  };
  auto last_use_of = [&](const std::vector<int>& ord) {
    std::vector<int> lu(n, -1);
    for (size_t i = 0; i < ord.size(); ++i) {
      const GNode& nd = g->nodes[ord[i]];
      lu[nd.a] = std::max(lu[nd.a], (int)i);
      if (nd.kind != K_UN) lu[nd.b] = std::max(lu[nd.b], (int)i);
    }
    return lu;
  };
  auto flags = [&](const std::vector<int>& roots) {
    std::vector<char> f(n, 0);
    for (int r : roots) f[r] = 1;
    return f;
  };
  const std::vector<int> no_pos;
  auto* p = new jx_program();
  p->n_inputs = g->n_inputs;
  p->input_nodes.assign(g->n_inputs, -1);
  for (int v = 0; v < n; ++v)
    if (g->nodes[v].kind == K_INPUT) p->input_nodes[g->nodes[v].input] = v;
  p->outputs.assign(outs, outs + n_out);
  int rc = JX_OK;
  // Outputs in groups of up to four whose cones fit one tape; each tape
  // recomputes what it needs from the program inputs (elementwise values are
  // cheaper to recompute than to round-trip through HBM).
  for (size_t i = 0; !rc && i < couts.size();) {
    std::vector<int> grp = {couts[i]};
    std::vector<int> ord = cone(grp);
    Range r = analyse(g, ord, 0, (int)ord.size() - 1, last_use_of(ord), flags(grp), no_pos, {});
    if (!fits(r)) {
      // one output whose cone exceeds a tape: split its topological order into
      // consecutive tapes, values crossing them through scratch buffers
      const std::vector<int> lu = last_use_of(ord);
      const std::vector<char> of = flags(grp);
      const int m = (int)ord.size();
      for (int s0 = 0; !rc && s0 < m;) {
        int e = s0;
        Range best = analyse(g, ord, s0, e, lu, of, no_pos, {});
        if (!fits(best)) {
          rc = jx::fail(JX_EINTERNAL, "graph: node %d alone does not fit a tape", ord[s0]);
          break;
        }
        while (e + 1 < m) {
          Range r2 = analyse(g, ord, s0, e + 1, lu, of, no_pos, {});
          if (!fits(r2)) break;
          best = r2;
          ++e;
        }
        jx_program::TapeRun tr;
        rc = emit(g, ord, s0, e, best, &tr);
        if (!rc) p->tapes.push_back(tr);
        s0 = e + 1;
      }
      ++i;
      continue;
    }
    size_t j = i + 1;
    while (j < couts.size() && grp.size() < (size_t)JX_TAPE_MAX_IO) {
      std::vector<int> g2 = grp;
      g2.push_back(couts[j]);
      std::vector<int> ord2 = cone(g2);
      Range r2 = analyse(g, ord2, 0, (int)ord2.size() - 1, last_use_of(ord2), flags(g2), no_pos, {});
      if (!fits(r2)) break;
      grp.swap(g2);
      ord.swap(ord2);
      r = r2;
      ++j;
    }
    jx_program::TapeRun tr;
    rc = emit(g, ord, 0, (int)ord.size() - 1, r, &tr);
    if (!rc) p->tapes.push_back(tr);
    i = j;
  }
  // outputs that are program inputs or constants: store-only tapes
  for (size_t i = 0; !rc && i < passthrough.size(); i += JX_TAPE_MAX_IO) {
    std::vector<int> grp(passthrough.begin() + i,
                         passthrough.begin() + std::min(passthrough.size(), i + JX_TAPE_MAX_IO));
    const std::vector<int> empty;
    Range r = analyse(g, empty, 0, -1, std::vector<int>(n, -1), flags(grp), no_pos, grp);
    jx_program::TapeRun tr;
    rc = emit(g, empty, 0, -1, r, &tr);
    if (!rc) p->tapes.push_back(tr);
  }
  if (rc) {
    jx_program_destroy(p);
    return rc;
  }
  // values a tape writes that are not program outputs live in scratch
  std::set<int> produced_outputs(outs, outs + n_out);
  for (const auto& tr : p->tapes)
    for (int v : tr.out_vals)
      if (!produced_outputs.count(v) &&
          std::find(p->scratch_vals.begin(), p->scratch_vals.end(), v) == p->scratch_vals.end())
        p->scratch_vals.push_back(v);
  *out = p;
  return JX_OK;
}

int jx_program_info(const jx_program* p, int* n_tapes, int* n_inputs, int* n_outputs, int* n_scratch) {
  JX_TRACE("jx_program_info");
  JX_REQUIRE(p, "jx_program_info: NULL");
  if (n_tapes) *n_tapes = (int)p->tapes.size();
  if (n_inputs) *n_inputs = p->n_inputs;
  if (n_outputs) *n_outputs = (int)p->outputs.size();
  if (n_scratch) *n_scratch = (int)p->scratch_vals.size();
  return JX_OK;
}

int jx_program_tape(const jx_program* p, int i, const jx_tape** tape) {
  JX_TRACE("jx_program_tape");
  JX_REQUIRE(p && tape && i >= 0 && i < (int)p->tapes.size(), "jx_program_tape: bad index");
  *tape = p->tapes[i].tape;
  return JX_OK;
}

int jx_program_run(const jx_program* p, const float* const* ins, float* const* outs, int64_t n,
                   jx_stream_t stream) {
  JX_TRACE("jx_program_run");
  JX_REQUIRE(p && (ins || p->n_inputs == 0) && outs && n >= 0, "jx_program_run: bad arguments");
  if (n == 0) return JX_OK;
  cudaStream_t st = jx::as_stream(stream);
  // where each value lives: program inputs, caller outputs, scratch
  std::map<int, const float*> src;
  for (int i = 0; i < p->n_inputs; ++i)
    if (p->input_nodes[i] >= 0) {
      JX_REQUIRE(ins[i], "jx_program_run: input %d is NULL", i);
      src[p->input_nodes[i]] = ins[i];
    }
  std::map<int, std::vector<float*>> dst;  // value -> caller buffers (an output may repeat)
  for (size_t i = 0; i < p->outputs.size(); ++i) {
    JX_REQUIRE(outs[i], "jx_program_run: output %zu is NULL", i);
    dst[p->outputs[i]].push_back(outs[i]);
  }
  void* ws = nullptr;
  const size_t ns = p->scratch_vals.size();
  int rc = JX_OK;
  if (ns) {
    rc = jx::scratch_get(sizeof(float) * (size_t)n * ns, &ws, st);
    if (rc) return rc;
    for (size_t i = 0; i < ns; ++i) src[p->scratch_vals[i]] = reinterpret_cast<float*>(ws) + (size_t)n * i;
  }
  for (const auto& kv : dst) src.emplace(kv.first, kv.second[0]);
  for (size_t t = 0; !rc && t < p->tapes.size(); ++t) {
    const auto& tr = p->tapes[t];
    const float* tin[JX_TAPE_MAX_IO];
    float* tout[JX_TAPE_MAX_IO];
    for (size_t i = 0; i < tr.in_vals.size(); ++i) tin[i] = src.at(tr.in_vals[i]);
    for (size_t i = 0; i < tr.out_vals.size(); ++i) {
      const int v = tr.out_vals[i];
      auto it = dst.find(v);
      tout[i] = it != dst.end() ? it->second[0] : const_cast<float*>(src.at(v));
    }
    rc = jx_tape_run(tr.tape, tin, tout, n, stream);
  }
  // an output requested more than once: copy the first buffer to the others
  for (const auto& kv : dst)
    for (size_t k = 1; !rc && k < kv.second.size(); ++k)
      if (kv.second[k] != kv.second[0]) {
        cudaError_t e = cudaMemcpyAsync(kv.second[k], kv.second[0], sizeof(float) * (size_t)n,
                                        cudaMemcpyDeviceToDevice, st);
        if (e != cudaSuccess) rc = jx::check_cuda(e, "jx_program_run: output copy");
      }
  if (ws) {
    const int rc2 = jx::scratch_release(ws, st);
    if (!rc) rc = rc2;
  }
  return rc;
}

int jx_program_destroy(jx_program* p) {
  JX_TRACE("jx_program_destroy");
  if (!p) return JX_OK;
  for (auto& tr : p->tapes) jx_tape_destroy(tr.tape);
  delete p;
  return JX_OK;
}

}  // extern "C"
