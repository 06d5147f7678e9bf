// tape.cu -- the jit op-tape: one fused elementwise kernel per traced chain.
//
// Replaces the reference's fused groups (FusedGroup src/trace/ir.rs:8-17,
// generate_fused_shader src/trace/fusion.rs:296-346, the shader cache
// get_cached_shader src/backend/shaders.rs:1146-1217, gpu_fused_execute
// src/backend/ops.rs:283-437).  A tape is a straight-line register program
// {op, dst, src0, src1}.  jx_tape_create validates it; the first jx_tape_run
// of a tape *structure* on a device generates one CUDA kernel for it, compiles
// it for sm_100a with NVRTC and caches the function, keyed by the op sequence
// (not the constants).  Constants travel in the launch's parameter block, i.e.
// the constant bank, so re-running a tape with new scalars never recompiles.
//
// The generated kernel is straight-line code over SSA values: each thread
// loads two groups of 4 consecutive elements per input (one 128-bit load
// each, one grid sweep apart), applies the ops (the per-element semantics of
// jx_math.cuh, the same header the plain elementwise kernels use) and stores
// the same groups per output.  The reference
// formats literals with {:.6} (src/trace/fusion.rs:359) and turns constants
// it cannot see into 0.0 (:360-363); here constants keep all their bits.
#include <cudaTypedefs.h>
#include <math.h>
#include <nvrtc.h>
#include <string.h>

#include <map>
#include <mutex>
#include <new>
#include <string>
#include <vector>

#include "jx_common.cuh"

namespace {

// jx_math.cuh plus the op codes, embedded by build.py as a string literal.
const char* kPrelude =
#include "tape_prelude.inc"
    ;

constexpr int V = 4;  // elements per thread per input load

// Mirrors the struct the generated kernels declare (kParamsDecl).
struct TapeParams {
  const float* in[JX_TAPE_MAX_IO];
  float* out[JX_TAPE_MAX_IO];
  long long n;
  int vec_ok;
  int pad_;
  float k[JX_TAPE_MAX_CONSTS];
};
static_assert(JX_TAPE_MAX_IO == 4 && JX_TAPE_MAX_CONSTS == 64, "kParamsDecl spells these sizes out");

const char* kParamsDecl =
    "struct TapeParams { const float* in[4]; float* out[4]; long long n; int vec_ok; int pad_; float k[64]; };\n";

// ---- driver entry points (resolved through the runtime, no libcuda link) ----
PFN_cuModuleLoadData_v2000 p_load = nullptr;
PFN_cuModuleGetFunction_v2000 p_getfn = nullptr;
PFN_cuLaunchKernel_v4000 p_launch = nullptr;
std::once_flag g_entry_once;

int load_entry_points() {
  std::call_once(g_entry_once, [] {
    cudaDriverEntryPointQueryResult q;
    void* f = nullptr;
    if (cudaGetDriverEntryPoint("cuModuleLoadData", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      p_load = reinterpret_cast<PFN_cuModuleLoadData_v2000>(f);
    if (cudaGetDriverEntryPoint("cuModuleGetFunction", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      p_getfn = reinterpret_cast<PFN_cuModuleGetFunction_v2000>(f);
    if (cudaGetDriverEntryPoint("cuLaunchKernel", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      p_launch = reinterpret_cast<PFN_cuLaunchKernel_v4000>(f);
  });
  if (!p_load || !p_getfn || !p_launch) return jx::fail(JX_ECUDA, "tape: driver entry points unavailable");
  return JX_OK;
}

std::mutex g_cache_mu;
std::map<std::string, CUfunction> g_cache;  // "<device>|<structure key>" -> function

}  // namespace

struct jx_tape {
  int n_in, n_out, n_consts;
  std::vector<int4> code;  // register form, after constant folding and power-of-two division rewriting
  float consts[JX_TAPE_MAX_CONSTS];
  std::string key;         // op structure (no constant values)
};

namespace jx {

int tape_validate(const int32_t* code, int n_instr, int n_consts, int n_inputs, int n_outputs) {
  JX_REQUIRE(n_instr >= 0 && n_instr <= JX_TAPE_MAX_INSTR, "tape: %d instructions (max %d)", n_instr,
             JX_TAPE_MAX_INSTR);
  JX_REQUIRE(n_inputs >= 0 && n_inputs <= JX_TAPE_MAX_IO && n_outputs >= 1 && n_outputs <= JX_TAPE_MAX_IO,
             "tape: %d inputs / %d outputs (max %d each, >= 1 output)", n_inputs, n_outputs, JX_TAPE_MAX_IO);
  JX_REQUIRE(n_consts >= 0 && n_consts <= JX_TAPE_MAX_CONSTS, "tape: %d constants (max %d)", n_consts,
             JX_TAPE_MAX_CONSTS);
  JX_REQUIRE(n_instr == 0 || code, "tape: NULL code");
  bool defined[JX_TAPE_MAX_REGS] = {false};
  bool stored[JX_TAPE_MAX_IO] = {false};
  for (int i = 0; i < n_inputs; ++i) defined[i] = true;
  for (int pc = 0; pc < n_instr; ++pc) {
    const int op = code[4 * pc], dst = code[4 * pc + 1], s0 = code[4 * pc + 2], s1 = code[4 * pc + 3];
    auto reg_ok = [&](int r) { return r >= 0 && r < JX_TAPE_MAX_REGS; };
    if (op == JX_OP_CONST) {
      JX_REQUIRE(reg_ok(dst) && s0 >= 0 && s0 < n_consts, "tape[%d]: bad CONST (constant index %d)", pc, s0);
      defined[dst] = true;
    } else if (op == JX_OP_STORE) {
      JX_REQUIRE(dst >= 0 && dst < n_outputs && reg_ok(s0) && defined[s0], "tape[%d]: bad STORE", pc);
      stored[dst] = true;
    } else if ((op >= JX_OP_BINARY && op <= JX_OP_BINARY + JX_BIN_MAX) || op == JX_OP_SELECT_GT) {
      JX_REQUIRE(reg_ok(dst) && reg_ok(s0) && reg_ok(s1) && defined[s0] && defined[s1],
                 "tape[%d]: bad binary instruction (op %d): undefined source or register range", pc, op);
      defined[dst] = true;
    } else if (op >= JX_OP_UNARY && op <= JX_OP_UNARY + JX_UN_LOG2) {
      JX_REQUIRE(reg_ok(dst) && reg_ok(s0) && defined[s0],
                 "tape[%d]: bad unary instruction (op %d): undefined source or register range", pc, op);
      defined[dst] = true;
    } else {
      return fail(JX_EINVAL, "tape[%d]: unknown opcode %d", pc, op);
    }
  }
  for (int o = 0; o < n_outputs; ++o) JX_REQUIRE(stored[o], "tape: output %d never stored", o);
  return JX_OK;
}

namespace {

// Instructions whose operands are all constants, and whose op is exact in
// IEEE f32 (correctly rounded, so the host computes the same bits as the
// device), are evaluated here and become constant loads: a value_and_grad
// tape's -1/c scale costs nothing per element instead of a division.
// Transcendentals and pow stay on the device (the host's libm rounds
// differently); so do results that are NaN (payload bits differ between the
// host and the device), any subnormal operand or result (a host with
// flush-to-zero set would differ), and min/max/relu of signed zeros (the
// sign of the result is unspecified).
bool fold_value(int op, float a, float b, float& r) {
  auto sub = [](float v) { return fpclassify(v) == FP_SUBNORMAL; };
  if (sub(a) || sub(b)) return false;
  const bool zeros = a == 0.0f && b == 0.0f;
  if (op >= JX_OP_UNARY && op < JX_OP_BINARY) {
    switch (op - JX_OP_UNARY) {
      case JX_UN_NEG: r = -a; break;
      case JX_UN_ABS: r = fabsf(a); break;
      case JX_UN_SQRT: r = sqrtf(a); break;
      case JX_UN_RECIP: r = 1.0f / a; break;
      case JX_UN_SQUARE: r = a * a; break;
      case JX_UN_RELU: if (a == 0.0f) return false; r = fmaxf(a, 0.0f); break;
      case JX_UN_SIGN: r = a > 0.0f ? 1.0f : (a < 0.0f ? -1.0f : 0.0f); break;
      case JX_UN_CEIL: r = ceilf(a); break;
      case JX_UN_FLOOR: r = floorf(a); break;
      case JX_UN_ROUND: r = roundf(a); break;
      case JX_UN_TRUNC: r = truncf(a); break;
      default: return false;
    }
  } else if (op == JX_OP_SELECT_GT) {
    r = a > 0.0f ? b : 0.0f;
  } else {
    switch (op - JX_OP_BINARY) {
      case JX_BIN_ADD: r = a + b; break;
      case JX_BIN_SUB: r = a - b; break;
      case JX_BIN_MUL: r = a * b; break;
      case JX_BIN_DIV: r = a / b; break;
      case JX_BIN_MIN: if (zeros) return false; r = fminf(a, b); break;
      case JX_BIN_MAX: if (zeros) return false; r = fmaxf(a, b); break;
      default: return false;
    }
  }
  return !isnan(r) && !sub(r);
}

void fold_constants(std::vector<int4>& code, std::vector<float>& consts) {
  bool known[JX_TAPE_MAX_REGS] = {false};
  float val[JX_TAPE_MAX_REGS] = {0.0f};
  for (int4& ins : code) {
    const int op = ins.x;
    if (op == JX_OP_STORE) continue;
    if (op == JX_OP_CONST) {
      known[ins.y] = true;
      val[ins.y] = consts[ins.z];
      continue;
    }
    const bool unary = op >= JX_OP_UNARY && op < JX_OP_BINARY;
    float r = 0.0f;
    if (known[ins.z] && (unary || known[ins.w]) && consts.size() < JX_TAPE_MAX_CONSTS &&
        fold_value(op, val[ins.z], unary ? 0.0f : val[ins.w], r)) {
      consts.push_back(r);
      ins = make_int4(JX_OP_CONST, ins.y, (int)consts.size() - 1, 0);
      known[ins.y] = true;
      val[ins.y] = r;
    } else {
      known[ins.y] = false;
    }
  }
}

// Division by a constant that is a power of two becomes multiplication by its
// exact reciprocal: the same bits, without the division sequence.  The
// reciprocal lives in a register the tape never touches.
void rewrite_pow2_division(std::vector<int4>& code, std::vector<float>& consts) {
  int spare = -1;
  for (int r = JX_TAPE_MAX_REGS - 1; r >= 0 && spare < 0; --r) {
    bool used = false;
    for (const int4& j : code)
      if (j.y == r || j.z == r || (j.x != JX_OP_CONST && j.w == r)) used = true;
    if (!used) spare = r;
  }
  if (spare < 0) return;
  int const_of[JX_TAPE_MAX_REGS];
  for (int r = 0; r < JX_TAPE_MAX_REGS; ++r) const_of[r] = -1;
  std::vector<int4> out;
  for (const int4& ins : code) {
    if (ins.x == JX_OP_BINARY + JX_BIN_DIV && const_of[ins.w] >= 0 && consts.size() < JX_TAPE_MAX_CONSTS) {
      int e = 0;
      const float c = consts[const_of[ins.w]];
      const float m = frexpf(c, &e);
      // |c| = 2^(e-1); its reciprocal is exact while 2^(1-e) stays a normal float
      if (c != 0.0f && (m == 0.5f || m == -0.5f) && e > -124 && e < 126) {
        consts.push_back(1.0f / c);
        out.push_back(make_int4(JX_OP_CONST, spare, (int)consts.size() - 1, 0));
        out.push_back(make_int4(JX_OP_BINARY + JX_BIN_MUL, ins.y, ins.z, spare));
        const_of[ins.y] = -1;
        continue;
      }
    }
    out.push_back(ins);
    if (ins.x == JX_OP_CONST) const_of[ins.y] = ins.z;
    else if (ins.x != JX_OP_STORE) const_of[ins.y] = -1;
  }
  code.swap(out);
}

std::string structure_key(const jx_tape* t) {
  std::string k = "i" + std::to_string(t->n_in) + "o" + std::to_string(t->n_out) + ":";
  for (const int4& c : t->code)
    k += std::to_string(c.x) + "," + std::to_string(c.y) + "," + std::to_string(c.z) + "," + std::to_string(c.w) + ";";
  return k;
}

// CUDA source of the kernel for one tape structure.
std::string codegen(const jx_tape* t) {
  std::string s;
  s += kParamsDecl;
  s += "extern \"C\" __global__ void __launch_bounds__(256) jx_tape_kernel(const TapeParams p) {\n";
  // Each iteration: two 4-element groups per thread, one sweep of the grid
  // apart, so both 128-bit loads of a warp stay fully coalesced and the
  // second group's math overlaps the first's.
  s += "  const long long n = p.n;\n";
  s += "  const long long sweep = (long long)gridDim.x * blockDim.x * 4;\n";
  s += "  for (long long b0 = ((long long)blockIdx.x * blockDim.x + threadIdx.x) * 4; b0 < n; b0 += 2 * sweep) {\n";
  s += "    const long long bs[2] = {b0, b0 + sweep};\n";
  for (int i = 0; i < t->n_in; ++i) {
    const std::string I = std::to_string(i);
    s += "    float x" + I + "[8];\n";
    s += "#pragma unroll\n    for (int u = 0; u < 2; ++u) {\n";
    s += "      const long long base = bs[u];\n";
    s += "      if (p.vec_ok && base + 4 <= n) { const float4 q = __ldcs(reinterpret_cast<const float4*>(p.in[" + I +
         "] + base)); x" + I + "[4 * u] = q.x; x" + I + "[4 * u + 1] = q.y; x" + I + "[4 * u + 2] = q.z; x" + I +
         "[4 * u + 3] = q.w; }\n";
    s += "      else { for (int v = 0; v < 4; ++v) x" + I + "[4 * u + v] = base + v < n ? p.in[" + I +
         "][base + v] : 0.0f; }\n";
    s += "    }\n";
  }
  for (int o = 0; o < t->n_out; ++o) s += "    float y" + std::to_string(o) + "[8];\n";
  s += "#pragma unroll\n    for (int v = 0; v < 8; ++v) {\n";
  // SSA: every definition gets a fresh name; reg_name tracks the current one.
  // First pass: the SSA name each unary op reads, to find values that are fed
  // to both sigmoid and tanh, or to both gelu and its derivative (each pair
  // shares one exponential and one reciprocal: jxm::sigmoid_tanh,
  // jxm::gelu_pair).
  std::vector<std::string> src_name(t->code.size());
  {
    std::string rn[JX_TAPE_MAX_REGS];
    for (int i = 0; i < t->n_in; ++i) rn[i] = "x" + std::to_string(i) + "[v]";
    int nx = 0;
    for (size_t i = 0; i < t->code.size(); ++i) {
      const int4& c = t->code[i];
      if (c.x != JX_OP_CONST) src_name[i] = rn[c.z];  // a constant's src0 is a constant slot, not a register
      if (c.x != JX_OP_STORE) rn[c.y] = "t" + std::to_string(nx++);
    }
  }
  // pair kinds: 0 = sigmoid/tanh, 1 = gelu/gelu_grad; first op of each pair
  const int pair_op[2][2] = {{JX_OP_UNARY + JX_UN_SIGMOID, JX_OP_UNARY + JX_UN_TANH},
                             {JX_OP_UNARY + JX_UN_GELU, JX_OP_UNARY + JX_UN_GELU_GRAD}};
  const char* pair_fn[2] = {"sigmoid_tanh", "gelu_pair"};
  const char* pair_pre[2][2] = {{"sg_", "th_"}, {"gl_", "gd_"}};
  std::map<std::string, int> seen[2][2];  // SSA value -> uses, per pair kind and member
  for (size_t i = 0; i < t->code.size(); ++i)
    for (int k = 0; k < 2; ++k)
      for (int m = 0; m < 2; ++m)
        if (t->code[i].x == pair_op[k][m]) seen[k][m][src_name[i]]++;
  std::map<std::string, std::string> pair_done[2];  // SSA value -> suffix of its pair
  std::string reg_name[JX_TAPE_MAX_REGS];
  for (int i = 0; i < t->n_in; ++i) reg_name[i] = "x" + std::to_string(i) + "[v]";
  int next = 0;
  for (size_t i = 0; i < t->code.size(); ++i) {
    const int4& c = t->code[i];
    const int op = c.x;
    if (op == JX_OP_STORE) {
      s += "      y" + std::to_string(c.y) + "[v] = " + reg_name[c.z] + ";\n";
      continue;
    }
    const std::string nm = "t" + std::to_string(next++);
    std::string rhs;
    int pk = -1, pm = -1;
    for (int k = 0; k < 2; ++k)
      for (int m = 0; m < 2; ++m)
        if (op == pair_op[k][m] && seen[k][0].count(src_name[i]) && seen[k][1].count(src_name[i])) pk = k, pm = m;
    if (pk >= 0) {
      auto it = pair_done[pk].find(src_name[i]);
      if (it == pair_done[pk].end()) {
        const std::string k = std::to_string(pair_done[pk].size());
        const std::string a = pair_pre[pk][0] + k, b = pair_pre[pk][1] + k;
        s += "      float " + a + ", " + b + ";\n      jxm::" + pair_fn[pk] + "(" + src_name[i] + ", " + a + ", " + b +
             ");\n";
        it = pair_done[pk].emplace(src_name[i], k).first;
      }
      rhs = pair_pre[pk][pm] + it->second;
    } else if (op == JX_OP_CONST) {
      rhs = "p.k[" + std::to_string(c.z) + "]";
    } else if (op == JX_OP_SELECT_GT) {
      rhs = "jxm::binary_t<7>(" + reg_name[c.z] + ", " + reg_name[c.w] + ")";
    } else if (op >= JX_OP_BINARY) {
      rhs = "jxm::binary_t<" + std::to_string(op - JX_OP_BINARY) + ">(" + reg_name[c.z] + ", " + reg_name[c.w] + ")";
    } else {
      rhs = "jxm::unary_t<" + std::to_string(op - JX_OP_UNARY) + ">(" + reg_name[c.z] + ")";
    }
    s += "      const float " + nm + " = " + rhs + ";\n";
    reg_name[c.y] = nm;
  }
  s += "    }\n";
  s += "#pragma unroll\n    for (int u = 0; u < 2; ++u) {\n";
  s += "      const long long base = bs[u];\n";
  for (int o = 0; o < t->n_out; ++o) {
    const std::string O = std::to_string(o);
    s += "      if (p.vec_ok && base + 4 <= n) __stcs(reinterpret_cast<float4*>(p.out[" + O +
         "] + base), make_float4(y" + O + "[4 * u], y" + O + "[4 * u + 1], y" + O + "[4 * u + 2], y" + O +
         "[4 * u + 3]));\n";
    s += "      else { for (int v = 0; v < 4; ++v) if (base + v < n) p.out[" + O + "][base + v] = y" + O +
         "[4 * u + v]; }\n";
  }
  s += "    }\n  }\n}\n";
  return s;
}

// NVRTC: generated source -> sm_100a cubin.  Needs no GPU.
int nvrtc_build(const std::string& src, std::vector<char>& cubin) {
  nvrtcProgram prog;
  if (nvrtcCreateProgram(&prog, src.c_str(), "jx_tape.cu", 0, nullptr, nullptr) != NVRTC_SUCCESS)
    return fail(JX_ECUDA, "tape: nvrtcCreateProgram failed");
  const char* opts[] = {"--gpu-architecture=sm_100a", "-std=c++17", "-default-device", "-diag-suppress=177"};
  const nvrtcResult cr = nvrtcCompileProgram(prog, 4, opts);
  if (cr != NVRTC_SUCCESS) {
    size_t n = 0;
    nvrtcGetProgramLogSize(prog, &n);
    std::string log(n, '\0');
    nvrtcGetProgramLog(prog, &log[0]);
    nvrtcDestroyProgram(&prog);
    return fail(JX_ECUDA, "tape: NVRTC compile failed (%s): %.800s", nvrtcGetErrorString(cr), log.c_str());
  }
  size_t cubin_size = 0;
  nvrtcGetCUBINSize(prog, &cubin_size);
  cubin.resize(cubin_size);
  nvrtcGetCUBIN(prog, cubin.data());
  nvrtcDestroyProgram(&prog);
  return JX_OK;
}

int compile_tape(const jx_tape* t, CUfunction* fn) {
  int rc = load_entry_points();
  if (rc) return rc;
  int dev = 0;
  JX_CUDA(cudaGetDevice(&dev));
  const std::string cache_key = std::to_string(dev) + "|" + t->key;
  std::lock_guard<std::mutex> lk(g_cache_mu);
  auto it = g_cache.find(cache_key);
  if (it != g_cache.end()) {
    *fn = it->second;
    return JX_OK;
  }
  JX_CUDA(cudaFree(0));  // the device's primary context must be current for the driver calls
  std::vector<char> cubin;
  if ((rc = nvrtc_build(std::string(kPrelude) + codegen(t), cubin))) return rc;
  CUmodule mod;
  CUresult r = p_load(&mod, cubin.data());
  if (r != CUDA_SUCCESS) return fail(JX_ECUDA, "tape: cuModuleLoadData failed (%d)", (int)r);
  r = p_getfn(fn, mod, "jx_tape_kernel");
  if (r != CUDA_SUCCESS) return fail(JX_ECUDA, "tape: cuModuleGetFunction failed (%d)", (int)r);
  g_cache[cache_key] = *fn;  // modules live until the process exits
  return JX_OK;
}

}  // namespace
}  // namespace jx

extern "C" {

int jx_tape_create(const int32_t* code, int n_instr, const float* consts, int n_consts, int n_inputs, int n_outputs,
                   jx_tape** out) {
  JX_TRACE("jx_tape_create");
  JX_REQUIRE(out, "jx_tape_create: out is NULL");
  *out = nullptr;
  int rc = jx::tape_validate(code, n_instr, n_consts, n_inputs, n_outputs);
  if (rc) return rc;
  JX_REQUIRE(n_consts == 0 || consts, "tape: NULL constants");
  jx_tape* t = new (std::nothrow) jx_tape();
  if (!t) return jx::fail(JX_ENOMEM, "jx_tape_create: out of host memory");
  t->n_in = n_inputs;
  t->n_out = n_outputs;
  for (int i = 0; i < n_instr; ++i)
    t->code.push_back(make_int4(code[4 * i], code[4 * i + 1], code[4 * i + 2], code[4 * i + 3]));
  std::vector<float> kv;
  for (int i = 0; i < n_consts; ++i) kv.push_back(consts[i]);
  jx::fold_constants(t->code, kv);
  jx::rewrite_pow2_division(t->code, kv);
  t->n_consts = (int)kv.size();
  for (size_t i = 0; i < kv.size(); ++i) t->consts[i] = kv[i];
  t->key = jx::structure_key(t);
  *out = t;
  return JX_OK;
}

int jx_tape_destroy(jx_tape* tape) {
  JX_TRACE("jx_tape_destroy");
  delete tape;
  return JX_OK;
}

int jx_tape_source(const jx_tape* tape, char* buf, size_t cap, size_t* len) {
  JX_TRACE("jx_tape_source");
  JX_REQUIRE(tape && len, "jx_tape_source: NULL argument");
  const std::string src = jx::codegen(tape);
  *len = src.size() + 1;
  if (buf && cap > 0) {
    const size_t n = src.size() < cap - 1 ? src.size() : cap - 1;
    memcpy(buf, src.data(), n);
    buf[n] = '\0';
  }
  return JX_OK;
}

int jx_tape_check(const jx_tape* tape) {
  JX_TRACE("jx_tape_check");
  JX_REQUIRE(tape, "jx_tape_check: NULL tape");
  std::vector<char> cubin;
  return jx::nvrtc_build(std::string(kPrelude) + jx::codegen(tape), cubin);
}

int jx_tape_compile(const jx_tape* tape) {
  JX_TRACE("jx_tape_compile");
  JX_REQUIRE(tape, "jx_tape_compile: NULL tape");
  CUfunction f;
  return jx::compile_tape(tape, &f);
}

int jx_tape_info(const jx_tape* tape, int* n_inputs, int* n_outputs, int* n_instr) {
  JX_TRACE("jx_tape_info");
  JX_REQUIRE(tape, "jx_tape_info: NULL tape");
  if (n_inputs) *n_inputs = tape->n_in;
  if (n_outputs) *n_outputs = tape->n_out;
  if (n_instr) *n_instr = (int)tape->code.size();
  return JX_OK;
}

int jx_tape_run(const jx_tape* tape, const float* const* ins, float* const* outs, int64_t n, jx_stream_t stream) {
  JX_TRACE("jx_tape_run");
  JX_REQUIRE(tape, "jx_tape_run: NULL tape");
  JX_REQUIRE(n >= 0, "jx_tape_run: negative size");
  if (n == 0) return JX_OK;
  JX_REQUIRE(tape->n_in == 0 || ins, "jx_tape_run: NULL inputs");
  JX_REQUIRE(outs, "jx_tape_run: NULL outputs");
  TapeParams p;
  memset(&p, 0, sizeof(p));
  p.n = n;
  bool vec = true;
  auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  for (int i = 0; i < tape->n_in; ++i) {
    JX_REQUIRE(ins[i], "jx_tape_run: input %d is NULL", i);
    p.in[i] = ins[i];
    vec = vec && al16(ins[i]);
  }
  for (int i = 0; i < tape->n_out; ++i) {
    JX_REQUIRE(outs[i], "jx_tape_run: output %d is NULL", i);
    p.out[i] = outs[i];
    vec = vec && al16(outs[i]);
  }
  p.vec_ok = vec ? 1 : 0;
  memcpy(p.k, tape->consts, sizeof(float) * tape->n_consts);
  CUfunction f;
  int rc = jx::compile_tape(tape, &f);
  if (rc) return rc;
  const long long work = (n + 2 * V - 1) / (2 * V);  // threads: 2 groups of V elements each
  long long blocks = (work + 255) / 256;
  const long long cap = (long long)jx::num_sms() * 8;
  if (blocks > cap) blocks = cap;
  void* args[] = {&p};
  CUresult r = p_launch(f, (unsigned)blocks, 1, 1, 256, 1, 1, 0, reinterpret_cast<CUstream>(stream), args, nullptr);
  if (r != CUDA_SUCCESS) return jx::fail(JX_ECUDA, "tape: cuLaunchKernel failed (%d)", (int)r);
  return JX_OK;
}

}  // extern "C"
