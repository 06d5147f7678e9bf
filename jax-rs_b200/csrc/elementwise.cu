// elementwise.cu -- elementwise ops and the jit op-tape kernel.
//
// Replaces gpu_binary_op (src/backend/ops.rs:21-149, same-shape only) with a
// broadcasting kernel (binary_op src/ops/binary.rs:7-74, broadcast_index
// :134-168), the CPU-only unary_op (src/ops/unary.rs:30-49) and nn
// activations (src/nn.rs:22-26,111-140) with device kernels, and the
// generated-WGSL fused group (generate_fused_shader src/trace/fusion.rs:296-346,
// gpu_fused_execute src/backend/ops.rs:283-437) with one op-tape interpreter.
//
// The tape travels as a __grid_constant__ kernel parameter, i.e. in the
// constant bank: every thread reads the same instruction, so dispatch is
// warp-uniform.  The register file is 16 named register vectors of 4 lanes
// (4 consecutive elements per thread, one 128-bit load per input); operand
// selection goes through switch jump tables so values stay in real registers.
//
// Arithmetic follows the reference's f32 operation order with explicit
// round-to-nearest intrinsics (no FMA contraction), so ops without a
// transcendental are bit-identical to the reference; tanhf/expf/sinf/... are
// CUDA's own functions (within a few ulp of glibc's).
#include <math.h>
#include <string.h>

#include <new>
#include <vector>

#include "jx_common.cuh"

namespace {

constexpr int TAPE_V = 4;
constexpr float PI_F = 3.14159265358979323846f;
constexpr float GELU_C1 = 0.044715f;

struct TapeArgs {
  int n_instr;
  int n_in;
  int n_out;
  int vec_ok;
  long long n;
  const float* in[JX_TAPE_MAX_IO];
  float* out[JX_TAPE_MAX_IO];
  float consts[JX_TAPE_MAX_CONSTS];
  int4 code[JX_TAPE_MAX_INSTR];
};
static_assert(sizeof(TapeArgs) <= 4096, "tape must fit the kernel parameter space");

// --- scalar op semantics (shared by the tape and the plain kernels) ---------
__device__ __forceinline__ float gelu_f(float v) {
  // src/nn.rs:111-122; v.powi(3) = v*(v*v)
  const float coeff = sqrtf(__fdiv_rn(2.0f, PI_F));
  float v3 = __fmul_rn(v, __fmul_rn(v, v));
  float inner = __fmul_rn(coeff, __fadd_rn(v, __fmul_rn(GELU_C1, v3)));
  return __fmul_rn(__fmul_rn(0.5f, v), __fadd_rn(1.0f, tanhf(inner)));
}
__device__ __forceinline__ float gelu_grad_f(float u) {
  // d/du of the expression above (restated adjoint; same order as the oracle)
  const float coeff = sqrtf(__fdiv_rn(2.0f, PI_F));
  float u2 = __fmul_rn(u, u);
  float inner = __fmul_rn(coeff, __fadd_rn(u, __fmul_rn(GELU_C1, __fmul_rn(u, u2))));
  float t = tanhf(inner);
  float dinner = __fmul_rn(coeff, __fadd_rn(1.0f, __fmul_rn(__fmul_rn(3.0f, GELU_C1), u2)));
  float a = __fmul_rn(0.5f, __fadd_rn(1.0f, t));
  float b = __fmul_rn(__fmul_rn(__fmul_rn(0.5f, u), __fsub_rn(1.0f, __fmul_rn(t, t))), dinner);
  return __fadd_rn(a, b);
}
__device__ __forceinline__ float sigmoid_f(float v) {
  return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-v)));  // src/nn.rs:135-140
}

__device__ __forceinline__ float unary_f(int op, float x) {
  switch (op) {
    case JX_UN_NEG: return -x;
    case JX_UN_ABS: return fabsf(x);
    case JX_UN_SIN: return sinf(x);
    case JX_UN_COS: return cosf(x);
    case JX_UN_TANH: return tanhf(x);
    case JX_UN_EXP: return expf(x);
    case JX_UN_LOG: return logf(x);
    case JX_UN_SQRT: return __fsqrt_rn(x);
    case JX_UN_RECIP: return __fdiv_rn(1.0f, x);
    case JX_UN_SQUARE: return __fmul_rn(x, x);
    case JX_UN_RELU: return fmaxf(x, 0.0f);
    case JX_UN_GELU: return gelu_f(x);
    case JX_UN_SIGMOID: return sigmoid_f(x);
    case JX_UN_GELU_GRAD: return gelu_grad_f(x);
    default: return x;
  }
}

__device__ __forceinline__ float binary_f(int op, float a, float b) {
  switch (op) {
    case JX_BIN_ADD: return __fadd_rn(a, b);
    case JX_BIN_SUB: return __fsub_rn(a, b);
    case JX_BIN_MUL: return __fmul_rn(a, b);
    case JX_BIN_DIV: return __fdiv_rn(a, b);
    case JX_BIN_POW: return powf(a, b);
    case JX_BIN_MIN: return fminf(a, b);
    case JX_BIN_MAX: return fmaxf(a, b);
    default: return a;
  }
}

// --- tape interpreter ---------------------------------------------------------
#define JX_COPYV(d, s)                                 \
  _Pragma("unroll") for (int _v = 0; _v < TAPE_V; ++_v) \
    (d)[_v] = (s)[_v];

#define JX_FETCH(d, idx)           \
  switch (idx) {                   \
    case 0: JX_COPYV(d, r0); break;   \
    case 1: JX_COPYV(d, r1); break;   \
    case 2: JX_COPYV(d, r2); break;   \
    case 3: JX_COPYV(d, r3); break;   \
    case 4: JX_COPYV(d, r4); break;   \
    case 5: JX_COPYV(d, r5); break;   \
    case 6: JX_COPYV(d, r6); break;   \
    case 7: JX_COPYV(d, r7); break;   \
    case 8: JX_COPYV(d, r8); break;   \
    case 9: JX_COPYV(d, r9); break;   \
    case 10: JX_COPYV(d, r10); break; \
    case 11: JX_COPYV(d, r11); break; \
    case 12: JX_COPYV(d, r12); break; \
    case 13: JX_COPYV(d, r13); break; \
    case 14: JX_COPYV(d, r14); break; \
    default: JX_COPYV(d, r15); break; \
  }

#define JX_WRITE(idx, s)           \
  switch (idx) {                   \
    case 0: JX_COPYV(r0, s); break;   \
    case 1: JX_COPYV(r1, s); break;   \
    case 2: JX_COPYV(r2, s); break;   \
    case 3: JX_COPYV(r3, s); break;   \
    case 4: JX_COPYV(r4, s); break;   \
    case 5: JX_COPYV(r5, s); break;   \
    case 6: JX_COPYV(r6, s); break;   \
    case 7: JX_COPYV(r7, s); break;   \
    case 8: JX_COPYV(r8, s); break;   \
    case 9: JX_COPYV(r9, s); break;   \
    case 10: JX_COPYV(r10, s); break; \
    case 11: JX_COPYV(r11, s); break; \
    case 12: JX_COPYV(r12, s); break; \
    case 13: JX_COPYV(r13, s); break; \
    case 14: JX_COPYV(r14, s); break; \
    default: JX_COPYV(r15, s); break; \
  }

__global__ void __launch_bounds__(256) tape_kernel(const __grid_constant__ TapeArgs t) {
  float r0[TAPE_V], r1[TAPE_V], r2[TAPE_V], r3[TAPE_V], r4[TAPE_V], r5[TAPE_V], r6[TAPE_V], r7[TAPE_V];
  float r8[TAPE_V], r9[TAPE_V], r10[TAPE_V], r11[TAPE_V], r12[TAPE_V], r13[TAPE_V], r14[TAPE_V], r15[TAPE_V];
  const long long n = t.n;
  const long long stride = (long long)gridDim.x * blockDim.x * TAPE_V;
  for (long long base = ((long long)blockIdx.x * blockDim.x + threadIdx.x) * TAPE_V; base < n; base += stride) {
    const bool full = t.vec_ok && base + TAPE_V <= n;
    // load the inputs into r0..r(n_in-1)
    for (int i = 0; i < t.n_in; ++i) {
      float x[TAPE_V];
      if (full) {
        float4 q = __ldcs(reinterpret_cast<const float4*>(t.in[i] + base));
        x[0] = q.x; x[1] = q.y; x[2] = q.z; x[3] = q.w;
      } else {
#pragma unroll
        for (int v = 0; v < TAPE_V; ++v) x[v] = base + v < n ? t.in[i][base + v] : 0.0f;
      }
      JX_WRITE(i, x);
    }
    for (int pc = 0; pc < t.n_instr; ++pc) {
      const int4 ins = t.code[pc];
      const int op = ins.x;
      float a[TAPE_V], c[TAPE_V];
      if (op == JX_OP_CONST) {
        const float k = t.consts[ins.z];
#pragma unroll
        for (int v = 0; v < TAPE_V; ++v) c[v] = k;
        JX_WRITE(ins.y, c);
      } else if (op == JX_OP_STORE) {
        JX_FETCH(a, ins.z);
        float* o = t.out[ins.y];
        if (full) {
          __stcs(reinterpret_cast<float4*>(o + base), make_float4(a[0], a[1], a[2], a[3]));
        } else {
#pragma unroll
          for (int v = 0; v < TAPE_V; ++v)
            if (base + v < n) o[base + v] = a[v];
        }
      } else if (op >= JX_OP_BINARY && op < JX_OP_BINARY + 16) {
        float b[TAPE_V];
        JX_FETCH(a, ins.z);
        JX_FETCH(b, ins.w);
        const int bop = op - JX_OP_BINARY;
#pragma unroll
        for (int v = 0; v < TAPE_V; ++v) c[v] = binary_f(bop, a[v], b[v]);
        JX_WRITE(ins.y, c);
      } else if (op == JX_OP_SELECT_GT) {
        float b[TAPE_V];
        JX_FETCH(a, ins.z);
        JX_FETCH(b, ins.w);
#pragma unroll
        for (int v = 0; v < TAPE_V; ++v) c[v] = a[v] > 0.0f ? b[v] : 0.0f;
        JX_WRITE(ins.y, c);
      } else {
        JX_FETCH(a, ins.z);
        const int uop = op - JX_OP_UNARY;
#pragma unroll
        for (int v = 0; v < TAPE_V; ++v) c[v] = unary_f(uop, a[v]);
        JX_WRITE(ins.y, c);
      }
    }
  }
}

// --- plain kernels --------------------------------------------------------------
__global__ void unary_kernel(int op, const float* __restrict__ x, float* __restrict__ y, long long n, int vec_ok) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  if (vec_ok) {
    const long long n4 = n / 4;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4; i += stride) {
      float4 q = reinterpret_cast<const float4*>(x)[i];
      q.x = unary_f(op, q.x); q.y = unary_f(op, q.y); q.z = unary_f(op, q.z); q.w = unary_f(op, q.w);
      reinterpret_cast<float4*>(y)[i] = q;
    }
    for (long long i = n4 * 4 + blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += stride)
      y[i] = unary_f(op, x[i]);
  } else {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += stride) y[i] = unary_f(op, x[i]);
  }
}

constexpr int BMAX_DIMS = 8;
struct BroadcastArgs {
  int nd;
  long long n;
  long long out_dims[BMAX_DIMS];
  long long sa[BMAX_DIMS];  // element strides of a in output index space (0 = broadcast)
  long long sb[BMAX_DIMS];
};

__global__ void binary_bcast_kernel(int op, const float* __restrict__ a, const float* __restrict__ b,
                                    float* __restrict__ out, const __grid_constant__ BroadcastArgs g) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < g.n; i += stride) {
    long long rem = i, ia = 0, ib = 0;
    for (int d = g.nd - 1; d >= 0; --d) {
      const long long idx = rem % g.out_dims[d];
      rem /= g.out_dims[d];
      ia += idx * g.sa[d];
      ib += idx * g.sb[d];
    }
    out[i] = binary_f(op, a[ia], b[ib]);
  }
}

__global__ void binary_same_kernel(int op, const float* __restrict__ a, const float* __restrict__ b,
                                   float* __restrict__ out, long long n, int vec_ok) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  if (vec_ok) {
    const long long n4 = n / 4;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4; i += stride) {
      float4 p = reinterpret_cast<const float4*>(a)[i], q = reinterpret_cast<const float4*>(b)[i];
      reinterpret_cast<float4*>(out)[i] =
          make_float4(binary_f(op, p.x, q.x), binary_f(op, p.y, q.y), binary_f(op, p.z, q.z), binary_f(op, p.w, q.w));
    }
    for (long long i = n4 * 4 + blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += stride)
      out[i] = binary_f(op, a[i], b[i]);
  } else {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += stride)
      out[i] = binary_f(op, a[i], b[i]);
  }
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int grid_for(long long work, int threads) {
  long long blocks = (work + threads - 1) / threads;
  long long cap = (long long)jx::num_sms() * 8;
  if (blocks > cap) blocks = cap;
  return blocks < 1 ? 1 : (int)blocks;
}

}  // namespace

struct jx_tape {
  int n_instr, n_in, n_out, n_consts;
  int4 code[JX_TAPE_MAX_INSTR];
  float consts[JX_TAPE_MAX_CONSTS];
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
      JX_REQUIRE(reg_ok(dst) && s0 >= 0 && s0 < n_consts, "tape[%d]: bad CONST", pc);
      defined[dst] = true;
    } else if (op == JX_OP_STORE) {
      JX_REQUIRE(dst >= 0 && dst < n_outputs && reg_ok(s0) && defined[s0], "tape[%d]: bad STORE", pc);
      stored[dst] = true;
    } else if ((op >= JX_OP_BINARY && op <= JX_OP_BINARY + JX_BIN_MAX) || op == JX_OP_SELECT_GT) {
      JX_REQUIRE(reg_ok(dst) && reg_ok(s0) && reg_ok(s1) && defined[s0] && defined[s1],
                 "tape[%d]: bad binary instruction (op %d)", pc, op);
      defined[dst] = true;
    } else if (op >= JX_OP_UNARY && op <= JX_OP_UNARY + JX_UN_GELU_GRAD) {
      JX_REQUIRE(reg_ok(dst) && reg_ok(s0) && defined[s0], "tape[%d]: bad unary instruction (op %d)", pc, op);
      defined[dst] = true;
    } else {
      return fail(JX_EINVAL, "tape[%d]: unknown opcode %d", pc, op);
    }
  }
  for (int o = 0; o < n_outputs; ++o) JX_REQUIRE(stored[o], "tape: output %d never stored", o);
  return JX_OK;
}
}  // namespace jx

extern "C" {

int jx_tape_create(const int32_t* code, int n_instr, const float* consts, int n_consts, int n_inputs, int n_outputs,
                   jx_tape** out) {
  JX_REQUIRE(out, "jx_tape_create: out is NULL");
  *out = nullptr;
  int rc = jx::tape_validate(code, n_instr, n_consts, n_inputs, n_outputs);
  if (rc) return rc;
  JX_REQUIRE(n_consts == 0 || consts, "tape: NULL constants");
  jx_tape* t = new (std::nothrow) jx_tape();
  if (!t) return jx::fail(JX_ENOMEM, "jx_tape_create: out of host memory");
  t->n_instr = n_instr;
  t->n_in = n_inputs;
  t->n_out = n_outputs;
  t->n_consts = n_consts;
  for (int i = 0; i < n_instr; ++i) t->code[i] = make_int4(code[4 * i], code[4 * i + 1], code[4 * i + 2], code[4 * i + 3]);
  for (int i = 0; i < n_consts; ++i) t->consts[i] = consts[i];
  *out = t;
  return JX_OK;
}

int jx_tape_destroy(jx_tape* tape) {
  delete tape;
  return JX_OK;
}

int jx_tape_run(const jx_tape* tape, const float* const* ins, float* const* outs, int64_t n, jx_stream_t stream) {
  JX_REQUIRE(tape, "jx_tape_run: NULL tape");
  JX_REQUIRE(n >= 0, "jx_tape_run: negative size");
  if (n == 0) return JX_OK;
  JX_REQUIRE(tape->n_in == 0 || ins, "jx_tape_run: NULL inputs");
  JX_REQUIRE(outs, "jx_tape_run: NULL outputs");
  TapeArgs a;
  memset(&a, 0, sizeof(a));
  a.n_instr = tape->n_instr;
  a.n_in = tape->n_in;
  a.n_out = tape->n_out;
  a.n = n;
  bool vec = true;
  for (int i = 0; i < tape->n_in; ++i) {
    JX_REQUIRE(ins[i], "jx_tape_run: input %d is NULL", i);
    a.in[i] = ins[i];
    vec = vec && aligned16(ins[i]);
  }
  for (int i = 0; i < tape->n_out; ++i) {
    JX_REQUIRE(outs[i], "jx_tape_run: output %d is NULL", i);
    a.out[i] = outs[i];
    vec = vec && aligned16(outs[i]);
  }
  a.vec_ok = vec ? 1 : 0;
  memcpy(a.consts, tape->consts, sizeof(float) * tape->n_consts);
  memcpy(a.code, tape->code, sizeof(int4) * tape->n_instr);
  const long long work = (n + TAPE_V - 1) / TAPE_V;
  long long blocks = (work + 255) / 256;
  long long cap = (long long)jx::num_sms() * 8;
  if (blocks > cap) blocks = cap;
  tape_kernel<<<(int)blocks, 256, 0, jx::as_stream(stream)>>>(a);
  JX_LAUNCH_CHECK("tape_kernel");
  return JX_OK;
}

int jx_unary_f32(int op, const float* x, float* y, int64_t n, jx_stream_t stream) {
  JX_REQUIRE(op >= 0 && op <= JX_UN_GELU_GRAD, "unary: unknown op %d", op);
  JX_REQUIRE(n >= 0, "unary: negative size");
  if (n == 0) return JX_OK;
  JX_REQUIRE(x && y, "unary: NULL pointer");
  unary_kernel<<<grid_for((n + 3) / 4, 256), 256, 0, jx::as_stream(stream)>>>(op, x, y, n,
                                                                              aligned16(x) && aligned16(y));
  JX_LAUNCH_CHECK("unary_kernel");
  return JX_OK;
}

int jx_binary_f32(int op, const float* a, const int64_t* a_shape, int a_ndim, const float* b, const int64_t* b_shape,
                  int b_ndim, float* out, jx_stream_t stream) {
  JX_REQUIRE(op >= 0 && op <= JX_BIN_MAX, "binary: unknown op %d", op);
  JX_REQUIRE(a_ndim >= 0 && a_ndim <= BMAX_DIMS && b_ndim >= 0 && b_ndim <= BMAX_DIMS, "binary: rank > %d",
             BMAX_DIMS);
  JX_REQUIRE((a_ndim == 0 || a_shape) && (b_ndim == 0 || b_shape), "binary: NULL shape");
  const int nd = a_ndim > b_ndim ? a_ndim : b_ndim;
  BroadcastArgs g;
  memset(&g, 0, sizeof(g));
  g.nd = nd;
  long long total = 1;
  bool same = a_ndim == b_ndim;
  // NumPy broadcasting (src/shape.rs:87-113): align trailing dims.
  long long stride_a = 1, stride_b = 1;
  for (int d = nd - 1; d >= 0; --d) {
    const int ia = d - (nd - a_ndim), ib = d - (nd - b_ndim);
    const long long da = ia >= 0 ? a_shape[ia] : 1, db = ib >= 0 ? b_shape[ib] : 1;
    JX_REQUIRE(da >= 0 && db >= 0, "binary: negative dimension");
    if (da != db && da != 1 && db != 1)
      return jx::fail(JX_EINVAL, "Shapes are not broadcast-compatible (dim %d: %lld vs %lld)", d, da, db);
    if (da != db) same = false;
    const long long od = da == 1 ? db : da;
    g.out_dims[d] = od;
    g.sa[d] = (da == 1) ? 0 : stride_a;
    g.sb[d] = (db == 1) ? 0 : stride_b;
    stride_a *= da;
    stride_b *= db;
    total *= od;
  }
  g.n = total;
  if (total == 0) return JX_OK;
  JX_REQUIRE(a && b && out, "binary: NULL pointer");
  cudaStream_t st = jx::as_stream(stream);
  if (same) {
    binary_same_kernel<<<grid_for((total + 3) / 4, 256), 256, 0, st>>>(op, a, b, out, total,
                                                                       aligned16(a) && aligned16(b) && aligned16(out));
  } else {
    binary_bcast_kernel<<<grid_for(total, 256), 256, 0, st>>>(op, a, b, out, g);
  }
  JX_LAUNCH_CHECK("binary kernel");
  return JX_OK;
}

}  // extern "C"
