/*
 * jaxrs_oracle.c -- CPU restatement of the jax-rs (v0.5.1) CPU code paths that
 * the CUDA backend replaces.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker: only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference legs
 * may load it.  The product path (libjaxrs_cuda.so) never calls into it.
 *
 * Every routine follows a named reference function line by line, in the same
 * f32 operation order, so results are bit-identical to what the reference's
 * Rust code computes on the same inputs (Rust never contracts a*b+c into an
 * FMA, so this file is compiled with -ffp-contract=off and no fast-math, and
 * uses glibc's expf/tanhf/logf/cosf/sinf/sqrtf/powf, which are what Rust's f32
 * methods call on Linux).  Parity pins: the known-answer tests in the
 * reference's tests/ directory (*.rs) and doc-tests (see tests/golden/known_answers.json).
 *
 * Routines marked "restated adjoint" (conv2d dX/dW, the chain's VJP, the MLP
 * backward) have no reference implementation; they are the exact derivative
 * of the reference forward, written in the loop order stated beside each one.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <pthread.h>

#define JXO_PI_F 3.14159265358979323846264338327950288f

/* ------------------------------------------------------------------------- */
/* PRNGKey: xorshift128+ (src/random.rs:15-97)                                */
/* ------------------------------------------------------------------------- */
typedef struct { uint64_t s0, s1; } jxo_key;

static inline uint64_t rotl64(uint64_t x, unsigned r) { return (x << r) | (x >> (64u - r)); }
static inline uint64_t rotr64(uint64_t x, unsigned r) { return (x >> r) | (x << (64u - r)); }

/* src/random.rs:29-32 PRNGKey::from_seed */
void jxo_key_from_seed(uint64_t seed, jxo_key *out) {
    out->s0 = seed;
    out->s1 = seed * 0x9e3779b97f4a7c15ULL;
}

/* src/random.rs:43-56 PRNGKey::split */
void jxo_key_split(const jxo_key *k, jxo_key *k1, jxo_key *k2) {
    jxo_key a = *k, b = *k;
    a.s0 = a.s0 + 0x9e3779b97f4a7c15ULL;
    b.s0 = b.s0 + 0x3c6ef372fe94f82aULL;
    a.s1 = rotl64(a.s1, 27);
    b.s1 = rotr64(b.s1, 17);
    *k1 = a;
    *k2 = b;
}

/* src/random.rs:67-76 PRNGKey::split_n */
void jxo_key_split_n(const jxo_key *k, int64_t n, jxo_key *out) {
    jxo_key cur = *k;
    for (int64_t i = 0; i < n; ++i) {
        jxo_key key, next;
        jxo_key_split(&cur, &key, &next);
        out[i] = key;
        cur = next;
    }
}

/* src/random.rs:78-90 PRNGKey::next_u64 */
uint64_t jxo_next_u64(jxo_key *k) {
    uint64_t s1 = k->s0;
    uint64_t s0 = k->s1;
    k->s0 = s0;
    s1 ^= s1 << 23;
    s1 ^= s1 >> 17;
    s1 ^= s0;
    s1 ^= s0 >> 26;
    k->s1 = s1;
    return s1 + s0;
}

/* src/random.rs:93-97 PRNGKey::next_f32 */
static inline float next_f32(jxo_key *k) {
    uint64_t u = jxo_next_u64(k);
    return (float)(u >> 40) / (float)(1ULL << 24);
}

/* src/random.rs:128-150 uniform_device (CPU arm): n draws of next_f32 */
void jxo_uniform(jxo_key key, float *out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) out[i] = next_f32(&key);
}

/* src/random.rs:161-181 uniform_range: min + (max - min) * next_f32 */
void jxo_uniform_range(jxo_key key, float *out, int64_t n, float minval, float maxval) {
    for (int64_t i = 0; i < n; ++i) {
        float u = next_f32(&key);
        out[i] = minval + (maxval - minval) * u;
    }
}

/* src/random.rs:189-210 randint: (next_u64 % range) as i32 + minval, stored as f32 */
void jxo_randint(jxo_key key, float *out, int64_t n, int32_t minval, int32_t maxval) {
    uint64_t range = (uint64_t)(int64_t)(maxval - minval);
    for (int64_t i = 0; i < n; ++i) {
        int32_t r = (int32_t)(jxo_next_u64(&key) % range) + minval;
        out[i] = (float)r;
    }
}

/* src/random.rs:259-285 normal_device (CPU arm): Box-Muller, cos first then sin */
void jxo_normal(jxo_key key, float *out, int64_t n) {
    int64_t i = 0;
    while (i < n) {
        float u1 = next_f32(&key);
        float u2 = next_f32(&key);
        u1 = fmaxf(u1, 1e-10f);
        float r = sqrtf(-2.0f * logf(u1));
        float theta = 2.0f * JXO_PI_F * u2;
        out[i++] = r * cosf(theta);
        if (i < n) out[i++] = r * sinf(theta);
    }
}

/* ------------------------------------------------------------------------- */
/* Small parallel-for used only to time the CPU path on several host cores.  */
/* Each worker runs the same per-row arithmetic, so results do not depend on */
/* the thread count.                                                         */
/* ------------------------------------------------------------------------- */
typedef void (*row_fn)(void *ctx, int64_t r0, int64_t r1);
typedef struct { row_fn fn; void *ctx; int64_t r0, r1; } pf_job;
static void *pf_tramp(void *p) { pf_job *j = (pf_job *)p; j->fn(j->ctx, j->r0, j->r1); return NULL; }

static void parallel_rows(row_fn fn, void *ctx, int64_t rows, int nthreads) {
    if (nthreads <= 1 || rows < 2) { fn(ctx, 0, rows); return; }
    if (nthreads > 256) nthreads = 256;
    if (nthreads > rows) nthreads = (int)rows;
    pthread_t th[256];
    pf_job jobs[256];
    int64_t per = (rows + nthreads - 1) / nthreads;
    int started = 0;
    for (int t = 0; t < nthreads; ++t) {
        int64_t a = t * per, b = a + per < rows ? a + per : rows;
        if (a >= b) break;
        jobs[t].fn = fn; jobs[t].ctx = ctx; jobs[t].r0 = a; jobs[t].r1 = b;
        if (pthread_create(&th[t], NULL, pf_tramp, &jobs[t]) != 0) { fn(ctx, a, b); continue; }
        started = t + 1;
    }
    for (int t = 0; t < started; ++t) pthread_join(th[t], NULL);
}

/* ------------------------------------------------------------------------- */
/* GEMM: src/ops/linalg.rs:215-232 (i-j-p loop, sequential f32 sum from 0)   */
/* batched: src/ops/einsum.rs:505-519 (same loop per batch)                  */
/* ------------------------------------------------------------------------- */
typedef struct { const float *a, *b; float *c; int64_t m, n, k; } mm_ctx;

static void mm_rows(void *p, int64_t r0, int64_t r1) {
    mm_ctx *c = (mm_ctx *)p;
    for (int64_t i = r0; i < r1; ++i)
        for (int64_t j = 0; j < c->n; ++j) {
            float sum = 0.0f;
            for (int64_t q = 0; q < c->k; ++q) sum += c->a[i * c->k + q] * c->b[q * c->n + j];
            c->c[i * c->n + j] = sum;
        }
}

/* Rows [r0, r1) of C = A.B (A row-major [m,k], B [k,n]); C holds only those rows. */
void jxo_matmul_rows(const float *a, const float *b, float *c, int64_t m, int64_t n, int64_t k,
                     int64_t r0, int64_t r1, int nthreads) {
    (void)m;
    mm_ctx ctx = {a + r0 * k, b, c, r1 - r0, n, k};
    parallel_rows(mm_rows, &ctx, r1 - r0, nthreads);
}

void jxo_matmul(const float *a, const float *b, float *c, int64_t m, int64_t n, int64_t k, int nthreads) {
    jxo_matmul_rows(a, b, c, m, n, k, 0, m, nthreads);
}

/* f64 twin of the same loop (not a reference routine: the exact-arithmetic yardstick). */
void jxo_matmul_f64(const float *a, const float *b, double *c, int64_t m, int64_t n, int64_t k) {
    for (int64_t i = 0; i < m; ++i)
        for (int64_t j = 0; j < n; ++j) {
            double s = 0.0;
            for (int64_t q = 0; q < k; ++q) s += (double)a[i * k + q] * (double)b[q * n + j];
            c[i * n + j] = s;
        }
}

void jxo_bmm(const float *a, const float *b, float *c, int64_t batch, int64_t m, int64_t n, int64_t k,
             int nthreads) {
    for (int64_t bb = 0; bb < batch; ++bb)
        jxo_matmul(a + bb * m * k, b + bb * k * n, c + bb * m * n, m, n, k, nthreads);
}

/* src/ops/linalg.rs:20-51 transpose of a 2-D array */
void jxo_transpose(const float *x, float *y, int64_t rows, int64_t cols) {
    for (int64_t i = 0; i < rows; ++i)
        for (int64_t j = 0; j < cols; ++j) y[j * rows + i] = x[i * cols + j];
}

/* ------------------------------------------------------------------------- */
/* Elementwise (src/ops/binary.rs:89-101, src/ops/unary.rs:30-49,87-93,      */
/* src/nn.rs:22-26,111-140)                                                  */
/* ------------------------------------------------------------------------- */
static const float GELU_C1 = 0.044715f;

/* src/nn.rs:111-122: coeff = sqrt(2/pi); inner = coeff*(v + 0.044715*v^3);
 * 0.5*v*(1+tanh(inner)); v.powi(3) lowers to v*(v*v). */
static inline float gelu1(float v) {
    float coeff = sqrtf(2.0f / JXO_PI_F);
    float v3 = v * (v * v);
    float inner = coeff * (v + GELU_C1 * v3);
    return 0.5f * v * (1.0f + tanhf(inner));
}
/* src/nn.rs:135-140 */
static inline float sigmoid1(float v) { return 1.0f / (1.0f + expf(-v)); }
/* src/nn.rs:22-26 (Rust f32::max ignores NaN like fmaxf) */
static inline float relu1(float v) { return fmaxf(v, 0.0f); }

void jxo_gelu(const float *x, float *y, int64_t n) { for (int64_t i = 0; i < n; ++i) y[i] = gelu1(x[i]); }
/* Derivative of gelu1 (the mathematical derivative of src/nn.rs:111-122, which
 * the reference leaves untraced): 0.5*(1+t) + 0.5*v*(1-t^2)*coeff*(1 + 3*0.044715*v^2),
 * t = tanh(inner), the same expression jxo_chain_vjp uses for its gelu term. */
void jxo_gelu_grad(const float *x, float *y, int64_t n) {
    const float coeff = sqrtf(2.0f / JXO_PI_F);
    for (int64_t i = 0; i < n; ++i) {
        float v = x[i], v2 = v * v;
        float t = tanhf(coeff * (v + GELU_C1 * (v * v2)));
        float dinner = coeff * (1.0f + 3.0f * GELU_C1 * v2);
        y[i] = 0.5f * (1.0f + t) + 0.5f * v * (1.0f - t * t) * dinner;
    }
}
void jxo_sigmoid(const float *x, float *y, int64_t n) { for (int64_t i = 0; i < n; ++i) y[i] = sigmoid1(x[i]); }
void jxo_relu(const float *x, float *y, int64_t n) { for (int64_t i = 0; i < n; ++i) y[i] = relu1(x[i]); }
void jxo_tanh(const float *x, float *y, int64_t n) { for (int64_t i = 0; i < n; ++i) y[i] = tanhf(x[i]); }
void jxo_exp(const float *x, float *y, int64_t n) { for (int64_t i = 0; i < n; ++i) y[i] = expf(x[i]); }

/* Rust std's own f32 formulas for the inverse hyperbolic functions (they do
 * not call libm's asinhf/acoshf/atanhf): asinh = copysign(ln_1p(|x| +
 * |x| / (hypot(1, 1/|x|) + 1/|x|)), x); acosh = x < 1 ? NaN :
 * ln(x + sqrt(x - 1) * sqrt(x + 1)); atanh = 0.5 * ln_1p(2x / (1 - x)). */
static inline float rust_asinh(float x) {
    float ax = fabsf(x), ix = 1.0f / ax;
    return copysignf(log1pf(ax + (ax / (hypotf(1.0f, ix) + ix))), x);
}
static inline float rust_acosh(float x) {
    return x < 1.0f ? NAN : logf(x + (sqrtf(x - 1.0f) * sqrtf(x + 1.0f)));
}
static inline float rust_atanh(float x) { return 0.5f * log1pf((2.0f * x) / (1.0f - x)); }
/* Array::sign (src/ops/unary.rs:117-127): 1, -1, else 0 (NaN included). */
static inline float sign1(float x) { return x > 0.0f ? 1.0f : (x < 0.0f ? -1.0f : 0.0f); }

/* unary_op (src/ops/unary.rs:30-49) with the element function of each method
 * (neg, abs, sin, cos, tanh, exp, ln, sqrt, recip, square at :60-160; relu,
 * gelu, sigmoid from src/nn.rs; tan through log2 at :82-541).  Codes follow
 * JX_UN_* of the C ABI. */
static inline float unary1(int op, float x) {
    switch (op) {
    case 0: return -x;
    case 1: return fabsf(x);
    case 2: return sinf(x);
    case 3: return cosf(x);
    case 4: return tanhf(x);
    case 5: return expf(x);
    case 6: return logf(x);
    case 7: return sqrtf(x);
    case 8: return 1.0f / x;
    case 9: return x * x;
    case 10: return relu1(x);
    case 11: return gelu1(x);
    case 12: return sigmoid1(x);
    case 14: return tanf(x);
    case 15: return sign1(x);
    case 16: return sinhf(x);
    case 17: return coshf(x);
    case 18: return asinf(x);
    case 19: return acosf(x);
    case 20: return atanf(x);
    case 21: return rust_asinh(x);
    case 22: return rust_acosh(x);
    case 23: return rust_atanh(x);
    case 24: return ceilf(x);
    case 25: return floorf(x);
    case 26: return roundf(x);
    case 27: return truncf(x);
    case 28: return expm1f(x);
    case 29: return log1pf(x);
    case 30: return cbrtf(x);
    case 31: return log2f(x);
    default: return x;
    }
}
void jxo_unary(int op, const float *x, float *y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) y[i] = unary1(op, x[i]);
}

/* Binary ops with the reference's broadcasting rule (src/ops/binary.rs:7-74,
 * src/shape.rs:87-113, broadcast_index src/ops/binary.rs:134-168).
 * op: 0 add, 1 sub, 2 mul, 3 div, 4 pow, 5 min, 6 max. */
static inline float binop(int op, float a, float b) {
    switch (op) {
    case 0: return a + b;
    case 1: return a - b;
    case 2: return a * b;
    case 3: return a / b;
    case 4: return powf(a, b);
    case 5: return fminf(a, b);
    default: return fmaxf(a, b);
    }
}

int jxo_binary_broadcast(int op, const float *a, const int64_t *ad, int an, const float *b,
                         const int64_t *bd, int bn, float *out, int64_t *od, int *on) {
    int nd = an > bn ? an : bn;
    int64_t dims[16];
    if (nd > 16) return -1;
    for (int i = 0; i < nd; ++i) {
        int ia = i - (nd - an), ib = i - (nd - bn);
        int64_t da = ia >= 0 ? ad[ia] : 1, db = ib >= 0 ? bd[ib] : 1;
        if (da != db && da != 1 && db != 1) return -1;
        dims[i] = da == 1 ? db : da;
    }
    int64_t total = 1;
    for (int i = 0; i < nd; ++i) { od[i] = dims[i]; total *= dims[i]; }
    *on = nd;
    for (int64_t f = 0; f < total; ++f) {
        int64_t rem = f, ia = 0, ib = 0, sa = 1, sb = 1;
        for (int i = nd - 1; i >= 0; --i) {
            int64_t idx = rem % dims[i];
            rem /= dims[i];
            int xa = i - (nd - an), xb = i - (nd - bn);
            if (xa >= 0) { if (ad[xa] != 1) ia += idx * sa; sa *= ad[xa]; }
            if (xb >= 0) { if (bd[xb] != 1) ib += idx * sb; sb *= bd[xb]; }
        }
        out[f] = binop(op, a[ia], b[ib]);
    }
    return 0;
}

/* The fused chain as the reference composes it:
 *   x.mul(a).add(b) -> nn::gelu -> .mul(&nn::sigmoid(x)) -> .sub(&x.tanh().div(2))
 * i.e. y = gelu(x*a + b) * sigmoid(x) - tanh(x)/2, every op rounded to f32.
 * Computing it per element in one loop gives the same bits as the 8 eager
 * passes because every intermediate is an f32 value either way. */
static inline float chain1(float x, float a, float b) {
    float u = x * a + b; /* two roundings: mul then add (no FMA under -ffp-contract=off) */
    float g = gelu1(u);
    float s = sigmoid1(x);
    float t = tanhf(x) / 2.0f;
    return g * s - t;
}

void jxo_chain_fwd(const float *x, float *y, int64_t n, float a, float b) {
    for (int64_t i = 0; i < n; ++i) y[i] = chain1(x[i], a, b);
}

/* The same chain as the reference executes it: eight eager passes, each
 * allocating a fresh output array (src/ops/binary.rs:7-74, src/nn.rs:111-140,
 * src/ops/unary.rs:30-49).  Used only to time the reference CPU path. */
void jxo_chain_fwd_eager(const float *x, float *y, int64_t n, float a, float b) {
    float *t1 = (float *)malloc(sizeof(float) * n); for (int64_t i = 0; i < n; ++i) t1[i] = x[i] * a;
    float *t2 = (float *)malloc(sizeof(float) * n); for (int64_t i = 0; i < n; ++i) t2[i] = t1[i] + b;
    float *t3 = (float *)malloc(sizeof(float) * n); for (int64_t i = 0; i < n; ++i) t3[i] = gelu1(t2[i]);
    float *t4 = (float *)malloc(sizeof(float) * n); for (int64_t i = 0; i < n; ++i) t4[i] = sigmoid1(x[i]);
    float *t5 = (float *)malloc(sizeof(float) * n); for (int64_t i = 0; i < n; ++i) t5[i] = t3[i] * t4[i];
    float *t6 = (float *)malloc(sizeof(float) * n); for (int64_t i = 0; i < n; ++i) t6[i] = tanhf(x[i]);
    float *t7 = (float *)malloc(sizeof(float) * n); for (int64_t i = 0; i < n; ++i) t7[i] = t6[i] / 2.0f;
    for (int64_t i = 0; i < n; ++i) y[i] = t5[i] - t7[i];
    free(t1); free(t2); free(t3); free(t4); free(t5); free(t6); free(t7);
}

/* Restated adjoint: VJP of the chain with cotangent ct (ones for grad).
 * dy/dx = gelu'(u)*a*s + g*s*(1-s) - (1 - tanh(x)^2)/2,   u = x*a+b,
 * gelu'(u) = 0.5*(1+t) + 0.5*u*(1-t^2)*coeff*(1 + 3*0.044715*u^2), t = tanh(inner).
 * Per-primitive rules: transpose_mul src/trace/transpose_rules.rs:279-307,
 * transpose_tanh :136-154; the gelu and sigmoid derivatives are the
 * mathematical derivatives of src/nn.rs:111-140 (the reference leaves them untraced). */
void jxo_chain_vjp(const float *x, const float *ct, float *y, float *dx, int64_t n, float a, float b) {
    const float coeff = sqrtf(2.0f / JXO_PI_F);
    for (int64_t i = 0; i < n; ++i) {
        float xv = x[i];
        float u = xv * a + b;
        float u2 = u * u;
        float inner = coeff * (u + GELU_C1 * (u * u2));
        float t = tanhf(inner);
        float g = 0.5f * u * (1.0f + t);
        float s = 1.0f / (1.0f + expf(-xv));
        float th = tanhf(xv);
        if (y) y[i] = g * s - th / 2.0f;
        float dinner = coeff * (1.0f + 3.0f * GELU_C1 * u2);
        float dg = 0.5f * (1.0f + t) + 0.5f * u * (1.0f - t * t) * dinner;
        float d = dg * a * s + g * (s * (1.0f - s)) - (1.0f - th * th) / 2.0f;
        dx[i] = ct ? d * ct[i] : d;
    }
}

/* f64 twin of the chain and its derivative (accuracy yardstick only). */
void jxo_chain_f64(const float *x, double *y, double *dx, int64_t n, float a, float b) {
    const double coeff = sqrt(2.0 / 3.14159265358979323846);
    for (int64_t i = 0; i < n; ++i) {
        double xv = x[i], u = xv * a + b, u2 = u * u;
        double t = tanh(coeff * (u + 0.044715 * u * u2));
        double g = 0.5 * u * (1.0 + t);
        double s = 1.0 / (1.0 + exp(-xv));
        double th = tanh(xv);
        if (y) y[i] = g * s - th / 2.0;
        if (dx) {
            double dg = 0.5 * (1.0 + t) + 0.5 * u * (1.0 - t * t) * coeff * (1.0 + 3.0 * 0.044715 * u2);
            dx[i] = dg * a * s + g * s * (1.0 - s) - (1.0 - th * th) / 2.0;
        }
    }
}

/* ------------------------------------------------------------------------- */
/* Reductions (src/ops/reduce.rs)                                            */
/* op: 0 sum, 1 max, 2 min, 3 prod                                           */
/* ------------------------------------------------------------------------- */
static inline float red_init(int op) {
    return op == 0 ? 0.0f : op == 1 ? -INFINITY : op == 2 ? INFINITY : 1.0f;
}
static inline float red_f(int op, float acc, float x) {
    return op == 0 ? acc + x : op == 1 ? fmaxf(acc, x) : op == 2 ? fminf(acc, x) : acc * x;
}

/* src/ops/reduce.rs:19-50 reduce_all_gpu_aware CPU arm: fold from init. */
float jxo_reduce_all(const float *x, int64_t n, int op) {
    float acc = red_init(op);
    for (int64_t i = 0; i < n; ++i) acc = red_f(op, acc, x[i]);
    return acc;
}

double jxo_sum_all_f64(const float *x, int64_t n) {
    double s = 0.0, c = 0.0; /* Kahan */
    for (int64_t i = 0; i < n; ++i) {
        double y = (double)x[i] - c, t = s + y;
        c = (t - s) - y;
        s = t;
    }
    return s;
}

/* src/ops/reduce.rs:53-135 reduce_axis: for each output, fold over the axis
 * from init in index order.  The array is viewed as [outer, len, inner]. */
typedef struct { const float *x; float *y; int64_t len, inner; int op; } ra_ctx;
static void ra_rows(void *p, int64_t o0, int64_t o1) {
    ra_ctx *c = (ra_ctx *)p;
    for (int64_t o = o0; o < o1; ++o)
        for (int64_t in = 0; in < c->inner; ++in) {
            float acc = red_init(c->op);
            const float *base = c->x + o * c->len * c->inner + in;
            for (int64_t a = 0; a < c->len; ++a) acc = red_f(c->op, acc, base[a * c->inner]);
            c->y[o * c->inner + in] = acc;
        }
}
void jxo_reduce_axis(const float *x, float *y, int64_t outer, int64_t len, int64_t inner, int op, int nthreads) {
    ra_ctx ctx = {x, y, len, inner, op};
    parallel_rows(ra_rows, &ctx, outer, nthreads);
}

/* f64 twin of the last-axis sum. */
void jxo_sum_rows_f64(const float *x, double *y, int64_t rows, int64_t cols) {
    for (int64_t r = 0; r < rows; ++r) {
        double s = 0.0;
        for (int64_t c = 0; c < cols; ++c) s += x[r * cols + c];
        y[r] = s;
    }
}

/* src/ops/reduce.rs:301-309 argmax: Iterator::max_by(partial_cmp) keeps the
 * LAST of equal maxima.  :281-289 argmin: min_by keeps the FIRST of equal
 * minima.  Restated per row of a [rows, cols] array.  Returns -1 (the
 * reference panics) if a NaN is met. */
typedef struct { const float *x; int32_t *idx; int64_t cols; int is_max; int bad; } am_ctx;
static void am_rows(void *p, int64_t r0, int64_t r1) {
    am_ctx *c = (am_ctx *)p;
    for (int64_t r = r0; r < r1; ++r) {
        const float *row = c->x + r * c->cols;
        int64_t best = 0;
        float bv = row[0];
        if (bv != bv) c->bad = 1;
        for (int64_t j = 1; j < c->cols; ++j) {
            float v = row[j];
            if (v != v) { c->bad = 1; continue; }
            if (c->is_max ? (v >= bv) : (v < bv)) { bv = v; best = j; }
        }
        c->idx[r] = (int32_t)best;
    }
}
int jxo_arg_rows(const float *x, int32_t *idx, int64_t rows, int64_t cols, int is_max, int nthreads) {
    am_ctx ctx = {x, idx, cols, is_max, 0};
    parallel_rows(am_rows, &ctx, rows, nthreads);
    return ctx.bad ? -1 : 0;
}

/* VJP of sum over the last axis (transpose_sum_axis src/trace/transpose_rules.rs:409-418):
 * dx[r, c] = ct[r]. */
void jxo_sum_rows_vjp(const float *ct, float *dx, int64_t rows, int64_t cols) {
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t c = 0; c < cols; ++c) dx[r * cols + c] = ct[r];
}

/* VJP of max over the last axis, applying transpose_max_all's rule per row
 * (src/trace/transpose_rules.rs:444-469): mask = (x == max); count = sum(mask);
 * if count > 1 the mask is scaled by (1/count); times the cotangent. */
void jxo_max_rows_vjp(const float *x, const float *ct, float *dx, int64_t rows, int64_t cols) {
    for (int64_t r = 0; r < rows; ++r) {
        const float *row = x + r * cols;
        float m = -INFINITY;
        for (int64_t c = 0; c < cols; ++c) m = fmaxf(m, row[c]);
        float count = 0.0f;
        for (int64_t c = 0; c < cols; ++c) count += (row[c] == m) ? 1.0f : 0.0f;
        float scale = count > 1.0f ? 1.0f / count : 1.0f;
        for (int64_t c = 0; c < cols; ++c) {
            float mask = (row[c] == m) ? 1.0f : 0.0f;
            float nm = count > 1.0f ? mask * scale : mask;
            dx[r * cols + c] = nm * ct[r];
        }
    }
}

/* ------------------------------------------------------------------------- */
/* FFT: src/ops/fft.rs:25-70 (recursive radix-2 DIT, twiddles in f32),        */
/* ifft 1/n scaling :174-179, fft2/ifft2 row-then-column order :261-396.      */
/* Complex values are interleaved [re, im] f32.                              */
/* ------------------------------------------------------------------------- */
typedef struct { float re, im; } cpx;

/* src/ops/fft.rs:33-37 twiddle_factor: angle = 2*PI*k/n in f32; (cos, -+sin) */
static inline cpx twiddle(int64_t k, int64_t n, int inverse) {
    float angle = 2.0f * JXO_PI_F * (float)k / (float)n;
    float sign = inverse ? 1.0f : -1.0f;
    cpx t = {cosf(angle), sign * sinf(angle)};
    return t;
}

static void fft_rec(const cpx *in, cpx *out, int64_t n, int inverse, cpx *scratch) {
    if (n <= 1) { if (n == 1) out[0] = in[0]; return; }
    int64_t h = n / 2;
    cpx *even = scratch, *odd = scratch + h;
    for (int64_t i = 0; i < h; ++i) { even[i] = in[2 * i]; odd[i] = in[2 * i + 1]; }
    cpx *fe = out, *fo = out + h; /* results of the halves, combined below */
    cpx *sub = scratch + n;
    fft_rec(even, fe, h, inverse, sub);
    fft_rec(odd, fo, h, inverse, sub);
    /* combine (src/ops/fft.rs:61-66); copy halves first since out aliases them */
    cpx *tmp = scratch; /* even/odd inputs are no longer needed */
    memcpy(tmp, out, sizeof(cpx) * n);
    for (int64_t k = 0; k < h; ++k) {
        cpx w = twiddle(k, n, inverse);
        cpx o = tmp[h + k], e = tmp[k];
        /* complex_mul src/ops/fft.rs:27-29: (a.re*b.re - a.im*b.im, a.re*b.im + a.im*b.re) */
        cpx t = {w.re * o.re - w.im * o.im, w.re * o.im + w.im * o.re};
        out[k].re = e.re + t.re; out[k].im = e.im + t.im;
        out[k + h].re = e.re - t.re; out[k + h].im = e.im - t.im;
    }
}

/* Batched complex-to-complex 1-D FFT of length n (power of two).  Forward
 * calls fft_recursive(.., false); inverse calls fft_recursive(.., true) and
 * scales by 1/n as ifft does. */
typedef struct { const float *in; float *out; int64_t n; int inverse; } fft_ctx;
static void fft_rows(void *p, int64_t b0, int64_t b1) {
    fft_ctx *c = (fft_ctx *)p;
    int64_t n = c->n;
    cpx *scratch = (cpx *)malloc(sizeof(cpx) * (4 * n + 4));
    for (int64_t b = b0; b < b1; ++b) {
        const cpx *in = (const cpx *)(c->in + 2 * n * b);
        cpx *out = (cpx *)(c->out + 2 * n * b);
        fft_rec(in, out, n, c->inverse, scratch);
        if (c->inverse) {
            float scale = 1.0f / (float)n;
            for (int64_t i = 0; i < n; ++i) { out[i].re *= scale; out[i].im *= scale; }
        }
    }
    free(scratch);
}
int jxo_fft_c2c(const float *in, float *out, int64_t n, int64_t batch, int inverse, int nthreads) {
    if (n <= 0 || (n & (n - 1)) != 0) return -1;
    fft_ctx ctx = {in, out, n, inverse};
    parallel_rows(fft_rows, &ctx, batch, nthreads);
    return 0;
}

/* 2-D: rows of length w first, then columns of length h (fft2 / ifft2 order). */
int jxo_fft2_c2c(const float *in, float *out, int64_t h, int64_t w, int64_t batch, int inverse, int nthreads) {
    if (jxo_fft_c2c(in, out, w, h * batch, inverse, nthreads) != 0) return -1;
    if (h <= 0 || (h & (h - 1)) != 0) return -1;
    float *col = (float *)malloc(sizeof(float) * 2 * h);
    float *colo = (float *)malloc(sizeof(float) * 2 * h);
    for (int64_t b = 0; b < batch; ++b) {
        float *img = out + 2 * h * w * b;
        for (int64_t j = 0; j < w; ++j) {
            for (int64_t i = 0; i < h; ++i) { col[2 * i] = img[2 * (i * w + j)]; col[2 * i + 1] = img[2 * (i * w + j) + 1]; }
            jxo_fft_c2c(col, colo, h, 1, inverse, 1);
            for (int64_t i = 0; i < h; ++i) { img[2 * (i * w + j)] = colo[2 * i]; img[2 * (i * w + j) + 1] = colo[2 * i + 1]; }
        }
    }
    free(col); free(colo);
    return 0;
}

/* Real-input and real-output transforms, per batch row.  fft (real input,
 * src/ops/fft.rs:91-126): widen to complex (imaginary 0), fft_recursive,
 * all n bins.  rfft (:212-234): the same, first n/2+1 bins. */
int jxo_fft_real(const float *in, float *out, int64_t n, int64_t batch, int full) {
    if (n <= 0 || (n & (n - 1)) != 0) return -1;
    int64_t bins = full ? n : n / 2 + 1;
    cpx *x = (cpx *)malloc(sizeof(cpx) * n), *y = (cpx *)malloc(sizeof(cpx) * n);
    cpx *scratch = (cpx *)malloc(sizeof(cpx) * (4 * n + 4));
    for (int64_t b = 0; b < batch; ++b) {
        for (int64_t i = 0; i < n; ++i) { x[i].re = in[b * n + i]; x[i].im = 0.0f; }
        fft_rec(x, y, n, 0, scratch);
        for (int64_t k = 0; k < bins; ++k) { out[2 * (b * bins + k)] = y[k].re; out[2 * (b * bins + k) + 1] = y[k].im; }
    }
    free(x); free(y); free(scratch);
    return 0;
}

/* irfft (src/ops/fft.rs:417-462): bins 0..m-1 as given, then conj(X[i]) for
 * i = n-m down to 1; fft_recursive(.., inverse); times 1/n; real parts. */
int jxo_irfft(const float *in, float *out, int64_t n, int64_t batch) {
    if (n <= 0 || (n & (n - 1)) != 0) return -1;
    int64_t m = n / 2 + 1;
    cpx *x = (cpx *)malloc(sizeof(cpx) * n), *y = (cpx *)malloc(sizeof(cpx) * n);
    cpx *scratch = (cpx *)malloc(sizeof(cpx) * (4 * n + 4));
    for (int64_t b = 0; b < batch; ++b) {
        const float *d = in + 2 * m * b;
        int64_t p = 0;
        for (int64_t i = 0; i < m; ++i) { x[p].re = d[2 * i]; x[p].im = d[2 * i + 1]; ++p; }
        for (int64_t i = n - m; i >= 1; --i) { x[p].re = d[2 * i]; x[p].im = -d[2 * i + 1]; ++p; }
        fft_rec(x, y, n, 1, scratch);
        float scale = 1.0f / (float)n;
        for (int64_t i = 0; i < n; ++i) out[b * n + i] = y[i].re * scale;
    }
    free(x); free(y); free(scratch);
    return 0;
}

/* rfftn 2-D (src/ops/fft.rs:474-553): full fft of each row, then fft of each
 * of the first w/2+1 columns; result [h][w/2+1] complex. */
int jxo_rfftn2(const float *in, float *out, int64_t h, int64_t w, int64_t batch) {
    int64_t m = w / 2 + 1;
    float *rows = (float *)malloc(sizeof(float) * 2 * h * w);
    float *col = (float *)malloc(sizeof(float) * 2 * h), *colo = (float *)malloc(sizeof(float) * 2 * h);
    for (int64_t b = 0; b < batch; ++b) {
        if (jxo_fft_real(in + b * h * w, rows, w, h, 1) != 0) return -1;
        for (int64_t j = 0; j < m; ++j) {
            for (int64_t i = 0; i < h; ++i) { col[2 * i] = rows[2 * (i * w + j)]; col[2 * i + 1] = rows[2 * (i * w + j) + 1]; }
            if (jxo_fft_c2c(col, colo, h, 1, 0, 1) != 0) return -1;
            for (int64_t i = 0; i < h; ++i) {
                out[2 * (b * h * m + i * m + j)] = colo[2 * i];
                out[2 * (b * h * m + i * m + j) + 1] = colo[2 * i + 1];
            }
        }
    }
    free(rows); free(col); free(colo);
    return 0;
}

/* irfftn 2-D (src/ops/fft.rs:554-628): inverse fft of each of the w/2+1
 * columns (times 1/h), then per row the conjugate-symmetric extension, the
 * inverse fft and times 1/w, real parts. */
int jxo_irfftn2(const float *in, float *out, int64_t h, int64_t w, int64_t batch) {
    int64_t m = w / 2 + 1;
    float *cols = (float *)malloc(sizeof(float) * 2 * h * m);
    float *col = (float *)malloc(sizeof(float) * 2 * h), *colo = (float *)malloc(sizeof(float) * 2 * h);
    for (int64_t b = 0; b < batch; ++b) {
        const float *d = in + 2 * h * m * b;
        for (int64_t j = 0; j < m; ++j) {
            for (int64_t i = 0; i < h; ++i) { col[2 * i] = d[2 * (i * m + j)]; col[2 * i + 1] = d[2 * (i * m + j) + 1]; }
            /* fft_recursive(.., true), then * (1/h) */
            cpx *scratch = (cpx *)malloc(sizeof(cpx) * (4 * h + 4));
            fft_rec((const cpx *)col, (cpx *)colo, h, 1, scratch);
            free(scratch);
            float scale = 1.0f / (float)h;
            for (int64_t i = 0; i < h; ++i) {
                cols[2 * (i * m + j)] = colo[2 * i] * scale;
                cols[2 * (i * m + j) + 1] = colo[2 * i + 1] * scale;
            }
        }
        if (jxo_irfft(cols, out + b * h * w, w, h) != 0) return -1;
    }
    free(cols); free(col); free(colo);
    return 0;
}

/* Plain O(n^2) DFT in f64 (yardstick for the FFT tests). */
void jxo_dft_f64(const float *in, double *out, int64_t n, int inverse) {
    for (int64_t k = 0; k < n; ++k) {
        double sr = 0.0, si = 0.0;
        for (int64_t t = 0; t < n; ++t) {
            double ang = (inverse ? 2.0 : -2.0) * 3.14159265358979323846 * (double)((k * t) % n) / (double)n;
            double c = cos(ang), s = sin(ang);
            sr += in[2 * t] * c - in[2 * t + 1] * s;
            si += in[2 * t] * s + in[2 * t + 1] * c;
        }
        out[2 * k] = inverse ? sr / n : sr;
        out[2 * k + 1] = inverse ? si / n : si;
    }
}

/* ------------------------------------------------------------------------- */
/* conv2d (src/nn.rs:2097-2138): NCHW input, OIHW kernel, loop order        */
/* b -> oc -> oh -> ow -> ic -> kh -> kw, f32 accumulate, padding skipped.   */
/* ------------------------------------------------------------------------- */
typedef struct {
    const float *x, *w, *dy; float *y;
    int64_t B, C, H, W, O, KH, KW, stride, pad, OH, OW;
} conv_ctx;

static void conv_fwd_rows(void *p, int64_t b0, int64_t b1) {
    conv_ctx *c = (conv_ctx *)p;
    for (int64_t b = b0; b < b1; ++b)
        for (int64_t oc = 0; oc < c->O; ++oc)
            for (int64_t oh = 0; oh < c->OH; ++oh)
                for (int64_t ow = 0; ow < c->OW; ++ow) {
                    float sum = 0.0f;
                    for (int64_t ic = 0; ic < c->C; ++ic)
                        for (int64_t kh = 0; kh < c->KH; ++kh)
                            for (int64_t kw = 0; kw < c->KW; ++kw) {
                                int64_t ih = oh * c->stride + kh - c->pad;
                                int64_t iw = ow * c->stride + kw - c->pad;
                                if (ih >= 0 && ih < c->H && iw >= 0 && iw < c->W)
                                    sum += c->x[((b * c->C + ic) * c->H + ih) * c->W + iw] *
                                           c->w[((oc * c->C + ic) * c->KH + kh) * c->KW + kw];
                            }
                    c->y[((b * c->O + oc) * c->OH + oh) * c->OW + ow] = sum;
                }
}

void jxo_conv2d_fwd(const float *x, const float *w, float *y, int64_t B, int64_t C, int64_t H, int64_t W,
                    int64_t O, int64_t KH, int64_t KW, int64_t stride, int64_t pad, int nthreads) {
    conv_ctx c = {x, w, NULL, y, B, C, H, W, O, KH, KW, stride, pad,
                  (H + 2 * pad - KH) / stride + 1, (W + 2 * pad - KW) / stride + 1};
    parallel_rows(conv_fwd_rows, &c, B, nthreads);
}

/* Restated adjoint of the forward loop (no reference implementation):
 * dx[b,ic,ih,iw] = sum over (oc, kh, kw) with oh = (ih+pad-kh)/stride integral,
 * in loop order oc -> kh -> kw, f32 accumulate. */
static void conv_dx_rows(void *p, int64_t b0, int64_t b1) {
    conv_ctx *c = (conv_ctx *)p;
    for (int64_t b = b0; b < b1; ++b)
        for (int64_t ic = 0; ic < c->C; ++ic)
            for (int64_t ih = 0; ih < c->H; ++ih)
                for (int64_t iw = 0; iw < c->W; ++iw) {
                    float sum = 0.0f;
                    for (int64_t oc = 0; oc < c->O; ++oc)
                        for (int64_t kh = 0; kh < c->KH; ++kh)
                            for (int64_t kw = 0; kw < c->KW; ++kw) {
                                int64_t th = ih + c->pad - kh, tw = iw + c->pad - kw;
                                if (th < 0 || tw < 0 || th % c->stride || tw % c->stride) continue;
                                int64_t oh = th / c->stride, ow = tw / c->stride;
                                if (oh >= c->OH || ow >= c->OW) continue;
                                sum += c->dy[((b * c->O + oc) * c->OH + oh) * c->OW + ow] *
                                       c->w[((oc * c->C + ic) * c->KH + kh) * c->KW + kw];
                            }
                    c->y[((b * c->C + ic) * c->H + ih) * c->W + iw] = sum;
                }
}
void jxo_conv2d_bwd_data(const float *dy, const float *w, float *dx, int64_t B, int64_t C, int64_t H,
                         int64_t W, int64_t O, int64_t KH, int64_t KW, int64_t stride, int64_t pad, int nthreads) {
    conv_ctx c = {NULL, w, dy, dx, B, C, H, W, O, KH, KW, stride, pad,
                  (H + 2 * pad - KH) / stride + 1, (W + 2 * pad - KW) / stride + 1};
    parallel_rows(conv_dx_rows, &c, B, nthreads);
}

/* Restated adjoint: dw[oc,ic,kh,kw] = sum over (b, oh, ow) of dy*x, loop order b -> oh -> ow. */
static void conv_dw_rows(void *p, int64_t o0, int64_t o1) {
    conv_ctx *c = (conv_ctx *)p;
    for (int64_t oc = o0; oc < o1; ++oc)
        for (int64_t ic = 0; ic < c->C; ++ic)
            for (int64_t kh = 0; kh < c->KH; ++kh)
                for (int64_t kw = 0; kw < c->KW; ++kw) {
                    float sum = 0.0f;
                    for (int64_t b = 0; b < c->B; ++b)
                        for (int64_t oh = 0; oh < c->OH; ++oh)
                            for (int64_t ow = 0; ow < c->OW; ++ow) {
                                int64_t ih = oh * c->stride + kh - c->pad;
                                int64_t iw = ow * c->stride + kw - c->pad;
                                if (ih >= 0 && ih < c->H && iw >= 0 && iw < c->W)
                                    sum += c->dy[((b * c->O + oc) * c->OH + oh) * c->OW + ow] *
                                           c->x[((b * c->C + ic) * c->H + ih) * c->W + iw];
                            }
                    c->y[((oc * c->C + ic) * c->KH + kh) * c->KW + kw] = sum;
                }
}
void jxo_conv2d_bwd_filter(const float *x, const float *dy, float *dw, int64_t B, int64_t C, int64_t H,
                           int64_t W, int64_t O, int64_t KH, int64_t KW, int64_t stride, int64_t pad, int nthreads) {
    conv_ctx c = {x, NULL, dy, dw, B, C, H, W, O, KH, KW, stride, pad,
                  (H + 2 * pad - KH) / stride + 1, (W + 2 * pad - KW) / stride + 1};
    parallel_rows(conv_dw_rows, &c, O, nthreads);
}

/* ------------------------------------------------------------------------- */
/* nn: softmax (src/nn.rs:155-168, applied per row), log_softmax (:181-193), */
/* one_hot (:205-221), cross_entropy_loss (:300-318)                         */
/* ------------------------------------------------------------------------- */
void jxo_softmax_rows(const float *x, float *y, int64_t rows, int64_t cols) {
    for (int64_t r = 0; r < rows; ++r) {
        const float *in = x + r * cols;
        float *out = y + r * cols;
        float m = -INFINITY;
        for (int64_t c = 0; c < cols; ++c) m = fmaxf(m, in[c]);
        float sum = 0.0f;
        for (int64_t c = 0; c < cols; ++c) { out[c] = expf(in[c] - m); sum += out[c]; }
        for (int64_t c = 0; c < cols; ++c) out[c] = out[c] / sum;
    }
}

void jxo_log_softmax_rows(const float *x, float *y, int64_t rows, int64_t cols) {
    for (int64_t r = 0; r < rows; ++r) {
        const float *in = x + r * cols;
        float m = -INFINITY;
        for (int64_t c = 0; c < cols; ++c) m = fmaxf(m, in[c]);
        float s = 0.0f;
        for (int64_t c = 0; c < cols; ++c) s += expf(in[c] - m);
        float lse = logf(s);
        for (int64_t c = 0; c < cols; ++c) y[r * cols + c] = (in[c] - m) - lse;
    }
}

void jxo_one_hot(const float *idx, float *out, int64_t n, int64_t classes) {
    memset(out, 0, sizeof(float) * n * classes);
    for (int64_t i = 0; i < n; ++i) {
        float v = idx[i];
        /* `idx as usize` saturates negatives to 0 and truncates toward zero */
        uint64_t cls = v <= 0.0f ? 0 : (uint64_t)v;
        if (v != v) cls = 0;
        if (cls < (uint64_t)classes) out[i * classes + cls] = 1.0f;
    }
}

/* src/nn.rs:300-318: -sum(t * ln(p + 1e-7)) / len, summed in element order. */
float jxo_cross_entropy(const float *p, const float *t, int64_t n) {
    float sum = 0.0f;
    for (int64_t i = 0; i < n; ++i) sum += -t[i] * logf(p[i] + 1e-7f);
    return sum / (float)n;
}

/* ------------------------------------------------------------------------- */
/* Adam: src/optim.rs:138-189, elementwise in the reference's op order.      */
/* first != 0 means state.m/state.v are None (step 1).                       */
/* ------------------------------------------------------------------------- */
void jxo_adam_update(float *p, const float *g, float *m, float *v, int64_t n, float lr, float b1, float b2,
                     float eps, int64_t step, int first) {
    float t = (float)step;
    float bc1 = 1.0f - powf(b1, t);
    float bc2 = 1.0f - powf(b2, t);
    float r1 = 1.0f / bc1, r2 = 1.0f / bc2;
    float omb1 = 1.0f - b1, omb2 = 1.0f - b2;
    for (int64_t i = 0; i < n; ++i) {
        float gi = g[i];
        float mi = first ? gi * omb1 : m[i] * b1 + gi * omb1;
        float g2 = gi * gi;
        float vi = first ? g2 * omb2 : v[i] * b2 + g2 * omb2;
        float mh = mi * r1;
        float vh = vi * r2;
        float upd = (mh / (sqrtf(vh) + eps)) * lr;
        p[i] = p[i] - upd;
        m[i] = mi;
        v[i] = vi;
    }
}

/* ------------------------------------------------------------------------- */
/* Dense layer pieces used by the MLP training step (composition of         */
/* Array::matmul, broadcast_to + add, relu/gelu, softmax, cross_entropy).    */
/* ------------------------------------------------------------------------- */

/* y[B,N] = x[B,K].w[K,N] + bias[N]  (matmul then broadcast add, src/ops/manipulation.rs:919-946) */
void jxo_dense_fwd(const float *x, const float *w, const float *bias, float *y, int64_t B, int64_t K, int64_t N,
                   int nthreads) {
    jxo_matmul(x, w, y, B, N, K, nthreads);
    for (int64_t i = 0; i < B; ++i)
        for (int64_t j = 0; j < N; ++j) y[i * N + j] = y[i * N + j] + bias[j];
}

/* Restated adjoint of softmax (per row) followed by cross_entropy_loss over
 * all B*C elements (src/nn.rs:155-168,300-318), with the epsilon kept:
 * dp = -t / ((p + 1e-7) * (B*C)); dz = p * (dp - sum_k p_k*dp_k), per row in index order. */
void jxo_softmax_xent_bwd(const float *p, const float *t, float *dz, int64_t rows, int64_t cols) {
    float inv = (float)(rows * cols);
    for (int64_t r = 0; r < rows; ++r) {
        const float *pr = p + r * cols, *tr = t + r * cols;
        float s = 0.0f;
        for (int64_t c = 0; c < cols; ++c) {
            float dp = -tr[c] / ((pr[c] + 1e-7f) * inv);
            s += pr[c] * dp;
        }
        for (int64_t c = 0; c < cols; ++c) {
            float dp = -tr[c] / ((pr[c] + 1e-7f) * inv);
            dz[r * cols + c] = pr[c] * (dp - s);
        }
    }
}

/* Column sums of dY[B,N] (bias gradient: transpose of broadcast_to), row order. */
void jxo_col_sum(const float *dy, float *db, int64_t B, int64_t N) {
    for (int64_t j = 0; j < N; ++j) db[j] = 0.0f;
    for (int64_t i = 0; i < B; ++i)
        for (int64_t j = 0; j < N; ++j) db[j] = db[j] + dy[i * N + j];
}

/* ------------------------------------------------------------------------- */
/* Layers that the reference runs as WGSL-only kernels or CPU loops:          */
/* conv1d, 2-D pooling, global pooling, batch / layer normalisation.         */
/* ------------------------------------------------------------------------- */

/* Batched multi-channel 1-D convolution, the conv1d shader's loop
 * (src/backend/shaders.rs:449-519, launched by gpu_conv1d
 * src/backend/ops.rs:1014-1200): y[b,o,p] = sum over ic, then k, of
 * x[b,ic,p*stride+k-pad] * w[o,ic,k], padded taps skipped, f32 accumulate from
 * 0.  With batch = channels = 1, stride 1 and pad 0 this is nn::conv1d's CPU
 * loop (src/nn.rs:1662-1722). */
typedef struct { const float *x, *w; float *y; int64_t B, C, L, O, K, S, P, OL; } conv1_ctx;
static void conv1_rows(void *p, int64_t r0, int64_t r1) {
    conv1_ctx *c = (conv1_ctx *)p;
    for (int64_t r = r0; r < r1; ++r) {  /* r = b*O + o */
        int64_t b = r / c->O, o = r % c->O;
        for (int64_t q = 0; q < c->OL; ++q) {
            float sum = 0.0f;
            int64_t start = q * c->S - c->P;
            for (int64_t ic = 0; ic < c->C; ++ic)
                for (int64_t k = 0; k < c->K; ++k) {
                    int64_t ip = start + k;
                    if (ip < 0 || ip >= c->L) continue;
                    sum += c->x[(b * c->C + ic) * c->L + ip] * c->w[(o * c->C + ic) * c->K + k];
                }
            c->y[r * c->OL + q] = sum;
        }
    }
}
int jxo_conv1d(const float *x, const float *w, float *y, int64_t B, int64_t C, int64_t L, int64_t O, int64_t K,
               int64_t stride, int64_t pad, int nthreads) {
    if (K < 1 || stride < 1 || pad < 0 || L + 2 * pad < K) return -1;
    conv1_ctx c = {x, w, y, B, C, L, O, K, stride, pad, (L + 2 * pad - K) / stride + 1};
    parallel_rows(conv1_rows, &c, B * O, nthreads);
    return 0;
}

/* 2-D pooling over [N, H, W] planes (N = batch*channels) with separate
 * window, stride and padding per axis.  Max: init -inf, f32::max over the
 * in-range taps in (ph, pw) order (nn::maxpool2d src/nn.rs:2164-2211,
 * max_pool2d :1121-1184, max_pool1d :1002-1047 with h = 1).  Average: the
 * in-range taps summed in (ph, pw) order from 0 and divided by their count, 0
 * if none (nn::avgpool2d :2231-2280; avg_pool2d :1199-1261 and avg_pool1d
 * :1059-1100 divide by the window area, the same count without padding). */
int jxo_pool2d(const float *x, float *y, int64_t N, int64_t H, int64_t W, int64_t kh, int64_t kw, int64_t sh,
               int64_t sw, int64_t ph_, int64_t pw_, int is_max) {
    if (kh < 1 || kw < 1 || sh < 1 || sw < 1 || ph_ < 0 || pw_ < 0 || H + 2 * ph_ < kh || W + 2 * pw_ < kw)
        return -1;
    int64_t OH = (H + 2 * ph_ - kh) / sh + 1, OW = (W + 2 * pw_ - kw) / sw + 1;
    for (int64_t n = 0; n < N; ++n)
        for (int64_t oh = 0; oh < OH; ++oh)
            for (int64_t ow = 0; ow < OW; ++ow) {
                float acc = is_max ? -INFINITY : 0.0f;
                int64_t count = 0;
                for (int64_t a = 0; a < kh; ++a)
                    for (int64_t b = 0; b < kw; ++b) {
                        int64_t ih = oh * sh + a - ph_, iw = ow * sw + b - pw_;
                        if (ih < 0 || ih >= H || iw < 0 || iw >= W) continue;
                        float v = x[(n * H + ih) * W + iw];
                        if (is_max) acc = fmaxf(acc, v); else acc += v;
                        ++count;
                    }
                y[(n * OH + oh) * OW + ow] = is_max ? acc : (count > 0 ? acc / (float)count : 0.0f);
            }
    return 0;
}

/* Global pooling of [N, S] rows (N = batch*channels, S = H*W):
 * global_avg_pool2d (src/nn.rs:2383-2408): sequential sum / S;
 * global_max_pool2d (:2431-2455): fold from -inf with f32::max. */
void jxo_global_pool(const float *x, float *y, int64_t N, int64_t S, int is_max) {
    for (int64_t n = 0; n < N; ++n) {
        float acc = is_max ? -INFINITY : 0.0f;
        for (int64_t i = 0; i < S; ++i) acc = is_max ? fmaxf(acc, x[n * S + i]) : acc + x[n * S + i];
        y[n] = is_max ? acc : acc / (float)S;
    }
}

/* Normalisation of x viewed as [outer, C, inner], statistics per channel over
 * outer*inner elements, in the reference's order: mean = sequential f32 sum /
 * count, var = sequential f32 sum of (x-mean)^2 / count, std = sqrt(var+eps),
 * y = (x - mean) / std * gamma + beta (batch_norm_2d src/nn.rs:2303-2360).
 * gamma == NULL skips the affine step: batch_norm [batch, features]
 * (:656-699, outer = batch, inner = 1) and layer_norm (:712-725, one
 * channel over the whole array). */
void jxo_batchnorm(const float *x, const float *gamma, const float *beta, float *y, int64_t outer, int64_t C,
                   int64_t inner, float eps, float *mean_out, float *var_out) {
    float count = (float)(outer * inner);
    for (int64_t c = 0; c < C; ++c) {
        float mean = 0.0f;
        for (int64_t o = 0; o < outer; ++o)
            for (int64_t i = 0; i < inner; ++i) mean += x[(o * C + c) * inner + i];
        mean /= count;
        float var = 0.0f;
        for (int64_t o = 0; o < outer; ++o)
            for (int64_t i = 0; i < inner; ++i) {
                float d = x[(o * C + c) * inner + i] - mean;
                var += d * d;
            }
        var /= count;
        float sd = sqrtf(var + eps);
        for (int64_t o = 0; o < outer; ++o)
            for (int64_t i = 0; i < inner; ++i) {
                int64_t idx = (o * C + c) * inner + i;
                float z = (x[idx] - mean) / sd;
                y[idx] = gamma ? z * gamma[c] + beta[c] : z;
            }
        if (mean_out) mean_out[c] = mean;
        if (var_out) var_out[c] = var;
    }
}

/* f64 statistics per channel (two passes in double) for checking device
 * statistics independently of the f32 summation order. */
void jxo_channel_stats_f64(const float *x, int64_t outer, int64_t C, int64_t inner, double *mean, double *var) {
    double cnt = (double)(outer * inner);
    for (int64_t c = 0; c < C; ++c) {
        double s = 0.0;
        for (int64_t o = 0; o < outer; ++o)
            for (int64_t i = 0; i < inner; ++i) s += x[(o * C + c) * inner + i];
        double m = s / cnt, v = 0.0;
        for (int64_t o = 0; o < outer; ++o)
            for (int64_t i = 0; i < inner; ++i) {
                double d = x[(o * C + c) * inner + i] - m;
                v += d * d;
            }
        mean[c] = m;
        var[c] = v / cnt;
    }
}

const char *jxo_version(void) { return "jaxrs-oracle 1 (restates jax-rs 0.5.1 CPU paths)"; }
