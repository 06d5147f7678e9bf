/*
 * jaxrs_cuda.h -- C ABI of the jax-rs B200 (sm_100a) compute backend.
 *
 * This is the FFI surface a `Device::Cuda(n)` arm of jax-rs binds.  Each entry
 * point names the reference interface it replaces (paths relative to the
 * jax-rs 0.5.1 source tree).  Conventions, mirroring the reference's
 * `gpu_*` launchers (src/backend/ops.rs):
 *   - outputs are pre-allocated by the caller, as `gpu_*` takes `&Buffer` outputs;
 *   - pointers are device pointers unless a parameter says "host";
 *   - all work is enqueued on `stream` (NULL = the legacy default stream) and
 *     nothing blocks except jx_memcpy_d2h / jx_stream_sync, the equivalent of
 *     the reference's blocking readback (src/buffer.rs:711-749);
 *   - every function returns JX_OK (0) or a JX_E* status; jx_last_error()
 *     returns the message of the calling thread's last failure.  The reference
 *     panics on the same conditions (e.g. src/backend/ops.rs:30-36); a Rust
 *     shim turns a non-zero status into that panic.
 */
#ifndef JAXRS_CUDA_H
#define JAXRS_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes --------------------------------------------------------- */
#define JX_OK 0
#define JX_EINVAL 1      /* bad argument (the reference's assert!/panic!) */
#define JX_ENOMEM 2      /* device allocation failed */
#define JX_ECUDA 3       /* CUDA runtime/driver error */
#define JX_ENCCL 4       /* NCCL error */
#define JX_ETIMEOUT 5    /* a bounded wait (device or host watchdog) expired */
#define JX_EUNSUPPORTED 6
#define JX_EDEVICE 7     /* a kernel flagged bad input (see jx_device_status) */
#define JX_EINTERNAL 8   /* a library invariant did not hold (a bug in this library) */

typedef void *jx_stream_t; /* a cudaStream_t */

#if defined(__GNUC__)
#define JX_API __attribute__((visibility("default")))
#else
#define JX_API
#endif

/* ---- context / device (src/backend/webgpu.rs:31-75, src/device.rs:10-80) -- */
JX_API const char *jx_last_error(void);
JX_API int jx_version(void);
/* WebGpuContext::init (src/backend/webgpu.rs:31-64): select and initialise a device.
 * device < 0 selects the process default: the JAXRS_DEVICE environment
 * variable, else device 0 (the reference's set-once default device,
 * src/device.rs:55-80). */
JX_API int jx_init(int device);
JX_API int jx_device_count(int *count);
JX_API int jx_set_device(int device);
JX_API int jx_get_device(int *device);
/* Device-side error word (bit 0: NaN met by an arg-reduction, bit 1: a bounded
 * wait timed out).  Reads and clears it, together with the fixed error word of
 * jx_gemm_f32_noalloc's launches (ORed in); synchronises the device. */
JX_API int jx_device_status(unsigned int *flags);

/* ---- storage (src/buffer.rs:40-122,581-590,700-749) ------------------------ */
/* Buffer::zeros (src/buffer.rs:40-74) when zero != 0; stream-ordered allocation. */
JX_API int jx_malloc(void **ptr, size_t nbytes, int zero, jx_stream_t stream);
/* Last drop of a Buffer (Arc<BufferInner>); stream-ordered free.  With
 * JAXRS_CHECK=1 set when the buffer was allocated, jx_malloc puts 256 canary
 * bytes after its end and jx_free checks them (synchronising the stream):
 * JX_EDEVICE if a kernel wrote past the end. */
JX_API int jx_free(void *ptr, jx_stream_t stream);
/* JAXRS_CHECK (no reference counterpart): checks the canary tails of every
 * live guarded buffer (synchronises the device); *corrupted = how many were
 * overwritten. */
JX_API int jx_check_guards(int *corrupted);
/* Fault injection on the host (no reference counterpart): the next `count`
 * device allocations (jx_malloc and the library's own scratch) fail with
 * JX_ENOMEM; 0 disarms. */
JX_API int jx_selftest_fail_alloc(int count);
/* Buffer::from_f32 upload (src/buffer.rs:81-122).  `src` is host memory. */
JX_API int jx_memcpy_h2d(void *dst, const void *src, size_t nbytes, jx_stream_t stream);
/* Buffer::to_f32_vec readback (src/buffer.rs:581-590,711-749): blocks until the
 * copy lands in host memory `dst`. */
JX_API int jx_memcpy_d2h(void *dst, const void *src, size_t nbytes, jx_stream_t stream);
JX_API int jx_memcpy_d2d(void *dst, const void *src, size_t nbytes, jx_stream_t stream);
JX_API int jx_stream_create(jx_stream_t *stream);
JX_API int jx_stream_destroy(jx_stream_t stream);
JX_API int jx_stream_sync(jx_stream_t stream);
/* Page-lock an existing host range (a Vec<f32>'s storage) so the *_host entry
 * points and jx_memcpy_* overlap their copies with the math; no reference
 * counterpart (its readback maps a staging buffer, src/buffer.rs:711-749).
 * Unregister before the memory is freed. */
JX_API int jx_host_register(void *ptr, size_t nbytes);
JX_API int jx_host_unregister(void *ptr);

/* ---- GEMM (gpu_matmul src/backend/ops.rs:460-467; Array::matmul
 *      src/ops/linalg.rs:154-237; einsum "bij,bjk->bik" src/ops/einsum.rs:488-523) */
/* tcgen05 kind::tf32, A=Ah+Al, B=Bh+Bl, Ah.Bh+Ah.Bl+Al.Bh in TMEM f32.  Products
 * with at least one 256x256 tile per SM pair and TMA-compatible operands
 * (16-byte aligned, lda/ldb/batch strides multiples of 4) run on the SM-pair
 * kernel (see JX_PREC_3XTF32_PAIR); others split the operands into library
 * scratch first. */
#define JX_PREC_3XTF32 0
#define JX_PREC_EXACT 1  /* sequential-k f32, no FMA: the reference's CPU loop order, bit-exact */
/* JX_PREC_3XTF32 with the hi/lo split done inside the GEMM kernel from the
 * caller's f32 buffers: no split pass and no workspace.  Needs untransposed A
 * and B, 16-byte aligned, lda, ldb and batch strides multiples of 4 (and non-zero
 * batch strides when batch > 1); otherwise JX_EINVAL.  JX_PREC_3XTF32 picks
 * this kernel where it is faster and the SM-pair kernel does not apply (products of at least one 128x256 tile
 * per SM with small M or N). */
#define JX_PREC_3XTF32_FUSED 2
/* JX_PREC_3XTF32 on SM pairs (tcgen05 cta_group::2, a 256x256 tile per pair
 * of SMs, each SM holding half of B), the hi/lo split done in shared memory
 * from the caller's f32 buffers: no split pass, no workspace, any
 * transposition.  Needs 16-byte aligned A and B with lda, ldb and batch
 * strides multiples of 4 and at least one 256x256 tile per SM pair;
 * otherwise JX_EINVAL. */
#define JX_PREC_3XTF32_PAIR 3
/* C[b] = op(A[b]) . op(B[b]) for b < batch, row-major.  op(X) = X or X^T per
 * trans flags: A is [M,K] (or [K,M] when transA), B is [K,N] (or [N,K]).
 * lda/ldb/ldc: row strides in elements; stride*: batch strides in elements. */
JX_API int jx_gemm_f32(const float *A, const float *B, float *C, int64_t M, int64_t N, int64_t K, int transA,
                int transB, int64_t lda, int64_t ldb, int64_t ldc, int64_t batch, int64_t strideA,
                int64_t strideB, int64_t strideC, int precision, jx_stream_t stream);
/* Scratch bytes jx_gemm_f32 uses (library-owned) for JX_PREC_3XTF32. */
JX_API int jx_gemm_workspace_size(int64_t M, int64_t N, int64_t K, int64_t batch, size_t *bytes);
/* The two stages of JX_PREC_3XTF32, for operands reused across calls (a weight
 * matrix split once per step).  jx_gemm_kpad: K rounded up to the k-block.
 * jx_gemm_split_f32 writes hi = tf32(x), lo = tf32(x - hi) K-major:
 * hi/lo are [batch][rows][Kp]; element (r,k) is src[b*stride + r*ld + k], or
 * src[b*stride + k*ld + r] when trans != 0.  jx_gemm_presplit_f32 computes
 * C[b] = Ah.Bh^T + Ah.Bl^T + Al.Bh^T from such buffers (A rows = M, B rows = N);
 * a single product with fewer 128x256 tiles than SMs is cut along K and its
 * partial products added in order (split-K, library scratch). */
JX_API int jx_gemm_kpad(int64_t K, int64_t *Kp);
JX_API int jx_gemm_split_f32(const float *src, float *hi, float *lo, int64_t rows, int64_t K, int64_t ld,
                             int trans, int64_t batch, int64_t stride, jx_stream_t stream);
JX_API int jx_gemm_presplit_f32(const float *Ah, const float *Al, const float *Bh, const float *Bl, float *C,
                                int64_t M, int64_t N, int64_t Kp, int64_t ldc, int64_t batch, int64_t strideC,
                                jx_stream_t stream);
/* No counterpart in the reference (its readback is one blocking copy,
 * src/buffer.rs:711-749).  C = A . B (3xTF32) with A, B and C in host memory
 * (pinned for overlap), untransposed: B is uploaded and split once, then row
 * blocks of block_rows rows (0: about M/8) of A stream through the device
 * while the product of the previous block runs and the block before that
 * downloads, on three streams.  The caller's stream waits for the last
 * download. */
JX_API int jx_gemm_f32_host(const float *A, const float *B, float *C, int64_t M, int64_t N, int64_t K, int64_t lda,
                            int64_t ldb, int64_t ldc, int64_t block_rows, jx_stream_t stream);
/* Batched counterpart over host buffers (einsum "bij,bjk->bik" on host
 * arrays, src/ops/einsum.rs:488-523): A [batch][M][K], B [batch][K][N],
 * C [batch][M][N], contiguous; blocks of block_items entries (0: about 96 MiB
 * of operands) stream through the device, uploads, the batched 3xTF32
 * product and downloads overlapping on three streams. */
JX_API int jx_gemm_batched_f32_host(const float *A, const float *B, float *C, int64_t M, int64_t N, int64_t K,
                                    int64_t batch, int64_t block_items, jx_stream_t stream);
/* No counterpart in the reference.  jx_gemm_f32 (JX_PREC_3XTF32) for callers
 * that cannot let a library allocate device memory: a process whose own arena
 * or caching allocator already owns the device's memory, a latency-critical
 * loop that cannot afford an allocator call, or a plugin host that forbids
 * allocation behind its back.  It allocates nothing; its operand-split
 * workspace is a fixed 64 MiB device array inside the library, held by every
 * GPU that loads the library until the process exits.  Limit:
 * 2*batch*(M+N)*round_up(K,32) <= 16777216 floats, else JX_EINVAL.  The first
 * call on each device does that device's one-time set-up under a mutex (the
 * array's address by cudaGetSymbolAddress, the tensor-map encoder, the
 * kernel's shared-memory limit), so make that first call before any stream
 * capture.  All calls share the array: calls that overlap on the GPU race and
 * must be serialised by the caller.  K == 0 zero-fills C, as jx_gemm_f32.  A
 * bounded wait that gives up inside its launches is reported by
 * jx_device_status. */
JX_API int jx_gemm_f32_noalloc(const float *A, const float *B, float *C, int64_t M, int64_t N, int64_t K,
                               int transA, int transB, int64_t lda, int64_t ldb, int64_t ldc, int64_t batch,
                               int64_t strideA, int64_t strideB, int64_t strideC, jx_stream_t stream);

/* ---- elementwise (gpu_binary_op src/backend/ops.rs:21-26; binary_op with
 *      broadcasting src/ops/binary.rs:7-74,134-168; unary_op src/ops/unary.rs:30-49;
 *      nn::relu/gelu/sigmoid src/nn.rs:22-26,111-140) ----------------------- */
#define JX_BIN_ADD 0
#define JX_BIN_SUB 1
#define JX_BIN_MUL 2
#define JX_BIN_DIV 3
#define JX_BIN_POW 4
#define JX_BIN_MIN 5
#define JX_BIN_MAX 6
/* out = a op b with NumPy broadcasting of a_shape/b_shape (ndim <= 8). */
JX_API int jx_binary_f32(int op, const float *a, const int64_t *a_shape, int a_ndim, const float *b,
                  const int64_t *b_shape, int b_ndim, float *out, jx_stream_t stream);
#define JX_UN_NEG 0
#define JX_UN_ABS 1
#define JX_UN_SIN 2
#define JX_UN_COS 3
#define JX_UN_TANH 4
#define JX_UN_EXP 5
#define JX_UN_LOG 6
#define JX_UN_SQRT 7
#define JX_UN_RECIP 8
#define JX_UN_SQUARE 9
#define JX_UN_RELU 10
#define JX_UN_GELU 11
#define JX_UN_SIGMOID 12
#define JX_UN_GELU_GRAD 13 /* d/dx nn::gelu (restated adjoint, used by grad tapes) */
/* The remaining Array unary methods (src/ops/unary.rs:82-541): Rust f32 semantics;
 * ceil/floor/round (half away from zero)/trunc and sign (NaN -> 0) bit-identical. */
#define JX_UN_TAN 14
#define JX_UN_SIGN 15
#define JX_UN_SINH 16
#define JX_UN_COSH 17
#define JX_UN_ASIN 18
#define JX_UN_ACOS 19
#define JX_UN_ATAN 20
#define JX_UN_ASINH 21
#define JX_UN_ACOSH 22
#define JX_UN_ATANH 23
#define JX_UN_CEIL 24
#define JX_UN_FLOOR 25
#define JX_UN_ROUND 26
#define JX_UN_TRUNC 27
#define JX_UN_EXPM1 28
#define JX_UN_LOG1P 29
#define JX_UN_CBRT 30
#define JX_UN_LOG2 31
JX_API int jx_unary_f32(int op, const float *x, float *y, int64_t n, jx_stream_t stream);

/* ---- jit op-tape (FusedGroup src/trace/ir.rs:8-17; gpu_fused_execute
 *      src/backend/ops.rs:283-437; generate_fused_shader src/trace/fusion.rs:296-346)
 * A tape is a straight-line register program over per-element values.  Each
 * instruction is 4 int32 words {opcode, dst, src0, src1}; registers 0..nin-1
 * hold the inputs on entry; JX_OP_CONST loads consts[src0]; JX_OP_STORE writes
 * register src0 to output dst; registers 0..15 are usable.  The tape is
 * validated on creation (operands defined before use, every output stored).
 * Each distinct op structure is turned into one straight-line kernel (NVRTC,
 * sm_100a, cached per process and device); constants are passed in the
 * launch's parameter block, i.e. the constant bank, on every run. */
#define JX_OP_CONST 1
#define JX_OP_STORE 2
#define JX_OP_UNARY 16  /* opcode = 16 + JX_UN_* */
#define JX_OP_BINARY 48 /* opcode = 48 + JX_BIN_* */
#define JX_OP_SELECT_GT 64 /* dst = (src0 > 0) ? src1 : 0 (relu-style masks) */
#define JX_TAPE_MAX_INSTR 128
#define JX_TAPE_MAX_REGS 16
#define JX_TAPE_MAX_CONSTS 64
#define JX_TAPE_MAX_IO 4
typedef struct jx_tape jx_tape;
JX_API int jx_tape_create(const int32_t *code, int n_instr, const float *consts, int n_consts, int n_inputs,
                   int n_outputs, jx_tape **out);
JX_API int jx_tape_destroy(jx_tape *tape);
/* Generates and compiles (NVRTC, sm_100a) the kernel for this tape's op
 * structure on the current device, if the process has not already; the
 * first jx_tape_run does the same implicitly.  Tapes that differ only in their
 * constants share one compiled kernel. */
JX_API int jx_tape_compile(const jx_tape *tape);
/* The generated CUDA source of the tape's kernel (without the shared op
 * definitions), NUL-terminated into buf[cap]; *len = bytes needed. */
JX_API int jx_tape_source(const jx_tape *tape, char *buf, size_t cap, size_t *len);
/* Generates and NVRTC-compiles the tape's kernel without loading it (needs no GPU). */
JX_API int jx_tape_check(const jx_tape *tape);
/* ins/outs: host arrays of device pointers, each of n elements. */
JX_API int jx_tape_run(const jx_tape *tape, const float *const *ins, float *const *outs, int64_t n,
                jx_stream_t stream);
/* Inputs, outputs and instructions (after the tape's own rewrites). */
JX_API int jx_tape_info(const jx_tape *tape, int *n_inputs, int *n_outputs, int *n_instr);
/* jx_tape_run over host buffers (pinned for overlap): blocks of block_elems
 * elements (0: 8 Mi) stream through the device, uploads, the tape and
 * downloads on three streams overlapping.  The caller's stream waits for the
 * last download. */
JX_API int jx_tape_run_host(const jx_tape *tape, const float *const *ins, float *const *outs, int64_t n,
                            int64_t block_elems, jx_stream_t stream);

/* ---- random streams (PRNGKey src/random.rs:15-97; uniform_range :161-181;
 *      randint :189-210; normal's CPU arm :259-285)
 * (s0, s1) is a PRNGKey's state.  out[i] is exactly what the reference's
 * host loop writes at position i for the same key: uniform and randint
 * bit-identical, normal (Box-Muller, cos then sin per pair) within a few ulp
 * (CUDA's logf/cosf/sinf against glibc).  The device reaches position i by a
 * GF(2) jump-ahead of the xorshift128+ state, so any n runs fully parallel. */
JX_API int jx_random_uniform_f32(uint64_t s0, uint64_t s1, float *out, int64_t n, float minval, float maxval,
                                 jx_stream_t stream);
JX_API int jx_random_randint_f32(uint64_t s0, uint64_t s1, float *out, int64_t n, int32_t minval, int32_t maxval,
                                 jx_stream_t stream);
JX_API int jx_random_normal_f32(uint64_t s0, uint64_t s1, float *out, int64_t n, jx_stream_t stream);
/* Host: advance a key's state by `steps` draws of next_u64 (no GPU needed). */
JX_API int jx_random_jump(uint64_t *s0, uint64_t *s1, uint64_t steps);
/* Host: PRNGKey::from_seed and PRNGKey::split (src/random.rs:29-48). */
JX_API int jx_random_key_from_seed(uint64_t seed, uint64_t *s0, uint64_t *s1);
JX_API int jx_random_key_split(uint64_t s0, uint64_t s1, uint64_t *a0, uint64_t *a1, uint64_t *b0, uint64_t *b1);

/* ---- tracer: record, differentiate and fuse elementwise programs
 *      (TraceContext src/trace/tracer.rs:22-165; IRNode src/trace/ir.rs:8-386;
 *      find_fusible_groups src/trace/fusion.rs:97-294; VJPEngine
 *      src/trace/grad.rs:450-837 over src/trace/transpose_rules.rs;
 *      JitFunction::call src/trace/jit.rs:44-107)
 * A graph holds nodes over equal-length f32 vectors; node ids come back
 * through the last argument and are in topological order.  Identical nodes
 * are shared.  jx_graph_vjp appends, for cotangent nodes cts[i] of outputs
 * outs[i], the reverse-mode gradient nodes of every wrt[j] into grads[j]
 * (a zero constant when wrt[j] does not reach any output).  jx_graph_compile
 * fuses the nodes the outputs need into op-tapes (as many as the tape limits
 * require, with scratch buffers between them); jx_program_run runs them:
 * ins[i] is graph input i (in jx_graph_input call order), outs[j] receives
 * outs[j] of the compile call, all of n elements. */
typedef struct jx_graph jx_graph;
typedef struct jx_program jx_program;
JX_API int jx_graph_create(jx_graph **out);
JX_API int jx_graph_destroy(jx_graph *g);
JX_API int jx_graph_input(jx_graph *g, int *node);
JX_API int jx_graph_const(jx_graph *g, float value, int *node);
JX_API int jx_graph_unary(jx_graph *g, int op /* JX_UN_* */, int x, int *node);
JX_API int jx_graph_binary(jx_graph *g, int op /* JX_BIN_* */, int x, int y, int *node);
JX_API int jx_graph_select_gt(jx_graph *g, int x, int y, int *node); /* x > 0 ? y : 0 */
JX_API int jx_graph_size(const jx_graph *g, int *n_nodes, int *n_inputs);
JX_API int jx_graph_vjp(jx_graph *g, int n_out, const int *outs, const int *cts, int n_wrt, const int *wrt,
                        int *grads);
JX_API int jx_graph_compile(const jx_graph *g, int n_out, const int *outs, jx_program **out);
JX_API int jx_program_info(const jx_program *p, int *n_tapes, int *n_inputs, int *n_outputs, int *n_scratch);
JX_API int jx_program_tape(const jx_program *p, int index, const jx_tape **tape);
JX_API int jx_program_run(const jx_program *p, const float *const *ins, float *const *outs, int64_t n,
                          jx_stream_t stream);
JX_API int jx_program_destroy(jx_program *p);

/* ---- reductions (gpu_reduce_all src/backend/ops.rs:639-643; reduce_axis
 *      src/ops/reduce.rs:53-135; argmax/argmin src/ops/reduce.rs:281-309) ---- */
#define JX_RED_SUM 0
#define JX_RED_MAX 1
#define JX_RED_MIN 2
#define JX_RED_PROD 3
/* out[0] = fold(op) over n elements (device scalar). */
JX_API int jx_reduce_all_f32(const float *x, float *out, int64_t n, int op, jx_stream_t stream);
/* x viewed as [outer, len, inner]; out[outer, inner] = fold over len. */
JX_API int jx_reduce_axis_f32(const float *x, float *out, int64_t outer, int64_t len, int64_t inner, int op,
                       jx_stream_t stream);
/* Per-row arg reduction of x[rows, cols]: argmax keeps the LAST index among
 * equal maxima, argmin the FIRST among equal minima (Iterator::max_by/min_by).
 * A NaN sets JX_DEVERR_NAN in the device error word (the reference panics).
 * out_val may be NULL. */
JX_API int jx_argreduce_rows_f32(const float *x, int32_t *out_idx, float *out_val, int64_t rows, int64_t cols,
                          int is_max, jx_stream_t stream);
/* VJPs (transpose_sum_axis src/trace/transpose_rules.rs:409-418; transpose_max_all
 * :444-469 applied per row): dx[r,c] = ct[r]; dx[r,c] = ct[r]*(x==max)/(count>1?count:1). */
JX_API int jx_sum_rows_vjp_f32(const float *ct, float *dx, int64_t rows, int64_t cols, jx_stream_t stream);
JX_API int jx_max_rows_vjp_f32(const float *x, const float *ct, float *dx, int64_t rows, int64_t cols,
                        jx_stream_t stream);

/* ---- FFT (gpu_fft_complex src/backend/ops.rs:1736-1741; fft_recursive
 *      src/ops/fft.rs:40-70; ifft :146-191; fft2/ifft2 :261-396) ----------- */
/* Batched complex-to-complex FFT, interleaved [re,im] f32, n a power of two.
 * inverse != 0 applies the 1/n scale as ifft does.  in may equal out. */
JX_API int jx_fft_c2c_f32(const float *in, float *out, int64_t n, int64_t batch, int inverse, jx_stream_t stream);
/* Batched 2-D transform of [batch, h, w] complex images: rows, then columns. */
JX_API int jx_fft2_c2c_f32(const float *in, float *out, int64_t h, int64_t w, int64_t batch, int inverse,
                    jx_stream_t stream);
/* jx_fft_c2c_f32 / jx_fft2_c2c_f32 over host buffers (pinned for overlap):
 * blocks of block_items transforms or images (0: about 32 MiB) stream through
 * the device, uploads, transforms and downloads overlapping on three
 * streams; the caller's stream waits for the last download. */
JX_API int jx_fft_c2c_f32_host(const float *in, float *out, int64_t n, int64_t batch, int inverse,
                               int64_t block_items, jx_stream_t stream);
JX_API int jx_fft2_c2c_f32_host(const float *in, float *out, int64_t h, int64_t w, int64_t batch, int inverse,
                                int64_t block_items, jx_stream_t stream);
/* Real input / real output (ops::fft::fft with real input :91-126, rfft
 * :212-234, irfft :417-462, rfftn / irfftn in 2-D :474-628).  in [batch][n]
 * real -> out [batch][bins] interleaved complex, bins = full ? n : n/2+1
 * (full = 1 is fft's whole spectrum, 0 is rfft's).  n >= 2, a power of two,
 * up to 16384. */
JX_API int jx_fft_r2c_f32(const float *in, float *out, int64_t n, int64_t batch, int full, jx_stream_t stream);
/* irfft: in [batch][n/2+1] complex -> out [batch][n] real, scaled 1/n; the
 * imaginary parts of the DC and Nyquist bins do not affect the result. */
JX_API int jx_fft_c2r_f32(const float *in, float *out, int64_t n, int64_t batch, jx_stream_t stream);
/* rfftn / irfftn of [batch][h][w] real <-> [batch][h][w/2+1] complex. */
JX_API int jx_rfft2_f32(const float *in, float *out, int64_t h, int64_t w, int64_t batch, jx_stream_t stream);
JX_API int jx_irfft2_f32(const float *in, float *out, int64_t h, int64_t w, int64_t batch, jx_stream_t stream);

/* ---- conv2d (gpu_conv2d src/backend/ops.rs:815-828; nn::conv2d_batched
 *      src/nn.rs:2048-2144), NCHW input, OIHW weight --------------------- */
JX_API int jx_conv2d_fwd_f32(const float *x, const float *w, float *y, int64_t B, int64_t C, int64_t H, int64_t W,
                      int64_t O, int64_t KH, int64_t KW, int64_t stride, int64_t pad, jx_stream_t stream);
JX_API int jx_conv2d_bwd_data_f32(const float *dy, const float *w, float *dx, int64_t B, int64_t C, int64_t H,
                           int64_t W, int64_t O, int64_t KH, int64_t KW, int64_t stride, int64_t pad,
                           jx_stream_t stream);
JX_API int jx_conv2d_bwd_filter_f32(const float *x, const float *dy, float *dw, int64_t B, int64_t C, int64_t H,
                             int64_t W, int64_t O, int64_t KH, int64_t KW, int64_t stride, int64_t pad,
                             jx_stream_t stream);
/* Kernel of the implicit convolutions above (no reference counterpart; for
 * tests and tuning), process-wide.  JX_CONV_AUTO: the SM-pair kernel
 * (tcgen05 cta_group::2, 256x256 tiles) when the pass's tiles fill at least
 * 90% of the SM pairs, else the one-CTA kernel (128x256 tiles).  The two compute the
 * same sums in the same order.  Shapes beyond the implicit kernels (more
 * than 4096 gathered indices or 32 filter taps) take the explicit path
 * whatever the setting.  Returns JX_EINVAL for another value. */
#define JX_CONV_AUTO 0
#define JX_CONV_ONE_CTA 1
#define JX_CONV_PAIR 2
JX_API int jx_conv_set_kernel(int which);

/* ---- layers: conv1d, pooling, normalisation ------------------------------- */
/* gpu_conv1d (src/backend/ops.rs:1014-1025; shader src/backend/shaders.rs:449-519),
 * nn::conv1d (src/nn.rs:1662-1722: batch = channels = 1, stride 1, padding 0).
 * x [batch, in_channels, input_len], w [out_channels, in_channels, kernel_len]
 * -> y [batch, out_channels, (input_len + 2 padding - kernel_len) / stride + 1].
 * Per output: sum over in-channel, then tap, padded taps skipped, unfused f32:
 * bit-identical to the reference's loop.  "Kernel size must be <= input size"
 * (JX_EINVAL) when kernel_len > input_len + 2 padding. */
JX_API int jx_conv1d_f32(const float *x, const float *w, float *y, int64_t batch, int64_t in_channels,
                         int64_t out_channels, int64_t input_len, int64_t kernel_len, int64_t stride,
                         int64_t padding, jx_stream_t stream);
#define JX_POOL_MAX 0
#define JX_POOL_AVG 1
/* Pooling of NCHW planes with a pool_h x pool_w window, per-axis stride and
 * padding.  Max folds from -inf with f32::max over the in-range taps; average
 * sums them in row-major order and divides by their count (0 if none):
 * nn::maxpool2d / avgpool2d (src/nn.rs:2164-2280), and with batch = 1 or
 * channels = 1 and no padding max_pool2d / avg_pool2d (:1121-1261) and, with
 * input_h = pool_h = 1, max_pool1d / avg_pool1d (:1002-1100).  Bit-identical. */
JX_API int jx_pool2d_f32(const float *x, float *y, int64_t batch, int64_t channels, int64_t input_h,
                         int64_t input_w, int64_t pool_h, int64_t pool_w, int64_t stride_h, int64_t stride_w,
                         int64_t pad_h, int64_t pad_w, int op, jx_stream_t stream);
/* jx_pool2d_f32 over host buffers: blocks of block_items images (0: about
 * 32 MiB of input) stream through the device, uploads, pooling and downloads
 * overlapping on three streams; the caller's stream waits for the last
 * download. */
JX_API int jx_pool2d_f32_host(const float *x, float *y, int64_t batch, int64_t channels, int64_t input_h,
                              int64_t input_w, int64_t pool_h, int64_t pool_w, int64_t stride_h, int64_t stride_w,
                              int64_t pad_h, int64_t pad_w, int op, int64_t block_items, jx_stream_t stream);
/* gpu_maxpool2d / gpu_avgpool2d (src/backend/ops.rs:1204-1215,1359-1370): one
 * stride and one padding for both axes. */
JX_API int jx_maxpool2d_f32(const float *x, float *y, int64_t batch, int64_t channels, int64_t input_h,
                            int64_t input_w, int64_t pool_h, int64_t pool_w, int64_t stride, int64_t padding,
                            jx_stream_t stream);
JX_API int jx_avgpool2d_f32(const float *x, float *y, int64_t batch, int64_t channels, int64_t input_h,
                            int64_t input_w, int64_t pool_h, int64_t pool_w, int64_t stride, int64_t padding,
                            jx_stream_t stream);
/* global_avg_pool2d / global_max_pool2d (src/nn.rs:2383-2455): [batch,
 * channels, height, width] -> [batch, channels].  Max is exact; the average
 * is a tree sum divided by height*width. */
JX_API int jx_global_pool2d_f32(const float *x, float *y, int64_t batch, int64_t channels, int64_t height,
                                int64_t width, int op, jx_stream_t stream);
/* gpu_batchnorm (src/backend/ops.rs:1516-1525) / nn::batch_norm_2d (src/nn.rs:
 * 2303-2360): x [batch, channels, spatial]; per channel, mean and variance
 * (biased) over batch*spatial, y = (x - mean) / sqrt(var + epsilon) * gamma +
 * beta.  gamma = beta = NULL drops the affine step: nn::batch_norm [batch,
 * features] (:656-699) is spatial = 1, nn::layer_norm (:712-725) is batch =
 * channels = 1.  mean_out / var_out (may be NULL) receive the statistics. */
JX_API int jx_batchnorm_f32(const float *x, const float *gamma, const float *beta, float *y, int64_t batch,
                            int64_t channels, int64_t spatial, float epsilon, float *mean_out, float *var_out,
                            jx_stream_t stream);

/* ---- nn / optim (src/nn.rs:155-221,300-318; src/optim.rs:138-189) -------- */
/* y[r,:] = softmax(x[r,:]) (src/nn.rs:155-168 applied per row). */
JX_API int jx_softmax_rows_f32(const float *x, float *y, int64_t rows, int64_t cols, jx_stream_t stream);
/* Fused softmax + cross_entropy_loss (src/nn.rs:300-318, eps 1e-7) forward and
 * backward.  labels are class indices stored as f32, as randint returns them,
 * with one_hot's semantics (src/nn.rs:205-221).  The loss is
 * -sum(t*ln(p+eps)) / count, where the reference's count is rows*cols; a
 * data-parallel caller passes the global element count so that summing the
 * ranks' gradients gives the gradient of the global loss.  Writes probs (may be
 * NULL), dlogits = dL/dlogits (may be NULL) and loss_out[0] (device scalar). */
JX_API int jx_softmax_xent_f32(const float *logits, const float *labels, float *probs, float *dlogits,
                               float *loss_out, int64_t rows, int64_t cols, int64_t count, jx_stream_t stream);
/* y[r,c] = act(y[r,c] + bias[c]); act: 0 none, 1 relu, 2 gelu (broadcast_to +
 * add src/ops/manipulation.rs:919-946, then src/nn.rs:22-26 / :111-122).
 * pre (may be NULL) receives the pre-activation. */
JX_API int jx_bias_act_f32(float *y, const float *bias, float *pre, int64_t rows, int64_t cols, int act,
                    jx_stream_t stream);
/* dz = dy * act'(pre) (act 1 relu, 2 gelu); db[c] = sum_r dz[r,c] (db may be NULL). */
JX_API int jx_act_bwd_f32(const float *dy, const float *pre, float *dz, float *db, int64_t rows, int64_t cols,
                   int act, jx_stream_t stream);
/* Column sums db[c] = sum_r dy[r,c] (bias gradient). */
JX_API int jx_col_sum_f32(const float *dy, float *db, int64_t rows, int64_t cols, jx_stream_t stream);
/* optim::adam_update (src/optim.rs:138-189) over `count` tensors in one launch,
 * in the reference's op order (bit-exact): step is the new step number (>=1);
 * step == 1 treats m and v as absent (state.m == None). */
JX_API int jx_adam_step_f32(float *const *params, const float *const *grads, float *const *m, float *const *v,
                     const int64_t *sizes, int count, float lr, float beta1, float beta2, float eps,
                     int64_t step, jx_stream_t stream);

/* ---- Dense-stack trainer (examples/mlp_training.rs:94-145 trains with finite
 *      differences + SGD; here: analytic backward, optim::adam_update
 *      src/optim.rs:138-189, Array::matmul + broadcast bias + nn activations) --
 * widths[0..n_layers]; acts[l] (0 none, 1 relu, 2 gelu) for hidden layers
 * l < n_layers-1; the last layer feeds fused softmax cross-entropy.  Params
 * are one flat f32 vector [W1, b1, W2, b2, ...], W row-major [in, out], each
 * block starting at the offsets jx_mlp_param_offsets reports. */
typedef struct jx_mlp jx_mlp;
JX_API int jx_mlp_create(const int64_t *widths, int n_layers, const int *acts, int64_t batch, int precision,
                         jx_mlp **out);
JX_API int jx_mlp_param_count(const jx_mlp *mlp, int64_t *count);
JX_API int jx_mlp_param_offsets(const jx_mlp *mlp, int64_t *w_off, int64_t *b_off);
JX_API int jx_mlp_set_params(jx_mlp *mlp, const float *host_params, int64_t count);
JX_API int jx_mlp_get_params(const jx_mlp *mlp, float *host_params, int64_t count);
/* Resets the optimiser state (adam_init) and sets its hyper-parameters. */
JX_API int jx_mlp_set_adam(jx_mlp *mlp, float lr, float beta1, float beta2, float eps);
/* Data parallel: gradients are summed over the communicator's ranks; the loss
 * is normalised by the global batch (global_batch = batch * world). */
JX_API int jx_mlp_attach_comm(jx_mlp *mlp, void *comm, int world, int64_t global_batch);
/* One step: forward, backward, (all-reduce), Adam.  x [batch, widths[0]] and
 * labels [batch] are device pointers; loss_out (device scalar) may be NULL. */
JX_API int jx_mlp_train_step(jx_mlp *mlp, const float *x, const float *labels, float *loss_out,
                             jx_stream_t stream);
/* With JX_PREC_EXACT and no communicator, a step runs as one cooperative
 * kernel (forward, loss, backward, Adam, grid barriers between phases; the
 * same arithmetic as the separate kernels, bit-identical).  enable = 0 selects
 * the captured graph of separate kernels instead.  On by default. */
JX_API int jx_mlp_set_fused(jx_mlp *mlp, int enable);
/* Phase timing of training steps (no reference counterpart: the reference has
 * no profiler, timestamp_writes: None at src/backend/ops.rs:139).  enable != 0
 * records CUDA events in every following step (which then runs as separate
 * launches, not a captured graph or the fused kernel); jx_mlp_step_times
 * waits for the last timed step and returns ms[0] forward (through the
 * softmax cross-entropy), ms[1] backward as enqueued on the caller's stream,
 * ms[2] the tail after it: the wait for outstanding gradient all-reduces and
 * Adam updates on the communication stream (with a communicator), else the
 * flat Adam update. */
JX_API int jx_mlp_set_timing(jx_mlp *mlp, int enable);
/* Data-parallel update form (no reference counterpart).  enable != 0 (the
 * default): each gradient bucket whose size divides by the rank count is
 * reduce-scattered, Adam updates this rank's 1/world of it, and the updated
 * parameters are all-gathered (ZeRO-1-style; each rank keeps Adam moments for
 * its own shards only).  enable = 0: all-reduce and Adam over every bucket on
 * every rank.  Call before the first step. */
JX_API int jx_mlp_set_dp_sharded(jx_mlp *mlp, int enable);
JX_API int jx_mlp_step_times(jx_mlp *mlp, float *ms);
/* Self-test of the bounded waits (no reference counterpart): a two-block
 * grid barrier waiting for one arrival more than the grid has.  Each block's
 * wait gives up after timeout_ms (1..5000), records JX_DEVERR_TIMEOUT in the
 * device error word and returns; *timed_out = 1 if the kernel reported it.
 * The context stays usable. */
JX_API int jx_selftest_barrier_timeout(int timeout_ms, int *timed_out);
/* Test hook (no reference counterpart): ORs flags into the current device's
 * jx_gemm_f32_noalloc error word, so a test can check that the word reaches
 * jx_device_status without making a wait run out. */
JX_API int jx_selftest_noalloc_flag(unsigned int flags);
JX_API int jx_mlp_destroy(jx_mlp *mlp);

/* ---- data-parallel collectives (no reference counterpart: the reference has
 *      a single global device, src/backend/webgpu.rs:6) -------------------- */
JX_API int jx_nccl_unique_id_size(void);
JX_API int jx_nccl_get_unique_id(void *id_out /* jx_nccl_unique_id_size() bytes */);
/* Non-blocking communicator init with a host watchdog of timeout_ms; a
 * timeout_ms <= 0 takes JAXRS_NCCL_TIMEOUT_MS from the environment, else
 * 120000. */
JX_API int jx_nccl_init(const void *id, int nranks, int rank, int timeout_ms, void **comm_out);
/* In-place sum all-reduce of count floats; polls for async errors up to timeout_ms. */
JX_API int jx_nccl_allreduce_sum_f32(void *comm, float *buf, int64_t count, jx_stream_t stream);
JX_API int jx_nccl_wait(void *comm, jx_stream_t stream, int timeout_ms);
JX_API int jx_nccl_destroy(void *comm);

#ifdef __cplusplus
}
#endif
#endif /* JAXRS_CUDA_H */
