// conv.cu -- conv2d forward, input gradient and weight gradient on the
// tcgen05 3xTF32 GEMM core.
//
// Replaces nn::conv2d_batched (src/nn.rs:2048-2144: NCHW input, OIHW weight,
// stride and zero padding, the CPU loop b -> oc -> oh -> ow -> ic -> kh -> kw)
// and gpu_conv2d (src/backend/ops.rs:815-998: one output per thread, no data
// reuse, forward only).  The reference has no conv backward; dX and dW here
// are the exact adjoints of its forward loop.
//
// With K = C*KH*KW and P = OH*OW (output pixels):
//   forward   Y_b[O, P]  = W[O, K] . Xcol_b[K, P]          (batch = images, W shared)
//   input     dXcol_b[K, P] = W^T[K, O] . dY_b[O, P], then col2im (gather)
//   weight    dW[O, K] = sum_b dY_b[O, P] . Xcol_b^T[P, K] (contraction over
//             B*P, split in S slices, partial results added in slice order)
// The GEMM takes K-major hi/lo operand pairs (see gemm.cu).  The producers
// below write those pairs directly from the NCHW tensors -- im2col and the
// tf32 split fused into one pass -- so no plain im2col matrix is ever stored.
#include <algorithm>

#include "jx_common.cuh"

namespace jx {
int gemm_presplit_err(const float* Ah, const float* Al, const float* Bh, const float* Bl, float* C, int M, int N,
                      int Kp, long long ldc, long long strideC, int batch, cudaStream_t st, unsigned int* err,
                      bool a_bcast, bool b_bcast);
int gemm_split_operand(const float* src, float* hi, float* lo, int rows, int K, int Kp, long long ld, long long sb,
                       int batch, bool transposed, cudaStream_t st);
long long gemm_kpad(long long K);
}  // namespace jx

namespace {

struct Geo {
  int C, H, W, O, KH, KW, S, P, OH, OW;
  __host__ __device__ int K() const { return C * KH * KW; }
  __host__ __device__ int NP() const { return OH * OW; }
};

// Forward B operand: rows (b, p) of Kp values, element k = (c, kh, kw) is
// x[b, c, oh*S + kh - P, ow*S + kw - P] (0 outside the image and for k >= K).
__global__ void im2col_rows_split(const float* __restrict__ x, float* __restrict__ hi, float* __restrict__ lo,
                                  long long rows, int Kp, const Geo g) {
  const int K = g.K(), kk = g.KH * g.KW, np = g.NP();
  for (long long r = blockIdx.x; r < rows; r += gridDim.x) {
    const long long b = r / np;
    const int p = (int)(r - b * np);
    const int oh = p / g.OW, ow = p - (p / g.OW) * g.OW;
    const float* xb = x + b * g.C * g.H * g.W;
    float* hr = hi + r * Kp;
    float* lr = lo + r * Kp;
    for (int k = threadIdx.x; k < Kp; k += blockDim.x) {
      float v = 0.0f;
      if (k < K) {
        const int c = k / kk, rem = k - (k / kk) * kk;
        const int kh = rem / g.KW, kw = rem - (rem / g.KW) * g.KW;
        const int ih = oh * g.S + kh - g.P, iw = ow * g.S + kw - g.P;
        if (ih >= 0 && ih < g.H && iw >= 0 && iw < g.W) v = __ldg(xb + ((long long)c * g.H + ih) * g.W + iw);
      }
      float h, l;
      jxd::split_tf32(v, h, l);
      hr[k] = h;
      lr[k] = l;
    }
  }
}

// Weight-gradient B operand: for slice s, row k holds x at q = s*Ks + j for
// j < Ksp (q = b*P + p over all images and output pixels; 0 past the end).
__global__ void im2col_cols_split(const float* __restrict__ x, float* __restrict__ hi, float* __restrict__ lo,
                                  long long Q, long long Ks, int Ksp, int S_slices, const Geo g) {
  const int K = g.K(), kk = g.KH * g.KW, np = g.NP();
  const long long rows = (long long)S_slices * K;
  for (long long r = blockIdx.x; r < rows; r += gridDim.x) {
    const int s = (int)(r / K);
    const int k = (int)(r - (long long)s * K);
    const int c = k / kk, rem = k - (k / kk) * kk;
    const int kh = rem / g.KW, kw = rem - (rem / g.KW) * g.KW;
    float* hr = hi + r * Ksp;
    float* lr = lo + r * Ksp;
    for (int j = threadIdx.x; j < Ksp; j += blockDim.x) {
      const long long q = (long long)s * Ks + j;
      float v = 0.0f;
      if (j < Ks && q < Q) {
        const long long b = q / np;
        const int p = (int)(q - b * np);
        const int oh = p / g.OW, ow = p - (p / g.OW) * g.OW;
        const int ih = oh * g.S + kh - g.P, iw = ow * g.S + kw - g.P;
        if (ih >= 0 && ih < g.H && iw >= 0 && iw < g.W)
          v = __ldg(x + ((b * g.C + c) * g.H + ih) * (long long)g.W + iw);
      }
      float h, l;
      jxd::split_tf32(v, h, l);
      hr[j] = h;
      lr[j] = l;
    }
  }
}

// Weight-gradient A operand: for slice s, row o holds dY[b, o, p] at q = b*P + p.
__global__ void dy_rows_split(const float* __restrict__ dy, float* __restrict__ hi, float* __restrict__ lo,
                              long long Q, long long Ks, int Ksp, int S_slices, const Geo g) {
  const int np = g.NP();
  const long long rows = (long long)S_slices * g.O;
  for (long long r = blockIdx.x; r < rows; r += gridDim.x) {
    const int s = (int)(r / g.O);
    const int o = (int)(r - (long long)s * g.O);
    float* hr = hi + r * Ksp;
    float* lr = lo + r * Ksp;
    for (int j = threadIdx.x; j < Ksp; j += blockDim.x) {
      const long long q = (long long)s * Ks + j;
      float v = 0.0f;
      if (j < Ks && q < Q) {
        const long long b = q / np;
        const int p = (int)(q - b * np);
        v = __ldg(dy + (b * g.O + o) * (long long)np + p);
      }
      float h, l;
      jxd::split_tf32(v, h, l);
      hr[j] = h;
      lr[j] = l;
    }
  }
}

// dx[b, c, ih, iw] = sum over (kh, kw) with oh*S = ih + P - kh and
// ow*S = iw + P - kw in range of dcol[b, (c, kh, kw), (oh, ow)].
__global__ void col2im_gather(const float* __restrict__ dcol, float* __restrict__ dx, long long nb, const Geo g) {
  const long long total = nb * g.C * g.H * g.W;
  const int K = g.K(), np = g.NP();
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int iw = (int)(i % g.W);
    const int ih = (int)((i / g.W) % g.H);
    const int c = (int)((i / ((long long)g.W * g.H)) % g.C);
    const long long b = i / ((long long)g.W * g.H * g.C);
    const float* db = dcol + b * (long long)K * np;
    float acc = 0.0f;
    for (int kh = 0; kh < g.KH; ++kh) {
      const int th = ih + g.P - kh;
      if (th < 0 || th % g.S) continue;
      const int oh = th / g.S;
      if (oh >= g.OH) continue;
      for (int kw = 0; kw < g.KW; ++kw) {
        const int tw = iw + g.P - kw;
        if (tw < 0 || tw % g.S) continue;
        const int ow = tw / g.S;
        if (ow >= g.OW) continue;
        acc += db[((long long)(c * g.KH + kh) * g.KW + kw) * np + oh * g.OW + ow];
      }
    }
    dx[i] = acc;
  }
}

// out[i] = sum over s of part[s * n + i], in slice order.
__global__ void slice_sum(const float* __restrict__ part, float* __restrict__ out, long long n, int slices) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    float acc = 0.0f;
    for (int s = 0; s < slices; ++s) acc += part[(long long)s * n + i];
    out[i] = acc;
  }
}

int blocks_for(long long work, int cap_per_sm) {
  long long b = work;
  const long long cap = (long long)jx::num_sms() * cap_per_sm;
  if (b > cap) b = cap;
  return b < 1 ? 1 : (int)b;
}

int check_geo(long long B, long long C, long long H, long long W, long long O, long long KH, long long KW,
              long long stride, long long pad, Geo* g) {
  JX_REQUIRE(B >= 0 && C >= 1 && H >= 1 && W >= 1 && O >= 1 && KH >= 1 && KW >= 1, "conv2d: bad shape");
  JX_REQUIRE(stride > 0, "Stride must be positive");
  JX_REQUIRE(pad >= 0, "conv2d: negative padding");
  JX_REQUIRE(KH <= H + 2 * pad, "Kernel height too large");
  JX_REQUIRE(KW <= W + 2 * pad, "Kernel width too large");
  const long long OH = (H + 2 * pad - KH) / stride + 1, OW = (W + 2 * pad - KW) / stride + 1;
  JX_REQUIRE(C * KH * KW < (1LL << 30) && OH * OW < (1LL << 30) && O < (1LL << 30) && H * W < (1LL << 30),
             "conv2d: dimensions too large");
  *g = Geo{(int)C, (int)H, (int)W, (int)O, (int)KH, (int)KW, (int)stride, (int)pad, (int)OH, (int)OW};
  return JX_OK;
}

// Images per pass so one pass's operand workspace stays under ~4 GiB.
long long images_per_pass(long long B, long long per_image_floats) {
  const long long budget = (4LL << 30) / 4;
  long long nb = per_image_floats > 0 ? budget / per_image_floats : B;
  if (nb < 1) nb = 1;
  return nb < B ? nb : B;
}

}  // namespace

extern "C" {

int jx_conv2d_fwd_f32(const float* x, const float* w, float* y, int64_t B, int64_t C, int64_t H, int64_t W, int64_t O,
                      int64_t KH, int64_t KW, int64_t stride, int64_t pad, jx_stream_t stream) {
  Geo g;
  int rc = check_geo(B, C, H, W, O, KH, KW, stride, pad, &g);
  if (rc) return rc;
  if (B == 0) return JX_OK;
  JX_REQUIRE(x && w && y, "conv2d: NULL pointer");
  cudaStream_t st = jx::as_stream(stream);
  const long long K = g.K(), Kp = jx::gemm_kpad(K), NP = g.NP();
  const long long nb = images_per_pass(B, 2 * NP * Kp);
  void* ws = nullptr;
  if ((rc = jx::scratch_get(sizeof(float) * (size_t)(2 * O * Kp + 2 * nb * NP * Kp), &ws, st))) return rc;
  float* Wh = reinterpret_cast<float*>(ws);
  float* Wl = Wh + O * Kp;
  float* Xh = Wl + O * Kp;
  float* Xl = Xh + nb * NP * Kp;
  rc = jx::gemm_split_operand(w, Wh, Wl, (int)O, (int)K, (int)Kp, K, 0, 1, false, st);
  for (long long b0 = 0; !rc && b0 < B; b0 += nb) {
    const long long n = std::min(nb, B - b0);
    im2col_rows_split<<<blocks_for(n * NP, 16), 256, 0, st>>>(x + b0 * C * H * W, Xh, Xl, n * NP, (int)Kp, g);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) rc = jx::check_cuda(e, "im2col_rows_split");
    // Y_b[O, NP] = W . Xcol_b for each image of the pass
    if (!rc)
      rc = jx::gemm_presplit_err(Wh, Wl, Xh, Xl, y + b0 * O * NP, (int)O, (int)NP, (int)Kp, NP, O * NP, (int)n, st,
                                 jx::device_error_word(), true, false);
  }
  const int rc2 = jx::scratch_release(ws, st);
  return rc ? rc : rc2;
}

int jx_conv2d_bwd_data_f32(const float* dy, const float* w, float* dx, int64_t B, int64_t C, int64_t H, int64_t W,
                           int64_t O, int64_t KH, int64_t KW, int64_t stride, int64_t pad, jx_stream_t stream) {
  Geo g;
  int rc = check_geo(B, C, H, W, O, KH, KW, stride, pad, &g);
  if (rc) return rc;
  if (B == 0) return JX_OK;
  JX_REQUIRE(dy && w && dx, "conv2d: NULL pointer");
  cudaStream_t st = jx::as_stream(stream);
  const long long K = g.K(), Op = jx::gemm_kpad(O), NP = g.NP();
  const long long nb = images_per_pass(B, 2 * NP * Op + K * NP);
  void* ws = nullptr;
  if ((rc = jx::scratch_get(sizeof(float) * (size_t)(2 * K * Op + nb * (2 * NP * Op + K * NP)), &ws, st))) return rc;
  float* Ah = reinterpret_cast<float*>(ws);  // W^T split: rows k, contraction over o
  float* Al = Ah + K * Op;
  float* Bh = Al + K * Op;  // dY_b^T split: rows p, contraction over o
  float* Bl = Bh + nb * NP * Op;
  float* dcol = Bl + nb * NP * Op;
  rc = jx::gemm_split_operand(w, Ah, Al, (int)K, (int)O, (int)Op, K, 0, 1, true, st);
  for (long long b0 = 0; !rc && b0 < B; b0 += nb) {
    const long long n = std::min(nb, B - b0);
    rc = jx::gemm_split_operand(dy + b0 * O * NP, Bh, Bl, (int)NP, (int)O, (int)Op, NP, O * NP, (int)n, true, st);
    if (!rc)
      rc = jx::gemm_presplit_err(Ah, Al, Bh, Bl, dcol, (int)K, (int)NP, (int)Op, NP, K * NP, (int)n, st,
                                 jx::device_error_word(), true, false);
    if (!rc) {
      col2im_gather<<<blocks_for((n * C * H * W + 255) / 256, 8), 256, 0, st>>>(dcol, dx + b0 * C * H * W, n, g);
      cudaError_t e = cudaGetLastError();
      if (e != cudaSuccess) rc = jx::check_cuda(e, "col2im_gather");
    }
  }
  const int rc2 = jx::scratch_release(ws, st);
  return rc ? rc : rc2;
}

int jx_conv2d_bwd_filter_f32(const float* x, const float* dy, float* dw, int64_t B, int64_t C, int64_t H, int64_t W,
                             int64_t O, int64_t KH, int64_t KW, int64_t stride, int64_t pad, jx_stream_t stream) {
  Geo g;
  int rc = check_geo(B, C, H, W, O, KH, KW, stride, pad, &g);
  if (rc) return rc;
  JX_REQUIRE(dw, "conv2d: NULL pointer");
  cudaStream_t st = jx::as_stream(stream);
  const long long K = g.K(), NP = g.NP();
  if (B == 0) {
    JX_CUDA(cudaMemsetAsync(dw, 0, sizeof(float) * O * K, st));
    return JX_OK;
  }
  JX_REQUIRE(x && dy, "conv2d: NULL pointer");
  const long long Q = B * NP;  // contraction length: every image's every output pixel
  // slices: enough output tiles to fill the GPU twice over, each slice >= 1024 long
  const long long tiles = ((O + 127) / 128) * ((K + 255) / 256);
  long long S = (2LL * jx::num_sms() + tiles - 1) / tiles;
  S = std::max(1LL, std::min(S, std::min(64LL, Q / 1024)));
  const long long Ks = (Q + S - 1) / S, Ksp = jx::gemm_kpad(Ks);
  void* ws = nullptr;
  const size_t floats = (size_t)(2 * S * O * Ksp + 2 * S * K * Ksp + (S > 1 ? S * O * K : 0));
  if ((rc = jx::scratch_get(sizeof(float) * floats, &ws, st))) return rc;
  float* Ah = reinterpret_cast<float*>(ws);
  float* Al = Ah + S * O * Ksp;
  float* Bh = Al + S * O * Ksp;
  float* Bl = Bh + S * K * Ksp;
  float* part = S > 1 ? Bl + S * K * Ksp : dw;
  dy_rows_split<<<blocks_for(S * O, 16), 256, 0, st>>>(dy, Ah, Al, Q, Ks, (int)Ksp, (int)S, g);
  im2col_cols_split<<<blocks_for(S * K, 16), 256, 0, st>>>(x, Bh, Bl, Q, Ks, (int)Ksp, (int)S, g);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) rc = jx::check_cuda(e, "conv2d dW operand kernels");
  if (!rc)
    rc = jx::gemm_presplit_err(Ah, Al, Bh, Bl, part, (int)O, (int)K, (int)Ksp, K, O * K, (int)S, st,
                               jx::device_error_word(), false, false);
  if (!rc && S > 1) {
    slice_sum<<<blocks_for((O * K + 255) / 256, 8), 256, 0, st>>>(part, dw, O * K, (int)S);
    e = cudaGetLastError();
    if (e != cudaSuccess) rc = jx::check_cuda(e, "slice_sum");
  }
  const int rc2 = jx::scratch_release(ws, st);
  return rc ? rc : rc2;
}

}  // extern "C"
