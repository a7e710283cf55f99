// 2-D convolution forward, backward-data and backward-filter.
//
// Replaces dlprim::core::Conv2DForward / Conv2DBackwardData /
// Conv2DBackwardFilter / BiasBackwardFilter as called from
// src/vision_ops.cpp:61-186 (convolution_overrideable and
// convolution_backward_overrideable).
//
// Dispatch:
//   * depthwise (groups == C == K): direct shared-memory-free stencil kernels.
//   * otherwise, math == TF32 and the shape suits it: tcgen05 implicit GEMM
//     (conv_tc.cu).
//   * else: exact-fp32 SIMT implicit GEMM (igemm_simt.cuh) over NCHW.
// All layouts here are NCHW-contiguous; W is [K, C/g, R, S] contiguous.
#include "igemm_simt.cuh"

namespace pvb2 {

int conv_tc_fwd(const pvb2_conv2d_desc* d, const float* x, const float* w, const float* b, float* y, void* ws,
                size_t ws_bytes, cudaStream_t s, bool* handled, float* staged, bool* staged_written);
int conv_tc_bwd_data(const pvb2_conv2d_desc* d, const float* dy, const float* w, float* dx, void* ws,
                     size_t ws_bytes, cudaStream_t s, bool* handled, float* staged_dy, bool* staged_written);
int conv_tc_bwd_filter(const pvb2_conv2d_desc* d, const float* x, const float* dy, float* dw, void* ws,
                       size_t ws_bytes, cudaStream_t s, bool* handled, const float* staged,
                       const float* staged_dy);
size_t conv_tc_staged_grad_bytes(const pvb2_conv2d_desc* d);
size_t conv_tc_workspace(const pvb2_conv2d_desc* d, int which);
size_t conv_tc_staged_bytes(const pvb2_conv2d_desc* d);
bool conv_tc_path(const pvb2_conv2d_desc* d, int which);
size_t dw_wgrad_workspace(const pvb2_conv2d_desc* d);
int dw_fwd(const pvb2_conv2d_desc* d, const float* x, const float* w, const float* b, float* y, cudaStream_t s,
           bool* handled);
int dw_dgrad(const pvb2_conv2d_desc* d, const float* dy, const float* w, float* dx, cudaStream_t s, bool* handled);
int dw_wgrad(const pvb2_conv2d_desc* d, const float* x, const float* dy, float* dw, void* ws, size_t ws_bytes,
             cudaStream_t s, bool* handled);
bool conv_tc_bwd_data_acc_ok(const pvb2_conv2d_desc* d, const void* dy, const void* w, const void* dx,
                             const void* addend);
int conv_tc_bwd_data_acc(const pvb2_conv2d_desc* d, const float* dy, const float* w, float* dx, const float* addend,
                         cudaStream_t s);

struct ConvGeom {
  int N, C, H, W, K, R, S, P, Q, sh, sw, ph, pw, dh, dw, G, Cg, Kg;
};

static ConvGeom geom(const pvb2_conv2d_desc* d) {
  ConvGeom g;
  const int groups = d->groups > 0 ? d->groups : 1;
  g.N = d->N; g.C = d->C; g.H = d->H; g.W = d->W; g.K = d->K; g.R = d->R; g.S = d->S; g.P = d->P; g.Q = d->Q;
  g.sh = d->stride_h; g.sw = d->stride_w; g.ph = d->pad_h; g.pw = d->pad_w; g.dh = d->dil_h; g.dw = d->dil_w;
  g.G = groups; g.Cg = d->C / groups; g.Kg = d->K / groups;
  return g;
}

// ---------------------------------------------------------------- forward
// M = Kg (output channels of group z), N = N*P*Q, K = Cg*R*S
struct ConvFwdProb {
  int64_t M, N;
  int zcount;
  ConvGeom g;
  const float* x;
  const float* w;
  const float* bias;
  float* y;
  struct BCol {
    int64_t xbase;  // &x[nn, z*Cg, 0, 0] offset
    int h0, w0;     // p*sh - ph, q*sw - pw
    bool valid;
  };
  __device__ int64_t k_begin(int) const { return 0; }
  __device__ int64_t k_end(int) const { return (int64_t)g.Cg * g.R * g.S; }
  __device__ BCol bcol(int z, int64_t n) const {
    BCol c;
    c.valid = n < N;
    int64_t nn = 0;
    int p = 0, q = 0;
    if (c.valid) {
      q = (int)(n % g.Q);
      p = (int)((n / g.Q) % g.P);
      nn = n / ((int64_t)g.P * g.Q);
    }
    c.xbase = (nn * g.C + (int64_t)z * g.Cg) * g.H * g.W;
    c.h0 = p * g.sh - g.ph;
    c.w0 = q * g.sw - g.pw;
    return c;
  }
  __device__ float a(int z, int64_t m, int64_t k) const {
    return __ldg(w + ((int64_t)z * g.Kg + m) * ((int64_t)g.Cg * g.R * g.S) + k);
  }
  __device__ float b(int, const BCol& c, int64_t k) const {
    const int s = (int)(k % g.S);
    const int r = (int)((k / g.S) % g.R);
    const int64_t cc = k / ((int64_t)g.R * g.S);
    const int h = c.h0 + r * g.dh, ww = c.w0 + s * g.dw;
    if ((unsigned)h >= (unsigned)g.H || (unsigned)ww >= (unsigned)g.W) return 0.f;
    return __ldg(x + c.xbase + (cc * g.H + h) * g.W + ww);
  }
  __device__ void store(int z, int64_t m, int64_t n, float acc) const {
    const int64_t pq = (int64_t)g.P * g.Q;
    const int64_t nn = n / pq, rem = n % pq;
    const int64_t co = (int64_t)z * g.Kg + m;
    if (bias) acc += bias[co];
    y[(nn * g.K + co) * pq + rem] = acc;
  }
};

// ------------------------------------------------------------ backward data
// M = Cg (input channels of group z), N = N*H*W, K = Kg*R*S
struct ConvBwdDataProb {
  int64_t M, N;
  int zcount;
  ConvGeom g;
  const float* dy;
  const float* w;
  float* dx;
  struct BCol {
    int64_t ybase;  // &dy[nn, z*Kg, 0, 0]
    int hp, wp;     // h + ph, w + pw
  };
  __device__ int64_t k_begin(int) const { return 0; }
  __device__ int64_t k_end(int) const { return (int64_t)g.Kg * g.R * g.S; }
  __device__ BCol bcol(int z, int64_t n) const {
    BCol c;
    int64_t nn = 0;
    int h = 0, ww = 0;
    if (n < N) {
      ww = (int)(n % g.W);
      h = (int)((n / g.W) % g.H);
      nn = n / ((int64_t)g.H * g.W);
    }
    c.ybase = (nn * g.K + (int64_t)z * g.Kg) * g.P * g.Q;
    c.hp = h + g.ph;
    c.wp = ww + g.pw;
    return c;
  }
  __device__ float a(int z, int64_t m, int64_t k) const {
    // W[z*Kg + kk, m, r, s] with k = (kk, r, s)
    const int64_t rs = (int64_t)g.R * g.S;
    const int64_t kk = k / rs, t = k % rs;
    return __ldg(w + (((int64_t)z * g.Kg + kk) * g.Cg + m) * rs + t);
  }
  __device__ float b(int, const BCol& c, int64_t k) const {
    const int s = (int)(k % g.S);
    const int r = (int)((k / g.S) % g.R);
    const int64_t kk = k / ((int64_t)g.R * g.S);
    const int ht = c.hp - r * g.dh, wt = c.wp - s * g.dw;
    if (ht < 0 || wt < 0) return 0.f;
    if (ht % g.sh != 0 || wt % g.sw != 0) return 0.f;
    const int p = ht / g.sh, q = wt / g.sw;
    if (p >= g.P || q >= g.Q) return 0.f;
    return __ldg(dy + c.ybase + (kk * g.P + p) * g.Q + q);
  }
  __device__ void store(int z, int64_t m, int64_t n, float acc) const {
    const int64_t hw = (int64_t)g.H * g.W;
    const int64_t nn = n / hw, rem = n % hw;
    dx[(nn * g.C + (int64_t)z * g.Cg + m) * hw + rem] = acc;
  }
};

// ---------------------------------------------------------- backward filter
// M = Kg, N = Cg*R*S, K = N*P*Q split into `splits` ranges; z = g*splits + split.
// Partial sums go to ws[split][K][Cg*R*S], reduced afterwards.
struct ConvBwdFilterProb {
  int64_t M, N;
  int zcount;
  int splits;
  int64_t kchunk;
  ConvGeom g;
  const float* x;
  const float* dy;
  float* part;
  struct BCol {
    int64_t cc;
    int r, s;
  };
  __device__ int64_t k_begin(int z) const { return (int64_t)(z % splits) * kchunk; }
  __device__ int64_t k_end(int z) const {
    const int64_t total = (int64_t)g.N * g.P * g.Q;
    const int64_t e = (int64_t)(z % splits + 1) * kchunk;
    return e < total ? e : total;
  }
  __device__ BCol bcol(int, int64_t n) const {
    BCol c;
    c.s = (int)(n % g.S);
    c.r = (int)((n / g.S) % g.R);
    c.cc = n / ((int64_t)g.R * g.S);
    return c;
  }
  __device__ float a(int z, int64_t m, int64_t k) const {
    const int grp = z / splits;
    const int64_t pq = (int64_t)g.P * g.Q;
    const int64_t nn = k / pq, rem = k % pq;
    return __ldg(dy + (nn * g.K + (int64_t)grp * g.Kg + m) * pq + rem);
  }
  __device__ float b(int z, const BCol& c, int64_t k) const {
    const int grp = z / splits;
    const int q = (int)(k % g.Q);
    const int p = (int)((k / g.Q) % g.P);
    const int64_t nn = k / ((int64_t)g.P * g.Q);
    const int h = p * g.sh - g.ph + c.r * g.dh, ww = q * g.sw - g.pw + c.s * g.dw;
    if ((unsigned)h >= (unsigned)g.H || (unsigned)ww >= (unsigned)g.W) return 0.f;
    return __ldg(x + ((nn * g.C + (int64_t)grp * g.Cg + c.cc) * g.H + h) * g.W + ww);
  }
  __device__ void store(int z, int64_t m, int64_t n, float acc) const {
    const int grp = z / splits, sp = z % splits;
    part[((int64_t)sp * g.K + (int64_t)grp * g.Kg + m) * N + n] = acc;
  }
};

__global__ void reduce_splits_kernel(const float* __restrict__ part, int splits, int64_t n, float* __restrict__ out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int k = 0; k < splits; ++k) s += part[(int64_t)k * n + i];
    out[i] = s;
  }
}

// bias gradient: db[k] = sum over n, p, q of dy[n, k, p, q]; one CTA per channel
__global__ void conv_bias_grad_kernel(const float* __restrict__ dy, int N, int K, int64_t PQ, float* __restrict__ db) {
  __shared__ float sh[32];
  const int k = blockIdx.x;
  float s = 0.f;
  for (int n = 0; n < N; ++n) {
    const float* p = dy + ((int64_t)n * K + k) * PQ;
    for (int64_t i = threadIdx.x; i < PQ; i += blockDim.x) s += p[i];
  }
  for (int o = 16; o > 0; o >>= 1) s += __shfl_down_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    s = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0.f;
    for (int o = 16; o > 0; o >>= 1) s += __shfl_down_sync(0xffffffffu, s, o);
    if (threadIdx.x == 0) db[k] = s;
  }
}

// ------------------------------------------------------------- depthwise
// groups == C == K (channel multiplier 1): each output reads an R x S window
// of its own channel.  These direct kernels serve the filter sizes the
// shared-memory-staged stencils of depthwise.cu do not take (3x3, 5x5).
__global__ void dw_fwd_kernel(ConvGeom g, const float* __restrict__ x, const float* __restrict__ w,
                              const float* __restrict__ bias, float* __restrict__ y) {
  const int64_t total = (int64_t)g.N * g.K * g.P * g.Q;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int q = (int)(i % g.Q);
    const int p = (int)((i / g.Q) % g.P);
    const int64_t plane = i / ((int64_t)g.P * g.Q);
    const int c = (int)(plane % g.K);
    const float* xp = x + plane * g.H * g.W;
    const float* wp = w + (int64_t)c * g.R * g.S;
    float acc = bias ? bias[c] : 0.f;
    for (int r = 0; r < g.R; ++r) {
      const int h = p * g.sh - g.ph + r * g.dh;
      if ((unsigned)h >= (unsigned)g.H) continue;
      for (int s = 0; s < g.S; ++s) {
        const int ww = q * g.sw - g.pw + s * g.dw;
        if ((unsigned)ww >= (unsigned)g.W) continue;
        acc = fmaf(__ldg(xp + (int64_t)h * g.W + ww), __ldg(wp + r * g.S + s), acc);
      }
    }
    y[i] = acc;
  }
}

__global__ void dw_bwd_data_kernel(ConvGeom g, const float* __restrict__ dy, const float* __restrict__ w,
                                   float* __restrict__ dx) {
  const int64_t total = (int64_t)g.N * g.C * g.H * g.W;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int ww = (int)(i % g.W);
    const int h = (int)((i / g.W) % g.H);
    const int64_t plane = i / ((int64_t)g.H * g.W);
    const int c = (int)(plane % g.C);
    const float* gp = dy + plane * g.P * g.Q;
    const float* wp = w + (int64_t)c * g.R * g.S;
    float acc = 0.f;
    for (int r = 0; r < g.R; ++r) {
      const int ht = h + g.ph - r * g.dh;
      if (ht < 0 || ht % g.sh) continue;
      const int p = ht / g.sh;
      if (p >= g.P) continue;
      for (int s = 0; s < g.S; ++s) {
        const int wt = ww + g.pw - s * g.dw;
        if (wt < 0 || wt % g.sw) continue;
        const int q = wt / g.sw;
        if (q >= g.Q) continue;
        acc = fmaf(__ldg(gp + (int64_t)p * g.Q + q), __ldg(wp + r * g.S + s), acc);
      }
    }
    dx[i] = acc;
  }
}

// one CTA per (channel, tap): reduce over n, p, q
__global__ void dw_bwd_filter_kernel(ConvGeom g, const float* __restrict__ x, const float* __restrict__ dy,
                                     float* __restrict__ dw) {
  __shared__ float sh[32];
  const int c = blockIdx.x / (g.R * g.S);
  const int tap = blockIdx.x % (g.R * g.S);
  const int r = tap / g.S, s = tap % g.S;
  const int64_t pq = (int64_t)g.P * g.Q;
  float acc = 0.f;
  for (int n = 0; n < g.N; ++n) {
    const float* xp = x + ((int64_t)n * g.C + c) * g.H * g.W;
    const float* gp = dy + ((int64_t)n * g.K + c) * pq;
    for (int64_t i = threadIdx.x; i < pq; i += blockDim.x) {
      const int q = (int)(i % g.Q), p = (int)(i / g.Q);
      const int h = p * g.sh - g.ph + r * g.dh, ww = q * g.sw - g.pw + s * g.dw;
      if ((unsigned)h < (unsigned)g.H && (unsigned)ww < (unsigned)g.W) acc = fmaf(gp[i], xp[(int64_t)h * g.W + ww], acc);
    }
  }
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_down_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    acc = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0.f;
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_down_sync(0xffffffffu, acc, o);
    if (threadIdx.x == 0) dw[(int64_t)c * g.R * g.S + tap] = acc;
  }
}

static bool is_depthwise(const ConvGeom& g) { return g.G > 1 && g.G == g.C && g.G == g.K; }

static int wgrad_splits(const ConvGeom& g) {
  const int64_t kdim = (int64_t)g.N * g.P * g.Q;
  const int64_t tiles = (int64_t)((g.Kg + 63) / 64) * (((int64_t)g.Cg * g.R * g.S + 63) / 64) * g.G;
  if (tiles <= 0) return 1;
  int64_t want = ((int64_t)num_sms() * 2 + tiles - 1) / tiles;
  int64_t max_by_k = (kdim + 255) / 256;
  if (want > max_by_k) want = max_by_k;
  if (want > 64) want = 64;
  if (want < 1) want = 1;
  return (int)want;
}

static int check_desc(const pvb2_conv2d_desc* d) {
  if (d->math != PVB2_MATH_TF32 && d->math != PVB2_MATH_FP32)
    return fail(PVB2_ERR_UNSUPPORTED, "conv2d: math mode %d is not implemented (0 = TF32, 1 = exact fp32)", d->math);
  PVB2_CHECK_ARG(d->groups >= 1 && d->C % d->groups == 0 && d->K % d->groups == 0,
                 "conv2d: channels must divide groups");
  PVB2_CHECK_ARG(d->stride_h > 0 && d->stride_w > 0 && d->dil_h > 0 && d->dil_w > 0,
                 "conv2d: stride and dilation must be positive");
  PVB2_CHECK_ARG(d->P == (d->H + 2 * d->pad_h - d->dil_h * (d->R - 1) - 1) / d->stride_h + 1 &&
                     d->Q == (d->W + 2 * d->pad_w - d->dil_w * (d->S - 1) - 1) / d->stride_w + 1,
                 "conv2d: output size inconsistent with the descriptor");
  return PVB2_OK;
}

static int check_t(const pvb2_tensor* t, int64_t n, int64_t c, int64_t h, int64_t w, const char* what) {
  PVB2_CHECK_ARG(t->dtype == PVB2_F32 && t->ndim == 4, "conv2d: %s must be a 4-D float32 tensor", what);
  PVB2_CHECK_ARG(t->sizes[0] == n && t->sizes[1] == c && t->sizes[2] == h && t->sizes[3] == w,
                 "conv2d: %s shape mismatch", what);
  PVB2_CHECK_ARG(is_contiguous(t), "conv2d: %s must be NCHW-contiguous", what);
  return PVB2_OK;
}

}  // namespace pvb2

using namespace pvb2;

extern "C" {

size_t pvb2_conv2d_workspace_size(const pvb2_conv2d_desc* d, int which) {
  ConvGeom g = geom(d);
  size_t need = 0;
  if (which == 2 && !is_depthwise(g)) {
    need = (size_t)wgrad_splits(g) * g.K * ((size_t)g.Cg * g.R * g.S) * sizeof(float);
  }
  if (which == 2 && is_depthwise(g)) need = dw_wgrad_workspace(d);
  size_t tc = conv_tc_workspace(d, which);
  return need > tc ? need : tc;
}

int pvb2_conv2d_path(const pvb2_conv2d_desc* d, int which) {
  if (check_desc(d) != PVB2_OK || which < 0 || which > 2) return -1;
  if (is_depthwise(geom(d))) return 0;
  return conv_tc_path(d, which) ? 1 : 0;
}

size_t pvb2_conv2d_staged_input_bytes(const pvb2_conv2d_desc* d) {
  if (check_desc(d) != PVB2_OK || d->math != PVB2_MATH_TF32 || is_depthwise(geom(d))) return 0;
  return conv_tc_staged_bytes(d);
}

size_t pvb2_conv2d_staged_grad_bytes(const pvb2_conv2d_desc* d) {
  if (check_desc(d) != PVB2_OK || d->math != PVB2_MATH_TF32 || is_depthwise(geom(d))) return 0;
  return conv_tc_staged_grad_bytes(d);
}

int pvb2_conv2d_fwd(const pvb2_conv2d_desc* d, const pvb2_tensor* x, const float* w, const float* b,
                    const pvb2_tensor* y, void* workspace, size_t workspace_bytes, pvb2_stream stream) {
  return pvb2_conv2d_fwd_staged(d, x, w, b, y, workspace, workspace_bytes, nullptr, 0, nullptr, stream);
}

int pvb2_conv2d_fwd_staged(const pvb2_conv2d_desc* d, const pvb2_tensor* x, const float* w, const float* b,
                           const pvb2_tensor* y, void* workspace, size_t workspace_bytes, float* staged,
                           size_t staged_bytes, int* staged_written, pvb2_stream stream) {
  if (staged_written) *staged_written = 0;
  PVB2_TRY(check_desc(d));
  PVB2_TRY(check_t(x, d->N, d->C, d->H, d->W, "input"));
  PVB2_TRY(check_t(y, d->N, d->K, d->P, d->Q, "output"));
  ConvGeom g = geom(d);
  cudaStream_t s = as_stream(stream);
  if ((int64_t)g.N * g.K * g.P * g.Q == 0) return PVB2_OK;
  if (is_depthwise(g)) {
    PVB2_CHECK_ARG(is_contiguous(x) && is_contiguous(y), "conv2d: depthwise tensors must be contiguous NCHW");
    bool handled = false;
    PVB2_TRY(dw_fwd(d, (const float*)x->data, w, b, (float*)y->data, s, &handled));
    if (handled) return PVB2_OK;
    const int64_t total = (int64_t)g.N * g.K * g.P * g.Q;
    dw_fwd_kernel<<<grid_for(total, 256), 256, 0, s>>>(g, (const float*)x->data, w, b, (float*)y->data);
    PVB2_LAUNCH_CHECK();
    return PVB2_OK;
  }
  if (d->math == PVB2_MATH_TF32) {
    bool handled = false, written = false;
    if (staged) {
      PVB2_CHECK_ARG(staged_bytes >= conv_tc_staged_bytes(d) && ((uintptr_t)staged & 15) == 0,
                     "conv2d_fwd_staged: staged buffer too small or not 16-byte aligned");
    }
    PVB2_TRY(conv_tc_fwd(d, (const float*)x->data, w, b, (float*)y->data, workspace, workspace_bytes, s, &handled,
                         staged && conv_tc_staged_bytes(d) > 0 ? staged : nullptr, &written));
    if (staged_written) *staged_written = written ? 1 : 0;
    if (handled) return PVB2_OK;
  }
  ConvFwdProb pb;
  pb.M = g.Kg;
  pb.N = (int64_t)g.N * g.P * g.Q;
  pb.zcount = g.G;
  pb.g = g;
  pb.x = (const float*)x->data;
  pb.w = w;
  pb.bias = b;
  pb.y = (float*)y->data;
  return launch_igemm_simt(pb, s);
}

int pvb2_conv2d_bwd_data(const pvb2_conv2d_desc* d, const pvb2_tensor* dy, const float* w, const pvb2_tensor* dx,
                         void* workspace, size_t workspace_bytes, pvb2_stream stream) {
  return pvb2_conv2d_bwd_data_staged(d, dy, w, dx, workspace, workspace_bytes, nullptr, 0, nullptr, stream);
}

int pvb2_conv2d_bwd_data_staged(const pvb2_conv2d_desc* d, const pvb2_tensor* dy, const float* w,
                                const pvb2_tensor* dx, void* workspace, size_t workspace_bytes, float* staged_dy,
                                size_t staged_dy_bytes, int* staged_written, pvb2_stream stream) {
  if (staged_written) *staged_written = 0;
  PVB2_TRY(check_desc(d));
  PVB2_TRY(check_t(dy, d->N, d->K, d->P, d->Q, "grad_output"));
  PVB2_TRY(check_t(dx, d->N, d->C, d->H, d->W, "grad_input"));
  ConvGeom g = geom(d);
  cudaStream_t s = as_stream(stream);
  if ((int64_t)g.N * g.C * g.H * g.W == 0) return PVB2_OK;
  if (is_depthwise(g)) {
    PVB2_CHECK_ARG(is_contiguous(dy) && is_contiguous(dx), "conv2d: depthwise tensors must be contiguous NCHW");
    bool handled = false;
    PVB2_TRY(dw_dgrad(d, (const float*)dy->data, w, (float*)dx->data, s, &handled));
    if (handled) return PVB2_OK;
    const int64_t total = (int64_t)g.N * g.C * g.H * g.W;
    dw_bwd_data_kernel<<<grid_for(total, 256), 256, 0, s>>>(g, (const float*)dy->data, w, (float*)dx->data);
    PVB2_LAUNCH_CHECK();
    return PVB2_OK;
  }
  if (d->math == PVB2_MATH_TF32) {
    bool handled = false, written = false;
    if (staged_dy) {
      PVB2_CHECK_ARG(staged_dy_bytes >= conv_tc_staged_grad_bytes(d) && ((uintptr_t)staged_dy & 15) == 0,
                     "conv2d_bwd_data_staged: staged buffer too small or not 16-byte aligned");
    }
    PVB2_TRY(conv_tc_bwd_data(d, (const float*)dy->data, w, (float*)dx->data, workspace, workspace_bytes, s,
                              &handled, staged_dy, &written));
    if (staged_written) *staged_written = written ? 1 : 0;
    if (handled) return PVB2_OK;
  }
  ConvBwdDataProb pb;
  pb.M = g.Cg;
  pb.N = (int64_t)g.N * g.H * g.W;
  pb.zcount = g.G;
  pb.g = g;
  pb.dy = (const float*)dy->data;
  pb.w = w;
  pb.dx = (float*)dx->data;
  return launch_igemm_simt(pb, s);
}

int pvb2_conv2d_bwd_data_acc_ok(const pvb2_conv2d_desc* d, const void* dy, const float* w, const void* dx,
                                 const void* addend) {
  if (check_desc(d) != PVB2_OK || is_depthwise(geom(d))) return 0;
  return conv_tc_bwd_data_acc_ok(d, dy, w, dx, addend) ? 1 : 0;
}

int pvb2_conv2d_bwd_data_acc(const pvb2_conv2d_desc* d, const pvb2_tensor* dy, const float* w, const pvb2_tensor* dx,
                             const pvb2_tensor* addend, pvb2_stream stream) {
  PVB2_TRY(check_desc(d));
  PVB2_TRY(check_t(dy, d->N, d->K, d->P, d->Q, "grad_output"));
  PVB2_TRY(check_t(dx, d->N, d->C, d->H, d->W, "grad_input"));
  PVB2_TRY(check_t(addend, d->N, d->C, d->H, d->W, "addend"));
  if (!pvb2_conv2d_bwd_data_acc_ok(d, dy->data, w, dx->data, addend->data))
    return fail(PVB2_ERR_UNSUPPORTED, "conv2d_bwd_data_acc: not a tensor-core 1x1 stride-1 convolution");
  if ((int64_t)d->N * d->C * d->H * d->W == 0) return PVB2_OK;
  return conv_tc_bwd_data_acc(d, (const float*)dy->data, w, (float*)dx->data, (const float*)addend->data,
                              as_stream(stream));
}

int pvb2_conv2d_bwd_filter(const pvb2_conv2d_desc* d, const pvb2_tensor* x, const pvb2_tensor* dy, float* dw,
                           float* db, void* workspace, size_t workspace_bytes, pvb2_stream stream) {
  return pvb2_conv2d_bwd_filter_staged(d, x, dy, dw, db, workspace, workspace_bytes, nullptr, 0, stream);
}

int pvb2_conv2d_bwd_filter_staged(const pvb2_conv2d_desc* d, const pvb2_tensor* x, const pvb2_tensor* dy,
                                  float* dw, float* db, void* workspace, size_t workspace_bytes,
                                  const float* staged, size_t staged_bytes, pvb2_stream stream) {
  return pvb2_conv2d_bwd_filter_staged_grad(d, x, dy, dw, db, workspace, workspace_bytes, staged, staged_bytes,
                                            nullptr, 0, stream);
}

int pvb2_conv2d_bwd_filter_staged_grad(const pvb2_conv2d_desc* d, const pvb2_tensor* x, const pvb2_tensor* dy,
                                       float* dw, float* db, void* workspace, size_t workspace_bytes,
                                       const float* staged, size_t staged_bytes, const float* staged_dy,
                                       size_t staged_dy_bytes, pvb2_stream stream) {
  PVB2_TRY(check_desc(d));
  PVB2_TRY(check_t(x, d->N, d->C, d->H, d->W, "input"));
  PVB2_TRY(check_t(dy, d->N, d->K, d->P, d->Q, "grad_output"));
  ConvGeom g = geom(d);
  cudaStream_t s = as_stream(stream);
  const int64_t wnum = (int64_t)g.K * g.Cg * g.R * g.S;
  if (db) {
    if ((int64_t)g.N * g.P * g.Q == 0) {
      PVB2_CUDA_TRY(cudaMemsetAsync(db, 0, g.K * sizeof(float), s));
    } else {
      conv_bias_grad_kernel<<<g.K, 256, 0, s>>>((const float*)dy->data, g.N, g.K, (int64_t)g.P * g.Q, db);
      PVB2_LAUNCH_CHECK();
    }
  }
  if (!dw) return PVB2_OK;
  if ((int64_t)g.N * g.P * g.Q == 0) {
    PVB2_CUDA_TRY(cudaMemsetAsync(dw, 0, wnum * sizeof(float), s));
    return PVB2_OK;
  }
  if (is_depthwise(g)) {
    PVB2_CHECK_ARG(is_contiguous(x) && is_contiguous(dy), "conv2d: depthwise tensors must be contiguous NCHW");
    bool handled = false;
    PVB2_TRY(dw_wgrad(d, (const float*)x->data, (const float*)dy->data, dw, workspace, workspace_bytes, s, &handled));
    if (handled) return PVB2_OK;
    dw_bwd_filter_kernel<<<g.C * g.R * g.S, 256, 0, s>>>(g, (const float*)x->data, (const float*)dy->data, dw);
    PVB2_LAUNCH_CHECK();
    return PVB2_OK;
  }
  if (d->math == PVB2_MATH_TF32) {
    bool handled = false;
    if (staged) {
      PVB2_CHECK_ARG(conv_tc_staged_bytes(d) > 0 && staged_bytes >= conv_tc_staged_bytes(d) &&
                         ((uintptr_t)staged & 15) == 0,
                     "conv2d_bwd_filter_staged: staged input does not match this convolution");
    }
    if (staged_dy) {
      PVB2_CHECK_ARG(conv_tc_staged_grad_bytes(d) > 0 && staged_dy_bytes >= conv_tc_staged_grad_bytes(d) &&
                         ((uintptr_t)staged_dy & 15) == 0,
                     "conv2d_bwd_filter_staged_grad: staged grad_output does not match this convolution");
    }
    PVB2_TRY(conv_tc_bwd_filter(d, (const float*)x->data, (const float*)dy->data, dw, workspace, workspace_bytes, s,
                                &handled, staged, staged_dy));
    if (handled) return PVB2_OK;
  }
  const int splits = wgrad_splits(g);
  const size_t need = (size_t)splits * wnum * sizeof(float);
  float* part = dw;
  if (splits > 1) {
    PVB2_CHECK_ARG(workspace && workspace_bytes >= need, "conv2d_bwd_filter: workspace too small (%zu < %zu)",
                   workspace_bytes, need);
    part = (float*)workspace;
  }
  ConvBwdFilterProb pb;
  pb.M = g.Kg;
  pb.N = (int64_t)g.Cg * g.R * g.S;
  pb.splits = splits;
  const int64_t kdim = (int64_t)g.N * g.P * g.Q;
  pb.kchunk = ((kdim + splits - 1) / splits + kSimtBK - 1) / kSimtBK * kSimtBK;
  pb.zcount = g.G * splits;
  pb.g = g;
  pb.x = (const float*)x->data;
  pb.dy = (const float*)dy->data;
  pb.part = part;
  // the exact path accumulates the long N*P*Q reduction in fp64: weight
  // gradients sum many cancelling terms
  if (d->math == PVB2_MATH_FP32) {
    PVB2_TRY((launch_igemm_simt<ConvBwdFilterProb, double>(pb, s)));
  } else {
    PVB2_TRY(launch_igemm_simt(pb, s));
  }
  if (splits > 1) {
    reduce_splits_kernel<<<grid_for(wnum, 256), 256, 0, s>>>(part, splits, wnum, dw);
    PVB2_LAUNCH_CHECK();
  }
  return PVB2_OK;
}

}  // extern "C"
