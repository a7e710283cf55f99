// 2-D pooling: max (with int64 indices), average, adaptive average.
//
// Replaces dlprim::core::Pooling2DForward / MaxPooling2DBackward /
// AvgPooling2DBackward as called from src/vision_ops.cpp:188-241 (adaptive
// avg), :353-445 (max_pool2d_cls) and :448-511 (avg_pool2d).  The reference
// recomputed the argmax from x in backward; here the forward writes torch's
// flat h*W+w index so max-pool indices are bit-exact with the CPU, and the
// backward scatters each output's gradient to its index in classes of
// non-overlapping windows (no atomics), so dx is deterministic.
#include <algorithm>
#include "common.cuh"

namespace pvb2 {

// grid (ceil(P*Q / block), min(ceil(planes / 2), 65535)): x covers the
// positions of one plane (32-bit arithmetic), y strides over pairs of planes
__global__ void maxpool_fwd_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t* __restrict__ ind,
                                   int64_t planes, int H, int W, int P, int Q, pvb2_pool2d_desc d) {
  const int o = blockIdx.x * blockDim.x + threadIdx.x;
  if (o >= P * Q) return;
  const int q = o % Q, p = o / Q;
  int h0 = p * d.sh - d.ph, w0 = q * d.sw - d.pw;
  const int h1 = min(h0 + (d.kh - 1) * d.dh + 1, H);
  const int w1 = min(w0 + (d.kw - 1) * d.dw + 1, W);
  while (h0 < 0) h0 += d.dh;
  while (w0 < 0) w0 += d.dw;
  constexpr int kPlanes = 2;
  for (int64_t plane0 = (int64_t)blockIdx.y * kPlanes; plane0 < planes; plane0 += (int64_t)gridDim.y * kPlanes) {
    int best[kPlanes];
    float bv[kPlanes];
#pragma unroll
    for (int u = 0; u < kPlanes; ++u) {
      best[u] = h0 * W + w0;
      bv[u] = -INFINITY;
    }
    for (int h = h0; h < h1; h += d.dh) {
      for (int w = w0; w < w1; w += d.dw) {
        const int idx = h * W + w;
#pragma unroll
        for (int u = 0; u < kPlanes; ++u) {
          if (plane0 + u < planes) {
            const float v = __ldg(x + (plane0 + u) * H * W + idx);
            if (v > bv[u] || v != v) {
              bv[u] = v;
              best[u] = idx;
            }
          }
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kPlanes; ++u) {
      if (plane0 + u < planes) {
        const int64_t oi = (plane0 + u) * P * Q + o;
        y[oi] = bv[u];
        if (ind) ind[oi] = best[u];
      }
    }
  }
}

// first output index whose window [o*s - pad, o*s - pad + (k-1)*dil] can include position `pos`
__device__ __forceinline__ int first_out(int pos, int k, int s, int pad, int dil) {
  int num = pos + pad - (k - 1) * dil;
  if (num <= 0) return 0;
  return (num + s - 1) / s;
}

// Backward as a gather: each input element sums, in increasing output index
// (the order in which torch-CPU's scatter adds them, so the sums are the
// same), the gradients of the outputs whose window can hold it and whose
// recorded argmax it is.  Every dX element is written once, coalesced, so
// there is no clearing pass and no read-modify-write; the few outputs each
// element consults are read by its neighbours too and come from L1.
// grid (ceil(H*W / block), min(planes, 128)): each thread works its
// position's candidate outputs out once and walks planes.
__global__ void maxpool_bwd_gather_kernel(const float* __restrict__ dy, const int64_t* __restrict__ ind,
                                          float* __restrict__ dx, int64_t planes, int H, int W, int P, int Q,
                                          pvb2_pool2d_desc d) {
  const int HW = H * W;
  const int pos = blockIdx.x * blockDim.x + threadIdx.x;
  if (pos >= HW) return;
  const int h = pos / W, w = pos - h * W;
  const int p0 = first_out(h, d.kh, d.sh, d.ph, d.dh), p1 = min(P - 1, (h + d.ph) / d.sh);
  const int q0 = first_out(w, d.kw, d.sw, d.pw, d.dw), q1 = min(Q - 1, (w + d.pw) / d.sw);
  const int64_t PQ = (int64_t)P * Q;
  // four planes at a time, their loads issued together
  constexpr int kU = 4;
  for (int64_t plane0 = blockIdx.y; plane0 < planes; plane0 += (int64_t)kU * gridDim.y) {
    float acc[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) acc[u] = 0.f;
    for (int p = p0; p <= p1; ++p)
      for (int q = q0; q <= q1; ++q) {
        const int o = p * Q + q;
        int64_t iv[kU];
        float gv[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int64_t plane = plane0 + (int64_t)u * gridDim.y;
          iv[u] = plane < planes ? __ldg(ind + plane * PQ + o) : -1;
          gv[u] = plane < planes ? __ldg(dy + plane * PQ + o) : 0.f;
        }
#pragma unroll
        for (int u = 0; u < kU; ++u)
          if (iv[u] == pos) acc[u] += gv[u];
      }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int64_t plane = plane0 + (int64_t)u * gridDim.y;
      if (plane < planes) dx[plane * HW + pos] = acc[u];
    }
  }
}

__device__ __forceinline__ int avg_divisor(const pvb2_pool2d_desc& d, int H, int W, int p, int q, int& hs, int& he,
                                           int& ws, int& we) {
  hs = p * d.sh - d.ph;
  ws = q * d.sw - d.pw;
  he = min(hs + d.kh, H + d.ph);
  we = min(ws + d.kw, W + d.pw);
  const int pool_size = (he - hs) * (we - ws);
  hs = max(hs, 0);
  ws = max(ws, 0);
  he = min(he, H);
  we = min(we, W);
  if (d.divisor_override) return d.divisor_override;
  if (d.count_include_pad) return pool_size;
  return (he - hs) * (we - ws);
}

__global__ void avgpool_fwd_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t planes, int H, int W,
                                   int P, int Q, pvb2_pool2d_desc d) {
  const int64_t total = planes * P * Q;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int q = (int)(i % Q);
    const int p = (int)((i / Q) % P);
    const int64_t plane = i / ((int64_t)P * Q);
    int hs, he, ws, we;
    const int div = avg_divisor(d, H, W, p, q, hs, he, ws, we);
    const float* xp = x + plane * H * W;
    float s = 0.f;
    for (int h = hs; h < he; ++h)
      for (int w = ws; w < we; ++w) s += xp[(int64_t)h * W + w];
    y[i] = s / (float)div;
  }
}

__global__ void avgpool_bwd_kernel(const float* __restrict__ dy, float* __restrict__ dx, int64_t planes, int H, int W,
                                   int P, int Q, pvb2_pool2d_desc d) {
  const int64_t total = planes * H * W;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int w = (int)(i % W);
    const int h = (int)((i / W) % H);
    const int64_t plane = i / ((int64_t)H * W);
    const int p0 = first_out(h, d.kh, d.sh, d.ph, 1);
    const int q0 = first_out(w, d.kw, d.sw, d.pw, 1);
    const int p1 = min((h + d.ph) / d.sh + 1, P);
    const int q1 = min((w + d.pw) / d.sw + 1, Q);
    float acc = 0.f;
    for (int p = p0; p < p1; ++p)
      for (int q = q0; q < q1; ++q) {
        int hs, he, ws, we;
        const int div = avg_divisor(d, H, W, p, q, hs, he, ws, we);
        if (h >= hs && h < he && w >= ws && w < we) acc += dy[plane * P * Q + (int64_t)p * Q + q] / (float)div;
      }
    dx[i] = acc;
  }
}

// adaptive average pooling: window [floor(o*I/O), ceil((o+1)*I/O))
__device__ __forceinline__ int ad_start(int o, int O, int I) { return (int)(((int64_t)o * I) / O); }
__device__ __forceinline__ int ad_end(int o, int O, int I) { return (int)((((int64_t)o + 1) * I + O - 1) / O); }

// global pooling (P=Q=1): one warp per plane
__global__ void global_avgpool_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t planes, int64_t HW) {
  const int lane = threadIdx.x & 31;
  const int64_t plane = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (plane >= planes) return;
  const float* xp = x + plane * HW;
  float s = 0.f;
  for (int64_t i = lane; i < HW; i += 32) s += xp[i];
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) y[plane] = s / (float)HW;
}

__global__ void adaptive_avgpool_fwd_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t planes, int H,
                                            int W, int P, int Q) {
  const int64_t total = planes * P * Q;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int q = (int)(i % Q);
    const int p = (int)((i / Q) % P);
    const int64_t plane = i / ((int64_t)P * Q);
    const int hs = ad_start(p, P, H), he = ad_end(p, P, H);
    const int ws = ad_start(q, Q, W), we = ad_end(q, Q, W);
    const float* xp = x + plane * H * W;
    float s = 0.f;
    for (int h = hs; h < he; ++h)
      for (int w = ws; w < we; ++w) s += xp[(int64_t)h * W + w];
    y[i] = s / (float)((he - hs) * (we - ws));
  }
}

__global__ void adaptive_avgpool_bwd_kernel(const float* __restrict__ dy, float* __restrict__ dx, int64_t planes,
                                            int H, int W, int P, int Q) {
  const int64_t total = planes * H * W;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int w = (int)(i % W);
    const int h = (int)((i / W) % H);
    const int64_t plane = i / ((int64_t)H * W);
    float acc = 0.f;
    // output rows whose window contains h
    for (int p = 0; p < P; ++p) {
      const int hs = ad_start(p, P, H), he = ad_end(p, P, H);
      if (h < hs || h >= he) continue;
      for (int q = 0; q < Q; ++q) {
        const int ws = ad_start(q, Q, W), we = ad_end(q, Q, W);
        if (w < ws || w >= we) continue;
        acc += dy[plane * P * Q + (int64_t)p * Q + q] / (float)((he - hs) * (we - ws));
      }
    }
    dx[i] = acc;
  }
}

// ------------------------------------------------------------ upsample
// source coordinate of output index o along one axis (torch's rules, fp32)
__device__ __forceinline__ int nearest_src(int o, float scale, int in, int out, bool exact) {
  if (out == in) return o;
  if (!exact && out == 2 * in) return o >> 1;
  const int s = exact ? (int)floorf(((float)o + 0.5f) * scale) : (int)floorf((float)o * scale);
  return min(s, in - 1);
}

__device__ __forceinline__ float linear_src(int o, float scale, bool align) {
  if (align) return scale * (float)o;
  const float s = scale * ((float)o + 0.5f) - 0.5f;
  return s < 0.f ? 0.f : s;
}

// bilinear taps of output index o: i0 = floor(src), i1 = i0 + (i0 < in - 1), weights l0, l1
__device__ __forceinline__ void linear_taps(int o, float scale, bool align, int in, int& i0, int& i1, float& l0,
                                            float& l1) {
  const float src = linear_src(o, scale, align);
  i0 = (int)src;
  i1 = i0 + (i0 < in - 1 ? 1 : 0);
  l1 = src - (float)i0;
  l0 = 1.f - l1;
}

// grid (ceil(OH*OW / 256), min(planes, 65535))
__global__ void upsample_fwd_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t planes, int H, int W,
                                    int OH, int OW, int mode, int align, float sh, float sw) {
  const int o = blockIdx.x * blockDim.x + threadIdx.x;
  if (o >= OH * OW) return;
  const int oh = o / OW, ow = o - (o / OW) * OW;
  for (int64_t plane = blockIdx.y; plane < planes; plane += gridDim.y) {
    const float* xp = x + plane * H * W;
    float v;
    if (mode == PVB2_UPSAMPLE_BILINEAR) {
      int h0, h1, w0, w1;
      float a0, a1, b0, b1;
      linear_taps(oh, sh, align != 0, H, h0, h1, a0, a1);
      linear_taps(ow, sw, align != 0, W, w0, w1, b0, b1);
      v = a0 * (b0 * __ldg(xp + h0 * W + w0) + b1 * __ldg(xp + h0 * W + w1)) +
          a1 * (b0 * __ldg(xp + h1 * W + w0) + b1 * __ldg(xp + h1 * W + w1));
    } else {
      const bool exact = mode == PVB2_UPSAMPLE_NEAREST_EXACT;
      v = __ldg(xp + nearest_src(oh, sh, H, OH, exact) * W + nearest_src(ow, sw, W, OW, exact));
    }
    y[plane * OH * OW + o] = v;
  }
}

// outputs along one axis whose taps may reach input index i: a conservative
// range (checked exactly by the caller); scale 0 maps every output to 0
__device__ __forceinline__ void out_range(int i, float scale, int out, int& lo, int& hi) {
  if (!(scale > 0.f)) {
    lo = 0;
    hi = out - 1;
    return;
  }
  lo = max(0, (int)floorf(((float)i - 1.f) / scale) - 2);
  hi = min(out - 1, (int)ceilf(((float)i + 2.f) / scale) + 2);
}

// backward as a gather: each input element sums the outputs that sampled it,
// in increasing output order.  grid (ceil(H*W / 256), min(planes, 65535))
__global__ void upsample_bwd_kernel(const float* __restrict__ dy, float* __restrict__ dx, int64_t planes, int H, int W,
                                    int OH, int OW, int mode, int align, float sh, float sw) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= H * W) return;
  const int ih = i / W, iw = i - (i / W) * W;
  int ohl, ohh, owl, owh;
  out_range(ih, sh, OH, ohl, ohh);
  out_range(iw, sw, OW, owl, owh);
  const bool exact = mode == PVB2_UPSAMPLE_NEAREST_EXACT;
  for (int64_t plane = blockIdx.y; plane < planes; plane += gridDim.y) {
    const float* gp = dy + plane * OH * OW;
    float acc = 0.f;
    for (int oh = ohl; oh <= ohh; ++oh) {
      float wh;
      if (mode == PVB2_UPSAMPLE_BILINEAR) {
        int h0, h1;
        float a0, a1;
        linear_taps(oh, sh, align != 0, H, h0, h1, a0, a1);
        wh = (h0 == ih ? a0 : 0.f) + (h1 == ih ? a1 : 0.f);
      } else {
        wh = nearest_src(oh, sh, H, OH, exact) == ih ? 1.f : 0.f;
      }
      if (wh == 0.f) continue;
      for (int ow = owl; ow <= owh; ++ow) {
        float ww;
        if (mode == PVB2_UPSAMPLE_BILINEAR) {
          int w0, w1;
          float b0, b1;
          linear_taps(ow, sw, align != 0, W, w0, w1, b0, b1);
          ww = (w0 == iw ? b0 : 0.f) + (w1 == iw ? b1 : 0.f);
        } else {
          ww = nearest_src(ow, sw, W, OW, exact) == iw ? 1.f : 0.f;
        }
        if (ww != 0.f) acc += wh * ww * __ldg(gp + oh * OW + ow);
      }
    }
    dx[plane * H * W + i] = acc;
  }
}

static int check_nchw(const pvb2_tensor* t, const char* what) {
  PVB2_CHECK_ARG(t->dtype == PVB2_F32, "%s: only float32 is supported", what);
  PVB2_CHECK_ARG(t->ndim == 4, "%s: expected a 4-D NCHW tensor", what);
  PVB2_CHECK_ARG(is_contiguous(t), "%s: expected NCHW-contiguous memory", what);
  return PVB2_OK;
}

}  // namespace pvb2

using namespace pvb2;

extern "C" {

int pvb2_max_pool2d_fwd(const pvb2_pool2d_desc* d, const pvb2_tensor* x, const pvb2_tensor* y, int64_t* indices,
                        pvb2_stream stream) {
  PVB2_TRY(check_nchw(x, "max_pool2d"));
  PVB2_TRY(check_nchw(y, "max_pool2d"));
  PVB2_CHECK_ARG(d->kh > 0 && d->kw > 0 && d->sh > 0 && d->sw > 0 && d->dh > 0 && d->dw > 0,
                 "max_pool2d: kernel, stride and dilation must be positive");
  const int64_t planes = x->sizes[0] * x->sizes[1];
  const int64_t total = planes * y->sizes[2] * y->sizes[3];
  if (total == 0) return PVB2_OK;
  PVB2_CHECK_ARG(x->sizes[2] * x->sizes[3] < (int64_t)1 << 31, "max_pool2d: plane too large");
  const int64_t pq = y->sizes[2] * y->sizes[3];
  const dim3 grid((unsigned)((pq + 255) / 256), (unsigned)std::min<int64_t>((planes + 1) / 2, 65535));
  maxpool_fwd_kernel<<<grid, 256, 0, as_stream(stream)>>>(
      (const float*)x->data, (float*)y->data, indices, planes, (int)x->sizes[2], (int)x->sizes[3], (int)y->sizes[2],
      (int)y->sizes[3], *d);
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

int pvb2_max_pool2d_bwd(const pvb2_pool2d_desc* d, const pvb2_tensor* dy, const int64_t* indices,
                        const pvb2_tensor* dx, pvb2_stream stream) {
  PVB2_TRY(check_nchw(dy, "max_pool2d_backward"));
  PVB2_TRY(check_nchw(dx, "max_pool2d_backward"));
  PVB2_CHECK_ARG(d->kh > 0 && d->kw > 0 && d->sh > 0 && d->sw > 0 && d->dh > 0 && d->dw > 0,
                 "max_pool2d_backward: kernel, stride and dilation must be positive");
  const int64_t planes = dx->sizes[0] * dx->sizes[1];
  const int64_t hw = dx->sizes[2] * dx->sizes[3];
  const int64_t pq = dy->sizes[2] * dy->sizes[3];
  if (planes * hw == 0) return PVB2_OK;
  PVB2_CHECK_ARG(hw < (int64_t)1 << 31 && pq < (int64_t)1 << 31, "max_pool2d_backward: plane too large");
  cudaStream_t s = as_stream(stream);
  if (pq == 0) {
    PVB2_CUDA_TRY(cudaMemsetAsync(dx->data, 0, (size_t)(planes * hw) * sizeof(float), s));
    return PVB2_OK;
  }
  const dim3 grid((unsigned)((hw + 255) / 256), (unsigned)std::min<int64_t>(planes, 128));
  maxpool_bwd_gather_kernel<<<grid, 256, 0, s>>>((const float*)dy->data, indices, (float*)dx->data, planes,
                                                 (int)dx->sizes[2], (int)dx->sizes[3], (int)dy->sizes[2],
                                                 (int)dy->sizes[3], *d);
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

static int upsample_launch(bool bwd, int mode, int align, float sh, float sw, const pvb2_tensor* in,
                           const pvb2_tensor* out, pvb2_stream stream) {
  const char* what = bwd ? "upsample2d_backward" : "upsample2d";
  PVB2_TRY(check_nchw(in, what));
  PVB2_TRY(check_nchw(out, what));
  PVB2_CHECK_ARG(mode >= PVB2_UPSAMPLE_NEAREST && mode <= PVB2_UPSAMPLE_BILINEAR, "%s: unknown mode %d", what, mode);
  PVB2_CHECK_ARG(in->sizes[0] == out->sizes[0] && in->sizes[1] == out->sizes[1], "%s: N, C mismatch", what);
  // forward: in = x (H, W), out = y (OH, OW); backward: in = dy (OH, OW), out = dx (H, W)
  const pvb2_tensor* small = bwd ? out : in;
  const pvb2_tensor* big = bwd ? in : out;
  const int64_t planes = small->sizes[0] * small->sizes[1];
  const int64_t H = small->sizes[2], W = small->sizes[3], OH = big->sizes[2], OW = big->sizes[3];
  PVB2_CHECK_ARG(H * W < (int64_t)1 << 31 && OH * OW < (int64_t)1 << 31, "%s: plane too large", what);
  if (planes == 0 || H * W == 0 || OH * OW == 0) {
    if (bwd && planes * H * W) PVB2_CUDA_TRY(cudaMemsetAsync(out->data, 0, planes * H * W * 4, as_stream(stream)));
    return PVB2_OK;
  }
  const int64_t pos = bwd ? H * W : OH * OW;
  const dim3 grid((unsigned)((pos + 255) / 256), (unsigned)std::min<int64_t>(planes, 65535));
  if (bwd)
    upsample_bwd_kernel<<<grid, 256, 0, as_stream(stream)>>>((const float*)in->data, (float*)out->data, planes, (int)H,
                                                             (int)W, (int)OH, (int)OW, mode, align, sh, sw);
  else
    upsample_fwd_kernel<<<grid, 256, 0, as_stream(stream)>>>((const float*)in->data, (float*)out->data, planes, (int)H,
                                                             (int)W, (int)OH, (int)OW, mode, align, sh, sw);
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

int pvb2_upsample2d_fwd(int mode, int align_corners, float scale_h, float scale_w, const pvb2_tensor* x,
                        const pvb2_tensor* y, pvb2_stream stream) {
  return upsample_launch(false, mode, align_corners, scale_h, scale_w, x, y, stream);
}

int pvb2_upsample2d_bwd(int mode, int align_corners, float scale_h, float scale_w, const pvb2_tensor* dy,
                        const pvb2_tensor* dx, pvb2_stream stream) {
  return upsample_launch(true, mode, align_corners, scale_h, scale_w, dy, dx, stream);
}

int pvb2_avg_pool2d_fwd(const pvb2_pool2d_desc* d, const pvb2_tensor* x, const pvb2_tensor* y, pvb2_stream stream) {
  PVB2_TRY(check_nchw(x, "avg_pool2d"));
  PVB2_TRY(check_nchw(y, "avg_pool2d"));
  const int64_t planes = x->sizes[0] * x->sizes[1];
  const int64_t total = planes * y->sizes[2] * y->sizes[3];
  if (total == 0) return PVB2_OK;
  avgpool_fwd_kernel<<<grid_for(total, 256), 256, 0, as_stream(stream)>>>(
      (const float*)x->data, (float*)y->data, planes, (int)x->sizes[2], (int)x->sizes[3], (int)y->sizes[2],
      (int)y->sizes[3], *d);
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

int pvb2_avg_pool2d_bwd(const pvb2_pool2d_desc* d, const pvb2_tensor* dy, const pvb2_tensor* dx, pvb2_stream stream) {
  PVB2_TRY(check_nchw(dy, "avg_pool2d_backward"));
  PVB2_TRY(check_nchw(dx, "avg_pool2d_backward"));
  const int64_t planes = dx->sizes[0] * dx->sizes[1];
  const int64_t total = planes * dx->sizes[2] * dx->sizes[3];
  if (total == 0) return PVB2_OK;
  avgpool_bwd_kernel<<<grid_for(total, 256), 256, 0, as_stream(stream)>>>(
      (const float*)dy->data, (float*)dx->data, planes, (int)dx->sizes[2], (int)dx->sizes[3], (int)dy->sizes[2],
      (int)dy->sizes[3], *d);
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

int pvb2_adaptive_avg_pool2d_fwd(const pvb2_tensor* x, const pvb2_tensor* y, pvb2_stream stream) {
  PVB2_TRY(check_nchw(x, "adaptive_avg_pool2d"));
  PVB2_TRY(check_nchw(y, "adaptive_avg_pool2d"));
  const int64_t planes = x->sizes[0] * x->sizes[1];
  const int H = (int)x->sizes[2], W = (int)x->sizes[3], P = (int)y->sizes[2], Q = (int)y->sizes[3];
  if (planes * P * Q == 0) return PVB2_OK;
  if (P == 1 && Q == 1) {
    const int warps = 8;
    global_avgpool_kernel<<<(unsigned)((planes + warps - 1) / warps), warps * 32, 0, as_stream(stream)>>>(
        (const float*)x->data, (float*)y->data, planes, (int64_t)H * W);
  } else {
    const int64_t total = planes * P * Q;
    adaptive_avgpool_fwd_kernel<<<grid_for(total, 256), 256, 0, as_stream(stream)>>>(
        (const float*)x->data, (float*)y->data, planes, H, W, P, Q);
  }
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

int pvb2_adaptive_avg_pool2d_bwd(const pvb2_tensor* dy, const pvb2_tensor* dx, pvb2_stream stream) {
  PVB2_TRY(check_nchw(dy, "adaptive_avg_pool2d_backward"));
  PVB2_TRY(check_nchw(dx, "adaptive_avg_pool2d_backward"));
  const int64_t planes = dx->sizes[0] * dx->sizes[1];
  const int64_t total = planes * dx->sizes[2] * dx->sizes[3];
  if (total == 0) return PVB2_OK;
  adaptive_avgpool_bwd_kernel<<<grid_for(total, 256), 256, 0, as_stream(stream)>>>(
      (const float*)dy->data, (float*)dx->data, planes, (int)dx->sizes[2], (int)dx->sizes[3], (int)dy->sizes[2],
      (int)dy->sizes[3]);
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

}  // extern "C"
