// (log_)softmax forward/backward over one dim of an (outer, dim, inner)
// view, and the NLL loss.
//
// Replaces dlprim::core::softmax_forward / softmax_backward and
// nll_loss_forward / nll_loss_backward as called from src/loss_ops.cpp:23-65
// and :137-213.  Unlike the reference, nll_loss accepts class weights and any
// ignore_index (the reference required ignore_index < 0, loss_ops.cpp:26-27).
#include "common.cuh"

namespace pvb2 {

__device__ __forceinline__ float warp_max(float v) {
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sumf(float v) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// block-wide all-reduce (max or sum); every thread gets the result
template <bool MAX>
__device__ __forceinline__ float block_all(float v) {
  __shared__ float sh[32];
  v = MAX ? warp_max(v) : warp_sumf(v);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) sh[wid] = v;
  __syncthreads();
  float r = lane < nw ? sh[lane] : (MAX ? -INFINITY : 0.f);
  r = MAX ? warp_max(r) : warp_sumf(r);
  return r;
}

// inner == 1: one CTA per row
template <bool LOG>
__global__ void softmax_row_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t rows, int64_t D) {
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float* xr = x + r * D;
    float* yr = y + r * D;
    float m = -INFINITY;
    for (int64_t j = threadIdx.x; j < D; j += blockDim.x) m = fmaxf(m, xr[j]);
    m = block_all<true>(m);
    float s = 0.f;
    for (int64_t j = threadIdx.x; j < D; j += blockDim.x) s += expf(xr[j] - m);
    s = block_all<false>(s);
    if (LOG) {
      const float ls = logf(s);
      for (int64_t j = threadIdx.x; j < D; j += blockDim.x) yr[j] = xr[j] - m - ls;
    } else {
      const float inv = 1.f / s;
      for (int64_t j = threadIdx.x; j < D; j += blockDim.x) yr[j] = expf(xr[j] - m) * inv;
    }
  }
}

// inner > 1: one thread per (outer, inner) column
template <bool LOG>
__global__ void softmax_col_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t outer, int64_t D,
                                   int64_t inner) {
  const int64_t total = outer * inner;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t o = i / inner, k = i % inner;
    const float* xp = x + o * D * inner + k;
    float* yp = y + o * D * inner + k;
    float m = -INFINITY;
    for (int64_t j = 0; j < D; ++j) m = fmaxf(m, xp[j * inner]);
    float s = 0.f;
    for (int64_t j = 0; j < D; ++j) s += expf(xp[j * inner] - m);
    if (LOG) {
      const float ls = logf(s);
      for (int64_t j = 0; j < D; ++j) yp[j * inner] = xp[j * inner] - m - ls;
    } else {
      const float inv = 1.f / s;
      for (int64_t j = 0; j < D; ++j) yp[j * inner] = expf(xp[j * inner] - m) * inv;
    }
  }
}

template <bool LOG>
__global__ void softmax_bwd_row_kernel(const float* __restrict__ dy, const float* __restrict__ y,
                                       float* __restrict__ dx, int64_t rows, int64_t D) {
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float* g = dy + r * D;
    const float* yr = y + r * D;
    float* o = dx + r * D;
    float s = 0.f;
    for (int64_t j = threadIdx.x; j < D; j += blockDim.x) s += LOG ? g[j] : g[j] * yr[j];
    s = block_all<false>(s);
    for (int64_t j = threadIdx.x; j < D; j += blockDim.x) o[j] = LOG ? g[j] - expf(yr[j]) * s : yr[j] * (g[j] - s);
  }
}

template <bool LOG>
__global__ void softmax_bwd_col_kernel(const float* __restrict__ dy, const float* __restrict__ y,
                                       float* __restrict__ dx, int64_t outer, int64_t D, int64_t inner) {
  const int64_t total = outer * inner;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t o = i / inner, k = i % inner;
    const int64_t base = o * D * inner + k;
    float s = 0.f;
    for (int64_t j = 0; j < D; ++j) s += LOG ? dy[base + j * inner] : dy[base + j * inner] * y[base + j * inner];
    for (int64_t j = 0; j < D; ++j) {
      const int64_t e = base + j * inner;
      dx[e] = LOG ? dy[e] - expf(y[e]) * s : y[e] * (dy[e] - s);
    }
  }
}

// single CTA: loss terms summed in a fixed order (deterministic)
__global__ void nll_fwd_reduce_kernel(const float* __restrict__ x, const int64_t* __restrict__ t,
                                      const float* __restrict__ w, int64_t N, int64_t C, int reduction,
                                      int64_t ignore, float* __restrict__ out, float* __restrict__ total_w) {
  float s = 0.f, tw = 0.f;
  for (int64_t i = threadIdx.x; i < N; i += blockDim.x) {
    const int64_t c = t[i];
    if (c == ignore || c < 0 || c >= C) continue;  // out-of-range targets contribute nothing
    const float wt = w ? w[c] : 1.f;
    s -= x[i * C + c] * wt;
    tw += wt;
  }
  s = block_all<false>(s);
  tw = block_all<false>(tw);
  if (threadIdx.x == 0) {
    *total_w = tw;
    *out = reduction == 1 ? s / tw : s;
  }
}

__global__ void nll_fwd_none_kernel(const float* __restrict__ x, const int64_t* __restrict__ t,
                                    const float* __restrict__ w, int64_t N, int64_t C, int64_t ignore,
                                    float* __restrict__ out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < N; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t c = t[i];
    if (c == ignore || c < 0 || c >= C) {
      out[i] = 0.f;
      continue;
    }
    out[i] = -x[i * C + c] * (w ? w[c] : 1.f);
  }
}

__global__ void nll_bwd_kernel(const float* __restrict__ go, const int64_t* __restrict__ t,
                               const float* __restrict__ w, const float* __restrict__ total_w, int64_t N, int64_t C,
                               int reduction, int64_t ignore, float* __restrict__ gi) {
  const int64_t total = N * C;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = e / C, c = e % C;
    const int64_t tc = t[i];
    float v = 0.f;
    if (c == tc && tc != ignore) {
      const float wt = w ? w[c] : 1.f;
      if (reduction == 0) v = -wt * go[i];
      else if (reduction == 1) v = -wt * go[0] / total_w[0];
      else v = -wt * go[0];
    }
    gi[e] = v;
  }
}

static int threads_for(int64_t D) {
  if (D >= 4096) return 1024;
  if (D >= 1024) return 512;
  if (D >= 256) return 256;
  if (D >= 64) return 64;
  return 32;
}

}  // namespace pvb2

using namespace pvb2;

extern "C" {

int pvb2_softmax_fwd(int log_softmax, const float* x, float* y, int64_t outer, int64_t dim, int64_t inner,
                     pvb2_stream stream) {
  if (outer * dim * inner == 0) return PVB2_OK;
  cudaStream_t s = as_stream(stream);
  if (inner == 1) {
    const int g = (int)std::min<int64_t>(outer, (int64_t)num_sms() * 16);
    if (log_softmax) softmax_row_kernel<true><<<g, threads_for(dim), 0, s>>>(x, y, outer, dim);
    else softmax_row_kernel<false><<<g, threads_for(dim), 0, s>>>(x, y, outer, dim);
  } else {
    const int64_t total = outer * inner;
    if (log_softmax) softmax_col_kernel<true><<<grid_for(total, 256), 256, 0, s>>>(x, y, outer, dim, inner);
    else softmax_col_kernel<false><<<grid_for(total, 256), 256, 0, s>>>(x, y, outer, dim, inner);
  }
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

int pvb2_softmax_bwd(int log_softmax, const float* dy, const float* y, float* dx, int64_t outer, int64_t dim,
                     int64_t inner, pvb2_stream stream) {
  if (outer * dim * inner == 0) return PVB2_OK;
  cudaStream_t s = as_stream(stream);
  if (inner == 1) {
    const int g = (int)std::min<int64_t>(outer, (int64_t)num_sms() * 16);
    if (log_softmax) softmax_bwd_row_kernel<true><<<g, threads_for(dim), 0, s>>>(dy, y, dx, outer, dim);
    else softmax_bwd_row_kernel<false><<<g, threads_for(dim), 0, s>>>(dy, y, dx, outer, dim);
  } else {
    const int64_t total = outer * inner;
    if (log_softmax) softmax_bwd_col_kernel<true><<<grid_for(total, 256), 256, 0, s>>>(dy, y, dx, outer, dim, inner);
    else softmax_bwd_col_kernel<false><<<grid_for(total, 256), 256, 0, s>>>(dy, y, dx, outer, dim, inner);
  }
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

int pvb2_nll_loss_fwd(const float* x, const int64_t* target, const float* weight, int64_t N, int64_t C,
                      int reduction, int64_t ignore_index, float* out, float* total_weight, pvb2_stream stream) {
  PVB2_CHECK_ARG(reduction >= 0 && reduction <= 2, "nll_loss: bad reduction %d", reduction);
  cudaStream_t s = as_stream(stream);
  if (reduction == 0) {
    if (N == 0) return PVB2_OK;
    nll_fwd_none_kernel<<<grid_for(N, 256), 256, 0, s>>>(x, target, weight, N, C, ignore_index, out);
    PVB2_LAUNCH_CHECK();
    if (total_weight) PVB2_CUDA_TRY(cudaMemsetAsync(total_weight, 0, sizeof(float), s));
    return PVB2_OK;
  }
  nll_fwd_reduce_kernel<<<1, 1024, 0, s>>>(x, target, weight, N, C, reduction, ignore_index, out, total_weight);
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

int pvb2_nll_loss_bwd(const float* grad_out, const int64_t* target, const float* weight, const float* total_weight,
                      int64_t N, int64_t C, int reduction, int64_t ignore_index, float* grad_in, pvb2_stream stream) {
  if (N * C == 0) return PVB2_OK;
  nll_bwd_kernel<<<grid_for(N * C, 256), 256, 0, as_stream(stream)>>>(grad_out, target, weight, total_weight, N, C,
                                                                      reduction, ignore_index, grad_in);
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

}  // extern "C"
