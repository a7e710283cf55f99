// Batch norm and layer norm, forward and backward.
//
// Replaces dlprim::core::BatchNormFwdBwd as driven by native_batch_norm /
// native_batch_norm_backward (src/norm_ops.cpp:19-164) and the
// batch-norm-over-(1,B,N) trick the reference used for layer norm
// (norm_ops.cpp:167-351).
//
// Training batch norm runs as two streaming launches over fixed element
// ranges of each channel (bn_st_* below: statistics, then apply in reverse
// channel order so the second read mostly hits L2).  Tensors with more than
// 65535 channels or 2^30 elements per channel use the plane-based kernels:
//   1. stats:   grid (C, splits); each CTA reduces whole (n, c) planes with
//               128-bit loads into a shifted sum / sum of squares; the
//               per-CTA partials go to the caller's workspace.
//   2. apply:   grid over planes; each CTA folds its channel's partials
//               (few, in double), computes mean / invstd, and writes
//               y = x * a + b with a = invstd*gamma, b = beta - mean*a.
//               The CTA that owns plane (0, c) also writes save_mean /
//               save_invstd and updates the running statistics.
// The backward pass has the same shape: a reduction of (sum dy,
// sum dy*(x-mean)) per channel, then an apply pass for dx.
#include <algorithm>
#include <mutex>
#include "common.cuh"


namespace pvb2 {

constexpr int kBnThreads = 256;

struct BnGeom {
  int64_t N, C, HW;
  int splits;          // CTAs per channel in the reduction pass
  int64_t planes_per;  // planes of one channel handled by one reduction CTA
};

static BnGeom bn_geom(const pvb2_tensor* x) {
  BnGeom g;
  g.N = x->sizes[0];
  g.C = x->sizes[1];
  g.HW = 1;
  for (int d = 2; d < x->ndim; ++d) g.HW *= x->sizes[d];
  int64_t target = (int64_t)num_sms() * 4;
  int64_t splits = (target + g.C - 1) / g.C;
  if (splits > g.N) splits = g.N;
  if (splits < 1) splits = 1;
  if (g.N == 0) {
    g.planes_per = 1;
    g.splits = 1;
    return g;
  }
  g.planes_per = (g.N + splits - 1) / splits;
  g.splits = (int)((g.N + g.planes_per - 1) / g.planes_per);
  return g;
}

__device__ __forceinline__ float warp_sum(float v) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
  return v;
}

// block-wide sum of two values; result valid in thread 0
__device__ __forceinline__ void block_sum2(float& a, float& b) {
  __shared__ float sa[32], sb[32];
  a = warp_sum(a);
  b = warp_sum(b);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) {
    sa[wid] = a;
    sb[wid] = b;
  }
  __syncthreads();
  if (wid == 0) {
    const int nw = blockDim.x >> 5;
    a = lane < nw ? sa[lane] : 0.f;
    b = lane < nw ? sb[lane] : 0.f;
    a = warp_sum(a);
    b = warp_sum(b);
  }
  __syncthreads();
}

// shifted sums over a run of contiguous floats
__device__ __forceinline__ void plane_sums(const float* __restrict__ p, int64_t HW, float shift, float& s1, float& s2) {
  if ((HW & 3) == 0 && (((uintptr_t)p) & 15) == 0) {
    const float4* p4 = reinterpret_cast<const float4*>(p);
    const int64_t n4 = HW >> 2;
    for (int64_t i = threadIdx.x; i < n4; i += blockDim.x) {
      float4 v = __ldg(p4 + i);
      float a = v.x - shift, b = v.y - shift, c = v.z - shift, d = v.w - shift;
      s1 += (a + b) + (c + d);
      s2 += (a * a + b * b) + (c * c + d * d);
    }
  } else {
    for (int64_t i = threadIdx.x; i < HW; i += blockDim.x) {
      float a = __ldg(p + i) - shift;
      s1 += a;
      s2 += a * a;
    }
  }
}

__global__ void bn_stats_kernel(const float* __restrict__ x, int64_t N, int64_t C, int64_t HW, int64_t planes_per,
                                int splits, float* __restrict__ part /* [C][splits][2] */) {
  const int64_t c = blockIdx.x;
  const int sidx = blockIdx.y;
  const float shift = __ldg(x + c * HW);  // sample (0, c, 0): keeps the sums well conditioned
  float s1 = 0.f, s2 = 0.f;
  const int64_t n0 = (int64_t)sidx * planes_per;
  const int64_t n1 = min(N, n0 + planes_per);
  for (int64_t n = n0; n < n1; ++n) plane_sums(x + (n * C + c) * HW, HW, shift, s1, s2);
  block_sum2(s1, s2);
  if (threadIdx.x == 0) {
    part[(c * splits + sidx) * 2 + 0] = s1;
    part[(c * splits + sidx) * 2 + 1] = s2;
  }
}

// fold the per-CTA shifted partials of channel c into mean / biased var
__device__ __forceinline__ void bn_fold(const float* __restrict__ part, int splits, int64_t c, double count,
                                        float shift, double& mean, double& var) {
  double s1 = 0.0, s2 = 0.0;
  for (int k = 0; k < splits; ++k) {
    s1 += (double)part[(c * splits + k) * 2 + 0];
    s2 += (double)part[(c * splits + k) * 2 + 1];
  }
  double m = s1 / count;
  var = s2 / count - m * m;
  if (var < 0.0) var = 0.0;
  mean = m + (double)shift;
}

__global__ void bn_apply_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t N, int64_t C, int64_t HW,
                                int splits, const float* __restrict__ part, const float* __restrict__ gamma,
                                const float* __restrict__ beta, float* __restrict__ running_mean,
                                float* __restrict__ running_var, float momentum, float eps,
                                float* __restrict__ save_mean, float* __restrict__ save_invstd) {
  __shared__ float s_a, s_b;
  const int64_t plane = blockIdx.x;  // n * C + c
  const int64_t c = plane % C;
  if (threadIdx.x == 0) {
    const double count = (double)N * (double)HW;
    double mean, var;
    bn_fold(part, splits, c, count, __ldg(x + c * HW), mean, var);
    const float invstd = (float)(1.0 / sqrt(var + (double)eps));
    const float meanf = (float)mean;
    const float g = gamma ? gamma[c] : 1.f;
    const float b = beta ? beta[c] : 0.f;
    const float a = invstd * g;
    s_a = a;
    s_b = b - meanf * a;
    if (plane < C) {  // n == 0: one CTA per channel publishes the statistics
      if (save_mean) save_mean[c] = meanf;
      if (save_invstd) save_invstd[c] = invstd;
      if (running_mean) running_mean[c] = (1.f - momentum) * running_mean[c] + momentum * meanf;
      if (running_var) {
        const double unbiased = count > 1.0 ? var * count / (count - 1.0) : var;
        running_var[c] = (1.f - momentum) * running_var[c] + momentum * (float)unbiased;
      }
    }
  }
  __syncthreads();
  const float a = s_a, b = s_b;
  const float* xp = x + plane * HW;
  float* yp = y + plane * HW;
  if ((HW & 3) == 0 && (((uintptr_t)xp) & 15) == 0 && (((uintptr_t)yp) & 15) == 0) {
    const float4* x4 = reinterpret_cast<const float4*>(xp);
    float4* y4 = reinterpret_cast<float4*>(yp);
    for (int64_t i = threadIdx.x; i < (HW >> 2); i += blockDim.x) {
      float4 v = x4[i];
      v.x = fmaf(v.x, a, b);
      v.y = fmaf(v.y, a, b);
      v.z = fmaf(v.z, a, b);
      v.w = fmaf(v.w, a, b);
      y4[i] = v;
    }
  } else {
    for (int64_t i = threadIdx.x; i < HW; i += blockDim.x) yp[i] = fmaf(xp[i], a, b);
  }
}

__global__ void bn_eval_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t C, int64_t HW,
                               const float* __restrict__ gamma, const float* __restrict__ beta,
                               const float* __restrict__ rmean, const float* __restrict__ rvar, float eps) {
  __shared__ float s_a, s_b;
  const int64_t plane = blockIdx.x;
  const int64_t c = plane % C;
  if (threadIdx.x == 0) {
    const float invstd = 1.f / sqrtf(rvar[c] + eps);
    const float g = gamma ? gamma[c] : 1.f;
    const float b = beta ? beta[c] : 0.f;
    s_a = invstd * g;
    s_b = b - rmean[c] * s_a;
  }
  __syncthreads();
  const float a = s_a, b = s_b;
  const float* xp = x + plane * HW;
  float* yp = y + plane * HW;
  for (int64_t i = threadIdx.x; i < HW; i += blockDim.x) yp[i] = fmaf(xp[i], a, b);
}

// backward reduction: per channel sum(dy) and sum(dy * (x - mean))
__global__ void bn_bwd_reduce_kernel(const float* __restrict__ dy, const float* __restrict__ x,
                                     const float* __restrict__ mean, int64_t N, int64_t C, int64_t HW,
                                     int64_t planes_per, int splits, float* __restrict__ part) {
  const int64_t c = blockIdx.x;
  const int sidx = blockIdx.y;
  const float m = mean[c];
  float s_dy = 0.f, s_dot = 0.f;
  const int64_t n0 = (int64_t)sidx * planes_per;
  const int64_t n1 = min(N, n0 + planes_per);
  for (int64_t n = n0; n < n1; ++n) {
    const float* g = dy + (n * C + c) * HW;
    const float* xp = x + (n * C + c) * HW;
    if ((HW & 3) == 0 && (((uintptr_t)g) & 15) == 0 && (((uintptr_t)xp) & 15) == 0) {
      const float4* g4 = reinterpret_cast<const float4*>(g);
      const float4* x4 = reinterpret_cast<const float4*>(xp);
      for (int64_t i = threadIdx.x; i < (HW >> 2); i += blockDim.x) {
        float4 a = __ldg(g4 + i), b = __ldg(x4 + i);
        s_dy += (a.x + a.y) + (a.z + a.w);
        s_dot += (a.x * (b.x - m) + a.y * (b.y - m)) + (a.z * (b.z - m) + a.w * (b.w - m));
      }
    } else {
      for (int64_t i = threadIdx.x; i < HW; i += blockDim.x) {
        float a = __ldg(g + i);
        s_dy += a;
        s_dot += a * (__ldg(xp + i) - m);
      }
    }
  }
  block_sum2(s_dy, s_dot);
  if (threadIdx.x == 0) {
    part[(c * splits + sidx) * 2 + 0] = s_dy;
    part[(c * splits + sidx) * 2 + 1] = s_dot;
  }
}

__global__ void bn_bwd_apply_kernel(const float* __restrict__ dy, const float* __restrict__ x,
                                    const float* __restrict__ mean, const float* __restrict__ invstd,
                                    const float* __restrict__ gamma, int64_t N, int64_t C, int64_t HW, int splits,
                                    const float* __restrict__ part, float* __restrict__ dx,
                                    float* __restrict__ dgamma, float* __restrict__ dbeta) {
  __shared__ float s_k, s_gm, s_mul, s_mean;
  const int64_t plane = blockIdx.x;
  const int64_t c = plane % C;
  if (threadIdx.x == 0) {
    double sdy = 0.0, sdot = 0.0;
    for (int k = 0; k < splits; ++k) {
      sdy += (double)part[(c * splits + k) * 2 + 0];
      sdot += (double)part[(c * splits + k) * 2 + 1];
    }
    const double count = (double)N * (double)HW;
    const float is = invstd[c];
    s_mean = mean[c];
    s_gm = (float)(sdy / count);                          // mean of dy
    s_k = (float)(sdot / count) * is * is;                // dotp * invstd^2 / count
    s_mul = is * (gamma ? gamma[c] : 1.f);
    if (plane < C) {
      if (dgamma) dgamma[c] = (float)sdot * is;
      if (dbeta) dbeta[c] = (float)sdy;
    }
  }
  __syncthreads();
  if (!dx) return;
  const float k = s_k, gm = s_gm, mul = s_mul, m = s_mean;
  const float* g = dy + plane * HW;
  const float* xp = x + plane * HW;
  float* o = dx + plane * HW;
  for (int64_t i = threadIdx.x; i < HW; i += blockDim.x) o[i] = (g[i] - gm - (xp[i] - m) * k) * mul;
}

__global__ void bn_bwd_eval_kernel(const float* __restrict__ dy, const float* __restrict__ rvar,
                                   const float* __restrict__ gamma, float eps, int64_t C, int64_t HW,
                                   float* __restrict__ dx) {
  const int64_t plane = blockIdx.x;
  const int64_t c = plane % C;
  const float mul = (gamma ? gamma[c] : 1.f) / sqrtf(rvar[c] + eps);
  const float* g = dy + plane * HW;
  float* o = dx + plane * HW;
  for (int64_t i = threadIdx.x; i < HW; i += blockDim.x) o[i] = g[i] * mul;
}

// Position of element e = n*HW + i of one channel, advanced by a fixed step
// without dividing in the loop.
struct ChanWalk {
  int n, i, dn, di, HW;
  __device__ __forceinline__ ChanWalk(int e0, int step, int hw) : HW(hw) {
    n = e0 / hw;
    i = e0 - n * hw;
    dn = step / hw;
    di = step - dn * hw;
  }
  __device__ __forceinline__ void next() {
    i += di;
    n += dn;
    if (i >= HW) {
      i -= HW;
      ++n;
    }
  }
};

// ------------------------------------------ batch norm, two streaming passes
// Training batch norm as two grid-wide passes over fixed element ranges:
//   stats  grid (splits, C): CTA (s, c) reduces elements [s*chunk, (s+1)*chunk)
//          of channel c's (n, hw) range to a shifted sum and sum of squares
//          (shift = the channel's first element) in the workspace;
//   apply  grid (splits, C), channels in reverse order so that the ranges the
//          stats pass read last (still in L2) are read first: thread 0 folds
//          the channel's partials in double, then the CTA writes its range.
// A channel's range is walked with 128-bit accesses when HW % 4 == 0.  The
// backward has the same shape: sums of dy and dy*(x - mean), then dx.
constexpr int kBnStThreads = 256;
constexpr int kBnStChunk = 16384;  // elements of one channel per CTA (64 KB)

struct BnStream {
  int splits, chunk;
  bool vec;
};

// channels on grid y, 32-bit element indices within a channel
static bool bn_streamable(const BnGeom& g) {
  return g.C <= 65535 && g.N * g.HW < ((int64_t)1 << 30) && g.N * g.HW > 0;
}

static BnStream bn_stream_plan(const BnGeom& g, const void* const* ptrs, int nptr) {
  BnStream p;
  const int64_t M = g.N * g.HW;
  int64_t splits = (M + kBnStChunk - 1) / kBnStChunk;
  // enough CTAs for every SM twice, but no range below 1024 elements
  const int64_t want = (2 * (int64_t)num_sms() + g.C - 1) / std::max<int64_t>(g.C, 1);
  splits = std::max(splits, std::min(want, (M + 1023) / 1024));
  splits = std::max<int64_t>(1, std::min<int64_t>(splits, 65535));
  int64_t chunk = (M + splits - 1) / splits;
  chunk = (chunk + 3) / 4 * 4;
  p.chunk = (int)chunk;
  p.splits = (int)((M + chunk - 1) / chunk);
  p.vec = (g.HW & 3) == 0;
  for (int i = 0; i < nptr; ++i)
    if (ptrs[i] && ((uintptr_t)ptrs[i] & 15)) p.vec = false;
  return p;
}

// sum of two values over the block; every thread gets the results
__device__ __forceinline__ void block_allsum2(float& a, float& b, float* red) {
  a = warp_sum(a);
  b = warp_sum(b);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) {
    red[wid] = a;
    red[32 + wid] = b;
  }
  __syncthreads();
  a = 0.f;
  b = 0.f;
  for (int i = 0; i < nw; ++i) {
    a += red[i];
    b += red[32 + i];
  }
}

// counter (or null): an int64 the first CTA's first thread increments (the
// module's num_batches_tracked, whose `+= 1` the host hands over instead of
// launching a kernel for it)
__global__ void __launch_bounds__(kBnStThreads) bn_st_stats_kernel(const float* __restrict__ x, int N, int C, int HW,
                                                                   int chunk, int splits, int vec,
                                                                   float* __restrict__ part,
                                                                   long long* __restrict__ counter) {
  __shared__ float red[64];
  const int s = blockIdx.x, c = blockIdx.y;
  if (counter && s == 0 && c == 0 && threadIdx.x == 0) *counter += 1;
  const int M = N * HW, start = s * chunk, end = min(M, start + chunk);
  const int64_t nstride = (int64_t)C * HW;
  const float* xc = x + (int64_t)c * HW;
  const float shift = __ldg(xc);
  float s1 = 0.f, s2 = 0.f;
  const int vw = vec ? 4 : 1, step = vw * blockDim.x;
  int e = start + vw * threadIdx.x;
  if (e < end) {
    ChanWalk w(e, step, HW);
    if (vec) {
      // four 128-bit loads in flight per thread
      for (; e < end; e += 4 * step) {
        float4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          v[u] = e + u * step < end ? __ldg(reinterpret_cast<const float4*>(xc + w.n * nstride + w.i))
                                    : make_float4(shift, shift, shift, shift);
          w.next();
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float a = v[u].x - shift, b = v[u].y - shift, d = v[u].z - shift, f = v[u].w - shift;
          s1 += (a + b) + (d + f);
          s2 += (a * a + b * b) + (d * d + f * f);
        }
      }
    } else {
      for (; e < end; e += 4 * step) {
        float v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          v[u] = e + u * step < end ? __ldg(xc + w.n * nstride + w.i) : shift;
          w.next();
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float a = v[u] - shift;
          s1 += a;
          s2 += a * a;
        }
      }
    }
  }
  block_allsum2(s1, s2, red);
  if (threadIdx.x == 0) {
    part[((int64_t)c * splits + s) * 2 + 0] = s1;
    part[((int64_t)c * splits + s) * 2 + 1] = s2;
  }
}

// y = act(a * x + b + residual): residual optional (same layout as x), act
// the identity (0), ReLU (1) or ReLU6 = hardtanh(0, 6) (2), NaN kept in both
// as torch's relu and hardtanh keep it; the epilogue of `bn(x) (+ identity)`
// followed by an in-place activation, fused by the host
__device__ __forceinline__ float bn_epi(float v, const float* res, int64_t o, int act) {
  if (res) v += __ldg(res + o);
  if (act == 1) v = v != v ? v : (v > 0.f ? v : 0.f);
  if (act == 2) v = v != v ? v : (v < 0.f ? 0.f : (v > 6.f ? 6.f : v));
  return v;
}

// the gradient below the activation bn_epi applied, from its output r and the
// gradient g above it: ReLU as threshold_backward (r <= 0 ? 0 : g), ReLU6 as
// hardtanh_backward ((r <= 0 || r >= 6) ? 0 : g); NaN outputs pass g
__device__ __forceinline__ float act_grad(float r, float g, int act) {
  return (r <= 0.f || (act == 2 && r >= 6.f)) ? 0.f : g;
}

__global__ void __launch_bounds__(kBnStThreads) bn_st_apply_kernel(
    const float* __restrict__ x, float* __restrict__ y, int N, int C, int HW, int chunk, int splits, int vec,
    const float* __restrict__ part, const float* __restrict__ gamma, const float* __restrict__ beta,
    float* __restrict__ running_mean, float* __restrict__ running_var, float momentum, float eps,
    float* __restrict__ save_mean, float* __restrict__ save_invstd, const float* __restrict__ residual, int act,
    float* __restrict__ sum_out, float* __restrict__ ab_out) {
  // ab_out (or null): the channel's (a, b) of y = fmaf(x, a, b), a at [c],
  // b at [C + c], for a backward that forms the activation's mask from x
  __shared__ float s_ab[2];
  const int s = blockIdx.x, c = C - 1 - blockIdx.y;
  const int M = N * HW, start = s * chunk, end = min(M, start + chunk);
  const int64_t nstride = (int64_t)C * HW;
  const float* xc = x + (int64_t)c * HW;
  if (threadIdx.x == 0) {
    double s1 = 0.0, s2 = 0.0;
    for (int k = 0; k < splits; ++k) {
      s1 += (double)part[((int64_t)c * splits + k) * 2 + 0];
      s2 += (double)part[((int64_t)c * splits + k) * 2 + 1];
    }
    const double count = (double)M;
    const double m = s1 / count;
    double var = s2 / count - m * m;
    if (var < 0.0) var = 0.0;
    const double mean = m + (double)__ldg(xc);
    const float invstd = (float)(1.0 / sqrt(var + (double)eps));
    const float meanf = (float)mean;
    const float g = gamma ? gamma[c] : 1.f;
    const float b = beta ? beta[c] : 0.f;
    const float a = invstd * g;
    s_ab[0] = a;
    s_ab[1] = b - meanf * a;
    if (s == 0) {
      if (ab_out) {
        ab_out[c] = a;
        ab_out[C + c] = s_ab[1];
      }
      if (save_mean) save_mean[c] = meanf;
      if (save_invstd) save_invstd[c] = invstd;
      if (running_mean) running_mean[c] = (1.f - momentum) * running_mean[c] + momentum * meanf;
      if (running_var) {
        const double unbiased = count > 1.0 ? var * count / (count - 1.0) : var;
        running_var[c] = (1.f - momentum) * running_var[c] + momentum * (float)unbiased;
      }
    }
  }
  __syncthreads();
  const float a = s_ab[0], b = s_ab[1];
  float* yc = y + (int64_t)c * HW;
  const float* rc = residual ? residual + (int64_t)c * HW : nullptr;
  // with sum_out: y keeps the normalised values and the epilogue result goes
  // to sum_out (which may be the residual itself: each element is read, then
  // written, by the same thread)
  float* sc = sum_out ? sum_out + (int64_t)c * HW : nullptr;
  const int vw = vec ? 4 : 1, step = vw * blockDim.x;
  int e = start + vw * threadIdx.x;
  if (e >= end) return;
  ChanWalk w(e, step, HW);
  const bool plain = rc == nullptr && !act;
  if (vec) {
    for (; e < end; e += 4 * step) {
      float4 v[4];
      int64_t o[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        o[u] = w.n * nstride + w.i;
        if (e + u * step < end) v[u] = __ldg(reinterpret_cast<const float4*>(xc + o[u]));
        w.next();
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (e + u * step < end) {
          float4 r = v[u];
          r.x = fmaf(r.x, a, b);
          r.y = fmaf(r.y, a, b);
          r.z = fmaf(r.z, a, b);
          r.w = fmaf(r.w, a, b);
          if (sc) *reinterpret_cast<float4*>(yc + o[u]) = r;
          if (!plain) {
            r.x = bn_epi(r.x, rc, o[u], act);
            r.y = bn_epi(r.y, rc, o[u] + 1, act);
            r.z = bn_epi(r.z, rc, o[u] + 2, act);
            r.w = bn_epi(r.w, rc, o[u] + 3, act);
          }
          *reinterpret_cast<float4*>((sc ? sc : yc) + o[u]) = r;
        }
      }
    }
  } else {
    for (; e < end; e += 4 * step) {
      float v[4];
      int64_t o[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        o[u] = w.n * nstride + w.i;
        if (e + u * step < end) v[u] = __ldg(xc + o[u]);
        w.next();
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (e + u * step < end) {
          const float r = fmaf(v[u], a, b);
          if (sc) {
            yc[o[u]] = r;
            sc[o[u]] = bn_epi(r, rc, o[u], act);
          } else {
            yc[o[u]] = bn_epi(r, rc, o[u], act);
          }
        }
    }
  }
}

// How the backward forms the gradient below an activation (GATE):
// 0 none (dy is the batch norm's output gradient); 1 / 2 ReLU / ReLU6 whose
// output relu_y is read; 3 / 4 ReLU / ReLU6 whose output act(fmaf(x, a, b))
// is formed from x with the forward's (a, b), bit for bit as the forward
// formed it.  A compile-time mode keeps each form's loop to its own math
// (these loops are latency-bound: every instruction between a load and the
// next one counts).
template <int GATE>
struct BnGate {
  static constexpr bool on = GATE != 0;
  static constexpr bool from_x = GATE >= 3;
  static constexpr int act = (GATE == 1 || GATE == 3) ? 1 : 2;
  __device__ __forceinline__ static float grad(float g, float v, float r, float fa, float fb) {
    if (!on) return g;
    return act_grad(from_x ? bn_epi(fmaf(v, fa, fb), nullptr, 0, act) : r, g, act);
  }
};

// VEC: 128-bit accesses (HW % 4 == 0, aligned pointers).  dy_out (or null):
// where the gradient below the activation is stored.
template <bool VEC, int GATE>
__global__ void __launch_bounds__(kBnStThreads) bn_st_bwd_reduce_kernel(
    const float* __restrict__ dy, const float* __restrict__ x, const float* __restrict__ mean, int N, int C, int HW,
    int chunk, int splits, float* __restrict__ part, const float* __restrict__ relu_y, float* __restrict__ dy_out,
    const float* __restrict__ ab) {
  using G = BnGate<GATE>;
  constexpr bool read_y = G::on && !G::from_x;
  __shared__ float red[64];
  const int s = blockIdx.x, c = blockIdx.y;
  const int M = N * HW, start = s * chunk, end = min(M, start + chunk);
  const int64_t nstride = (int64_t)C * HW;
  const float* gc = dy + (int64_t)c * HW;
  const float* xc = x + (int64_t)c * HW;
  const float* yc = read_y ? relu_y + (int64_t)c * HW : nullptr;
  float* oc = G::on && dy_out ? dy_out + (int64_t)c * HW : nullptr;
  const float fa = G::from_x ? ab[c] : 0.f, fb = G::from_x ? ab[C + c] : 0.f;
  const float m = mean[c];
  float sg = 0.f, sd = 0.f;
  const int vw = VEC ? 4 : 1, step = vw * blockDim.x;
  int e = start + vw * threadIdx.x;
  if (e < end) {
    ChanWalk w(e, step, HW);
    if (VEC) {
      for (; e < end; e += step, w.next()) {
        const int64_t o = w.n * nstride + w.i;
        float4 g = __ldg(reinterpret_cast<const float4*>(gc + o));
        const float4 v = __ldg(reinterpret_cast<const float4*>(xc + o));
        if (G::on) {
          float4 r = make_float4(0.f, 0.f, 0.f, 0.f);
          if (read_y) r = __ldg(reinterpret_cast<const float4*>(yc + o));
          g.x = G::grad(g.x, v.x, r.x, fa, fb);
          g.y = G::grad(g.y, v.y, r.y, fa, fb);
          g.z = G::grad(g.z, v.z, r.z, fa, fb);
          g.w = G::grad(g.w, v.w, r.w, fa, fb);
          if (oc) *reinterpret_cast<float4*>(oc + o) = g;
        }
        sg += (g.x + g.y) + (g.z + g.w);
        sd += (g.x * (v.x - m) + g.y * (v.y - m)) + (g.z * (v.z - m) + g.w * (v.w - m));
      }
    } else {
      for (; e < end; e += 4 * step) {
        float g[4], v[4], r[4];
        int64_t o[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {  // every load first
          o[u] = w.n * nstride + w.i;
          g[u] = 0.f;
          v[u] = m;
          r[u] = 0.f;
          if (e + u * step < end) {
            g[u] = __ldg(gc + o[u]);
            v[u] = __ldg(xc + o[u]);
            if (read_y) r[u] = __ldg(yc + o[u]);
          }
          w.next();
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (G::on && e + u * step < end) {
            g[u] = G::grad(g[u], v[u], r[u], fa, fb);
            if (oc) oc[o[u]] = g[u];
          }
          sg += g[u];
          sd += g[u] * (v[u] - m);
        }
      }
    }
  }
  block_allsum2(sg, sd, red);
  if (threadIdx.x == 0) {
    part[((int64_t)c * splits + s) * 2 + 0] = sg;
    part[((int64_t)c * splits + s) * 2 + 1] = sd;
  }
}

// GATE 0, 3 or 4 (the reading forms hand this pass the stored gradient)
template <bool VEC, int GATE>
__global__ void __launch_bounds__(kBnStThreads) bn_st_bwd_apply_kernel(
    const float* __restrict__ dy, const float* __restrict__ x, const float* __restrict__ mean,
    const float* __restrict__ invstd, const float* __restrict__ gamma, int N, int C, int HW, int chunk, int splits,
    const float* __restrict__ part, float* __restrict__ dx, float* __restrict__ dgamma, float* __restrict__ dbeta,
    const float* __restrict__ ab) {
  using G = BnGate<GATE>;
  static_assert(GATE == 0 || G::from_x, "the apply pass forms the gradient from x or takes it formed");
  __shared__ float s_k[3];
  const int s = blockIdx.x, c = C - 1 - blockIdx.y;
  const int M = N * HW, start = s * chunk, end = min(M, start + chunk);
  const int64_t nstride = (int64_t)C * HW;
  if (threadIdx.x == 0) {
    double sg = 0.0, sd = 0.0;
    for (int k = 0; k < splits; ++k) {
      sg += (double)part[((int64_t)c * splits + k) * 2 + 0];
      sd += (double)part[((int64_t)c * splits + k) * 2 + 1];
    }
    const double count = (double)M;
    const float is = invstd[c];
    s_k[0] = (float)(sg / count);             // mean of dy
    s_k[1] = (float)(sd / count) * is * is;   // dotp * invstd^2 / count
    s_k[2] = is * (gamma ? gamma[c] : 1.f);
    if (s == 0) {
      if (dgamma) dgamma[c] = (float)sd * is;
      if (dbeta) dbeta[c] = (float)sg;
    }
  }
  __syncthreads();
  if (!dx) return;
  const float gm = s_k[0], kk = s_k[1], mul = s_k[2], m = mean[c];
  const float fa = G::from_x ? ab[c] : 0.f, fb = G::from_x ? ab[C + c] : 0.f;
  const float* gc = dy + (int64_t)c * HW;
  const float* xc = x + (int64_t)c * HW;
  float* dc = dx + (int64_t)c * HW;
  const int vw = VEC ? 4 : 1, step = vw * blockDim.x;
  int e = start + vw * threadIdx.x;
  if (e >= end) return;
  ChanWalk w(e, step, HW);
  if (VEC) {
    // two float4 steps per iteration, both loads issued before the math
    for (; e < end; e += 2 * step) {
      float4 g[2], v[2];
      int64_t o[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        o[u] = w.n * nstride + w.i;
        if (e + u * step < end) {
          g[u] = __ldg(reinterpret_cast<const float4*>(gc + o[u]));
          v[u] = __ldg(reinterpret_cast<const float4*>(xc + o[u]));
        }
        w.next();
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        if (e + u * step >= end) continue;
        float4 gg = g[u];
        const float4 vv = v[u];
        gg.x = G::grad(gg.x, vv.x, 0.f, fa, fb);
        gg.y = G::grad(gg.y, vv.y, 0.f, fa, fb);
        gg.z = G::grad(gg.z, vv.z, 0.f, fa, fb);
        gg.w = G::grad(gg.w, vv.w, 0.f, fa, fb);
        float4 r;
        r.x = (gg.x - gm - (vv.x - m) * kk) * mul;
        r.y = (gg.y - gm - (vv.y - m) * kk) * mul;
        r.z = (gg.z - gm - (vv.z - m) * kk) * mul;
        r.w = (gg.w - gm - (vv.w - m) * kk) * mul;
        *reinterpret_cast<float4*>(dc + o[u]) = r;
      }
    }
  } else {
    for (; e < end; e += 4 * step) {
      float g[4], v[4];
      int64_t o[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {  // every load first
        o[u] = w.n * nstride + w.i;
        if (e + u * step < end) {
          g[u] = __ldg(gc + o[u]);
          v[u] = __ldg(xc + o[u]);
        }
        w.next();
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (e + u * step < end) dc[o[u]] = (G::grad(g[u], v[u], 0.f, fa, fb) - gm - (v[u] - m) * kk) * mul;
    }
  }
}

template <bool VEC>
static int launch_bn_bwd(const BnGeom& g, const BnStream& p, int gate, const float* dy, const float* x,
                          const float* mean, const float* invstd, const float* gamma, float* dx, float* dgamma,
                          float* dbeta, float* part, const float* relu_y, float* dy_out, const float* ab,
                          cudaStream_t s) {
  using R = void (*)(const float*, const float*, const float*, int, int, int, int, int, float*, const float*, float*,
                     const float*);
  using A = void (*)(const float*, const float*, const float*, const float*, const float*, int, int, int, int, int,
                     const float*, float*, float*, float*, const float*);
  static const R reduce[5] = {bn_st_bwd_reduce_kernel<VEC, 0>, bn_st_bwd_reduce_kernel<VEC, 1>,
                              bn_st_bwd_reduce_kernel<VEC, 2>, bn_st_bwd_reduce_kernel<VEC, 3>,
                              bn_st_bwd_reduce_kernel<VEC, 4>};
  static const A apply[3] = {bn_st_bwd_apply_kernel<VEC, 0>, bn_st_bwd_apply_kernel<VEC, 3>,
                             bn_st_bwd_apply_kernel<VEC, 4>};
  const dim3 grid((unsigned)p.splits, (unsigned)g.C);
  reduce[gate]<<<grid, kBnStThreads, 0, s>>>(dy, x, mean, (int)g.N, (int)g.C, (int)g.HW, p.chunk, p.splits, part,
                                            relu_y, dy_out, ab);
  PVB2_LAUNCH_CHECK();
  // the apply pass reads the stored gradient below a read activation, or
  // forms it again from x
  if (gate == 1 || gate == 2) dy = dy_out;
  apply[gate >= 3 ? gate - 2 : 0]<<<grid, kBnStThreads, 0, s>>>(dy, x, mean, invstd, gamma, (int)g.N, (int)g.C,
                                                                (int)g.HW, p.chunk, p.splits, part, dx, dgamma,
                                                                dbeta, ab);
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

static int bn_fwd_stream(const BnGeom& g, const BnStream& p, const float* x, float* y, const float* gamma,
                         const float* beta, float* running_mean, float* running_var, double momentum, double eps,
                         float* save_mean, float* save_invstd, float* part, cudaStream_t s) {
  const dim3 grid((unsigned)p.splits, (unsigned)g.C);
  bn_st_stats_kernel<<<grid, kBnStThreads, 0, s>>>(x, (int)g.N, (int)g.C, (int)g.HW, p.chunk, p.splits, p.vec ? 1 : 0,
                                                    part, nullptr);
  PVB2_LAUNCH_CHECK();
  bn_st_apply_kernel<<<grid, kBnStThreads, 0, s>>>(x, y, (int)g.N, (int)g.C, (int)g.HW, p.chunk, p.splits,
                                                    p.vec ? 1 : 0, part, gamma, beta, running_mean, running_var,
                                                    (float)momentum, (float)eps, save_mean, save_invstd, nullptr, 0,
                                                    nullptr, nullptr);
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

static int bn_bwd_stream(const BnGeom& g, const BnStream& p, const float* dy, const float* x, const float* mean,
                         const float* invstd, const float* gamma, float* dx, float* dgamma, float* dbeta, float* part,
                         cudaStream_t s, const float* relu_y = nullptr, float* dy_out = nullptr, int act = 0,
                         const float* ab = nullptr) {
  // gate: 0 none, 1 / 2 ReLU / ReLU6 read from relu_y, 3 / 4 formed from x
  const int gate = ab ? (act == 1 ? 3 : 4) : (relu_y ? act : 0);
  if (p.vec)
    return launch_bn_bwd<true>(g, p, gate, dy, x, mean, invstd, gamma, dx, dgamma, dbeta, part, relu_y, dy_out, ab,
                               s);
  return launch_bn_bwd<false>(g, p, gate, dy, x, mean, invstd, gamma, dx, dgamma, dbeta, part, relu_y, dy_out, ab,
                              s);
}

// ------------------------------------------------------------- layer norm
// one warp per row; the row is held in registers (N <= 32 * kLnMaxPerLane)
constexpr int kLnMaxPerLane = 32;

__global__ void ln_fwd_kernel(const float* __restrict__ x, const float* __restrict__ gamma,
                              const float* __restrict__ beta, int64_t M, int64_t N, float eps, float* __restrict__ y,
                              float* __restrict__ mean_out, float* __restrict__ rstd_out) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= M) return;
  const float* xr = x + row * N;
  float v[kLnMaxPerLane];
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < kLnMaxPerLane; ++k) {
    int64_t j = (int64_t)k * 32 + lane;
    v[k] = j < N ? xr[j] : 0.f;
    s += v[k];
  }
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float mean = s / (float)N;
  float q = 0.f;
#pragma unroll
  for (int k = 0; k < kLnMaxPerLane; ++k) {
    int64_t j = (int64_t)k * 32 + lane;
    float d = j < N ? v[k] - mean : 0.f;
    q += d * d;
  }
  for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
  const float rstd = 1.f / sqrtf(q / (float)N + eps);
  float* yr = y + row * N;
#pragma unroll
  for (int k = 0; k < kLnMaxPerLane; ++k) {
    int64_t j = (int64_t)k * 32 + lane;
    if (j < N) {
      float o = (v[k] - mean) * rstd;
      if (gamma) o = o * gamma[j];
      if (beta) o = o + beta[j];
      yr[j] = o;
    }
  }
  if (lane == 0) {
    if (mean_out) mean_out[row] = mean;
    if (rstd_out) rstd_out[row] = rstd;
  }
}

// generic (large N) layer norm forward: one CTA per row, two passes over gmem
__global__ void ln_fwd_big_kernel(const float* __restrict__ x, const float* __restrict__ gamma,
                                  const float* __restrict__ beta, int64_t M, int64_t N, float eps,
                                  float* __restrict__ y, float* __restrict__ mean_out, float* __restrict__ rstd_out) {
  __shared__ float s_mean, s_rstd;
  const int64_t row = blockIdx.x;
  const float* xr = x + row * N;
  float s = 0.f, dummy = 0.f;
  for (int64_t j = threadIdx.x; j < N; j += blockDim.x) s += xr[j];
  block_sum2(s, dummy);
  if (threadIdx.x == 0) s_mean = s / (float)N;
  __syncthreads();
  const float mean = s_mean;
  float q = 0.f;
  dummy = 0.f;
  for (int64_t j = threadIdx.x; j < N; j += blockDim.x) {
    float d = xr[j] - mean;
    q += d * d;
  }
  block_sum2(q, dummy);
  if (threadIdx.x == 0) s_rstd = 1.f / sqrtf(q / (float)N + eps);
  __syncthreads();
  const float rstd = s_rstd;
  float* yr = y + row * N;
  for (int64_t j = threadIdx.x; j < N; j += blockDim.x) {
    float o = (xr[j] - mean) * rstd;
    if (gamma) o = o * gamma[j];
    if (beta) o = o + beta[j];
    yr[j] = o;
  }
  if (threadIdx.x == 0) {
    if (mean_out) mean_out[row] = mean;
    if (rstd_out) rstd_out[row] = rstd;
  }
}

// dx for one row per CTA:  dx = rstd * (g - mean(g) - xhat * mean(g * xhat)),  g = dy * gamma
__global__ void ln_bwd_dx_kernel(const float* __restrict__ dy, const float* __restrict__ x,
                                 const float* __restrict__ mean, const float* __restrict__ rstd,
                                 const float* __restrict__ gamma, int64_t N, float* __restrict__ dx) {
  __shared__ float s_a, s_b;
  const int64_t row = blockIdx.x;
  const float* g = dy + row * N;
  const float* xr = x + row * N;
  const float m = mean[row], r = rstd[row];
  float sg = 0.f, sgx = 0.f;
  for (int64_t j = threadIdx.x; j < N; j += blockDim.x) {
    float gv = g[j] * (gamma ? gamma[j] : 1.f);
    float xh = (xr[j] - m) * r;
    sg += gv;
    sgx += gv * xh;
  }
  block_sum2(sg, sgx);
  if (threadIdx.x == 0) {
    s_a = sg / (float)N;
    s_b = sgx / (float)N;
  }
  __syncthreads();
  const float a = s_a, b = s_b;
  float* o = dx + row * N;
  for (int64_t j = threadIdx.x; j < N; j += blockDim.x) {
    float gv = g[j] * (gamma ? gamma[j] : 1.f);
    float xh = (xr[j] - m) * r;
    o[j] = r * (gv - a - xh * b);
  }
}

// dgamma / dbeta partial column sums: CTA (colblock, rowsplit)
__global__ void ln_bwd_param_partial_kernel(const float* __restrict__ dy, const float* __restrict__ x,
                                            const float* __restrict__ mean, const float* __restrict__ rstd, int64_t M,
                                            int64_t N, int64_t rows_per, float* __restrict__ part /* [splits][2][N] */) {
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int sidx = blockIdx.y;
  if (j >= N) return;
  const int64_t r0 = (int64_t)sidx * rows_per, r1 = min(M, r0 + rows_per);
  float sg = 0.f, sgx = 0.f;
  for (int64_t r = r0; r < r1; ++r) {
    float gv = dy[r * N + j];
    sg += gv;
    sgx += gv * (x[r * N + j] - mean[r]) * rstd[r];
  }
  part[((int64_t)sidx * 2 + 0) * N + j] = sgx;
  part[((int64_t)sidx * 2 + 1) * N + j] = sg;
}

__global__ void ln_bwd_param_final_kernel(const float* __restrict__ part, int splits, int64_t N,
                                          float* __restrict__ dgamma, float* __restrict__ dbeta) {
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= N) return;
  float a = 0.f, b = 0.f;
  for (int k = 0; k < splits; ++k) {
    a += part[((int64_t)k * 2 + 0) * N + j];
    b += part[((int64_t)k * 2 + 1) * N + j];
  }
  if (dgamma) dgamma[j] = a;
  if (dbeta) dbeta[j] = b;
}

// ---- rows of N = 128 * NC floats (N <= 1024, 16-byte aligned): a warp per
// row, lane l owning the float4 columns 4 l + 128 k (k < NC), the row held in
// registers
template <int NC>
__global__ void __launch_bounds__(256) ln_fwd_v4_kernel(const float* __restrict__ x, const float* __restrict__ gamma,
                                                        const float* __restrict__ beta, int64_t M, float eps,
                                                        float* __restrict__ y, float* __restrict__ mean_out,
                                                        float* __restrict__ rstd_out) {
  constexpr int N = 128 * NC;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= M) return;
  const float4* xr = reinterpret_cast<const float4*>(x + row * N);
  float4 v[NC];
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < NC; ++k) {
    v[k] = __ldg(xr + lane + 32 * k);
    s += (v[k].x + v[k].y) + (v[k].z + v[k].w);
  }
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float mean = s / (float)N;
  float q = 0.f;
#pragma unroll
  for (int k = 0; k < NC; ++k) {
    const float a = v[k].x - mean, b = v[k].y - mean, c = v[k].z - mean, d = v[k].w - mean;
    q += (a * a + b * b) + (c * c + d * d);
  }
  for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
  const float rstd = 1.f / sqrtf(q / (float)N + eps);
  float4* yr = reinterpret_cast<float4*>(y + row * N);
#pragma unroll
  for (int k = 0; k < NC; ++k) {
    float4 o = make_float4((v[k].x - mean) * rstd, (v[k].y - mean) * rstd, (v[k].z - mean) * rstd,
                           (v[k].w - mean) * rstd);
    if (gamma) {
      const float4 g = __ldg(reinterpret_cast<const float4*>(gamma) + lane + 32 * k);
      o = make_float4(o.x * g.x, o.y * g.y, o.z * g.z, o.w * g.w);
    }
    if (beta) {
      const float4 b = __ldg(reinterpret_cast<const float4*>(beta) + lane + 32 * k);
      o = make_float4(o.x + b.x, o.y + b.y, o.z + b.z, o.w + b.w);
    }
    yr[lane + 32 * k] = o;
  }
  if (lane == 0) {
    if (mean_out) mean_out[row] = mean;
    if (rstd_out) rstd_out[row] = rstd;
  }
}

// Backward for such rows: CTA b (8 warps) takes rows [b R, (b + 1) R), a warp
// per row; dx = rstd (g - mean(g) - xhat mean(g xhat)) with g = dy gamma, and
// each lane accumulates its columns' dy xhat and dy over the CTA's rows; the
// eight warps' sums are added in warp order into part[b][0 | 1][N]
// (gamma, beta), which ln_bwd_param_final_kernel sums over CTAs in order.
template <int NC>
__global__ void __launch_bounds__(256, NC <= 6 ? 2 : 1) ln_bwd_v4_kernel(const float* __restrict__ dy, const float* __restrict__ x,
                                                           const float* __restrict__ mean,
                                                           const float* __restrict__ rstd,
                                                           const float* __restrict__ gamma, int64_t M, int R,
                                                           float* __restrict__ dx, float* __restrict__ part) {
  constexpr int N = 128 * NC;
  __shared__ float4 acc[2][32 * NC];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float4* g4 = reinterpret_cast<const float4*>(gamma);
  float4 dg[NC], db[NC];
#pragma unroll
  for (int k = 0; k < NC; ++k) dg[k] = db[k] = make_float4(0.f, 0.f, 0.f, 0.f);
  const int64_t r0 = (int64_t)blockIdx.x * R, r1 = min(M, r0 + R);
  for (int64_t row = r0 + warp; row < r1; row += 8) {
    const float4* gr = reinterpret_cast<const float4*>(dy + row * N);
    const float4* xr = reinterpret_cast<const float4*>(x + row * N);
    const float m = __ldg(mean + row), r = __ldg(rstd + row);
    float4 d[NC], v[NC];  // v becomes xhat
    float sg = 0.f, sgx = 0.f;
#pragma unroll
    for (int k = 0; k < NC; ++k) {
      d[k] = __ldg(gr + lane + 32 * k);
      v[k] = __ldg(xr + lane + 32 * k);
      v[k] = make_float4((v[k].x - m) * r, (v[k].y - m) * r, (v[k].z - m) * r, (v[k].w - m) * r);
      dg[k] = make_float4(fmaf(d[k].x, v[k].x, dg[k].x), fmaf(d[k].y, v[k].y, dg[k].y),
                          fmaf(d[k].z, v[k].z, dg[k].z), fmaf(d[k].w, v[k].w, dg[k].w));
      db[k] = make_float4(db[k].x + d[k].x, db[k].y + d[k].y, db[k].z + d[k].z, db[k].w + d[k].w);
      const float4 gm = gamma ? __ldg(g4 + lane + 32 * k) : make_float4(1.f, 1.f, 1.f, 1.f);
      d[k] = make_float4(d[k].x * gm.x, d[k].y * gm.y, d[k].z * gm.z, d[k].w * gm.w);  // d becomes g
      sg += (d[k].x + d[k].y) + (d[k].z + d[k].w);
      sgx += (d[k].x * v[k].x + d[k].y * v[k].y) + (d[k].z * v[k].z + d[k].w * v[k].w);
    }
    for (int o = 16; o > 0; o >>= 1) {
      sg += __shfl_xor_sync(0xffffffffu, sg, o);
      sgx += __shfl_xor_sync(0xffffffffu, sgx, o);
    }
    if (dx) {
      const float a = sg / (float)N, b = sgx / (float)N;
      float4* o = reinterpret_cast<float4*>(dx + row * N);
#pragma unroll
      for (int k = 0; k < NC; ++k)
        o[lane + 32 * k] = make_float4(r * (d[k].x - a - v[k].x * b), r * (d[k].y - a - v[k].y * b),
                                       r * (d[k].z - a - v[k].z * b), r * (d[k].w - a - v[k].w * b));
    }
  }
  if (!part) return;
  for (int w = 0; w < 8; ++w) {
    if (warp == w) {
#pragma unroll
      for (int k = 0; k < NC; ++k) {
        float4& a = acc[0][lane + 32 * k];
        float4& b = acc[1][lane + 32 * k];
        if (w == 0) {
          a = dg[k];
          b = db[k];
        } else {
          a = make_float4(a.x + dg[k].x, a.y + dg[k].y, a.z + dg[k].z, a.w + dg[k].w);
          b = make_float4(b.x + db[k].x, b.y + db[k].y, b.z + db[k].z, b.w + db[k].w);
        }
      }
    }
    __syncthreads();
  }
  float4* pg = reinterpret_cast<float4*>(part + ((int64_t)blockIdx.x * 2) * N);
  for (int i = threadIdx.x; i < 32 * NC; i += blockDim.x) {
    pg[i] = acc[0][i];
    pg[32 * NC + i] = acc[1][i];
  }
}

// rows per CTA of ln_bwd_v4_kernel: about two CTAs per SM, a multiple of 8
static int ln_bwd_rows(int64_t M) {
  int64_t r = (M + 2 * num_sms() - 1) / (2 * num_sms());
  r = (r + 7) / 8 * 8;
  return (int)std::max<int64_t>(r, 8);
}
static bool ln_vec_ok(int64_t N, std::initializer_list<const void*> ptrs) {
  if (N % 128 != 0 || N > 1024) return false;
  for (const void* p : ptrs)
    if (p && ((uintptr_t)p & 15)) return false;
  return true;
}

static int ln_splits(int64_t M) {
  int64_t s = (M + 63) / 64;
  if (s > 256) s = 256;
  if (s < 1) s = 1;
  return (int)s;
}

static int check_bn_x(const pvb2_tensor* x) {
  PVB2_CHECK_ARG(x->dtype == PVB2_F32, "batch_norm: only float32 is supported");
  PVB2_CHECK_ARG(x->ndim >= 2, "batch_norm: input must have >= 2 dims");
  PVB2_CHECK_ARG(is_contiguous(x), "batch_norm: input must be NCHW-contiguous");
  return PVB2_OK;
}

// Fixed scratch of the allocation-free batch-norm forward: a file-scope
// device array (every GPU that loads the library holds its own copy until the
// process exits).  In host code the symbol is only a host-side handle, never
// a device address; the device address comes from cudaGetSymbolAddress,
// looked up once per device with that device current.
static __device__ __align__(256) float g_bn_scratch[PVB2_BN_NOALLOC_SCRATCH_BYTES / sizeof(float)];

static int bn_scratch_address(float** out) {
  static std::mutex m;
  static float* addr[64] = {nullptr};
  int dev = 0;
  PVB2_CUDA_TRY(cudaGetDevice(&dev));
  PVB2_CHECK_ARG(dev >= 0 && dev < 64, "batch_norm_noalloc: device index %d out of range", dev);
  std::lock_guard<std::mutex> g(m);
  if (!addr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_bn_scratch);
    if (e != cudaSuccess || !p)
      return fail(PVB2_ERR_CUDA, "batch_norm_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
                  cudaGetErrorString(e));
    addr[dev] = (float*)p;
  }
  *out = addr[dev];
  return PVB2_OK;
}

}  // namespace pvb2

using namespace pvb2;

extern "C" {

size_t pvb2_batch_norm_workspace_size(const pvb2_tensor* x) {
  if (x->ndim < 2) return 0;
  BnGeom g = bn_geom(x);
  size_t need = (size_t)g.C * g.splits * 2 * sizeof(float);
  if (bn_streamable(g)) need = std::max(need, (size_t)g.C * bn_stream_plan(g, nullptr, 0).splits * 2 * sizeof(float));
  return need;
}

int pvb2_batch_norm_fwd_train(const pvb2_tensor* x, const float* gamma, const float* beta, float* running_mean,
                              float* running_var, double momentum, double eps, const pvb2_tensor* y, float* save_mean,
                              float* save_invstd, void* workspace, size_t workspace_bytes, pvb2_stream stream) {
  PVB2_TRY(check_bn_x(x));
  PVB2_CHECK_ARG(is_contiguous(y) && y->dtype == PVB2_F32, "batch_norm: output must be contiguous float32");
  BnGeom g = bn_geom(x);
  if (g.N * g.HW == 0 || g.C == 0) return PVB2_OK;
  cudaStream_t s = as_stream(stream);
  if (bn_streamable(g)) {
    const void* ptrs[2] = {x->data, y->data};
    const BnStream p = bn_stream_plan(g, ptrs, 2);
    const size_t need = (size_t)g.C * p.splits * 2 * sizeof(float);
    PVB2_CHECK_ARG(workspace && workspace_bytes >= need, "batch_norm: workspace too small (%zu < %zu)",
                   workspace_bytes, need);
    return bn_fwd_stream(g, p, (const float*)x->data, (float*)y->data, gamma, beta, running_mean, running_var,
                         momentum, eps, save_mean, save_invstd, (float*)workspace, s);
  }
  const size_t need = (size_t)g.C * g.splits * 2 * sizeof(float);
  PVB2_CHECK_ARG(workspace && workspace_bytes >= need, "batch_norm: workspace too small (%zu < %zu)",
                 workspace_bytes, need);
  float* part = (float*)workspace;
  bn_stats_kernel<<<dim3((unsigned)g.C, (unsigned)g.splits), kBnThreads, 0, s>>>(
      (const float*)x->data, g.N, g.C, g.HW, g.planes_per, g.splits, part);
  PVB2_LAUNCH_CHECK();
  int threads = g.HW >= 1024 ? 256 : (g.HW >= 256 ? 128 : 64);
  bn_apply_kernel<<<(unsigned)(g.N * g.C), threads, 0, s>>>((const float*)x->data, (float*)y->data, g.N, g.C, g.HW,
                                                            g.splits, part, gamma, beta, running_mean, running_var,
                                                            (float)momentum, (float)eps, save_mean, save_invstd);
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

int pvb2_batch_norm_fwd_split_ok(const pvb2_tensor* x) {
  if (!x || x->ndim < 2 || x->dtype != PVB2_F32 || !is_contiguous(x)) return 0;
  const BnGeom g = bn_geom(x);
  return g.N * g.HW > 0 && g.C > 0 && bn_streamable(g) ? 1 : 0;
}

int pvb2_batch_norm_fwd_stats(const pvb2_tensor* x, void* workspace, size_t workspace_bytes, pvb2_stream stream) {
  return pvb2_batch_norm_fwd_stats_count(x, workspace, workspace_bytes, nullptr, stream);
}

int pvb2_batch_norm_fwd_stats_count(const pvb2_tensor* x, void* workspace, size_t workspace_bytes, int64_t* counter,
                                    pvb2_stream stream) {
  PVB2_TRY(check_bn_x(x));
  PVB2_CHECK_ARG(pvb2_batch_norm_fwd_split_ok(x), "batch_norm: input not supported by the split forward");
  const BnGeom g = bn_geom(x);
  const void* ptrs[1] = {x->data};
  const BnStream p = bn_stream_plan(g, ptrs, 1);
  const size_t need = (size_t)g.C * p.splits * 2 * sizeof(float);
  PVB2_CHECK_ARG(workspace && workspace_bytes >= need, "batch_norm: workspace too small (%zu < %zu)", workspace_bytes,
                 need);
  const dim3 grid((unsigned)p.splits, (unsigned)g.C);
  bn_st_stats_kernel<<<grid, kBnStThreads, 0, as_stream(stream)>>>((const float*)x->data, (int)g.N, (int)g.C,
                                                                  (int)g.HW, p.chunk, p.splits, p.vec ? 1 : 0,
                                                                  (float*)workspace, (long long*)counter);
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

int pvb2_batch_norm_fwd_apply(const pvb2_tensor* x, const float* gamma, const float* beta, float* running_mean,
                              float* running_var, double momentum, double eps, const pvb2_tensor* y,
                              float* save_mean, float* save_invstd, const pvb2_tensor* residual, int act,
                              const pvb2_tensor* sum_out, const void* workspace, size_t workspace_bytes,
                              pvb2_stream stream) {
  return pvb2_batch_norm_fwd_apply_ab(x, gamma, beta, running_mean, running_var, momentum, eps, y, save_mean,
                                      save_invstd, residual, act, sum_out, workspace, workspace_bytes, nullptr,
                                      stream);
}

int pvb2_batch_norm_fwd_apply_ab(const pvb2_tensor* x, const float* gamma, const float* beta, float* running_mean,
                                 float* running_var, double momentum, double eps, const pvb2_tensor* y,
                                 float* save_mean, float* save_invstd, const pvb2_tensor* residual, int act,
                                 const pvb2_tensor* sum_out, const void* workspace, size_t workspace_bytes,
                                 float* ab_out, pvb2_stream stream) {
  PVB2_TRY(check_bn_x(x));
  PVB2_CHECK_ARG(act >= 0 && act <= 2, "batch_norm: activation %d is not 0 (none), 1 (ReLU) or 2 (ReLU6)", act);
  PVB2_CHECK_ARG(pvb2_batch_norm_fwd_split_ok(x), "batch_norm: input not supported by the split forward");
  PVB2_CHECK_ARG(is_contiguous(y) && y->dtype == PVB2_F32 && numel(y) == numel(x),
                 "batch_norm: output must be contiguous float32 of the input's size");
  if (residual) {
    PVB2_CHECK_ARG(is_contiguous(residual) && residual->dtype == PVB2_F32 && residual->ndim == x->ndim,
                   "batch_norm: residual must be contiguous float32 of the input's shape");
    for (int d = 0; d < x->ndim; ++d)
      PVB2_CHECK_ARG(residual->sizes[d] == x->sizes[d], "batch_norm: residual shape differs at dim %d", d);
  }
  if (sum_out) {
    PVB2_CHECK_ARG(is_contiguous(sum_out) && sum_out->dtype == PVB2_F32 && numel(sum_out) == numel(x),
                   "batch_norm: sum_out must be contiguous float32 of the input's size");
  }
  const BnGeom g = bn_geom(x);
  const void* ptrs[4] = {x->data, y->data, residual ? residual->data : nullptr, sum_out ? sum_out->data : nullptr};
  const BnStream p = bn_stream_plan(g, ptrs, 4);
  const size_t need = (size_t)g.C * p.splits * 2 * sizeof(float);
  PVB2_CHECK_ARG(workspace && workspace_bytes >= need, "batch_norm: workspace too small (%zu < %zu)", workspace_bytes,
                 need);
  const dim3 grid((unsigned)p.splits, (unsigned)g.C);
  bn_st_apply_kernel<<<grid, kBnStThreads, 0, as_stream(stream)>>>(
      (const float*)x->data, (float*)y->data, (int)g.N, (int)g.C, (int)g.HW, p.chunk, p.splits, p.vec ? 1 : 0,
      (const float*)workspace, gamma, beta, running_mean, running_var, (float)momentum, (float)eps, save_mean,
      save_invstd, residual ? (const float*)residual->data : nullptr, act,
      sum_out ? (float*)sum_out->data : nullptr, ab_out);
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

// Allocation-free variant of pvb2_batch_norm_fwd_train for callers that
// cannot allocate device memory when they call (inside stream capture, or
// when every device byte belongs to another allocator).  The per-CTA partial
// sums live in g_bn_scratch below instead of a caller workspace.  Every
// partial slot the apply kernel reads is written by the stats kernel of the
// same call, so nothing in the array has to be cleared between calls; it
// simply keeps the last call's partials.  Calls that overlap on the GPU
// share the array and race.
int pvb2_batch_norm_fwd_train_noalloc(const pvb2_tensor* x, const float* gamma, const float* beta,
                                      float* running_mean, float* running_var, double momentum, double eps,
                                      const pvb2_tensor* y, float* save_mean, float* save_invstd,
                                      pvb2_stream stream) {
  PVB2_TRY(check_bn_x(x));
  PVB2_CHECK_ARG(is_contiguous(y) && y->dtype == PVB2_F32, "batch_norm: output must be contiguous float32");
  BnGeom g = bn_geom(x);
  if (g.N * g.HW == 0 || g.C == 0) return PVB2_OK;
  if (bn_streamable(g)) {
    const void* ptrs[2] = {x->data, y->data};
    const BnStream p = bn_stream_plan(g, ptrs, 2);
    const size_t need = (size_t)g.C * p.splits * 2 * sizeof(float);
    PVB2_CHECK_ARG(need <= sizeof(g_bn_scratch),
                   "batch_norm_noalloc: %lld channels x %d splits need %zu bytes of partials, more than the "
                   "%zu-byte scratch; use pvb2_batch_norm_fwd_train with a workspace",
                   (long long)g.C, p.splits, need, sizeof(g_bn_scratch));
    float* part = nullptr;
    PVB2_TRY(bn_scratch_address(&part));
    return bn_fwd_stream(g, p, (const float*)x->data, (float*)y->data, gamma, beta, running_mean, running_var,
                         momentum, eps, save_mean, save_invstd, part, as_stream(stream));
  }
  const size_t need = (size_t)g.C * g.splits * 2 * sizeof(float);
  PVB2_CHECK_ARG(need <= sizeof(g_bn_scratch),
                 "batch_norm_noalloc: %lld channels x %d splits need %zu bytes of partials, more than the "
                 "%zu-byte scratch; use pvb2_batch_norm_fwd_train with a workspace",
                 (long long)g.C, g.splits, need, sizeof(g_bn_scratch));
  float* part = nullptr;
  PVB2_TRY(bn_scratch_address(&part));
  cudaStream_t s = as_stream(stream);
  bn_stats_kernel<<<dim3((unsigned)g.C, (unsigned)g.splits), kBnThreads, 0, s>>>(
      (const float*)x->data, g.N, g.C, g.HW, g.planes_per, g.splits, part);
  PVB2_LAUNCH_CHECK();
  int threads = g.HW >= 1024 ? 256 : (g.HW >= 256 ? 128 : 64);
  bn_apply_kernel<<<(unsigned)(g.N * g.C), threads, 0, s>>>((const float*)x->data, (float*)y->data, g.N, g.C, g.HW,
                                                            g.splits, part, gamma, beta, running_mean, running_var,
                                                            (float)momentum, (float)eps, save_mean, save_invstd);
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

int pvb2_batch_norm_fwd_eval(const pvb2_tensor* x, const float* gamma, const float* beta, const float* running_mean,
                             const float* running_var, double eps, const pvb2_tensor* y, pvb2_stream stream) {
  PVB2_TRY(check_bn_x(x));
  PVB2_CHECK_ARG(running_mean && running_var, "batch_norm eval: running stats required");
  BnGeom g = bn_geom(x);
  if (g.N * g.HW * g.C == 0) return PVB2_OK;
  int threads = g.HW >= 1024 ? 256 : (g.HW >= 256 ? 128 : 64);
  bn_eval_kernel<<<(unsigned)(g.N * g.C), threads, 0, as_stream(stream)>>>(
      (const float*)x->data, (float*)y->data, g.C, g.HW, gamma, beta, running_mean, running_var, (float)eps);
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

int pvb2_batch_norm_bwd(const pvb2_tensor* dy, const pvb2_tensor* x, const float* gamma, const float* mean,
                        const float* invstd, int train, const pvb2_tensor* dx, float* dgamma, float* dbeta,
                        void* workspace, size_t workspace_bytes, pvb2_stream stream) {
  PVB2_TRY(check_bn_x(x));
  PVB2_CHECK_ARG(is_contiguous(dy), "batch_norm_backward: grad must be contiguous");
  BnGeom g = bn_geom(x);
  if (g.C == 0) return PVB2_OK;
  cudaStream_t s = as_stream(stream);
  int threads = g.HW >= 1024 ? 256 : (g.HW >= 256 ? 128 : 64);
  if (!train) {
    // `mean` is unused; `invstd` carries running_var and the eps is folded
    // by the caller into running_var (var + eps passed as var, eps = 0).
    PVB2_CHECK_ARG(false, "batch_norm_backward: use pvb2_batch_norm_bwd_eval for eval mode");
  }
  if (g.N * g.HW == 0) {
    if (dgamma) PVB2_CUDA_TRY(cudaMemsetAsync(dgamma, 0, g.C * sizeof(float), s));
    if (dbeta) PVB2_CUDA_TRY(cudaMemsetAsync(dbeta, 0, g.C * sizeof(float), s));
    return PVB2_OK;
  }
  if (bn_streamable(g)) {
    const void* ptrs[3] = {dy->data, x->data, dx ? dx->data : nullptr};
    const BnStream p = bn_stream_plan(g, ptrs, 3);
    const size_t need = (size_t)g.C * p.splits * 2 * sizeof(float);
    PVB2_CHECK_ARG(workspace && workspace_bytes >= need, "batch_norm_backward: workspace too small");
    return bn_bwd_stream(g, p, (const float*)dy->data, (const float*)x->data, mean, invstd, gamma,
                         dx ? (float*)dx->data : nullptr, dgamma, dbeta, (float*)workspace, s);
  }
  const size_t need = (size_t)g.C * g.splits * 2 * sizeof(float);
  PVB2_CHECK_ARG(workspace && workspace_bytes >= need, "batch_norm_backward: workspace too small");
  float* part = (float*)workspace;
  bn_bwd_reduce_kernel<<<dim3((unsigned)g.C, (unsigned)g.splits), kBnThreads, 0, s>>>(
      (const float*)dy->data, (const float*)x->data, mean, g.N, g.C, g.HW, g.planes_per, g.splits, part);
  PVB2_LAUNCH_CHECK();
  bn_bwd_apply_kernel<<<(unsigned)(g.N * g.C), threads, 0, s>>>(
      (const float*)dy->data, (const float*)x->data, mean, invstd, gamma, g.N, g.C, g.HW, g.splits, part,
      dx ? (float*)dx->data : nullptr, dgamma, dbeta);
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

int pvb2_batch_norm_bwd_relu(const pvb2_tensor* grad_above, const pvb2_tensor* relu_out, const pvb2_tensor* x,
                             const float* gamma, const float* mean, const float* invstd, const pvb2_tensor* dy,
                             const pvb2_tensor* dx, float* dgamma, float* dbeta, void* workspace,
                             size_t workspace_bytes, pvb2_stream stream) {
  return pvb2_batch_norm_bwd_act(1, grad_above, relu_out, x, gamma, mean, invstd, dy, dx, dgamma, dbeta, workspace,
                                 workspace_bytes, stream);
}

int pvb2_batch_norm_bwd_act(int act, const pvb2_tensor* grad_above, const pvb2_tensor* relu_out,
                            const pvb2_tensor* x, const float* gamma, const float* mean, const float* invstd,
                            const pvb2_tensor* dy, const pvb2_tensor* dx, float* dgamma, float* dbeta,
                            void* workspace, size_t workspace_bytes, pvb2_stream stream) {
  PVB2_CHECK_ARG(act == 1 || act == 2, "batch_norm_backward: activation %d is not 1 (ReLU) or 2 (ReLU6)", act);
  PVB2_TRY(check_bn_x(x));
  for (const pvb2_tensor* t : {grad_above, relu_out, dy}) {
    PVB2_CHECK_ARG(t && is_contiguous(t) && t->dtype == PVB2_F32 && numel(t) == numel(x),
                   "batch_norm_backward_relu: gradients and ReLU output must be contiguous float32 like x");
  }
  PVB2_CHECK_ARG(pvb2_batch_norm_fwd_split_ok(x), "batch_norm_backward_relu: input not supported");
  const BnGeom g = bn_geom(x);
  const void* ptrs[5] = {grad_above->data, relu_out->data, x->data, dy->data, dx ? dx->data : nullptr};
  const BnStream p = bn_stream_plan(g, ptrs, 5);
  const size_t need = (size_t)g.C * p.splits * 2 * sizeof(float);
  PVB2_CHECK_ARG(workspace && workspace_bytes >= need, "batch_norm_backward: workspace too small");
  return bn_bwd_stream(g, p, (const float*)grad_above->data, (const float*)x->data, mean, invstd, gamma,
                       dx ? (float*)dx->data : nullptr, dgamma, dbeta, (float*)workspace, as_stream(stream),
                       (const float*)relu_out->data, (float*)dy->data, act);
}

int pvb2_batch_norm_bwd_act_ab(int act, const pvb2_tensor* grad_above, const pvb2_tensor* x, const float* ab,
                               const float* gamma, const float* mean, const float* invstd, const pvb2_tensor* dy,
                               const pvb2_tensor* dx, float* dgamma, float* dbeta, void* workspace,
                               size_t workspace_bytes, pvb2_stream stream) {
  PVB2_CHECK_ARG(act == 1 || act == 2, "batch_norm_backward: activation %d is not 1 (ReLU) or 2 (ReLU6)", act);
  PVB2_CHECK_ARG(ab != nullptr, "batch_norm_backward_act_ab: the forward's (a, b) are required");
  PVB2_TRY(check_bn_x(x));
  for (const pvb2_tensor* t : {grad_above, dy}) {
    PVB2_CHECK_ARG(!t || (is_contiguous(t) && t->dtype == PVB2_F32 && numel(t) == numel(x)),
                   "batch_norm_backward_act_ab: gradients must be contiguous float32 like x");
  }
  PVB2_CHECK_ARG(grad_above != nullptr, "batch_norm_backward_act_ab: grad_above is required");
  PVB2_CHECK_ARG(pvb2_batch_norm_fwd_split_ok(x), "batch_norm_backward_act_ab: input not supported");
  const BnGeom g = bn_geom(x);
  const void* ptrs[4] = {grad_above->data, x->data, dy ? dy->data : nullptr, dx ? dx->data : nullptr};
  const BnStream p = bn_stream_plan(g, ptrs, 4);
  const size_t need = (size_t)g.C * p.splits * 2 * sizeof(float);
  PVB2_CHECK_ARG(workspace && workspace_bytes >= need, "batch_norm_backward: workspace too small");
  return bn_bwd_stream(g, p, (const float*)grad_above->data, (const float*)x->data, mean, invstd, gamma,
                       dx ? (float*)dx->data : nullptr, dgamma, dbeta, (float*)workspace, as_stream(stream), nullptr,
                       dy ? (float*)dy->data : nullptr, act, ab);
}

int pvb2_batch_norm_bwd_eval(const pvb2_tensor* dy, const float* gamma, const float* running_var, double eps,
                             const pvb2_tensor* dx, pvb2_stream stream) {
  PVB2_CHECK_ARG(dy->dtype == PVB2_F32 && is_contiguous(dy) && is_contiguous(dx), "batch_norm_backward eval: layout");
  BnGeom g = bn_geom(dy);
  if (g.N * g.HW * g.C == 0) return PVB2_OK;
  int threads = g.HW >= 1024 ? 256 : (g.HW >= 256 ? 128 : 64);
  bn_bwd_eval_kernel<<<(unsigned)(g.N * g.C), threads, 0, as_stream(stream)>>>(
      (const float*)dy->data, running_var, gamma, (float)eps, g.C, g.HW, (float*)dx->data);
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

int pvb2_layer_norm_fwd(const float* x, const float* gamma, const float* beta, int64_t M, int64_t N, double eps,
                        float* y, float* mean, float* rstd, pvb2_stream stream) {
  if (M == 0) return PVB2_OK;
  PVB2_CHECK_ARG(N > 0, "layer_norm: N must be positive");
  cudaStream_t s = as_stream(stream);
  if (ln_vec_ok(N, {x, gamma, beta, y})) {
    const unsigned grid = (unsigned)((M + 7) / 8);
    switch (N / 128) {
#define LN_FWD(NC) \
  case NC: ln_fwd_v4_kernel<NC><<<grid, 256, 0, s>>>(x, gamma, beta, M, (float)eps, y, mean, rstd); break;
      LN_FWD(1) LN_FWD(2) LN_FWD(3) LN_FWD(4) LN_FWD(5) LN_FWD(6) LN_FWD(7) LN_FWD(8)
#undef LN_FWD
    }
  } else if (N <= 32 * kLnMaxPerLane) {
    const int warps = 8;
    ln_fwd_kernel<<<(unsigned)((M + warps - 1) / warps), warps * 32, 0, s>>>(x, gamma, beta, M, N, (float)eps, y,
                                                                            mean, rstd);
  } else {
    ln_fwd_big_kernel<<<(unsigned)M, 256, 0, s>>>(x, gamma, beta, M, N, (float)eps, y, mean, rstd);
  }
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

size_t pvb2_layer_norm_bwd_workspace_size(int64_t M, int64_t N) {
  const int64_t ctas = (M + ln_bwd_rows(M) - 1) / ln_bwd_rows(M);
  return (size_t)std::max<int64_t>(ln_splits(M), ctas) * 2 * (size_t)N * sizeof(float);
}

int pvb2_layer_norm_bwd(const float* dy, const float* x, const float* mean, const float* rstd, const float* gamma,
                        int64_t M, int64_t N, float* dx, float* dgamma, float* dbeta, void* workspace,
                        size_t workspace_bytes, pvb2_stream stream) {
  cudaStream_t s = as_stream(stream);
  if (M == 0) {
    if (dgamma) PVB2_CUDA_TRY(cudaMemsetAsync(dgamma, 0, N * sizeof(float), s));
    if (dbeta) PVB2_CUDA_TRY(cudaMemsetAsync(dbeta, 0, N * sizeof(float), s));
    return PVB2_OK;
  }
  if (ln_vec_ok(N, {dy, x, gamma, dx, workspace}) && M < ((int64_t)1 << 31)) {
    const int R = ln_bwd_rows(M);
    const int64_t ctas = (M + R - 1) / R;
    const bool params = dgamma || dbeta;
    PVB2_CHECK_ARG(!params || (workspace && workspace_bytes >= (size_t)ctas * 2 * N * sizeof(float)),
                   "layer_norm_backward: workspace too small");
    float* part = params ? (float*)workspace : nullptr;
    switch (N / 128) {
#define LN_BWD(NC) \
  case NC: ln_bwd_v4_kernel<NC><<<(unsigned)ctas, 256, 0, s>>>(dy, x, mean, rstd, gamma, M, R, dx, part); break;
      LN_BWD(1) LN_BWD(2) LN_BWD(3) LN_BWD(4) LN_BWD(5) LN_BWD(6) LN_BWD(7) LN_BWD(8)
#undef LN_BWD
    }
    PVB2_LAUNCH_CHECK();
    if (params) {
      ln_bwd_param_final_kernel<<<(unsigned)((N + 255) / 256), 256, 0, s>>>(part, (int)ctas, N, dgamma, dbeta);
      PVB2_LAUNCH_CHECK();
    }
    return PVB2_OK;
  }
  if (dx) {
    ln_bwd_dx_kernel<<<(unsigned)M, 256, 0, s>>>(dy, x, mean, rstd, gamma, N, dx);
    PVB2_LAUNCH_CHECK();
  }
  if (dgamma || dbeta) {
    const int splits = ln_splits(M);
    const size_t need = (size_t)splits * 2 * N * sizeof(float);
    PVB2_CHECK_ARG(workspace && workspace_bytes >= need, "layer_norm_backward: workspace too small");
    const int64_t rows_per = (M + splits - 1) / splits;
    float* part = (float*)workspace;
    dim3 grid((unsigned)((N + 127) / 128), (unsigned)splits);
    ln_bwd_param_partial_kernel<<<grid, 128, 0, s>>>(dy, x, mean, rstd, M, N, rows_per, part);
    PVB2_LAUNCH_CHECK();
    ln_bwd_param_final_kernel<<<(unsigned)((N + 255) / 256), 256, 0, s>>>(part, splits, N, dgamma, dbeta);
    PVB2_LAUNCH_CHECK();
  }
  return PVB2_OK;
}

}  // extern "C"
