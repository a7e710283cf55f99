// Batch norm and layer norm, forward and backward.
//
// Replaces dlprim::core::BatchNormFwdBwd as driven by native_batch_norm /
// native_batch_norm_backward (src/norm_ops.cpp:19-164) and the
// batch-norm-over-(1,B,N) trick the reference used for layer norm
// (norm_ops.cpp:167-351).
//
// Training batch norm on NCHW-contiguous x whose channels each fit the shared
// memory of one thread-block cluster (<= 8 CTAs, up to 1.7 MB of fp32 per
// channel in the forward, 0.85 MB per tensor in the backward) runs as ONE
// cluster-resident launch that reads its inputs once (bn_fwd_cluster_kernel,
// bn_bwd_cluster_kernel below).  Larger channels run as two launches:
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
#include <cooperative_groups.h>
#include <mutex>
#include "common.cuh"

namespace cg = cooperative_groups;

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

// ------------------------------------------- batch norm, cluster-resident
// When one channel's data fits the shared memory of a thread-block cluster
// (<= 8 CTAs), the training forward and backward each read their inputs from
// HBM once: grid (k, C) with clusters of k CTAs along x, CTA r of channel c
// holds elements [r*chunk, (r+1)*chunk) of the channel's (n, hw) range in
// shared memory, partial sums meet through distributed shared memory, and
// the output is written from the resident copy.  Each CTA reduces its own
// elements first (the forward in two passes over shared memory: mean, then
// squared deviations), one cluster barrier publishes the per-CTA results,
// and every CTA combines them in double in rank order (the forward with
// Chan's pairwise formula for (count, mean, M2)).
constexpr int kBnClThreads = 512;
constexpr int kBnClMaxCluster = 8;
constexpr int kBnClSmallBytes = 110 * 1024;  // two CTAs per SM
constexpr int kBnClBigBytes = 220 * 1024;    // one CTA per SM

// sum over the block; every thread gets the result
__device__ __forceinline__ float block_allsum(float v, float* red) {
  v = warp_sum(v);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  __syncthreads();  // red may still be read by a previous call
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float t = 0.f;
  const int nw = blockDim.x >> 5;
  for (int i = 0; i < nw; ++i) t += red[i];
  return t;
}

// split cluster barrier: arrive (release) once this CTA's distributed
// shared-memory reads are done, wait (acquire) before leaving
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }

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

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Start asynchronous copies of this CTA's elements [start, end) of channel c
// into shared memory (16-byte copies when vec: HW % 4 == 0 and aligned).
// The caller waits with cp_async_wait_all + __syncthreads.
__device__ __forceinline__ void bn_cl_load(const float* __restrict__ src, float* __restrict__ dst, int start, int end,
                                           int HW, int64_t nstride, bool vec) {
  const int vw = vec ? 4 : 1;
  const int step = vw * blockDim.x;
  int e = start + vw * threadIdx.x;
  if (e >= end) return;
  ChanWalk w(e, step, HW);
  if (vec) {
    for (; e < end; e += step, w.next()) cp_async16(dst + (e - start), src + w.n * nstride + w.i);
  } else {
    for (; e < end; e += step, w.next()) cp_async4(dst + (e - start), src + w.n * nstride + w.i);
  }
}

__global__ void __launch_bounds__(kBnClThreads) bn_fwd_cluster_kernel(
    const float* __restrict__ x, float* __restrict__ y, int N, int C, int HW, int chunk, int vec,
    const float* __restrict__ gamma, const float* __restrict__ beta, float* __restrict__ running_mean,
    float* __restrict__ running_var, float momentum, float eps, float* __restrict__ save_mean,
    float* __restrict__ save_invstd) {
  extern __shared__ __align__(16) float sx[];
  __shared__ float red[32];
  __shared__ float cl_part[3];  // count, mean, M2 of this CTA's elements
  __shared__ float s_coef[2];
  cg::cluster_group cl = cg::this_cluster();
  const int r = (int)cl.block_rank(), k = (int)cl.num_blocks();
  const int c = blockIdx.y;
  const int M = N * HW;
  const int start = r * chunk, end = min(M, start + chunk), len = max(0, end - start);
  const int64_t nstride = (int64_t)C * HW;
  bn_cl_load(x + (int64_t)c * HW, sx, start, end, HW, nstride, vec != 0);
  cp_async_wait_all();
  __syncthreads();
  // this CTA's mean and sum of squared deviations: two passes over shared memory
  float s = 0.f;
  for (int i = threadIdx.x; i < len; i += blockDim.x) s += sx[i];
  const float lmean = len ? block_allsum(s, red) / (float)len : 0.f;
  float s2 = 0.f;
  for (int i = threadIdx.x; i < len; i += blockDim.x) {
    const float d = sx[i] - lmean;
    s2 += d * d;
  }
  s2 = block_allsum(s2, red);
  if (threadIdx.x == 0) {
    cl_part[0] = (float)len;
    cl_part[1] = lmean;
    cl_part[2] = s2;
  }
  cl.sync();
  if (threadIdx.x == 0) {
    // Chan's pairwise combination, in double, in rank order
    double n = 0.0, mean = 0.0, m2 = 0.0;
    for (int q = 0; q < k; ++q) {
      const float* pq = cl.map_shared_rank(cl_part, q);
      const double nq = pq[0];
      if (nq == 0.0) continue;
      const double nn = n + nq, d = (double)pq[1] - mean;
      mean += d * nq / nn;
      m2 += (double)pq[2] + d * d * n * nq / nn;
      n = nn;
    }
    const double var = m2 / n;
    const float invstd = (float)(1.0 / sqrt(var + (double)eps));
    const float meanf = (float)mean;
    const float g = gamma ? gamma[c] : 1.f;
    const float b = beta ? beta[c] : 0.f;
    const float a = invstd * g;
    s_coef[0] = a;
    s_coef[1] = b - meanf * a;
    if (r == 0) {
      if (save_mean) save_mean[c] = meanf;
      if (save_invstd) save_invstd[c] = invstd;
      if (running_mean) running_mean[c] = (1.f - momentum) * running_mean[c] + momentum * meanf;
      if (running_var) {
        const double unbiased = n > 1.0 ? var * n / (n - 1.0) : var;
        running_var[c] = (1.f - momentum) * running_var[c] + momentum * (float)unbiased;
      }
    }
  }
  cluster_arrive();  // this CTA is done reading its peers' statistics
  __syncthreads();
  const float a = s_coef[0], b = s_coef[1];
  float* yc = y + (int64_t)c * HW;
  const int vw = vec ? 4 : 1, step = vw * blockDim.x;
  int e = start + vw * threadIdx.x;
  if (e < end) {
    ChanWalk w(e, step, HW);
    if (vec) {
      for (; e < end; e += step, w.next()) {
        float4 v = *reinterpret_cast<const float4*>(sx + (e - start));
        v.x = fmaf(v.x, a, b);
        v.y = fmaf(v.y, a, b);
        v.z = fmaf(v.z, a, b);
        v.w = fmaf(v.w, a, b);
        *reinterpret_cast<float4*>(yc + w.n * nstride + w.i) = v;
      }
    } else {
      for (; e < end; e += step, w.next()) yc[w.n * nstride + w.i] = fmaf(sx[e - start], a, b);
    }
  }
  cluster_wait();  // no CTA leaves while a peer may still read its statistics
}

__global__ void __launch_bounds__(kBnClThreads) bn_bwd_cluster_kernel(
    const float* __restrict__ dy, const float* __restrict__ x, const float* __restrict__ mean,
    const float* __restrict__ invstd, const float* __restrict__ gamma, int N, int C, int HW, int chunk, int vec,
    float* __restrict__ dx, float* __restrict__ dgamma, float* __restrict__ dbeta) {
  extern __shared__ __align__(16) float smem_bn[];
  float* sdy = smem_bn;
  float* sx = smem_bn + chunk;
  __shared__ float red[32];
  __shared__ float cl_part[2];
  __shared__ float s_coef[3];
  cg::cluster_group cl = cg::this_cluster();
  const int r = (int)cl.block_rank(), k = (int)cl.num_blocks();
  const int c = blockIdx.y;
  const int M = N * HW;
  const int start = r * chunk, end = min(M, start + chunk), len = max(0, end - start);
  const int64_t nstride = (int64_t)C * HW;
  bn_cl_load(dy + (int64_t)c * HW, sdy, start, end, HW, nstride, vec != 0);
  bn_cl_load(x + (int64_t)c * HW, sx, start, end, HW, nstride, vec != 0);
  cp_async_wait_all();
  __syncthreads();
  const float m = mean[c];
  float s_dy = 0.f, s_dot = 0.f;
  for (int i = threadIdx.x; i < len; i += blockDim.x) {
    const float g = sdy[i];
    s_dy += g;
    s_dot += g * (sx[i] - m);
  }
  s_dy = block_allsum(s_dy, red);
  s_dot = block_allsum(s_dot, red);
  if (threadIdx.x == 0) {
    cl_part[0] = s_dy;
    cl_part[1] = s_dot;
  }
  cl.sync();
  if (threadIdx.x == 0) {
    double sdy_all = 0.0, sdot_all = 0.0;
    for (int q = 0; q < k; ++q) {
      const float* pq = cl.map_shared_rank(cl_part, q);
      sdy_all += (double)pq[0];
      sdot_all += (double)pq[1];
    }
    const double count = (double)M;
    const float is = invstd[c];
    s_coef[0] = (float)(sdy_all / count);              // mean of dy
    s_coef[1] = (float)(sdot_all / count) * is * is;   // dotp * invstd^2 / count
    s_coef[2] = is * (gamma ? gamma[c] : 1.f);
    if (r == 0) {
      if (dgamma) dgamma[c] = (float)sdot_all * is;
      if (dbeta) dbeta[c] = (float)sdy_all;
    }
  }
  cluster_arrive();  // this CTA is done reading its peers' sums
  __syncthreads();
  if (dx) {
    const float gm = s_coef[0], kk = s_coef[1], mul = s_coef[2];
    float* dxc = dx + (int64_t)c * HW;
    const int vw = vec ? 4 : 1, step = vw * blockDim.x;
    int e = start + vw * threadIdx.x;
    if (e < end) {
      ChanWalk w(e, step, HW);
      if (vec) {
        for (; e < end; e += step, w.next()) {
          const float4 g = *reinterpret_cast<const float4*>(sdy + (e - start));
          const float4 v = *reinterpret_cast<const float4*>(sx + (e - start));
          float4 o;
          o.x = (g.x - gm - (v.x - m) * kk) * mul;
          o.y = (g.y - gm - (v.y - m) * kk) * mul;
          o.z = (g.z - gm - (v.z - m) * kk) * mul;
          o.w = (g.w - gm - (v.w - m) * kk) * mul;
          *reinterpret_cast<float4*>(dxc + w.n * nstride + w.i) = o;
        }
      } else {
        for (; e < end; e += step, w.next())
          dxc[w.n * nstride + w.i] = (sdy[e - start] - gm - (sx[e - start] - m) * kk) * mul;
      }
    }
  }
  cluster_wait();  // no CTA leaves while a peer may still read its sums
}

struct BnCluster {
  int k, chunk, smem;
  bool vec;
};

// plan a cluster-resident launch holding `arrays` fp32 tensors per element;
// false when a channel does not fit 8 CTAs' shared memory
static bool bn_cluster_plan(const BnGeom& g, int arrays, const void* const* ptrs, int nptr, BnCluster* p) {
  const int64_t M = g.N * g.HW;
  if (M <= 0 || g.C > 65535 || M > (int64_t)1 << 30) return false;
  bool vec = (g.HW & 3) == 0;
  for (int i = 0; i < nptr; ++i)
    if (ptrs[i] && ((uintptr_t)ptrs[i] & 15)) vec = false;
  for (int budget : {kBnClSmallBytes, kBnClBigBytes}) {
    const int64_t per = budget / (4 * arrays) / 4 * 4;  // elements per CTA, multiple of 4
    const int64_t k = (M + per - 1) / per;
    if (k > kBnClMaxCluster) continue;
    int64_t chunk = (M + k - 1) / k;
    chunk = (chunk + 3) / 4 * 4;
    p->k = (int)k;
    p->chunk = (int)chunk;
    p->smem = (int)(chunk * 4 * arrays);
    p->vec = vec;
    return true;
  }
  return false;
}

// launch configuration of a cluster-resident kernel: grid (k, C), clusters (k, 1, 1)
struct BnClusterLaunch {
  cudaLaunchConfig_t cfg;
  cudaLaunchAttribute attr[1];
  BnClusterLaunch(const BnCluster& p, int C, cudaStream_t s) {
    cfg = cudaLaunchConfig_t{};
    cfg.gridDim = dim3((unsigned)p.k, (unsigned)C, 1);
    cfg.blockDim = dim3(kBnClThreads, 1, 1);
    cfg.dynamicSmemBytes = (size_t)p.smem;
    cfg.stream = s;
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)p.k;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
};

static int bn_fwd_cluster(const BnGeom& g, const BnCluster& p, const float* x, float* y, const float* gamma,
                          const float* beta, float* running_mean, float* running_var, double momentum, double eps,
                          float* save_mean, float* save_invstd, cudaStream_t s) {
  static std::atomic<uint64_t> attr_done{0};
  if (first_on_device(attr_done))
    PVB2_CUDA_TRY(cudaFuncSetAttribute(bn_fwd_cluster_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kBnClBigBytes));
  BnClusterLaunch L(p, (int)g.C, s);
  PVB2_CUDA_TRY(cudaLaunchKernelEx(&L.cfg, bn_fwd_cluster_kernel, x, y, (int)g.N, (int)g.C, (int)g.HW, p.chunk,
                                   p.vec ? 1 : 0, gamma, beta, running_mean, running_var, (float)momentum, (float)eps,
                                   save_mean, save_invstd));
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

static int bn_bwd_cluster(const BnGeom& g, const BnCluster& p, const float* dy, const float* x, const float* mean,
                          const float* invstd, const float* gamma, float* dx, float* dgamma, float* dbeta,
                          cudaStream_t s) {
  static std::atomic<uint64_t> attr_done{0};
  if (first_on_device(attr_done))
    PVB2_CUDA_TRY(cudaFuncSetAttribute(bn_bwd_cluster_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kBnClBigBytes));
  BnClusterLaunch L(p, (int)g.C, s);
  PVB2_CUDA_TRY(cudaLaunchKernelEx(&L.cfg, bn_bwd_cluster_kernel, dy, x, mean, invstd, gamma, (int)g.N, (int)g.C,
                                   (int)g.HW, p.chunk, p.vec ? 1 : 0, dx, dgamma, dbeta));
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
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
  return (size_t)g.C * g.splits * 2 * sizeof(float);
}

int pvb2_batch_norm_fwd_train(const pvb2_tensor* x, const float* gamma, const float* beta, float* running_mean,
                              float* running_var, double momentum, double eps, const pvb2_tensor* y, float* save_mean,
                              float* save_invstd, void* workspace, size_t workspace_bytes, pvb2_stream stream) {
  PVB2_TRY(check_bn_x(x));
  PVB2_CHECK_ARG(is_contiguous(y) && y->dtype == PVB2_F32, "batch_norm: output must be contiguous float32");
  BnGeom g = bn_geom(x);
  if (g.N * g.HW == 0 || g.C == 0) return PVB2_OK;
  cudaStream_t s = as_stream(stream);
  BnCluster cp;
  const void* ptrs[2] = {x->data, y->data};
  if (bn_cluster_plan(g, 1, ptrs, 2, &cp))
    return bn_fwd_cluster(g, cp, (const float*)x->data, (float*)y->data, gamma, beta, running_mean, running_var,
                          momentum, eps, save_mean, save_invstd, s);
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
  BnCluster cp;
  const void* ptrs[2] = {x->data, y->data};
  if (bn_cluster_plan(g, 1, ptrs, 2, &cp))  // needs no scratch at all
    return bn_fwd_cluster(g, cp, (const float*)x->data, (float*)y->data, gamma, beta, running_mean, running_var,
                          momentum, eps, save_mean, save_invstd, as_stream(stream));
  const size_t need = (size_t)g.C * g.splits * 2 * sizeof(float);
  PVB2_CHECK_ARG(need <= sizeof(g_bn_scratch),
                 "batch_norm_noalloc: %lld channels need %zu bytes of partials, more than the %zu-byte scratch; "
                 "use pvb2_batch_norm_fwd_train with a workspace",
                 (long long)g.C, need, sizeof(g_bn_scratch));
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
  BnCluster cp;
  const void* ptrs[3] = {dy->data, x->data, dx ? dx->data : nullptr};
  if (bn_cluster_plan(g, 2, ptrs, 3, &cp))
    return bn_bwd_cluster(g, cp, (const float*)dy->data, (const float*)x->data, mean, invstd, gamma,
                          dx ? (float*)dx->data : nullptr, dgamma, dbeta, s);
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
  if (N <= 32 * kLnMaxPerLane) {
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
  return (size_t)ln_splits(M) * 2 * (size_t)N * sizeof(float);
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
