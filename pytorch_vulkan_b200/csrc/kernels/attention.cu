// Fused scaled-dot-product attention, forward and backward, fp32.
//
// Replaces the math path the reference's ViT attention took: two batched
// GEMMs and a softmax through mm_bmm_out (src/vision_ops.cpp:541-626) and
// _softmax_out / _softmax_backward_data_out (src/loss_ops.cpp:137-213), each
// writing the [B*H, Lq, Lk] score matrix to memory.  Here the scores never
// leave shared memory.
//
// Layout: Q [B, H, Lq, D], K and V [B, H, Lk, D], any strides over (b, h, l),
// unit stride along d.  O [B, H, Lq, D] contiguous, logsumexp [B, H, Lq].
// D is 32, 64 or 128.  No attention mask, no dropout; optional causal mask
// (query i sees keys j <= i).
//
// Forward: one CTA per (64 queries, head); key blocks of 64 stream through
// shared memory with the online softmax (running row max m and sum l, the
// accumulator rescaled by exp(m_old - m_new)).  Thread t owns query row
// t / 4 and, of that row, keys j = t%4 + 4u of each block and output
// columns (t%4)*D/4 .. +D/4; the four threads of a row are adjacent lanes.
// Backward (with D_i = sum_d dO_i,d O_i,d, P_ij = exp(s_ij - lse_i),
// dS_ij = P_ij (dO_i . V_j - D_i)):
//   dK, dV: one CTA per (64 keys, head), looping over query blocks:
//           dV_j += sum_i P_ij dO_i,  dK_j += scale * sum_i dS_ij Q_i
//   dQ:     one CTA per (64 queries, head), looping over key blocks:
//           dQ_i += scale * sum_j dS_ij K_j
// All arithmetic is fp32 on the CUDA cores; the exponentials use expf.
#include <cfloat>
#include "common.cuh"

namespace pvb2 {

constexpr int kAtB = 64;        // rows (queries or keys) per block
constexpr int kAtThreads = 256;

struct AtView {  // one of Q, K, V, O, dO, dQ, dK, dV
  float* p;
  int64_t sb, sh, sl;
};

struct AtArgs {
  int B, H, Lq, Lk;
  float scale;
  int causal;
};

__device__ __forceinline__ const float* at_row(const AtView& v, int b, int h, int l) {
  return v.p + b * v.sb + h * v.sh + (int64_t)l * v.sl;
}
__device__ __forceinline__ float* at_row_w(const AtView& v, int b, int h, int l) {
  return v.p + b * v.sb + h * v.sh + (int64_t)l * v.sl;
}

// rows [l0, l0+64) of a view into shared memory (pitch floats per row),
// scaled, zero past `len`
template <int D>
__device__ __forceinline__ void at_load(float* s, int pitch, const AtView& v, int b, int h, int l0, int len,
                                        float mul) {
  for (int e = threadIdx.x; e < kAtB * (D / 4); e += blockDim.x) {
    const int r = e / (D / 4), c4 = (e % (D / 4)) * 4;
    float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
    if (l0 + r < len) x = __ldg(reinterpret_cast<const float4*>(at_row(v, b, h, l0 + r) + c4));
    float* d = s + r * pitch + c4;
    d[0] = x.x * mul;
    d[1] = x.y * mul;
    d[2] = x.z * mul;
    d[3] = x.w * mul;
  }
}

__device__ __forceinline__ float quad_max(float v) {
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1));
  return fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2));
}
__device__ __forceinline__ float quad_sum(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 1);
  return v + __shfl_xor_sync(0xffffffffu, v, 2);
}

template <int D>
struct AtFwdSmem {
  static constexpr int PQ = D + 1, PK = D + 1, PV = D + 4, PP = kAtB + 1;
  static constexpr int Q = 0, K = Q + kAtB * PQ, V = K + kAtB * PK, P = V + kAtB * PV;
  static constexpr int FLOATS = P + kAtB * PP;
};

template <int D>
__global__ void __launch_bounds__(kAtThreads) sdpa_fwd_kernel(AtView q, AtView k, AtView v, AtView o,
                                                              float* __restrict__ lse, AtArgs a) {
  using L = AtFwdSmem<D>;
  constexpr int DC = D / 4;
  extern __shared__ __align__(16) float at_smem[];
  float* Qs = at_smem + L::Q;
  float* Ks = at_smem + L::K;
  float* Vs = at_smem + L::V;
  float* Ps = at_smem + L::P;
  const int bh = blockIdx.y, b = bh / a.H, h = bh % a.H;
  const int q0 = blockIdx.x * kAtB;
  const int r = threadIdx.x >> 2, g = threadIdx.x & 3;
  const int qi = q0 + r;
  at_load<D>(Qs, L::PQ, q, b, h, q0, a.Lq, a.scale);
  float acc[DC];
#pragma unroll
  for (int e = 0; e < DC; ++e) acc[e] = 0.f;
  float m = -FLT_MAX, l = 0.f;
  const int kend = a.causal ? min(a.Lk, q0 + kAtB) : a.Lk;
  for (int k0 = 0; k0 < kend; k0 += kAtB) {
    __syncthreads();  // previous block's K / V / P no longer read
    at_load<D>(Ks, L::PK, k, b, h, k0, a.Lk, 1.f);
    at_load<D>(Vs, L::PV, v, b, h, k0, a.Lk, 1.f);
    __syncthreads();
    float s[16];
#pragma unroll
    for (int u = 0; u < 16; ++u) s[u] = 0.f;
    for (int d = 0; d < D; ++d) {
      const float qd = Qs[r * L::PQ + d];
#pragma unroll
      for (int u = 0; u < 16; ++u) s[u] = fmaf(qd, Ks[(g + 4 * u) * L::PK + d], s[u]);
    }
    float mx = -FLT_MAX;
#pragma unroll
    for (int u = 0; u < 16; ++u) {
      const int kj = k0 + g + 4 * u;
      const bool ok = kj < a.Lk && !(a.causal && kj > qi);
      s[u] = ok ? s[u] : -FLT_MAX;
      mx = fmaxf(mx, s[u]);
    }
    mx = quad_max(mx);
    const float mnew = fmaxf(m, mx);
    const float alpha = expf(m - mnew);
    float ps = 0.f;
#pragma unroll
    for (int u = 0; u < 16; ++u) {
      const float p = s[u] == -FLT_MAX ? 0.f : expf(s[u] - mnew);
      Ps[r * L::PP + g + 4 * u] = p;
      ps += p;
    }
    l = l * alpha + quad_sum(ps);
    m = mnew;
#pragma unroll
    for (int e = 0; e < DC; ++e) acc[e] *= alpha;
    __syncwarp();  // the row's probabilities come from the four adjacent lanes
    for (int j = 0; j < kAtB; ++j) {
      const float pj = Ps[r * L::PP + j];
      const float* vr = Vs + j * L::PV + g * DC;
#pragma unroll
      for (int e = 0; e < DC; e += 4) {
        const float4 vv = *reinterpret_cast<const float4*>(vr + e);
        acc[e] = fmaf(pj, vv.x, acc[e]);
        acc[e + 1] = fmaf(pj, vv.y, acc[e + 1]);
        acc[e + 2] = fmaf(pj, vv.z, acc[e + 2]);
        acc[e + 3] = fmaf(pj, vv.w, acc[e + 3]);
      }
    }
  }
  if (qi < a.Lq) {
    const float inv = l > 0.f ? 1.f / l : 0.f;
    float* orow = at_row_w(o, b, h, qi) + g * DC;
#pragma unroll
    for (int e = 0; e < DC; e += 4)
      *reinterpret_cast<float4*>(orow + e) =
          make_float4(acc[e] * inv, acc[e + 1] * inv, acc[e + 2] * inv, acc[e + 3] * inv);
    if (g == 0) lse[(int64_t)bh * a.Lq + qi] = l > 0.f ? m + logf(l) : -FLT_MAX;
  }
}

// D_i = sum_d dO_i,d * O_i,d, one warp per query row
template <int D>
__global__ void sdpa_bwd_di_kernel(AtView dout, AtView out, float* __restrict__ di, AtArgs a) {
  const int64_t rows = (int64_t)a.B * a.H * a.Lq;
  const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int i = (int)(row % a.Lq), bh = (int)(row / a.Lq), b = bh / a.H, h = bh % a.H;
  const float* gr = at_row(dout, b, h, i);
  const float* orow = at_row(out, b, h, i);
  float s = 0.f;
  for (int d = lane; d < D; d += 32) s = fmaf(__ldg(gr + d), __ldg(orow + d), s);
  for (int o = 16; o > 0; o >>= 1) s += __shfl_down_sync(0xffffffffu, s, o);
  if (lane == 0) di[row] = s;
}

template <int D>
struct AtKvSmem {
  static constexpr int PK = D + 1, PV = D + 1, PQ = D + 4, PG = D + 4, PT = kAtB + 1;
  static constexpr int K = 0, V = K + kAtB * PK, Q = V + kAtB * PV, G = Q + kAtB * PQ, P = G + kAtB * PG,
                       S = P + kAtB * PT, LSE = S + kAtB * PT, DI = LSE + kAtB;
  static constexpr int FLOATS = DI + kAtB;
};

template <int D>
__global__ void __launch_bounds__(kAtThreads) sdpa_bwd_dkdv_kernel(AtView q, AtView k, AtView v, AtView dout,
                                                                   const float* __restrict__ lse,
                                                                   const float* __restrict__ di, AtView dk,
                                                                   AtView dv, AtArgs a) {
  using L = AtKvSmem<D>;
  constexpr int DC = D / 4;
  extern __shared__ __align__(16) float at_smem[];
  float* Ks = at_smem + L::K;
  float* Vs = at_smem + L::V;
  float* Qs = at_smem + L::Q;
  float* Gs = at_smem + L::G;
  float* Pt = at_smem + L::P;
  float* St = at_smem + L::S;
  float* Ls = at_smem + L::LSE;
  float* Ds = at_smem + L::DI;
  const int bh = blockIdx.y, b = bh / a.H, h = bh % a.H;
  const int k0 = blockIdx.x * kAtB;
  const int j = threadIdx.x >> 2, g = threadIdx.x & 3;
  const int kj = k0 + j;
  at_load<D>(Ks, L::PK, k, b, h, k0, a.Lk, 1.f);
  at_load<D>(Vs, L::PV, v, b, h, k0, a.Lk, 1.f);
  float dka[DC], dva[DC];
#pragma unroll
  for (int e = 0; e < DC; ++e) dka[e] = dva[e] = 0.f;
  const int qstart = a.causal ? (k0 / kAtB) * kAtB : 0;
  for (int q0 = qstart; q0 < a.Lq; q0 += kAtB) {
    __syncthreads();
    at_load<D>(Qs, L::PQ, q, b, h, q0, a.Lq, 1.f);
    at_load<D>(Gs, L::PG, dout, b, h, q0, a.Lq, 1.f);
    if (threadIdx.x < kAtB) {
      const int qi = q0 + threadIdx.x;
      Ls[threadIdx.x] = qi < a.Lq ? lse[(int64_t)bh * a.Lq + qi] : 0.f;
      Ds[threadIdx.x] = qi < a.Lq ? di[(int64_t)bh * a.Lq + qi] : 0.f;
    }
    __syncthreads();
    float s[16], dp[16];
#pragma unroll
    for (int u = 0; u < 16; ++u) s[u] = dp[u] = 0.f;
    for (int d = 0; d < D; ++d) {
      const float kd = Ks[j * L::PK + d], vd = Vs[j * L::PV + d];
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        const int i = g + 4 * u;
        s[u] = fmaf(Qs[i * L::PQ + d], kd, s[u]);
        dp[u] = fmaf(Gs[i * L::PG + d], vd, dp[u]);
      }
    }
#pragma unroll
    for (int u = 0; u < 16; ++u) {
      const int i = g + 4 * u, qi = q0 + i;
      const bool ok = qi < a.Lq && kj < a.Lk && !(a.causal && kj > qi);
      const float p = ok ? expf(s[u] * a.scale - Ls[i]) : 0.f;
      Pt[j * L::PT + i] = p;
      St[j * L::PT + i] = p * (dp[u] - Ds[i]);
    }
    __syncwarp();  // row j of Pt / St comes from the four adjacent lanes
    for (int i = 0; i < kAtB; ++i) {
      const float p = Pt[j * L::PT + i], ds = St[j * L::PT + i];
      const float* gr = Gs + i * L::PG + g * DC;
      const float* qr = Qs + i * L::PQ + g * DC;
#pragma unroll
      for (int e = 0; e < DC; e += 4) {
        const float4 gg = *reinterpret_cast<const float4*>(gr + e);
        const float4 qq = *reinterpret_cast<const float4*>(qr + e);
        dva[e] = fmaf(p, gg.x, dva[e]);
        dva[e + 1] = fmaf(p, gg.y, dva[e + 1]);
        dva[e + 2] = fmaf(p, gg.z, dva[e + 2]);
        dva[e + 3] = fmaf(p, gg.w, dva[e + 3]);
        dka[e] = fmaf(ds, qq.x, dka[e]);
        dka[e + 1] = fmaf(ds, qq.y, dka[e + 1]);
        dka[e + 2] = fmaf(ds, qq.z, dka[e + 2]);
        dka[e + 3] = fmaf(ds, qq.w, dka[e + 3]);
      }
    }
  }
  if (kj < a.Lk) {
    float* kr = at_row_w(dk, b, h, kj) + g * DC;
    float* vr = at_row_w(dv, b, h, kj) + g * DC;
#pragma unroll
    for (int e = 0; e < DC; e += 4) {
      *reinterpret_cast<float4*>(kr + e) =
          make_float4(dka[e] * a.scale, dka[e + 1] * a.scale, dka[e + 2] * a.scale, dka[e + 3] * a.scale);
      *reinterpret_cast<float4*>(vr + e) = make_float4(dva[e], dva[e + 1], dva[e + 2], dva[e + 3]);
    }
  }
}

template <int D>
struct AtQSmem {
  static constexpr int PQ = D + 1, PG = D + 1, PK = D + 4, PV = D + 1, PS = kAtB + 1;
  static constexpr int Q = 0, G = Q + kAtB * PQ, K = G + kAtB * PG, V = K + kAtB * PK, S = V + kAtB * PV;
  static constexpr int FLOATS = S + kAtB * PS;
};

template <int D>
__global__ void __launch_bounds__(kAtThreads) sdpa_bwd_dq_kernel(AtView q, AtView k, AtView v, AtView dout,
                                                                 const float* __restrict__ lse,
                                                                 const float* __restrict__ di, AtView dq, AtArgs a) {
  using L = AtQSmem<D>;
  constexpr int DC = D / 4;
  extern __shared__ __align__(16) float at_smem[];
  float* Qs = at_smem + L::Q;
  float* Gs = at_smem + L::G;
  float* Ks = at_smem + L::K;
  float* Vs = at_smem + L::V;
  float* Ss = at_smem + L::S;
  const int bh = blockIdx.y, b = bh / a.H, h = bh % a.H;
  const int q0 = blockIdx.x * kAtB;
  const int r = threadIdx.x >> 2, g = threadIdx.x & 3;
  const int qi = q0 + r;
  at_load<D>(Qs, L::PQ, q, b, h, q0, a.Lq, 1.f);
  at_load<D>(Gs, L::PG, dout, b, h, q0, a.Lq, 1.f);
  const float lse_i = qi < a.Lq ? lse[(int64_t)bh * a.Lq + qi] : 0.f;
  const float di_i = qi < a.Lq ? di[(int64_t)bh * a.Lq + qi] : 0.f;
  float dqa[DC];
#pragma unroll
  for (int e = 0; e < DC; ++e) dqa[e] = 0.f;
  const int kend = a.causal ? min(a.Lk, q0 + kAtB) : a.Lk;
  for (int k0 = 0; k0 < kend; k0 += kAtB) {
    __syncthreads();
    at_load<D>(Ks, L::PK, k, b, h, k0, a.Lk, 1.f);
    at_load<D>(Vs, L::PV, v, b, h, k0, a.Lk, 1.f);
    __syncthreads();
    float s[16], dp[16];
#pragma unroll
    for (int u = 0; u < 16; ++u) s[u] = dp[u] = 0.f;
    for (int d = 0; d < D; ++d) {
      const float qd = Qs[r * L::PQ + d], gd = Gs[r * L::PG + d];
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        const int jj = g + 4 * u;
        s[u] = fmaf(qd, Ks[jj * L::PK + d], s[u]);
        dp[u] = fmaf(gd, Vs[jj * L::PV + d], dp[u]);
      }
    }
#pragma unroll
    for (int u = 0; u < 16; ++u) {
      const int jj = g + 4 * u, kj = k0 + jj;
      const bool ok = qi < a.Lq && kj < a.Lk && !(a.causal && kj > qi);
      const float p = ok ? expf(s[u] * a.scale - lse_i) : 0.f;
      Ss[r * L::PS + jj] = p * (dp[u] - di_i);
    }
    __syncwarp();
    for (int jj = 0; jj < kAtB; ++jj) {
      const float ds = Ss[r * L::PS + jj];
      const float* kr = Ks + jj * L::PK + g * DC;
#pragma unroll
      for (int e = 0; e < DC; e += 4) {
        const float4 kk = *reinterpret_cast<const float4*>(kr + e);
        dqa[e] = fmaf(ds, kk.x, dqa[e]);
        dqa[e + 1] = fmaf(ds, kk.y, dqa[e + 1]);
        dqa[e + 2] = fmaf(ds, kk.z, dqa[e + 2]);
        dqa[e + 3] = fmaf(ds, kk.w, dqa[e + 3]);
      }
    }
  }
  if (qi < a.Lq) {
    float* qr = at_row_w(dq, b, h, qi) + g * DC;
#pragma unroll
    for (int e = 0; e < DC; e += 4)
      *reinterpret_cast<float4*>(qr + e) =
          make_float4(dqa[e] * a.scale, dqa[e + 1] * a.scale, dqa[e + 2] * a.scale, dqa[e + 3] * a.scale);
  }
}

// ------------------------------------------------------------ host side
static int at_view(const pvb2_tensor* t, int B, int H, int L, int D, const char* what, AtView* v) {
  PVB2_CHECK_ARG(t && t->dtype == PVB2_F32 && t->ndim == 4, "sdpa: %s must be a 4-D float32 tensor", what);
  PVB2_CHECK_ARG(t->sizes[0] == B && t->sizes[1] == H && t->sizes[2] == L && t->sizes[3] == D,
                 "sdpa: %s has the wrong shape", what);
  PVB2_CHECK_ARG(t->strides[3] == 1, "sdpa: %s must be contiguous along the head dimension", what);
  PVB2_CHECK_ARG(((uintptr_t)t->data & 15) == 0 && t->strides[0] % 4 == 0 && t->strides[1] % 4 == 0 &&
                     t->strides[2] % 4 == 0,
                 "sdpa: %s rows must be 16-byte aligned", what);
  v->p = (float*)t->data;
  v->sb = t->strides[0];
  v->sh = t->strides[1];
  v->sl = t->strides[2];
  return PVB2_OK;
}

static int at_check(const pvb2_sdpa_desc* d) {
  PVB2_CHECK_ARG(d->D == 32 || d->D == 64 || d->D == 128, "sdpa: head dimension %d not supported (32, 64, 128)",
                 d->D);
  PVB2_CHECK_ARG(d->B >= 0 && d->H >= 0 && d->Lq >= 0 && d->Lk >= 0, "sdpa: negative size");
  PVB2_CHECK_ARG((int64_t)d->B * d->H <= 65535, "sdpa: more than 65535 heads");
  return PVB2_OK;
}

// `done`: the calling kernel's own per-device flag
template <typename K>
static int at_smem_attr(K kernel, int bytes, std::atomic<uint64_t>& done) {
  if (first_on_device(done))
    PVB2_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  return PVB2_OK;
}

template <int D>
static int at_fwd(const AtView& q, const AtView& k, const AtView& v, const AtView& o, float* lse, const AtArgs& a,
                  cudaStream_t s) {
  const int smem = AtFwdSmem<D>::FLOATS * 4;
  static std::atomic<uint64_t> attr{0};
  PVB2_TRY(at_smem_attr(sdpa_fwd_kernel<D>, smem, attr));
  const dim3 grid((unsigned)((a.Lq + kAtB - 1) / kAtB), (unsigned)(a.B * a.H));
  sdpa_fwd_kernel<D><<<grid, kAtThreads, smem, s>>>(q, k, v, o, lse, a);
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

template <int D>
static int at_bwd(const AtView& q, const AtView& k, const AtView& v, const AtView& o, const AtView& g,
                  const float* lse, float* di, const AtView& dq, const AtView& dk, const AtView& dv, const AtArgs& a,
                  cudaStream_t s) {
  const int64_t rows = (int64_t)a.B * a.H * a.Lq;
  sdpa_bwd_di_kernel<D><<<(unsigned)((rows * 32 + 255) / 256), 256, 0, s>>>(g, o, di, a);
  PVB2_LAUNCH_CHECK();
  const int skv = AtKvSmem<D>::FLOATS * 4, sq = AtQSmem<D>::FLOATS * 4;
  static std::atomic<uint64_t> attr_kv{0}, attr_q{0};
  PVB2_TRY(at_smem_attr(sdpa_bwd_dkdv_kernel<D>, skv, attr_kv));
  PVB2_TRY(at_smem_attr(sdpa_bwd_dq_kernel<D>, sq, attr_q));
  const dim3 gk((unsigned)((a.Lk + kAtB - 1) / kAtB), (unsigned)(a.B * a.H));
  sdpa_bwd_dkdv_kernel<D><<<gk, kAtThreads, skv, s>>>(q, k, v, g, lse, di, dk, dv, a);
  PVB2_LAUNCH_CHECK();
  const dim3 gq((unsigned)((a.Lq + kAtB - 1) / kAtB), (unsigned)(a.B * a.H));
  sdpa_bwd_dq_kernel<D><<<gq, kAtThreads, sq, s>>>(q, k, v, g, lse, di, dq, a);
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

}  // namespace pvb2

using namespace pvb2;

extern "C" {

int pvb2_sdpa_fwd(const pvb2_sdpa_desc* d, const pvb2_tensor* q, const pvb2_tensor* k, const pvb2_tensor* v,
                  const pvb2_tensor* out, float* lse, pvb2_stream stream) {
  PVB2_TRY(at_check(d));
  AtView qv, kv, vv, ov;
  PVB2_TRY(at_view(q, d->B, d->H, d->Lq, d->D, "query", &qv));
  PVB2_TRY(at_view(k, d->B, d->H, d->Lk, d->D, "key", &kv));
  PVB2_TRY(at_view(v, d->B, d->H, d->Lk, d->D, "value", &vv));
  PVB2_TRY(at_view(out, d->B, d->H, d->Lq, d->D, "output", &ov));
  PVB2_CHECK_ARG(lse || (int64_t)d->B * d->H * d->Lq == 0, "sdpa: logsumexp buffer required");
  if ((int64_t)d->B * d->H * d->Lq == 0) return PVB2_OK;
  const AtArgs a{d->B, d->H, d->Lq, d->Lk, d->scale, d->causal};
  cudaStream_t s = as_stream(stream);
  if (d->D == 32) return at_fwd<32>(qv, kv, vv, ov, lse, a, s);
  if (d->D == 64) return at_fwd<64>(qv, kv, vv, ov, lse, a, s);
  return at_fwd<128>(qv, kv, vv, ov, lse, a, s);
}

size_t pvb2_sdpa_bwd_workspace_size(const pvb2_sdpa_desc* d) { return (size_t)d->B * d->H * d->Lq * sizeof(float); }

int pvb2_sdpa_bwd(const pvb2_sdpa_desc* d, const pvb2_tensor* q, const pvb2_tensor* k, const pvb2_tensor* v,
                  const pvb2_tensor* out, const pvb2_tensor* dout, const float* lse, const pvb2_tensor* dq,
                  const pvb2_tensor* dk, const pvb2_tensor* dv, void* workspace, size_t workspace_bytes,
                  pvb2_stream stream) {
  PVB2_TRY(at_check(d));
  AtView qv, kv, vv, ov, gv, dqv, dkv, dvv;
  PVB2_TRY(at_view(q, d->B, d->H, d->Lq, d->D, "query", &qv));
  PVB2_TRY(at_view(k, d->B, d->H, d->Lk, d->D, "key", &kv));
  PVB2_TRY(at_view(v, d->B, d->H, d->Lk, d->D, "value", &vv));
  PVB2_TRY(at_view(out, d->B, d->H, d->Lq, d->D, "output", &ov));
  PVB2_TRY(at_view(dout, d->B, d->H, d->Lq, d->D, "grad_output", &gv));
  PVB2_TRY(at_view(dq, d->B, d->H, d->Lq, d->D, "grad_query", &dqv));
  PVB2_TRY(at_view(dk, d->B, d->H, d->Lk, d->D, "grad_key", &dkv));
  PVB2_TRY(at_view(dv, d->B, d->H, d->Lk, d->D, "grad_value", &dvv));
  cudaStream_t s = as_stream(stream);
  if ((int64_t)d->B * d->H == 0) return PVB2_OK;
  if (d->Lq == 0 || d->Lk == 0) {  // nothing flows: zero gradients
    if (d->Lk > 0) {
      PVB2_TRY(pvb2_fill(dk, 0.0, stream));
      PVB2_TRY(pvb2_fill(dv, 0.0, stream));
    }
    if (d->Lq > 0) PVB2_TRY(pvb2_fill(dq, 0.0, stream));
    return PVB2_OK;
  }
  const size_t need = pvb2_sdpa_bwd_workspace_size(d);
  PVB2_CHECK_ARG(workspace && workspace_bytes >= need, "sdpa_bwd: workspace too small (%zu < %zu)", workspace_bytes,
                 need);
  const AtArgs a{d->B, d->H, d->Lq, d->Lk, d->scale, d->causal};
  float* di = (float*)workspace;
  if (d->D == 32) return at_bwd<32>(qv, kv, vv, ov, gv, lse, di, dqv, dkv, dvv, a, s);
  if (d->D == 64) return at_bwd<64>(qv, kv, vv, ov, gv, lse, di, dqv, dkv, dvv, a, s);
  return at_bwd<128>(qv, kv, vv, ov, gv, lse, di, dqv, dkv, dvv, a, s);
}

}  // extern "C"
