// Fused scaled-dot-product attention, forward and backward, fp32.
//
// Replaces the math path the reference's ViT attention took: two batched
// GEMMs and a softmax through mm_bmm_out (src/vision_ops.cpp:541-626) and
// _softmax_out / _softmax_backward_data_out (src/loss_ops.cpp:137-213), each
// writing the [B*H, Lq, Lk] score matrix to memory.  Here the scores never
// leave shared memory.
//
// Layout: Q [B, H, Lq, D], K and V [B, H, Lk, D], any strides over (b, h, l),
// unit stride along d.  O [B, H, Lq, D], logsumexp [B, H, Lq].  D is 32, 64
// or 128.  No attention mask, no dropout; optional causal mask (query i sees
// keys j <= i).
//
// Tiles are 64 queries x 64 keys in shared memory, row-major with 4 floats
// of padding per row.  256 threads, t = 16 * tr + tc; each tile product is
// register-blocked so that a thread does 16 FMAs per pair of 16-byte shared
// loads:
//   NT  C[m][n] = sum_d A[m][d] B[n][d]   (S = Q K^T, dP = dO V^T)
//       thread rows m = tr + 16 i, columns n = tc + 16 j (i, j < 4): the 64
//       scores of a row sit in one half-warp, so row max / sum are four
//       xor-shuffles;
//   NN  C[m][c] += sum_k A[m][k] B[k][c]  (O += P V, dQ = dS K), rows as NT;
//   TN  C[m][c] += sum_r A[r][m] B[r][c]  (dV += P^T dO, dK += dS^T Q),
//       rows m = 4 tr .. 4 tr + 3;
// where a thread owns D / 16 of the D output columns c: 2 at 2 tc (D = 32),
// 4 at 4 tc (D = 64), 4 at 4 tc and 4 at 4 tc + 64 (D = 128), so a
// half-warp reads a tile row without bank conflicts.
//
// Forward: one CTA per (64 queries, head), key blocks streamed with the
// online softmax (running max m and sum l per row, O rescaled by
// exp(m_old - m_new)); logsumexp = m + log l.
// Backward, with D_i = sum_d dO_i,d O_i,d, P_ij = exp(s_ij - lse_i),
// dS_ij = P_ij (dP_ij - D_i): one CTA per (64 keys, head) loops over the
// query blocks, accumulating dV_j and dK_j in registers and writing its
// contribution dS K_j to dQ into a per-key-block slice of the workspace;
// a reduction kernel sums the slices in key-block order (deterministic).
// When the caller's workspace cannot hold the slices, a second kernel per
// (64 queries, head) recomputes S and dP and accumulates dQ instead.
// In exact-fp32 math mode all arithmetic is fp32 on the CUDA cores; in the
// default TF32 mode (D = 32 or 64) the tile products run on the tensor cores
// (the kernels below the SIMT ones).  The exponentials use expf.
#include <cfloat>
#include "common.cuh"

namespace pvb2 {

constexpr int kAtB = 64;  // rows (queries or keys) per tile
constexpr int kAtThreads = 256;
constexpr int kAtPS = kAtB + 4;  // pitch of the 64-wide P / dS tiles

template <int D>
struct AtCfg {
  static constexpr int PD = D + 4;   // pitch of the D-wide Q / K / V / dO tiles
  static constexpr int NC = D / 16;  // output columns per thread in NN / TN
  static constexpr int TILE = kAtB * PD;
  static constexpr int PTILE = kAtB * kAtPS;
};

struct AtView {  // one of Q, K, V, O, dO, dQ, dK, dV
  float* p;
  int64_t sb, sh, sl;
};

struct AtArgs {
  int B, H, Lq, Lk;
  float scale;
  int causal;
};

__device__ __forceinline__ float* at_row(const AtView& v, int b, int h, int l) {
  return v.p + b * v.sb + h * v.sh + (int64_t)l * v.sl;
}

__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }

__device__ __forceinline__ float f4(const float4& v, int i) { return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w; }

// the thread's D / 16 columns of one tile row
template <int D>
__device__ __forceinline__ void at_frag(const float* row, int tc, float (&b)[AtCfg<D>::NC]) {
  if constexpr (D == 32) {
    const float2 v = *reinterpret_cast<const float2*>(row + tc * 2);
    b[0] = v.x;
    b[1] = v.y;
  } else {
#pragma unroll
    for (int h = 0; h < D / 64; ++h) {
      const float4 v = ld4(row + tc * 4 + 64 * h);
      b[4 * h] = v.x;
      b[4 * h + 1] = v.y;
      b[4 * h + 2] = v.z;
      b[4 * h + 3] = v.w;
    }
  }
}

// store a thread's D / 16 columns of one output row, times `mul`
template <int D>
__device__ __forceinline__ void at_store_row(float* row, int tc, const float (&v)[AtCfg<D>::NC], float mul) {
  if constexpr (D == 32) {
    *reinterpret_cast<float2*>(row + tc * 2) = make_float2(v[0] * mul, v[1] * mul);
  } else {
#pragma unroll
    for (int h = 0; h < D / 64; ++h)
      *reinterpret_cast<float4*>(row + tc * 4 + 64 * h) =
          make_float4(v[4 * h] * mul, v[4 * h + 1] * mul, v[4 * h + 2] * mul, v[4 * h + 3] * mul);
  }
}

// rows [l0, l0 + 64) of a view into a D-wide tile, times `mul`, zero past `len`
template <int D>
__device__ __forceinline__ void at_load(float* s, const AtView& v, int b, int h, int l0, int len, float mul) {
  for (int e = threadIdx.x; e < kAtB * (D / 4); e += kAtThreads) {
    const int r = e / (D / 4), c4 = (e % (D / 4)) * 4;
    float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
    if (l0 + r < len) x = __ldg(reinterpret_cast<const float4*>(at_row(v, b, h, l0 + r) + c4));
    x.x *= mul;
    x.y *= mul;
    x.z *= mul;
    x.w *= mul;
    *reinterpret_cast<float4*>(s + r * AtCfg<D>::PD + c4) = x;
  }
}

// C = A B^T over the head dimension (both D-wide tiles)
template <int D>
__device__ __forceinline__ void at_nt(const float* A, const float* B, int tr, int tc, float (&c)[4][4]) {
  constexpr int PD = AtCfg<D>::PD;
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) c[i][j] = 0.f;
#pragma unroll 2
  for (int d = 0; d < D; d += 4) {
    float4 a[4], b[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) a[i] = ld4(A + (tr + 16 * i) * PD + d);
#pragma unroll
    for (int j = 0; j < 4; ++j) b[j] = ld4(B + (tc + 16 * j) * PD + d);
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        c[i][j] = fmaf(a[i].x, b[j].x, c[i][j]);
        c[i][j] = fmaf(a[i].y, b[j].y, c[i][j]);
        c[i][j] = fmaf(a[i].z, b[j].z, c[i][j]);
        c[i][j] = fmaf(a[i].w, b[j].w, c[i][j]);
      }
  }
}

// C += A B, A a 64-wide tile (rows tr + 16 i), B a D-wide tile; k < kn
// (kn a multiple of 4)
template <int D>
__device__ __forceinline__ void at_nn(const float* A, const float* B, int kn, int tr, int tc,
                                      float (&c)[4][AtCfg<D>::NC]) {
  constexpr int PD = AtCfg<D>::PD, NC = AtCfg<D>::NC;
  for (int k = 0; k < kn; k += 4) {
    float4 a[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) a[i] = ld4(A + (tr + 16 * i) * kAtPS + k);
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      float b[NC];
      at_frag<D>(B + (k + kk) * PD, tc, b);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float av = f4(a[i], kk);
#pragma unroll
        for (int e = 0; e < NC; ++e) c[i][e] = fmaf(av, b[e], c[i][e]);
      }
    }
  }
}

// C += A^T B, A a 64-wide tile (columns 4 tr .. 4 tr + 3), B a D-wide tile;
// rows r < rn
template <int D>
__device__ __forceinline__ void at_tn(const float* A, const float* B, int rn, int tr, int tc,
                                      float (&c)[4][AtCfg<D>::NC]) {
  constexpr int PD = AtCfg<D>::PD, NC = AtCfg<D>::NC;
#pragma unroll 2
  for (int r = 0; r < rn; ++r) {
    const float4 a = ld4(A + r * kAtPS + tr * 4);
    float b[NC];
    at_frag<D>(B + r * PD, tc, b);
#pragma unroll
    for (int e = 0; e < NC; ++e) {
      c[0][e] = fmaf(a.x, b[e], c[0][e]);
      c[1][e] = fmaf(a.y, b[e], c[1][e]);
      c[2][e] = fmaf(a.z, b[e], c[2][e]);
      c[3][e] = fmaf(a.w, b[e], c[3][e]);
    }
  }
}

__device__ __forceinline__ float half_max(float v) {
#pragma unroll
  for (int o = 1; o < 16; o <<= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float half_sum(float v) {
#pragma unroll
  for (int o = 1; o < 16; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// keys (or queries) of a tile that can matter, rounded up to a multiple of 4
__device__ __forceinline__ int at_span(int l0, int len) { return (min(kAtB, len - l0) + 3) & ~3; }

template <int D>
__global__ void __launch_bounds__(kAtThreads) sdpa_fwd_kernel(AtView q, AtView k, AtView v, AtView o,
                                                              float* __restrict__ lse, AtArgs a) {
  using C = AtCfg<D>;
  constexpr int NC = C::NC;
  extern __shared__ __align__(16) float at_smem[];
  float* Qs = at_smem;
  float* Ks = Qs + C::TILE;
  float* Vs = Ks + C::TILE;
  float* Ps = Vs + C::TILE;
  const int bh = blockIdx.y, b = bh / a.H, h = bh % a.H;
  const int q0 = blockIdx.x * kAtB;
  const int tr = threadIdx.x >> 4, tc = threadIdx.x & 15;
  at_load<D>(Qs, q, b, h, q0, a.Lq, a.scale);
  float acc[4][NC];
  float m[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m[i] = -FLT_MAX;
    l[i] = 0.f;
#pragma unroll
    for (int e = 0; e < NC; ++e) acc[i][e] = 0.f;
  }
  const int kend = a.causal ? min(a.Lk, q0 + kAtB) : a.Lk;
  for (int k0 = 0; k0 < kend; k0 += kAtB) {
    __syncthreads();  // previous block's K / V no longer read
    at_load<D>(Ks, k, b, h, k0, a.Lk, 1.f);
    at_load<D>(Vs, v, b, h, k0, a.Lk, 1.f);
    __syncthreads();
    float s[4][4];
    at_nt<D>(Qs, Ks, tr, tc, s);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int qi = q0 + tr + 16 * i;
      float mx = -FLT_MAX;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int kj = k0 + tc + 16 * j;
        const bool ok = kj < a.Lk && !(a.causal && kj > qi);
        s[i][j] = ok ? s[i][j] : -FLT_MAX;
        mx = fmaxf(mx, s[i][j]);
      }
      const float mnew = fmaxf(m[i], half_max(mx));
      const float alpha = expf(m[i] - mnew);
      float ps = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float p = s[i][j] == -FLT_MAX ? 0.f : expf(s[i][j] - mnew);
        Ps[(tr + 16 * i) * kAtPS + tc + 16 * j] = p;
        ps += p;
      }
      l[i] = l[i] * alpha + half_sum(ps);
      m[i] = mnew;
#pragma unroll
      for (int e = 0; e < NC; ++e) acc[i][e] *= alpha;
    }
    __syncwarp();  // a row of P is written and read by the same half-warp
    at_nn<D>(Ps, Vs, at_span(k0, a.Lk), tr, tc, acc);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int qi = q0 + tr + 16 * i;
    if (qi >= a.Lq) continue;
    at_store_row<D>(at_row(o, b, h, qi), tc, acc[i], l[i] > 0.f ? 1.f / l[i] : 0.f);
    if (tc == 0) lse[(int64_t)bh * a.Lq + qi] = l[i] > 0.f ? m[i] + logf(l[i]) : -FLT_MAX;
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

// per-query-row logsumexp and D_i of a query block into shared memory
__device__ __forceinline__ void at_load_rows(float* Ls, float* Ds, const float* lse, const float* di, int64_t bh,
                                             int q0, int Lq) {
  if (threadIdx.x < kAtB) {
    const int qi = q0 + threadIdx.x;
    Ls[threadIdx.x] = qi < Lq ? lse[bh * Lq + qi] : 0.f;
    Ds[threadIdx.x] = qi < Lq ? di[bh * Lq + qi] : 0.f;
  }
}

// P and dS of one (query block, key block) pair into the 64-wide tiles
// (P only when Ps is given); rows tr + 16 i, keys tc + 16 j
template <int D>
__device__ __forceinline__ void at_probs(const float* Qs, const float* Gs, const float* Ks, const float* Vs,
                                         const float* Ls, const float* Ds, float* Ps, float* Ss, int q0, int k0,
                                         const AtArgs& a, int tr, int tc) {
  float s[4][4];
  at_nt<D>(Qs, Ks, tr, tc, s);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = tr + 16 * i, qi = q0 + r;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int kj = k0 + tc + 16 * j;
      const bool ok = qi < a.Lq && kj < a.Lk && !(a.causal && kj > qi);
      s[i][j] = ok ? expf(s[i][j] - Ls[r]) : 0.f;
      if (Ps) Ps[r * kAtPS + tc + 16 * j] = s[i][j];
    }
  }
  float dp[4][4];
  at_nt<D>(Gs, Vs, tr, tc, dp);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = tr + 16 * i;
#pragma unroll
    for (int j = 0; j < 4; ++j) Ss[r * kAtPS + tc + 16 * j] = s[i][j] * (dp[i][j] - Ds[r]);
  }
}

// dK, dV of one key block; with dq_part, also this key block's slice dS K of
// dQ (not yet times scale) at dq_part[kb][bh][q][:]
template <int D>
__global__ void __launch_bounds__(kAtThreads) sdpa_bwd_kv_kernel(AtView q, AtView k, AtView v, AtView dout,
                                                                 const float* __restrict__ lse,
                                                                 const float* __restrict__ di, AtView dk,
                                                                 AtView dv, float* __restrict__ dq_part, AtArgs a) {
  using C = AtCfg<D>;
  constexpr int NC = C::NC;
  extern __shared__ __align__(16) float at_smem[];
  float* Ks = at_smem;
  float* Vs = Ks + C::TILE;
  float* Qs = Vs + C::TILE;
  float* Gs = Qs + C::TILE;
  float* Ps = Gs + C::TILE;
  float* Ss = Ps + C::PTILE;
  float* Ls = Ss + C::PTILE;
  float* Ds = Ls + kAtB;
  const int bh = blockIdx.y, b = bh / a.H, h = bh % a.H;
  const int kb = blockIdx.x, k0 = kb * kAtB;
  const int tr = threadIdx.x >> 4, tc = threadIdx.x & 15;
  at_load<D>(Ks, k, b, h, k0, a.Lk, 1.f);
  at_load<D>(Vs, v, b, h, k0, a.Lk, 1.f);
  float dka[4][NC], dva[4][NC];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int e = 0; e < NC; ++e) dka[i][e] = dva[i][e] = 0.f;
  const int kspan = at_span(k0, a.Lk);
  for (int q0 = a.causal ? k0 : 0; q0 < a.Lq; q0 += kAtB) {
    __syncthreads();  // previous query block's tiles no longer read
    at_load<D>(Qs, q, b, h, q0, a.Lq, a.scale);
    at_load<D>(Gs, dout, b, h, q0, a.Lq, 1.f);
    at_load_rows(Ls, Ds, lse, di, bh, q0, a.Lq);
    __syncthreads();
    at_probs<D>(Qs, Gs, Ks, Vs, Ls, Ds, Ps, Ss, q0, k0, a, tr, tc);
    __syncthreads();  // TN reads columns written by every half-warp
    const int rn = min(kAtB, a.Lq - q0);
    at_tn<D>(Ps, Gs, rn, tr, tc, dva);
    at_tn<D>(Ss, Qs, rn, tr, tc, dka);  // Qs holds scale * Q: dK = scale * dS^T Q
    if (dq_part) {
      float dqa[4][NC];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int e = 0; e < NC; ++e) dqa[i][e] = 0.f;
      at_nn<D>(Ss, Ks, kspan, tr, tc, dqa);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int qi = q0 + tr + 16 * i;
        if (qi < a.Lq)
          at_store_row<D>(dq_part + (((int64_t)kb * a.B * a.H + bh) * a.Lq + qi) * D, tc, dqa[i], 1.f);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int kj = k0 + tr * 4 + i;
    if (kj >= a.Lk) continue;
    at_store_row<D>(at_row(dk, b, h, kj), tc, dka[i], 1.f);
    at_store_row<D>(at_row(dv, b, h, kj), tc, dva[i], 1.f);
  }
}

// dQ = scale * sum of the per-key-block slices, in key-block order; a causal
// query row q has slices only from key blocks kb <= q / 64
template <int D>
__global__ void sdpa_bwd_dq_reduce_kernel(const float* __restrict__ dq_part, AtView dq, AtArgs a, int nkb) {
  const int64_t n4 = (int64_t)a.B * a.H * a.Lq * (D / 4);
  const int64_t slice = (int64_t)a.B * a.H * a.Lq * D;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n4; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = e / (D / 4);
    const int c4 = (int)(e % (D / 4)) * 4;
    const int qi = (int)(row % a.Lq), bh = (int)(row / a.Lq);
    const int last = a.causal ? min(nkb - 1, qi / kAtB) : nkb - 1;
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    const float* p = dq_part + row * D + c4;
    for (int kb = 0; kb <= last; ++kb) {
      const float4 x = __ldg(reinterpret_cast<const float4*>(p + kb * slice));
      s.x += x.x;
      s.y += x.y;
      s.z += x.z;
      s.w += x.w;
    }
    *reinterpret_cast<float4*>(at_row(dq, bh / a.H, bh % a.H, qi) + c4) =
        make_float4(s.x * a.scale, s.y * a.scale, s.z * a.scale, s.w * a.scale);
  }
}

// dQ of one query block, recomputing S and dP per key block (used when the
// workspace has no room for the per-key-block slices)
template <int D>
__global__ void __launch_bounds__(kAtThreads) sdpa_bwd_dq_kernel(AtView q, AtView k, AtView v, AtView dout,
                                                                 const float* __restrict__ lse,
                                                                 const float* __restrict__ di, AtView dq, AtArgs a) {
  using C = AtCfg<D>;
  constexpr int NC = C::NC;
  extern __shared__ __align__(16) float at_smem[];
  float* Qs = at_smem;
  float* Gs = Qs + C::TILE;
  float* Ks = Gs + C::TILE;
  float* Vs = Ks + C::TILE;
  float* Ss = Vs + C::TILE;
  float* Ls = Ss + C::PTILE;
  float* Ds = Ls + kAtB;
  const int bh = blockIdx.y, b = bh / a.H, h = bh % a.H;
  const int q0 = blockIdx.x * kAtB;
  const int tr = threadIdx.x >> 4, tc = threadIdx.x & 15;
  at_load<D>(Qs, q, b, h, q0, a.Lq, a.scale);
  at_load<D>(Gs, dout, b, h, q0, a.Lq, 1.f);
  at_load_rows(Ls, Ds, lse, di, bh, q0, a.Lq);
  float dqa[4][NC];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int e = 0; e < NC; ++e) dqa[i][e] = 0.f;
  const int kend = a.causal ? min(a.Lk, q0 + kAtB) : a.Lk;
  for (int k0 = 0; k0 < kend; k0 += kAtB) {
    __syncthreads();
    at_load<D>(Ks, k, b, h, k0, a.Lk, 1.f);
    at_load<D>(Vs, v, b, h, k0, a.Lk, 1.f);
    __syncthreads();
    at_probs<D>(Qs, Gs, Ks, Vs, Ls, Ds, nullptr, Ss, q0, k0, a, tr, tc);
    __syncwarp();  // a row of dS is written and read by the same half-warp
    at_nn<D>(Ss, Ks, at_span(k0, a.Lk), tr, tc, dqa);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int qi = q0 + tr + 16 * i;
    if (qi < a.Lq) at_store_row<D>(at_row(dq, b, h, qi), tc, dqa[i], a.scale);
  }
}

// ------------------------------------------------- TF32 tensor-core kernels
// The default math mode (TF32, as for convolutions and GEMMs) runs the tile
// products on the tensor cores with warp-level mma.sync.m16n8k8 TF32
// (operands rounded to TF32 with cvt.rna, fp32 accumulation); D = 32 or 64.
// 128 threads, four warps of 16 rows each; fragment layouts of m16n8k8
// (g = lane / 4, t = lane % 4):  A a0 (g, t) a1 (g+8, t) a2 (g, t+4)
// a3 (g+8, t+4);  B b0 (t, g) b1 (t+4, g);  C c0 (g, 2t) c1 (g, 2t+1)
// c2 (g+8, 2t) c3 (g+8, 2t+1).  Shared tiles use a row pitch of D + 4
// (4 mod 32 banks: the (g, t) fragment reads are conflict-free).
constexpr int kTcThreads = 128;
constexpr int kTcPS = kAtB + 4;  // pitch of the 64-wide P / dS tiles

__device__ __forceinline__ uint32_t tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}

__device__ __forceinline__ void mma8(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// A fragment of rows r0 .. r0+15, columns k0 .. k0+7 of a row-major tile
__device__ __forceinline__ void frag_a(uint32_t (&a)[4], const float* T, int pitch, int r0, int k0, int g, int t) {
  a[0] = __float_as_uint(T[(r0 + g) * pitch + k0 + t]);
  a[1] = __float_as_uint(T[(r0 + g + 8) * pitch + k0 + t]);
  a[2] = __float_as_uint(T[(r0 + g) * pitch + k0 + t + 4]);
  a[3] = __float_as_uint(T[(r0 + g + 8) * pitch + k0 + t + 4]);
}
// A fragment read transposed: element (m, k) at T[k][m]
__device__ __forceinline__ void frag_a_t(uint32_t (&a)[4], const float* T, int pitch, int m0, int k0, int g, int t) {
  a[0] = __float_as_uint(T[(k0 + t) * pitch + m0 + g]);
  a[1] = __float_as_uint(T[(k0 + t) * pitch + m0 + g + 8]);
  a[2] = __float_as_uint(T[(k0 + t + 4) * pitch + m0 + g]);
  a[3] = __float_as_uint(T[(k0 + t + 4) * pitch + m0 + g + 8]);
}

// rows [l0, l0 + 64) of a view into a tile of pitch PITCH, times `mul`,
// rounded to TF32
template <int D, int PITCH>
__device__ __forceinline__ void tc_load(float* s, const AtView& v, int b, int h, int l0, int len, float mul) {
  for (int e = threadIdx.x; e < kAtB * (D / 4); e += kTcThreads) {
    const int r = e / (D / 4), c4 = (e % (D / 4)) * 4;
    float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
    if (l0 + r < len) x = __ldg(reinterpret_cast<const float4*>(at_row(v, b, h, l0 + r) + c4));
    x.x = __uint_as_float(tf32(x.x * mul));
    x.y = __uint_as_float(tf32(x.y * mul));
    x.z = __uint_as_float(tf32(x.z * mul));
    x.w = __uint_as_float(tf32(x.w * mul));
    *reinterpret_cast<float4*>(s + r * PITCH + c4) = x;
  }
}

// tiles hold TF32-rounded values (rounded once when stored), so fragments
// are plain reinterpretations
__device__ __forceinline__ uint32_t u32(float x) { return __float_as_uint(x); }

__device__ __forceinline__ float quad_max2(float v) {
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1));
  return fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2));
}
__device__ __forceinline__ float quad_sum2(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 1);
  return v + __shfl_xor_sync(0xffffffffu, v, 2);
}

// forward: CTA = 64 queries of a head; warp w owns query rows 16 w .. 16 w + 15
template <int D>
__global__ void __launch_bounds__(kTcThreads) sdpa_fwd_tc_kernel(AtView q, AtView k, AtView v, AtView o,
                                                                 float* __restrict__ lse, AtArgs a) {
  constexpr int PQ = D + 4, PV = D + 8, NT = D / 8;
  extern __shared__ __align__(16) float at_smem[];
  float* Qs = at_smem;
  float* Ks = Qs + kAtB * PQ;
  float* Vs = Ks + kAtB * PQ;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  float* Ps = Vs + kAtB * PV + warp * 16 * kTcPS;
  const int bh = blockIdx.y, b = bh / a.H, h = bh % a.H;
  const int q0 = blockIdx.x * kAtB, r0 = warp * 16;
  tc_load<D, PQ>(Qs, q, b, h, q0, a.Lq, a.scale);
  float acc[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
  float m[2] = {-FLT_MAX, -FLT_MAX}, l[2] = {0.f, 0.f};
  const int kend = a.causal ? min(a.Lk, q0 + kAtB) : a.Lk;
  for (int k0 = 0; k0 < kend; k0 += kAtB) {
    __syncthreads();  // previous block's K / V no longer read
    tc_load<D, PQ>(Ks, k, b, h, k0, a.Lk, 1.f);
    tc_load<D, PV>(Vs, v, b, h, k0, a.Lk, 1.f);
    __syncthreads();
    float s[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D; kk += 8) {
      uint32_t af[4];
      frag_a(af, Qs, PQ, r0, kk, g, t);
#pragma unroll
      for (int n = 0; n < 8; ++n)
        mma8(s[n], af, u32(Ks[(n * 8 + g) * PQ + kk + t]), u32(Ks[(n * 8 + g) * PQ + kk + t + 4]));
    }
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      const int qi = q0 + r0 + g + 8 * hr;
      float mx = -FLT_MAX;
#pragma unroll
      for (int n = 0; n < 8; ++n)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int kj = k0 + n * 8 + 2 * t + j;
          const bool ok = kj < a.Lk && !(a.causal && kj > qi);
          s[n][2 * hr + j] = ok ? s[n][2 * hr + j] : -FLT_MAX;
          mx = fmaxf(mx, s[n][2 * hr + j]);
        }
      const float mnew = fmaxf(m[hr], quad_max2(mx));
      const float alpha = expf(m[hr] - mnew);
      float ps = 0.f;
#pragma unroll
      for (int n = 0; n < 8; ++n)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const float p = s[n][2 * hr + j] == -FLT_MAX ? 0.f : expf(s[n][2 * hr + j] - mnew);
          Ps[(g + 8 * hr) * kTcPS + n * 8 + 2 * t + j] = __uint_as_float(tf32(p));
          ps += p;
        }
      l[hr] = l[hr] * alpha + quad_sum2(ps);
      m[hr] = mnew;
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        acc[n][2 * hr] *= alpha;
        acc[n][2 * hr + 1] *= alpha;
      }
    }
    __syncwarp();  // the warp's P rows are read back as A fragments
    const int kspan = at_span(k0, a.Lk);
    for (int kk = 0; kk < kspan; kk += 8) {
      uint32_t af[4];
      frag_a(af, Ps, kTcPS, 0, kk, g, t);
#pragma unroll
      for (int n = 0; n < NT; ++n)
        mma8(acc[n], af, u32(Vs[(kk + t) * PV + n * 8 + g]), u32(Vs[(kk + t + 4) * PV + n * 8 + g]));
    }
    __syncwarp();  // P rows may be rewritten by the next block
  }
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int qi = q0 + r0 + g + 8 * hr;
    if (qi >= a.Lq) continue;
    const float inv = l[hr] > 0.f ? 1.f / l[hr] : 0.f;
    float* orow = at_row(o, b, h, qi);
#pragma unroll
    for (int n = 0; n < NT; ++n)
      *reinterpret_cast<float2*>(orow + n * 8 + 2 * t) = make_float2(acc[n][2 * hr] * inv, acc[n][2 * hr + 1] * inv);
    if (t == 0) lse[(int64_t)bh * a.Lq + qi] = l[hr] > 0.f ? m[hr] + logf(l[hr]) : -FLT_MAX;
  }
}

// backward per 64-key block: warp w owns keys 16 w .. 16 w + 15 for S^T, dP^T,
// dV, dK and query rows 16 w .. 16 w + 15 for this block's dQ slice
template <int D>
__global__ void __launch_bounds__(kTcThreads) sdpa_bwd_kv_tc_kernel(AtView q, AtView k, AtView v, AtView dout,
                                                                    const float* __restrict__ lse,
                                                                    const float* __restrict__ di, AtView dk,
                                                                    AtView dv, float* __restrict__ dq_part,
                                                                    AtArgs a) {
  constexpr int PQ = D + 4, NT = D / 8;
  extern __shared__ __align__(16) float at_smem[];
  float* Ks = at_smem;
  float* Vs = Ks + kAtB * PQ;
  float* Qs = Vs + kAtB * PQ;
  float* Gs = Qs + kAtB * PQ;
  float* PTs = Gs + kAtB * PQ;  // P^T  [key][query]
  float* STs = PTs + kAtB * kTcPS;  // dS^T [key][query]
  float* Ls = STs + kAtB * kTcPS;
  float* Ds = Ls + kAtB;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int bh = blockIdx.y, b = bh / a.H, h = bh % a.H;
  const int kb = blockIdx.x, k0 = kb * kAtB, r0 = warp * 16;
  tc_load<D, PQ>(Ks, k, b, h, k0, a.Lk, 1.f);
  tc_load<D, PQ>(Vs, v, b, h, k0, a.Lk, 1.f);
  float dka[NT][4], dva[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) dka[n][e] = dva[n][e] = 0.f;
  for (int q0 = a.causal ? k0 : 0; q0 < a.Lq; q0 += kAtB) {
    __syncthreads();  // previous query block's tiles no longer read
    tc_load<D, PQ>(Qs, q, b, h, q0, a.Lq, a.scale);
    tc_load<D, PQ>(Gs, dout, b, h, q0, a.Lq, 1.f);
    at_load_rows(Ls, Ds, lse, di, bh, q0, a.Lq);
    __syncthreads();
    // S^T and dP^T for the warp's 16 keys x 64 queries
    float st[8][4], dp[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) st[n][e] = dp[n][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D; kk += 8) {
      uint32_t ak[4], av[4];
      frag_a(ak, Ks, PQ, r0, kk, g, t);
      frag_a(av, Vs, PQ, r0, kk, g, t);
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        const int qr = (n * 8 + g) * PQ + kk + t;
        mma8(st[n], ak, u32(Qs[qr]), u32(Qs[qr + 4]));
        mma8(dp[n], av, u32(Gs[qr]), u32(Gs[qr + 4]));
      }
    }
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      const int kr = r0 + g + 8 * hr, kj = k0 + kr;
#pragma unroll
      for (int n = 0; n < 8; ++n)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int qc = n * 8 + 2 * t + j, qi = q0 + qc;
          const bool ok = qi < a.Lq && kj < a.Lk && !(a.causal && kj > qi);
          const float p = ok ? expf(st[n][2 * hr + j] - Ls[qc]) : 0.f;
          PTs[kr * kTcPS + qc] = __uint_as_float(tf32(p));
          STs[kr * kTcPS + qc] = __uint_as_float(tf32(p * (dp[n][2 * hr + j] - Ds[qc])));
        }
    }
    __syncwarp();  // the warp's own P^T / dS^T rows are its A fragments below
    const int rn = at_span(q0, a.Lq);
    for (int kk = 0; kk < rn; kk += 8) {
      uint32_t ap[4], as[4];
      frag_a(ap, PTs, kTcPS, r0, kk, g, t);
      frag_a(as, STs, kTcPS, r0, kk, g, t);
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        const int r = (kk + t) * PQ + n * 8 + g;
        mma8(dva[n], ap, u32(Gs[r]), u32(Gs[r + 4 * PQ]));
        mma8(dka[n], as, u32(Qs[r]), u32(Qs[r + 4 * PQ]));  // Qs holds scale * Q
      }
    }
    if (dq_part) {
      __syncthreads();  // every warp's dS^T rows are read below
      float dqa[NT][4];
#pragma unroll
      for (int n = 0; n < NT; ++n) dqa[n][0] = dqa[n][1] = dqa[n][2] = dqa[n][3] = 0.f;
      const int kspan = at_span(k0, a.Lk);
      for (int kk = 0; kk < kspan; kk += 8) {
        uint32_t as[4];
        frag_a_t(as, STs, kTcPS, r0, kk, g, t);  // dS (query r0.., key kk..) = dS^T transposed
#pragma unroll
        for (int n = 0; n < NT; ++n) {
          const int r = (kk + t) * PQ + n * 8 + g;
          mma8(dqa[n], as, u32(Ks[r]), u32(Ks[r + 4 * PQ]));
        }
      }
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        const int qi = q0 + r0 + g + 8 * hr;
        if (qi >= a.Lq) continue;
        float* row = dq_part + (((int64_t)kb * a.B * a.H + bh) * a.Lq + qi) * D;
#pragma unroll
        for (int n = 0; n < NT; ++n)
          *reinterpret_cast<float2*>(row + n * 8 + 2 * t) = make_float2(dqa[n][2 * hr], dqa[n][2 * hr + 1]);
      }
    }
  }
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int kj = k0 + r0 + g + 8 * hr;
    if (kj >= a.Lk) continue;
    float* kr = at_row(dk, b, h, kj);
    float* vr = at_row(dv, b, h, kj);
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      *reinterpret_cast<float2*>(kr + n * 8 + 2 * t) = make_float2(dka[n][2 * hr], dka[n][2 * hr + 1]);
      *reinterpret_cast<float2*>(vr + n * 8 + 2 * t) = make_float2(dva[n][2 * hr], dva[n][2 * hr + 1]);
    }
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
                  bool tc, cudaStream_t s) {
  const dim3 grid((unsigned)((a.Lq + kAtB - 1) / kAtB), (unsigned)(a.B * a.H));
  if constexpr (D <= 64) {
    if (tc) {
      const int smem = (2 * kAtB * (D + 4) + kAtB * (D + 8) + 4 * 16 * kTcPS) * 4;
      static std::atomic<uint64_t> attr_tc{0};
      PVB2_TRY(at_smem_attr(sdpa_fwd_tc_kernel<D>, smem, attr_tc));
      sdpa_fwd_tc_kernel<D><<<grid, kTcThreads, smem, s>>>(q, k, v, o, lse, a);
      PVB2_LAUNCH_CHECK();
      return PVB2_OK;
    }
  }
  const int smem = (3 * AtCfg<D>::TILE + AtCfg<D>::PTILE) * 4;
  static std::atomic<uint64_t> attr{0};
  PVB2_TRY(at_smem_attr(sdpa_fwd_kernel<D>, smem, attr));
  sdpa_fwd_kernel<D><<<grid, kAtThreads, smem, s>>>(q, k, v, o, lse, a);
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

// workspace: D_i (rounded up to 256 bytes), then, when they fit, the
// per-key-block dQ slices
static size_t at_di_bytes(const pvb2_sdpa_desc* d) {
  return ((size_t)d->B * d->H * d->Lq * sizeof(float) + 255) & ~(size_t)255;
}
static size_t at_slice_bytes(const pvb2_sdpa_desc* d) {
  const size_t nkb = (size_t)(d->Lk + kAtB - 1) / kAtB;
  return nkb * d->B * d->H * d->Lq * d->D * sizeof(float);
}
constexpr size_t kAtSliceCap = (size_t)2 << 30;  // larger slices: dQ is recomputed instead

template <int D>
static int at_bwd(const AtView& q, const AtView& k, const AtView& v, const AtView& o, const AtView& g,
                  const float* lse, float* di, float* dq_part, const AtView& dq, const AtView& dk, const AtView& dv,
                  const AtArgs& a, bool tc, cudaStream_t s) {
  const int64_t rows = (int64_t)a.B * a.H * a.Lq;
  sdpa_bwd_di_kernel<D><<<(unsigned)((rows * 32 + 255) / 256), 256, 0, s>>>(g, o, di, a);
  PVB2_LAUNCH_CHECK();
  using C = AtCfg<D>;
  static std::atomic<uint64_t> attr_kv{0}, attr_q{0}, attr_tc{0};
  const int nkb = (a.Lk + kAtB - 1) / kAtB;
  const dim3 gk((unsigned)nkb, (unsigned)(a.B * a.H));
  bool done = false;
  if constexpr (D <= 64) {
    if (tc) {
      const int stc = (4 * kAtB * (D + 4) + 2 * kAtB * kTcPS + 2 * kAtB) * 4;
      PVB2_TRY(at_smem_attr(sdpa_bwd_kv_tc_kernel<D>, stc, attr_tc));
      sdpa_bwd_kv_tc_kernel<D><<<gk, kTcThreads, stc, s>>>(q, k, v, g, lse, di, dk, dv, dq_part, a);
      PVB2_LAUNCH_CHECK();
      done = true;
    }
  }
  if (!done) {
    const int skv = (4 * C::TILE + 2 * C::PTILE + 2 * kAtB) * 4;
    PVB2_TRY(at_smem_attr(sdpa_bwd_kv_kernel<D>, skv, attr_kv));
    sdpa_bwd_kv_kernel<D><<<gk, kAtThreads, skv, s>>>(q, k, v, g, lse, di, dk, dv, dq_part, a);
    PVB2_LAUNCH_CHECK();
  }
  if (dq_part) {
    sdpa_bwd_dq_reduce_kernel<D><<<grid_for(rows * (D / 4), 256), 256, 0, s>>>(dq_part, dq, a, nkb);
    PVB2_LAUNCH_CHECK();
    return PVB2_OK;
  }
  const int sq = (4 * C::TILE + C::PTILE + 2 * kAtB) * 4;
  PVB2_TRY(at_smem_attr(sdpa_bwd_dq_kernel<D>, sq, attr_q));
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
  const bool tc = d->math == PVB2_MATH_TF32;
  if (d->D == 32) return at_fwd<32>(qv, kv, vv, ov, lse, a, tc, s);
  if (d->D == 64) return at_fwd<64>(qv, kv, vv, ov, lse, a, tc, s);
  return at_fwd<128>(qv, kv, vv, ov, lse, a, tc, s);
}

size_t pvb2_sdpa_bwd_workspace_size(const pvb2_sdpa_desc* d) {
  const size_t slices = at_slice_bytes(d);
  return at_di_bytes(d) + (slices <= kAtSliceCap ? slices : 0);
}

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
  const size_t di_bytes = at_di_bytes(d);
  PVB2_CHECK_ARG(workspace && workspace_bytes >= di_bytes, "sdpa_bwd: workspace too small (%zu < %zu)",
                 workspace_bytes, di_bytes);
  const AtArgs a{d->B, d->H, d->Lq, d->Lk, d->scale, d->causal};
  float* di = (float*)workspace;
  // dQ through the per-key-block slices when they fit, else recomputed
  float* dq_part =
      workspace_bytes >= di_bytes + at_slice_bytes(d) ? (float*)((char*)workspace + di_bytes) : nullptr;
  const bool tc = d->math == PVB2_MATH_TF32;
  if (d->D == 32) return at_bwd<32>(qv, kv, vv, ov, gv, lse, di, dq_part, dqv, dkv, dvv, a, tc, s);
  if (d->D == 64) return at_bwd<64>(qv, kv, vv, ov, gv, lse, di, dq_part, dqv, dkv, dvv, a, tc, s);
  return at_bwd<128>(qv, kv, vv, ov, gv, lse, di, dq_part, dqv, dkv, dvv, a, tc, s);
}

}  // extern "C"
