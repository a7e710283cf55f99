// Depthwise convolution (groups == C == K, one filter per channel) as
// shared-memory-staged stencils; MobileNet-v2's 3x3 layers at stride 1 and 2.
//
// Replaces dlprim's grouped Conv2DForward / Conv2DBackwardData /
// Conv2DBackwardFilter as convolution_overrideable reached them with
// groups = C (src/vision_ops.cpp:30-59, 61-186).  All three are bound by
// HBM (4 B per input and output element, the filter is tiny), so each CTA
// reads a tile of its input plane once into shared memory, halo included,
// and every thread computes its outputs from there.
//
//   forward  a CTA covers a TH x TW output tile of PP consecutive planes
//            (n, c) (several whole planes when a plane is small: 7x7, 14x14),
//            staging the (TH-1)*sh + (R-1)*dh + 1 by (TW-1)*sw + (S-1)*dw + 1
//            input window of each and the planes' filters.
//   dgrad    the same over a TH x TW tile of dX: the dY rows and columns the
//            tile's taps reach are staged, each dX element sums the taps
//            whose source position is a multiple of the stride.
//   wgrad    a CTA takes one channel and a range of images; for each image
//            it stages x and dY tile by tile and every thread adds its
//            outputs' R*S products into registers.  The CTA's per-tap sums
//            (fixed-order block reduction) are partials [C][chunks][R*S],
//            summed in chunk order by dw_wgrad_reduce_kernel, so the result
//            depends only on the shapes.
#include <algorithm>

#include "common.cuh"

namespace pvb2 {

constexpr int kDwThreads = 256;
constexpr int kDwMaxTaps = 49;                 // R * S <= 49 (7 x 7)
constexpr int kDwSmemFloats = 46 * 1024 / 4;   // dynamic shared memory budget per CTA

struct DwGeom {
  int N, C, H, W, P, Q, R, S, sh, sw, ph, pw, dh, dw;
  int TH, TW, PP;        // output (dgrad: input) tile and planes per CTA
  int tiles_h, tiles_w;  // tiles per plane
  int IH, IW;            // staged window of one plane
};

// outputs [OH x OW] of each plane in tiles of TH x TW, about kDwOuts per CTA
// (16 per thread, so each thread keeps several loads in flight): whole
// planes, PP of them, when a plane has at most half that many outputs, else
// strips of full rows (rows cut at 128) as tall as the shared-memory budget
// allows
constexpr int kDwOuts = 4096;

static void dw_window(DwGeom& g, bool dgrad) {
  if (!dgrad) {
    g.IH = (g.TH - 1) * g.sh + (g.R - 1) * g.dh + 1;
    g.IW = (g.TW - 1) * g.sw + (g.S - 1) * g.dw + 1;
  } else {
    // dY rows p with h0 <= p*sh - ph + r*dh <= h0 + TH - 1 for some r
    g.IH = (g.TH - 1 + (g.R - 1) * g.dh) / g.sh + 2;
    g.IW = (g.TW - 1 + (g.S - 1) * g.dw) / g.sw + 2;
  }
}

static DwGeom dw_plan(int N, int C, int H, int W, int P, int Q, int R, int S, int sh, int sw, int ph, int pw, int dh,
                      int dw, bool dgrad) {
  DwGeom g{N, C, H, W, P, Q, R, S, sh, sw, ph, pw, dh, dw, 0, 0, 1, 1, 1, 0, 0};
  const int OH = dgrad ? H : P, OW = dgrad ? W : Q;  // the grid this pass writes
  if (OH * OW <= kDwOuts / 2) {
    g.TH = OH;
    g.TW = OW;
    dw_window(g, dgrad);
    g.PP = std::max(1, kDwOuts / (OH * OW));
    while (g.PP > 1 && g.PP * (g.IH * g.IW + R * S) > kDwSmemFloats) --g.PP;
  } else {
    g.TW = std::min(OW, 128);
    g.TH = std::max(1, std::min(OH, kDwOuts / g.TW));
    dw_window(g, dgrad);
    while (g.TH > 1 && g.IH * g.IW + R * S > kDwSmemFloats) {
      --g.TH;
      dw_window(g, dgrad);
    }
    g.PP = 1;
  }
  g.tiles_h = (OH + g.TH - 1) / g.TH;
  g.tiles_w = (OW + g.TW - 1) / g.TW;
  return g;
}

static bool dw_fits(const DwGeom& g) {
  return g.R * g.S <= kDwMaxTaps && (int64_t)g.PP * (g.IH * g.IW + g.R * g.S) <= kDwSmemFloats;
}

// floor division for possibly negative a, b > 0
__host__ __device__ __forceinline__ int floordiv(int a, int b) { return a >= 0 ? a / b : -((-a + b - 1) / b); }

// Loops run over (row, column) with a 32 x 8 thread block: threadIdx.x
// along a row (coalesced), threadIdx.y over rows, and no integer division
// per element.  SH / SW are the strides when they are compile-time (1, 2),
// 0 for the runtime values in g.

// ---------------------------------------------------------------- forward
template <int KR, int KS, int SH, int SW>
__global__ void __launch_bounds__(kDwThreads) dw_fwd_tile_kernel(DwGeom g, const float* __restrict__ x,
                                                                 const float* __restrict__ w,
                                                                 const float* __restrict__ bias,
                                                                 float* __restrict__ y) {
  extern __shared__ float sm[];
  constexpr int RS = KR * KS;
  const int sh = SH ? SH : g.sh, sw = SW ? SW : g.sw;
  const int tiles = g.tiles_h * g.tiles_w;
  const int64_t grp = blockIdx.x / tiles;
  const int tile = (int)(blockIdx.x - grp * tiles);
  const int p0 = (tile / g.tiles_w) * g.TH, q0 = (tile % g.tiles_w) * g.TW;
  const int64_t plane0 = grp * g.PP;
  const int pp = (int)min((int64_t)g.PP, (int64_t)g.N * g.C - plane0);
  const int win = g.IH * g.IW;
  float* wsm = sm + g.PP * win;  // filters [PP][RS]
  const int h0 = p0 * sh - g.ph, w0 = q0 * sw - g.pw;
  const int64_t HW = (int64_t)g.H * g.W;
  const int tx = threadIdx.x, ty = threadIdx.y, tid = ty * 32 + tx;
  for (int pl = 0; pl < pp; ++pl) {
    const float* xp = x + (plane0 + pl) * HW;
    float* dst = sm + pl * win;
    for (int i = ty; i < g.IH; i += 8) {
      const int h = h0 + i;
      const bool hok = (unsigned)h < (unsigned)g.H;
#pragma unroll 4
      for (int j = tx; j < g.IW; j += 32) {
        const int ww = w0 + j;
        dst[i * g.IW + j] = hok && (unsigned)ww < (unsigned)g.W ? __ldg(xp + (int64_t)h * g.W + ww) : 0.f;
      }
    }
  }
  for (int e = tid; e < pp * RS; e += kDwThreads) {
    const int pl = e / RS;
    wsm[e] = __ldg(w + (int64_t)((plane0 + pl) % g.C) * RS + (e - pl * RS));
  }
  __syncthreads();
  const int th = min(g.TH, g.P - p0), tw = min(g.TW, g.Q - q0);
  const int64_t PQ = (int64_t)g.P * g.Q;
  for (int pl = 0; pl < pp; ++pl) {
    const float* src = sm + pl * win;
    float wk[RS];
#pragma unroll
    for (int t = 0; t < RS; ++t) wk[t] = wsm[pl * RS + t];
    const float b0 = bias ? __ldg(bias + (plane0 + pl) % g.C) : 0.f;
    float* yp = y + (plane0 + pl) * PQ + (int64_t)p0 * g.Q + q0;
    for (int i = ty; i < th; i += 8) {
      const float* row = src + i * sh * g.IW;
#pragma unroll 2
      for (int j = tx; j < tw; j += 32) {
        const float* base = row + j * sw;
        float acc = b0;
#pragma unroll
        for (int a = 0; a < KR; ++a)
#pragma unroll
          for (int b = 0; b < KS; ++b) acc = fmaf(base[a * g.dh * g.IW + b * g.dw], wk[a * KS + b], acc);
        yp[(int64_t)i * g.Q + j] = acc;
      }
    }
  }
}

// ------------------------------------------------------------ input grad
// tile of dX at (h0, w0); staged dY rows pb .., columns qb .. with
// pb = ceil((h0 + ph - (R-1) dh) / sh): the first row any tap of the tile reads
template <int KR, int KS, int SH, int SW>
__global__ void __launch_bounds__(kDwThreads) dw_dgrad_tile_kernel(DwGeom g, const float* __restrict__ dy,
                                                                   const float* __restrict__ w,
                                                                   float* __restrict__ dx) {
  extern __shared__ float sm[];
  constexpr int RS = KR * KS;
  const int sh = SH ? SH : g.sh, sw = SW ? SW : g.sw;
  const int tiles = g.tiles_h * g.tiles_w;
  const int64_t grp = blockIdx.x / tiles;
  const int tile = (int)(blockIdx.x - grp * tiles);
  const int h0 = (tile / g.tiles_w) * g.TH, w0 = (tile % g.tiles_w) * g.TW;
  const int64_t plane0 = grp * g.PP;
  const int pp = (int)min((int64_t)g.PP, (int64_t)g.N * g.C - plane0);
  const int win = g.IH * g.IW;
  float* wsm = sm + g.PP * win;
  const int pb = floordiv(h0 + g.ph - (KR - 1) * g.dh + sh - 1, sh);
  const int qb = floordiv(w0 + g.pw - (KS - 1) * g.dw + sw - 1, sw);
  const int64_t PQ = (int64_t)g.P * g.Q, HW = (int64_t)g.H * g.W;
  const int tx = threadIdx.x, ty = threadIdx.y, tid = ty * 32 + tx;
  for (int pl = 0; pl < pp; ++pl) {
    const float* gp = dy + (plane0 + pl) * PQ;
    float* dst = sm + pl * win;
    for (int i = ty; i < g.IH; i += 8) {
      const int p = pb + i;
      const bool pok = (unsigned)p < (unsigned)g.P;
#pragma unroll 4
      for (int j = tx; j < g.IW; j += 32) {
        const int q = qb + j;
        dst[i * g.IW + j] = pok && (unsigned)q < (unsigned)g.Q ? __ldg(gp + (int64_t)p * g.Q + q) : 0.f;
      }
    }
  }
  for (int e = tid; e < pp * RS; e += kDwThreads) {
    const int pl = e / RS;
    wsm[e] = __ldg(w + (int64_t)((plane0 + pl) % g.C) * RS + (e - pl * RS));
  }
  __syncthreads();
  const int th = min(g.TH, g.H - h0), tw = min(g.TW, g.W - w0);
  for (int pl = 0; pl < pp; ++pl) {
    const float* src = sm + pl * win;
    float wk[RS];
#pragma unroll
    for (int t = 0; t < RS; ++t) wk[t] = wsm[pl * RS + t];
    float* xp = dx + (plane0 + pl) * HW + (int64_t)h0 * g.W + w0;
    for (int i = ty; i < th; i += 8) {
      const int h = h0 + i;
      for (int j = tx; j < tw; j += 32) {
        const int ww = w0 + j;
        float acc = 0.f;
#pragma unroll
        for (int a = 0; a < KR; ++a) {
          const int vh = h + g.ph - a * g.dh, p = floordiv(vh, sh);
          if (p * sh != vh) continue;
#pragma unroll
          for (int b = 0; b < KS; ++b) {
            const int vw = ww + g.pw - b * g.dw, q = floordiv(vw, sw);
            if (q * sw != vw) continue;
            acc = fmaf(src[(p - pb) * g.IW + (q - qb)], wk[a * KS + b], acc);
          }
        }
        xp[(int64_t)i * g.W + j] = acc;
      }
    }
  }
}

// ----------------------------------------- 3x3 forward, four outputs a thread
// Division by a runtime divisor d as a multiply-high and shift (Granlund and
// Montgomery's method, as CUTLASS's FastDivmod states it): m = ceil(2^p / d),
// p = 31 + ceil(log2 d); exact for dividends below 2^31.
struct FastDiv {
  int d;
  uint32_t m, s;
};
static FastDiv fast_div(int d) {
  FastDiv f{d, 0, 0};
  if (d > 1) {
    int l = 0;
    while ((1ll << l) < d) ++l;
    const int p = 31 + l;
    f.m = (uint32_t)(((1ull << p) + (uint64_t)d - 1) / (uint64_t)d);
    f.s = (uint32_t)(p - 32);
  }
  return f;
}
__device__ __forceinline__ int fdiv(int n, const FastDiv& f) {
  return f.d > 1 ? (int)(__umulhi((uint32_t)n, f.m) >> f.s) : n;
}
__device__ __forceinline__ FastDiv fast_div_device(int d) {
  FastDiv f{d, 0, 0};
  if (d > 1) {
    const int l = 32 - __clz(d - 1);  // ceil(log2 d)
    const int p = 31 + l;
    f.m = (uint32_t)(((1ull << p) + (uint64_t)d - 1) / (uint64_t)d);
    f.s = (uint32_t)(p - 32);
  }
  return f;
}

// 3x3 depthwise, dilation 1, stride SH in both dimensions (1 or 2), as a
// forward over planes H x W into P x Q.  A CTA stages PP whole planes or a
// strip of TH output rows of one plane (rows of IW4 floats, a multiple of 4,
// smem column c holding input column c - pw), then each thread computes
// items of four adjacent outputs of a row from registers: per filter row it
// reads the 6 (SH = 1) or 9 (SH = 2) inputs the four windows span with
// 16-byte shared loads.  FLIP reverses the filter: the stride-1 input
// gradient is this forward over dY with the flipped filter and padding
// 2 - pad.
// Staging of rows [0, ih) of pp planes into [pp][IH][IW4]: smem column c
// holds input column c - pw of input row h0 + i (zero outside the plane).
// Wide rows go one warp per row, four rows' loads in flight per warp;
// narrow rows (small planes) as one flat element loop, so no lane idles.
__device__ __forceinline__ void dw_stage_rows(float* __restrict__ sm, const float* __restrict__ x, int64_t plane0,
                                              int64_t pstride, int pp, int ih, int IH, int IW4, int h0, int pw, int H,
                                              int W, int64_t HW, const FastDiv& fiw4, const FastDiv& fih) {
  if (IW4 >= 64) {
    const int rows = pp * ih, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int r0 = warp; r0 < rows; r0 += 4 * (kDwThreads / 32)) {
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int rr = r0 + u * (kDwThreads / 32);
        if (rr >= rows) break;
        const int pl = rr / ih, i = rr - pl * ih, h = h0 + i;
        const float* xr = x + (plane0 + pl) * pstride + (int64_t)h * W;
        float* dst = sm + (pl * IH + i) * IW4;
        const bool hok = (unsigned)h < (unsigned)H;
        for (int c = lane; c < IW4; c += 32) {
          const int ww = c - pw;
          dst[c] = hok && (unsigned)ww < (unsigned)W ? __ldg(xr + ww) : 0.f;
        }
      }
    }
  } else {
    const int total = pp * ih * IW4;
#pragma unroll 4
    for (int e = threadIdx.x; e < total; e += kDwThreads) {
      const int rr = fdiv(e, fiw4), c = e - rr * IW4;
      const int pl = fdiv(rr, fih), i = rr - pl * ih, h = h0 + i, ww = c - pw;
      sm[(pl * IH + i) * IW4 + c] = (unsigned)h < (unsigned)H && (unsigned)ww < (unsigned)W
                                        ? __ldg(x + (plane0 + pl) * pstride + (int64_t)h * W + ww)
                                        : 0.f;
    }
  }
  (void)HW;
}

template <int SH, bool FLIP>
__global__ void __launch_bounds__(kDwThreads) dw3_fwd4_kernel(DwGeom g, int IW4, FastDiv fnq, FastDiv fth,
                                                              FastDiv fiw4, FastDiv fih,
                                                              const float* __restrict__ x,
                                                              const float* __restrict__ w,
                                                              const float* __restrict__ bias, float* __restrict__ y) {
  extern __shared__ __align__(16) float sm[];
  const int tiles = g.tiles_h;
  const int64_t grp = blockIdx.x / tiles;
  const int p0 = (int)(blockIdx.x - grp * tiles) * g.TH;
  const int64_t plane0 = grp * g.PP;
  const int pp = (int)min((int64_t)g.PP, (int64_t)g.N * g.C - plane0);
  const int win = g.IH * IW4;
  float* wsm = sm + g.PP * win;  // filters [PP][9]
  const int h0 = p0 * SH - g.ph;
  const int64_t HW = (int64_t)g.H * g.W, PQ = (int64_t)g.P * g.Q;
  // stage the rows this CTA's outputs read (a short last strip reads fewer)
  const int th0 = min(g.TH, g.P - p0), ih = (th0 - 1) * SH + 3;
  dw_stage_rows(sm, x, plane0, HW, pp, pp > 1 ? g.IH : ih, g.IH, IW4, h0, g.pw, g.H, g.W, HW, fiw4,
                pp > 1 ? fih : fast_div_device(ih));
  for (int e = threadIdx.x; e < pp * 9; e += kDwThreads) {
    const int pl = e / 9, t = e - pl * 9;
    wsm[e] = __ldg(w + (int64_t)((plane0 + pl) % g.C) * 9 + (FLIP ? 8 - t : t));
  }
  __syncthreads();
  const int th = min(g.TH, g.P - p0), nq = fnq.d;
  const int items = pp * th * nq;
  const bool vec_out = (g.Q & 3) == 0;
  for (int e = threadIdx.x; e < items; e += kDwThreads) {
    const int rowall = fdiv(e, fnq), jq = e - rowall * nq;
    const int pl = pp > 1 ? fdiv(rowall, fth) : 0, i = rowall - pl * th;
    const float* wk = wsm + pl * 9;
    const float b0 = bias ? __ldg(bias + (plane0 + pl) % g.C) : 0.f;
    float acc[4] = {b0, b0, b0, b0};
    const float* src = sm + pl * win + (i * SH) * IW4 + jq * 4 * SH;
#pragma unroll
    for (int a = 0; a < 3; ++a) {
      const float* r = src + a * IW4;
      float v[4 * SH + 2];
      const float4 v0 = *reinterpret_cast<const float4*>(r);
      v[0] = v0.x; v[1] = v0.y; v[2] = v0.z; v[3] = v0.w;
      if (SH == 1) {
        const float2 v1 = *reinterpret_cast<const float2*>(r + 4);
        v[4] = v1.x; v[5] = v1.y;
      } else {
        const float4 v1 = *reinterpret_cast<const float4*>(r + 4);
        v[4] = v1.x; v[5] = v1.y; v[6] = v1.z; v[7] = v1.w;
        v[8] = r[8];
      }
      const float w0 = wk[a * 3], w1 = wk[a * 3 + 1], w2 = wk[a * 3 + 2];
#pragma unroll
      for (int o = 0; o < 4; ++o) {
        acc[o] = fmaf(v[o * SH], w0, acc[o]);
        acc[o] = fmaf(v[o * SH + 1], w1, acc[o]);
        acc[o] = fmaf(v[o * SH + 2], w2, acc[o]);
      }
    }
    const int q0 = jq * 4;
    float* yr = y + (plane0 + pl) * PQ + (int64_t)(p0 + i) * g.Q + q0;
    if (vec_out) {
      *reinterpret_cast<float4*>(yr) = make_float4(acc[0], acc[1], acc[2], acc[3]);
    } else {
#pragma unroll
      for (int o = 0; o < 4; ++o)
        if (q0 + o < g.Q) yr[o] = acc[o];
    }
  }
}

// 3x3 weight gradient (dilation 1, stride SH): CTA (channel, image chunk)
// stages, per step, pp images' x rows ([pp][IH][IW4], as the forward) and
// dY rows ([pp][TH][Q4], zero past Q), then each thread takes items of four
// adjacent outputs and adds dY * x for the 9 taps into registers; the CTA's
// sums go to part[c][chunk][9] by a fixed-order block reduction.
template <int SH>
__global__ void __launch_bounds__(kDwThreads) dw3_wgrad4_kernel(DwGeom g, int IW4, FastDiv fnq, FastDiv fth,
                                                                FastDiv fiw4, FastDiv fih, FastDiv fq4,
                                                                const float* __restrict__ x,
                                                                const float* __restrict__ dy, int per_chunk,
                                                                float* __restrict__ part) {
  extern __shared__ __align__(16) float sm[];
  __shared__ float red[kDwThreads / 32][9];
  const int c = blockIdx.x, k = blockIdx.y;
  const int n0 = k * per_chunk, n1 = min(g.N, n0 + per_chunk);
  const int nq = fnq.d, Q4 = nq * 4;
  float* dsm = sm + g.PP * g.IH * IW4;
  const int64_t HW = (int64_t)g.H * g.W, PQ = (int64_t)g.P * g.Q;
  const int64_t xstride = (int64_t)g.C * HW, ystride = (int64_t)g.C * PQ;
  float acc[9];
#pragma unroll
  for (int t = 0; t < 9; ++t) acc[t] = 0.f;
  for (int n = n0; n < n1; n += g.PP) {
    const int pp = min(g.PP, n1 - n);
    const float* xb = x + ((int64_t)n * g.C + c) * HW;
    const float* yb = dy + ((int64_t)n * g.C + c) * PQ;
    for (int t = 0; t < g.tiles_h; ++t) {
      const int p0 = t * g.TH, th = min(g.TH, g.P - p0), ih = (th - 1) * SH + 3, h0 = p0 * SH - g.ph;
      const FastDiv fthr = pp > 1 ? fth : fast_div_device(th);
      __syncthreads();  // the previous step's rows are no longer read
      dw_stage_rows(sm, xb, 0, xstride, pp, pp > 1 ? g.IH : ih, g.IH, IW4, h0, g.pw, g.H, g.W, HW, fiw4,
                    pp > 1 ? fih : fast_div_device(ih));
      const int dtotal = pp * th * Q4;
#pragma unroll 4
      for (int e = threadIdx.x; e < dtotal; e += kDwThreads) {
        const int rr = fdiv(e, fq4), j = e - rr * Q4, pl = fdiv(rr, fthr), i = rr - pl * th;
        dsm[(pl * g.TH + i) * Q4 + j] = j < g.Q ? __ldg(yb + pl * ystride + (int64_t)(p0 + i) * g.Q + j) : 0.f;
      }
      __syncthreads();
      const int items = pp * th * nq;
      for (int e = threadIdx.x; e < items; e += kDwThreads) {
        const int rowall = fdiv(e, fnq), jq = e - rowall * nq;
        const int pl = fdiv(rowall, fthr), i = rowall - pl * th;
        const float4 d = *reinterpret_cast<const float4*>(dsm + (pl * g.TH + i) * Q4 + jq * 4);
        const float dv[4] = {d.x, d.y, d.z, d.w};
        const float* src = sm + (pl * g.IH + i * SH) * IW4 + jq * 4 * SH;
#pragma unroll
        for (int a = 0; a < 3; ++a) {
          const float* r = src + a * IW4;
          float v[4 * SH + 2];
          const float4 v0 = *reinterpret_cast<const float4*>(r);
          v[0] = v0.x; v[1] = v0.y; v[2] = v0.z; v[3] = v0.w;
          if (SH == 1) {
            const float2 v1 = *reinterpret_cast<const float2*>(r + 4);
            v[4] = v1.x; v[5] = v1.y;
          } else {
            const float4 v1 = *reinterpret_cast<const float4*>(r + 4);
            v[4] = v1.x; v[5] = v1.y; v[6] = v1.z; v[7] = v1.w;
            v[8] = r[8];
          }
#pragma unroll
          for (int o = 0; o < 4; ++o)
#pragma unroll
            for (int b = 0; b < 3; ++b) acc[a * 3 + b] = fmaf(dv[o], v[o * SH + b], acc[a * 3 + b]);
        }
      }
    }
  }
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
  for (int t = 0; t < 9; ++t) {
    float v = acc[t];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) red[wid][t] = v;
  }
  __syncthreads();
  if (threadIdx.x < 9) {
    float v = 0.f;
    for (int i = 0; i < kDwThreads / 32; ++i) v += red[i][threadIdx.x];
    part[((int64_t)c * gridDim.y + k) * 9 + threadIdx.x] = v;
  }
}

// ---------------------------------------------------------- weight grad
// CTA (channel c, image chunk k) over grid (C, chunks): for each of its
// images and each output tile, x's window and dY's tile are staged and each
// thread adds dY * x for all taps of its outputs; the per-tap sums are
// reduced over the block in a fixed order into part[c][k][tap].
template <int KR, int KS, int SH, int SW>
__global__ void __launch_bounds__(kDwThreads) dw_wgrad_tile_kernel(DwGeom g, const float* __restrict__ x,
                                                                   const float* __restrict__ dy, int per_chunk,
                                                                   float* __restrict__ part) {
  extern __shared__ float sm[];
  __shared__ float red[kDwThreads / 32][KR * KS];
  constexpr int RS = KR * KS;
  const int sh = SH ? SH : g.sh, sw = SW ? SW : g.sw;
  const int c = blockIdx.x, k = blockIdx.y;
  const int n0 = k * per_chunk, n1 = min(g.N, n0 + per_chunk);
  const int win = g.IH * g.IW;
  float* dsm = sm + win;  // dY tile [TH][TW]
  const int64_t HW = (int64_t)g.H * g.W, PQ = (int64_t)g.P * g.Q;
  const int tx = threadIdx.x, ty = threadIdx.y;
  float acc[RS];
#pragma unroll
  for (int t = 0; t < RS; ++t) acc[t] = 0.f;
  for (int n = n0; n < n1; ++n) {
    const float* xp = x + ((int64_t)n * g.C + c) * HW;
    const float* gp = dy + ((int64_t)n * g.C + c) * PQ;
    for (int tile = 0; tile < g.tiles_h * g.tiles_w; ++tile) {
      const int p0 = (tile / g.tiles_w) * g.TH, q0 = (tile % g.tiles_w) * g.TW;
      const int h0 = p0 * sh - g.ph, w0 = q0 * sw - g.pw;
      const int th = min(g.TH, g.P - p0), tw = min(g.TW, g.Q - q0);
      __syncthreads();  // the previous tile's values are no longer read
      for (int i = ty; i < g.IH; i += 8) {
        const int h = h0 + i;
        const bool hok = (unsigned)h < (unsigned)g.H;
#pragma unroll 4
        for (int j = tx; j < g.IW; j += 32) {
          const int ww = w0 + j;
          sm[i * g.IW + j] = hok && (unsigned)ww < (unsigned)g.W ? __ldg(xp + (int64_t)h * g.W + ww) : 0.f;
        }
      }
      for (int i = ty; i < th; i += 8)
#pragma unroll 4
        for (int j = tx; j < tw; j += 32) dsm[i * g.TW + j] = __ldg(gp + (int64_t)(p0 + i) * g.Q + q0 + j);
      __syncthreads();
      for (int i = ty; i < th; i += 8) {
        const float* row = sm + i * sh * g.IW;
        for (int j = tx; j < tw; j += 32) {
          const float d = dsm[i * g.TW + j];
          const float* base = row + j * sw;
#pragma unroll
          for (int a = 0; a < KR; ++a)
#pragma unroll
            for (int b = 0; b < KS; ++b)
              acc[a * KS + b] = fmaf(d, base[a * g.dh * g.IW + b * g.dw], acc[a * KS + b]);
        }
      }
    }
  }
  // block sums per tap: warp butterfly, then the warps' sums in order
  const int wid = ty;
#pragma unroll
  for (int t = 0; t < RS; ++t) {
    float v = acc[t];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (tx == 0) red[wid][t] = v;
  }
  __syncthreads();
  const int tid = ty * 32 + tx;
  if (tid < RS) {
    float v = 0.f;
    for (int i = 0; i < kDwThreads / 32; ++i) v += red[i][tid];
    part[((int64_t)c * gridDim.y + k) * RS + tid] = v;
  }
}

// dw[c][tap] = sum over chunks in order
__global__ void dw_wgrad_reduce_kernel(const float* __restrict__ part, int C, int chunks, int RS,
                                       float* __restrict__ dw) {
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= C * RS) return;
  const int c = e / RS, t = e - c * RS;
  float v = 0.f;
  for (int k = 0; k < chunks; ++k) v += part[((int64_t)c * chunks + k) * RS + t];
  dw[e] = v;
}

// ----------------------------------------------------------- host side
static DwGeom dw_geom(const pvb2_conv2d_desc* d, bool dgrad) {
  return dw_plan(d->N, d->C, d->H, d->W, d->P, d->Q, d->R, d->S, d->stride_h, d->stride_w, d->pad_h, d->pad_w,
                 d->dil_h, d->dil_w, dgrad);
}

// the tiled kernels take 3x3 and 5x5 filters whose staged windows fit
static bool dw_tiled_ok(const pvb2_conv2d_desc* d, bool dgrad) {
  if (!((d->R == 3 && d->S == 3) || (d->R == 5 && d->S == 5))) return false;
  const DwGeom g = dw_geom(d, dgrad);
  if (!dw_fits(g)) return false;
  const int64_t groups = ((int64_t)d->N * d->C + g.PP - 1) / g.PP;
  return groups * g.tiles_h * g.tiles_w < ((int64_t)1 << 31);
}

// image chunks of the weight gradient: about eight CTAs per SM, each taking
// a run of images of one channel
static int dw_chunks(const pvb2_conv2d_desc* d, int* per_chunk) {
  int chunks = std::max(1, std::min(d->N, (8 * num_sms() + d->C - 1) / std::max(d->C, 1)));
  *per_chunk = (d->N + chunks - 1) / chunks;
  chunks = (d->N + *per_chunk - 1) / *per_chunk;
  return std::min(chunks, 65535);
}

// scratch of the tiled weight gradient (0: the tiled path does not apply)
static bool dw3_ok(const pvb2_conv2d_desc* d);

size_t dw_wgrad_workspace(const pvb2_conv2d_desc* d) {
  const DwGeom g = dw_geom(d, false);
  if (!((d->R == 3 && d->S == 3) || (d->R == 5 && d->S == 5))) return 0;
  if (!dw3_ok(d) && g.IH * g.IW + g.TH * g.TW > kDwSmemFloats) return 0;
  int per = 0;
  const int chunks = dw_chunks(d, &per);
  return (size_t)d->C * chunks * d->R * d->S * sizeof(float);
}

// dw3_fwd4_kernel over planes H x W -> P x Q (3x3, dilation 1, stride st in
// both dimensions): about 1024 four-output items per CTA, whole planes when a
// plane has at most 512 items, else strips of rows; false when the staged
// rows do not fit
static bool dw3_plan(DwGeom& g, int st, int* iw4, FastDiv* fnq, FastDiv* fth) {
  const int nq = (g.Q + 3) / 4;
  *iw4 = (4 * nq * st + 3 + 3) / 4 * 4;
  auto ih = [&](int th) { return (th - 1) * st + 3; };
  if (g.P * nq <= 512) {
    g.TH = g.P;
    g.PP = std::max(1, 1024 / (g.P * nq));
    while (g.PP > 1 && g.PP * (ih(g.TH) * *iw4 + 9) > kDwSmemFloats) --g.PP;
  } else {
    g.PP = 1;
    g.TH = std::max(1, std::min(g.P, 1024 / nq));
    while (g.TH > 1 && ih(g.TH) * *iw4 + 9 > kDwSmemFloats) --g.TH;
  }
  g.IH = ih(g.TH);
  g.TW = g.Q;
  g.tiles_h = (g.P + g.TH - 1) / g.TH;
  g.tiles_w = 1;
  *fnq = fast_div(nq);
  *fth = fast_div(g.TH);
  return g.PP * (g.IH * *iw4 + 9) <= kDwSmemFloats && (int64_t)g.N * g.C * g.P * g.Q < ((int64_t)1 << 31);
}

static bool dw3_ok(const pvb2_conv2d_desc* d) {
  return d->R == 3 && d->S == 3 && d->dil_h == 1 && d->dil_w == 1 && d->stride_h == d->stride_w &&
         (d->stride_h == 1 || d->stride_h == 2);
}

template <bool FLIP>
static bool dw3_launch(DwGeom g, int st, const float* x, const float* w, const float* b, float* y, cudaStream_t s) {
  int iw4 = 0;
  FastDiv fnq, fth;
  if (!dw3_plan(g, st, &iw4, &fnq, &fth)) return false;
  const int64_t blocks = ((int64_t)g.N * g.C + g.PP - 1) / g.PP * g.tiles_h;
  if (blocks >= ((int64_t)1 << 31)) return false;
  const size_t smem = (size_t)g.PP * (g.IH * iw4 + 9) * sizeof(float);
  const FastDiv fiw4 = fast_div(iw4), fih = fast_div(g.IH);
  if (st == 1)
    dw3_fwd4_kernel<1, FLIP><<<(unsigned)blocks, kDwThreads, smem, s>>>(g, iw4, fnq, fth, fiw4, fih, x, w, b, y);
  else
    dw3_fwd4_kernel<2, FLIP><<<(unsigned)blocks, kDwThreads, smem, s>>>(g, iw4, fnq, fth, fiw4, fih, x, w, b, y);
  return true;
}

// *handled = false: not a shape the tiled kernels take (the caller runs the
// direct kernels)
int dw_fwd(const pvb2_conv2d_desc* d, const float* x, const float* w, const float* b, float* y, cudaStream_t s,
           bool* handled) {
  if (dw3_ok(d) && dw3_launch<false>(dw_geom(d, false), d->stride_h, x, w, b, y, s)) {
    PVB2_LAUNCH_CHECK();
    *handled = true;
    return PVB2_OK;
  }
  *handled = dw_tiled_ok(d, false);
  if (!*handled) return PVB2_OK;
  const DwGeom g = dw_geom(d, false);
  const int64_t blocks = ((int64_t)d->N * d->C + g.PP - 1) / g.PP * g.tiles_h * g.tiles_w;
  const size_t smem = (size_t)g.PP * (g.IH * g.IW + d->R * d->S) * sizeof(float);
  const dim3 blk(32, kDwThreads / 32);
  if (d->R == 3 && d->stride_h == 1 && d->stride_w == 1)
    dw_fwd_tile_kernel<3, 3, 1, 1><<<(unsigned)blocks, blk, smem, s>>>(g, x, w, b, y);
  else if (d->R == 3 && d->stride_h == 2 && d->stride_w == 2)
    dw_fwd_tile_kernel<3, 3, 2, 2><<<(unsigned)blocks, blk, smem, s>>>(g, x, w, b, y);
  else if (d->R == 3)
    dw_fwd_tile_kernel<3, 3, 0, 0><<<(unsigned)blocks, blk, smem, s>>>(g, x, w, b, y);
  else
    dw_fwd_tile_kernel<5, 5, 0, 0><<<(unsigned)blocks, blk, smem, s>>>(g, x, w, b, y);
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

int dw_dgrad(const pvb2_conv2d_desc* d, const float* dy, const float* w, float* dx, cudaStream_t s, bool* handled) {
  if (dw3_ok(d) && d->stride_h == 1) {
    // stride 1: the forward of dY with the flipped filter and padding 2 - pad
    DwGeom g = dw_geom(d, false);
    g.H = d->P;
    g.W = d->Q;
    g.P = d->H;
    g.Q = d->W;
    g.ph = 2 - d->pad_h;
    g.pw = 2 - d->pad_w;
    if (dw3_launch<true>(g, 1, dy, w, nullptr, dx, s)) {
      PVB2_LAUNCH_CHECK();
      *handled = true;
      return PVB2_OK;
    }
  }
  *handled = dw_tiled_ok(d, true);
  if (!*handled) return PVB2_OK;
  const DwGeom g = dw_geom(d, true);
  const int64_t blocks = ((int64_t)d->N * d->C + g.PP - 1) / g.PP * g.tiles_h * g.tiles_w;
  const size_t smem = (size_t)g.PP * (g.IH * g.IW + d->R * d->S) * sizeof(float);
  const dim3 blk(32, kDwThreads / 32);
  if (d->R == 3 && d->stride_h == 1 && d->stride_w == 1)
    dw_dgrad_tile_kernel<3, 3, 1, 1><<<(unsigned)blocks, blk, smem, s>>>(g, dy, w, dx);
  else if (d->R == 3 && d->stride_h == 2 && d->stride_w == 2)
    dw_dgrad_tile_kernel<3, 3, 2, 2><<<(unsigned)blocks, blk, smem, s>>>(g, dy, w, dx);
  else if (d->R == 3)
    dw_dgrad_tile_kernel<3, 3, 0, 0><<<(unsigned)blocks, blk, smem, s>>>(g, dy, w, dx);
  else
    dw_dgrad_tile_kernel<5, 5, 0, 0><<<(unsigned)blocks, blk, smem, s>>>(g, dy, w, dx);
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

// dw3_wgrad4_kernel's steps: about 1024 items per step, whole planes of up to
// `per` images when a plane has at most 512 items, else strips of rows
static bool dw3_wgrad_plan(const pvb2_conv2d_desc* d, int per, DwGeom& g, int* iw4) {
  g = dw_geom(d, false);
  const int st = d->stride_h, nq = (d->Q + 3) / 4, Q4 = nq * 4;
  *iw4 = (4 * nq * st + 3 + 3) / 4 * 4;
  auto ih = [&](int th) { return (th - 1) * st + 3; };
  auto fl = [&](int pp, int th) { return (int64_t)pp * (ih(th) * *iw4 + th * Q4); };
  if (d->P * nq <= 512) {
    g.TH = d->P;
    g.PP = std::max(1, std::min(per, 1024 / (d->P * nq)));
    while (g.PP > 1 && fl(g.PP, g.TH) > kDwSmemFloats) --g.PP;
  } else {
    g.PP = 1;
    g.TH = std::max(1, std::min(d->P, 1024 / nq));
    while (g.TH > 1 && fl(1, g.TH) > kDwSmemFloats) --g.TH;
  }
  g.IH = ih(g.TH);
  g.tiles_h = (d->P + g.TH - 1) / g.TH;
  return fl(g.PP, g.TH) <= kDwSmemFloats;
}

int dw_wgrad(const pvb2_conv2d_desc* d, const float* x, const float* dy, float* dw, void* ws, size_t ws_bytes,
             cudaStream_t s, bool* handled) {
  const size_t need = dw_wgrad_workspace(d);
  *handled = need > 0 && ws && ws_bytes >= need;
  if (!*handled) return PVB2_OK;
  if (dw3_ok(d)) {
    int per = 0, iw4 = 0;
    const int chunks = dw_chunks(d, &per);
    DwGeom g;
    if (dw3_wgrad_plan(d, per, g, &iw4)) {
      const int nq = (d->Q + 3) / 4;
      const size_t smem = (size_t)g.PP * (g.IH * iw4 + g.TH * nq * 4) * sizeof(float);
      const FastDiv fnq = fast_div(nq), fth = fast_div(g.TH), fiw4 = fast_div(iw4), fih = fast_div(g.IH),
                    fq4 = fast_div(nq * 4);
      float* part = (float*)ws;
      const dim3 grid((unsigned)d->C, (unsigned)chunks);
      if (d->stride_h == 1)
        dw3_wgrad4_kernel<1><<<grid, kDwThreads, smem, s>>>(g, iw4, fnq, fth, fiw4, fih, fq4, x, dy, per, part);
      else
        dw3_wgrad4_kernel<2><<<grid, kDwThreads, smem, s>>>(g, iw4, fnq, fth, fiw4, fih, fq4, x, dy, per, part);
      PVB2_LAUNCH_CHECK();
      dw_wgrad_reduce_kernel<<<grid_for((int64_t)d->C * 9, 256), 256, 0, s>>>(part, d->C, chunks, 9, dw);
      PVB2_LAUNCH_CHECK();
      return PVB2_OK;
    }
  }
  DwGeom g = dw_geom(d, false);
  g.PP = 1;
  int per = 0;
  const int chunks = dw_chunks(d, &per);
  float* part = (float*)ws;
  const dim3 grid((unsigned)d->C, (unsigned)chunks);
  const size_t smem = (size_t)(g.IH * g.IW + g.TH * g.TW) * sizeof(float);
  const dim3 blk(32, kDwThreads / 32);
  if (d->R == 3 && d->stride_h == 1 && d->stride_w == 1)
    dw_wgrad_tile_kernel<3, 3, 1, 1><<<grid, blk, smem, s>>>(g, x, dy, per, part);
  else if (d->R == 3 && d->stride_h == 2 && d->stride_w == 2)
    dw_wgrad_tile_kernel<3, 3, 2, 2><<<grid, blk, smem, s>>>(g, x, dy, per, part);
  else if (d->R == 3)
    dw_wgrad_tile_kernel<3, 3, 0, 0><<<grid, blk, smem, s>>>(g, x, dy, per, part);
  else
    dw_wgrad_tile_kernel<5, 5, 0, 0><<<grid, blk, smem, s>>>(g, x, dy, per, part);
  PVB2_LAUNCH_CHECK();
  const int RS = d->R * d->S;
  dw_wgrad_reduce_kernel<<<grid_for((int64_t)d->C * RS, 256), 256, 0, s>>>(part, d->C, chunks, RS, dw);
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

}  // namespace pvb2
