// Depthwise convolution (groups == C == K, one filter per channel);
// MobileNet-v2's 3x3 layers at stride 1 and 2.
//
// Replaces dlprim's grouped Conv2DForward / Conv2DBackwardData /
// Conv2DBackwardFilter as convolution_overrideable reached them with
// groups = C (src/vision_ops.cpp:30-59, 61-186).  All three are bound by
// HBM (4 B per input and output element, the filter is tiny).
//
//   3x3 (dilation 1, stride 1 or 2): direct register-blocked kernels, each
//   thread four adjacent outputs of a row from 16-byte global loads, the
//   overlap between neighbours served by L1 (dw3_*):
//     forward  over x; the stride-1 input gradient is the same kernel over
//              dY with the flipped filter and padding 2 - pad.
//     dgrad    stride 2 (pad 1) by sub-pixel phases: a thread makes a 2 x 8
//              block of dX from a 2 x 5 block of dY.
//     wgrad    CTA (channel, chunk of its (image, row, column-group) items)
//              sums dY * x per tap in registers, block-reduces in a fixed
//              order to partials [C][9][chunks], and one warp per (c, tap)
//              sums those in a fixed order, so the result depends only on
//              the shapes.
//   Other filters (5x5, other strides): shared-memory-staged tiles, each
//   CTA staging a tile of its input plane with its halo and every thread
//   computing its outputs from there (dw_*_tile_kernel); their weight
//   gradient writes partials [C][chunks][taps] summed in chunk order.
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

// ------------------------------------------------- 3x3 direct kernels
// 3x3 depthwise, dilation 1, stride SH in both dimensions (1 or 2), pad 0..2.
// Each thread computes an "item" of four adjacent outputs of one row
// straight from global memory: per filter row it loads the inputs the four
// windows span into registers (16-byte loads for the aligned interior when
// VEC) and does the 36 multiply-adds there.  Neighbouring items read
// overlapping inputs, which the L1 cache serves, so HBM sees each input about
// once.  There is no shared-memory staging and no barrier, so every thread's
// loads are in flight together and the warps of an SM overlap them; the
// staged version of these kernels (rows to shared memory, barrier, compute)
// ran at a third of the bandwidth.
//
// dw3_row: v[t] = row[c0 + t] for t <= 3*SH + 2 (the span of four windows),
// zero outside [0, W) or when the row lies outside the plane (rok false).
// VEC: pad 1, so c0 + 1 = 4*SH*jq, and the 4*SH columns from there lie inside
// the row (W a multiple of 4*SH, rows 16-byte aligned); they come as 16-byte
// loads, and the halo columns (c0, and c0 + 5 at stride 1) from the
// neighbouring lanes, which hold items jq - 1 and jq + 1 of the same row
// (items run jq fastest); only a lane at the warp's edge loads one itself,
// and at the row's ends the halo is padding.  Every lane of the warp must
// call it (it shuffles); a lane past the last item passes rok = false.
template <int SH, bool VEC>
__device__ __forceinline__ void dw3_row(const float* __restrict__ row, bool rok, int c0, int W, int jq, int nq,
                                        float (&v)[4 * SH + 2]) {
  if (VEC) {
    const int lane = threadIdx.x & 31;
    // the lanes that cannot take a halo column from a neighbour load it, in
    // the same batch as the 16-byte loads (not after the shuffles, which
    // would add a second memory round trip for the whole warp)
    const bool own_left = lane == 0 && jq > 0, own_right = SH == 1 && (lane == 31 || jq == nq - 1);
    const float eL = own_left && rok ? __ldg(row + c0) : 0.f;
    const float eR = own_right && rok && c0 + 5 < W ? __ldg(row + c0 + 5) : 0.f;
#pragma unroll
    for (int k = 0; k < SH; ++k) {
      float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
      if (rok) t = __ldg(reinterpret_cast<const float4*>(row + c0 + 1 + 4 * k));
      v[1 + 4 * k] = t.x;
      v[2 + 4 * k] = t.y;
      v[3 + 4 * k] = t.z;
      v[4 + 4 * k] = t.w;
    }
    const float left = __shfl_up_sync(0xffffffffu, v[4 * SH], 1);
    v[0] = jq == 0 ? 0.f : (lane > 0 ? left : eL);
    if (SH == 1) {
      const float right = __shfl_down_sync(0xffffffffu, v[1], 1);
      v[5] = own_right ? eR : right;
    } else {
      v[4 * SH + 1] = 0.f;  // stride 2 spans 4 * SH + 1 columns
    }
  } else {
#pragma unroll
    for (int t = 0; t < 4 * SH + 2; ++t) {
      const int c = c0 + t;
      v[t] = rok && t <= 3 * SH + 2 && (unsigned)c < (unsigned)W ? __ldg(row + c) : 0.f;
    }
  }
}

// Forward over planes [planes][H][W] into [planes][P][Q]; items in
// (plane, p, jq) order, jq fastest, so a warp's loads and stores run along
// rows.  FLIP reverses the filter: the stride-1 input gradient is this
// forward over dY with the flipped filter and padding 2 - pad.
template <int SH, bool FLIP, bool VEC>
__global__ void __launch_bounds__(kDwThreads) dw3_fwd_kernel(int items, int H, int W, int P, int Q, int ph, int pw,
                                                             FastDiv fpq, FastDiv fnq, FastDiv fc,
                                                             const float* __restrict__ x,
                                                             const float* __restrict__ w,
                                                             const float* __restrict__ bias, float* __restrict__ y) {
  // a lane past the last item computes item items - 1 with zero inputs and
  // stores nothing: it only takes part in dw3_row's shuffles
  const int e0 = blockIdx.x * kDwThreads + threadIdx.x;
  const bool valid = e0 < items;
  const int e = valid ? e0 : items - 1;
  const int plane = fdiv(e, fpq), rem = e - plane * fpq.d;
  const int p = fdiv(rem, fnq), jq = rem - p * fnq.d;
  const int c = plane - fdiv(plane, fc) * fc.d;
  float wk[9];
#pragma unroll
  for (int t = 0; t < 9; ++t) wk[t] = __ldg(w + c * 9 + (FLIP ? 8 - t : t));
  const float b0 = bias ? __ldg(bias + c) : 0.f;
  float acc[4] = {b0, b0, b0, b0};
  const float* xp = x + (int64_t)plane * H * W;
  const int h0 = p * SH - ph, c0 = jq * 4 * SH - pw;
#pragma unroll
  for (int a = 0; a < 3; ++a) {
    const int h = h0 + a;
    const bool rok = valid && (unsigned)h < (unsigned)H;
    float v[4 * SH + 2];
    dw3_row<SH, VEC>(xp + (int64_t)((unsigned)h < (unsigned)H ? h : 0) * W, rok, c0, W, jq, fnq.d, v);
#pragma unroll
    for (int o = 0; o < 4; ++o) {
      acc[o] = fmaf(v[o * SH], wk[a * 3], acc[o]);
      acc[o] = fmaf(v[o * SH + 1], wk[a * 3 + 1], acc[o]);
      acc[o] = fmaf(v[o * SH + 2], wk[a * 3 + 2], acc[o]);
    }
  }
  if (!valid) return;
  const int q0 = jq * 4;
  float* yr = y + (int64_t)plane * P * Q + (int64_t)p * Q + q0;
  if (VEC) {
    *reinterpret_cast<float4*>(yr) = make_float4(acc[0], acc[1], acc[2], acc[3]);
  } else {
#pragma unroll
    for (int o = 0; o < 4; ++o)
      if (q0 + o < Q) yr[o] = acc[o];
  }
}

// Stride-2 input gradient, pad 1, by sub-pixel phases: with
// y[p][q] = sum_ab x[2p-1+a][2q-1+b] w[a][b], the even rows of dX take filter
// row 1 of dY row i, the odd rows filter row 2 of dY row i and filter row 0
// of dY row i + 1 (columns alike).  An item is dX rows 2i, 2i+1 by columns
// 8j .. 8j+7, made from dY rows i, i+1, columns 4j .. 4j+4 (zero past the
// plane).  VEC: H = 2P, W = 2Q, Q a multiple of 4 (every store in range,
// 16-byte aligned).
template <bool VEC>
__global__ void __launch_bounds__(kDwThreads) dw3_s2_dgrad_kernel(int items, int H, int W, int P, int Q, FastDiv fij,
                                                                  FastDiv fnj, FastDiv fc,
                                                                  const float* __restrict__ dy,
                                                                  const float* __restrict__ w,
                                                                  float* __restrict__ dx) {
  // a lane past the last item takes part in the shuffles with zeros
  const int e0 = blockIdx.x * kDwThreads + threadIdx.x;
  const bool valid = e0 < items;
  const int e = valid ? e0 : items - 1;
  const int plane = fdiv(e, fij), rem = e - plane * fij.d;
  const int i = fdiv(rem, fnj), j = rem - i * fnj.d;
  const int c = plane - fdiv(plane, fc) * fc.d;
  float wk[9];
#pragma unroll
  for (int t = 0; t < 9; ++t) wk[t] = __ldg(w + c * 9 + t);
  const float* gp = dy + (int64_t)plane * P * Q;
  const int q0 = 4 * j;
  float d[2][5];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int pr = i + r;
    const bool rok = valid && pr < P;
    const float* row = gp + (int64_t)(pr < P ? pr : 0) * Q;
    if (VEC) {
      // column 4j + 4 is the next lane's first (item j + 1 of the same row),
      // padding past the row's last item; a lane at the warp's edge loads it
      const bool edge = (threadIdx.x & 31) == 31 && j < fnj.d - 1;
      const float eR = edge && rok ? __ldg(row + q0 + 4) : 0.f;
      float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
      if (rok) t = __ldg(reinterpret_cast<const float4*>(row + q0));
      d[r][0] = t.x;
      d[r][1] = t.y;
      d[r][2] = t.z;
      d[r][3] = t.w;
      const float right = __shfl_down_sync(0xffffffffu, t.x, 1);
      d[r][4] = j == fnj.d - 1 ? 0.f : (edge ? eR : right);
    } else {
#pragma unroll
      for (int u = 0; u < 5; ++u) d[r][u] = rok && q0 + u < Q ? __ldg(row + q0 + u) : 0.f;
    }
  }
  if (!valid) return;
  float ev[8], od[8];  // dX rows 2i and 2i + 1
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    ev[2 * u] = d[0][u] * wk[4];
    ev[2 * u + 1] = fmaf(d[0][u + 1], wk[3], d[0][u] * wk[5]);
    od[2 * u] = fmaf(d[1][u], wk[1], d[0][u] * wk[7]);
    od[2 * u + 1] = fmaf(d[1][u + 1], wk[0], fmaf(d[1][u], wk[2], fmaf(d[0][u + 1], wk[6], d[0][u] * wk[8])));
  }
  const int h = 2 * i, w0 = 8 * j;
  float* xr = dx + (int64_t)plane * H * W + (int64_t)h * W + w0;
  if (VEC) {
    *reinterpret_cast<float4*>(xr) = make_float4(ev[0], ev[1], ev[2], ev[3]);
    *reinterpret_cast<float4*>(xr + 4) = make_float4(ev[4], ev[5], ev[6], ev[7]);
    *reinterpret_cast<float4*>(xr + W) = make_float4(od[0], od[1], od[2], od[3]);
    *reinterpret_cast<float4*>(xr + W + 4) = make_float4(od[4], od[5], od[6], od[7]);
  } else {
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (w0 + u < W) {
        xr[u] = ev[u];
        if (h + 1 < H) xr[W + u] = od[u];
      }
  }
}

// Weight gradient: CTA (channel c, chunk k) over grid (C, J) sums, for its
// items (n, p, jq) of channel c, dY[n][c][p][4jq..] * x under each of the 9
// taps in registers, then reduces them over the block in a fixed order into
// part[(c * 9 + tap) * J + k]; dw3_wgrad_reduce_kernel sums the J partials.
template <int SH, bool VEC>
__global__ void __launch_bounds__(kDwThreads) dw3_wgrad_kernel(int C, int H, int W, int P, int Q, int ph, int pw,
                                                               int total, int per, FastDiv fpq, FastDiv fnq,
                                                               const float* __restrict__ x,
                                                               const float* __restrict__ dy,
                                                               float* __restrict__ part) {
  __shared__ float red[kDwThreads / 32][9];
  const int c = blockIdx.x, k = blockIdx.y;
  const int e0 = k * per, e1 = min(total, e0 + per);
  const int64_t HW = (int64_t)H * W, PQ = (int64_t)P * Q;
  float acc[9];
#pragma unroll
  for (int t = 0; t < 9; ++t) acc[t] = 0.f;
  // every thread runs the same number of iterations (dw3_row shuffles); a
  // lane past e1 loads the inputs of its item (the chunk may end inside a
  // row, and the last item's halo column comes from that lane) but adds
  // nothing (zero dY); past the last item of all it takes that one
  for (int base = e0; base < e1; base += kDwThreads) {
    const bool valid = base + (int)threadIdx.x < e1;
    const int e = min(base + (int)threadIdx.x, total - 1);
    const int n = fdiv(e, fpq), rem = e - n * fpq.d;
    const int p = fdiv(rem, fnq), jq = rem - p * fnq.d;
    const int64_t plane = (int64_t)n * C + c;
    const int q0 = jq * 4;
    const float* gr = dy + plane * PQ + (int64_t)p * Q + q0;
    float dv[4] = {0.f, 0.f, 0.f, 0.f};
    if (VEC) {
      if (valid) {
        const float4 t = __ldg(reinterpret_cast<const float4*>(gr));
        dv[0] = t.x;
        dv[1] = t.y;
        dv[2] = t.z;
        dv[3] = t.w;
      }
    } else {
#pragma unroll
      for (int o = 0; o < 4; ++o) dv[o] = valid && q0 + o < Q ? __ldg(gr + o) : 0.f;
    }
    const float* xp = x + plane * HW;
    const int h0 = p * SH - ph, c0 = jq * 4 * SH - pw;
#pragma unroll
    for (int a = 0; a < 3; ++a) {
      const int h = h0 + a;
      const bool rok = (unsigned)h < (unsigned)H;
      float v[4 * SH + 2];
      dw3_row<SH, VEC>(xp + (int64_t)(rok ? h : 0) * W, rok, c0, W, jq, fnq.d, v);
#pragma unroll
      for (int o = 0; o < 4; ++o)
#pragma unroll
        for (int b = 0; b < 3; ++b) acc[a * 3 + b] = fmaf(dv[o], v[o * SH + b], acc[a * 3 + b]);
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
    part[((int64_t)c * 9 + threadIdx.x) * gridDim.y + k] = v;
  }
}

// dw[c * 9 + tap] = the J partials of (c, tap), one warp each: lane l sums
// partials l, l + 32, ... in order, then a fixed butterfly (the result
// depends only on the shapes)
__global__ void dw3_wgrad_reduce_kernel(const float* __restrict__ part, int rows, int J, float* __restrict__ dw) {
  const int r = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (r >= rows) return;
  const float* pr = part + (int64_t)r * J;
  float v = 0.f;
  for (int i = lane; i < J; i += 32) v += pr[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if (lane == 0) dw[r] = v;
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

// ---------------------------------------------- 3x3 direct: host side
// 3x3, dilation 1, equal strides of 1 or 2, pads up to 2 (the stride-1 input
// gradient runs as a forward with padding 2 - pad)
static bool dw3_ok(const pvb2_conv2d_desc* d) {
  return d->R == 3 && d->S == 3 && d->dil_h == 1 && d->dil_w == 1 && d->stride_h == d->stride_w &&
         (d->stride_h == 1 || d->stride_h == 2) && d->pad_h >= 0 && d->pad_h <= 2 && d->pad_w >= 0 &&
         d->pad_w <= 2;
}

static bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

// the 16-byte paths of dw3_row and the four-output stores: pad 1, rows and
// planes 16-byte aligned, every item's interior inside the row
static bool dw3_vec(int W, int Q, int st, int pw, const void* a, const void* b) {
  return pw == 1 && W % 4 == 0 && Q % 4 == 0 && W >= st * Q && aligned16(a) && aligned16(b);
}

// forward over [planes][H][W] -> [planes][P][Q] with stride st and pads
// (ph, pw); false when the item count does not fit an int
template <bool FLIP>
static bool dw3_launch(int64_t planes, int C, int H, int W, int P, int Q, int st, int ph, int pw, const float* x,
                       const float* w, const float* b, float* y, cudaStream_t s) {
  const int nq = (Q + 3) / 4;
  const int64_t items = planes * P * nq;
  if (items >= ((int64_t)1 << 31) - kDwThreads) return false;
  const unsigned blocks = (unsigned)((items + kDwThreads - 1) / kDwThreads);
  const FastDiv fpq = fast_div(P * nq), fnq = fast_div(nq), fc = fast_div(C);
  const bool vec = dw3_vec(W, Q, st, pw, x, y);
#define PVB2_DW3_FWD(SH, V)                                                                                        \
  dw3_fwd_kernel<SH, FLIP, V><<<blocks, kDwThreads, 0, s>>>((int)items, H, W, P, Q, ph, pw, fpq, fnq, fc, x, w, b, \
                                                            y)
  if (st == 1) {
    if (vec) PVB2_DW3_FWD(1, true);
    else PVB2_DW3_FWD(1, false);
  } else {
    if (vec) PVB2_DW3_FWD(2, true);
    else PVB2_DW3_FWD(2, false);
  }
#undef PVB2_DW3_FWD
  return true;
}

// weight-gradient chunks per channel: about eight CTAs per SM in all, each
// with at least eight items per thread
static int dw3_wgrad_chunks(const pvb2_conv2d_desc* d, int* per) {
  const int64_t total = (int64_t)d->N * d->P * ((d->Q + 3) / 4);
  const int64_t most = std::max<int64_t>(1, total / (8 * kDwThreads));
  int64_t J = std::min<int64_t>(most, std::max(1, (8 * num_sms() + d->C - 1) / std::max(d->C, 1)));
  J = std::min<int64_t>(J, 65535);
  *per = (int)((total + J - 1) / J);
  return (int)((total + *per - 1) / *per);
}

static bool dw3_wgrad_ok(const pvb2_conv2d_desc* d) {
  return dw3_ok(d) && (int64_t)d->N * d->P * ((d->Q + 3) / 4) < ((int64_t)1 << 31) - kDwThreads;
}

// image chunks of the tiled weight gradient: about eight CTAs per SM, each
// taking a run of images of one channel
static int dw_chunks(const pvb2_conv2d_desc* d, int* per_chunk) {
  int chunks = std::max(1, std::min(d->N, (8 * num_sms() + d->C - 1) / std::max(d->C, 1)));
  *per_chunk = (d->N + chunks - 1) / chunks;
  chunks = (d->N + *per_chunk - 1) / *per_chunk;
  return std::min(chunks, 65535);
}

// scratch of the weight gradient (0: neither the direct nor the tiled path
// applies)
size_t dw_wgrad_workspace(const pvb2_conv2d_desc* d) {
  if (dw3_wgrad_ok(d)) {
    int per = 0;
    return (size_t)d->C * 9 * dw3_wgrad_chunks(d, &per) * sizeof(float);
  }
  const DwGeom g = dw_geom(d, false);
  if (!((d->R == 3 && d->S == 3) || (d->R == 5 && d->S == 5))) return 0;
  if (g.IH * g.IW + g.TH * g.TW > kDwSmemFloats) return 0;
  int per = 0;
  const int chunks = dw_chunks(d, &per);
  return (size_t)d->C * chunks * d->R * d->S * sizeof(float);
}

// *handled = false: not a shape the direct or tiled kernels take (the
// caller runs the generic kernels)
int dw_fwd(const pvb2_conv2d_desc* d, const float* x, const float* w, const float* b, float* y, cudaStream_t s,
           bool* handled) {
  if (dw3_ok(d) && dw3_launch<false>((int64_t)d->N * d->C, d->C, d->H, d->W, d->P, d->Q, d->stride_h, d->pad_h,
                                     d->pad_w, x, w, b, y, s)) {
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
  // stride 1: the forward of dY with the flipped filter and padding 2 - pad
  if (dw3_ok(d) && d->stride_h == 1 &&
      dw3_launch<true>((int64_t)d->N * d->C, d->C, d->P, d->Q, d->H, d->W, 1, 2 - d->pad_h, 2 - d->pad_w, dy, w,
                       nullptr, dx, s)) {
    PVB2_LAUNCH_CHECK();
    *handled = true;
    return PVB2_OK;
  }
  // stride 2, pad 1: sub-pixel phases, an item of 2 x 8 dX outputs a thread
  if (dw3_ok(d) && d->stride_h == 2 && d->pad_h == 1 && d->pad_w == 1) {
    const int ir = (d->H + 1) / 2, nj = (d->W + 7) / 8;
    const int64_t items = (int64_t)d->N * d->C * ir * nj;
    if (items < ((int64_t)1 << 31) - kDwThreads) {
      const unsigned blocks = (unsigned)((items + kDwThreads - 1) / kDwThreads);
      const FastDiv fij = fast_div(ir * nj), fnj = fast_div(nj), fc = fast_div(d->C);
      const bool vec = d->H == 2 * d->P && d->W == 2 * d->Q && d->Q % 4 == 0 && aligned16(dy) && aligned16(dx);
      if (vec)
        dw3_s2_dgrad_kernel<true><<<blocks, kDwThreads, 0, s>>>((int)items, d->H, d->W, d->P, d->Q, fij, fnj, fc,
                                                                dy, w, dx);
      else
        dw3_s2_dgrad_kernel<false><<<blocks, kDwThreads, 0, s>>>((int)items, d->H, d->W, d->P, d->Q, fij, fnj, fc,
                                                                 dy, w, dx);
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

int dw_wgrad(const pvb2_conv2d_desc* d, const float* x, const float* dy, float* dw, void* ws, size_t ws_bytes,
             cudaStream_t s, bool* handled) {
  const size_t need = dw_wgrad_workspace(d);
  *handled = need > 0 && ws && ws_bytes >= need;
  if (!*handled) return PVB2_OK;
  float* part = (float*)ws;
  if (dw3_wgrad_ok(d)) {
    int per = 0;
    const int J = dw3_wgrad_chunks(d, &per);
    const int nq = (d->Q + 3) / 4, total = d->N * d->P * nq;
    const FastDiv fpq = fast_div(d->P * nq), fnq = fast_div(nq);
    const bool vec = dw3_vec(d->W, d->Q, d->stride_h, d->pad_w, x, dy);
    const dim3 grid((unsigned)d->C, (unsigned)J);
#define PVB2_DW3_WG(SH, V)                                                                                   \
  dw3_wgrad_kernel<SH, V><<<grid, kDwThreads, 0, s>>>(d->C, d->H, d->W, d->P, d->Q, d->pad_h, d->pad_w, total, \
                                                      per, fpq, fnq, x, dy, part)
    if (d->stride_h == 1) {
      if (vec) PVB2_DW3_WG(1, true);
      else PVB2_DW3_WG(1, false);
    } else {
      if (vec) PVB2_DW3_WG(2, true);
      else PVB2_DW3_WG(2, false);
    }
#undef PVB2_DW3_WG
    PVB2_LAUNCH_CHECK();
    const int rows = d->C * 9;
    dw3_wgrad_reduce_kernel<<<(rows + 7) / 8, 256, 0, s>>>(part, rows, J, dw);
    PVB2_LAUNCH_CHECK();
    return PVB2_OK;
  }
  DwGeom g = dw_geom(d, false);
  g.PP = 1;
  int per = 0;
  const int chunks = dw_chunks(d, &per);
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
