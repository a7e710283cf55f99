// Reductions over arbitrary dims: sum / mean / prod / max / min / argmax /
// argmin / sum of squares.
//
// Replaces dlprim::core::PointwiseOperationBroadcastReduce as used by
// red_op_out (src/pointwise_ops.cpp:501-555), amax/amin/argmax
// (:1030-1102) and the bias/gamma/beta gradient sums in norm_ops.cpp and
// vision_ops.cpp.  Reduction order is a fixed tree, so results are
// deterministic run to run.
#include "common.cuh"

namespace pvb2 {

struct RedShape {
  // kept dims: iterate outputs; reduced dims: iterate inputs per output
  int kdim;
  int64_t ksizes[PVB2_MAX_DIMS];
  int64_t k_in_strides[PVB2_MAX_DIMS];
  int64_t k_out_strides[PVB2_MAX_DIMS];
  int rdim;
  int64_t rsizes[PVB2_MAX_DIMS];
  int64_t r_in_strides[PVB2_MAX_DIMS];
};

template <typename T>
struct Acc {
  T v;
  int64_t idx;
};

template <typename T>
__device__ __forceinline__ Acc<T> red_init(int op) {
  Acc<T> a;
  a.idx = -1;
  switch (op) {
    case PVB2_RED_PROD: a.v = (T)1; break;
    case PVB2_RED_MAX:
    case PVB2_RED_ARGMAX: a.v = std::numeric_limits<T>::lowest(); break;
    case PVB2_RED_MIN:
    case PVB2_RED_ARGMIN: a.v = std::numeric_limits<T>::max(); break;
    default: a.v = (T)0;
  }
  if constexpr (std::is_floating_point<T>::value) {
    if (op == PVB2_RED_MAX || op == PVB2_RED_ARGMAX) a.v = -std::numeric_limits<T>::infinity();
    if (op == PVB2_RED_MIN || op == PVB2_RED_ARGMIN) a.v = std::numeric_limits<T>::infinity();
  }
  return a;
}

template <typename T>
__device__ __forceinline__ bool isnan_(T x) {
  if constexpr (std::is_floating_point<T>::value) return x != x;
  else return false;
}

// combine, keeping the first index on ties and propagating NaN (NaN wins,
// first NaN kept), matching torch's CPU semantics.
template <typename T>
__device__ __forceinline__ Acc<T> red_combine(int op, Acc<T> a, Acc<T> b) {
  switch (op) {
    case PVB2_RED_SUM:
    case PVB2_RED_SUMSQ: a.v = a.v + b.v; return a;
    case PVB2_RED_PROD: a.v = a.v * b.v; return a;
    case PVB2_RED_MAX:
    case PVB2_RED_ARGMAX: {
      if (b.idx < 0 && op == PVB2_RED_ARGMAX) return a;
      if (a.idx < 0 && op == PVB2_RED_ARGMAX) return b;
      bool an = isnan_(a.v), bn = isnan_(b.v);
      if (an || bn) {
        if (an && bn) return a.idx <= b.idx ? a : b;
        return an ? a : b;
      }
      if (b.v > a.v || (b.v == a.v && b.idx < a.idx)) return b;
      return a;
    }
    case PVB2_RED_MIN:
    case PVB2_RED_ARGMIN: {
      if (b.idx < 0 && op == PVB2_RED_ARGMIN) return a;
      if (a.idx < 0 && op == PVB2_RED_ARGMIN) return b;
      bool an = isnan_(a.v), bn = isnan_(b.v);
      if (an || bn) {
        if (an && bn) return a.idx <= b.idx ? a : b;
        return an ? a : b;
      }
      if (b.v < a.v || (b.v == a.v && b.idx < a.idx)) return b;
      return a;
    }
  }
  return a;
}

template <typename T>
__device__ __forceinline__ Acc<T> red_elem(int op, T x, int64_t idx) {
  Acc<T> a;
  a.v = op == PVB2_RED_SUMSQ ? x * x : x;
  a.idx = idx;
  return a;
}

template <typename T>
__device__ __forceinline__ Acc<T> shfl_down(Acc<T> a, int off) {
  Acc<T> b;
  b.v = __shfl_down_sync(0xffffffffu, a.v, off);
  b.idx = __shfl_down_sync(0xffffffffu, a.idx, off);
  return b;
}

__device__ __forceinline__ int64_t offset_of(int nd, const int64_t* sizes, const int64_t* strides, int64_t lin) {
  int64_t off = 0;
  for (int d = nd - 1; d >= 0; --d) {
    int64_t sz = sizes[d];
    off += (lin % sz) * strides[d];
    lin /= sz;
  }
  return off;
}

// one block per output element; threads split the reduced index space
template <typename T>
__global__ void reduce_row_kernel(RedShape rs, int op, const void* in, int idt, void* out, int odt, int64_t n_out,
                                  int64_t n_red, T scale) {
  __shared__ Acc<T> warp_acc[32];
  for (int64_t o = blockIdx.x; o < n_out; o += gridDim.x) {
    const int64_t base_in = offset_of(rs.kdim, rs.ksizes, rs.k_in_strides, o);
    const int64_t off_out = offset_of(rs.kdim, rs.ksizes, rs.k_out_strides, o);
    Acc<T> acc = red_init<T>(op);
    for (int64_t r = threadIdx.x; r < n_red; r += blockDim.x) {
      int64_t off = base_in + offset_of(rs.rdim, rs.rsizes, rs.r_in_strides, r);
      acc = red_combine<T>(op, acc, red_elem<T>(op, load_as<T>(in, off, idt), r));
    }
    for (int s = 16; s > 0; s >>= 1) acc = red_combine<T>(op, acc, shfl_down(acc, s));
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    if (lane == 0) warp_acc[wid] = acc;
    __syncthreads();
    if (wid == 0) {
      const int nw = blockDim.x >> 5;
      acc = lane < nw ? warp_acc[lane] : red_init<T>(op);
      for (int s = 16; s > 0; s >>= 1) acc = red_combine<T>(op, acc, shfl_down(acc, s));
      if (lane == 0) {
        if (op == PVB2_RED_ARGMAX || op == PVB2_RED_ARGMIN) store_as<int64_t>(out, off_out, odt, acc.idx < 0 ? 0 : acc.idx);
        else store_as<T>(out, off_out, odt, (op == PVB2_RED_SUM || op == PVB2_RED_SUMSQ) ? acc.v * scale : acc.v);
      }
    }
    __syncthreads();
  }
}

// column mode: consecutive outputs are consecutive in memory; threads in x
// own outputs, threads in y split the reduced range, combined in smem.
template <typename T>
__global__ void reduce_col_kernel(RedShape rs, int op, const void* in, int idt, void* out, int odt, int64_t n_out,
                                  int64_t n_red, T scale) {
  __shared__ Acc<T> part[8][33];
  const int64_t o = (int64_t)blockIdx.x * 32 + threadIdx.x;
  Acc<T> acc = red_init<T>(op);
  int64_t base_in = 0;
  if (o < n_out) {
    base_in = offset_of(rs.kdim, rs.ksizes, rs.k_in_strides, o);
    for (int64_t r = threadIdx.y; r < n_red; r += blockDim.y) {
      int64_t off = base_in + offset_of(rs.rdim, rs.rsizes, rs.r_in_strides, r);
      acc = red_combine<T>(op, acc, red_elem<T>(op, load_as<T>(in, off, idt), r));
    }
  }
  part[threadIdx.y][threadIdx.x] = acc;
  __syncthreads();
  if (threadIdx.y == 0 && o < n_out) {
    for (int k = 1; k < (int)blockDim.y; ++k) acc = red_combine<T>(op, acc, part[k][threadIdx.x]);
    const int64_t off_out = offset_of(rs.kdim, rs.ksizes, rs.k_out_strides, o);
    if (op == PVB2_RED_ARGMAX || op == PVB2_RED_ARGMIN) store_as<int64_t>(out, off_out, odt, acc.idx < 0 ? 0 : acc.idx);
    else store_as<T>(out, off_out, odt, (op == PVB2_RED_SUM || op == PVB2_RED_SUMSQ) ? acc.v * scale : acc.v);
  }
}

// ---------------------------------------------------------------- 2-D paths
// After adjacent dims are merged, most reductions are one of
//   column: out[c] = red_r in[r * rstride + c]      (bias / gamma gradients)
//   row:    out[k] = red_r in[k * kstride + r]      (last-dim reductions, full sums)
// with a single reduced stride.  These walk pointers (no index division) and
// may split the reduced range over S blocks: block s reduces its chunk into
// partial[s][k], and red_partials_kernel combines the S partials of each
// output in order s = 0..S-1, so the result depends only on the shape.

template <typename T>
__device__ __forceinline__ T vinit(int op) {
  switch (op) {
    case PVB2_RED_PROD: return (T)1;
    case PVB2_RED_MAX: return -std::numeric_limits<T>::infinity();
    case PVB2_RED_MIN: return std::numeric_limits<T>::infinity();
  }
  return (T)0;
}

// NaN wins for max / min, as in red_combine
template <typename T>
__device__ __forceinline__ T vcombine(int op, T a, T b) {
  switch (op) {
    case PVB2_RED_PROD: return a * b;
    case PVB2_RED_MAX: return a != a ? a : (b != b ? b : (b > a ? b : a));
    case PVB2_RED_MIN: return a != a ? a : (b != b ? b : (b < a ? b : a));
  }
  return a + b;
}

template <typename T>
__device__ __forceinline__ T velem(int op, T x) {
  return op == PVB2_RED_SUMSQ ? x * x : x;
}

template <typename T>
__device__ __forceinline__ T vfinal(int op, T v, T scale) {
  return (op == PVB2_RED_SUM || op == PVB2_RED_SUMSQ) ? v * scale : v;
}

struct Red2d {
  int64_t n_out, n_red;
  int64_t kstride_in, kstride_out;  // kept dim (column mode: kstride_in == 1)
  int64_t rstride;                  // reduced dim (row mode: rstride == 1)
  int64_t chunk;                    // reduced elements per split
  int splits;
};

// block (32, 8): x = column, y = row lane; grid (ceil(n_out / 32), splits)
template <typename T>
__global__ void __launch_bounds__(256) red2d_col_kernel(Red2d g, int op, const T* __restrict__ in, void* out,
                                                        int odt, T* __restrict__ partial, T scale) {
  __shared__ T part[8][33];
  const int64_t c = (int64_t)blockIdx.x * 32 + threadIdx.x;
  const int64_t r0 = (int64_t)blockIdx.y * g.chunk;
  const int64_t r1 = min(g.n_red, r0 + g.chunk);
  T acc = vinit<T>(op);
  if (c < g.n_out) {
    const T* p = in + c + (r0 + threadIdx.y) * g.rstride;
    const int64_t step = 8 * g.rstride;
    int64_t r = r0 + threadIdx.y;
    for (; r + 24 < r1; r += 32, p += 4 * step) {
      const T x0 = __ldg(p), x1 = __ldg(p + step), x2 = __ldg(p + 2 * step), x3 = __ldg(p + 3 * step);
      acc = vcombine<T>(op, acc, velem<T>(op, x0));
      acc = vcombine<T>(op, acc, velem<T>(op, x1));
      acc = vcombine<T>(op, acc, velem<T>(op, x2));
      acc = vcombine<T>(op, acc, velem<T>(op, x3));
    }
    for (; r < r1; r += 8, p += step) acc = vcombine<T>(op, acc, velem<T>(op, __ldg(p)));
  }
  part[threadIdx.y][threadIdx.x] = acc;
  __syncthreads();
  if (threadIdx.y == 0 && c < g.n_out) {
#pragma unroll
    for (int k = 1; k < 8; ++k) acc = vcombine<T>(op, acc, part[k][threadIdx.x]);
    if (g.splits > 1) partial[(int64_t)blockIdx.y * g.n_out + c] = acc;
    else store_as<T>(out, c * g.kstride_out, odt, vfinal<T>(op, acc, scale));
  }
}

// one warp per output row (short rows); 8 rows per 256-thread block
template <typename T>
__global__ void __launch_bounds__(256) red2d_row_warp_kernel(Red2d g, int op, const T* __restrict__ in, void* out,
                                                             int odt, T scale) {
  const int64_t k = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (k >= g.n_out) return;
  const T* p = in + k * g.kstride_in;
  T acc = vinit<T>(op);
  for (int64_t r = lane; r < g.n_red; r += 32) acc = vcombine<T>(op, acc, velem<T>(op, __ldg(p + r)));
  for (int s = 16; s > 0; s >>= 1) acc = vcombine<T>(op, acc, __shfl_down_sync(0xffffffffu, acc, s));
  if (lane == 0) store_as<T>(out, k * g.kstride_out, odt, vfinal<T>(op, acc, scale));
}

// one 256-thread block per (output row, split)
template <typename T>
__global__ void __launch_bounds__(256) red2d_row_block_kernel(Red2d g, int op, const T* __restrict__ in, void* out,
                                                              int odt, T* __restrict__ partial, T scale) {
  __shared__ T wacc[8];
  const int64_t k = blockIdx.x;
  const int64_t r0 = (int64_t)blockIdx.y * g.chunk;
  const int64_t r1 = min(g.n_red, r0 + g.chunk);
  const T* p = in + k * g.kstride_in;
  T acc = vinit<T>(op);
  int64_t r = r0 + threadIdx.x;
  for (; r + 768 < r1; r += 1024) {
    const T x0 = __ldg(p + r), x1 = __ldg(p + r + 256), x2 = __ldg(p + r + 512), x3 = __ldg(p + r + 768);
    acc = vcombine<T>(op, acc, velem<T>(op, x0));
    acc = vcombine<T>(op, acc, velem<T>(op, x1));
    acc = vcombine<T>(op, acc, velem<T>(op, x2));
    acc = vcombine<T>(op, acc, velem<T>(op, x3));
  }
  for (; r < r1; r += 256) acc = vcombine<T>(op, acc, velem<T>(op, __ldg(p + r)));
  for (int s = 16; s > 0; s >>= 1) acc = vcombine<T>(op, acc, __shfl_down_sync(0xffffffffu, acc, s));
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) wacc[wid] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    acc = wacc[0];
#pragma unroll
    for (int w = 1; w < 8; ++w) acc = vcombine<T>(op, acc, wacc[w]);
    if (g.splits > 1) partial[(int64_t)blockIdx.y * g.n_out + k] = acc;
    else store_as<T>(out, k * g.kstride_out, odt, vfinal<T>(op, acc, scale));
  }
}

// out[k] = final(combine_s partial[s][k]); one warp per output, lanes take
// s = lane, lane + 32, ... and a fixed shuffle tree joins them
template <typename T>
__global__ void __launch_bounds__(256) red_partials_kernel(Red2d g, int op, const T* __restrict__ partial, void* out,
                                                           int odt, T scale) {
  const int64_t k = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (k >= g.n_out) return;
  T acc = vinit<T>(op);
  for (int s = lane; s < g.splits; s += 32) acc = vcombine<T>(op, acc, partial[(int64_t)s * g.n_out + k]);
  for (int s = 16; s > 0; s >>= 1) acc = vcombine<T>(op, acc, __shfl_down_sync(0xffffffffu, acc, s));
  if (lane == 0) store_as<T>(out, k * g.kstride_out, odt, vfinal<T>(op, acc, scale));
}

enum { kRedGeneric = 0, kRedCol = 1, kRedRowWarp = 2, kRedRowBlock = 3 };

template <typename T>
static int launch_red2d(int mode, const Red2d& g, int op, const void* in, const pvb2_tensor* out, void* partial,
                        double scale, cudaStream_t s) {
  T* part = static_cast<T*>(partial);
  const T* x = static_cast<const T*>(in);
  if (mode == kRedCol) {
    dim3 grid((unsigned)((g.n_out + 31) / 32), (unsigned)g.splits);
    red2d_col_kernel<T><<<grid, dim3(32, 8), 0, s>>>(g, op, x, out->data, out->dtype, part, (T)scale);
  } else if (mode == kRedRowWarp) {
    red2d_row_warp_kernel<T><<<(unsigned)((g.n_out + 7) / 8), 256, 0, s>>>(g, op, x, out->data, out->dtype,
                                                                           (T)scale);
  } else {
    dim3 grid((unsigned)g.n_out, (unsigned)g.splits);
    red2d_row_block_kernel<T><<<grid, 256, 0, s>>>(g, op, x, out->data, out->dtype, part, (T)scale);
  }
  PVB2_LAUNCH_CHECK();
  if (g.splits > 1) {
    red_partials_kernel<T><<<(unsigned)((g.n_out + 7) / 8), 256, 0, s>>>(g, op, part, out->data, out->dtype,
                                                                         (T)scale);
    PVB2_LAUNCH_CHECK();
  }
  return PVB2_OK;
}

template <typename T>
static int launch_reduce(const RedShape& rs, bool col, int op, const pvb2_tensor* in, const pvb2_tensor* out,
                         int64_t n_out, int64_t n_red, double scale, cudaStream_t s) {
  if (col) {
    dim3 block(32, 8);
    int64_t g = (n_out + 31) / 32;
    reduce_col_kernel<T><<<(unsigned)g, block, 0, s>>>(rs, op, in->data, in->dtype, out->data, out->dtype, n_out,
                                                       n_red, (T)scale);
  } else {
    int threads = n_red >= 1024 ? 512 : (n_red >= 256 ? 256 : (n_red >= 64 ? 64 : 32));
    int64_t g = std::min<int64_t>(n_out, (int64_t)num_sms() * 32);
    reduce_row_kernel<T><<<(unsigned)g, threads, 0, s>>>(rs, op, in->data, in->dtype, out->data, out->dtype, n_out,
                                                         n_red, (T)scale);
  }
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

}  // namespace pvb2

using namespace pvb2;

namespace pvb2 {

struct RedPlan {
  RedShape rs;
  int64_t n_out = 1, n_red = 1;
  bool col = false;  // generic kernels: inner memory dim is kept
  int mode = kRedGeneric;
  Red2d g;
  size_t elem = 0;  // partial element size when splitting
};

// Classify dims (kept / reduced), merge neighbours that are contiguous with
// one another, and pick a kernel.  Identical for the size query and the launch.
static int plan_reduce(int op, const pvb2_tensor* out, const pvb2_tensor* in, int compute_dtype, RedPlan& P) {
  PVB2_CHECK_ARG(out->ndim == in->ndim, "pvb2_reduce: out must keep reduced dims (ndim %d vs %d)", out->ndim,
                 in->ndim);
  RedShape& rs = P.rs;
  rs.kdim = 0;
  rs.rdim = 0;
  int inner_mem_dim = -1;
  int64_t best = INT64_MAX;
  for (int d = 0; d < in->ndim; ++d) {
    if (in->sizes[d] != 1 && in->strides[d] != 0 && in->strides[d] < best) {
      best = in->strides[d];
      inner_mem_dim = d;
    }
  }
  // merged dims, outermost first
  int nm = 0;
  bool mk[PVB2_MAX_DIMS];
  int64_t msz[PVB2_MAX_DIMS], mis[PVB2_MAX_DIMS], mos[PVB2_MAX_DIMS];
  bool inner_kept = false;
  for (int d = 0; d < in->ndim; ++d) {
    const bool kept = out->sizes[d] == in->sizes[d];
    PVB2_CHECK_ARG(kept || out->sizes[d] == 1, "pvb2_reduce: out dim %d must be 1 or match", d);
    if (in->sizes[d] == 1) continue;
    if (kept) {
      P.n_out *= in->sizes[d];
      if (d == inner_mem_dim) inner_kept = true;
    } else {
      P.n_red *= in->sizes[d];
    }
    const int64_t os = kept ? out->strides[d] : 0;
    if (nm > 0 && mk[nm - 1] == kept && mis[nm - 1] == in->sizes[d] * in->strides[d] &&
        mos[nm - 1] == in->sizes[d] * os) {
      msz[nm - 1] *= in->sizes[d];
      mis[nm - 1] = in->strides[d];
      mos[nm - 1] = os;
      continue;
    }
    mk[nm] = kept;
    msz[nm] = in->sizes[d];
    mis[nm] = in->strides[d];
    mos[nm] = os;
    ++nm;
  }
  for (int i = 0; i < nm; ++i) {
    if (mk[i]) {
      rs.ksizes[rs.kdim] = msz[i];
      rs.k_in_strides[rs.kdim] = mis[i];
      rs.k_out_strides[rs.kdim] = mos[i];
      rs.kdim++;
    } else {
      rs.rsizes[rs.rdim] = msz[i];
      rs.r_in_strides[rs.rdim] = mis[i];
      rs.rdim++;
    }
  }
  P.col = inner_kept && P.n_out >= 32;
  P.mode = kRedGeneric;
  const bool fp = compute_dtype == PVB2_F32 || compute_dtype == PVB2_F64;
  const bool arg = op == PVB2_RED_ARGMAX || op == PVB2_RED_ARGMIN;
  if (!fp || arg || in->dtype != compute_dtype || P.n_out == 0 || P.n_red == 0 || rs.rdim != 1 || rs.kdim > 1)
    return PVB2_OK;
  Red2d& g = P.g;
  g.n_out = P.n_out;
  g.n_red = P.n_red;
  g.kstride_in = rs.kdim ? rs.k_in_strides[0] : 0;
  g.kstride_out = rs.kdim ? rs.k_out_strides[0] : 0;
  g.rstride = rs.r_in_strides[0];
  g.splits = 1;
  g.chunk = g.n_red;
  P.elem = compute_dtype == PVB2_F64 ? 8 : 4;
  const int64_t target = (int64_t)num_sms() * 4;  // 256-thread blocks
  if (rs.kdim == 1 && g.kstride_in == 1) {
    P.mode = kRedCol;
    const int64_t tiles = (g.n_out + 31) / 32;
    const int64_t s = std::min<int64_t>(std::max<int64_t>(target / tiles, 1), std::max<int64_t>(g.n_red / 64, 1));
    g.chunk = (g.n_red + s - 1) / s;
  } else if (g.rstride == 1) {
    if (g.n_red <= 1024) {
      P.mode = kRedRowWarp;
      return PVB2_OK;
    }
    P.mode = kRedRowBlock;
    const int64_t s = std::min<int64_t>(std::max<int64_t>(target / g.n_out, 1), std::max<int64_t>(g.n_red / 4096, 1));
    g.chunk = (g.n_red + s - 1) / s;
  } else {
    return PVB2_OK;
  }
  g.chunk = std::max<int64_t>(g.chunk, 1);
  g.splits = (int)((g.n_red + g.chunk - 1) / g.chunk);
  return PVB2_OK;
}

static size_t plan_workspace(const RedPlan& P) {
  return P.mode != kRedGeneric && P.mode != kRedRowWarp && P.g.splits > 1
             ? (size_t)P.g.splits * (size_t)P.g.n_out * P.elem
             : 0;
}

}  // namespace pvb2

extern "C" size_t pvb2_reduce_workspace_size(int op, const pvb2_tensor* out, const pvb2_tensor* in,
                                             int compute_dtype) {
  RedPlan P;
  if (plan_reduce(op, out, in, compute_dtype, P) != PVB2_OK) return 0;
  return plan_workspace(P);
}

extern "C" int pvb2_reduce_ws(int op, const pvb2_tensor* out, const pvb2_tensor* in, double scale,
                              int compute_dtype, void* workspace, size_t workspace_bytes, pvb2_stream stream) {
  RedPlan P;
  const int rc = plan_reduce(op, out, in, compute_dtype, P);
  if (rc != PVB2_OK) return rc;
  if (P.n_out == 0) return PVB2_OK;
  cudaStream_t s = as_stream(stream);
  if (P.n_red == 0) {
    // empty reduction: identity (sum 0, prod 1); max/min of empty is an error upstream
    double ident = op == PVB2_RED_PROD ? 1.0 : 0.0;
    return pvb2_fill(out, ident, stream);
  }
  if (P.mode != kRedGeneric) {
    if (workspace == nullptr) {  // no scratch: one block per output (column tile) covers the whole range
      P.g.splits = 1;
      P.g.chunk = P.g.n_red;
    } else {
      const size_t need = plan_workspace(P);
      PVB2_CHECK_ARG(workspace_bytes >= need, "pvb2_reduce_ws: workspace %zu bytes, need %zu", workspace_bytes, need);
    }
    if (compute_dtype == PVB2_F64) return launch_red2d<double>(P.mode, P.g, op, in->data, out, workspace, scale, s);
    return launch_red2d<float>(P.mode, P.g, op, in->data, out, workspace, scale, s);
  }
  switch (compute_dtype) {
    case PVB2_F32: return launch_reduce<float>(P.rs, P.col, op, in, out, P.n_out, P.n_red, scale, s);
    case PVB2_F64: return launch_reduce<double>(P.rs, P.col, op, in, out, P.n_out, P.n_red, scale, s);
    case PVB2_I64:
    case PVB2_I32:
    case PVB2_I16:
    case PVB2_I8:
    case PVB2_U8:
    case PVB2_BOOL: return launch_reduce<int64_t>(P.rs, P.col, op, in, out, P.n_out, P.n_red, scale, s);
  }
  return fail(PVB2_ERR_UNSUPPORTED, "pvb2_reduce: compute dtype %d", compute_dtype);
}

extern "C" int pvb2_reduce(int op, const pvb2_tensor* out, const pvb2_tensor* in, double scale, int compute_dtype,
                           pvb2_stream stream) {
  return pvb2_reduce_ws(op, out, in, scale, compute_dtype, nullptr, 0, stream);
}
