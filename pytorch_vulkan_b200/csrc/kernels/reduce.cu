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

extern "C" int pvb2_reduce(int op, const pvb2_tensor* out, const pvb2_tensor* in, double scale, int compute_dtype,
                           pvb2_stream stream) {
  PVB2_CHECK_ARG(out->ndim == in->ndim, "pvb2_reduce: out must keep reduced dims (ndim %d vs %d)", out->ndim,
                 in->ndim);
  RedShape rs;
  rs.kdim = 0;
  rs.rdim = 0;
  int64_t n_out = 1, n_red = 1;
  int inner_mem_dim = -1;
  int64_t best = INT64_MAX;
  for (int d = 0; d < in->ndim; ++d) {
    if (in->sizes[d] != 1 && in->strides[d] != 0 && in->strides[d] < best) {
      best = in->strides[d];
      inner_mem_dim = d;
    }
  }
  bool inner_kept = false;
  for (int d = 0; d < in->ndim; ++d) {
    if (out->sizes[d] == in->sizes[d]) {
      if (in->sizes[d] == 1) continue;
      rs.ksizes[rs.kdim] = in->sizes[d];
      rs.k_in_strides[rs.kdim] = in->strides[d];
      rs.k_out_strides[rs.kdim] = out->strides[d];
      rs.kdim++;
      n_out *= in->sizes[d];
      if (d == inner_mem_dim) inner_kept = true;
    } else {
      PVB2_CHECK_ARG(out->sizes[d] == 1, "pvb2_reduce: out dim %d must be 1 or match", d);
      rs.rsizes[rs.rdim] = in->sizes[d];
      rs.r_in_strides[rs.rdim] = in->strides[d];
      rs.rdim++;
      n_red *= in->sizes[d];
    }
  }
  if (n_out == 0) return PVB2_OK;
  cudaStream_t s = as_stream(stream);
  if (n_red == 0) {
    // empty reduction: identity (sum 0, prod 1); max/min of empty is an error upstream
    double ident = op == PVB2_RED_PROD ? 1.0 : 0.0;
    return pvb2_fill(out, ident, stream);
  }
  const bool col = inner_kept && n_out >= 32;
  switch (compute_dtype) {
    case PVB2_F32: return launch_reduce<float>(rs, col, op, in, out, n_out, n_red, scale, s);
    case PVB2_F64: return launch_reduce<double>(rs, col, op, in, out, n_out, n_red, scale, s);
    case PVB2_I64:
    case PVB2_I32:
    case PVB2_I16:
    case PVB2_I8:
    case PVB2_U8:
    case PVB2_BOOL: return launch_reduce<int64_t>(rs, col, op, in, out, n_out, n_red, scale, s);
  }
  return fail(PVB2_ERR_UNSUPPORTED, "pvb2_reduce: compute dtype %d", compute_dtype);
}
