// Pointwise kernels: unary, binary and ternary element maps with torch's
// broadcasting already applied by the caller (stride-0 dims).
//
// Replaces the runtime-JIT OpenCL expressions that src/pointwise_ops.cpp
// builds with dlprim::core::pointwise_operation[_broadcast] (e.g.
// pointwise_ops.cpp:133-172 add, :407-411 mul, :437-455 threshold_backward,
// :559-603 hardtanh, :1324-1393 gelu).  Here every expression is compiled
// ahead of time; contiguous fp32 operands take a 128-bit vectorised path.
#include "common.cuh"

namespace pvb2 {

// ----------------------------------------------------------- op bodies
template <typename T>
__device__ __forceinline__ T sat_nan_max(T a, T b) {
  if (a != a) return a;
  if (b != b) return b;
  return a > b ? a : b;
}
template <typename T>
__device__ __forceinline__ T sat_nan_min(T a, T b) {
  if (a != a) return a;
  if (b != b) return b;
  return a < b ? a : b;
}

template <typename T>
__device__ __forceinline__ T f_exp(T x) { return (T)exp((double)x); }
template <>
__device__ __forceinline__ float f_exp<float>(float x) { return expf(x); }

template <typename T>
struct Math {
  static __device__ __forceinline__ T exp_(T x) { return exp(x); }
  static __device__ __forceinline__ T log_(T x) { return log(x); }
  static __device__ __forceinline__ T log1p_(T x) { return log1p(x); }
  static __device__ __forceinline__ T sqrt_(T x) { return sqrt(x); }
  static __device__ __forceinline__ T erf_(T x) { return erf(x); }
  static __device__ __forceinline__ T tanh_(T x) { return tanh(x); }
  static __device__ __forceinline__ T pow_(T x, T y) { return pow(x, y); }
  static __device__ __forceinline__ T atan_(T x) { return atan(x); }
  static __device__ __forceinline__ T atan2_(T x, T y) { return atan2(x, y); }
  static __device__ __forceinline__ T ceil_(T x) { return ceil(x); }
  static __device__ __forceinline__ T floor_(T x) { return floor(x); }
  static __device__ __forceinline__ T trunc_(T x) { return trunc(x); }
  static __device__ __forceinline__ T rint_(T x) { return rint(x); }
  static __device__ __forceinline__ T fabs_(T x) { return fabs(x); }
  static __device__ __forceinline__ T fmod_(T x, T y) { return fmod(x, y); }
};
template <>
struct Math<float> {
  static __device__ __forceinline__ float exp_(float x) { return expf(x); }
  static __device__ __forceinline__ float log_(float x) { return logf(x); }
  static __device__ __forceinline__ float log1p_(float x) { return log1pf(x); }
  static __device__ __forceinline__ float sqrt_(float x) { return sqrtf(x); }
  static __device__ __forceinline__ float erf_(float x) { return erff(x); }
  static __device__ __forceinline__ float tanh_(float x) { return tanhf(x); }
  static __device__ __forceinline__ float pow_(float x, float y) { return powf(x, y); }
  static __device__ __forceinline__ float atan_(float x) { return atanf(x); }
  static __device__ __forceinline__ float atan2_(float x, float y) { return atan2f(x, y); }
  static __device__ __forceinline__ float ceil_(float x) { return ceilf(x); }
  static __device__ __forceinline__ float floor_(float x) { return floorf(x); }
  static __device__ __forceinline__ float trunc_(float x) { return truncf(x); }
  static __device__ __forceinline__ float rint_(float x) { return rintf(x); }
  static __device__ __forceinline__ float fabs_(float x) { return fabsf(x); }
  static __device__ __forceinline__ float fmod_(float x, float y) { return fmodf(x, y); }
};

template <typename T>
__device__ __forceinline__ bool is_nan(T x) { return x != x; }

template <typename T>
__device__ __forceinline__ T unary_float(int op, T x, T p0, T p1) {
  using M = Math<T>;
  const T zero = (T)0, one = (T)1;
  switch (op) {
    case PVB2_UN_COPY: return x;
    case PVB2_UN_RELU: return is_nan(x) ? x : (x > zero ? x : zero);
    case PVB2_UN_HARDTANH: return is_nan(x) ? x : (x < p0 ? p0 : (x > p1 ? p1 : x));
    case PVB2_UN_GELU_ERF: return x * (T)0.5 * (one + M::erf_(x * (T)0.70710678118654752440));
    case PVB2_UN_GELU_TANH: {
      const T kBeta = (T)0.79788456080286535588;  // sqrt(2/pi)
      const T kKappa = (T)0.044715;
      T inner = kBeta * (x + kKappa * x * x * x);
      return (T)0.5 * x * (one + M::tanh_(inner));
    }
    case PVB2_UN_NEG: return -x;
    case PVB2_UN_EXP: return M::exp_(x);
    case PVB2_UN_LOG: return M::log_(x);
    case PVB2_UN_SQRT: return M::sqrt_(x);
    case PVB2_UN_RSQRT: return one / M::sqrt_(x);
    case PVB2_UN_ABS: return M::fabs_(x);
    case PVB2_UN_SIGMOID: return one / (one + M::exp_(-x));
    case PVB2_UN_TANH: return M::tanh_(x);
    case PVB2_UN_RECIPROCAL: return one / x;
    case PVB2_UN_SILU: return x / (one + M::exp_(-x));
    case PVB2_UN_AFFINE: return x * p0 + p1;
    case PVB2_UN_POW: {
      if (p0 == (T)2) return x * x;
      if (p0 == (T)3) return x * x * x;
      if (p0 == (T)0.5) return M::sqrt_(x);
      if (p0 == (T)-0.5) return one / M::sqrt_(x);
      if (p0 == (T)-1) return one / x;
      if (p0 == (T)-2) return one / (x * x);
      if (p0 == (T)1) return x;
      if (p0 == (T)0) return one;
      return M::pow_(x, p0);
    }
    case PVB2_UN_CLAMP: return is_nan(x) ? x : (x < p0 ? p0 : (x > p1 ? p1 : x));
    case PVB2_UN_CLAMP_MIN: return is_nan(x) ? x : (x < p0 ? p0 : x);
    case PVB2_UN_LEAKY_RELU: return x > zero ? x : x * p0;
    case PVB2_UN_SGN: return (T)((x > zero) - (x < zero));
    case PVB2_UN_HARDSIGMOID: {
      T t = x + (T)3;
      t = t < zero ? zero : (t > (T)6 ? (T)6 : t);
      return t / (T)6;
    }
    case PVB2_UN_HARDSWISH: {
      T t = x + (T)3;
      t = t < zero ? zero : (t > (T)6 ? (T)6 : t);
      return x * t / (T)6;
    }
    case PVB2_UN_CEIL: return M::ceil_(x);
    case PVB2_UN_FLOOR: return M::floor_(x);
    case PVB2_UN_TRUNC: return M::trunc_(x);
    case PVB2_UN_ROUND: return M::rint_(x);
    case PVB2_UN_ATAN: return M::atan_(x);
    case PVB2_UN_LOG_SIGMOID: {
      T mn = x < zero ? x : zero;
      return mn - M::log1p_(M::exp_(-M::fabs_(x)));
    }
    case PVB2_UN_LOGICAL_NOT: return x == zero ? one : zero;
    case PVB2_UN_ISNAN: return is_nan(x) ? one : zero;
    case PVB2_UN_ISINF: return (!is_nan(x) && M::fabs_(x) == (T)INFINITY) ? one : zero;
    case PVB2_UN_ISPOSINF: return x == (T)INFINITY ? one : zero;
    case PVB2_UN_ISNEGINF: return x == (T)-INFINITY ? one : zero;
    case PVB2_UN_ISFINITE: return (!is_nan(x) && M::fabs_(x) != (T)INFINITY) ? one : zero;
    case PVB2_UN_LOGIT: {
      T z = x;
      if (p0 >= zero) z = z < p0 ? p0 : (z > one - p0 ? one - p0 : z);
      return M::log_(z / (one - z));
    }
  }
  return x;
}

template <typename T>
__device__ __forceinline__ T unary_int(int op, T x, T p0, T p1) {
  switch (op) {
    case PVB2_UN_COPY: return x;
    case PVB2_UN_RELU: return x > 0 ? x : 0;
    case PVB2_UN_HARDTANH:
    case PVB2_UN_CLAMP: return x < p0 ? p0 : (x > p1 ? p1 : x);
    case PVB2_UN_CLAMP_MIN: return x < p0 ? p0 : x;
    case PVB2_UN_NEG: return -x;
    case PVB2_UN_ABS: return x < 0 ? -x : x;
    case PVB2_UN_AFFINE: return x * p0 + p1;
    case PVB2_UN_SGN: return (T)((x > 0) - (x < 0));
    case PVB2_UN_BITWISE_NOT: return ~x;
    case PVB2_UN_LOGICAL_NOT: return x == 0 ? 1 : 0;
    case PVB2_UN_ISNAN:
    case PVB2_UN_ISINF:
    case PVB2_UN_ISPOSINF:
    case PVB2_UN_ISNEGINF: return 0;
    case PVB2_UN_ISFINITE: return 1;
    case PVB2_UN_CEIL:
    case PVB2_UN_FLOOR:
    case PVB2_UN_TRUNC:
    case PVB2_UN_ROUND: return x;
  }
  return x;
}

template <typename T>
__device__ __forceinline__ T unary_apply(int op, T x, T p0, T p1) {
  if constexpr (std::is_floating_point<T>::value) return unary_float<T>(op, x, p0, p1);
  else return unary_int<T>(op, x, p0, p1);
}

// binary ops producing a value of the compute type
template <typename T>
__device__ __forceinline__ T binary_float(int op, T a, T b, T p0, T p1) {
  using M = Math<T>;
  const T zero = (T)0, one = (T)1;
  switch (op) {
    case PVB2_BIN_ADD: return p0 == one ? a + b : fma(p0, b, a);
    case PVB2_BIN_SUB: return p0 == one ? a - b : fma(-p0, b, a);
    case PVB2_BIN_MUL: return a * b;
    case PVB2_BIN_DIV: return a / b;
    case PVB2_BIN_DIV_TRUNC: return M::trunc_(a / b);
    case PVB2_BIN_DIV_FLOOR: {
      if (b == zero) return a / b;
      T mod = M::fmod_(a, b);
      T div = (a - mod) / b;
      if ((mod != zero) && ((b < zero) != (mod < zero))) div -= one;
      if (div == zero) return copysign(zero, a / b);
      T fl = M::floor_(div);
      if (div - fl > (T)0.5) fl += one;
      return fl;
    }
    case PVB2_BIN_REMAINDER: {
      T m = M::fmod_(a, b);
      if (m != zero && ((b < zero) != (m < zero))) m += b;
      return m;
    }
    case PVB2_BIN_MAXIMUM: return sat_nan_max(a, b);
    case PVB2_BIN_MINIMUM: return sat_nan_min(a, b);
    case PVB2_BIN_THRESHOLD_BWD: return b <= p0 ? zero : a;
    case PVB2_BIN_HARDTANH_BWD: return (b <= p0 || b >= p1) ? zero : a;
    case PVB2_BIN_GELU_ERF_BWD: {
      const T kAlpha = (T)0.70710678118654752440;   // 1/sqrt(2)
      const T kBeta = (T)0.39894228040143267794;    // 1/sqrt(2*pi)
      T cdf = (T)0.5 * (one + M::erf_(b * kAlpha));
      T pdf = kBeta * M::exp_((T)-0.5 * b * b);
      return a * (cdf + b * pdf);
    }
    case PVB2_BIN_GELU_TANH_BWD: {
      const T kBeta = (T)0.79788456080286535588;
      const T kKappa = (T)0.044715;
      T x_sq = b * b;
      T x_cube = x_sq * b;
      T inner = kBeta * (b + kKappa * x_cube);
      T tanh_inner = M::tanh_(inner);
      T left = (T)0.5 * b;
      T right = one + tanh_inner;
      T left_derivative = (T)0.5 * right;
      T right_derivative = left * (one - tanh_inner * tanh_inner) * kBeta * (one + (T)3 * kKappa * x_sq);
      return a * (left_derivative + right_derivative);
    }
    case PVB2_BIN_SIGMOID_BWD: return a * (one - b) * b;
    case PVB2_BIN_TANH_BWD: return a * (one - b * b);
    case PVB2_BIN_SILU_BWD: {
      T s = one / (one + M::exp_(-b));
      return a * s * (one + b * (one - s));
    }
    case PVB2_BIN_LEAKY_RELU_BWD: return b > zero ? a : a * p0;
    case PVB2_BIN_HARDSIGMOID_BWD: return (b > (T)-3 && b < (T)3) ? a / (T)6 : zero;
    case PVB2_BIN_HARDSWISH_BWD:
      return b < (T)-3 ? zero : (b <= (T)3 ? a * ((b / (T)3) + (T)0.5) : a);
    case PVB2_BIN_LOG_SIGMOID_BWD: {
      // d/dx log(sigmoid(x)) = 1 - sigmoid(x) = sigmoid(-x)
      T s = one / (one + M::exp_(b));
      return a * s;
    }
    case PVB2_BIN_LERP: {
      T w = p0;
      return (M::fabs_(w) < (T)0.5) ? a + w * (b - a) : b - (b - a) * (one - w);
    }
    case PVB2_BIN_POW: return M::pow_(a, b);
    case PVB2_BIN_ATAN2: return M::atan2_(a, b);
    case PVB2_BIN_MSE_BWD: return p0 * (a - b);
  }
  return a;
}

template <typename T>
__device__ __forceinline__ T binary_int(int op, T a, T b, T p0, T p1) {
  switch (op) {
    case PVB2_BIN_ADD: return a + p0 * b;
    case PVB2_BIN_SUB: return a - p0 * b;
    case PVB2_BIN_MUL: return a * b;
    case PVB2_BIN_DIV:
    case PVB2_BIN_DIV_TRUNC: return b == 0 ? 0 : a / b;
    case PVB2_BIN_DIV_FLOOR: {
      if (b == 0) return 0;
      T q = a / b;
      if ((a % b != 0) && ((a < 0) != (b < 0))) q -= 1;
      return q;
    }
    case PVB2_BIN_REMAINDER: {
      if (b == 0) return 0;
      T m = a % b;
      if (m != 0 && ((b < 0) != (m < 0))) m += b;
      return m;
    }
    case PVB2_BIN_MAXIMUM: return a > b ? a : b;
    case PVB2_BIN_MINIMUM: return a < b ? a : b;
    case PVB2_BIN_THRESHOLD_BWD: return b <= p0 ? 0 : a;
    case PVB2_BIN_BITWISE_AND: return a & b;
    case PVB2_BIN_BITWISE_OR: return a | b;
    case PVB2_BIN_BITWISE_XOR: return a ^ b;
    case PVB2_BIN_MSE_BWD: return p0 * (a - b);
  }
  return a;
}

template <typename T>
__device__ __forceinline__ T binary_apply(int op, T a, T b, T p0, T p1) {
  if constexpr (std::is_floating_point<T>::value) return binary_float<T>(op, a, b, p0, p1);
  else return binary_int<T>(op, a, b, p0, p1);
}

__device__ __forceinline__ bool is_compare(int op) { return op >= PVB2_BIN_EQ && op <= PVB2_BIN_GE; }

template <typename T>
__device__ __forceinline__ bool compare_apply(int op, T a, T b) {
  switch (op) {
    case PVB2_BIN_EQ: return a == b;
    case PVB2_BIN_NE: return a != b;
    case PVB2_BIN_LT: return a < b;
    case PVB2_BIN_LE: return a <= b;
    case PVB2_BIN_GT: return a > b;
    case PVB2_BIN_GE: return a >= b;
  }
  return false;
}

template <typename T>
__device__ __forceinline__ T ternary_apply(int op, T a, T b, T c, T p0) {
  switch (op) {
    case PVB2_TER_ADDCMUL: return a + p0 * b * c;
    case PVB2_TER_ADDCDIV: return a + (p0 * b) / c;
    case PVB2_TER_WHERE: return a != (T)0 ? b : c;
  }
  return a;
}

// ------------------------------------------------------------ kernels
// generic strided, dtype-converting kernels (compute type T)
template <typename T>
__global__ void unary_generic_kernel(IterShape it, int op, void* out, int odt, const void* x, int xdt,
                                     T p0, T p1, int64_t n) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t step = (int64_t)gridDim.x * blockDim.x;
  for (; i < n; i += step) {
    int64_t o[kMaxArgs];
    iter_offsets(it, 2, i, o);
    T v = load_as<T>(x, o[1], xdt);
    store_as<T>(out, o[0], odt, unary_apply<T>(op, v, p0, p1));
  }
}

template <typename T>
__global__ void binary_generic_kernel(IterShape it, int op, void* out, int odt, const void* a, int adt,
                                      const void* b, int bdt, T p0, T p1, int64_t n) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t step = (int64_t)gridDim.x * blockDim.x;
  const bool cmp = is_compare(op);
  for (; i < n; i += step) {
    int64_t o[kMaxArgs];
    iter_offsets(it, 3, i, o);
    T va = load_as<T>(a, o[1], adt);
    T vb = load_as<T>(b, o[2], bdt);
    if (cmp) store_as<int>(out, o[0], odt, compare_apply<T>(op, va, vb) ? 1 : 0);
    else store_as<T>(out, o[0], odt, binary_apply<T>(op, va, vb, p0, p1));
  }
}

// fp32 operands whose innermost (merged) dim has unit stride in the output
// and unit or zero stride in each input (a transposed-batch residual add, a
// row broadcast): rows of `len` elements, a group of G lanes per row, row
// offsets from the outer dims computed once per row.
// A long row is cut into pieces of `piece` elements (a group per piece) so
// that few-row shapes (a [B, L*C] broadcast add) still fill the GPU.
__global__ void __launch_bounds__(256) binary_f32_rows_kernel(IterShape outer, int64_t rows, int64_t len,
                                                              int64_t piece, int group, int op,
                                                              float* __restrict__ out, const float* __restrict__ a,
                                                              int a_unit, const float* __restrict__ b, int b_unit,
                                                              float p0, float p1) {
  const int lane = threadIdx.x % group;
  const int64_t pieces = (len + piece - 1) / piece;
  const int64_t g0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / group;
  const int64_t gstep = (int64_t)gridDim.x * blockDim.x / group;
  for (int64_t gi = g0; gi < rows * pieces; gi += gstep) {
    const int64_t r = gi / pieces, u0 = (gi - r * pieces) * piece, u1 = min(len, u0 + piece);
    int64_t o[kMaxArgs];
    iter_offsets(outer, 3, r, o);
    float* dst = out + o[0];
    const float* x = a + o[1];
    const float* y = b + o[2];
    for (int64_t u = u0 + lane; u < u1; u += group)
      dst[u] = binary_apply<float>(op, __ldg(x + u * a_unit), __ldg(y + u * b_unit), p0, p1);
  }
}

template <typename T>
__global__ void binary_scalar_generic_kernel(IterShape it, int op, void* out, int odt, const void* a, int adt,
                                             T sc, int scalar_first, T p0, T p1, int64_t n) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t step = (int64_t)gridDim.x * blockDim.x;
  const bool cmp = is_compare(op);
  for (; i < n; i += step) {
    int64_t o[kMaxArgs];
    iter_offsets(it, 2, i, o);
    T v = load_as<T>(a, o[1], adt);
    T x = scalar_first ? sc : v, y = scalar_first ? v : sc;
    if (cmp) store_as<int>(out, o[0], odt, compare_apply<T>(op, x, y) ? 1 : 0);
    else store_as<T>(out, o[0], odt, binary_apply<T>(op, x, y, p0, p1));
  }
}

// contiguous fp32 tensor op scalar value
template <int OP>
__global__ void binary_f32_value_kernel(float* __restrict__ out, const float* __restrict__ a, float b, int64_t n,
                                        float p0, float p1) {
  const int64_t n4 = n >> 2;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t step = (int64_t)gridDim.x * blockDim.x;
  const float4* a4 = reinterpret_cast<const float4*>(a);
  float4* o4 = reinterpret_cast<float4*>(out);
  for (int64_t k = i; k < n4; k += step) {
    float4 va = a4[k];
    va.x = binary_float<float>(OP, va.x, b, p0, p1);
    va.y = binary_float<float>(OP, va.y, b, p0, p1);
    va.z = binary_float<float>(OP, va.z, b, p0, p1);
    va.w = binary_float<float>(OP, va.w, b, p0, p1);
    o4[k] = va;
  }
  for (int64_t k = (n4 << 2) + i; k < n; k += step) out[k] = binary_float<float>(OP, a[k], b, p0, p1);
}

template <typename T>
__global__ void ternary_generic_kernel(IterShape it, int op, void* out, int odt, const void* a, int adt,
                                       const void* b, int bdt, const void* c, int cdt, T p0, int64_t n) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t step = (int64_t)gridDim.x * blockDim.x;
  for (; i < n; i += step) {
    int64_t o[kMaxArgs];
    iter_offsets(it, 4, i, o);
    T va = load_as<T>(a, o[1], adt);
    T vb = load_as<T>(b, o[2], bdt);
    T vc = load_as<T>(c, o[3], cdt);
    store_as<T>(out, o[0], odt, ternary_apply<T>(op, va, vb, vc, p0));
  }
}

// contiguous fp32 fast paths, 128-bit vectorised
template <int OP>
__global__ void unary_f32_vec_kernel(float* __restrict__ out, const float* __restrict__ x, int64_t n, float p0,
                                     float p1) {
  const int64_t n4 = n >> 2;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t step = (int64_t)gridDim.x * blockDim.x;
  const float4* x4 = reinterpret_cast<const float4*>(x);
  float4* o4 = reinterpret_cast<float4*>(out);
  for (int64_t k = i; k < n4; k += step) {
    float4 v = x4[k];
    v.x = unary_float<float>(OP, v.x, p0, p1);
    v.y = unary_float<float>(OP, v.y, p0, p1);
    v.z = unary_float<float>(OP, v.z, p0, p1);
    v.w = unary_float<float>(OP, v.w, p0, p1);
    o4[k] = v;
  }
  for (int64_t k = (n4 << 2) + i; k < n; k += step) out[k] = unary_float<float>(OP, x[k], p0, p1);
}

template <int OP>
__global__ void binary_f32_vec_kernel(float* __restrict__ out, const float* __restrict__ a,
                                      const float* __restrict__ b, int64_t n, float p0, float p1) {
  const int64_t n4 = n >> 2;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t step = (int64_t)gridDim.x * blockDim.x;
  const float4* a4 = reinterpret_cast<const float4*>(a);
  const float4* b4 = reinterpret_cast<const float4*>(b);
  float4* o4 = reinterpret_cast<float4*>(out);
  for (int64_t k = i; k < n4; k += step) {
    float4 va = a4[k], vb = b4[k];
    va.x = binary_float<float>(OP, va.x, vb.x, p0, p1);
    va.y = binary_float<float>(OP, va.y, vb.y, p0, p1);
    va.z = binary_float<float>(OP, va.z, vb.z, p0, p1);
    va.w = binary_float<float>(OP, va.w, vb.w, p0, p1);
    o4[k] = va;
  }
  for (int64_t k = (n4 << 2) + i; k < n; k += step) out[k] = binary_float<float>(OP, a[k], b[k], p0, p1);
}

// a contiguous, b a broadcast scalar (all strides 0)
template <int OP>
__global__ void binary_f32_scalar_kernel(float* __restrict__ out, const float* __restrict__ a,
                                         const float* __restrict__ bptr, int64_t n, float p0, float p1) {
  const float b = *bptr;
  const int64_t n4 = n >> 2;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t step = (int64_t)gridDim.x * blockDim.x;
  const float4* a4 = reinterpret_cast<const float4*>(a);
  float4* o4 = reinterpret_cast<float4*>(out);
  for (int64_t k = i; k < n4; k += step) {
    float4 va = a4[k];
    va.x = binary_float<float>(OP, va.x, b, p0, p1);
    va.y = binary_float<float>(OP, va.y, b, p0, p1);
    va.z = binary_float<float>(OP, va.z, b, p0, p1);
    va.w = binary_float<float>(OP, va.w, b, p0, p1);
    o4[k] = va;
  }
  for (int64_t k = (n4 << 2) + i; k < n; k += step) out[k] = binary_float<float>(OP, a[k], b, p0, p1);
}

// a contiguous 4-D NCHW, b broadcast per channel ([1,C,1,1] or [C,1,1])
template <int OP>
__global__ void binary_f32_channel_kernel(float* __restrict__ out, const float* __restrict__ a,
                                          const float* __restrict__ b, int64_t b_stride, int64_t rows, int64_t C,
                                          int64_t inner, float p0, float p1) {
  // one block row per (n, c) plane
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float bv = b[(r % C) * b_stride];
    const float* ap = a + r * inner;
    float* op = out + r * inner;
    for (int64_t k = threadIdx.x; k < inner; k += blockDim.x) op[k] = binary_float<float>(OP, ap[k], bv, p0, p1);
  }
}

static bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

template <int OP>
static int launch_unary_fast(float* out, const float* x, int64_t n, float p0, float p1, cudaStream_t s) {
  const int block = 256;
  unary_f32_vec_kernel<OP><<<grid_for((n + 3) / 4, block), block, 0, s>>>(out, x, n, p0, p1);
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

template <int OP>
static int launch_binary_fast(float* out, const float* a, const float* b, int64_t n, float p0, float p1,
                              cudaStream_t s) {
  const int block = 256;
  binary_f32_vec_kernel<OP><<<grid_for((n + 3) / 4, block), block, 0, s>>>(out, a, b, n, p0, p1);
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

template <int OP>
static int launch_binary_scalar(float* out, const float* a, const float* b, int64_t n, float p0, float p1,
                                cudaStream_t s) {
  const int block = 256;
  binary_f32_scalar_kernel<OP><<<grid_for((n + 3) / 4, block), block, 0, s>>>(out, a, b, n, p0, p1);
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

static bool all_zero_strides(const pvb2_tensor* t) {
  for (int d = 0; d < t->ndim; ++d)
    if (t->sizes[d] != 1 && t->strides[d] != 0) return false;
  return true;
}

}  // namespace pvb2

using namespace pvb2;

#define UNARY_FAST_CASE(OPC) \
  case OPC: return launch_unary_fast<OPC>((float*)out->data, (const float*)x->data, n, (float)p0, (float)p1, s);
#define BINARY_FAST_CASE(OPC)                                                                                   \
  case OPC:                                                                                                     \
    return launch_binary_fast<OPC>((float*)out->data, (const float*)a->data, (const float*)b->data, n, (float)p0, \
                                   (float)p1, s);
#define BINARY_SCALAR_CASE(OPC)                                                                                   \
  case OPC:                                                                                                       \
    return launch_binary_scalar<OPC>((float*)out->data, (const float*)a->data, (const float*)b->data, n, (float)p0, \
                                     (float)p1, s);

extern "C" {

int pvb2_unary(int op, const pvb2_tensor* out, const pvb2_tensor* x, double p0, double p1, int compute_dtype,
               pvb2_stream stream) {
  const int64_t n = numel(out);
  if (n == 0) return PVB2_OK;
  PVB2_CHECK_ARG(x->ndim == out->ndim, "pvb2_unary: ndim mismatch");
  cudaStream_t s = as_stream(stream);
  if (compute_dtype == PVB2_F32 && out->dtype == PVB2_F32 && x->dtype == PVB2_F32 && is_contiguous(out) &&
      is_contiguous(x) && aligned16(out->data) && aligned16(x->data)) {
    switch (op) {
      UNARY_FAST_CASE(PVB2_UN_RELU)
      UNARY_FAST_CASE(PVB2_UN_HARDTANH)
      UNARY_FAST_CASE(PVB2_UN_GELU_ERF)
      UNARY_FAST_CASE(PVB2_UN_GELU_TANH)
      UNARY_FAST_CASE(PVB2_UN_AFFINE)
      UNARY_FAST_CASE(PVB2_UN_COPY)
      UNARY_FAST_CASE(PVB2_UN_SQRT)
      UNARY_FAST_CASE(PVB2_UN_EXP)
      UNARY_FAST_CASE(PVB2_UN_NEG)
      default: break;
    }
  }
  IterShape it;
  const pvb2_tensor* ts[2] = {out, x};
  make_iter(&it, ts, 2);
  const int block = 256;
  const int grid = grid_for(n, block);
  switch (compute_dtype) {
    case PVB2_F32:
      unary_generic_kernel<float><<<grid, block, 0, s>>>(it, op, out->data, out->dtype, x->data, x->dtype,
                                                         (float)p0, (float)p1, n);
      break;
    case PVB2_F64:
      unary_generic_kernel<double><<<grid, block, 0, s>>>(it, op, out->data, out->dtype, x->data, x->dtype, p0,
                                                          p1, n);
      break;
    case PVB2_I64:
    case PVB2_I32:
    case PVB2_I16:
    case PVB2_I8:
    case PVB2_U8:
    case PVB2_BOOL:
      unary_generic_kernel<int64_t><<<grid, block, 0, s>>>(it, op, out->data, out->dtype, x->data, x->dtype,
                                                           (int64_t)p0, (int64_t)p1, n);
      break;
    default:
      return fail(PVB2_ERR_UNSUPPORTED, "pvb2_unary: compute dtype %d not supported", compute_dtype);
  }
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

static inline bool is_compare_op(int op) { return op >= PVB2_BIN_EQ && op <= PVB2_BIN_GE; }

int pvb2_binary(int op, const pvb2_tensor* out, const pvb2_tensor* a, const pvb2_tensor* b, double p0, double p1,
                int compute_dtype, pvb2_stream stream) {
  const int64_t n = numel(out);
  if (n == 0) return PVB2_OK;
  PVB2_CHECK_ARG(a->ndim == out->ndim && b->ndim == out->ndim, "pvb2_binary: ndim mismatch");
  cudaStream_t s = as_stream(stream);
  const bool f32 = compute_dtype == PVB2_F32 && out->dtype == PVB2_F32 && a->dtype == PVB2_F32 &&
                   b->dtype == PVB2_F32;
  if (f32 && is_contiguous(out) && is_contiguous(a) && aligned16(out->data) && aligned16(a->data)) {
    if (is_contiguous(b) && aligned16(b->data)) {
      switch (op) {
        BINARY_FAST_CASE(PVB2_BIN_ADD)
        BINARY_FAST_CASE(PVB2_BIN_SUB)
        BINARY_FAST_CASE(PVB2_BIN_MUL)
        BINARY_FAST_CASE(PVB2_BIN_DIV)
        BINARY_FAST_CASE(PVB2_BIN_THRESHOLD_BWD)
        BINARY_FAST_CASE(PVB2_BIN_HARDTANH_BWD)
        BINARY_FAST_CASE(PVB2_BIN_GELU_ERF_BWD)
        BINARY_FAST_CASE(PVB2_BIN_GELU_TANH_BWD)
        default: break;
      }
    } else if (all_zero_strides(b)) {
      switch (op) {
        BINARY_SCALAR_CASE(PVB2_BIN_ADD)
        BINARY_SCALAR_CASE(PVB2_BIN_SUB)
        BINARY_SCALAR_CASE(PVB2_BIN_MUL)
        BINARY_SCALAR_CASE(PVB2_BIN_DIV)
        default: break;
      }
    } else if (out->ndim == 4 && b->strides[0] == 0 && b->strides[2] == 0 && b->strides[3] == 0 &&
               (op == PVB2_BIN_ADD || op == PVB2_BIN_MUL || op == PVB2_BIN_SUB || op == PVB2_BIN_DIV)) {
      const int64_t C = out->sizes[1], rows = out->sizes[0] * C, inner = out->sizes[2] * out->sizes[3];
      const int grid = (int)std::min<int64_t>(rows, (int64_t)num_sms() * 16);
      const float* bp = (const float*)b->data;
      float* op_ = (float*)out->data;
      const float* ap = (const float*)a->data;
      switch (op) {
        case PVB2_BIN_ADD:
          binary_f32_channel_kernel<PVB2_BIN_ADD><<<grid, 256, 0, s>>>(op_, ap, bp, b->strides[1], rows, C, inner,
                                                                       (float)p0, (float)p1);
          break;
        case PVB2_BIN_SUB:
          binary_f32_channel_kernel<PVB2_BIN_SUB><<<grid, 256, 0, s>>>(op_, ap, bp, b->strides[1], rows, C, inner,
                                                                       (float)p0, (float)p1);
          break;
        case PVB2_BIN_MUL:
          binary_f32_channel_kernel<PVB2_BIN_MUL><<<grid, 256, 0, s>>>(op_, ap, bp, b->strides[1], rows, C, inner,
                                                                       (float)p0, (float)p1);
          break;
        default:
          binary_f32_channel_kernel<PVB2_BIN_DIV><<<grid, 256, 0, s>>>(op_, ap, bp, b->strides[1], rows, C, inner,
                                                                       (float)p0, (float)p1);
          break;
      }
      PVB2_LAUNCH_CHECK();
      return PVB2_OK;
    }
  }
  IterShape it;
  const pvb2_tensor* ts[3] = {out, a, b};
  make_iter(&it, ts, 3);
  const int block = 256;
  const int grid = grid_for(n, block);
  const int nd = it.ndim;
  if (f32 && !is_compare_op(op) && nd >= 1 && it.sizes[nd - 1] >= 32 && it.strides[0][nd - 1] == 1 &&
      (it.strides[1][nd - 1] == 0 || it.strides[1][nd - 1] == 1) &&
      (it.strides[2][nd - 1] == 0 || it.strides[2][nd - 1] == 1)) {
    IterShape outer;
    outer.ndim = nd - 1;
    int64_t rows = 1;
    for (int d = 0; d < nd - 1; ++d) {
      outer.sizes[d] = it.sizes[d];
      for (int k = 0; k < 3; ++k) outer.strides[k][d] = it.strides[k][d];
      rows *= it.sizes[d];
    }
    const int64_t len = it.sizes[nd - 1];
    int group = 32;
    while (group > 4 && group / 2 >= len) group >>= 1;
    const int64_t piece = 1024;
    const int64_t groups = rows * ((len + piece - 1) / piece);
    binary_f32_rows_kernel<<<grid_for(groups * group, block), block, 0, s>>>(
        outer, rows, len, piece, group, op, (float*)out->data, (const float*)a->data, (int)it.strides[1][nd - 1],
        (const float*)b->data, (int)it.strides[2][nd - 1], (float)p0, (float)p1);
    PVB2_LAUNCH_CHECK();
    return PVB2_OK;
  }
  switch (compute_dtype) {
    case PVB2_F32:
      binary_generic_kernel<float><<<grid, block, 0, s>>>(it, op, out->data, out->dtype, a->data, a->dtype, b->data,
                                                          b->dtype, (float)p0, (float)p1, n);
      break;
    case PVB2_F64:
      binary_generic_kernel<double><<<grid, block, 0, s>>>(it, op, out->data, out->dtype, a->data, a->dtype,
                                                           b->data, b->dtype, p0, p1, n);
      break;
    case PVB2_I64:
    case PVB2_I32:
    case PVB2_I16:
    case PVB2_I8:
    case PVB2_U8:
    case PVB2_BOOL:
      binary_generic_kernel<int64_t><<<grid, block, 0, s>>>(it, op, out->data, out->dtype, a->data, a->dtype,
                                                            b->data, b->dtype, (int64_t)p0, (int64_t)p1, n);
      break;
    default:
      return fail(PVB2_ERR_UNSUPPORTED, "pvb2_binary: compute dtype %d not supported", compute_dtype);
  }
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

int pvb2_binary_scalar(int op, const pvb2_tensor* out, const pvb2_tensor* t, double scalar, int scalar_first,
                       double p0, double p1, int compute_dtype, pvb2_stream stream) {
  const int64_t n = numel(out);
  if (n == 0) return PVB2_OK;
  PVB2_CHECK_ARG(t->ndim == out->ndim, "pvb2_binary_scalar: ndim mismatch");
  cudaStream_t s = as_stream(stream);
  const int block = 256;
  if (!scalar_first && compute_dtype == PVB2_F32 && out->dtype == PVB2_F32 && t->dtype == PVB2_F32 &&
      is_contiguous(out) && is_contiguous(t) && aligned16(out->data) && aligned16(t->data)) {
    float* o = (float*)out->data;
    const float* a = (const float*)t->data;
    const float b = (float)scalar;
    const int grid = grid_for((n + 3) / 4, block);
    switch (op) {
      case PVB2_BIN_ADD:
        binary_f32_value_kernel<PVB2_BIN_ADD><<<grid, block, 0, s>>>(o, a, b, n, (float)p0, (float)p1);
        PVB2_LAUNCH_CHECK();
        return PVB2_OK;
      case PVB2_BIN_SUB:
        binary_f32_value_kernel<PVB2_BIN_SUB><<<grid, block, 0, s>>>(o, a, b, n, (float)p0, (float)p1);
        PVB2_LAUNCH_CHECK();
        return PVB2_OK;
      case PVB2_BIN_MUL:
        binary_f32_value_kernel<PVB2_BIN_MUL><<<grid, block, 0, s>>>(o, a, b, n, (float)p0, (float)p1);
        PVB2_LAUNCH_CHECK();
        return PVB2_OK;
      case PVB2_BIN_DIV:
        binary_f32_value_kernel<PVB2_BIN_DIV><<<grid, block, 0, s>>>(o, a, b, n, (float)p0, (float)p1);
        PVB2_LAUNCH_CHECK();
        return PVB2_OK;
      default: break;
    }
  }
  IterShape it;
  const pvb2_tensor* ts[2] = {out, t};
  make_iter(&it, ts, 2);
  const int grid = grid_for(n, block);
  switch (compute_dtype) {
    case PVB2_F32:
      binary_scalar_generic_kernel<float><<<grid, block, 0, s>>>(it, op, out->data, out->dtype, t->data, t->dtype,
                                                                 (float)scalar, scalar_first, (float)p0, (float)p1, n);
      break;
    case PVB2_F64:
      binary_scalar_generic_kernel<double><<<grid, block, 0, s>>>(it, op, out->data, out->dtype, t->data, t->dtype,
                                                                  scalar, scalar_first, p0, p1, n);
      break;
    case PVB2_I64:
    case PVB2_I32:
    case PVB2_I16:
    case PVB2_I8:
    case PVB2_U8:
    case PVB2_BOOL:
      binary_scalar_generic_kernel<int64_t><<<grid, block, 0, s>>>(it, op, out->data, out->dtype, t->data, t->dtype,
                                                                   (int64_t)scalar, scalar_first, (int64_t)p0,
                                                                   (int64_t)p1, n);
      break;
    default:
      return fail(PVB2_ERR_UNSUPPORTED, "pvb2_binary_scalar: compute dtype %d not supported", compute_dtype);
  }
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

int pvb2_ternary(int op, const pvb2_tensor* out, const pvb2_tensor* a, const pvb2_tensor* b, const pvb2_tensor* c,
                 double p0, int compute_dtype, pvb2_stream stream) {
  const int64_t n = numel(out);
  if (n == 0) return PVB2_OK;
  PVB2_CHECK_ARG(a->ndim == out->ndim && b->ndim == out->ndim && c->ndim == out->ndim,
                 "pvb2_ternary: ndim mismatch");
  cudaStream_t s = as_stream(stream);
  IterShape it;
  const pvb2_tensor* ts[4] = {out, a, b, c};
  make_iter(&it, ts, 4);
  const int block = 256;
  const int grid = grid_for(n, block);
  switch (compute_dtype) {
    case PVB2_F32:
      ternary_generic_kernel<float><<<grid, block, 0, s>>>(it, op, out->data, out->dtype, a->data, a->dtype, b->data,
                                                           b->dtype, c->data, c->dtype, (float)p0, n);
      break;
    case PVB2_F64:
      ternary_generic_kernel<double><<<grid, block, 0, s>>>(it, op, out->data, out->dtype, a->data, a->dtype,
                                                            b->data, b->dtype, c->data, c->dtype, p0, n);
      break;
    case PVB2_I64:
    case PVB2_I32:
    case PVB2_BOOL:
    case PVB2_U8:
      ternary_generic_kernel<int64_t><<<grid, block, 0, s>>>(it, op, out->data, out->dtype, a->data, a->dtype,
                                                             b->data, b->dtype, c->data, c->dtype, (int64_t)p0, n);
      break;
    default:
      return fail(PVB2_ERR_UNSUPPORTED, "pvb2_ternary: compute dtype %d not supported", compute_dtype);
  }
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

}  // extern "C"
