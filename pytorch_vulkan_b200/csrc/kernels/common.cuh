// Shared helpers for the libpvb2 kernels: status handling, launch
// accounting, dtype conversion and strided-index arithmetic.
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>
#include <atomic>
#include <string>
#include "../../../include/pvb2.h"

namespace pvb2 {

// ---------------------------------------------------------------- errors
void set_error(const char* fmt, ...);
int fail(int code, const char* fmt, ...);
extern std::atomic<int64_t> g_launches;

#define PVB2_CHECK_ARG(cond, ...)                                   \
  do {                                                              \
    if (!(cond)) return ::pvb2::fail(PVB2_ERR_INVALID, __VA_ARGS__); \
  } while (0)

#define PVB2_CUDA_TRY(expr)                                                         \
  do {                                                                              \
    cudaError_t _e = (expr);                                                        \
    if (_e != cudaSuccess)                                                          \
      return ::pvb2::fail(PVB2_ERR_CUDA, "%s failed: %s (%s:%d)", #expr,           \
                          cudaGetErrorString(_e), __FILE__, __LINE__);              \
  } while (0)

// Call after every <<<>>> launch: counts the launch and reports a launch error.
#define PVB2_LAUNCH_CHECK()                                                         \
  do {                                                                              \
    ::pvb2::g_launches.fetch_add(1, std::memory_order_relaxed);                     \
    cudaError_t _e = cudaGetLastError();                                            \
    if (_e != cudaSuccess)                                                          \
      return ::pvb2::fail(PVB2_ERR_CUDA, "kernel launch failed: %s (%s:%d)",       \
                          cudaGetErrorString(_e), __FILE__, __LINE__);              \
  } while (0)

#define PVB2_TRY(expr)          \
  do {                          \
    int _s = (expr);            \
    if (_s != PVB2_OK) return _s; \
  } while (0)

inline cudaStream_t as_stream(pvb2_stream s) { return reinterpret_cast<cudaStream_t>(s); }

int num_sms();

inline int dtype_size(int dt) {
  switch (dt) {
    case PVB2_F32: return 4;
    case PVB2_F64: return 8;
    case PVB2_F16: return 2;
    case PVB2_BF16: return 2;
    case PVB2_I64: return 8;
    case PVB2_I32: return 4;
    case PVB2_I16: return 2;
    case PVB2_I8: return 1;
    case PVB2_U8: return 1;
    case PVB2_BOOL: return 1;
  }
  return 0;
}

inline int64_t numel(const pvb2_tensor* t) {
  int64_t n = 1;
  for (int i = 0; i < t->ndim; ++i) n *= t->sizes[i];
  return n;
}

inline bool is_contiguous(const pvb2_tensor* t) {
  if (numel(t) == 0) return true;  // torch treats empty tensors as contiguous
  int64_t expect = 1;
  for (int i = t->ndim - 1; i >= 0; --i) {
    if (t->sizes[i] != 1 && t->strides[i] != expect) return false;
    expect *= t->sizes[i];
  }
  return true;
}

// channels-last (NHWC storage) test for a 4-D NCHW-indexed tensor
inline bool is_channels_last(const pvb2_tensor* t) {
  if (t->ndim != 4) return false;
  const int64_t N = t->sizes[0], C = t->sizes[1], H = t->sizes[2], W = t->sizes[3];
  (void)N;
  auto ok = [&](int d, int64_t s) { return t->sizes[d] == 1 || t->strides[d] == s; };
  return ok(1, 1) && ok(3, C) && ok(2, C * W) && ok(0, C * W * H);
}

// ------------------------------------------------------- dtype load/store
template <typename T>
__device__ __forceinline__ T load_as(const void* base, int64_t off, int dt) {
  switch (dt) {
    case PVB2_F32: return (T)(static_cast<const float*>(base)[off]);
    case PVB2_F64: return (T)(static_cast<const double*>(base)[off]);
    case PVB2_I64: return (T)(static_cast<const int64_t*>(base)[off]);
    case PVB2_I32: return (T)(static_cast<const int32_t*>(base)[off]);
    case PVB2_I16: return (T)(static_cast<const int16_t*>(base)[off]);
    case PVB2_I8: return (T)(static_cast<const int8_t*>(base)[off]);
    case PVB2_U8: return (T)(static_cast<const uint8_t*>(base)[off]);
    case PVB2_BOOL: return (T)(static_cast<const uint8_t*>(base)[off] != 0);
    case PVB2_F16: {
      uint16_t h = static_cast<const uint16_t*>(base)[off];
      return (T)__half2float(*reinterpret_cast<const __half*>(&h));
    }
    case PVB2_BF16: {
      uint32_t u = ((uint32_t) static_cast<const uint16_t*>(base)[off]) << 16;
      return (T)__uint_as_float(u);
    }
  }
  return (T)0;
}

template <typename T>
__device__ __forceinline__ void store_as(void* base, int64_t off, int dt, T v) {
  switch (dt) {
    case PVB2_F32: static_cast<float*>(base)[off] = (float)v; break;
    case PVB2_F64: static_cast<double*>(base)[off] = (double)v; break;
    case PVB2_I64: static_cast<int64_t*>(base)[off] = (int64_t)v; break;
    case PVB2_I32: static_cast<int32_t*>(base)[off] = (int32_t)v; break;
    case PVB2_I16: static_cast<int16_t*>(base)[off] = (int16_t)v; break;
    case PVB2_I8: static_cast<int8_t*>(base)[off] = (int8_t)v; break;
    case PVB2_U8: static_cast<uint8_t*>(base)[off] = (uint8_t)v; break;
    case PVB2_BOOL: static_cast<uint8_t*>(base)[off] = (v != (T)0) ? 1 : 0; break;
    case PVB2_F16: {
      __half h = __float2half_rn((float)v);
      static_cast<__half*>(base)[off] = h;
      break;
    }
    case PVB2_BF16: {
      // round-to-nearest-even, NaN preserved
      float f = (float)v;
      uint32_t u = __float_as_uint(f);
      uint16_t r;
      if ((u & 0x7fffffffu) > 0x7f800000u) r = (uint16_t)((u >> 16) | 0x40);
      else r = (uint16_t)((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
      static_cast<uint16_t*>(base)[off] = r;
      break;
    }
  }
}

// ------------------------------------------------- strided index helper
// Up to MAX_ARGS operands sharing one iteration shape, dims coalesced on
// the host.  offsets computed from a linear index by div/mod per dim.
constexpr int kMaxArgs = 6;
struct IterShape {
  int ndim;
  int64_t sizes[PVB2_MAX_DIMS];
  int64_t strides[kMaxArgs][PVB2_MAX_DIMS];
};

// Build a coalesced iteration shape over `n` operands with identical sizes.
// Size-1 dims are dropped; adjacent dims merge when every operand's strides
// allow it.  Dim order is kept (last dim fastest).
void make_iter(IterShape* it, const pvb2_tensor* const* ts, int n);

__device__ __forceinline__ void iter_offsets(const IterShape& it, int nargs, int64_t linear, int64_t* offs) {
#pragma unroll
  for (int a = 0; a < kMaxArgs; ++a) offs[a] = 0;
  for (int d = it.ndim - 1; d >= 0; --d) {
    int64_t sz = it.sizes[d];
    int64_t idx = linear % sz;
    linear /= sz;
#pragma unroll
    for (int a = 0; a < kMaxArgs; ++a)
      if (a < nargs) offs[a] += idx * it.strides[a][d];
  }
}

// true the first time it is called with `mask` on the current device (for
// per-device one-time setup such as cudaFuncSetAttribute)
inline bool first_on_device(std::atomic<uint64_t>& mask) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return true;
  const uint64_t bit = 1ull << (dev & 63);
  return (mask.fetch_or(bit) & bit) == 0;
}

// Division by a runtime divisor d as a multiply-high and shift (Granlund and
// Montgomery's method, as CUTLASS's FastDivmod states it): m = ceil(2^p / d),
// p = 31 + ceil(log2 d); exact for dividends below 2^31.
struct FastDiv {
  int d;
  uint32_t m, s;
};
inline FastDiv fast_div(int d) {
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

inline int grid_for(int64_t n, int block, int max_blocks_per_sm = 8) {
  int64_t b = (n + block - 1) / block;
  int64_t cap = (int64_t)num_sms() * max_blocks_per_sm;
  if (b > cap) b = cap;
  if (b < 1) b = 1;
  return (int)b;
}

}  // namespace pvb2
