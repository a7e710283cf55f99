// Multi-tensor kernels: SGD with momentum, _foreach_* binary maps, and
// flatten/unflatten of many tensors into one bucket.
//
// In the reference, torch.optim.SGD's foreach path has no kernel on the
// device and falls back to one mul_/add_ launch per parameter (add_out and
// mul_out, src/pointwise_ops.cpp:115-172,407-411: ~3 launches x 161 tensors
// for ResNet-50).  Here one launch walks every tensor: the host packs the
// tensor list into the kernel parameter block and each CTA finds its tensor
// by binary search over per-tensor chunk prefix sums.
#include "common.cuh"

namespace pvb2 {

constexpr int kMtMax = 192;           // tensors per launch
constexpr int64_t kMtChunk = 8192;    // elements per CTA

struct MtPack {
  int n;
  int total_chunks;
  float* p0[kMtMax];
  const float* p1[kMtMax];
  float* p2[kMtMax];
  int64_t numel[kMtMax];
  int chunk_prefix[kMtMax + 1];
};

__device__ __forceinline__ int mt_find(const MtPack& pk, int chunk) {
  int lo = 0, hi = pk.n - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (pk.chunk_prefix[mid] <= chunk) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

struct SgdArgs {
  float lr, momentum, dampening, weight_decay, grad_scale;
  int nesterov, first_step;
};

// p0 = params, p1 = grads, p2 = momentum buffers (may be null when momentum == 0)
__global__ void sgd_kernel(MtPack pk, SgdArgs a) {
  for (int chunk = blockIdx.x; chunk < pk.total_chunks; chunk += gridDim.x) {
    const int t = mt_find(pk, chunk);
    const int64_t c = chunk - pk.chunk_prefix[t];
    const int64_t start = c * kMtChunk;
    const int64_t end = min(pk.numel[t], start + kMtChunk);
    float* p = pk.p0[t];
    const float* g = pk.p1[t];
    float* buf = pk.p2[t];
    for (int64_t i = start + threadIdx.x; i < end; i += blockDim.x) {
      float d = g[i];
      if (a.grad_scale != 1.f) d *= a.grad_scale;
      if (a.weight_decay != 0.f) d = fmaf(a.weight_decay, p[i], d);
      if (a.momentum != 0.f) {
        float b;
        if (a.first_step) b = d;
        else b = fmaf(1.f - a.dampening, d, buf[i] * a.momentum);
        buf[i] = b;
        d = a.nesterov ? fmaf(a.momentum, b, d) : b;
      }
      p[i] = fmaf(-a.lr, d, p[i]);
    }
  }
}

// out[i] = a[i] op b[i] (or scalar);  p0 = out, p1 = a, p2 = b (as float*)
__global__ void foreach_binary_kernel(MtPack pk, int op, float scalar, float alpha, int has_b) {
  for (int chunk = blockIdx.x; chunk < pk.total_chunks; chunk += gridDim.x) {
    const int t = mt_find(pk, chunk);
    const int64_t c = chunk - pk.chunk_prefix[t];
    const int64_t start = c * kMtChunk;
    const int64_t end = min(pk.numel[t], start + kMtChunk);
    float* o = pk.p0[t];
    const float* x = pk.p1[t];
    const float* y = pk.p2[t];
    for (int64_t i = start + threadIdx.x; i < end; i += blockDim.x) {
      const float b = has_b ? y[i] : scalar;
      float r;
      switch (op) {
        case PVB2_BIN_ADD: r = fmaf(alpha, b, x[i]); break;
        case PVB2_BIN_SUB: r = fmaf(-alpha, b, x[i]); break;
        case PVB2_BIN_MUL: r = x[i] * b; break;
        default: r = x[i] / b; break;
      }
      o[i] = r;
    }
  }
}

// direction 0: flat[off_t + i] = t[i] * scale ;  1: t[i] = flat[off_t + i] * scale
struct FlatPack {
  int n;
  int total_chunks;
  float* t[kMtMax];
  int64_t numel[kMtMax];
  int64_t offset[kMtMax];
  int chunk_prefix[kMtMax + 1];
};

__global__ void flatten_kernel(FlatPack pk, float* flat, int direction, float scale) {
  for (int chunk = blockIdx.x; chunk < pk.total_chunks; chunk += gridDim.x) {
    int lo = 0, hi = pk.n - 1;
    while (lo < hi) {
      int mid = (lo + hi + 1) >> 1;
      if (pk.chunk_prefix[mid] <= chunk) lo = mid;
      else hi = mid - 1;
    }
    const int t = lo;
    const int64_t start = (int64_t)(chunk - pk.chunk_prefix[t]) * kMtChunk;
    const int64_t end = min(pk.numel[t], start + kMtChunk);
    float* tp = pk.t[t];
    float* fp = flat + pk.offset[t];
    if (direction == 0) {
      for (int64_t i = start + threadIdx.x; i < end; i += blockDim.x) fp[i] = tp[i] * scale;
    } else {
      for (int64_t i = start + threadIdx.x; i < end; i += blockDim.x) tp[i] = fp[i] * scale;
    }
  }
}

template <typename Pack>
static int fill_prefix(Pack& pk, const int64_t* numels, int base, int cnt) {
  pk.n = cnt;
  int acc = 0;
  for (int k = 0; k < cnt; ++k) {
    pk.numel[k] = numels[base + k];
    pk.chunk_prefix[k] = acc;
    acc += (int)((numels[base + k] + kMtChunk - 1) / kMtChunk);
  }
  pk.chunk_prefix[cnt] = acc;
  pk.total_chunks = acc;
  return acc;
}

}  // namespace pvb2

using namespace pvb2;

extern "C" {

int pvb2_sgd_multi(int n, float* const* params, const float* const* grads, float* const* momentum_bufs,
                   const int64_t* numels, double lr, double momentum, double dampening, double weight_decay,
                   int nesterov, int first_step, double grad_scale, pvb2_stream stream) {
  PVB2_CHECK_ARG(n >= 0, "sgd: negative tensor count");
  PVB2_CHECK_ARG(momentum == 0.0 || momentum_bufs != nullptr, "sgd: momentum buffers required");
  SgdArgs a{(float)lr, (float)momentum, (float)dampening, (float)weight_decay, (float)grad_scale, nesterov,
            first_step};
  cudaStream_t s = as_stream(stream);
  for (int base = 0; base < n; base += kMtMax) {
    const int cnt = std::min(kMtMax, n - base);
    MtPack pk;
    for (int k = 0; k < cnt; ++k) {
      pk.p0[k] = params[base + k];
      pk.p1[k] = grads[base + k];
      pk.p2[k] = momentum_bufs ? momentum_bufs[base + k] : nullptr;
    }
    const int chunks = fill_prefix(pk, numels, base, cnt);
    if (chunks == 0) continue;
    const int grid = std::min(chunks, num_sms() * 8);
    sgd_kernel<<<grid, 256, 0, s>>>(pk, a);
    PVB2_LAUNCH_CHECK();
  }
  return PVB2_OK;
}

int pvb2_foreach_binary(int op, int n, float* const* out, const float* const* a, const float* const* b,
                        const int64_t* numels, double scalar, double alpha, pvb2_stream stream) {
  PVB2_CHECK_ARG(op == PVB2_BIN_ADD || op == PVB2_BIN_SUB || op == PVB2_BIN_MUL || op == PVB2_BIN_DIV,
                 "foreach_binary: unsupported op %d", op);
  cudaStream_t s = as_stream(stream);
  for (int base = 0; base < n; base += kMtMax) {
    const int cnt = std::min(kMtMax, n - base);
    MtPack pk;
    for (int k = 0; k < cnt; ++k) {
      pk.p0[k] = out[base + k];
      pk.p1[k] = a[base + k];
      pk.p2[k] = b ? const_cast<float*>(b[base + k]) : nullptr;
    }
    const int chunks = fill_prefix(pk, numels, base, cnt);
    if (chunks == 0) continue;
    const int grid = std::min(chunks, num_sms() * 8);
    foreach_binary_kernel<<<grid, 256, 0, s>>>(pk, op, (float)scalar, (float)alpha, b ? 1 : 0);
    PVB2_LAUNCH_CHECK();
  }
  return PVB2_OK;
}

int pvb2_flatten_multi(int n, float* const* tensors, const int64_t* numels, float* flat, int direction, double scale,
                       pvb2_stream stream) {
  cudaStream_t s = as_stream(stream);
  int64_t off = 0;
  for (int base = 0; base < n; base += kMtMax) {
    const int cnt = std::min(kMtMax, n - base);
    FlatPack pk;
    for (int k = 0; k < cnt; ++k) {
      pk.t[k] = tensors[base + k];
      pk.offset[k] = off;
      off += numels[base + k];
    }
    const int chunks = fill_prefix(pk, numels, base, cnt);
    if (chunks == 0) continue;
    const int grid = std::min(chunks, num_sms() * 8);
    flatten_kernel<<<grid, 256, 0, s>>>(pk, flat, direction, (float)scale);
    PVB2_LAUNCH_CHECK();
  }
  return PVB2_OK;
}

}  // extern "C"
