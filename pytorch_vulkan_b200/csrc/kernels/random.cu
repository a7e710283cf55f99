// Philox-4x32-10 counter-based random numbers, and dropout.
//
// Replaces dlprim::core::fill_random as used by bernoulli_/normal_/uniform_
// and native_dropout (src/random_ops.cpp:37-105).  Philox-4x32 with 10
// rounds is the generator of Salmon, Moraes, Dror and Shaw, "Parallel random
// numbers: as easy as 1, 2, 3" (SC'11): a 128-bit counter is mixed with a
// 64-bit key by ten rounds of two 32x32->64 multiplies, with the key bumped
// by the Weyl constants between rounds.  Element i of a fill uses counter
// (offset + i/4, 0) and output lane i%4, so a result depends only on
// (seed, offset, i) and not on the launch shape.
#include "common.cuh"

namespace pvb2 {

struct U4 {
  uint32_t x, y, z, w;
};

__device__ __forceinline__ U4 philox4x32_10(U4 ctr, uint32_t k0, uint32_t k1) {
  const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u;
  const uint32_t W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(M0, ctr.x), lo0 = M0 * ctr.x;
    const uint32_t hi1 = __umulhi(M1, ctr.z), lo1 = M1 * ctr.z;
    U4 n;
    n.x = hi1 ^ ctr.y ^ k0;
    n.y = lo1;
    n.z = hi0 ^ ctr.w ^ k1;
    n.w = lo0;
    ctr = n;
    k0 += W0;
    k1 += W1;
  }
  return ctr;
}

__device__ __forceinline__ float u32_to_unit(uint32_t v) {
  // 24 random bits -> [0, 1)
  return (float)(v >> 8) * (1.0f / 16777216.0f);
}

__device__ __forceinline__ U4 philox_block(uint64_t seed, uint64_t offset, uint64_t block) {
  const uint64_t c = offset + block;
  U4 ctr{(uint32_t)c, (uint32_t)(c >> 32), 0u, 0u};
  return philox4x32_10(ctr, (uint32_t)seed, (uint32_t)(seed >> 32));
}

__device__ __forceinline__ uint32_t lane_of(const U4& r, int k) {
  return k == 0 ? r.x : (k == 1 ? r.y : (k == 2 ? r.z : r.w));
}

__global__ void philox_fill_kernel(IterShape it, void* out, int dt, int dist, uint64_t seed, uint64_t offset,
                                   float p0, float p1, int64_t n) {
  const int64_t nblocks = (n + 3) / 4;
  for (int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; b < nblocks; b += (int64_t)gridDim.x * blockDim.x) {
    const U4 r = philox_block(seed, offset, (uint64_t)b);
    float v[4];
    if (dist == PVB2_RNG_NORMAL) {
      // Box-Muller on two pairs of uniforms
      for (int k = 0; k < 4; k += 2) {
        float u1 = u32_to_unit(lane_of(r, k));
        float u2 = u32_to_unit(lane_of(r, k + 1));
        u1 = fmaxf(u1, 1.0e-7f);
        const float rad = sqrtf(-2.f * logf(u1));
        float sn, cs;
        sincospif(2.f * u2, &sn, &cs);
        v[k] = p0 + p1 * rad * cs;
        v[k + 1] = p0 + p1 * rad * sn;
      }
    } else {
      for (int k = 0; k < 4; ++k) {
        const float u = u32_to_unit(lane_of(r, k));
        v[k] = dist == PVB2_RNG_UNIFORM ? p0 + (p1 - p0) * u : (u < p0 ? 1.f : 0.f);
      }
    }
    for (int k = 0; k < 4; ++k) {
      const int64_t i = b * 4 + k;
      if (i >= n) break;
      int64_t offs[kMaxArgs];
      iter_offsets(it, 1, i, offs);
      store_as<float>(out, offs[0], dt, v[k]);
    }
  }
}

__global__ void dropout_fwd_kernel(const float* __restrict__ x, float* __restrict__ y, uint8_t* __restrict__ mask,
                                   int64_t n, float p, float scale, uint64_t seed, uint64_t offset) {
  const int64_t nblocks = (n + 3) / 4;
  for (int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; b < nblocks; b += (int64_t)gridDim.x * blockDim.x) {
    const U4 r = philox_block(seed, offset, (uint64_t)b);
    for (int k = 0; k < 4; ++k) {
      const int64_t i = b * 4 + k;
      if (i >= n) break;
      const bool keep = u32_to_unit(lane_of(r, k)) >= p;
      if (mask) mask[i] = keep ? 1 : 0;
      y[i] = keep ? x[i] * scale : 0.f;
    }
  }
}

__global__ void dropout_bwd_kernel(const float* __restrict__ dy, const uint8_t* __restrict__ mask,
                                   float* __restrict__ dx, int64_t n, float scale) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    dx[i] = mask[i] ? dy[i] * scale : 0.f;
}

}  // namespace pvb2

using namespace pvb2;

extern "C" {

int pvb2_philox_fill(int dist, const pvb2_tensor* out, uint64_t seed, uint64_t offset, double p0, double p1,
                     pvb2_stream stream) {
  const int64_t n = numel(out);
  if (n == 0) return PVB2_OK;
  PVB2_CHECK_ARG(dist >= 0 && dist <= 2, "philox_fill: bad distribution %d", dist);
  IterShape it;
  const pvb2_tensor* ts[1] = {out};
  make_iter(&it, ts, 1);
  const int64_t nb = (n + 3) / 4;
  philox_fill_kernel<<<grid_for(nb, 256), 256, 0, as_stream(stream)>>>(it, out->data, out->dtype, dist, seed, offset,
                                                                       (float)p0, (float)p1, n);
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

int pvb2_dropout_fwd(const float* x, float* y, uint8_t* mask, int64_t n, double p, uint64_t seed, uint64_t offset,
                     pvb2_stream stream) {
  if (n == 0) return PVB2_OK;
  PVB2_CHECK_ARG(p >= 0.0 && p <= 1.0, "dropout: p must be in [0, 1]");
  const float scale = p < 1.0 ? (float)(1.0 / (1.0 - p)) : 0.f;
  const int64_t nb = (n + 3) / 4;
  dropout_fwd_kernel<<<grid_for(nb, 256), 256, 0, as_stream(stream)>>>(x, y, mask, n, (float)p, scale, seed, offset);
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

int pvb2_dropout_bwd(const float* dy, const uint8_t* mask, float* dx, int64_t n, double scale, pvb2_stream stream) {
  if (n == 0) return PVB2_OK;
  dropout_bwd_kernel<<<grid_for(n, 256), 256, 0, as_stream(stream)>>>(dy, mask, dx, n, (float)scale);
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

}  // extern "C"
