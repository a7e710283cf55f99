// Exact-fp32 SIMT implicit GEMM: a 64x64x16 CTA tile, 256 threads each
// owning a 4x4 register block, double-buffered shared memory.  A problem
// type supplies the operand gathers A(m,k), B(k,n) and the epilogue; the
// same engine serves strided GEMM and the three convolution passes.  It is
// the fp32-exact path (math=FP32) and the fallback for shapes the tensor-
// core kernels do not take.
#pragma once
#include "common.cuh"

namespace pvb2 {

constexpr int kSimtBM = 64, kSimtBN = 64, kSimtBK = 16, kSimtThreads = 256;

// Prob must provide:
//   int64_t M, N, K (per z-slice), int zcount
//   __device__ void begin(int z, int64_t k_lo, int64_t k_hi)     (optional state)
//   __device__ float a(int z, int64_t m, int64_t k) const
//   __device__ float b(int z, int64_t k, int64_t n) const         (thread-fixed n; see bprep)
//   __device__ void store(int z, int64_t m, int64_t n, float acc) const
//   k range per z: [k_begin(z), k_end(z))
template <class Prob, typename Acc = float>
__global__ void __launch_bounds__(kSimtThreads) igemm_simt_kernel(Prob pb) {
  __shared__ __align__(16) float As[2][kSimtBK][kSimtBM + 4];
  __shared__ __align__(16) float Bs[2][kSimtBK][kSimtBN + 4];
  const int tid = threadIdx.x;
  const int tm = tid >> 4, tn = tid & 15;
  const int z = blockIdx.z;
  const int64_t m0 = (int64_t)blockIdx.y * kSimtBM;
  const int64_t n0 = (int64_t)blockIdx.x * kSimtBN;
  const int64_t kb = pb.k_begin(z), ke = pb.k_end(z);

  // loader coordinates: A with k fastest, B with n fastest
  const int a_k = tid & 15, a_m = tid >> 4;   // + 16*i
  const int b_n = tid & 63, b_k = tid >> 6;   // + 4*i
  typename Prob::BCol bcol = pb.bcol(z, n0 + b_n);

  Acc acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = (Acc)0;

  float ra[4], rb[4];
  auto load_regs = [&](int64_t k0) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t m = m0 + a_m + 16 * i, k = k0 + a_k;
      ra[i] = (m < pb.M && k < ke) ? pb.a(z, m, k) : 0.f;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t k = k0 + b_k + 4 * i, n = n0 + b_n;
      rb[i] = (n < pb.N && k < ke) ? pb.b(z, bcol, k) : 0.f;
    }
  };
  auto store_smem = [&](int buf) {
#pragma unroll
    for (int i = 0; i < 4; ++i) As[buf][a_k][a_m + 16 * i] = ra[i];
#pragma unroll
    for (int i = 0; i < 4; ++i) Bs[buf][b_k + 4 * i][b_n] = rb[i];
  };

  int buf = 0;
  if (kb < ke) {
    load_regs(kb);
    store_smem(0);
  }
  __syncthreads();
  for (int64_t k0 = kb; k0 < ke; k0 += kSimtBK) {
    const bool more = k0 + kSimtBK < ke;
    if (more) load_regs(k0 + kSimtBK);
#pragma unroll
    for (int kk = 0; kk < kSimtBK; ++kk) {
      const float4 av = *reinterpret_cast<const float4*>(&As[buf][kk][tm * 4]);
      const float4 bv = *reinterpret_cast<const float4*>(&Bs[buf][kk][tn * 4]);
      const float a4[4] = {av.x, av.y, av.z, av.w};
      const float b4[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fma((Acc)a4[i], (Acc)b4[j], acc[i][j]);
    }
    if (more) {
      store_smem(buf ^ 1);
      __syncthreads();
      buf ^= 1;
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t m = m0 + tm * 4 + i;
    if (m >= pb.M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t n = n0 + tn * 4 + j;
      if (n < pb.N) pb.store(z, m, n, (float)acc[i][j]);
    }
  }
}

template <class Prob, typename Acc = float>
inline int launch_igemm_simt(const Prob& pb, cudaStream_t s) {
  if (pb.M == 0 || pb.N == 0 || pb.zcount == 0) return PVB2_OK;
  dim3 grid((unsigned)((pb.N + kSimtBN - 1) / kSimtBN), (unsigned)((pb.M + kSimtBM - 1) / kSimtBM),
            (unsigned)pb.zcount);
  if (grid.y > 65535 || grid.z > 65535) return fail(PVB2_ERR_UNSUPPORTED, "igemm_simt: grid too large");
  igemm_simt_kernel<Prob, Acc><<<grid, kSimtThreads, 0, s>>>(pb);
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

}  // namespace pvb2
