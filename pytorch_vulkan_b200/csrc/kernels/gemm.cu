// Strided, batched GEMM with alpha/beta and an optional bias:
//   C[b] = alpha * A[b] @ B[b] + beta * C[b] (+ bias)
//
// Replaces dlprim's gpu::GEMM / batch_sgemm and IPForward / IPBackwardData /
// IPBackwardFilter as used by mm/bmm/addmm (src/vision_ops.cpp:513-673) and
// linear (vision_ops.cpp:243-351).  math == TF32 routes to the tcgen05
// kernel (gemm_tc.cu) whenever the operands satisfy its alignment rules;
// everything else, and math == FP32, runs the exact SIMT engine.
#include "igemm_simt.cuh"

namespace pvb2 {

int gemm_tc(const pvb2_tensor* A, const pvb2_tensor* B, const pvb2_tensor* C, const float* bias, int bias_dim,
            float alpha, float beta, int math, cudaStream_t s, bool* handled, void* workspace,
            size_t workspace_bytes);
size_t gemm_tc_workspace(const pvb2_tensor* A, const pvb2_tensor* B, const pvb2_tensor* C, int math);
bool gemm_tc_path(const pvb2_tensor* A, const pvb2_tensor* B, const pvb2_tensor* C, int math);

struct GemmProb {
  int64_t M, N;
  int zcount;
  int64_t K;
  const float* A;
  const float* B;
  float* C;
  int64_t sab, sam, sak, sbb, sbk, sbn, scb, scm, scn;
  float alpha, beta;
  const float* bias;
  int bias_dim;
  struct BCol {
    int64_t off;
  };
  __device__ int64_t k_begin(int) const { return 0; }
  __device__ int64_t k_end(int) const { return K; }
  __device__ BCol bcol(int z, int64_t n) const { return BCol{(int64_t)z * sbb + n * sbn}; }
  __device__ float a(int z, int64_t m, int64_t k) const { return __ldg(A + (int64_t)z * sab + m * sam + k * sak); }
  __device__ float b(int, const BCol& c, int64_t k) const { return __ldg(B + c.off + k * sbk); }
  __device__ void store(int z, int64_t m, int64_t n, float acc) const {
    float* p = C + (int64_t)z * scb + m * scm + n * scn;
    float v = alpha * acc;
    if (beta != 0.f) v = fmaf(beta, *p, v);
    if (bias) v += bias[bias_dim == 1 ? n : m];
    *p = v;
  }
};

}  // namespace pvb2

using namespace pvb2;

static int gemm_check(const pvb2_tensor* A, const pvb2_tensor* B, const pvb2_tensor* C, int bias_dim) {
  PVB2_CHECK_ARG(A->ndim == 3 && B->ndim == 3 && C->ndim == 3, "gemm: operands must be 3-D [batch, rows, cols]");
  PVB2_CHECK_ARG(A->dtype == PVB2_F32 && B->dtype == PVB2_F32 && C->dtype == PVB2_F32, "gemm: float32 only");
  const int64_t batch = C->sizes[0], M = C->sizes[1], N = C->sizes[2], K = A->sizes[2];
  PVB2_CHECK_ARG(A->sizes[0] == batch && B->sizes[0] == batch, "gemm: batch mismatch");
  PVB2_CHECK_ARG(A->sizes[1] == M && B->sizes[1] == K && B->sizes[2] == N, "gemm: shape mismatch");
  PVB2_CHECK_ARG(bias_dim == 0 || bias_dim == 1, "gemm: bias_dim must be 0 or 1");
  return PVB2_OK;
}

extern "C" size_t pvb2_gemm_workspace_size(const pvb2_tensor* A, const pvb2_tensor* B, const pvb2_tensor* C,
                                           int math) {
  if (gemm_check(A, B, C, 0) != PVB2_OK) return 0;
  if ((int64_t)C->sizes[0] * C->sizes[1] * C->sizes[2] == 0) return 0;
  return gemm_tc_workspace(A, B, C, math);
}

extern "C" int pvb2_gemm_path(const pvb2_tensor* A, const pvb2_tensor* B, const pvb2_tensor* C, int math) {
  if (gemm_check(A, B, C, 0) != PVB2_OK) return -1;
  if (math != PVB2_MATH_TF32 && math != PVB2_MATH_FP32) return -1;
  if ((int64_t)C->sizes[0] * C->sizes[1] * C->sizes[2] == 0) return 0;
  return gemm_tc_path(A, B, C, math) ? 1 : 0;
}

extern "C" int pvb2_gemm(const pvb2_tensor* A, const pvb2_tensor* B, const pvb2_tensor* C, const float* bias,
                         int bias_dim, double alpha, double beta, int math, pvb2_stream stream) {
  return pvb2_gemm_ws(A, B, C, bias, bias_dim, alpha, beta, math, nullptr, 0, stream);
}

extern "C" int pvb2_gemm_ws(const pvb2_tensor* A, const pvb2_tensor* B, const pvb2_tensor* C, const float* bias,
                            int bias_dim, double alpha, double beta, int math, void* workspace,
                            size_t workspace_bytes, pvb2_stream stream) {
  PVB2_TRY(gemm_check(A, B, C, bias_dim));
  if (math != PVB2_MATH_TF32 && math != PVB2_MATH_FP32)
    return fail(PVB2_ERR_UNSUPPORTED, "gemm: math mode %d is not implemented (0 = TF32, 1 = exact fp32)", math);
  const int64_t batch = C->sizes[0], M = C->sizes[1], N = C->sizes[2], K = A->sizes[2];
  if (batch * M * N == 0) return PVB2_OK;
  cudaStream_t s = as_stream(stream);
  if (math != PVB2_MATH_FP32) {
    bool handled = false;
    PVB2_TRY(gemm_tc(A, B, C, bias, bias_dim, (float)alpha, (float)beta, math, s, &handled, workspace,
                     workspace_bytes));
    if (handled) return PVB2_OK;
  }
  PVB2_CHECK_ARG(batch <= 65535, "gemm: batch too large");
  GemmProb pb;
  pb.M = M;
  pb.N = N;
  pb.K = K;
  pb.zcount = (int)batch;
  pb.A = (const float*)A->data;
  pb.B = (const float*)B->data;
  pb.C = (float*)C->data;
  pb.sab = A->strides[0]; pb.sam = A->strides[1]; pb.sak = A->strides[2];
  pb.sbb = B->strides[0]; pb.sbk = B->strides[1]; pb.sbn = B->strides[2];
  pb.scb = C->strides[0]; pb.scm = C->strides[1]; pb.scn = C->strides[2];
  pb.alpha = (float)alpha;
  pb.beta = (float)beta;
  pb.bias = bias;
  pb.bias_dim = bias_dim;
  return launch_igemm_simt(pb, s);
}
