// tcgen05 TF32 GEMM for sm_100a:  C[z] = alpha * A[z] @ B[z] + beta * C[z] (+ bias)
//
// Persistent, warp-specialised kernel (one CTA per SM, 192 threads):
//   warp 0      TMA producer: one thread streams 128x32 A and BNx32 B tiles
//               (128-byte swizzle) into a shared-memory ring (4-8 stages);
//   warp 1      MMA issuer: allocates 2*BN TMEM columns, one thread issues
//               tcgen05.mma kind::tf32 (M=128, N=BN, K=8) four times per
//               32-deep K block and releases ring slots with tcgen05.commit;
//   warps 2-5   epilogue: drain a finished 128xBN fp32 accumulator from TMEM
//               (tcgen05.ld 32x32b), apply alpha / bias, stage each warp's
//               32x32 block in shared memory and write it with a TMA tensor
//               store (row-major C: 128-byte swizzled rows; column-major C:
//               plain 32x32 box); with beta != 0 or strides TMA cannot
//               express, per-element stores with C's strides.  Two TMEM
//               accumulators alternate so the epilogue of one tile overlaps
//               the main loop of the next.
// Either operand may be K-major (K contiguous) or MN-major (M/N contiguous),
// chosen from its strides, so transposed views (linear's W^T, dW = dY^T X)
// need no copies.  Every wait is bounded (tc_common.cuh).
//
// Replaces the dlprim gpu::GEMM / IP kernels behind mm / bmm / addmm / linear
// (src/vision_ops.cpp:243-351, 513-673).
#include <cudaTypedefs.h>
#include <mutex>
#include "tc_common.cuh"

namespace pvb2 {

// Warp roles: warps 0..3 issue TMA loads (one thread each, every fourth ring
// stage: a thread's bulk-tensor copies are processed one after another, so
// several issuing warps multiply the load rate), warp 4 allocates TMEM and
// issues the MMAs, warps 5..8 run the epilogue (TMEM lane quarter = warp % 4).
constexpr int kBM = 128, kBK = 32, kProducers = 4, kMmaWarp = kProducers, kThreads = (kProducers + 5) * 32;

struct GemmEpi {
  float* C;
  int64_t scb, scm, scn;  // C strides (elements)
  float alpha, beta;
  const float* bias;
  int bias_dim;           // 1: bias[n], 0: bias[m]
  int M, N, K, batch;
  int a_bcast, b_bcast;   // operand shared by all batches (batch stride 0)
  int store;              // kStoreScalar / kStoreRows / kStoreCols
  int splits, kb_per;     // split-K: split s covers K blocks [s * kb_per, (s + 1) * kb_per)
};

enum { kStoreScalar = 0, kStoreRows = 1, kStoreCols = 2 };

// Ring depth: as many stages as fit in 192 KB (8 at BN = 64, 6 at 128, 4 at
// 256).  Iteration i goes to stage i % STAGES and producer i % 4, so with 6
// stages a stage passes between producers; that is safe because every
// producer waits for the stage's previous use to be consumed (empty barrier)
// and the MMA consumes the ring in order, so no waiter is ever more than one
// phase ahead of a barrier.
template <int BN>
struct GemmSmem {
  static constexpr int A_BYTES = kBM * kBK * 4;
  static constexpr int B_BYTES = BN * kBK * 4;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (192 * 1024) / STAGE_BYTES;
  static constexpr int EPI_OFF = STAGES * STAGE_BYTES;  // 2 x 4 KB store boxes per epilogue warp
  static constexpr int BAR_OFF = EPI_OFF + 4 * 2 * 4096;
  // full[STAGES], empty[STAGES], acc_full[2], acc_empty[2], tmem slot, abort
  static constexpr int TOTAL = BAR_OFF + (2 * STAGES + 4) * 8 + 16;
};

template <int BN, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tf32_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmC, GemmEpi ep) {
  using L = GemmSmem<BN>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  constexpr int kStages = L::STAGES;
  uint64_t* full = (uint64_t*)(smem + L::BAR_OFF);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = (uint32_t*)(acc_empty + 2);
  volatile int* abort = (volatile int*)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles_m = (ep.M + kBM - 1) / kBM, tiles_n = (ep.N + BN - 1) / BN;
  const int base_tiles = tiles_m * tiles_n * ep.batch;
  const int total_tiles = base_tiles * ep.splits;  // split-major: tile = sp * base_tiles + base tile
  const int kblocks = (ep.K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    *abort = 0;
    fence_barrier_init();
  }
  if (warp == kMmaWarp) tmem_alloc(tmem_slot, 2 * BN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp < kProducers) {
    // ------------------------------------------------------------ producers
    if (lane == 0) {
      tma_prefetch(&tmA);
      tma_prefetch(&tmB);
      uint32_t it = 0;
      for (int tile = blockIdx.x; tile < total_tiles && !*abort; tile += gridDim.x) {
        const int bt = tile % base_tiles, sp = tile / base_tiles;
        const int nb = bt % tiles_n, mb = (bt / tiles_n) % tiles_m, z = bt / (tiles_n * tiles_m);
        const int za = ep.a_bcast ? 0 : z, zb = ep.b_bcast ? 0 : z;
        const int kb0 = sp * ep.kb_per, kb1 = min(kblocks, kb0 + ep.kb_per);
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % kStages;
          const uint32_t ph = (it / kStages) & 1;
          if ((int)(it % kProducers) != warp) continue;
          if (!mbar_wait(&empty[s], ph ^ 1, abort)) break;
          uint8_t* sa = smem + s * L::STAGE_BYTES;
          uint8_t* sb = sa + L::A_BYTES;
          mbar_arrive_expect_tx(&full[s], L::STAGE_BYTES);
          if (!A_MN) {
            tma_load_3d(sa, &tmA, &full[s], kb * kBK, mb * kBM, za);
          } else {
#pragma unroll
            for (int j = 0; j < kBM / 32; ++j) tma_load_3d(sa + j * 32 * kBK * 4, &tmA, &full[s], mb * kBM + 32 * j, kb * kBK, za);
          }
          if (!B_MN) {
            tma_load_3d(sb, &tmB, &full[s], kb * kBK, nb * BN, zb);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 32; ++j) tma_load_3d(sb + j * 32 * kBK * 4, &tmB, &full[s], nb * BN + 32 * j, kb * kBK, zb);
          }
        }
      }
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issue
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_tf32(kBM, BN, A_MN, B_MN);
      uint32_t it = 0;
      int local = 0;
      for (int tile = blockIdx.x; tile < total_tiles && !*abort; tile += gridDim.x, ++local) {
        const int buf = local & 1;
        const uint32_t aph = (local >> 1) & 1;
        if (!mbar_wait(&acc_empty[buf], aph ^ 1, abort)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        const int kb0 = (tile / base_tiles) * ep.kb_per, kb1 = min(kblocks, kb0 + ep.kb_per);
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % kStages;
          const uint32_t ph = (it / kStages) & 1;
          if (!mbar_wait(&full[s], ph, abort)) break;
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * L::STAGE_BYTES);
          const uint32_t sb = sa + L::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < kBK / 8; ++kk) {
            const uint64_t ad = A_MN ? desc_mnmajor(sa, kk, 32 * kBK * 4) : desc_kmajor(sa, kk);
            const uint64_t bd = B_MN ? desc_mnmajor(sb, kk, 32 * kBK * 4) : desc_kmajor(sb, kk);
            mma_tf32(d_tmem, ad, bd, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
          }
          mma_commit(&empty[s]);
        }
        mma_commit(&acc_full[buf]);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;  // TMEM lanes 32*quarter .. +31
    float* stage = (float*)(smem + L::EPI_OFF) + quarter * 2 * 1024;
    uint32_t echunk = 0;
    int local = 0;
    for (int tile = blockIdx.x; tile < total_tiles && !*abort; tile += gridDim.x, ++local) {
      const int bt = tile % base_tiles;
      const int nb = bt % tiles_n, mb = (bt / tiles_n) % tiles_m, z = bt / (tiles_n * tiles_m);
      const int zs = z + (tile / base_tiles) * ep.batch;  // z of the split's partial slab
      const int buf = local & 1;
      const uint32_t aph = (local >> 1) & 1;
      if (!mbar_wait(&acc_full[buf], aph, abort)) break;
      tc_fence_after();
      const int m0 = mb * kBM + quarter * 32;
      const int m = m0 + lane;
      const bool mrow = m < ep.M;
      const float bias_m = (ep.bias && ep.bias_dim == 0 && mrow) ? ep.bias[m] : 0.f;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        float v[32];
        tmem_ld32(tmem_base + ((uint32_t)(quarter * 32) << 16) + buf * BN + c * 32, v);
        const int n0 = nb * BN + c * 32;
        if (ep.store == kStoreScalar) {
          if (mrow) {
            float* crow = ep.C + (int64_t)z * ep.scb + (int64_t)m * ep.scm;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int n = n0 + j;
              if (n < ep.N) {
                float* p = crow + (int64_t)n * ep.scn;
                float r = ep.alpha * v[j];
                if (ep.beta != 0.f) r = fmaf(ep.beta, *p, r);
                if (ep.bias) r += ep.bias_dim == 1 ? ep.bias[n] : bias_m;
                *p = r;
              }
            }
          }
        } else if (m0 < ep.M && n0 < ep.N) {  // warp-uniform: the box has output to store
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            float r = ep.alpha * v[j];
            if (ep.bias) r += ep.bias_dim == 1 ? (n0 + j < ep.N ? ep.bias[n0 + j] : 0.f) : bias_m;
            v[j] = r;
          }
          // boxes alternate per issued store: wait until the store before the
          // most recent one has read this box
          float* st = stage + (echunk & 1) * 1024;
          if (lane == 0) bulk_wait_read<1>();
          __syncwarp();
          if (ep.store == kStoreRows) {
            // row `lane` of the box, 16-byte chunk q at chunk q ^ (lane % 8)
            // (the 128-byte swizzle the tensor map applies)
#pragma unroll
            for (int q = 0; q < 8; ++q)
              *reinterpret_cast<float4*>(st + lane * 32 + ((q ^ (lane & 7)) * 4)) =
                  make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) st[j * 32 + lane] = v[j];
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            if (ep.store == kStoreRows) tma_store_3d(&tmC, st, n0, m0, zs);
            else tma_store_3d(&tmC, st, m0, n0, zs);
            bulk_commit();
          }
          ++echunk;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
    if (lane == 0) bulk_wait_all();  // boxes stay valid until their stores finish
  }
  // ---------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    if (*abort) {
      // let any MMA still in flight finish before the columns are released
      if (lane == 0) {
        mma_commit(&acc_full[0]);
      }
      __syncwarp();
      const uint64_t t0 = globaltimer();
      while (globaltimer() - t0 < 10000000ull) {
      }
    }
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * BN);
  }
}

// ------------------------------------------------------------ host side
static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
  });
  return fn;
}

int encode_tiled(CUtensorMap* map, int rank, const void* base, const uint64_t* dims, const uint64_t* strides_bytes,
                 const uint32_t* box, CUtensorMapSwizzle swizzle, CUtensorMapL2promotion l2,
                 const uint32_t* elem_strides) {
  auto fn = get_encode();
  if (!fn) return fail(PVB2_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  if (elem_strides)
    for (int i = 0; i < rank; ++i) estr[i] = elem_strides[i];
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, rank, const_cast<void*>(base), dims, strides_bytes, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, l2, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(PVB2_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return PVB2_OK;
}

// A [batch, rows, cols] operand as a rank-3 TMA map whose innermost dim is
// its unit-stride dim.  For A, rows = M and cols = K; for B, rows = K and
// cols = N (`k_is_cols` says which).  *mn_major reports whether the unit-stride
// dim is M/N (true) or K (false).  Returns PVB2_ERR_UNSUPPORTED when TMA's
// alignment rules (16-byte base and strides) do not hold.
struct OperandLayout {
  bool mn_major;
  int bcast;
  uint64_t dims[3], str[2];
};

// the TMA view of an operand (no driver call): dims and byte strides, or
// PVB2_ERR_UNSUPPORTED when the alignment rules do not hold
static int operand_layout(const pvb2_tensor* t, bool k_is_cols, OperandLayout* o) {
  const int64_t Bt = t->sizes[0], R = t->sizes[1], Cc = t->sizes[2];
  const int64_t s0 = t->strides[0], s1 = t->strides[1], s2 = t->strides[2];
  int64_t inner, outer, ostride;
  bool inner_is_cols;
  if (s2 == 1 || Cc == 1) {
    inner_is_cols = true;
    inner = Cc;
    outer = R;
    ostride = s1;
  } else if (s1 == 1 || R == 1) {
    inner_is_cols = false;
    inner = R;
    outer = Cc;
    ostride = s2;
  } else {
    return PVB2_ERR_UNSUPPORTED;
  }
  const bool inner_is_k = inner_is_cols == k_is_cols;
  o->mn_major = !inner_is_k;
  if (outer == 1) ostride = (inner + 3) / 4 * 4;
  if (ostride <= 0 || (ostride * 4) % 16 != 0) return PVB2_ERR_UNSUPPORTED;
  o->bcast = (Bt > 1 && s0 == 0) ? 1 : 0;
  const int64_t nb = (o->bcast || Bt == 1) ? 1 : Bt;
  const int64_t bstride = nb == 1 ? ostride * outer : s0;
  if (bstride <= 0 || (bstride * 4) % 16 != 0) return PVB2_ERR_UNSUPPORTED;
  if ((uintptr_t)t->data % 16 != 0) return PVB2_ERR_UNSUPPORTED;
  o->dims[0] = (uint64_t)inner;
  o->dims[1] = (uint64_t)outer;
  o->dims[2] = (uint64_t)nb;
  o->str[0] = (uint64_t)ostride * 4;
  o->str[1] = (uint64_t)bstride * 4;
  return PVB2_OK;
}

static int make_operand_map(CUtensorMap* map, const pvb2_tensor* t, bool k_is_cols, int mn_box, bool* mn_major,
                            int* bcast) {
  OperandLayout o;
  const int st = operand_layout(t, k_is_cols, &o);
  if (st != PVB2_OK) return st;
  *mn_major = o.mn_major;
  *bcast = o.bcast;
  uint32_t box[3];
  if (*mn_major) {
    box[0] = 32;  // 128 bytes along M/N
    box[1] = kBK;
  } else {
    box[0] = kBK;  // 128 bytes along K
    box[1] = (uint32_t)mn_box;
  }
  box[2] = 1;
  return encode_tiled(map, 3, t->data, o.dims, o.str, box,
                      *mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B);
}

// C [batch, M, N] as the TMA store target of 32x32 boxes: kStoreRows when N
// is the unit-stride dim (boxes of 32 rows x 128 bytes, 128-byte swizzle),
// kStoreCols when M is, kStoreScalar when the strides or the base do not
// meet TMA's 16-byte rules.
static int make_output_map(CUtensorMap* map, const pvb2_tensor* C) {
  const int64_t Bt = C->sizes[0], M = C->sizes[1], N = C->sizes[2];
  const int64_t sb = C->strides[0], sm = C->strides[1], sn = C->strides[2];
  if ((uintptr_t)C->data % 16 != 0) return kStoreScalar;
  const bool rows = sn == 1 || N == 1;
  const bool cols = !rows && (sm == 1 || M == 1);
  if (!rows && !cols) return kStoreScalar;
  const int64_t inner = rows ? N : M, outer = rows ? M : N;
  int64_t ostride = rows ? sm : sn;
  if (outer == 1) ostride = (inner + 3) / 4 * 4;
  const int64_t bstride = Bt == 1 ? ostride * outer : sb;
  if (ostride < inner || (ostride * 4) % 16 != 0 || bstride <= 0 || (bstride * 4) % 16 != 0) return kStoreScalar;
  uint64_t dims[3] = {(uint64_t)inner, (uint64_t)outer, (uint64_t)Bt};
  uint64_t str[2] = {(uint64_t)ostride * 4, (uint64_t)bstride * 4};
  uint32_t box[3] = {32, 32, 1};
  if (encode_tiled(map, 3, C->data, dims, str, box, rows ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE) !=
      PVB2_OK)
    return kStoreScalar;
  return rows ? kStoreRows : kStoreCols;
}

template <int BN, bool A_MN, bool B_MN>
static int launch_gemm(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, const GemmEpi& ep,
                       cudaStream_t s) {
  constexpr int smem = GemmSmem<BN>::TOTAL + 1024;
  static std::atomic<uint64_t> attr_done{0};
  if (first_on_device(attr_done))
    PVB2_CUDA_TRY(cudaFuncSetAttribute(gemm_tf32_kernel<BN, A_MN, B_MN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       smem));
  const int tiles = ((ep.M + kBM - 1) / kBM) * ((ep.N + BN - 1) / BN) * ep.batch * ep.splits;
  const int grid = std::min(tiles, num_sms());
  gemm_tf32_kernel<BN, A_MN, B_MN><<<grid, kThreads, smem, s>>>(ma, mb, mc, ep);
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

template <int BN>
static int dispatch_majors(bool amn, bool bmn, const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc,
                           const GemmEpi& ep, cudaStream_t s) {
  if (!amn && !bmn) return launch_gemm<BN, false, false>(ma, mb, mc, ep, s);
  if (!amn && bmn) return launch_gemm<BN, false, true>(ma, mb, mc, ep, s);
  if (amn && !bmn) return launch_gemm<BN, true, false>(ma, mb, mc, ep, s);
  return launch_gemm<BN, true, true>(ma, mb, mc, ep, s);
}

// Split-K: out[z][m][n] = alpha * sum_s part[s][z][m][n] + beta * C + bias,
// the S partial slabs (row pitch n4) summed in order s = 0..S-1
__global__ void gemm_splitk_reduce_kernel(const float* __restrict__ part, int S, int64_t n4, GemmEpi ep) {
  const int64_t nq = (ep.N + 3) / 4;
  const int64_t total = (int64_t)ep.batch * ep.M * nq;
  const int64_t slab = (int64_t)ep.batch * ep.M * n4;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = e / nq;  // z * M + m
    const int n = (int)(e % nq) * 4;
    const int z = (int)(row / ep.M), m = (int)(row % ep.M);
    const float* p = part + row * n4 + n;
    float4 acc = __ldg(reinterpret_cast<const float4*>(p));
    for (int sp = 1; sp < S; ++sp) {
      const float4 x = __ldg(reinterpret_cast<const float4*>(p + sp * slab));
      acc.x += x.x;
      acc.y += x.y;
      acc.z += x.z;
      acc.w += x.w;
    }
    const float v[4] = {acc.x, acc.y, acc.z, acc.w};
    float* crow = ep.C + (int64_t)z * ep.scb + (int64_t)m * ep.scm;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (n + j >= ep.N) break;
      float* c = crow + (int64_t)(n + j) * ep.scn;
      float r = ep.alpha * v[j];
      if (ep.beta != 0.f) r = fmaf(ep.beta, *c, r);
      if (ep.bias) r += ep.bias[ep.bias_dim == 1 ? n + j : m];
      *c = r;
    }
  }
}

// Problem shape, tile width and split count, shared by the workspace query
// and the launch so both see the same plan.
struct GemmPlan {
  bool tc = false;
  int BN = 256;
  int splits = 1, kb_per = 0;
  int64_t n4 = 0;
  size_t ws_bytes = 0;
};

static GemmPlan plan_gemm(const pvb2_tensor* A, const pvb2_tensor* B, const pvb2_tensor* C, int math) {
  GemmPlan p;
  if (math != PVB2_MATH_TF32 || getenv("PVB2_DISABLE_TC")) return p;
  const int64_t batch = C->sizes[0], M = C->sizes[1], N = C->sizes[2], K = A->sizes[2];
  // small problems: the SIMT engine is as fast and exact
  if ((double)M * N * K * batch < (double)(1 << 22) || K < 8) return p;
  if (M > INT32_MAX / 2 || N > INT32_MAX / 2 || K > INT32_MAX / 2 || batch > 65535) return p;
  p.tc = true;
  p.BN = N <= 64 ? 64 : (N <= 128 ? 128 : 256);
  // too few output tiles to fill the SMs and a long K: split K so that every
  // SM gets work (dW = dY^T X of a linear layer: a small output, K = tokens)
  const int64_t tiles = ((M + kBM - 1) / kBM) * ((N + p.BN - 1) / p.BN) * batch;
  const int64_t kblocks = (K + kBK - 1) / kBK;
  const int sms = num_sms();
  if (tiles * 2 <= sms && kblocks >= 16) {
    const int64_t S = std::min<int64_t>(sms / tiles, kblocks / 8);
    if (S >= 2) {
      p.kb_per = (int)((kblocks + S - 1) / S);
      p.splits = (int)((kblocks + p.kb_per - 1) / p.kb_per);
      p.n4 = (N + 3) / 4 * 4;
      p.ws_bytes = (size_t)p.splits * batch * M * p.n4 * sizeof(float);
    }
  }
  if (p.splits < 2) {
    p.splits = 1;
    p.kb_per = (int)kblocks;
  }
  return p;
}

size_t gemm_tc_workspace(const pvb2_tensor* A, const pvb2_tensor* B, const pvb2_tensor* C, int math) {
  return plan_gemm(A, B, C, math).ws_bytes;
}

// whether gemm_tc runs this product on the tensor cores (host logic only)
bool gemm_tc_path(const pvb2_tensor* A, const pvb2_tensor* B, const pvb2_tensor* C, int math) {
  if (!plan_gemm(A, B, C, math).tc) return false;
  OperandLayout o;
  return operand_layout(A, true, &o) == PVB2_OK && operand_layout(B, false, &o) == PVB2_OK;
}

int gemm_tc(const pvb2_tensor* A, const pvb2_tensor* B, const pvb2_tensor* C, const float* bias, int bias_dim,
            float alpha, float beta, int math, cudaStream_t s, bool* handled, void* workspace,
            size_t workspace_bytes) {
  *handled = false;
  GemmPlan plan = plan_gemm(A, B, C, math);
  if (!plan.tc) return PVB2_OK;
  const int64_t batch = C->sizes[0], M = C->sizes[1], N = C->sizes[2], K = A->sizes[2];
  const int BN = plan.BN;
  CUtensorMap ma, mb;
  bool amn = false, bmn = false;
  int abc = 0, bbc = 0;
  if (make_operand_map(&ma, A, /*k_is_cols=*/true, kBM, &amn, &abc) != PVB2_OK) return PVB2_OK;
  if (make_operand_map(&mb, B, /*k_is_cols=*/false, BN, &bmn, &bbc) != PVB2_OK) return PVB2_OK;
  pvb2::set_error("");
  // without room for the partial slabs the product runs unsplit
  const bool split = plan.splits > 1 && workspace && workspace_bytes >= plan.ws_bytes;
  if (!split) {
    plan.splits = 1;
    plan.kb_per = (int)((K + kBK - 1) / kBK);
  }
  GemmEpi ep;
  ep.C = (float*)C->data;
  ep.scb = C->strides[0];
  ep.scm = C->strides[1];
  ep.scn = C->strides[2];
  ep.alpha = alpha;
  ep.beta = beta;
  ep.bias = bias;
  ep.bias_dim = bias_dim;
  ep.M = (int)M;
  ep.N = (int)N;
  ep.K = (int)K;
  ep.batch = (int)batch;
  ep.a_bcast = abc;
  ep.b_bcast = bbc;
  ep.splits = plan.splits;
  ep.kb_per = plan.kb_per;
  CUtensorMap mc;
  memset(&mc, 0, sizeof(mc));
  GemmEpi main = ep;
  if (split) {
    // the main kernel stores raw partial sums, slab s at z = s * batch + z
    uint64_t dims[3] = {(uint64_t)N, (uint64_t)M, (uint64_t)plan.splits * batch};
    uint64_t str[2] = {(uint64_t)plan.n4 * 4, (uint64_t)plan.n4 * M * 4};
    uint32_t box[3] = {32, 32, 1};
    PVB2_TRY(encode_tiled(&mc, 3, workspace, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B));
    main.store = kStoreRows;
    main.alpha = 1.f;
    main.beta = 0.f;
    main.bias = nullptr;
  } else {
    main.store = beta == 0.f ? make_output_map(&mc, C) : kStoreScalar;
  }
  int st;
  if (BN == 64) st = dispatch_majors<64>(amn, bmn, ma, mb, mc, main, s);
  else if (BN == 128) st = dispatch_majors<128>(amn, bmn, ma, mb, mc, main, s);
  else st = dispatch_majors<256>(amn, bmn, ma, mb, mc, main, s);
  if (st != PVB2_OK) return st;
  if (split) {
    const int64_t total = batch * M * ((N + 3) / 4);
    gemm_splitk_reduce_kernel<<<grid_for(total, 256), 256, 0, s>>>((const float*)workspace, plan.splits, plan.n4,
                                                                   ep);
    PVB2_LAUNCH_CHECK();
  }
  *handled = true;
  return PVB2_OK;
}

}  // namespace pvb2

extern "C" PVB2_API int pvb2_tc_status(int* timed_out, int reset) {
  return pvb2::tc_timeout_flag_local(timed_out, reset);
}
