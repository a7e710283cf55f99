// Tensor-core (tcgen05, TF32) implicit-GEMM convolution for sm_100a.
//
// Replaces dlprim's Conv2DForward / Conv2DBackwardData / Conv2DBackwardFilter
// (src/vision_ops.cpp:61-186) for groups == 1.  Activations arrive NCHW.
//
//   1x1 stride-1 (pointwise) convolutions read NCHW directly: the pixels of an
//   image are contiguous, so a 32-pixel x 32-channel TMA box is an MN-major
//   operand tile.  GEMM rows are four 32-pixel "slots" (n, hw0); an image
//   whose pixel count is not a multiple of 32 leaves its last slot part-empty
//   (TMA fills zeros, the store clips).
//     forward   Y[n, k, hw]  = sum_c W[k, c] X[n, c, hw]     (A = X slots, B = W K-major)
//     dgrad     dX[n, c, hw] = sum_k W[k, c] dY[n, k, hw]    (A = dY slots, B = W MN-major)
//     wgrad     dW[k, c]     = sum_{n,hw} dY[n, k, hw] X[n, c, hw]  (both K-major along pixels)
//   Other convolutions first stage their activations channels-last (NHWC,
//   channels zero-padded to a multiple of 4) in the caller's workspace,
//   because TMA can shift a tile by a filter tap along W and H only when the
//   contiguous dim is C.
//     forward   Y[pix, k] = sum_{r,s,c} Xnhwc[n, p*sh-ph+r*dh, q*sw-pw+s*dw, c] * Wp[k, r, s, c]
//               GEMM M = 128 output pixels (a BW x BH x BNI block), N = BN output
//               channels, K = R*S*ceil(C/32) blocks of 32 channels.  A: one 4-D
//               TMA box per K block, shifted by the tap, stride via the tensor
//               map's element strides (K-major).  B: packed weights (K-major).
//     dgrad     any stride, by sub-pixel phases: the dX rows/columns of one
//               residue class mod the stride receive a fixed subset of taps, so
//               each phase is a stride-1 correlation over dY (tap offsets in a
//               table, weights packed per phase) written to dX with strides.
//     small C   (the 3-channel stem): im2col columns Xcol[n, p, q, (c, r, s)]
//               (147 for a 7x7 filter on 3 channels, padded to 148) make the
//               forward a 1x1 GEMM with K = 148 and the weight gradient a
//               GEMM of Xcol (MN-major) against dY read NCHW (K-major).
//     wgrad     dW[k, c, r, s] = sum_pix dYnhwc[pix, k] * Xnhwc[shift_rs(pix), c]
//               GEMM M = 128 output channels, N = BN input channels, K = 32-pixel
//               blocks (MN-major A and B), one tap per tile.
//   Weight gradients split K (pixels) over CTAs into fp32 partials (stored
//   by TMA as row-contiguous 32 x 32 boxes) that a second kernel sums in a
//   fixed order while transposing them into dW's [K][C][R][S] layout.
//
// Epilogue of the forward-shaped launches: each epilogue warp owns 32
// accumulator rows; per 32-channel chunk it loads TMEM into registers, writes
// the chunk to a shared-memory box (double-buffered per warp) and issues one
// TMA tensor store, so global writes are full-line bulk transfers that run
// behind the next chunk.  The box is (32 q) x (32 k) of an NCHW row, or a
// (q, p) patch of up to 32 pixels, or a run of whole rows of a plane whose
// row pitch is not 16-byte aligned; outputs with strided pixels (dgrad
// phases of strided convolutions) use direct stores.
// Kernel structure (warp roles, TMA ring, TMEM double buffer, bounded waits)
// is the one of the GEMM in gemm_tc.cu.
#include <mutex>
#include "tc_common.cuh"

namespace pvb2 {

// Warp roles: warps 0..3 issue TMA loads (one thread each, every fourth ring
// stage: a thread's bulk-tensor copies are processed one after another, so
// several issuing warps multiply the load rate), warp 4 allocates TMEM and
// issues the MMAs, warps 5..12 run the epilogue.  A warp may read only the
// TMEM lane quarter warp % 4, so two epilogue warps share each quarter and
// split its 32-column chunks by parity: warp w takes chunks c with
// c % 2 == (w - 5) / 4.  Each epilogue warp stores through its own 4 KB box,
// so eight TMA stores per SM are in flight while the next chunks are loaded.
constexpr int cBM = 128, cBK = 32, cProducers = 4, cMmaWarp = cProducers, cEpiWarps = 8,
              cThreads = (cProducers + 1 + cEpiWarps) * 32;

constexpr int kMaxTaps = 8;

// where the operands of one launch come from
enum ConvMode : int {
  kImplicit = 0,  // forward / dgrad phase: A = channels-last tap boxes (K-major), B = packed weights (K-major)
  kPwFwd = 1,     // 1x1 stride-1 forward: A = NCHW 32-pixel slots (MN-major), B = W[K][C] (K-major)
  kPwDgrad = 2,   // 1x1 stride-1 dgrad: A = dY NCHW slots (MN-major), B = W[K][C] read along C (MN-major)
  kWgrad = 3,     // weight gradient over channels-last tap boxes (A and B MN-major)
  kPwWgrad = 4,   // 1x1 stride-1 weight gradient: A = dY, B = X, both NCHW, K-major along pixels
  kImWgrad = 5,   // weight gradient over im2col columns: A = Xcol[n][pix][j] (MN-major), B = dY NCHW (K-major)
  kWgradT = 6,    // weight gradient, at most 64 input and output channels: A = two taps' channels-last x
                  // boxes (M = tap pair x 64 channels), B = dY (N = output channels); both MN-major
};
// A launch stages KB K blocks per ring stage (the kernel's third template
// parameter): 2 for BN <= 128 in the implicit forward / dgrad (two 32-channel
// blocks of one tap) and the pointwise, implicit and two-tap weight
// gradients (two 32-pixel blocks), so that one mbarrier wait of the MMA
// thread covers eight MMAs instead of four.

// how a forward-shaped launch writes its output
enum EpiMode : int {
  kEpiScalar = 0,  // direct per-element stores (any output strides)
  kEpiBox = 1,     // TMA box (ebq q) x (ebp p) x 32 k of an NCHW-shaped output
  kEpiFlat = 2,    // TMA box of ebp whole rows (ebp * Q pixels) x 32 k, plane viewed flat
  kEpiSlots = 3,   // TMA box of one 32-pixel slot x 32 k (pointwise modes)
};

struct ConvTcArgs {
  int N, Cin, Cp, Kout, P, Q, R, S;   // the conv computed (for dgrad: the equivalent conv over dY)
  int sh, sw, ph, pw, dh, dw;
  // input coordinate of output (p, q) under tap (r, s): (p*sh + tap_h[r], q*sw + tap_w[s])
  int tap_h[kMaxTaps], tap_w[kMaxTaps];
  // forward-shaped output element (n, k, p, q) lives at
  // out[obase + n*on + k*ok + p*op + q*oq]
  int64_t obase, on, ok, op, oq;
  int cblocks;                        // ceil(Cp / 32)
  int bw, bh, bni;                    // pixel block (fwd: 128 pixels = M; wgrad: 32 pixels = K block)
  int tq, tp, tn;                     // pixel blocks along q, p, n
  int kt;                             // fwd: output-channel tiles ceil(Kout / BN); wgrad: ceil(Kout / 128)
  int ct;                             // wgrad: input-channel tiles ceil(Cin / BN)
  int splits, kb_per_split, total_kb; // wgrad split-K over pixel blocks
  int hwb, slots;                     // pointwise: 32-pixel slots per image, slots in all images
  int win, wq;                        // kImWgrad over filter-row windows (win = 1): output width Q
  int cpairs;                         // kImplicit with KB = 2: ceil(cblocks / 2), the channel-block pairs per tap
  int tiles;                          // tiles of this launch
  int epi, ebq, ebp;                  // EpiMode and its box extents
  float* out;
  const float* bias;
  // pointwise dgrad only: dX = dgrad + addend (same NCHW layout as dX; may be dX itself)
  const float* addend;
};

// Ring depth: as many stages as fit in 192 KB (8 at BN = 64, 6 at 128, 4 at
// 256).  Iteration i goes to stage i % STAGES and producer i % 4, so with 6
// stages a stage passes between producers; that is safe because every
// producer waits for the stage's previous use to be consumed (empty barrier)
// and the MMA consumes the ring in order, so no waiter is ever more than one
// phase ahead of a barrier.
//
// KB K blocks of 32 per stage.  An mbarrier wait costs
// the MMA-issuing thread about 180 cycles, as much as three 128x64x8 TF32
// MMAs; a stage of two channel blocks (eight MMAs) hides it at BN = 128.
template <int BN, int KB = 1>
struct ConvSmem {
  static constexpr int A_BYTES = KB * cBM * cBK * 4;
  static constexpr int B_BYTES = KB * BN * cBK * 4;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (192 * 1024) / STAGE_BYTES;
  static constexpr int EPI_OFF = STAGES * STAGE_BYTES;  // one box of 32 x 32 fp32 per epilogue warp
  static constexpr int EPI_BYTES = cEpiWarps * 32 * 32 * 4;
  static constexpr int BAR_OFF = EPI_OFF + EPI_BYTES;
  static constexpr int TOTAL = BAR_OFF + (2 * STAGES + 4) * 8 + 16;
};
static_assert(ConvSmem<256>::STAGES >= cProducers && ConvSmem<64>::TOTAL + 1024 <= 232448 && ConvSmem<128>::TOTAL + 1024 <= 232448 &&
                  ConvSmem<256>::TOTAL + 1024 <= 232448,
              "conv tile does not fit in shared memory");

// The addend's 32 x 32 box (pixels bx.., channels k0..) of image n, one
// 128-byte run per channel; indices past the plane or the channels are
// clamped to the box's last valid pixel / channel (read, then masked off by
// the caller), so the 32 loads carry no branches and issue back to back.
// Every address read lies in the box this warp stores next, so an addend
// that is the output itself is read before it is overwritten.
__device__ __forceinline__ void load_addend_chunk(const ConvTcArgs& a, int n, int bx, int k0, int lane,
                                                  float (&pre)[32]) {
  const int px = min(bx + lane, a.Q - 1);
  const float* ad = a.addend + (int64_t)n * a.Kout * a.Q + px;
#pragma unroll
  for (int j = 0; j < 32; ++j) pre[j] = ad[(int64_t)min(k0 + j, a.Kout - 1) * a.Q];
}

// L2 prefetch of a warp's chunks of the BN-channel addend box (pixels
// bx..bx+31 of image n; chunks c = half, half + 2, ...): lane j takes
// channel row 32 c + j of each; a 32-pixel run may straddle two 128-byte
// lines, so both ends are fetched.  Clamped like the loads.
template <int BN>
__device__ __forceinline__ void prefetch_addend_l2(const ConvTcArgs& a, int n, int bx, int k0, int lane, int half) {
  const float* img = a.addend + (int64_t)n * a.Kout * a.Q;
  const int p0 = min(bx, a.Q - 1), p1 = min(bx + 31, a.Q - 1);
#pragma unroll
  for (int c = half; c < BN / 32; c += 2) {
    const float* row = img + (int64_t)min(k0 + c * 32 + lane, a.Kout - 1) * a.Q;
    asm volatile("prefetch.global.L2 [%0];" ::"l"(row + p0));
    asm volatile("prefetch.global.L2 [%0];" ::"l"(row + p1));
  }
}

template <int BN, int MODE, int KB>
__global__ void __launch_bounds__(cThreads, 1)
    conv_tf32_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmC, ConvTcArgs a) {
  constexpr bool WG = MODE == kWgrad || MODE == kPwWgrad || MODE == kImWgrad || MODE == kWgradT;
  constexpr bool PW = MODE == kPwFwd || MODE == kPwDgrad;
  constexpr bool A_MN = MODE == kPwFwd || MODE == kPwDgrad || MODE == kWgrad || MODE == kImWgrad || MODE == kWgradT;
  constexpr bool B_MN = MODE == kPwDgrad || MODE == kWgrad || MODE == kWgradT;
  using L = ConvSmem<BN, KB>;
  constexpr int A_BLK = L::A_BYTES / KB, B_BLK = L::B_BYTES / KB;  // one K block's A / B bytes
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* full = (uint64_t*)(smem + L::BAR_OFF);
  constexpr int cStages = L::STAGES;
  uint64_t* empty = full + cStages;
  uint64_t* acc_full = empty + cStages;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = (uint32_t*)(acc_empty + 2);
  volatile int* abort = (volatile int*)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int RS = a.R * a.S;
  const int total_tiles = a.tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < cStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], cEpiWarps);
    }
    *abort = 0;
    fence_barrier_init();
  }
  if (warp == cMmaWarp) tmem_alloc(tmem_slot, 2 * BN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // tile -> coordinates
  auto fwd_tile = [&](int tile, int& kt, int& q0, int& p0, int& n0) {
    kt = tile % a.kt;
    const int pix = tile / a.kt;
    q0 = (pix % a.tq) * a.bw;
    p0 = ((pix / a.tq) % a.tp) * a.bh;
    n0 = (pix / (a.tq * a.tp)) * a.bni;
  };
  auto wg_tile = [&](int tile, int& sp, int& km, int& ctile, int& rs) {
    sp = tile % a.splits;
    int t = tile / a.splits;
    km = t % a.kt;
    t /= a.kt;
    ctile = t % a.ct;
    rs = t / a.ct;
  };
  auto wg_range = [&](int sp, int& kb0, int& kb1) {
    kb0 = sp * a.kb_per_split;
    kb1 = min(a.total_kb, kb0 + a.kb_per_split);
  };

  if (warp < cProducers) {
    // ------------------------------------------------------------ producers
    // issuing warps: at most one per ring stage, so that each warp's
    // previous stage had its use STAGES back consumed and no parity wait on
    // an empty barrier is ever two phases ahead of it
    constexpr int nissue = cStages < cProducers ? cStages : cProducers;
    if (lane == 0 && warp < nissue) {
      tma_prefetch(&tmA);
      tma_prefetch(&tmB);
      uint32_t it = 0;
      for (int tile = blockIdx.x; tile < total_tiles && !*abort; tile += gridDim.x) {
        if (MODE == kImplicit && KB == 2) {
          int kt, q0, p0, n0;
          fwd_tile(tile / a.splits, kt, q0, p0, n0);
          int kb0, kb1;
          wg_range(tile % a.splits, kb0, kb1);
          for (int kb = kb0; kb < kb1; ++kb, ++it) {
            const int s_ = it % cStages;
            const uint32_t ph = (it / cStages) & 1;
            if ((int)(it % nissue) != warp) continue;
            if (!mbar_wait(&empty[s_], ph ^ 1, abort)) break;
            // stage = tap rs, channel blocks 2 cp and 2 cp + 1 (past the
            // channels A reads zeros, so an odd last block adds nothing)
            const int rs = kb / a.cpairs, cp = kb - rs * a.cpairs;
            const int r = rs / a.S, s = rs % a.S;
            uint8_t* sa = smem + s_ * L::STAGE_BYTES;
            mbar_arrive_expect_tx(&full[s_], L::STAGE_BYTES);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int cb = 2 * cp + h;
              tma_load_4d(sa + h * cBM * cBK * 4, &tmA, &full[s_], cb * 32, q0 * a.sw + a.tap_w[s],
                          p0 * a.sh + a.tap_h[r], n0);
              tma_load_2d(sa + L::A_BYTES + h * BN * cBK * 4, &tmB, &full[s_], rs * a.Cp + cb * 32, kt * BN);
            }
          }
        } else if (MODE == kImplicit) {
          int kt, q0, p0, n0;
          fwd_tile(tile / a.splits, kt, q0, p0, n0);
          int kb0, kb1;
          wg_range(tile % a.splits, kb0, kb1);
          for (int kb = kb0; kb < kb1; ++kb, ++it) {
            const int s_ = it % cStages;
            const uint32_t ph = (it / cStages) & 1;
            if ((int)(it % nissue) != warp) continue;
            if (!mbar_wait(&empty[s_], ph ^ 1, abort)) break;
            const int rs = kb / a.cblocks, cb = kb % a.cblocks;
            const int r = rs / a.S, s = rs % a.S;
            uint8_t* sa = smem + s_ * L::STAGE_BYTES;
            mbar_arrive_expect_tx(&full[s_], L::STAGE_BYTES);
            tma_load_4d(sa, &tmA, &full[s_], cb * 32, q0 * a.sw + a.tap_w[s], p0 * a.sh + a.tap_h[r], n0);
            tma_load_2d(sa + L::A_BYTES, &tmB, &full[s_], rs * a.Cp + cb * 32, kt * BN);
          }
        } else if (PW) {
          const int kt = tile % a.kt, g = tile / a.kt;
          for (int kb = 0; kb < a.cblocks; ++kb, ++it) {
            const int s_ = it % cStages;
            const uint32_t ph = (it / cStages) & 1;
            if ((int)(it % nissue) != warp) continue;
            if (!mbar_wait(&empty[s_], ph ^ 1, abort)) break;
            uint8_t* sa = smem + s_ * L::STAGE_BYTES;
            uint8_t* sb = sa + L::A_BYTES;
            mbar_arrive_expect_tx(&full[s_], L::STAGE_BYTES);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              // slots past the last image read out of range: TMA fills zeros
              const int slot = g * 4 + j;
              const int n = slot / a.hwb;
              tma_load_3d(sa + j * 32 * cBK * 4, &tmA, &full[s_], (slot - n * a.hwb) * 32, kb * 32, n);
            }
            if (MODE == kPwFwd) {
              tma_load_2d(sb, &tmB, &full[s_], kb * 32, kt * BN);
            } else {
#pragma unroll
              for (int j = 0; j < BN / 32; ++j) tma_load_2d(sb + j * 32 * cBK * 4, &tmB, &full[s_], kt * BN + 32 * j, kb * 32);
            }
          }
        } else if (MODE == kWgradT) {
          // tile (split, tap pair): rows 32 j .. of A are tap 2 pair + j / 2,
          // input channels 32 (j % 2) ..; a pair past the last tap loads the
          // last tap again (its rows are not stored)
          int sp, km, ctile, pr;
          wg_tile(tile, sp, km, ctile, pr);
          int kb0, kb1;
          wg_range(sp, kb0, kb1);
          for (int kb = kb0; kb < kb1; ++kb, ++it) {
            const int s_ = it % cStages;
            const uint32_t ph = (it / cStages) & 1;
            if ((int)(it % nissue) != warp) continue;
            if (!mbar_wait(&empty[s_], ph ^ 1, abort)) break;
            mbar_arrive_expect_tx(&full[s_], L::STAGE_BYTES);
            // pixel blocks KB kb .. KB kb + KB - 1 (a block past the last
            // image lies outside the maps and loads zeros)
#pragma unroll
            for (int h = 0; h < KB; ++h) {
              const int pb = kb * KB + h;
              const int q0 = (pb % a.tq) * a.bw, p0 = ((pb / a.tq) % a.tp) * a.bh, n0 = (pb / (a.tq * a.tp)) * a.bni;
              uint8_t* sa = smem + s_ * L::STAGE_BYTES + h * A_BLK;
              uint8_t* sb = smem + s_ * L::STAGE_BYTES + L::A_BYTES + h * B_BLK;
#pragma unroll
              for (int j = 0; j < cBM / 32; ++j) {
                const int tap = min(2 * pr + (j >> 1), RS - 1), r = tap / a.S, s = tap - r * a.S;
                tma_load_4d(sa + j * 32 * cBK * 4, &tmA, &full[s_], 32 * (j & 1), q0 * a.sw + a.tap_w[s],
                            p0 * a.sh + a.tap_h[r], n0);
              }
#pragma unroll
              for (int j = 0; j < BN / 32; ++j)
                tma_load_4d(sb + j * 32 * cBK * 4, &tmB, &full[s_], ctile * BN + 32 * j, q0, p0, n0);
            }
          }
        } else if (MODE == kWgrad) {
          int sp, km, ctile, rs;
          wg_tile(tile, sp, km, ctile, rs);
          const int r = rs / a.S, s = rs % a.S;
          int kb0, kb1;
          wg_range(sp, kb0, kb1);
          for (int kb = kb0; kb < kb1; ++kb, ++it) {
            const int s_ = it % cStages;
            const uint32_t ph = (it / cStages) & 1;
            if ((int)(it % nissue) != warp) continue;
            if (!mbar_wait(&empty[s_], ph ^ 1, abort)) break;
            mbar_arrive_expect_tx(&full[s_], L::STAGE_BYTES);
#pragma unroll
            for (int h = 0; h < KB; ++h) {
              const int pb = kb * KB + h;
              const int q0 = (pb % a.tq) * a.bw, p0 = ((pb / a.tq) % a.tp) * a.bh, n0 = (pb / (a.tq * a.tp)) * a.bni;
              uint8_t* sa = smem + s_ * L::STAGE_BYTES + h * A_BLK;
              uint8_t* sb = smem + s_ * L::STAGE_BYTES + L::A_BYTES + h * B_BLK;
#pragma unroll
              for (int j = 0; j < cBM / 32; ++j)
                tma_load_4d(sa + j * 32 * cBK * 4, &tmA, &full[s_], km * cBM + 32 * j, q0, p0, n0);
#pragma unroll
              for (int j = 0; j < BN / 32; ++j)
                tma_load_4d(sb + j * 32 * cBK * 4, &tmB, &full[s_], ctile * BN + 32 * j, q0 * a.sw + a.tap_w[s],
                            p0 * a.sh + a.tap_h[r], n0);
            }
          }
        } else {  // kPwWgrad / kImWgrad: K blocks are (image, 32-pixel slot) pairs
          int sp, km, ctile, rs;
          wg_tile(tile, sp, km, ctile, rs);
          int kb0, kb1;
          wg_range(sp, kb0, kb1);
          for (int kb = kb0; kb < kb1; ++kb, ++it) {
            const int s_ = it % cStages;
            const uint32_t ph = (it / cStages) & 1;
            if ((int)(it % nissue) != warp) continue;
            if (!mbar_wait(&empty[s_], ph ^ 1, abort)) break;
            uint8_t* sa = smem + s_ * L::STAGE_BYTES;
            mbar_arrive_expect_tx(&full[s_], L::STAGE_BYTES);
            if (MODE == kPwWgrad) {
              // slots KB kb ..; one past the last image loads zeros
#pragma unroll
              for (int h = 0; h < KB; ++h) {
                const int sl = kb * KB + h, n = sl / a.hwb, hw0 = (sl - n * a.hwb) * 32;
                tma_load_3d(sa + h * A_BLK, &tmA, &full[s_], hw0, km * cBM, n);
                tma_load_3d(sa + L::A_BYTES + h * B_BLK, &tmB, &full[s_], hw0, ctile * BN, n);
              }
              continue;
            }
            const int n = kb / a.hwb, hw0 = (kb - n * a.hwb) * 32;
            if (a.win) {
              // rows km * 128 + 32 j .. : filter row 4 km + j, its 32-float
              // window of each pixel; the 32 pixels as two 16-pixel runs,
              // each inside one output row (Q % 16 == 0)
#pragma unroll
              for (int j = 0; j < cBM / 32; ++j)
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                  const int pq = hw0 + 16 * h, p = pq / a.wq, q = pq - p * a.wq;
                  tma_load_4d(sa + j * 32 * cBK * 4 + h * 16 * 128, &tmA, &full[s_], 0, q, p * a.sh + km * 4 + j, n);
                }
            } else {
#pragma unroll
              for (int j = 0; j < cBM / 32; ++j) tma_load_3d(sa + j * 32 * cBK * 4, &tmA, &full[s_], km * cBM + 32 * j, hw0, n);
            }
            tma_load_3d(sa + L::A_BYTES, &tmB, &full[s_], hw0, ctile * BN, n);
          }
        }
      }
    }
  } else if (warp == cMmaWarp) {
    // ------------------------------------------------------------ MMA issue
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_tf32(cBM, BN, A_MN, B_MN);
      uint32_t it = 0;
      int local = 0;
      for (int tile = blockIdx.x; tile < total_tiles && !*abort; tile += gridDim.x, ++local) {
        const int buf = local & 1;
        const uint32_t aph = (local >> 1) & 1;
        if (!mbar_wait(&acc_empty[buf], aph ^ 1, abort)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        int kb0 = 0, kb1 = RS * a.cblocks;
        if (WG) {
          int sp, km, ctile, rs;
          wg_tile(tile, sp, km, ctile, rs);
          wg_range(sp, kb0, kb1);
        } else if (MODE == kImplicit) {
          wg_range(tile % a.splits, kb0, kb1);
        }
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s_ = it % cStages;
          const uint32_t ph = (it / cStages) & 1;
          if (!mbar_wait(&full[s_], ph, abort)) break;
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s_ * L::STAGE_BYTES);
          const uint32_t sb = sa + L::A_BYTES;
#pragma unroll
          for (int h = 0; h < KB; ++h)
#pragma unroll
            for (int kk = 0; kk < cBK / 8; ++kk) {
              const uint32_t ah = sa + h * A_BLK, bh = sb + h * B_BLK;
              const uint64_t ad = A_MN ? desc_mnmajor(ah, kk, 32 * cBK * 4) : desc_kmajor(ah, kk);
              const uint64_t bd = B_MN ? desc_mnmajor(bh, kk, 32 * cBK * 4) : desc_kmajor(bh, kk);
              mma_tf32(d_tmem, ad, bd, idesc, (kb > kb0 || h > 0 || kk > 0) ? 1u : 0u);
            }
          mma_commit(&empty[s_]);
        }
        mma_commit(&acc_full[buf]);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int ew = warp - cMmaWarp - 1;   // epilogue warp 0..7
    const int quarter = warp & 3;         // TMEM lane quarter this warp may read
    const int half = ew >> 2;             // chunks c with c % 2 == half
    const int row = quarter * 32 + lane;  // TMEM lane = accumulator row
    float* st = (float*)(smem + L::EPI_OFF) + ew * 1024;
    int local = 0;
    for (int tile = blockIdx.x; tile < total_tiles && !*abort; tile += gridDim.x, ++local) {
      const int buf = local & 1;
      const uint32_t aph = (local >> 1) & 1;
      // pointwise dgrad with an addend: this warp's first chunk is loaded
      // before the accumulator is ready, each next one while a chunk is stored
      float pre[32];
      if (PW && a.addend) {
        const int slot = (tile / a.kt) * 4 + quarter;
        if (slot < a.slots) {
          const int n = slot / a.hwb;
          load_addend_chunk(a, n, (slot - n * a.hwb) * 32, (tile % a.kt) * BN + half * 32, lane, pre);
        }
        // and this warp's chunks of the next tile go to L2 now, a tile
        // ahead, so the per-chunk loads above find them there
        const int next = tile + gridDim.x;
        const int slot2 = (next / a.kt) * 4 + quarter;
        if (next < total_tiles && slot2 < a.slots) {
          const int n2 = slot2 / a.hwb;
          prefetch_addend_l2<BN>(a, n2, (slot2 - n2 * a.hwb) * 32, (next % a.kt) * BN, lane, half);
        }
      }
      if (!mbar_wait(&acc_full[buf], aph, abort)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + ((uint32_t)(quarter * 32) << 16) + buf * BN;
      if (!WG) {
        int kt;
        bool valid = false, bvalid;
        float* obase = nullptr;
        int bx, by = 0, bn;  // store-box origin of this warp's 32 rows
        if (PW) {
          kt = tile % a.kt;
          const int slot = (tile / a.kt) * 4 + quarter;
          bn = slot / a.hwb;
          bx = (slot - bn * a.hwb) * 32;
          bvalid = slot < a.slots;
        } else {
          int q0, p0, n0;
          fwd_tile(tile / a.splits, kt, q0, p0, n0);
          // split-K partial slab s holds images s * N .. s * N + N - 1
          const int nsh = (tile % a.splits) * a.N;
          const int q = q0 + row % a.bw, p = p0 + (row / a.bw) % a.bh, n = n0 + row / (a.bw * a.bh);
          valid = q < a.Q && p < a.P && n < a.N;
          obase = a.out + a.obase + (int64_t)(n + nsh) * a.on + (int64_t)p * a.op + (int64_t)q * a.oq;
          const int r0 = quarter * 32;
          const int wq = q0 + r0 % a.bw, wp = p0 + (r0 / a.bw) % a.bh;
          bn = n0 + r0 / (a.bw * a.bh);
          bvalid = wq < a.Q && wp < a.P && bn < a.N;
          bn += nsh;
          if (a.epi == kEpiBox) {
            bx = wq;
            by = wp;
          } else {
            bx = wp * a.Q;
          }
        }
#pragma unroll 1
        for (int c = half; c < BN / 32; c += 2) {
          float v[32];
          tmem_ld32(tbase + c * 32, v);
          const int k0 = kt * BN + c * 32;
          if (a.epi == kEpiScalar) {
            if (valid) {
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                const int k = k0 + j;
                if (k < a.Kout) obase[(int64_t)k * a.ok] = a.bias ? v[j] + a.bias[k] : v[j];
              }
            }
          } else if (bvalid && k0 < a.Kout) {  // warp-uniform: this chunk has output to store
            if (a.bias) {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (k0 + j < a.Kout) v[j] += a.bias[k0 + j];
            }
            if (PW && a.addend) {
              // a gradient accumulated into this one (prefetched in `pre`)
              const bool px_ok = bx + lane < a.Q;
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] += (px_ok && k0 + j < a.Kout) ? pre[j] : 0.0f;
              if (c + 2 < BN / 32 && k0 + 64 < a.Kout) load_addend_chunk(a, bn, bx, k0 + 64, lane, pre);
            }
            // the box's previous store must have read it before it is rewritten
            if (lane == 0) bulk_wait_read<0>();
            __syncwarp();
            if (a.epi == kEpiFlat) {
              const int qq = lane % a.bw, pp = lane / a.bw, pitch = a.ebp * a.Q;
              if (qq < a.Q) {
#pragma unroll
                for (int j = 0; j < 32; ++j) st[j * pitch + pp * a.Q + qq] = v[j];
              }
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j) st[j * 32 + lane] = v[j];
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              if (a.epi == kEpiBox) tma_store_4d(&tmC, st, bx, by, k0, bn);
              else tma_store_3d(&tmC, st, bx, k0, bn);
              bulk_commit();
            }
          }
        }
      } else if (MODE == kWgradT) {
        // partials [splits * taps][input channel][output channel]: TMEM row
        // (tap 2 pair + quarter / 2, channel 32 (quarter % 2) + lane) holds
        // the output channels along its columns, stored as a row-major
        // 128-byte-swizzled box (lane writes its eight 16-byte pieces at
        // piece ^ (lane % 8), conflict-free per quarter warp)
        int sp, km, ctile, pr;
        wg_tile(tile, sp, km, ctile, pr);
        const int tap = 2 * pr + (quarter >> 1), c0 = (quarter & 1) * 32;
        const bool rows_ok = tap < RS && c0 < a.Cin;
#pragma unroll 1
        for (int c = half; c < BN / 32; c += 2) {
          float v[32];
          tmem_ld32(tbase + c * 32, v);
          const int k0 = ctile * BN + c * 32;
          if (rows_ok && k0 < a.Kout) {  // warp-uniform
            if (lane == 0) bulk_wait_read<0>();
            __syncwarp();
            float4* rowp = reinterpret_cast<float4*>(st + lane * 32);
#pragma unroll
            for (int ch = 0; ch < 8; ++ch)
              rowp[ch ^ (lane & 7)] = make_float4(v[4 * ch], v[4 * ch + 1], v[4 * ch + 2], v[4 * ch + 3]);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_3d(&tmC, st, k0, c0, sp * RS + tap);
              bulk_commit();
            }
          }
        }
      } else {
        // weight-gradient partials [splits * taps][cols][rows] (rows contiguous):
        // one TMA store per 32 x 32 chunk, clipped at the row / column ends
        int sp, km, ctile, rs;
        wg_tile(tile, sp, km, ctile, rs);
        const int m0 = km * cBM + quarter * 32;
        const int z = sp * RS + rs;
#pragma unroll 1
        for (int c = half; c < BN / 32; c += 2) {
          float v[32];
          tmem_ld32(tbase + c * 32, v);
          const int n0 = ctile * BN + c * 32;
          if (m0 < a.Kout && n0 < a.Cin) {  // warp-uniform
            if (lane == 0) bulk_wait_read<0>();
            __syncwarp();
#pragma unroll
            for (int j = 0; j < 32; ++j) st[j * 32 + lane] = v[j];
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_3d(&tmC, st, m0, n0, z);
              bulk_commit();
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
    if (lane == 0) bulk_wait_all();
  }
  // ---------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  if (warp == cMmaWarp) {
    if (*abort) {
      const uint64_t t0 = globaltimer();
      while (globaltimer() - t0 < 10000000ull) {
      }
    }
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * BN);
  }
}

// ------------------------------------------------------ layout kernels
// x [N, C, HW] -> y [N, HW, Cp], channels C..Cp-1 zero
// Same transpose for any HW (7x7 planes) over the flattened pixel index
// g = n * HW + p: 64-pixel x 32-channel tiles run over the images back to
// back, so a 49-pixel plane leaves no part-empty tile.  A warp loads 32
// consecutive pixels of one channel (one run, split at most once at an image
// boundary) and stores 32 consecutive channels of one pixel.
__global__ void __launch_bounds__(256) nchw_to_nhwc_flat_kernel(const float* __restrict__ x, float* __restrict__ y,
                                                                int C, int Cp, int64_t HW, int64_t pixels) {
  __shared__ float tile[32][64 + 1];  // odd pitch: the column reads below hit 32 banks
  const int64_t g0 = (int64_t)blockIdx.x * 64;
  const int c0 = blockIdx.y * 32;
  const int pl = threadIdx.x & 63;
  const int64_t g = g0 + pl;
  const bool gv = g < pixels;
  int64_t base = 0;
  if (gv) {
    const int64_t n = g / HW;
    base = n * C * HW + (g - n * HW);
  }
#pragma unroll
  for (int k = threadIdx.x >> 6; k < 32; k += 4) {
    const int c = c0 + k;
    tile[k][pl] = (gv && c < C) ? __ldg(x + base + (int64_t)c * HW) : 0.f;
  }
  __syncthreads();
  const int cl = threadIdx.x & 31;
#pragma unroll
  for (int k = threadIdx.x >> 5; k < 64; k += 8) {
    const int64_t gp = g0 + k;
    if (gp < pixels && c0 + cl < Cp) y[gp * Cp + c0 + cl] = tile[cl][k];
  }
}

// Same transpose with 128-bit accesses when HW % 4 == 0 (Cp is a multiple
// of 4): a 64-pixel x 32-channel tile per 256-thread block; loads are float4
// runs of 4 pixels of one channel, stores float4 runs of 4 channels of one
// pixel.
__global__ void __launch_bounds__(256) nchw_to_nhwc_v4_kernel(const float* __restrict__ x, float* __restrict__ y,
                                                              int C, int Cp, int HW) {
  __shared__ float tile[32][64 + 1];  // odd pitch: the column reads below hit 32 banks
  const int64_t n = blockIdx.z;
  const int p0 = blockIdx.x * 64, c0 = blockIdx.y * 32;
  const float* xn = x + n * C * (int64_t)HW;
  float* yn = y + n * (int64_t)HW * Cp;
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int i = threadIdx.x + u * 256;  // 32 channels x 16 float4
    const int c = i >> 4, q4 = (i & 15) * 4;
    const int p = p0 + q4;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (c0 + c < C && p < HW) v = __ldg(reinterpret_cast<const float4*>(xn + (int64_t)(c0 + c) * HW + p));
    tile[c][q4 + 0] = v.x;
    tile[c][q4 + 1] = v.y;
    tile[c][q4 + 2] = v.z;
    tile[c][q4 + 3] = v.w;
  }
  __syncthreads();
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int i = threadIdx.x + u * 256;  // 64 pixels x 8 float4
    const int q = i >> 3, c4 = (i & 7) * 4;
    const int p = p0 + q;
    if (p < HW && c0 + c4 < Cp)
      *reinterpret_cast<float4*>(yn + (int64_t)p * Cp + c0 + c4) =
          make_float4(tile[c4][q], tile[c4 + 1][q], tile[c4 + 2][q], tile[c4 + 3][q]);
  }
}

// forward: W [K][C][R][S] -> Wp [K][R][S][Cp].  One warp per 32 channels
// of one k: lane c reads its R*S taps (its first load brings the warp's
// 32 x R*S contiguous values into L1, the others hit there) and each tap is
// one 128-byte run of Wp.  128-thread blocks, K * ceil(Cp / 32) warps.
__global__ void __launch_bounds__(128) pack_w_fwd_kernel(const float* __restrict__ w, float* __restrict__ wp, int K,
                                                         int C, int Cp, int RS) {
  const int nb = (Cp + 31) / 32;
  const int warp = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
  if (warp >= K * nb) return;
  const int k = warp / nb, c = (warp - k * nb) * 32 + lane;
  if (c >= Cp) return;
  const float* src = w + ((int64_t)k * C + c) * RS;
  float* dst = wp + (int64_t)k * RS * Cp + c;
  const bool in = c < C;
#pragma unroll 4
  for (int rs = 0; rs < RS; ++rs) dst[(int64_t)rs * Cp] = in ? __ldg(src + rs) : 0.f;
}

// dgrad phase: Wd[c][t][k] = W[k][c][r_t][s_t] over the phase's tap list
__global__ void pack_w_phase_kernel(const float* __restrict__ w, float* __restrict__ wd, int K, int Kp, int C, int R,
                                    int S, int nr, int ns, int4 rl, int4 rh, int4 sl, int4 shi) {
  __shared__ int tap_off[kMaxTaps * kMaxTaps];  // (r_t, s_t) -> r*S + s
  if (threadIdx.x < nr * ns) {
    const int a = threadIdx.x / ns, b = threadIdx.x % ns;
    const int rv[8] = {rl.x, rl.y, rl.z, rl.w, rh.x, rh.y, rh.z, rh.w};
    const int sv[8] = {sl.x, sl.y, sl.z, sl.w, shi.x, shi.y, shi.z, shi.w};
    tap_off[threadIdx.x] = rv[a] * S + sv[b];
  }
  __syncthreads();
  const int taps = nr * ns, RS = R * S;
  const int total = C * taps * Kp;  // weights: far below 2^31 elements (checked by the launcher)
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int k = i % Kp;
    const int u = i / Kp;
    const int t = u % taps, c = u / taps;
    wd[i] = k < K ? __ldg(w + (k * C + c) * RS + tap_off[t]) : 0.f;
  }
}

// small-C convolutions as a GEMM over im2col columns:
// Xcol[n, p, q, j] = X[n, c, p*sh - ph + r*dh, q*sw - pw + s*dw] with j = (c*R + r)*S + s
// (W's own flattening; 0 outside the image and for j >= C*R*S up to Kc).
// grid (P, N): one output row per CTA; each thread gathers four columns and
// writes them as one 16-byte store, consecutive threads consecutive stores.
constexpr int kIm2colMaxK = 1024;
__global__ void __launch_bounds__(256) im2col_kernel(const float* __restrict__ x, float* __restrict__ xcol, int C,
                                                     int H, int W, int P, int Q, int R, int S, int Kc, int sh, int sw,
                                                     int ph, int pw, int dh, int dw) {
  // per column j of this output row: the input row's offset (-1: zero column) and the tap's w shift
  __shared__ int joff[kIm2colMaxK], js[kIm2colMaxK];
  const int p = blockIdx.x;
  const int64_t n = blockIdx.y;
  const int crs = C * R * S;
  for (int j = threadIdx.x; j < Kc; j += blockDim.x) {
    const int c = j / (R * S), rs = j - c * R * S;
    const int h = p * sh + (rs / S) * dh - ph;
    joff[j] = (j < crs && h >= 0 && h < H) ? (c * H + h) * W : -1;
    js[j] = (rs % S) * dw - pw;
  }
  __syncthreads();
  const float* xn = x + n * C * H * W;
  // the row's Q x Kc columns as consecutive 16-byte stores; the gathered
  // loads of neighbouring threads hit the same few input rows (L1)
  const int kc4 = Kc / 4, total = Q * kc4;
  float4* out = reinterpret_cast<float4*>(xcol + ((n * P + p) * Q) * (int64_t)Kc);
  for (int t = threadIdx.x; t < total; t += blockDim.x) {
    const int q = t / kc4, j = (t - q * kc4) * 4;
    const int wq = q * sw;
    float v[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int ro = joff[j + e], w = wq + js[j + e];
      v[e] = (ro >= 0 && (unsigned)w < (unsigned)W) ? __ldg(xn + ro + w) : 0.f;
    }
    out[t] = make_float4(v[0], v[1], v[2], v[3]);
  }
}

// ------------------------------------------- windowed few-channel filters
// A convolution with few input channels (C <= 4) and a short filter row
// (S <= 8, the 3-channel 7x7 stem) reads its input as a zero-padded
// channels-last copy xw[n][hp][wp][4] (hp = h + pad_h, wp = w + pad_w, four
// channel slots, unused ones zero).  For output (p, q) and filter row r the
// S taps x 4 channels of the row are the 32 consecutive floats starting at
// xw[n][p*sh + r][q*sw][0] (8 pixels; the taps past S have zero weights), so
// a TMA map whose q dimension steps sw pixels (overlapping windows) gives
// each output pixel its row-r window as one 128-byte K block: the forward is
// an implicit GEMM over R K blocks with no im2col columns, and the weight
// gradient a GEMM of the windows (MN-major) against dY.
// Padded extents: rows (P - 1) * sh + 8 and columns (Q - 1) * sw + 8, so
// every window of filter rows 0..7 lies inside the copy.
__global__ void __launch_bounds__(256) pad_window_kernel(const float* __restrict__ x, float4* __restrict__ xw, int C,
                                                         int H, int W, int Hp, int Wp, int ph, int pw,
                                                         int64_t total) {
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int wp = (int)(e % Wp);
    const int64_t r = e / Wp;
    const int hp = (int)(r % Hp);
    const int64_t n = r / Hp;
    const int h = hp - ph, w = wp - pw;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if ((unsigned)h < (unsigned)H && (unsigned)w < (unsigned)W) {
      const float* xp = x + ((n * C) * H + h) * (int64_t)W + w;
#pragma unroll
      for (int c = 0; c < 4; ++c)
        if (c < C) v[c] = __ldg(xp + (int64_t)c * H * W);
    }
    xw[e] = make_float4(v[0], v[1], v[2], v[3]);
  }
}

// wp[k][r][s * 4 + c] = w[k][c][r][s] (zero for s >= S or c >= C)
__global__ void pack_w_window_kernel(const float* __restrict__ w, float* __restrict__ wp, int K, int C, int R, int S) {
  const int total = K * R * 32;
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < total; e += gridDim.x * blockDim.x) {
    const int j = e % 32, r = (e / 32) % R, k = e / (32 * R);
    const int s = j / 4, c = j % 4;
    wp[e] = (s < S && c < C) ? w[((k * C + c) * R + r) * S + s] : 0.f;
  }
}

// dw[k][c][r][s] = t[k][r * 32 + s * 4 + c]: the windowed weight gradient
// (rows = filter row x window element) back in the weight's layout
__global__ void unwindow_wgrad_kernel(const float* __restrict__ t, int ld, float* __restrict__ dw, int K, int C, int R,
                                      int S) {
  const int total = K * C * R * S;
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < total; e += gridDim.x * blockDim.x) {
    const int s = e % S, r = (e / S) % R, c = (e / (S * R)) % C, k = e / (S * R * C);
    dw[e] = t[(int64_t)k * ld + r * 32 + s * 4 + c];
  }
}

// Strided 1x1 convolutions (ResNet's downsampling projections) as
// pointwise ones over the sampled pixels.
// xs[plane][p][q] = x[plane][p*sh][q*sw]; one thread per sampled element,
// 32-bit index arithmetic (the host keeps the element count below 2^31),
// divisions by Q and P as multiply-highs
__global__ void subsample_kernel(const float* __restrict__ x, float* __restrict__ xs, int total, int H, int W,
                                 FastDiv Q, FastDiv P, int sh, int sw) {
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < total; e += gridDim.x * blockDim.x) {
    const int r = fdiv(e, Q), q = e - r * Q.d;
    const int pl = fdiv(r, P), p = r - pl * P.d;
    xs[e] = __ldg(x + ((int64_t)pl * H + p * sh) * W + q * sw);
  }
}

// dx[plane][h][w] = t[plane][h/sh][w/sw] on the sampled pixels, 0 elsewhere,
// written whole (no separate clearing pass) as 16-byte stores; W % 4 == 0
// and fewer than 2^31 float4 of dx (checked on the host).  ST is the stride
// in both dimensions when it is known at compile time (2), else 0 and the
// runtime sh, sw apply; the row and plane come from multiply-highs.
template <int ST>
__global__ void scatter_strided_kernel(const float* __restrict__ t, float* __restrict__ dx, int total4, FastDiv w4,
                                       FastDiv H, int P, int Q, int sh_rt, int sw_rt) {
  const int sh = ST ? ST : sh_rt, sw = ST ? ST : sw_rt;
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < total4; e += gridDim.x * blockDim.x) {
    const int r = fdiv(e, w4), w0 = (e - r * w4.d) * 4;
    const int pl = fdiv(r, H), h = r - pl * H.d;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (h % sh == 0 && h / sh < P) {
      const float* row = t + ((int64_t)pl * P + h / sh) * Q;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int w = w0 + u;
        if (w % sw == 0 && w / sw < Q) v[u] = __ldg(row + w / sw);
      }
    }
    reinterpret_cast<float4*>(dx)[e] = make_float4(v[0], v[1], v[2], v[3]);
  }
}

// W [K][crs] -> Wp [K][Kc], zero columns crs..Kc-1
__global__ void pack_w_rows_kernel(const float* __restrict__ w, float* __restrict__ wp, int K, int crs, int Kc) {
  const int64_t total = (int64_t)K * Kc;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int j = (int)(i % Kc);
    const int64_t k = i / Kc;
    wp[i] = j < crs ? w[k * crs + j] : 0.f;
  }
}

// ------------------------------------------------------------ host side
static int round4(int c) { return (c + 3) / 4 * 4; }
static int pow2_at_least(int v, int lo, int hi) {
  int p = lo;
  while (p < v && p < hi) p <<= 1;
  return p;
}
static size_t align256(size_t b) { return (b + 255) / 256 * 256; }
static int bn_for(int n) { return n <= 64 ? 64 : (n <= 128 ? 128 : 256); }
static bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

// pixel block of `pixels` (128 or 32) covering a P x Q grid
static void pixel_block(int P, int Q, int pixels, int& bw, int& bh, int& bni) {
  bw = pow2_at_least(Q, 8, pixels >= 64 ? 64 : pixels);
  if (bw > pixels) bw = pixels;
  bh = pow2_at_least(P, 1, pixels / bw);
  if (bh > pixels / bw) bh = pixels / bw;
  bni = pixels / (bw * bh);
}

static bool tc_conv_enabled() { return getenv("PVB2_DISABLE_TC") == nullptr; }

// implicit launches step their TMA boxes by the stride (bw * stride <= 256)
// and keep the filter taps of a row / column in fixed arrays
static bool stride_ok_for_boxes(const pvb2_conv2d_desc* d) {
  return d->stride_w <= 4 && d->stride_h <= 4 && d->R <= kMaxTaps && d->S <= kMaxTaps;
}

static bool tc_conv_shape_ok(const pvb2_conv2d_desc* d) {
  if (d->groups != 1 || d->math != PVB2_MATH_TF32 || !tc_conv_enabled()) return false;
  const double macs = (double)d->N * d->P * d->Q * d->K * d->C * d->R * d->S;
  if (macs < (double)(1 << 19)) return false;
  if (d->K < 8) return false;
  return true;
}

// 1x1, stride 1, no padding, and every NCHW row pitch a multiple of 16 bytes:
// the NCHW tensors themselves are the GEMM operands
static bool pointwise(const pvb2_conv2d_desc* d) {
  return d->R == 1 && d->S == 1 && d->stride_h == 1 && d->stride_w == 1 && d->pad_h == 0 && d->pad_w == 0 &&
         ((int64_t)d->H * d->W) % 4 == 0 && d->C % 4 == 0 && d->K % 4 == 0;
}

// 1x1, strided, no padding, with 16-byte sampled rows: a pointwise
// convolution over the sampled pixels xs (a dense [N][C][P][Q] copy)
static bool strided_pointwise(const pvb2_conv2d_desc* d) {
  return d->R == 1 && d->S == 1 && (d->stride_h > 1 || d->stride_w > 1) && d->pad_h == 0 && d->pad_w == 0 &&
         ((int64_t)d->P * d->Q) % 4 == 0 && d->C % 4 == 0 && d->K % 4 == 0 && d->W % 4 == 0 &&
         d->P == (d->H - 1) / d->stride_h + 1 && d->Q == (d->W - 1) / d->stride_w + 1 &&
         (int64_t)d->N * d->C * d->H * d->W < ((int64_t)1 << 31);
}
static size_t sampled_bytes(const pvb2_conv2d_desc* d) { return (size_t)d->N * d->C * d->P * d->Q * 4; }
static int subsample(const pvb2_conv2d_desc* d, const float* x, float* xs, cudaStream_t s) {
  const int64_t total = (int64_t)d->N * d->C * d->P * d->Q;
  subsample_kernel<<<grid_for(total, 256), 256, 0, s>>>(x, xs, (int)total, d->H, d->W, fast_div(d->Q),
                                                         fast_div(d->P), d->stride_h, d->stride_w);
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

// Few input channels and a spatial filter (the 3-channel stem): one GEMM
// over im2col columns instead of R*S taps of a few channels each.  The
// weight-gradient map needs 16-byte output-plane rows (P*Q % 4 == 0).
static int im2col_channels(const pvb2_conv2d_desc* d) { return round4(d->C * d->R * d->S); }
static bool use_im2col(const pvb2_conv2d_desc* d) {
  return d->C <= 8 && d->R * d->S > 1 && im2col_channels(d) <= kIm2colMaxK && ((int64_t)d->P * d->Q) % 4 == 0 &&
         d->N <= 65535 && d->P <= 65535;
}

// Few input channels and filter rows of at most 8 taps over a large image
// (ResNet's 3-channel 7x7 stem, MobileNet-v2's 3x3): filter-row windows of a padded channels-last
// copy instead of im2col columns (pad_window_kernel).  The weight gradient
// reads each 32-pixel K block as two 16-pixel runs of one output row.
static bool use_window(const pvb2_conv2d_desc* d) {
  return d->C <= 4 && d->S <= 8 && d->R <= kMaxTaps && d->R * d->S >= 9 && d->dil_h == 1 && d->dil_w == 1 &&
         d->stride_h <= 8 && d->stride_w <= 8 && d->Q % 16 == 0 && ((int64_t)d->P * d->Q) % 4 == 0 &&
         d->N <= 65535;
}
static int win_hp(const pvb2_conv2d_desc* d) { return (d->P - 1) * d->stride_h + 8; }
static int win_wp(const pvb2_conv2d_desc* d) { return (d->Q - 1) * d->stride_w + 8; }
static size_t win_bytes(const pvb2_conv2d_desc* d) { return (size_t)d->N * win_hp(d) * win_wp(d) * 16; }

static int pad_window(const pvb2_conv2d_desc* d, const float* x, float* xw, cudaStream_t s) {
  const int64_t total = (int64_t)d->N * win_hp(d) * win_wp(d);
  pad_window_kernel<<<grid_for(total, 256), 256, 0, s>>>(x, (float4*)xw, d->C, d->H, d->W, win_hp(d), win_wp(d),
                                                          d->pad_h, d->pad_w, total);
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

// the windows as a 4-D map (32 floats, Q output columns stepping sw pixels,
// padded rows, images); box (32, bq, brows, bn), row element stride es_h
static int window_map(CUtensorMap* m, const float* xw, const pvb2_conv2d_desc* d, uint32_t bq, uint32_t brows,
                      uint32_t bn, uint32_t es_h, bool mn_major) {
  const uint64_t wp = win_wp(d), hp = win_hp(d);
  uint64_t dims[4] = {32, (uint64_t)d->Q, hp, (uint64_t)d->N};
  uint64_t str[3] = {(uint64_t)d->stride_w * 16, wp * 16, hp * wp * 16};
  uint32_t box[4] = {32, bq, brows, bn};
  uint32_t es[4] = {1, 1, es_h, 1};
  return encode_tiled(m, 4, xw, dims, str, box, mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, es);
}

struct Taps {
  int nr, ns;
  int h[kMaxTaps], w[kMaxTaps];
};

template <int BN, int MODE, int KB = 1>
static int launch_conv(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, const ConvTcArgs& a,
                       cudaStream_t s) {
  constexpr int smem = ConvSmem<BN, KB>::TOTAL + 1024;
  static std::atomic<uint64_t> attr_done{0};
  if (first_on_device(attr_done))
    PVB2_CUDA_TRY(
        cudaFuncSetAttribute(conv_tf32_kernel<BN, MODE, KB>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  if (a.tiles <= 0) return PVB2_OK;
  const int grid = std::min(a.tiles, num_sms());
  conv_tf32_kernel<BN, MODE, KB><<<grid, cThreads, smem, s>>>(ma, mb, mc, a);
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

template <int MODE>
static int launch_bn(int BN, const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, const ConvTcArgs& a,
                     cudaStream_t s) {
  if (BN == 64) return launch_conv<64, MODE>(ma, mb, mc, a, s);
  if (BN == 128) return launch_conv<128, MODE>(ma, mb, mc, a, s);
  return launch_conv<256, MODE>(ma, mb, mc, a, s);
}

// the same with two K blocks per stage (BN <= 128 only)
template <int MODE>
static int launch_bn2(int BN, const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc,
                      const ConvTcArgs& a, cudaStream_t s) {
  PVB2_CHECK_ARG(BN <= 128, "conv: two K blocks per stage need BN <= 128");
  if (BN == 64) return launch_conv<64, MODE, 2>(ma, mb, mc, a, s);
  return launch_conv<128, MODE, 2>(ma, mb, mc, a, s);
}

// channels-last activations [N, H, W, Cp] as a 4-D map (Cp, W, H, N)
static int act_map(CUtensorMap* m, const float* base, int N, int H, int W, int Cp, int bw, int bh, int bni, int sw,
                   int sh, bool mn_major) {
  uint64_t dims[4] = {(uint64_t)Cp, (uint64_t)W, (uint64_t)H, (uint64_t)N};
  uint64_t str[3] = {(uint64_t)Cp * 4, (uint64_t)W * Cp * 4, (uint64_t)H * W * Cp * 4};
  uint32_t box[4] = {32, (uint32_t)(bw * sw), (uint32_t)(bh * sh), (uint32_t)bni};
  uint32_t es[4] = {1, (uint32_t)sw, (uint32_t)sh, 1};
  return encode_tiled(m, 4, base, dims, str, box, mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, es);
}

// an NCHW tensor [N, C, HW] as a 3-D map (HW, C, N) with box (32, rows, 1)
static int nchw_map(CUtensorMap* m, const float* base, int N, int C, int64_t hw, int rows, CUtensorMapSwizzle sw) {
  uint64_t dims[3] = {(uint64_t)hw, (uint64_t)C, (uint64_t)N};
  uint64_t str[2] = {(uint64_t)hw * 4, (uint64_t)C * hw * 4};
  uint32_t box[3] = {32, (uint32_t)rows, 1};
  return encode_tiled(m, 3, base, dims, str, box, sw);
}

static int to_nhwc(const float* x, float* y, int N, int C, int Cp, int64_t HW, cudaStream_t s) {
  if (HW % 4 == 0 && HW < ((int64_t)1 << 31) && aligned16(x) && aligned16(y)) {
    dim3 grid((unsigned)((HW + 63) / 64), (unsigned)((Cp + 31) / 32), (unsigned)N);
    nchw_to_nhwc_v4_kernel<<<grid, 256, 0, s>>>(x, y, C, Cp, (int)HW);
  } else {
    const int64_t pixels = (int64_t)N * HW;
    dim3 grid((unsigned)((pixels + 63) / 64), (unsigned)((Cp + 31) / 32));
    nchw_to_nhwc_flat_kernel<<<grid, 256, 0, s>>>(x, y, C, Cp, HW, pixels);
  }
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

// Choose the epilogue of a forward-shaped launch over a bw x bh x bni pixel
// block and build its store map.  TMA needs a 16-byte-aligned base, unit
// stride along q and 16-byte multiples for every other stride.
static int plan_epilogue(ConvTcArgs& a, CUtensorMap* mc, float* out, int N, int K, int P, int Q) {
  a.epi = kEpiScalar;
  float* base = out + a.obase;
  const bool ok = aligned16(base) && a.oq == 1 && (a.ok * 4) % 16 == 0 && (a.on * 4) % 16 == 0 &&
                  a.bw * a.bh >= 32;
  if (!ok) return PVB2_OK;
  if ((a.op * 4) % 16 == 0) {
    a.epi = kEpiBox;
    a.ebq = std::min(a.bw, 32);
    a.ebp = 32 / a.ebq;
    uint64_t dims[4] = {(uint64_t)Q, (uint64_t)P, (uint64_t)K, (uint64_t)N};
    uint64_t str[3] = {(uint64_t)a.op * 4, (uint64_t)a.ok * 4, (uint64_t)a.on * 4};
    uint32_t box[4] = {(uint32_t)a.ebq, (uint32_t)a.ebp, 32, 1};
    return encode_tiled(mc, 4, base, dims, str, box, CU_TENSOR_MAP_SWIZZLE_NONE);
  }
  // rows not 16-byte aligned (e.g. 14 x 14 planes): store whole rows of a contiguous plane
  const int ebp = 32 / std::max(a.bw, 1);
  if (a.op == Q && a.bw >= Q && a.bw <= 32 && (ebp * Q) % 4 == 0 && (a.bh * Q) % 4 == 0) {
    a.epi = kEpiFlat;
    a.ebq = Q;
    a.ebp = ebp;
    uint64_t dims[3] = {(uint64_t)P * Q, (uint64_t)K, (uint64_t)N};
    uint64_t str[2] = {(uint64_t)a.ok * 4, (uint64_t)a.on * 4};
    uint32_t box[3] = {(uint32_t)(ebp * Q), 32, 1};
    return encode_tiled(mc, 3, base, dims, str, box, CU_TENSOR_MAP_SWIZZLE_NONE);
  }
  return PVB2_OK;
}

// Split-K for forward-shaped launches whose output has too few 128 x BN
// tiles to occupy the SMs (ResNet's 7 x 7 and 14 x 14 stages): the taps x
// channel blocks are divided into S ranges, each range's partial output is
// TMA-stored raw into slab s of a dense [S][N][K][P][Q] buffer, and
// conv_splitk_reduce_kernel adds the slabs in order s = 0..S-1 plus the bias.
// S minimises rounds(S) x (K blocks per split) x (time of one K block)
// + (time to write and read the slabs), with 60% of the per-SM TF32 rate
// and 6 TB/s assumed.
struct FwdSplit {
  int splits = 1, kb_per = 0;
  size_t bytes = 0;
};

// the ring stage of a forward-shaped implicit launch: two channel blocks
// (KB = 2) when BN <= 128 and there are at least two
static bool implicit_pairs(int K, int Cp) { return bn_for(K) <= 128 && (Cp + 31) / 32 >= 2; }

static FwdSplit plan_fwd_split(int N, int P, int Q, int K, int taps, int Cp) {
  FwdSplit f;
  int bw, bh, bni;
  pixel_block(P, Q, cBM, bw, bh, bni);
  const int BN = bn_for(K);
  const int64_t tiles = (int64_t)((Q + bw - 1) / bw) * ((P + bh - 1) / bh) * ((N + bni - 1) / bni) * ((K + BN - 1) / BN);
  // K blocks here are ring stages (channel-block pairs when KB = 2)
  const int per_stage = implicit_pairs(K, Cp) ? 2 : 1;
  const int kblocks = taps * (((Cp + 31) / 32 + per_stage - 1) / per_stage);
  f.kb_per = kblocks;
  const int sms = num_sms();
  if (tiles >= sms || kblocks * per_stage < 8) return f;
  const double t_kb = per_stage * 2.0 * cBM * BN * cBK / (0.6 * 816e12 / sms);
  const double out_bytes = 4.0 * N * K * P * Q;
  double best = 1e30;
  for (int S = 1; S <= 8; ++S) {
    const int kb_per = (kblocks + S - 1) / S;
    if (S > 1 && kb_per < 4) break;
    const int Se = (kblocks + kb_per - 1) / kb_per;
    const int64_t rounds = (tiles * Se + sms - 1) / sms;
    const double cost = rounds * kb_per * t_kb + (Se > 1 ? 2.0 * Se * out_bytes / 6e12 : 0.0);
    if (cost < best * 0.97) {  // a split has to win clearly
      best = cost;
      f.splits = Se;
      f.kb_per = kb_per;
    }
  }
  f.bytes = f.splits > 1 ? (size_t)f.splits * N * K * P * Q * 4 : 0;
  return f;
}

// out[obase + n*on + k*ok + p*op + q*oq] = sum_s part[s][n][k][p][q] (+ bias[k])
__global__ void conv_splitk_reduce_kernel(const float* __restrict__ part, int S, int N, int K, int P, int Q,
                                          const float* __restrict__ bias, float* __restrict__ out, int64_t obase,
                                          int64_t on, int64_t ok, int64_t op, int64_t oq) {
  const int64_t slab = (int64_t)N * K * P * Q;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < slab; e += (int64_t)gridDim.x * blockDim.x) {
    const int q = (int)(e % Q);
    int64_t r = e / Q;
    const int p = (int)(r % P);
    r /= P;
    const int k = (int)(r % K);
    const int n = (int)(r / K);
    float acc = __ldg(part + e);
    for (int sp = 1; sp < S; ++sp) acc += __ldg(part + sp * slab + e);
    if (bias) acc += bias[k];
    out[obase + n * on + k * ok + p * op + q * oq] = acc;
  }
}

// the same for a dense NCHW output: 16-byte loads and stores over the flat index
__global__ void conv_splitk_reduce_dense_kernel(const float* __restrict__ part, int S, int n4, int K, int PQ,
                                                const float* __restrict__ bias, float* __restrict__ out) {
  const int64_t slab4 = n4;
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < n4; e += gridDim.x * blockDim.x) {
    float4 acc = __ldg(reinterpret_cast<const float4*>(part) + e);
    for (int sp = 1; sp < S; ++sp) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(part) + sp * slab4 + e);
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    if (bias) {
      const int i = e * 4;
      acc.x += bias[(i / PQ) % K];
      acc.y += bias[((i + 1) / PQ) % K];
      acc.z += bias[((i + 2) / PQ) % K];
      acc.w += bias[((i + 3) / PQ) % K];
    }
    reinterpret_cast<float4*>(out)[e] = acc;
  }
}

// Forward-shaped implicit GEMM.  act: channels-last [N, H, W, Cp]; wpacked:
// [K][taps][Cp]; output grid P x Q with strides (sh, sw) and tap offsets;
// out element (n, k, p, q) at out[obase + n*on + k*ok + p*op + q*oq].
// With a split plan (plan_fwd_split) and `part` holding its slabs, the
// launch is split-K and a reduction writes `out`.
// `win` (or null): act is that convolution's window copy (pad_window), read
// through window_map with the row stride sh (sw must be 1: the map's q
// dimension already steps the convolution's stride)
static int run_fwd_like(const float* act, const float* wpacked, const float* bias, float* out, int N, int Cp, int H,
                        int W, int K, const Taps& t, int P, int Q, int sh, int sw, int64_t obase, int64_t on,
                        int64_t ok, int64_t op, int64_t oq, float* part, size_t part_bytes, cudaStream_t s,
                        const pvb2_conv2d_desc* win = nullptr) {
  if (P <= 0 || Q <= 0 || N <= 0) return PVB2_OK;
  int bw, bh, bni;
  pixel_block(P, Q, cBM, bw, bh, bni);
  const int BN = bn_for(K);
  CUtensorMap ma, mb, mc;
  memset(&mc, 0, sizeof(mc));
  if (win) {
    PVB2_TRY(window_map(&ma, act, win, (uint32_t)bw, (uint32_t)(bh * sh), (uint32_t)bni, (uint32_t)sh, false));
  } else {
    PVB2_TRY(act_map(&ma, act, N, H, W, Cp, bw, bh, bni, sw, sh, false));
  }
  const int taps = t.nr * t.ns;
  uint64_t wd[2] = {(uint64_t)taps * Cp, (uint64_t)K};
  uint64_t wst[1] = {(uint64_t)taps * Cp * 4};
  uint32_t wbox[2] = {32, (uint32_t)BN};
  PVB2_TRY(encode_tiled(&mb, 2, wpacked, wd, wst, wbox, CU_TENSOR_MAP_SWIZZLE_128B));
  ConvTcArgs a;
  memset(&a, 0, sizeof(a));
  a.N = N; a.Cin = Cp; a.Cp = Cp; a.Kout = K; a.P = P; a.Q = Q; a.R = t.nr; a.S = t.ns;
  a.sh = sh; a.sw = sw;
  for (int i = 0; i < kMaxTaps; ++i) {
    a.tap_h[i] = t.h[i];
    a.tap_w[i] = t.w[i];
  }
  a.obase = obase; a.on = on; a.ok = ok; a.op = op; a.oq = oq;
  a.cblocks = (Cp + 31) / 32;
  a.cpairs = (a.cblocks + 1) / 2;
  a.bw = bw; a.bh = bh; a.bni = bni;
  a.tq = (Q + bw - 1) / bw;
  a.tp = (P + bh - 1) / bh;
  a.tn = (N + bni - 1) / bni;
  a.kt = (K + BN - 1) / BN;
  a.out = out;
  a.bias = bias;
  const bool pairs = implicit_pairs(K, Cp);
  const FwdSplit fs = plan_fwd_split(N, P, Q, K, t.nr * t.ns, Cp);
  const bool split = fs.splits > 1 && part && part_bytes >= fs.bytes;
  a.splits = split ? fs.splits : 1;
  a.total_kb = t.nr * t.ns * (pairs ? a.cpairs : a.cblocks);  // ring stages
  a.kb_per_split = split ? fs.kb_per : a.total_kb;
  a.tiles = a.tq * a.tp * a.tn * a.kt * a.splits;
  auto launch = [&]() {
    return pairs ? launch_bn2<kImplicit>(BN, ma, mb, mc, a, s) : launch_bn<kImplicit>(BN, ma, mb, mc, a, s);
  };
  if (!split) {
    PVB2_TRY(plan_epilogue(a, &mc, out, N, K, P, Q));
    return launch();
  }
  // partial slabs: dense NCHW images s * N + n, no bias
  a.out = part;
  a.bias = nullptr;
  a.obase = 0;
  a.on = (int64_t)K * P * Q;
  a.ok = (int64_t)P * Q;
  a.op = Q;
  a.oq = 1;
  PVB2_TRY(plan_epilogue(a, &mc, part, N * a.splits, K, P, Q));
  PVB2_TRY(launch());
  const int64_t slab = (int64_t)N * K * P * Q;
  const bool dense = obase == 0 && oq == 1 && op == Q && ok == (int64_t)P * Q && on == (int64_t)K * P * Q;
  if (dense && slab % 4 == 0 && aligned16(out) && slab < ((int64_t)1 << 31)) {
    conv_splitk_reduce_dense_kernel<<<grid_for(slab / 4, 256), 256, 0, s>>>(part, a.splits, (int)(slab / 4), K,
                                                                           P * Q, bias, out);
  } else {
    conv_splitk_reduce_kernel<<<grid_for(slab, 256), 256, 0, s>>>(part, a.splits, N, K, P, Q, bias, out, obase, on,
                                                                 ok, op, oq);
  }
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

// Pointwise forward (transpose = false): Y[n, k, hw] = sum_c W[k, c] X[n, c, hw] (+ bias[k]).
// Pointwise dgrad (transpose = true):    dX[n, c, hw] = sum_k W[k, c] dY[n, k, hw].
// src: [N, Cs, hw]; dst: [N, Cd, hw]; w: [K][C] with (Cs, Cd) = (C, K) or (K, C).
static int run_pointwise(const float* src, const float* w, const float* bias, float* dst, int N, int C, int K,
                         int64_t hw, bool transpose, cudaStream_t s, const float* addend = nullptr) {
  const int Cs = transpose ? K : C, Cd = transpose ? C : K;
  const int BN = bn_for(Cd);
  CUtensorMap ma, mb, mc;
  PVB2_TRY(nchw_map(&ma, src, N, Cs, hw, 32, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B));
  uint64_t wd[2] = {(uint64_t)C, (uint64_t)K};
  uint64_t wst[1] = {(uint64_t)C * 4};
  if (!transpose) {
    uint32_t wbox[2] = {32, (uint32_t)BN};
    PVB2_TRY(encode_tiled(&mb, 2, w, wd, wst, wbox, CU_TENSOR_MAP_SWIZZLE_128B));
  } else {
    uint32_t wbox[2] = {32, 32};
    PVB2_TRY(encode_tiled(&mb, 2, w, wd, wst, wbox, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B));
  }
  PVB2_TRY(nchw_map(&mc, dst, N, Cd, hw, 32, CU_TENSOR_MAP_SWIZZLE_NONE));
  ConvTcArgs a;
  memset(&a, 0, sizeof(a));
  a.N = N; a.Cin = Cs; a.Cp = Cs; a.Kout = Cd; a.P = 1; a.Q = (int)hw; a.R = 1; a.S = 1;
  a.sh = a.sw = 1;
  a.cblocks = (Cs + 31) / 32;
  a.kt = (Cd + BN - 1) / BN;
  a.hwb = (int)((hw + 31) / 32);
  a.slots = N * a.hwb;
  a.tiles = (a.slots + 3) / 4 * a.kt;
  a.epi = kEpiSlots;
  a.out = dst;
  a.bias = bias;
  a.addend = addend;
  if (transpose) return launch_bn<kPwDgrad>(BN, ma, mb, mc, a, s);
  return launch_bn<kPwFwd>(BN, ma, mb, mc, a, s);
}

// Weight-gradient split-K plan.  kb_total K blocks (32 pixels each) reduce
// into K x Cin x taps outputs; enough splits to give every SM two tiles,
// each split keeping at least 8 K blocks.
// total_kb, kb_per: ring stages of kbs 32-pixel blocks each (kbs = 2 when
// BN <= 128: one mbarrier wait per eight MMAs)
struct WgPlan {
  int bw, bh, bni, BN, splits, kb_per, total_kb, ct, kt;
  int kbs = 1;
};
static void set_stages(WgPlan& w, int blocks) {
  w.kbs = w.BN <= 128 && blocks >= 2 ? 2 : 1;
  w.total_kb = (blocks + w.kbs - 1) / w.kbs;
}

// out_elems: K x Cin x taps weights; in_bytes: the operand bytes the
// reduction streams.  Splits also cost their partials (written once, read
// once), so they stop where that traffic would pass the operands'.
// Launches aim at two tiles per SM, except pointwise ones of at most four
// 128 x BN tiles, which aim at one: measured on ResNet-50's and
// MobileNet-v2's 1x1 weight gradients at batch 64 / 128 (one wave: 56x56
// 64 -> 256 52 µs against 64 at two; 28x28 512 -> 256 49 against 67; the
// 14x14 layers, 8 to 16 tiles, 44 at two against 50 at one).
static void plan_splits(WgPlan& w, int taps, double out_elems, double in_bytes) {
  const int base_tiles = w.kt * w.ct * taps;
  const int waves = taps == 1 && base_tiles <= 4 ? 1 : 2;
  int splits = (waves * num_sms() + base_tiles - 1) / base_tiles;
  splits = std::min(splits, std::max(1, w.total_kb / 8));
  // no fixed cap: a weight gradient of one or two 128 x BN tiles (a 1x1
  // layer with <= 128 channels on each side) needs about two splits per SM
  // to occupy the GPU; the partials' traffic bounds it below
  splits = std::max(1, std::min(splits, 4 * num_sms()));
  while (splits > 1 && (double)splits * out_elems * 8.0 > in_bytes) --splits;
  w.kb_per = (w.total_kb + splits - 1) / splits;
  w.splits = (w.total_kb + w.kb_per - 1) / w.kb_per;
}

static WgPlan plan_wg(int N, int K, int Cin, int P, int Q, int taps) {
  WgPlan w;
  pixel_block(P, Q, cBK, w.bw, w.bh, w.bni);
  w.BN = bn_for(Cin);
  w.ct = (Cin + w.BN - 1) / w.BN;
  w.kt = (K + cBM - 1) / cBM;
  const int tq = (Q + w.bw - 1) / w.bw, tp = (P + w.bh - 1) / w.bh, tn = (N + w.bni - 1) / w.bni;
  set_stages(w, tq * tp * tn);
  plan_splits(w, taps, (double)K * Cin * taps, 4.0 * N * P * Q * ((double)K + Cin));
  return w;
}

// A pointwise weight gradient with fewer than 128 output channels would use
// half of each 128-row tile; with at least 128 input channels the roles swap
// (M = input channels, N = output channels: dW^T = X dY^T), filling it.
static bool pw_wg_swap(const pvb2_conv2d_desc* d) { return d->K < 128 && d->C >= 128; }

static WgPlan plan_pw_wg(int N, int K, int C, int64_t hw) {
  WgPlan w;
  w.bw = 32; w.bh = 1; w.bni = 1;
  w.BN = bn_for(C);
  w.ct = (C + w.BN - 1) / w.BN;
  w.kt = (K + cBM - 1) / cBM;
  set_stages(w, N * (int)((hw + 31) / 32));
  plan_splits(w, 1, (double)K * C, 4.0 * N * hw * ((double)K + C));
  return w;
}

// Weight-gradient partials: [splits * taps][cols][round4(rows)] fp32, rows
// (the GEMM M side) contiguous; the epilogue stores 32 x 32 boxes of it.
static size_t wg_partial_bytes(int rows, int cols, int z) { return (size_t)z * cols * round4(rows) * 4; }
static int wg_partial_map(CUtensorMap* mc, float* part, int rows, int cols, int z) {
  uint64_t dims[3] = {(uint64_t)rows, (uint64_t)cols, (uint64_t)z};
  uint64_t str[2] = {(uint64_t)round4(rows) * 4, (uint64_t)round4(rows) * cols * 4};
  uint32_t box[3] = {32, 32, 1};
  return encode_tiled(mc, 3, part, dims, str, box, CU_TENSOR_MAP_SWIZZLE_NONE);
}

// dW from the partials: out[m*osm + n*osn + t*ost] = sum_sp part[sp][t][n][m] for
// m < mv, n < nv (splits summed in order).  grid (ceil(mv/32), ceil(nv/32), taps),
// block (32, 8); a 32 x 32 shared tile turns row-contiguous reads into
// writes along whichever of m / n is contiguous in dW.
__global__ void wgrad_reduce_kernel(const float* __restrict__ part, int splits, int taps, int cols, int mp, int mv,
                                    int nv, float* __restrict__ out, int64_t osm, int64_t osn, int64_t ost) {
  __shared__ float tile[32][33];
  const int m0 = blockIdx.x * 32, n0 = blockIdx.y * 32, t = blockIdx.z;
  const int64_t zstride = (int64_t)taps * cols * mp;
  for (int ny = threadIdx.y; ny < 32; ny += blockDim.y) {
    const int n = n0 + ny, m = m0 + threadIdx.x;
    float acc = 0.f;
    if (n < nv && m < mv) {
      const float* src = part + ((int64_t)t * cols + n) * mp + m;
      int sp = 0;
      for (; sp + 4 <= splits; sp += 4) {
        const float v0 = __ldg(src + sp * zstride), v1 = __ldg(src + (sp + 1) * zstride);
        const float v2 = __ldg(src + (sp + 2) * zstride), v3 = __ldg(src + (sp + 3) * zstride);
        acc = (((acc + v0) + v1) + v2) + v3;
      }
      for (; sp < splits; ++sp) acc += __ldg(src + sp * zstride);
    }
    tile[ny][threadIdx.x] = acc;
  }
  __syncthreads();
  if (osm == 1) {
    for (int ny = threadIdx.y; ny < 32; ny += blockDim.y) {
      const int n = n0 + ny, m = m0 + threadIdx.x;
      if (n < nv && m < mv) out[m + n * osn + t * ost] = tile[ny][threadIdx.x];
    }
  } else {
    for (int my = threadIdx.y; my < 32; my += blockDim.y) {
      const int m = m0 + my, n = n0 + threadIdx.x;
      if (n < nv && m < mv) out[m * osm + n * osn + t * ost] = tile[threadIdx.x][my];
    }
  }
}

// Same sum for small weights with many splits (too few 32 x 32 tiles to
// occupy the GPU): one block per (32 m, one n, tap); its G thread rows take
// splits g, g + G, ... and the G row sums are added in order g = 0..G-1.
__global__ void wgrad_reduce_split_kernel(const float* __restrict__ part, int splits, int taps, int cols, int mp,
                                          int mv, float* __restrict__ out, int64_t osm, int64_t osn, int64_t ost) {
  extern __shared__ float rows_acc[];  // [G][32]
  const int m = blockIdx.x * 32 + threadIdx.x, n = blockIdx.y, t = blockIdx.z;
  const int G = blockDim.y;
  const int64_t zstride = (int64_t)taps * cols * mp;
  float acc = 0.f;
  if (m < mv) {
    const float* src = part + ((int64_t)t * cols + n) * mp + m;
#pragma unroll 4
    for (int sp = threadIdx.y; sp < splits; sp += G) acc += __ldg(src + sp * zstride);
  }
  rows_acc[threadIdx.y * 32 + threadIdx.x] = acc;
  __syncthreads();
  if (threadIdx.y == 0 && m < mv) {
    float sum = rows_acc[threadIdx.x];
    for (int g = 1; g < G; ++g) sum += rows_acc[g * 32 + threadIdx.x];
    out[m * osm + n * osn + t * ost] = sum;
  }
}

static int wgrad_reduce(const float* part, int splits, int taps, int rows, int cols, int mv, int nv, float* dw,
                        int64_t osm, int64_t osn, int64_t ost, cudaStream_t s) {
  const int64_t tiles = (int64_t)((mv + 31) / 32) * ((nv + 31) / 32) * taps;
  if (tiles >= 2 * num_sms() || splits < 8) {
    const dim3 grid((unsigned)((mv + 31) / 32), (unsigned)((nv + 31) / 32), (unsigned)taps);
    wgrad_reduce_kernel<<<grid, dim3(32, 8), 0, s>>>(part, splits, taps, cols, round4(rows), mv, nv, dw, osm, osn,
                                                     ost);
  } else {
    int G = 1;
    while (G < 32 && G * 8 <= splits) G <<= 1;  // at least 4 splits per thread row
    if (G < 32 && G * 4 <= splits && splits >= 128) G <<= 1;  // one batch of loads per row
    const dim3 grid((unsigned)((mv + 31) / 32), (unsigned)nv, (unsigned)taps);
    wgrad_reduce_split_kernel<<<grid, dim3(32, G), G * 32 * sizeof(float), s>>>(part, splits, taps, cols,
                                                                               round4(rows), mv, dw, osm, osn, ost);
  }
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

// dy: channels-last [N, P, Q, Kp]; x: channels-last [N, H, W, Cp] (Cin <= Cp real channels);
// partials [splits * taps][Cin][K]
static int run_wgrad(const float* dyn, int Kp, const float* xn, int Cp, int N, int H, int W, int P, int Q, int K,
                     int Cin, const Taps& t, int sh, int sw, const WgPlan& p, float* part, cudaStream_t s) {
  CUtensorMap ma, mb, mc;
  memset(&mc, 0, sizeof(mc));
  PVB2_TRY(act_map(&ma, dyn, N, P, Q, Kp, p.bw, p.bh, p.bni, 1, 1, true));
  PVB2_TRY(act_map(&mb, xn, N, H, W, Cp, p.bw, p.bh, p.bni, sw, sh, true));
  ConvTcArgs a;
  memset(&a, 0, sizeof(a));
  a.N = N; a.Cin = Cin; a.Cp = Cp; a.Kout = K; a.P = P; a.Q = Q; a.R = t.nr; a.S = t.ns;
  a.sh = sh; a.sw = sw;
  for (int i = 0; i < kMaxTaps; ++i) {
    a.tap_h[i] = t.h[i];
    a.tap_w[i] = t.w[i];
  }
  a.bw = p.bw; a.bh = p.bh; a.bni = p.bni;
  a.tq = (Q + p.bw - 1) / p.bw;
  a.tp = (P + p.bh - 1) / p.bh;
  a.tn = (N + p.bni - 1) / p.bni;
  a.kt = p.kt;
  a.ct = p.ct;
  a.splits = p.splits;
  a.kb_per_split = p.kb_per;
  a.total_kb = p.total_kb;
  a.out = part;
  a.tiles = a.kt * a.ct * t.nr * t.ns * a.splits;
  PVB2_TRY(wg_partial_map(&mc, part, K, Cin, p.splits * t.nr * t.ns));
  return p.kbs == 2 ? launch_bn2<kWgrad>(p.BN, ma, mb, mc, a, s) : launch_bn<kWgrad>(p.BN, ma, mb, mc, a, s);
}

// Weight gradients with at most 64 input and output channels (ResNet's
// layer1 3x3): two taps x 64 input channels fill the 128 accumulator rows
// (kWgradT) instead of 64 output channels leaving half of them empty.
static bool use_wgrad_t(const pvb2_conv2d_desc* d) { return d->K <= 64 && d->C <= 64 && d->R * d->S >= 2; }

static WgPlan plan_wg_t(int N, int K, int Cin, int P, int Q, int taps) {
  WgPlan w;
  pixel_block(P, Q, cBK, w.bw, w.bh, w.bni);
  w.BN = 64;
  w.kt = 1;
  w.ct = (K + 63) / 64;
  const int tq = (Q + w.bw - 1) / w.bw, tp = (P + w.bh - 1) / w.bh, tn = (N + w.bni - 1) / w.bni;
  set_stages(w, tq * tp * tn);
  plan_splits(w, (taps + 1) / 2, (double)K * Cin * taps, 4.0 * N * P * Q * ((double)K + Cin));
  return w;
}

// dy: channels-last [N, P, Q, Kp]; x: channels-last [N, H, W, Cp]; partials
// [splits * taps][Cin][K] (the layout run_wgrad writes)
static int run_wgrad_t(const float* dyn, int Kp, const float* xn, int Cp, int N, int H, int W, int P, int Q, int K,
                       int Cin, const Taps& t, int sh, int sw, const WgPlan& p, float* part, cudaStream_t s) {
  CUtensorMap ma, mb, mc;
  PVB2_TRY(act_map(&ma, xn, N, H, W, Cp, p.bw, p.bh, p.bni, sw, sh, true));
  PVB2_TRY(act_map(&mb, dyn, N, P, Q, Kp, p.bw, p.bh, p.bni, 1, 1, true));
  const int taps = t.nr * t.ns;
  {
    uint64_t dims[3] = {(uint64_t)K, (uint64_t)Cin, (uint64_t)p.splits * taps};
    uint64_t str[2] = {(uint64_t)round4(K) * 4, (uint64_t)round4(K) * Cin * 4};
    uint32_t box[3] = {32, 32, 1};
    PVB2_TRY(encode_tiled(&mc, 3, part, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B));
  }
  ConvTcArgs a;
  memset(&a, 0, sizeof(a));
  a.N = N; a.Cin = Cin; a.Cp = Cp; a.Kout = K; a.P = P; a.Q = Q; a.R = t.nr; a.S = t.ns;
  a.sh = sh; a.sw = sw;
  for (int i = 0; i < kMaxTaps; ++i) {
    a.tap_h[i] = t.h[i];
    a.tap_w[i] = t.w[i];
  }
  a.bw = p.bw; a.bh = p.bh; a.bni = p.bni;
  a.tq = (Q + p.bw - 1) / p.bw;
  a.tp = (P + p.bh - 1) / p.bh;
  a.tn = (N + p.bni - 1) / p.bni;
  a.kt = 1;
  a.ct = p.ct;
  a.splits = p.splits;
  a.kb_per_split = p.kb_per;
  a.total_kb = p.total_kb;
  a.out = part;
  a.tiles = a.ct * ((taps + 1) / 2) * a.splits;
  return p.kbs == 2 ? launch_conv<64, kWgradT, 2>(ma, mb, mc, a, s) : launch_conv<64, kWgradT>(ma, mb, mc, a, s);
}

// pointwise weight gradient into partials [splits][C][K]
static int run_pw_wgrad(const float* dy, const float* x, int N, int C, int K, int64_t hw, const WgPlan& p,
                        float* part, cudaStream_t s) {
  CUtensorMap ma, mb, mc;
  memset(&mc, 0, sizeof(mc));
  PVB2_TRY(nchw_map(&ma, dy, N, K, hw, cBM, CU_TENSOR_MAP_SWIZZLE_128B));
  PVB2_TRY(nchw_map(&mb, x, N, C, hw, p.BN, CU_TENSOR_MAP_SWIZZLE_128B));
  ConvTcArgs a;
  memset(&a, 0, sizeof(a));
  a.N = N; a.Cin = C; a.Cp = C; a.Kout = K; a.P = 1; a.Q = (int)hw; a.R = 1; a.S = 1;
  a.sh = a.sw = 1;
  a.kt = p.kt;
  a.ct = p.ct;
  a.splits = p.splits;
  a.kb_per_split = p.kb_per;
  a.total_kb = p.total_kb;
  a.hwb = (int)((hw + 31) / 32);
  a.out = part;
  a.tiles = a.kt * a.ct * a.splits;
  PVB2_TRY(wg_partial_map(&mc, part, K, C, p.splits));
  return p.kbs == 2 ? launch_bn2<kPwWgrad>(p.BN, ma, mb, mc, a, s) : launch_bn<kPwWgrad>(p.BN, ma, mb, mc, a, s);
}

// im2col weight-gradient plan: GEMM rows = Kc im2col columns, GEMM columns = K
static WgPlan plan_im_wg(int N, int K, int Kc, int64_t pq) {
  WgPlan w;
  w.bw = 32; w.bh = 1; w.bni = 1;
  w.BN = bn_for(K);
  w.ct = (K + w.BN - 1) / w.BN;
  w.kt = (Kc + cBM - 1) / cBM;
  w.total_kb = N * (int)((pq + 31) / 32);
  plan_splits(w, 1, (double)K * Kc, 4.0 * N * pq * ((double)K + Kc));
  return w;
}

// im2col weight gradient into partials [splits][K][Kc]; xcol: [N][pq][Kc], dy: NCHW [N][K][pq]
// `win` (or null): xcol is that convolution's window copy and Kc = R * 32
static int run_im_wgrad(const float* xcol, int Kc, const float* dy, int N, int K, int64_t pq, const WgPlan& p,
                        float* part, cudaStream_t s, const pvb2_conv2d_desc* win = nullptr) {
  CUtensorMap ma, mb, mc;
  memset(&mc, 0, sizeof(mc));
  if (win) {
    PVB2_TRY(window_map(&ma, xcol, win, 16, 1, 1, 1, true));
  } else {
    uint64_t dims[3] = {(uint64_t)Kc, (uint64_t)pq, (uint64_t)N};
    uint64_t str[2] = {(uint64_t)Kc * 4, (uint64_t)pq * Kc * 4};
    uint32_t box[3] = {32, 32, 1};
    PVB2_TRY(encode_tiled(&ma, 3, xcol, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B));
  }
  PVB2_TRY(nchw_map(&mb, dy, N, K, pq, p.BN, CU_TENSOR_MAP_SWIZZLE_128B));
  ConvTcArgs a;
  memset(&a, 0, sizeof(a));
  a.N = N; a.Cin = K; a.Cp = K; a.Kout = Kc; a.P = 1; a.Q = (int)pq; a.R = 1; a.S = 1;
  a.sh = a.sw = 1;
  a.kt = p.kt;
  a.ct = p.ct;
  a.splits = p.splits;
  a.kb_per_split = p.kb_per;
  a.total_kb = p.total_kb;
  a.hwb = (int)((pq + 31) / 32);
  if (win) {
    a.win = 1;
    a.wq = win->Q;
    a.sh = win->stride_h;
  }
  a.out = part;
  a.tiles = a.kt * a.ct * a.splits;
  PVB2_TRY(wg_partial_map(&mc, part, Kc, K, p.splits));
  return launch_bn<kImWgrad>(p.BN, ma, mb, mc, a, s);
}

static int im2col(const pvb2_conv2d_desc* d, const float* x, float* xcol, cudaStream_t s) {
  PVB2_CHECK_ARG((int64_t)d->C * d->H * d->W < ((int64_t)1 << 31), "conv2d: image too large for im2col");
  const dim3 grid((unsigned)d->P, (unsigned)d->N);
  im2col_kernel<<<grid, 256, 0, s>>>(x, xcol, d->C, d->H, d->W, d->P, d->Q, d->R, d->S, im2col_channels(d),
                                     d->stride_h, d->stride_w, d->pad_h, d->pad_w, d->dil_h, d->dil_w);
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

static Taps fwd_taps(const pvb2_conv2d_desc* d) {
  Taps t;
  t.nr = d->R;
  t.ns = d->S;
  for (int i = 0; i < kMaxTaps; ++i) {
    t.h[i] = i * d->dil_h - d->pad_h;
    t.w[i] = i * d->dil_w - d->pad_w;
  }
  return t;
}

// -------------------------------------------------------- workspace plans
struct Layout {
  size_t a, b, c, total;
  size_t part = 0, part_bytes = 0;  // split-K slabs of forward-shaped launches
};

static Layout fwd_layout(const pvb2_conv2d_desc* d) {
  Layout l;
  l.a = l.b = l.c = l.total = 0;
  if (pointwise(d)) return l;
  if (strided_pointwise(d)) {
    l.total = l.c = align256(sampled_bytes(d));  // xs
    return l;
  }
  if (use_window(d)) {
    l.b = align256(win_bytes(d));
    l.total = l.b + align256((size_t)d->K * d->R * 32 * 4);
    const FwdSplit fs = plan_fwd_split(d->N, d->P, d->Q, d->K, d->R, 32);
    l.part = l.total;
    l.part_bytes = fs.bytes;
    l.total += align256(fs.bytes);
  } else if (use_im2col(d)) {
    const int Kc = im2col_channels(d);
    l.b = align256((size_t)d->N * d->P * d->Q * Kc * 4);
    l.total = l.b + align256((size_t)d->K * Kc * 4);
  } else {
    const int Cp = round4(d->C);
    l.b = align256((size_t)d->N * d->H * d->W * Cp * 4);
    l.total = l.b + align256((size_t)d->K * d->R * d->S * Cp * 4);
    const FwdSplit fs = plan_fwd_split(d->N, d->P, d->Q, d->K, d->R * d->S, Cp);
    l.part = l.total;
    l.part_bytes = fs.bytes;
    l.total += align256(fs.bytes);
  }
  l.c = l.total;
  return l;
}

static Layout dgrad_layout(const pvb2_conv2d_desc* d) {
  Layout l;
  l.a = l.b = l.c = l.total = 0;
  if (pointwise(d)) return l;
  if (strided_pointwise(d)) {
    l.total = l.c = align256(sampled_bytes(d));  // dX on the sampled pixels
    return l;
  }
  const int Kp = round4(d->K);
  l.b = align256((size_t)d->N * d->P * d->Q * Kp * 4);
  l.total = l.b + align256((size_t)d->C * d->R * d->S * Kp * 4);  // one phase's packed weights at a time
  // split-K slabs: the largest any phase needs (phases run one after another)
  size_t pb = 0;
  for (int a = 0; a < d->stride_h; ++a)
    for (int b = 0; b < d->stride_w; ++b) {
      int nr = 0, ns = 0;
      for (int r = 0; r < d->R; ++r) nr += ((a + d->pad_h - r * d->dil_h) % d->stride_h + d->stride_h) % d->stride_h == 0;
      for (int c = 0; c < d->S; ++c) ns += ((b + d->pad_w - c * d->dil_w) % d->stride_w + d->stride_w) % d->stride_w == 0;
      const int Hph = (d->H - a + d->stride_h - 1) / d->stride_h, Wph = (d->W - b + d->stride_w - 1) / d->stride_w;
      if (Hph <= 0 || Wph <= 0 || nr == 0 || ns == 0) continue;
      pb = std::max(pb, plan_fwd_split(d->N, Hph, Wph, d->C, nr * ns, Kp).bytes);
    }
  l.part = l.total;
  l.part_bytes = pb;
  l.total += align256(pb);
  l.c = l.total;
  return l;
}

static Layout wgrad_layout(const pvb2_conv2d_desc* d, WgPlan* plan) {
  Layout l;
  l.a = l.b = l.c = l.total = 0;
  if (pointwise(d)) {
    WgPlan p = pw_wg_swap(d) ? plan_pw_wg(d->N, d->C, d->K, (int64_t)d->H * d->W)
                             : plan_pw_wg(d->N, d->K, d->C, (int64_t)d->H * d->W);
    if (plan) *plan = p;
    l.total = align256(wg_partial_bytes(d->K, d->C, p.splits));  // partials only
    return l;
  }
  if (strided_pointwise(d)) {
    WgPlan p = pw_wg_swap(d) ? plan_pw_wg(d->N, d->C, d->K, (int64_t)d->P * d->Q)
                             : plan_pw_wg(d->N, d->K, d->C, (int64_t)d->P * d->Q);
    if (plan) *plan = p;
    l.c = align256(sampled_bytes(d));  // xs, then partials
    l.total = l.c + align256(wg_partial_bytes(d->K, d->C, p.splits));
    return l;
  }
  if (use_window(d)) {
    const int Kc = d->R * 32;
    WgPlan p = plan_im_wg(d->N, d->K, Kc, (int64_t)d->P * d->Q);
    if (plan) *plan = p;
    l.c = align256(win_bytes(d));                                 // window copy, then partials,
    l.b = l.c + align256(wg_partial_bytes(Kc, d->K, p.splits));   // then the summed [K][Kc]
    l.total = l.b + align256((size_t)d->K * Kc * 4);
    return l;
  }
  if (use_im2col(d)) {
    const int Kc = im2col_channels(d);
    WgPlan p = plan_im_wg(d->N, d->K, Kc, (int64_t)d->P * d->Q);
    if (plan) *plan = p;
    l.c = align256((size_t)d->N * d->P * d->Q * Kc * 4);  // im2col columns, then partials
    l.total = l.c + align256(wg_partial_bytes(Kc, d->K, p.splits));
    return l;
  }
  const int Kp = round4(d->K);
  const int Cx = round4(d->C);
  const int taps = d->R * d->S;
  WgPlan p = use_wgrad_t(d) ? plan_wg_t(d->N, d->K, d->C, d->P, d->Q, taps)
                            : plan_wg(d->N, d->K, d->C, d->P, d->Q, taps);
  if (plan) *plan = p;
  l.a = 0;                                                     // x channels-last
  l.b = align256((size_t)d->N * d->H * d->W * Cx * 4);         // dy channels-last
  l.c = l.b + align256((size_t)d->N * d->P * d->Q * Kp * 4);   // partials
  l.total = l.c + align256(wg_partial_bytes(d->K, d->C, p.splits * taps));
  return l;
}

size_t conv_tc_workspace(const pvb2_conv2d_desc* d, int which) {
  if (!tc_conv_shape_ok(d)) return 0;
  if (which == 0) return fwd_layout(d).total;
  if (which == 1) return dgrad_layout(d).total;
  return wgrad_layout(d, nullptr).total;
}

// The input as the forward and weight-gradient launches read it (channels-
// last copy or im2col columns): its size when this path stages one, else 0.
// A caller may keep the forward's copy for the weight gradient.
size_t conv_tc_staged_bytes(const pvb2_conv2d_desc* d) {
  if (!tc_conv_shape_ok(d) || pointwise(d) || strided_pointwise(d)) return 0;
  if (use_window(d)) return win_bytes(d);
  if (use_im2col(d)) return (size_t)d->N * d->P * d->Q * im2col_channels(d) * 4;
  if (!stride_ok_for_boxes(d)) return 0;
  return (size_t)d->N * d->H * d->W * round4(d->C) * 4;
}

// The output gradient as the input- and weight-gradient launches of the
// tap-box path both read it (channels-last, K padded to 4): its size when
// both passes take that path, else 0.  A caller may keep the input
// gradient's copy for the weight gradient.
size_t conv_tc_staged_grad_bytes(const pvb2_conv2d_desc* d) {
  if (!tc_conv_shape_ok(d) || pointwise(d) || strided_pointwise(d) || use_window(d) || use_im2col(d)) return 0;
  if (!stride_ok_for_boxes(d)) return 0;
  return (size_t)d->N * d->P * d->Q * round4(d->K) * 4;
}

// whether conv_tc_fwd (which 0), conv_tc_bwd_data (1) or conv_tc_bwd_filter
// (2) take the tensor-core path, given 16-byte aligned tensors and the
// workspace that conv_tc_workspace reports; mirrors their conditions
bool conv_tc_path(const pvb2_conv2d_desc* d, int which) {
  if (!tc_conv_shape_ok(d)) return false;
  if (pointwise(d) || strided_pointwise(d)) return true;
  if (which != 1 && (use_window(d) || use_im2col(d))) return true;
  return stride_ok_for_boxes(d);
}

// `staged` (conv_tc_staged_bytes long, or null): where the staged input goes
// instead of the workspace; *staged_written says whether it was filled
int conv_tc_fwd(const pvb2_conv2d_desc* d, const float* x, const float* w, const float* b, float* y, void* ws,
                size_t ws_bytes, cudaStream_t s, bool* handled, float* staged, bool* staged_written) {
  *handled = false;
  if (staged_written) *staged_written = false;
  if (!tc_conv_shape_ok(d)) return PVB2_OK;
  const int64_t pq = (int64_t)d->P * d->Q;
  if (pointwise(d)) {
    if (!aligned16(x) || !aligned16(w) || !aligned16(y)) return PVB2_OK;
    PVB2_TRY(run_pointwise(x, w, b, y, d->N, d->C, d->K, pq, false, s));
    *handled = true;
    return PVB2_OK;
  }
  Layout l = fwd_layout(d);
  if (!ws || ws_bytes < l.total) return PVB2_OK;  // not enough scratch: exact path
  if (strided_pointwise(d)) {
    if (!aligned16(w) || !aligned16(y)) return PVB2_OK;
    float* xs = (float*)ws;
    PVB2_TRY(subsample(d, x, xs, s));
    PVB2_TRY(run_pointwise(xs, w, b, y, d->N, d->C, d->K, pq, false, s));
    *handled = true;
    return PVB2_OK;
  }
  float* act = staged ? staged : (float*)((char*)ws + l.a);
  float* wp = (float*)((char*)ws + l.b);
  if (use_window(d)) {
    PVB2_TRY(pad_window(d, x, act, s));
    const int64_t n2 = (int64_t)d->K * d->R * 32;
    pack_w_window_kernel<<<grid_for(n2, 256), 256, 0, s>>>(w, wp, d->K, d->C, d->R, d->S);
    PVB2_LAUNCH_CHECK();
    Taps t;
    memset(&t, 0, sizeof(t));
    t.nr = d->R;
    t.ns = 1;
    for (int r = 0; r < d->R; ++r) t.h[r] = r;
    PVB2_TRY(run_fwd_like(act, wp, b, y, d->N, 32, d->H, d->W, d->K, t, d->P, d->Q, d->stride_h, 1, 0,
                          (int64_t)d->K * pq, pq, d->Q, 1, (float*)((char*)ws + l.part), l.part_bytes, s, d));
  } else if (use_im2col(d)) {
    const int Kc = im2col_channels(d);
    PVB2_TRY(im2col(d, x, act, s));
    const int64_t n2 = (int64_t)d->K * Kc;
    pack_w_rows_kernel<<<grid_for(n2, 256), 256, 0, s>>>(w, wp, d->K, d->C * d->R * d->S, Kc);
    PVB2_LAUNCH_CHECK();
    Taps t;
    memset(&t, 0, sizeof(t));
    t.nr = t.ns = 1;
    PVB2_TRY(run_fwd_like(act, wp, b, y, d->N, Kc, d->P, d->Q, d->K, t, d->P, d->Q, 1, 1, 0, (int64_t)d->K * pq, pq,
                          d->Q, 1, nullptr, 0, s));
  } else {
    if (!stride_ok_for_boxes(d)) return PVB2_OK;
    const int Cp = round4(d->C);
    PVB2_TRY(to_nhwc(x, act, d->N, d->C, Cp, (int64_t)d->H * d->W, s));
    const int64_t fwarps = (int64_t)d->K * ((Cp + 31) / 32);
    pack_w_fwd_kernel<<<(unsigned)((fwarps + 3) / 4), 128, 0, s>>>(w, wp, d->K, d->C, Cp, d->R * d->S);
    PVB2_LAUNCH_CHECK();
    PVB2_TRY(run_fwd_like(act, wp, b, y, d->N, Cp, d->H, d->W, d->K, fwd_taps(d), d->P, d->Q, d->stride_h,
                          d->stride_w, 0, (int64_t)d->K * pq, pq, d->Q, 1, (float*)((char*)ws + l.part),
                          l.part_bytes, s));
  }
  if (staged_written) *staged_written = staged != nullptr;
  *handled = true;
  return PVB2_OK;
}

// dX = dgrad + addend in the dgrad's own epilogue, for the 1x1 stride-1
// convolutions whose dgrad is a pointwise GEMM (a residual block's first
// convolution, whose input gradient is summed with the identity branch's)
bool conv_tc_bwd_data_acc_ok(const pvb2_conv2d_desc* d, const void* dy, const void* w, const void* dx,
                             const void* addend) {
  return tc_conv_shape_ok(d) && pointwise(d) && aligned16(dy) && aligned16(w) && aligned16(dx) && aligned16(addend);
}

int conv_tc_bwd_data_acc(const pvb2_conv2d_desc* d, const float* dy, const float* w, float* dx, const float* addend,
                         cudaStream_t s) {
  return run_pointwise(dy, w, nullptr, dx, d->N, d->C, d->K, (int64_t)d->H * d->W, true, s, addend);
}

static int pos_mod(int a, int m) { return ((a % m) + m) % m; }

// dX by sub-pixel phases: output rows h = sh*i + ph_a receive only the taps r
// with (ph_a + pad_h - r*dil_h) divisible by sh, each reading dY row
// i + (ph_a + pad_h - r*dil_h)/sh; likewise for columns.  Each phase is a
// stride-1 correlation over dY with its own tap list, written to dX with
// strides (sh, sw).  Phases without taps are zero.
// `staged_dy` (conv_tc_staged_grad_bytes long, or null): where the
// channels-last dy goes instead of the workspace; *staged_written says
// whether it was filled
int conv_tc_bwd_data(const pvb2_conv2d_desc* d, const float* dy, const float* w, float* dx, void* ws, size_t ws_bytes,
                     cudaStream_t s, bool* handled, float* staged_dy, bool* staged_written) {
  *handled = false;
  if (staged_written) *staged_written = false;
  if (!tc_conv_shape_ok(d)) return PVB2_OK;
  if (pointwise(d)) {
    if (!aligned16(dy) || !aligned16(w) || !aligned16(dx)) return PVB2_OK;
    PVB2_TRY(run_pointwise(dy, w, nullptr, dx, d->N, d->C, d->K, (int64_t)d->H * d->W, true, s));
    *handled = true;
    return PVB2_OK;
  }
  Layout l = dgrad_layout(d);
  if (!ws || ws_bytes < l.total) return PVB2_OK;
  if (!strided_pointwise(d) && !stride_ok_for_boxes(d)) return PVB2_OK;
  if (strided_pointwise(d)) {
    if (!aligned16(dy) || !aligned16(w) || !aligned16(dx)) return PVB2_OK;
    float* t = (float*)ws;
    PVB2_TRY(run_pointwise(dy, w, nullptr, t, d->N, d->C, d->K, (int64_t)d->P * d->Q, true, s));
    const int64_t total4 = (int64_t)d->N * d->C * d->H * d->W / 4;
    const FastDiv w4 = fast_div(d->W / 4), hd = fast_div(d->H);
    if (d->stride_h == 2 && d->stride_w == 2)
      scatter_strided_kernel<2><<<grid_for(total4, 256), 256, 0, s>>>(t, dx, (int)total4, w4, hd, d->P, d->Q, 2, 2);
    else
      scatter_strided_kernel<0><<<grid_for(total4, 256), 256, 0, s>>>(t, dx, (int)total4, w4, hd, d->P, d->Q,
                                                                       d->stride_h, d->stride_w);
    PVB2_LAUNCH_CHECK();
    *handled = true;
    return PVB2_OK;
  }
  const int Kp = round4(d->K);
  const bool keep = staged_dy && conv_tc_staged_grad_bytes(d) > 0;
  float* dyn = keep ? staged_dy : (float*)((char*)ws + l.a);
  float* wd = (float*)((char*)ws + l.b);
  bool empty_phase = false;
  Taps ph[16];
  int nph = 0;
  int pa[16], pb[16];
  for (int a = 0; a < d->stride_h; ++a)
    for (int b = 0; b < d->stride_w; ++b) {
      Taps t;
      t.nr = t.ns = 0;
      for (int r = 0; r < d->R; ++r) {
        const int v = a + d->pad_h - r * d->dil_h;
        if (pos_mod(v, d->stride_h) == 0) {
          t.h[t.nr] = r;  // store r; offsets below
          ++t.nr;
        }
      }
      for (int s_ = 0; s_ < d->S; ++s_) {
        const int v = b + d->pad_w - s_ * d->dil_w;
        if (pos_mod(v, d->stride_w) == 0) {
          t.w[t.ns] = s_;
          ++t.ns;
        }
      }
      const int Hph = (d->H - a + d->stride_h - 1) / d->stride_h, Wph = (d->W - b + d->stride_w - 1) / d->stride_w;
      if (Hph <= 0 || Wph <= 0) continue;
      if (t.nr == 0 || t.ns == 0) {
        empty_phase = true;
        continue;
      }
      pa[nph] = a;
      pb[nph] = b;
      ph[nph++] = t;
    }
  if (empty_phase) PVB2_CUDA_TRY(cudaMemsetAsync(dx, 0, (size_t)d->N * d->C * d->H * d->W * sizeof(float), s));
  PVB2_TRY(to_nhwc(dy, dyn, d->N, d->K, Kp, (int64_t)d->P * d->Q, s));
  const int64_t hw = (int64_t)d->H * d->W;
  for (int i = 0; i < nph; ++i) {
    const int a = pa[i], b = pb[i];
    Taps t = ph[i];
    int rl[8] = {0}, sl[8] = {0};
    for (int j = 0; j < t.nr; ++j) rl[j] = t.h[j];
    for (int j = 0; j < t.ns; ++j) sl[j] = t.w[j];
    const int64_t wn = (int64_t)d->C * t.nr * t.ns * Kp;
    pack_w_phase_kernel<<<grid_for(wn, 256), 256, 0, s>>>(w, wd, d->K, Kp, d->C, d->R, d->S, t.nr, t.ns,
                                                          make_int4(rl[0], rl[1], rl[2], rl[3]),
                                                          make_int4(rl[4], rl[5], rl[6], rl[7]),
                                                          make_int4(sl[0], sl[1], sl[2], sl[3]),
                                                          make_int4(sl[4], sl[5], sl[6], sl[7]));
    PVB2_LAUNCH_CHECK();
    Taps off;
    off.nr = t.nr;
    off.ns = t.ns;
    for (int j = 0; j < kMaxTaps; ++j) off.h[j] = off.w[j] = 0;
    for (int j = 0; j < t.nr; ++j) off.h[j] = (a + d->pad_h - t.h[j] * d->dil_h) / d->stride_h;
    for (int j = 0; j < t.ns; ++j) off.w[j] = (b + d->pad_w - t.w[j] * d->dil_w) / d->stride_w;
    const int Hph = (d->H - a + d->stride_h - 1) / d->stride_h, Wph = (d->W - b + d->stride_w - 1) / d->stride_w;
    PVB2_TRY(run_fwd_like(dyn, wd, nullptr, dx, d->N, Kp, d->P, d->Q, d->C, off, Hph, Wph, 1, 1,
                          (int64_t)a * d->W + b, (int64_t)d->C * hw, hw, (int64_t)d->stride_h * d->W, d->stride_w,
                          (float*)((char*)ws + l.part), l.part_bytes, s));
  }
  if (staged_written) *staged_written = keep;
  *handled = true;
  return PVB2_OK;
}

// `staged`: the forward's staged copy of this x (conv_tc_fwd), or null;
// `staged_dy`: the input gradient's channels-last dy (conv_tc_bwd_data), or null
int conv_tc_bwd_filter(const pvb2_conv2d_desc* d, const float* x, const float* dy, float* dw, void* ws,
                       size_t ws_bytes, cudaStream_t s, bool* handled, const float* staged,
                       const float* staged_dy) {
  *handled = false;
  if (!tc_conv_shape_ok(d)) return PVB2_OK;
  WgPlan p;
  Layout l = wgrad_layout(d, &p);
  if (!ws || ws_bytes < l.total) return PVB2_OK;  // not enough scratch: exact path
  const int RS = d->R * d->S;
  if (pointwise(d)) {
    if (!aligned16(x) || !aligned16(dy)) return PVB2_OK;
    float* part = (float*)ws;
    if (pw_wg_swap(d)) {
      // partials [sp][k][c] -> dW[k][c]
      PVB2_TRY(run_pw_wgrad(x, dy, d->N, d->K, d->C, (int64_t)d->H * d->W, p, part, s));
      PVB2_TRY(wgrad_reduce(part, p.splits, 1, d->C, d->K, d->C, d->K, dw, 1, d->C, 0, s));
    } else {
      PVB2_TRY(run_pw_wgrad(dy, x, d->N, d->C, d->K, (int64_t)d->H * d->W, p, part, s));
      // partials [sp][c][k] -> dW[k][c]
      PVB2_TRY(wgrad_reduce(part, p.splits, 1, d->K, d->C, d->K, d->C, dw, d->C, 1, 0, s));
    }
    *handled = true;
    return PVB2_OK;
  }
  if (strided_pointwise(d)) {
    if (!aligned16(dy)) return PVB2_OK;
    float* xs = (float*)ws;
    float* part = (float*)((char*)ws + l.c);
    PVB2_TRY(subsample(d, x, xs, s));
    if (pw_wg_swap(d)) {
      PVB2_TRY(run_pw_wgrad(xs, dy, d->N, d->K, d->C, (int64_t)d->P * d->Q, p, part, s));
      PVB2_TRY(wgrad_reduce(part, p.splits, 1, d->C, d->K, d->C, d->K, dw, 1, d->C, 0, s));
    } else {
      PVB2_TRY(run_pw_wgrad(dy, xs, d->N, d->C, d->K, (int64_t)d->P * d->Q, p, part, s));
      PVB2_TRY(wgrad_reduce(part, p.splits, 1, d->K, d->C, d->K, d->C, dw, d->C, 1, 0, s));
    }
    *handled = true;
    return PVB2_OK;
  }
  if (use_window(d)) {
    const int Kc = d->R * 32;
    float* xw = staged ? const_cast<float*>(staged) : (float*)ws;
    float* part = (float*)((char*)ws + l.c);
    float* sum = (float*)((char*)ws + l.b);
    if (!staged) PVB2_TRY(pad_window(d, x, xw, s));
    PVB2_TRY(run_im_wgrad(xw, Kc, dy, d->N, d->K, (int64_t)d->P * d->Q, p, part, s, d));
    // partials [sp][k][r * 32 + j] -> sum[k][r * 32 + j] -> dW[k][c][r][s]
    PVB2_TRY(wgrad_reduce(part, p.splits, 1, Kc, d->K, Kc, d->K, sum, 1, Kc, 0, s));
    const int64_t nw = (int64_t)d->K * d->C * RS;
    unwindow_wgrad_kernel<<<grid_for(nw, 256), 256, 0, s>>>(sum, Kc, dw, d->K, d->C, d->R, d->S);
    PVB2_LAUNCH_CHECK();
    *handled = true;
    return PVB2_OK;
  }
  if (use_im2col(d)) {
    const int Kc = im2col_channels(d), crs = d->C * RS;
    float* xcol = staged ? const_cast<float*>(staged) : (float*)ws;
    float* part = (float*)((char*)ws + l.c);
    if (!staged) PVB2_TRY(im2col(d, x, xcol, s));
    PVB2_TRY(run_im_wgrad(xcol, Kc, dy, d->N, d->K, (int64_t)d->P * d->Q, p, part, s));
    // partials [sp][k][j] -> dW[k][j] for the crs real columns
    PVB2_TRY(wgrad_reduce(part, p.splits, 1, Kc, d->K, crs, d->K, dw, 1, crs, 0, s));
    *handled = true;
    return PVB2_OK;
  }
  if (!stride_ok_for_boxes(d)) return PVB2_OK;
  const int Kp = round4(d->K);
  float* xn = staged ? const_cast<float*>(staged) : (float*)((char*)ws + l.a);
  float* dyn = staged_dy ? const_cast<float*>(staged_dy) : (float*)((char*)ws + l.b);
  float* part = (float*)((char*)ws + l.c);
  if (!staged_dy) PVB2_TRY(to_nhwc(dy, dyn, d->N, d->K, Kp, (int64_t)d->P * d->Q, s));
  const int Cp = round4(d->C);
  if (!staged) PVB2_TRY(to_nhwc(x, xn, d->N, d->C, Cp, (int64_t)d->H * d->W, s));
  if (use_wgrad_t(d)) {
    PVB2_TRY(run_wgrad_t(dyn, Kp, xn, Cp, d->N, d->H, d->W, d->P, d->Q, d->K, d->C, fwd_taps(d), d->stride_h,
                         d->stride_w, p, part, s));
  } else {
    PVB2_TRY(run_wgrad(dyn, Kp, xn, Cp, d->N, d->H, d->W, d->P, d->Q, d->K, d->C, fwd_taps(d), d->stride_h,
                       d->stride_w, p, part, s));
  }
  // partials [sp][rs][c][k] -> dW[k][c][rs]
  PVB2_TRY(wgrad_reduce(part, p.splits, RS, d->K, d->C, d->K, d->C, dw, (int64_t)d->C * RS, RS, 1, s));
  *handled = true;
  return PVB2_OK;
}

}  // namespace pvb2

extern "C" PVB2_API int pvb2_conv_tc_status(int* timed_out, int reset) {
  return pvb2::tc_timeout_flag_local(timed_out, reset);
}
