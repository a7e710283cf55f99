// Stream compaction for masked_select and nonzero.
//
// The reference's masked_select copied tensor and mask to the host and
// selected there (src/tensor_ops.cpp:303-356).  Here it stays on the device:
//   count:  each CTA counts the true mask elements of its 4096-element chunk
//           (warp ballots), then one CTA turns the per-chunk counts into an
//           exclusive prefix and the total;
//   gather: each CTA re-reads its chunk and writes the selected elements at
//           prefix + rank-within-chunk, so the output keeps row-major order.
#include "common.cuh"

namespace pvb2 {

constexpr int kSelChunk = 4096;

__device__ __forceinline__ int dtype_size_dev(int dt) {
  return (dt == PVB2_F64 || dt == PVB2_I64) ? 8 : (dt == PVB2_F32 || dt == PVB2_I32) ? 4
       : (dt == PVB2_F16 || dt == PVB2_BF16 || dt == PVB2_I16) ? 2 : 1;
}
constexpr int kSelThreads = 256;

__device__ __forceinline__ bool mask_at(const IterShape& it, const void* m, int mdt, int64_t i) {
  int64_t offs[kMaxArgs];
  iter_offsets(it, 1, i, offs);
  return load_as<int64_t>(m, offs[0], mdt) != 0;
}

__global__ void select_count_kernel(IterShape it, const void* mask, int mdt, int64_t n, int64_t* counts) {
  __shared__ int warp_tot[kSelThreads / 32];
  const int64_t base = (int64_t)blockIdx.x * kSelChunk;
  int c = 0;
  for (int k = threadIdx.x; k < kSelChunk; k += blockDim.x) {
    const int64_t i = base + k;
    if (i < n && mask_at(it, mask, mdt, i)) ++c;
  }
  for (int o = 16; o > 0; o >>= 1) c += __shfl_down_sync(0xffffffffu, c, o);
  if ((threadIdx.x & 31) == 0) warp_tot[threadIdx.x >> 5] = c;
  __syncthreads();
  if (threadIdx.x == 0) {
    int t = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += warp_tot[w];
    counts[blockIdx.x] = t;
  }
}

// exclusive prefix over chunk counts, single CTA, sequential per thread slice
__global__ void select_prefix_kernel(int64_t* counts, int64_t nchunks, int64_t* total) {
  __shared__ int64_t part[1024];
  const int64_t per = (nchunks + blockDim.x - 1) / blockDim.x;
  const int64_t b = threadIdx.x * per, e = min(nchunks, b + per);
  int64_t s = 0;
  for (int64_t i = b; i < e; ++i) s += counts[i];
  part[threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    int64_t acc = 0;
    for (int t = 0; t < (int)blockDim.x; ++t) {
      const int64_t v = part[t];
      part[t] = acc;
      acc += v;
    }
    *total = acc;
  }
  __syncthreads();
  int64_t acc = part[threadIdx.x];
  for (int64_t i = b; i < e; ++i) {
    const int64_t v = counts[i];
    counts[i] = acc;
    acc += v;
  }
}

// one warp-ordered pass per chunk: ranks from ballots, warp totals from shared memory
__global__ void select_gather_kernel(IterShape mit, const void* mask, int mdt, IterShape sit, const void* src,
                                     int sdt, int64_t n, const int64_t* prefix, void* out, int ndim,
                                     IterShape shape_it) {
  __shared__ int warp_tot[kSelThreads / 32];
  __shared__ int64_t running;
  const int64_t base = (int64_t)blockIdx.x * kSelChunk;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (threadIdx.x == 0) running = prefix[blockIdx.x];
  __syncthreads();
  for (int k0 = 0; k0 < kSelChunk; k0 += blockDim.x) {
    const int64_t i = base + k0 + threadIdx.x;
    const bool sel = i < n && mask_at(mit, mask, mdt, i);
    const unsigned ballot = __ballot_sync(0xffffffffu, sel);
    if (lane == 0) warp_tot[wid] = __popc(ballot);
    __syncthreads();
    int before = 0;
    for (int w = 0; w < wid; ++w) before += warp_tot[w];
    const int64_t pos = running + before + __popc(ballot & ((1u << lane) - 1u));
    if (sel) {
      if (src) {
        int64_t offs[kMaxArgs];
        iter_offsets(sit, 1, i, offs);
        // raw element copy (exact for every dtype)
        switch (dtype_size_dev(sdt)) {
          case 8: static_cast<uint64_t*>(out)[pos] = static_cast<const uint64_t*>(src)[offs[0]]; break;
          case 4: static_cast<uint32_t*>(out)[pos] = static_cast<const uint32_t*>(src)[offs[0]]; break;
          case 2: static_cast<uint16_t*>(out)[pos] = static_cast<const uint16_t*>(src)[offs[0]]; break;
          default: static_cast<uint8_t*>(out)[pos] = static_cast<const uint8_t*>(src)[offs[0]]; break;
        }
      } else {
        // coordinates of linear index i in the logical shape
        int64_t lin = i;
        for (int d = ndim - 1; d >= 0; --d) {
          const int64_t sz = shape_it.sizes[d];
          static_cast<int64_t*>(out)[pos * ndim + d] = lin % sz;
          lin /= sz;
        }
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int t = 0;
      for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += warp_tot[w];
      running += t;
    }
    __syncthreads();
  }
}

struct IndexArgs {
  int n;
  const int64_t* idx[4];
  int64_t size[4];
  int64_t stride[4];
};

__global__ void index_gather_kernel(IterShape it, void* out, const void* src, int esize, IndexArgs ia, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t offs[kMaxArgs];
    iter_offsets(it, 2 + ia.n, i, offs);
    int64_t so = offs[1];
    for (int k = 0; k < ia.n; ++k) {
      int64_t v = ia.idx[k][offs[2 + k]];
      if (v < 0) v += ia.size[k];
      v = v < 0 ? 0 : (v >= ia.size[k] ? ia.size[k] - 1 : v);  // out-of-range indices are clamped, never read out of bounds
      so += v * ia.stride[k];
    }
    switch (esize) {
      case 8: static_cast<uint64_t*>(out)[offs[0]] = static_cast<const uint64_t*>(src)[so]; break;
      case 4: static_cast<uint32_t*>(out)[offs[0]] = static_cast<const uint32_t*>(src)[so]; break;
      case 2: static_cast<uint16_t*>(out)[offs[0]] = static_cast<const uint16_t*>(src)[so]; break;
      default: static_cast<uint8_t*>(out)[offs[0]] = static_cast<const uint8_t*>(src)[so]; break;
    }
  }
}

static int64_t nchunks_of(int64_t n) { return (n + kSelChunk - 1) / kSelChunk; }

}  // namespace pvb2

using namespace pvb2;

extern "C" {

int pvb2_index_gather(const pvb2_tensor* out, const pvb2_tensor* src, int n_index, const pvb2_tensor* indices,
                      const int64_t* index_sizes, const int64_t* index_strides, pvb2_stream stream) {
  const int64_t n = numel(out);
  if (n == 0) return PVB2_OK;
  PVB2_CHECK_ARG(n_index >= 1 && n_index <= 4, "index: 1 to 4 index tensors supported (got %d)", n_index);
  PVB2_CHECK_ARG(src->dtype == out->dtype && src->ndim == out->ndim, "index: src/out mismatch");
  IndexArgs ia;
  ia.n = n_index;
  const pvb2_tensor* ts[2 + 4] = {out, src};
  for (int k = 0; k < n_index; ++k) {
    PVB2_CHECK_ARG(indices[k].dtype == PVB2_I64 && indices[k].ndim == out->ndim, "index: int64 indices expected");
    ts[2 + k] = &indices[k];
    ia.idx[k] = (const int64_t*)indices[k].data;
    ia.size[k] = index_sizes[k];
    ia.stride[k] = index_strides[k];
    PVB2_CHECK_ARG(index_sizes[k] > 0, "index: indexing into an empty dimension");
  }
  IterShape it;
  make_iter(&it, ts, 2 + n_index);
  index_gather_kernel<<<grid_for(n, 256), 256, 0, as_stream(stream)>>>(it, out->data, src->data,
                                                                       dtype_size(out->dtype), ia, n);
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

size_t pvb2_select_workspace_size(int64_t n) { return (size_t)(nchunks_of(n) + 1) * sizeof(int64_t); }

int pvb2_select_count(const pvb2_tensor* mask, void* workspace, size_t workspace_bytes, int64_t* d_total,
                      pvb2_stream stream) {
  const int64_t n = numel(mask);
  cudaStream_t s = as_stream(stream);
  if (n == 0) {
    PVB2_CUDA_TRY(cudaMemsetAsync(d_total, 0, sizeof(int64_t), s));
    return PVB2_OK;
  }
  PVB2_CHECK_ARG(workspace && workspace_bytes >= pvb2_select_workspace_size(n), "select: workspace too small");
  IterShape it;
  const pvb2_tensor* ts[1] = {mask};
  make_iter(&it, ts, 1);
  const int64_t nc = nchunks_of(n);
  PVB2_CHECK_ARG(nc < (1ll << 31), "select: tensor too large");
  int64_t* counts = (int64_t*)workspace;
  select_count_kernel<<<(unsigned)nc, kSelThreads, 0, s>>>(it, mask->data, mask->dtype, n, counts);
  PVB2_LAUNCH_CHECK();
  select_prefix_kernel<<<1, 1024, 0, s>>>(counts, nc, d_total);
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

int pvb2_select_gather(const pvb2_tensor* src, const pvb2_tensor* mask, void* out, const void* workspace,
                       pvb2_stream stream) {
  const int64_t n = numel(mask);
  if (n == 0) return PVB2_OK;
  IterShape mit, sit, shp;
  const pvb2_tensor* tm[1] = {mask};
  make_iter(&mit, tm, 1);
  if (src) {
    PVB2_CHECK_ARG(numel(src) == n, "select: src and mask sizes differ");
    const pvb2_tensor* tsrc[1] = {src};
    make_iter(&sit, tsrc, 1);
  } else {
    sit = mit;
  }
  // the logical (uncoalesced) shape for nonzero's coordinates
  shp.ndim = mask->ndim;
  for (int d = 0; d < mask->ndim; ++d) shp.sizes[d] = mask->sizes[d];
  const int64_t nc = nchunks_of(n);
  select_gather_kernel<<<(unsigned)nc, kSelThreads, 0, as_stream(stream)>>>(
      mit, mask->data, mask->dtype, sit, src ? src->data : nullptr, src ? src->dtype : 0, n,
      (const int64_t*)workspace, out, mask->ndim, shp);
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

}  // extern "C"
