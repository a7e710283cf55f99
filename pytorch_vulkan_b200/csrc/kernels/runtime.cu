// Device runtime for the `ocl` backend: devices, memory, streams, events,
// and the tensor plumbing kernels (fill, strided copy, cat).
//
// Replaces the reference's CLContextManager (src/CLTensor.h:87-282), the
// OpenCL buffer calls behind CLCache (src/CLTensor.cpp:9-92) and the
// copy/fill kernels used by src/tensor_ops.cpp:118-225.
#include <stdarg.h>
#include <mutex>
#include <vector>
#include "common.cuh"

namespace pvb2 {

std::atomic<int64_t> g_launches{0};
static thread_local char t_err[1024];

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_err, sizeof(t_err), fmt, ap);
  va_end(ap);
}

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_err, sizeof(t_err), fmt, ap);
  va_end(ap);
  return code;
}

int num_sms() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

void make_iter(IterShape* it, const pvb2_tensor* const* ts, int n) {
  const pvb2_tensor* t0 = ts[0];
  int nd = 0;
  int64_t sizes[PVB2_MAX_DIMS];
  int64_t strides[kMaxArgs][PVB2_MAX_DIMS];
  for (int d = 0; d < t0->ndim; ++d) {
    if (t0->sizes[d] == 1) continue;
    sizes[nd] = t0->sizes[d];
    for (int a = 0; a < n; ++a) strides[a][nd] = ts[a]->strides[d];
    ++nd;
  }
  // merge dim i into dim i+1 (its inner neighbour) when contiguous for all operands
  int out = 0;
  for (int d = 0; d < nd; ++d) {
    if (out > 0) {
      bool can = true;
      for (int a = 0; a < n; ++a)
        if (strides[a][out - 1] != strides[a][d] * sizes[d]) { can = false; break; }
      if (can) {
        sizes[out - 1] *= sizes[d];
        for (int a = 0; a < n; ++a) strides[a][out - 1] = strides[a][d];
        continue;
      }
    }
    sizes[out] = sizes[d];
    for (int a = 0; a < n; ++a) strides[a][out] = strides[a][d];
    ++out;
  }
  it->ndim = out;
  for (int d = 0; d < out; ++d) {
    it->sizes[d] = sizes[d];
    for (int a = 0; a < kMaxArgs; ++a) it->strides[a][d] = a < n ? strides[a][d] : 0;
  }
}

// ------------------------------------------------------------------ fill
template <typename T>
__global__ void fill_contig_kernel(T* __restrict__ p, int64_t n, T v) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t step = (int64_t)gridDim.x * blockDim.x;
  for (; i < n; i += step) p[i] = v;
}

__global__ void fill_contig_f32x4_kernel(float4* __restrict__ p, int64_t n4, float v) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t step = (int64_t)gridDim.x * blockDim.x;
  float4 f = make_float4(v, v, v, v);
  for (; i < n4; i += step) p[i] = f;
}

__global__ void fill_strided_kernel(IterShape it, void* base, int dt, double v, int64_t n) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t step = (int64_t)gridDim.x * blockDim.x;
  for (; i < n; i += step) {
    int64_t offs[kMaxArgs];
    iter_offsets(it, 1, i, offs);
    store_as<double>(base, offs[0], dt, v);
  }
}

__global__ void arange_kernel(IterShape it, void* base, int dt, double start, double step, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t offs[kMaxArgs];
    iter_offsets(it, 1, i, offs);
    if (dt == PVB2_F32 || dt == PVB2_F64 || dt == PVB2_F16 || dt == PVB2_BF16)
      store_as<double>(base, offs[0], dt, start + (double)i * step);
    else
      store_as<int64_t>(base, offs[0], dt, (int64_t)start + (int64_t)i * (int64_t)step);
  }
}

// ------------------------------------------------------------------ copy
__global__ void copy_strided_kernel(IterShape it, void* dst, int ddt, const void* src, int sdt, int64_t n) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t step = (int64_t)gridDim.x * blockDim.x;
  const bool integral = !(sdt == PVB2_F32 || sdt == PVB2_F64 || sdt == PVB2_F16 || sdt == PVB2_BF16);
  for (; i < n; i += step) {
    int64_t offs[kMaxArgs];
    iter_offsets(it, 2, i, offs);
    if (integral && ddt != PVB2_F64 && ddt != PVB2_F32) {
      store_as<int64_t>(dst, offs[0], ddt, load_as<int64_t>(src, offs[1], sdt));
    } else {
      store_as<double>(dst, offs[0], ddt, load_as<double>(src, offs[1], sdt));
    }
  }
}

// Same-dtype copy whose innermost dim is unit-stride on both sides (the
// head split / merge permutes of attention, transposed-batch reshapes): rows
// of `units` V-sized words, a group of G lanes per row, row offsets from the
// outer dims computed once per row.  `outer` holds the outer dims with
// strides in V units.
// (long rows are cut into pieces of `piece` words, a group per piece)
template <typename V>
__global__ void __launch_bounds__(256) copy_rows_kernel(IterShape outer, int64_t rows, int64_t units, int64_t piece,
                                                        int group, V* __restrict__ dst, const V* __restrict__ src) {
  const int lane = threadIdx.x % group;
  const int64_t pieces = (units + piece - 1) / piece;
  const int64_t g0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / group;
  const int64_t gstep = (int64_t)gridDim.x * blockDim.x / group;
  for (int64_t gi = g0; gi < rows * pieces; gi += gstep) {
    const int64_t r = gi / pieces, u0 = (gi - r * pieces) * piece, u1 = min(units, u0 + piece);
    int64_t offs[kMaxArgs];
    iter_offsets(outer, 2, r, offs);
    V* d = dst + offs[0];
    const V* x = src + offs[1];
    for (int64_t u = u0 + lane; u < u1; u += group) d[u] = __ldg(x + u);
  }
}

// 2-D tiled transpose for the common "make contiguous" case of a permuted
// fp32 tensor: dst[r][c] = src[c*ld + r] blocks.
__global__ void transpose_f32_kernel(float* __restrict__ dst, const float* __restrict__ src, int64_t rows,
                                     int64_t cols, int64_t batch, int64_t src_row_stride,
                                     int64_t src_col_stride, int64_t src_batch_stride) {
  __shared__ float tile[32][33];
  int64_t b = blockIdx.z;
  int64_t r0 = (int64_t)blockIdx.y * 32, c0 = (int64_t)blockIdx.x * 32;
  const float* s = src + b * src_batch_stride;
  float* d = dst + b * rows * cols;
  // read with the source's unit-stride dim (rows) fastest
  for (int j = threadIdx.y; j < 32; j += blockDim.y) {
    int64_t c = c0 + j, r = r0 + threadIdx.x;
    if (r < rows && c < cols) tile[j][threadIdx.x] = s[r * src_row_stride + c * src_col_stride];
  }
  __syncthreads();
  for (int j = threadIdx.y; j < 32; j += blockDim.y) {
    int64_t r = r0 + j, c = c0 + threadIdx.x;
    if (r < rows && c < cols) d[r * cols + c] = tile[threadIdx.x][j];
  }
}

}  // namespace pvb2

using namespace pvb2;

extern "C" {

const char* pvb2_last_error(void) { return t_err; }
int pvb2_version(void) { return 1; }
int64_t pvb2_launch_count(void) { return g_launches.load(); }

int pvb2_device_count(int* count) {
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  *count = n;
  return PVB2_OK;
}

int pvb2_set_device(int device) {
  PVB2_CUDA_TRY(cudaSetDevice(device));
  return PVB2_OK;
}

int pvb2_get_device(int* device) {
  PVB2_CUDA_TRY(cudaGetDevice(device));
  return PVB2_OK;
}

int pvb2_device_name(int device, char* buf, int buflen) {
  cudaDeviceProp prop;
  PVB2_CUDA_TRY(cudaGetDeviceProperties(&prop, device));
  snprintf(buf, buflen, "%s", prop.name);
  return PVB2_OK;
}

int pvb2_device_synchronize(void) {
  PVB2_CUDA_TRY(cudaDeviceSynchronize());
  return PVB2_OK;
}

int pvb2_mem_get_info(size_t* free_bytes, size_t* total_bytes) {
  PVB2_CUDA_TRY(cudaMemGetInfo(free_bytes, total_bytes));
  return PVB2_OK;
}

int pvb2_malloc(void** ptr, size_t bytes) {
  *ptr = nullptr;
  if (bytes == 0) return PVB2_OK;
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e == cudaErrorMemoryAllocation) {
    cudaGetLastError();
    return fail(PVB2_ERR_OOM, "cudaMalloc of %zu bytes failed: out of memory", bytes);
  }
  PVB2_CUDA_TRY(e);
  return PVB2_OK;
}

int pvb2_free(void* ptr) {
  if (!ptr) return PVB2_OK;
  PVB2_CUDA_TRY(cudaFree(ptr));
  return PVB2_OK;
}

int pvb2_host_alloc(void** ptr, size_t bytes) {
  *ptr = nullptr;
  if (bytes == 0) return PVB2_OK;
  cudaError_t e = cudaHostAlloc(ptr, bytes, cudaHostAllocPortable);
  if (e == cudaErrorMemoryAllocation) {
    cudaGetLastError();
    return fail(PVB2_ERR_OOM, "cudaHostAlloc of %zu bytes failed", bytes);
  }
  PVB2_CUDA_TRY(e);
  return PVB2_OK;
}

int pvb2_host_free(void* ptr) {
  if (!ptr) return PVB2_OK;
  PVB2_CUDA_TRY(cudaFreeHost(ptr));
  return PVB2_OK;
}

int pvb2_pointer_info(const void* ptr, int* is_device, int* is_pinned_host, int* device) {
  *is_device = 0;
  *is_pinned_host = 0;
  *device = -1;
  cudaPointerAttributes attr;
  cudaError_t e = cudaPointerGetAttributes(&attr, ptr);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return PVB2_OK;
  }
  if (attr.type == cudaMemoryTypeDevice) {
    *is_device = 1;
    *device = attr.device;
  } else if (attr.type == cudaMemoryTypeHost) {
    *is_pinned_host = 1;
    *device = attr.device;
  } else if (attr.type == cudaMemoryTypeManaged) {
    *is_device = 1;
    *device = attr.device;
  }
  return PVB2_OK;
}

int pvb2_stream_create(pvb2_stream* stream, int priority) {
  cudaStream_t s;
  PVB2_CUDA_TRY(cudaStreamCreateWithPriority(&s, cudaStreamNonBlocking, priority));
  *stream = s;
  return PVB2_OK;
}

// ---------------------------------------------------------------- graphs
// A captured sequence of this library's work on one stream, replayed with
// one launch.  The number of kernels captured is kept so that each replay
// adds it to the launch counter, as launching them one by one would.
namespace {
struct Graph {
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  int64_t kernels = 0;
};
thread_local int64_t t_capture_start = -1;
}  // namespace

int pvb2_graph_capture_begin(pvb2_stream stream) {
  PVB2_CHECK_ARG(stream != nullptr, "graph capture needs a created stream, not the default stream");
  PVB2_CUDA_TRY(cudaStreamBeginCapture(as_stream(stream), cudaStreamCaptureModeRelaxed));
  t_capture_start = g_launches.load();
  return PVB2_OK;
}

int pvb2_graph_capture_end(pvb2_stream stream, pvb2_graph* graph) {
  PVB2_CHECK_ARG(graph != nullptr, "graph_capture_end: graph is NULL");
  *graph = nullptr;
  cudaGraph_t g = nullptr;
  cudaError_t e = cudaStreamEndCapture(as_stream(stream), &g);
  const int64_t kernels = t_capture_start >= 0 ? g_launches.load() - t_capture_start : 0;
  t_capture_start = -1;
  if (e != cudaSuccess || !g) {
    if (g) cudaGraphDestroy(g);
    cudaGetLastError();
    return fail(PVB2_ERR_CUDA, "graph capture failed: %s", cudaGetErrorString(e));
  }
  cudaGraphExec_t exec = nullptr;
  e = cudaGraphInstantiate(&exec, g, 0);
  if (e != cudaSuccess) {
    cudaGraphDestroy(g);
    cudaGetLastError();
    return fail(PVB2_ERR_CUDA, "graph instantiation failed: %s", cudaGetErrorString(e));
  }
  Graph* h = new Graph;
  h->graph = g;
  h->exec = exec;
  h->kernels = kernels;
  *graph = h;
  return PVB2_OK;
}

int pvb2_graph_launch(pvb2_graph graph, pvb2_stream stream) {
  PVB2_CHECK_ARG(graph != nullptr, "graph_launch: graph is NULL");
  Graph* h = static_cast<Graph*>(graph);
  PVB2_CUDA_TRY(cudaGraphLaunch(h->exec, as_stream(stream)));
  g_launches.fetch_add(h->kernels, std::memory_order_relaxed);
  return PVB2_OK;
}

int pvb2_graph_kernel_count(pvb2_graph graph, int64_t* kernels) {
  PVB2_CHECK_ARG(graph != nullptr && kernels != nullptr, "graph_kernel_count: NULL argument");
  *kernels = static_cast<Graph*>(graph)->kernels;
  return PVB2_OK;
}

int pvb2_graph_destroy(pvb2_graph graph) {
  if (!graph) return PVB2_OK;
  Graph* h = static_cast<Graph*>(graph);
  if (h->exec) cudaGraphExecDestroy(h->exec);
  if (h->graph) cudaGraphDestroy(h->graph);
  delete h;
  return PVB2_OK;
}

int pvb2_stream_is_capturing(pvb2_stream stream, int* capturing) {
  PVB2_CHECK_ARG(capturing != nullptr, "stream_is_capturing: NULL argument");
  cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
  PVB2_CUDA_TRY(cudaStreamIsCapturing(as_stream(stream), &st));
  *capturing = st == cudaStreamCaptureStatusActive ? 1 : 0;
  return PVB2_OK;
}

int pvb2_stream_destroy(pvb2_stream stream) {
  PVB2_CUDA_TRY(cudaStreamDestroy(as_stream(stream)));
  return PVB2_OK;
}

int pvb2_stream_synchronize(pvb2_stream stream) {
  PVB2_CUDA_TRY(cudaStreamSynchronize(as_stream(stream)));
  return PVB2_OK;
}

int pvb2_stream_query(pvb2_stream stream, int* done) {
  cudaError_t e = cudaStreamQuery(as_stream(stream));
  if (e == cudaErrorNotReady) {
    cudaGetLastError();
    *done = 0;
    return PVB2_OK;
  }
  PVB2_CUDA_TRY(e);
  *done = 1;
  return PVB2_OK;
}

int pvb2_stream_wait_event(pvb2_stream stream, pvb2_event event) {
  PVB2_CUDA_TRY(cudaStreamWaitEvent(as_stream(stream), (cudaEvent_t)event, 0));
  return PVB2_OK;
}

int pvb2_event_create(pvb2_event* event, int timing) {
  cudaEvent_t e;
  PVB2_CUDA_TRY(cudaEventCreateWithFlags(&e, timing ? cudaEventDefault : cudaEventDisableTiming));
  *event = e;
  return PVB2_OK;
}

int pvb2_event_destroy(pvb2_event event) {
  PVB2_CUDA_TRY(cudaEventDestroy((cudaEvent_t)event));
  return PVB2_OK;
}

int pvb2_event_record(pvb2_event event, pvb2_stream stream) {
  PVB2_CUDA_TRY(cudaEventRecord((cudaEvent_t)event, as_stream(stream)));
  return PVB2_OK;
}

int pvb2_event_synchronize(pvb2_event event) {
  PVB2_CUDA_TRY(cudaEventSynchronize((cudaEvent_t)event));
  return PVB2_OK;
}

int pvb2_event_query(pvb2_event event, int* done) {
  cudaError_t e = cudaEventQuery((cudaEvent_t)event);
  if (e == cudaErrorNotReady) {
    cudaGetLastError();
    *done = 0;
    return PVB2_OK;
  }
  PVB2_CUDA_TRY(e);
  *done = 1;
  return PVB2_OK;
}

int pvb2_event_elapsed_ms(pvb2_event start, pvb2_event end, float* ms) {
  PVB2_CUDA_TRY(cudaEventElapsedTime(ms, (cudaEvent_t)start, (cudaEvent_t)end));
  return PVB2_OK;
}

int pvb2_memcpy_async(void* dst, const void* src, size_t bytes, int kind, pvb2_stream stream) {
  if (bytes == 0) return PVB2_OK;
  cudaMemcpyKind k = kind == 0 ? cudaMemcpyHostToDevice
                   : kind == 1 ? cudaMemcpyDeviceToHost
                   : kind == 2 ? cudaMemcpyDeviceToDevice
                               : cudaMemcpyDefault;
  PVB2_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, k, as_stream(stream)));
  return PVB2_OK;
}

int pvb2_memset_async(void* dst, int value, size_t bytes, pvb2_stream stream) {
  if (bytes == 0) return PVB2_OK;
  PVB2_CUDA_TRY(cudaMemsetAsync(dst, value, bytes, as_stream(stream)));
  return PVB2_OK;
}

int pvb2_fill(const pvb2_tensor* out, double value, pvb2_stream stream) {
  const int64_t n = numel(out);
  if (n == 0) return PVB2_OK;
  cudaStream_t s = as_stream(stream);
  const int block = 256;
  if (is_contiguous(out)) {
    if (out->dtype == PVB2_F32) {
      float v = (float)value;
      if (((uintptr_t)out->data & 15) == 0 && n % 4 == 0) {
        fill_contig_f32x4_kernel<<<grid_for(n / 4, block), block, 0, s>>>((float4*)out->data, n / 4, v);
      } else {
        fill_contig_kernel<float><<<grid_for(n, block), block, 0, s>>>((float*)out->data, n, v);
      }
      PVB2_LAUNCH_CHECK();
      return PVB2_OK;
    }
    if (value == 0.0) {
      PVB2_CUDA_TRY(cudaMemsetAsync(out->data, 0, (size_t)n * dtype_size(out->dtype), s));
      return PVB2_OK;
    }
    if (out->dtype == PVB2_I64) {
      fill_contig_kernel<int64_t><<<grid_for(n, block), block, 0, s>>>((int64_t*)out->data, n, (int64_t)value);
      PVB2_LAUNCH_CHECK();
      return PVB2_OK;
    }
  }
  IterShape it;
  const pvb2_tensor* ts[1] = {out};
  make_iter(&it, ts, 1);
  fill_strided_kernel<<<grid_for(n, block), block, 0, s>>>(it, out->data, out->dtype, value, n);
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

int pvb2_copy(const pvb2_tensor* dst, const pvb2_tensor* src, pvb2_stream stream) {
  PVB2_CHECK_ARG(dst->ndim == src->ndim, "pvb2_copy: ndim mismatch %d vs %d", dst->ndim, src->ndim);
  for (int d = 0; d < dst->ndim; ++d)
    PVB2_CHECK_ARG(dst->sizes[d] == src->sizes[d], "pvb2_copy: size mismatch at dim %d", d);
  const int64_t n = numel(dst);
  if (n == 0) return PVB2_OK;
  cudaStream_t s = as_stream(stream);
  if (dst->dtype == src->dtype && is_contiguous(dst) && is_contiguous(src)) {
    PVB2_CUDA_TRY(cudaMemcpyAsync(dst->data, src->data, (size_t)n * dtype_size(dst->dtype),
                                  cudaMemcpyDeviceToDevice, s));
    return PVB2_OK;
  }
  IterShape it;
  const pvb2_tensor* ts[2] = {dst, src};
  make_iter(&it, ts, 2);
  // fp32 2-D (or batched 2-D) transpose into a contiguous destination
  if (dst->dtype == PVB2_F32 && src->dtype == PVB2_F32 && (it.ndim == 2 || it.ndim == 3) &&
      it.strides[0][it.ndim - 1] == 1 && it.strides[1][it.ndim - 1] != 1) {
    int nd = it.ndim;
    int64_t rows = it.sizes[nd - 2], cols = it.sizes[nd - 1];
    int64_t batch = nd == 3 ? it.sizes[0] : 1;
    bool dst_dense = it.strides[0][nd - 2] == cols && (nd == 2 || it.strides[0][0] == rows * cols);
    if (dst_dense && it.strides[1][nd - 2] == 1 && batch < 65536) {
      dim3 grid((unsigned)((cols + 31) / 32), (unsigned)((rows + 31) / 32), (unsigned)batch);
      transpose_f32_kernel<<<grid, dim3(32, 8), 0, s>>>((float*)dst->data, (const float*)src->data, rows, cols,
                                                        batch, it.strides[1][nd - 2], it.strides[1][nd - 1],
                                                        nd == 3 ? it.strides[1][0] : 0);
      PVB2_LAUNCH_CHECK();
      return PVB2_OK;
    }
  }
  const int esz = (int)dtype_size(dst->dtype);
  if (dst->dtype == src->dtype && it.ndim >= 2 && it.strides[0][it.ndim - 1] == 1 &&
      it.strides[1][it.ndim - 1] == 1 && it.sizes[it.ndim - 1] * esz >= 64 && esz <= 16) {
    // pick the widest word that every row start and the row length allow
    const int64_t inner_bytes = it.sizes[it.ndim - 1] * esz;
    int vb = 16;
    auto fits = [&](int w) {
      if (inner_bytes % w || ((uintptr_t)dst->data % w) || ((uintptr_t)src->data % w)) return false;
      for (int d = 0; d < it.ndim - 1; ++d)
        if ((it.strides[0][d] * esz) % w || (it.strides[1][d] * esz) % w) return false;
      return true;
    };
    while (vb > esz && !fits(vb)) vb >>= 1;
    if (vb >= 4 && fits(vb)) {
      IterShape outer;
      outer.ndim = it.ndim - 1;
      int64_t rows = 1;
      for (int d = 0; d < outer.ndim; ++d) {
        outer.sizes[d] = it.sizes[d];
        outer.strides[0][d] = it.strides[0][d] * esz / vb;
        outer.strides[1][d] = it.strides[1][d] * esz / vb;
        rows *= it.sizes[d];
      }
      const int64_t units = inner_bytes / vb;
      int group = 4;
      while (group < 32 && group < units) group <<= 1;
      const int64_t piece = 16384 / vb;  // 16 KB per group at most
      const int block = 256;
      const int grid = grid_for(rows * ((units + piece - 1) / piece) * group, block);
      if (vb == 16)
        copy_rows_kernel<float4><<<grid, block, 0, s>>>(outer, rows, units, piece, group, (float4*)dst->data,
                                                        (const float4*)src->data);
      else if (vb == 8)
        copy_rows_kernel<float2><<<grid, block, 0, s>>>(outer, rows, units, piece, group, (float2*)dst->data,
                                                        (const float2*)src->data);
      else
        copy_rows_kernel<float><<<grid, block, 0, s>>>(outer, rows, units, piece, group, (float*)dst->data,
                                                       (const float*)src->data);
      PVB2_LAUNCH_CHECK();
      return PVB2_OK;
    }
  }
  const int block = 256;
  copy_strided_kernel<<<grid_for(n, block), block, 0, s>>>(it, dst->data, dst->dtype, src->data, src->dtype, n);
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

int pvb2_arange(const pvb2_tensor* out, double start, double step, pvb2_stream stream) {
  const int64_t n = numel(out);
  if (n == 0) return PVB2_OK;
  PVB2_CHECK_ARG(out->ndim == 1, "pvb2_arange: out must be 1-D");
  IterShape it;
  const pvb2_tensor* ts[1] = {out};
  make_iter(&it, ts, 1);
  arange_kernel<<<grid_for(n, 256), 256, 0, as_stream(stream)>>>(it, out->data, out->dtype, start, step, n);
  PVB2_LAUNCH_CHECK();
  return PVB2_OK;
}

int pvb2_cat(const pvb2_tensor* out, const pvb2_tensor* inputs, int n_inputs, int dim, pvb2_stream stream) {
  PVB2_CHECK_ARG(dim >= 0 && dim < out->ndim, "pvb2_cat: bad dim %d", dim);
  int64_t off = 0;
  for (int i = 0; i < n_inputs; ++i) {
    const pvb2_tensor* in = &inputs[i];
    if (numel(in) == 0) continue;
    PVB2_CHECK_ARG(in->ndim == out->ndim, "pvb2_cat: ndim mismatch");
    pvb2_tensor slice = *out;
    slice.sizes[dim] = in->sizes[dim];
    slice.data = (char*)out->data + off * out->strides[dim] * dtype_size(out->dtype);
    PVB2_TRY(pvb2_copy(&slice, in, stream));
    off += in->sizes[dim];
  }
  PVB2_CHECK_ARG(off == out->sizes[dim], "pvb2_cat: sizes do not add up along dim %d", dim);
  return PVB2_OK;
}

}  // extern "C"
