// Host runtime of the `ocl` (PrivateUse1) backend.
//
//  * device / stream registry          replaces CLContextManager, src/CLTensor.h:87-282
//  * caching device allocator          replaces CLCache, src/CLTensor.h:39-84, CLTensor.cpp:9-92
//  * DeviceGuardImplInterface          replaces OCLDevImpl, src/registeration.cpp:31-82
//  * at::Allocator registration        replaces OCLAllocator, registeration.cpp:85-109
//  * PrivateUse1HooksInterface         replaces HooksInterface, registeration.cpp:111-127
//  * Philox generator state            replaces the per-device RandomState, CLTensor.h:154-157
//  * ExecGuard tracing + profiling     replaces src/guard.cpp and CLTensor.cpp:95-151
//  * pybind `impl_*` functions         replaces src/python_iface.cpp:1-88
#include <ATen/core/GeneratorForPrivateuseone.h>
#include <ATen/detail/PrivateUse1HooksInterface.h>
#include <c10/core/impl/DeviceGuardImplInterface.h>
#include <nvtx3/nvToolsExt.h>
#include <pthread.h>
#include <torch/extension.h>

#include <chrono>
#include <cstdlib>
#include <fstream>
#include <map>
#include <memory>
#include <mutex>
#include <random>
#include <unordered_map>

#include "ocl.h"

namespace ocl {

static bool env_flag(const char* a, const char* b = nullptr) {
  const char* v = getenv(a);
  if (!v && b) v = getenv(b);
  return v && *v && strcmp(v, "0") != 0;
}
static int env_int(const char* a, const char* b, int def) {
  const char* v = getenv(a);
  if (!v && b) v = getenv(b);
  return v && *v ? atoi(v) : def;
}

// ==================================================================== devices
static std::atomic<bool> g_bad_fork{false};
static const bool g_no_cache = env_flag("OPENCL_NO_MEM_CACHE", "B200_NO_MEM_CACHE");
static const bool g_debug_cache = env_flag("OPENCL_DEBUG_CACHE", "B200_DEBUG_CACHE");
static const bool g_cache_oversized = env_flag("OPENCL_CACHE_OVERSIZED", "B200_CACHE_OVERSIZED");

struct DeviceState {
  std::once_flag init;
  bool ready = false;
  pvb2_stream default_stream = nullptr;
  std::mutex m;
  std::vector<pvb2_stream> streams;  // id k >= 1 -> streams[k-1]
};

static int query_count() {
  int n = 0;
  pvb2_device_count(&n);
  return n;
}

int device_count() {
  static int n = query_count();
  return n;
}

static std::vector<DeviceState>& states() {
  static std::vector<DeviceState> s(std::max(device_count(), 1));
  return s;
}

static thread_local int t_device = -1;  // -1: not yet set on this thread
static thread_local std::vector<int64_t> t_stream_ids;

static void check_index(int d) {
  TORCH_CHECK(d >= 0 && d < device_count(), "ocl: invalid device index ", d, " (", device_count(),
              " device(s) visible)");
}

static DeviceState& dev_state(int d) {
  check_index(d);
  DeviceState& st = states()[d];
  std::call_once(st.init, [&] {
    int prev = 0;
    pvb2_get_device(&prev);
    OCL_CHECK(pvb2_set_device(d));
    OCL_CHECK(pvb2_stream_create(&st.default_stream, 0));
    st.ready = true;
    pvb2_set_device(prev);
  });
  return st;
}

int current_device() {
  if (t_device < 0) {
    t_device = 0;
    if (device_count() > 0) OCL_CHECK(pvb2_set_device(0));
  }
  return t_device;
}

void set_device(int d) {
  check_index(d);
  if (t_device != d) {
    OCL_CHECK(pvb2_set_device(d));
    t_device = d;
  }
}

void ensure_device(int d) {
  if (t_device != d) set_device(d);
}

static int64_t current_stream_id(int d) {
  if ((int)t_stream_ids.size() <= d) return 0;
  return t_stream_ids[d];
}

static void set_current_stream_id(int d, int64_t id) {
  if ((int)t_stream_ids.size() <= d) t_stream_ids.resize(d + 1, 0);
  t_stream_ids[d] = id;
}

static pvb2_stream stream_by_id(int d, int64_t id) {
  DeviceState& st = dev_state(d);
  if (id == 0) return st.default_stream;
  std::lock_guard<std::mutex> g(st.m);
  TORCH_CHECK(id >= 1 && id <= (int64_t)st.streams.size(), "ocl: unknown stream id ", id);
  return st.streams[id - 1];
}

static int64_t new_stream(int d, int priority) {
  DeviceState& st = dev_state(d);
  DeviceScope scope(d);
  pvb2_stream s = nullptr;
  OCL_CHECK(pvb2_stream_create(&s, priority));
  std::lock_guard<std::mutex> g(st.m);
  st.streams.push_back(s);
  return (int64_t)st.streams.size();
}

pvb2_stream stream_for(int d) { return stream_by_id(d, current_stream_id(d)); }
pvb2_stream current_stream() { return stream_for(current_device()); }

void after_op(int d) {
  if (g_no_cache) OCL_CHECK(pvb2_stream_synchronize(stream_for(d)));
}

DeviceScope::DeviceScope(const at::Tensor& t) : DeviceScope((int)t.device().index()) {}
DeviceScope::DeviceScope(int device, bool flush) {
  if (flush) flush_deferred();
  prev = current_device();
  changed = device >= 0 && device != prev;
  if (changed) set_device(device);
}
DeviceScope::~DeviceScope() {
  if (changed) {
    pvb2_set_device(prev);
    t_device = prev;
  }
}

// ================================================================ allocator
// Size classes: 512 B granules up to 1 MiB, then four classes per power of
// two (at most 25% padding; the reference padded to the next power of two,
// CLTensor.cpp:9-20).  Freed blocks are kept per (device, class) and reused
// in stream order.  A block that was also used on another stream
// (record_stream) is held back until an event recorded on that stream at
// free time has completed.
// Blocks allocated while a graph is being captured on a device come from a
// pool of their own and go back to it when freed: the graph's replays write
// them, so they stay reserved for it (never handed to other tensors, never
// released) until the graph is destroyed, when the pool is retired and its
// free blocks join the device's ordinary free lists.
struct CapturePool {
  std::unordered_map<size_t, std::vector<void*>> free_blocks;
  bool retired = false;
};

struct BlockCtx {
  void* ptr;
  size_t size;
  int device;
  std::vector<pvb2_stream> extra_streams;
  std::shared_ptr<CapturePool> cpool;  // set for blocks allocated during a capture
};

struct PendingFree {
  BlockCtx* blk;
  std::vector<pvb2_event> events;
};

struct Pool {
  std::mutex m;
  std::unordered_map<size_t, std::vector<void*>> free_blocks;
  std::vector<PendingFree> pending;
  std::shared_ptr<CapturePool> capturing;  // the pool of the graph being captured, if any
  size_t reserved = 0, allocated = 0, peak_allocated = 0, peak_reserved = 0;
  uint64_t n_malloc = 0, n_hits = 0;
};

static std::vector<Pool>& pools() {
  static std::vector<Pool> p(std::max(device_count(), 1));
  return p;
}

static size_t size_class(size_t n) {
  if (n <= 512) return 512;
  if (n <= (1u << 20)) return (n + 511) & ~size_t(511);
  size_t p = 1;
  while ((p << 1) <= n) p <<= 1;
  size_t step = p / 4;
  return (n + step - 1) / step * step;
}

static void process_pending(Pool& pool) {
  for (size_t i = 0; i < pool.pending.size();) {
    bool done = true;
    for (auto e : pool.pending[i].events) {
      int d = 0;
      pvb2_event_query(e, &d);
      if (!d) {
        done = false;
        break;
      }
    }
    if (done) {
      for (auto e : pool.pending[i].events) pvb2_event_destroy(e);
      BlockCtx* b = pool.pending[i].blk;
      pool.free_blocks[b->size].push_back(b->ptr);
      delete b;
      pool.pending[i] = pool.pending.back();
      pool.pending.pop_back();
    } else {
      ++i;
    }
  }
}

static void release_cached(int device, Pool& pool) {
  // caller holds pool.m; the device is current
  for (auto& kv : pool.free_blocks) {
    for (void* p : kv.second) {
      pvb2_free(p);
      pool.reserved -= kv.first;
    }
  }
  pool.free_blocks.clear();
}

static void free_block(void* raw_ctx);

class OclAllocator final : public c10::Allocator {
 public:
  c10::DataPtr allocate(size_t nbytes) override {
    const int d = current_device();
    const c10::Device dev(kOcl, d);
    if (nbytes == 0) return c10::DataPtr(nullptr, nullptr, &free_block, dev);
    dev_state(d);
    const size_t sz = size_class(nbytes);
    Pool& pool = pools()[d];
    void* p = nullptr;
    {
      std::lock_guard<std::mutex> g(pool.m);
      if (pool.capturing) return allocate_captured(pool, d, nbytes, sz);
      if (!pool.pending.empty()) process_pending(pool);
      auto it = pool.free_blocks.find(sz);
      if (it != pool.free_blocks.end() && !it->second.empty()) {
        p = it->second.back();
        it->second.pop_back();
        pool.n_hits++;
      } else if (g_cache_oversized) {
        // reuse a block of one of the next two classes
        size_t c = sz;
        for (int k = 0; k < 2 && !p; ++k) {
          c = size_class(c + 1);
          auto jt = pool.free_blocks.find(c);
          if (jt != pool.free_blocks.end() && !jt->second.empty()) {
            p = jt->second.back();
            jt->second.pop_back();
            pool.n_hits++;
          }
        }
      }
      if (!p) {
        int s = pvb2_malloc(&p, sz);
        if (s == PVB2_ERR_OOM) {
          // give cached blocks back and retry once
          pvb2_device_synchronize();
          release_cached(d, pool);
          s = pvb2_malloc(&p, sz);
        }
        TORCH_CHECK(s == PVB2_OK, "ocl: out of memory allocating ", nbytes, " bytes on device ", d, ": ",
                    pvb2_last_error(), " (reserved ", pool.reserved, " bytes)");
        pool.reserved += sz;
        pool.n_malloc++;
        pool.peak_reserved = std::max(pool.peak_reserved, pool.reserved);
      }
      pool.allocated += sz;
      pool.peak_allocated = std::max(pool.peak_allocated, pool.allocated);
      if (g_debug_cache)
        fprintf(stderr, "ocl cache: alloc %zu (class %zu) allocated=%zu reserved=%zu\n", nbytes, sz, pool.allocated,
                pool.reserved);
    }
    return c10::DataPtr(p, new BlockCtx{p, sz, d, {}}, &free_block, dev);
  }

  c10::DeleterFnPtr raw_deleter() const override { return nullptr; }

 private:
  // caller holds pool.m: a block of the capture pool (no event polling and
  // no release of cached blocks while capturing: neither may run then)
  c10::DataPtr allocate_captured(Pool& pool, int d, size_t nbytes, size_t sz) {
    const c10::Device dev(kOcl, d);
    void* p = nullptr;
    auto it = pool.capturing->free_blocks.find(sz);
    if (it != pool.capturing->free_blocks.end() && !it->second.empty()) {
      p = it->second.back();
      it->second.pop_back();
      pool.n_hits++;
    } else {
      const int s = pvb2_malloc(&p, sz);
      TORCH_CHECK(s == PVB2_OK, "ocl: out of memory allocating ", nbytes, " bytes on device ", d,
                  " while capturing a graph: ", pvb2_last_error());
      pool.reserved += sz;
      pool.n_malloc++;
      pool.peak_reserved = std::max(pool.peak_reserved, pool.reserved);
    }
    pool.allocated += sz;
    pool.peak_allocated = std::max(pool.peak_allocated, pool.allocated);
    return c10::DataPtr(p, new BlockCtx{p, sz, d, {}, pool.capturing}, &free_block, dev);
  }

 public:
  void copy_data(void* dest, const void* src, std::size_t count) const override {
    flush_deferred();
    OCL_CHECK(pvb2_memcpy_async(dest, src, count, 2, current_stream()));
  }
};

static OclAllocator g_allocator;

static void free_block(void* raw_ctx) {
  if (!raw_ctx) return;
  BlockCtx* b = static_cast<BlockCtx*>(raw_ctx);
  Pool& pool = pools()[b->device];
  std::lock_guard<std::mutex> g(pool.m);
  pool.allocated -= b->size;
  if (b->cpool) {  // a graph's block: back to its pool while the graph lives
    (b->cpool->retired ? pool.free_blocks : b->cpool->free_blocks)[b->size].push_back(b->ptr);
    delete b;
    return;
  }
  if (g_no_cache) {
    DeviceScope scope(b->device);
    pvb2_stream_synchronize(stream_for(b->device));
    pvb2_free(b->ptr);
    pool.reserved -= b->size;
    delete b;
    return;
  }
  if (!b->extra_streams.empty()) {
    PendingFree pf{b, {}};
    DeviceScope scope(b->device);
    for (auto s : b->extra_streams) {
      pvb2_event e = nullptr;
      if (pvb2_event_create(&e, 0) == PVB2_OK) {
        pvb2_event_record(e, s);
        pf.events.push_back(e);
      }
    }
    pool.pending.push_back(std::move(pf));
    return;
  }
  pool.free_blocks[b->size].push_back(b->ptr);
  delete b;
}

void allocator_record_stream(const c10::DataPtr& ptr, pvb2_stream stream) {
  if (ptr.get_deleter() != &free_block) return;
  BlockCtx* b = static_cast<BlockCtx*>(ptr.get_context());
  if (!b) return;
  if (stream == stream_for(b->device)) return;
  for (auto s : b->extra_streams)
    if (s == stream) return;
  b->extra_streams.push_back(stream);
}

c10::Allocator* allocator() { return &g_allocator; }

REGISTER_ALLOCATOR(c10::DeviceType::PrivateUse1, &g_allocator);

static void empty_cache_all() {
  for (int d = 0; d < device_count(); ++d) {
    if (!states()[d].ready) continue;
    Pool& pool = pools()[d];
    std::lock_guard<std::mutex> g(pool.m);
    TORCH_CHECK(!pool.capturing, "ocl: empty_cache() while a graph is being captured on device ", d);
  }
  clear_staged_inputs();
  for (int d = 0; d < device_count(); ++d) {
    if (!states()[d].ready) continue;
    DeviceScope scope(d);
    pvb2_device_synchronize();
    Pool& pool = pools()[d];
    std::lock_guard<std::mutex> g(pool.m);
    process_pending(pool);
    release_cached(d, pool);
  }
}

Workspace::Workspace(size_t n, int device) : bytes(n) {
  if (n == 0) return;
  DeviceScope scope(device);
  ptr = g_allocator.allocate(n);
}

// ------------------------------------------------------- pinned host memory
static void free_pinned(void* p) { pvb2_host_free(p); }

class PinnedAllocator final : public c10::Allocator {
 public:
  c10::DataPtr allocate(size_t n) override {
    void* p = nullptr;
    if (n) OCL_CHECK(pvb2_host_alloc(&p, n));
    return c10::DataPtr(p, p, &free_pinned, c10::Device(c10::DeviceType::CPU));
  }
  c10::DeleterFnPtr raw_deleter() const override { return &free_pinned; }
  void copy_data(void* dest, const void* src, std::size_t count) const override { memcpy(dest, src, count); }
};
static PinnedAllocator g_pinned;

// ================================================================= settings
static std::atomic<int> g_math{env_int("B200_MATH_MODE", "OCL_MATH_MODE", PVB2_MATH_TF32)};
int math_mode() { return g_math.load(); }
void set_math_mode(int m) {
  TORCH_CHECK(m == PVB2_MATH_TF32 || m == PVB2_MATH_FP32,
              "ocl: math mode must be 0 (TF32 tensor cores) or 1 (exact fp32); 3xTF32 (2) is not implemented");
  g_math = m;
}

// ================================================================== tracing
std::atomic<int> g_trace_mode{env_int("OPENCL_DEBUG_MODE", "B200_DEBUG_MODE", 0)};
std::atomic<bool> g_profiling{false};
static thread_local int t_depth = 0;
static thread_local std::vector<const char*> t_sections;

struct ProfRecord {
  std::string section, kernel;
  pvb2_event start, end;
};
struct ProfState {
  std::mutex m;
  bool enabled_before_init = false;
  bool active = false;
  std::vector<ProfRecord> records;
  pvb2_event origin = nullptr;
};
static std::vector<ProfState>& prof() {
  static std::vector<ProfState> p(std::max(device_count(), 1));
  return p;
}

ExecGuard::ExecGuard(const char* n, int dev) : name(n), device(dev), slot(-1) {
  flush_deferred();
  // a named range per op for timeline profilers (Nsight Systems, ncu --nvtx),
  // the counterpart of the reference's per-op section (src/guard.cpp:5-14);
  // without an attached tool this is a call through a null-checked pointer
  nvtxRangePushA(n);
  const int mode = g_trace_mode.load(std::memory_order_relaxed);
  if (mode == 2) fprintf(stderr, "%*s> %s (ocl:%d)\n", 2 * t_depth, "", n, dev);
  ++t_depth;
  t_sections.push_back(n);
  if (g_profiling.load(std::memory_order_relaxed) && dev >= 0 && dev < device_count() && prof()[dev].active) {
    ProfState& ps = prof()[dev];
    ProfRecord r;
    std::string sec;
    for (size_t i = 0; i + 1 < t_sections.size(); ++i) {
      if (i) sec += ":";
      sec += t_sections[i];
    }
    r.section = sec;
    r.kernel = n;
    pvb2_event_create(&r.start, 1);
    pvb2_event_create(&r.end, 1);
    pvb2_event_record(r.start, stream_for(dev));
    std::lock_guard<std::mutex> g(ps.m);
    slot = (int)ps.records.size();
    ps.records.push_back(r);
  }
}

ExecGuard::~ExecGuard() {
  --t_depth;
  t_sections.pop_back();
  if (slot >= 0) {
    ProfState& ps = prof()[device];
    std::lock_guard<std::mutex> g(ps.m);
    pvb2_event_record(ps.records[slot].end, stream_for(device));
  }
  if (std::uncaught_exceptions() > 0 && g_trace_mode.load() >= 1)
    fprintf(stderr, "ocl: exception in op %s (ocl:%d)\n", name, device);
  nvtxRangePop();
  if (device >= 0) after_op(device);
}

static bool enable_profiling(int d) {
  check_index(d);
  prof()[d].enabled_before_init = true;
  return true;
}

static void start_profiling(int d) {
  check_index(d);
  DeviceScope scope(d);
  ProfState& ps = prof()[d];
  std::lock_guard<std::mutex> g(ps.m);
  ps.records.clear();
  if (!ps.origin) pvb2_event_create(&ps.origin, 1);
  pvb2_event_record(ps.origin, stream_for(d));
  ps.active = true;
  g_profiling = true;
}

static void stop_profiling(int d, const std::string& path) {
  check_index(d);
  DeviceScope scope(d);
  OCL_CHECK(pvb2_stream_synchronize(stream_for(d)));
  ProfState& ps = prof()[d];
  std::lock_guard<std::mutex> g(ps.m);
  ps.active = false;
  bool any = false;
  for (auto& p : prof()) any = any || p.active;
  g_profiling = any;
  std::ofstream f(path);
  TORCH_CHECK(f.good(), "ocl: cannot open profile log ", path);
  // same header as the reference's log (CLTensor.cpp:95-140)
  f << "section,kernel,start (ms),end (ms),duraion(ms)\n";
  for (auto& r : ps.records) {
    float t0 = 0, t1 = 0;
    pvb2_event_elapsed_ms(ps.origin, r.start, &t0);
    pvb2_event_elapsed_ms(ps.origin, r.end, &t1);
    f << r.section << "," << r.kernel << "," << t0 << "," << t1 << "," << (t1 - t0) << "\n";
    pvb2_event_destroy(r.start);
    pvb2_event_destroy(r.end);
  }
  ps.records.clear();
}

// =============================================================== guard impl
class OclGuardImpl final : public c10::impl::DeviceGuardImplInterface {
 public:
  c10::DeviceType type() const override { return kOcl; }
  c10::Device exchangeDevice(c10::Device d) const override {
    const int old = current_device();
    if (d.index() >= 0 && d.index() != old) set_device(d.index());
    return c10::Device(kOcl, old);
  }
  c10::Device getDevice() const override { return c10::Device(kOcl, current_device()); }
  void setDevice(c10::Device d) const override {
    if (d.index() >= 0) set_device(d.index());
  }
  void uncheckedSetDevice(c10::Device d) const noexcept override {
    try {
      if (d.index() >= 0) set_device(d.index());
    } catch (...) {
    }
  }
  c10::Stream getStream(c10::Device d) const override {
    const int idx = d.index() < 0 ? current_device() : d.index();
    return c10::Stream(c10::Stream::UNSAFE, c10::Device(kOcl, idx), current_stream_id(idx));
  }
  c10::Stream getDefaultStream(c10::Device d) const override {
    const int idx = d.index() < 0 ? current_device() : d.index();
    return c10::Stream(c10::Stream::UNSAFE, c10::Device(kOcl, idx), 0);
  }
  c10::Stream getStreamFromGlobalPool(c10::Device d, bool isHighPriority) const override {
    return getNewStream(d, isHighPriority ? -1 : 0);
  }
  c10::Stream getNewStream(c10::Device d, int priority) const override {
    const int idx = d.index() < 0 ? current_device() : d.index();
    return c10::Stream(c10::Stream::UNSAFE, c10::Device(kOcl, idx), new_stream(idx, priority));
  }
  c10::Stream exchangeStream(c10::Stream s) const override {
    const int idx = s.device_index();
    c10::Stream old = getStream(s.device());
    set_current_stream_id(idx, s.id());
    return old;
  }
  void* getStreamNativeHandle(const c10::Stream s) const override {
    flush_deferred();  // the caller may launch its own work on the stream
    return stream_by_id(s.device_index(), s.id());
  }
  void destroyEvent(void* e, const c10::DeviceIndex) const noexcept override {
    if (e) pvb2_event_destroy(e);
  }
  void record(void** event, const c10::Stream& s, const c10::DeviceIndex idx, const c10::EventFlag flag) const override {
    TORCH_CHECK(idx == -1 || idx == s.device_index(), "ocl: event device does not match the stream's");
    DeviceScope scope(s.device_index());
    if (!*event) {
      pvb2_event e = nullptr;
      OCL_CHECK(pvb2_event_create(&e, flag == c10::EventFlag::BACKEND_DEFAULT ? 1 : 0));
      *event = e;
    }
    OCL_CHECK(pvb2_event_record(*event, stream_by_id(s.device_index(), s.id())));
  }
  void block(void* e, const c10::Stream& s) const override {
    if (!e) return;
    DeviceScope scope(s.device_index());
    OCL_CHECK(pvb2_stream_wait_event(stream_by_id(s.device_index(), s.id()), e));
  }
  bool queryEvent(void* e) const override {
    if (!e) return true;
    int done = 0;
    OCL_CHECK(pvb2_event_query(e, &done));
    return done != 0;
  }
  c10::DeviceIndex deviceCount() const noexcept override { return (c10::DeviceIndex)device_count(); }
  bool queryStream(const c10::Stream& s) const override {
    flush_deferred();
    int done = 0;
    OCL_CHECK(pvb2_stream_query(stream_by_id(s.device_index(), s.id()), &done));
    return done != 0;
  }
  void synchronizeStream(const c10::Stream& s) const override {
    flush_deferred();
    OCL_CHECK(pvb2_stream_synchronize(stream_by_id(s.device_index(), s.id())));
  }
  void synchronizeEvent(void* e) const override {
    if (e) OCL_CHECK(pvb2_event_synchronize(e));
  }
  void synchronizeDevice(const c10::DeviceIndex idx) const override {
    DeviceScope scope(idx < 0 ? current_device() : idx);
    OCL_CHECK(pvb2_device_synchronize());
  }
  void recordDataPtrOnStream(const c10::DataPtr& dp, const c10::Stream& s) const override {
    allocator_record_stream(dp, stream_by_id(s.device_index(), s.id()));
  }
  double elapsedTime(void* e1, void* e2, const c10::DeviceIndex) const override {
    float ms = 0;
    OCL_CHECK(pvb2_event_elapsed_ms(e1, e2, &ms));
    return ms;
  }
};

C10_REGISTER_GUARD_IMPL(PrivateUse1, OclGuardImpl);

// ================================================================ generator
// Philox state: (seed, offset).  Each random op reserves ceil(n/4) Philox
// counters, like get_random_seq in the reference (src/random_ops.cpp:26-34).
struct OclGenerator final : public c10::GeneratorImpl {
  explicit OclGenerator(c10::DeviceIndex idx)
      : c10::GeneratorImpl(c10::Device(kOcl, idx), c10::DispatchKeySet(c10::DispatchKey::PrivateUse1)) {}
  uint64_t seed_ = 67280421310721ull;
  uint64_t offset_ = 0;
  void set_current_seed(uint64_t s) override {
    seed_ = s;
    offset_ = 0;
  }
  void set_offset(uint64_t o) override { offset_ = o; }
  uint64_t get_offset() const override { return offset_; }
  uint64_t current_seed() const override { return seed_; }
  uint64_t seed() override {
    std::random_device rd;
    uint64_t s = ((uint64_t)rd() << 32) ^ rd();
    set_current_seed(s);
    return s;
  }
  void set_state(const c10::TensorImpl& st) override {
    TORCH_CHECK(st.numel() == 16 && st.dtype() == at::kByte, "ocl generator state must be 16 bytes");
    const uint8_t* p = static_cast<const uint8_t*>(st.data());
    memcpy(&seed_, p, 8);
    memcpy(&offset_, p + 8, 8);
  }
  c10::intrusive_ptr<c10::TensorImpl> get_state() const override {
    auto t = at::empty({16}, at::kByte);
    memcpy(t.data_ptr(), &seed_, 8);
    memcpy((uint8_t*)t.data_ptr() + 8, &offset_, 8);
    return t.getIntrusivePtr();
  }
  OclGenerator* clone_impl() const override {
    auto g = new OclGenerator(device().index());
    g->seed_ = seed_;
    g->offset_ = offset_;
    return g;
  }
  static c10::DeviceType device_type() { return kOcl; }
};

static std::vector<at::Generator>& default_generators() {
  static std::vector<at::Generator> g = [] {
    std::vector<at::Generator> v;
    for (int i = 0; i < std::max(device_count(), 1); ++i) v.push_back(at::make_generator<OclGenerator>((c10::DeviceIndex)i));
    return v;
  }();
  return g;
}

static at::Generator make_generator(c10::DeviceIndex idx) {
  return at::make_generator<OclGenerator>(idx < 0 ? (c10::DeviceIndex)current_device() : idx);
}

}  // namespace ocl

// exported for the random ops: reserve `n` values, return (seed, offset)
namespace ocl {
std::pair<uint64_t, uint64_t> philox_reserve(const std::optional<at::Generator>& gen, int device, int64_t n) {
  at::Generator g = gen.has_value() && gen->defined() ? *gen : default_generators().at(device);
  auto* impl = static_cast<OclGenerator*>(g.unsafeGetGeneratorImpl());
  std::lock_guard<std::mutex> lock(g.mutex());
  const uint64_t off = impl->offset_;
  impl->offset_ += (uint64_t)((n + 3) / 4);
  return {impl->seed_, off};
}
}  // namespace ocl

namespace ocl {
// ==================================================================== hooks
struct OclHooks final : public at::PrivateUse1HooksInterface {
  bool isBuilt() const override { return true; }
  bool isAvailable() const override { return device_count() > 0; }
  const at::Generator& getDefaultGenerator(c10::DeviceIndex idx) const override {
    const int d = idx < 0 ? current_device() : idx;
    return default_generators().at(d);
  }
  at::Generator getNewGenerator(c10::DeviceIndex idx) const override { return make_generator(idx); }
  at::Device getDeviceFromPtr(void* data) const override {
    int is_dev = 0, is_pinned = 0, dev = -1;
    pvb2_pointer_info(data, &is_dev, &is_pinned, &dev);
    return is_dev ? at::Device(kOcl, dev) : at::Device(at::kCPU);
  }
  bool isPinnedPtr(const void* data) const override {
    if (device_count() == 0) return false;
    int is_dev = 0, is_pinned = 0, dev = -1;
    pvb2_pointer_info(data, &is_dev, &is_pinned, &dev);
    return is_pinned != 0;
  }
  at::Allocator* getPinnedMemoryAllocator() const override { return &g_pinned; }
  bool hasPrimaryContext(c10::DeviceIndex idx) const override {
    return idx >= 0 && idx < device_count() && states()[idx].ready;
  }
  c10::DeviceIndex deviceCount() const override { return (c10::DeviceIndex)device_count(); }
  void setCurrentDevice(c10::DeviceIndex d) const override { set_device(d); }
  c10::DeviceIndex getCurrentDevice() const override { return (c10::DeviceIndex)current_device(); }
  c10::DeviceIndex exchangeDevice(c10::DeviceIndex d) const override {
    const int old = current_device();
    set_device(d);
    return (c10::DeviceIndex)old;
  }
  c10::DeviceIndex maybeExchangeDevice(c10::DeviceIndex d) const override { return exchangeDevice(d); }
  void resizePrivateUse1Bytes(const c10::Storage& storage, size_t newsize) const override {
    c10::StorageImpl* impl = storage.unsafeGetStorageImpl();
    const size_t old = impl->nbytes();
    if (newsize == old) return;
    DeviceScope scope(storage.device().index());
    c10::DataPtr fresh = g_allocator.allocate(newsize);
    const size_t keep = std::min(old, newsize);
    if (keep && impl->data()) OCL_CHECK(pvb2_memcpy_async(fresh.get(), impl->data(), keep, 2, current_stream()));
    impl->set_data_ptr_noswap(std::move(fresh));
    impl->set_nbytes(newsize);
  }
  void init() const override {}
};

static OclHooks g_hooks;
static bool register_hooks() {
  at::RegisterPrivateUse1HooksInterface(&g_hooks);
  return true;
}
static bool g_hooks_registered = register_hooks();

static void mark_bad_fork() { g_bad_fork = true; }
static bool register_fork() {
  pthread_atfork(nullptr, nullptr, &mark_bad_fork);
  return true;
}
static bool g_fork_registered = register_fork();

// ============================================================ python API
static void seed_all(uint64_t seed) {
  for (auto& g : default_generators()) {
    std::lock_guard<std::mutex> lock(g.mutex());
    g.set_current_seed(seed);
  }
}

static void synchronize_device(int index) {
  flush_deferred();
  if (index == -1) {
    for (int d = 0; d < device_count(); ++d) {
      if (!states()[d].ready) continue;
      DeviceScope scope(d);
      OCL_CHECK(pvb2_device_synchronize());
    }
    return;
  }
  check_index(index);
  DeviceScope scope(index);
  OCL_CHECK(pvb2_device_synchronize());
}

static pybind11::dict memory_stats(int d) {
  check_index(d);
  Pool& pool = pools()[d];
  std::lock_guard<std::mutex> g(pool.m);
  pybind11::dict r;
  r["allocated_bytes"] = pool.allocated;
  r["reserved_bytes"] = pool.reserved;
  r["peak_allocated_bytes"] = pool.peak_allocated;
  r["peak_reserved_bytes"] = pool.peak_reserved;
  r["num_device_mallocs"] = pool.n_malloc;
  r["num_cache_hits"] = pool.n_hits;
  return r;
}

static void reset_peak(int d) {
  check_index(d);
  Pool& pool = pools()[d];
  std::lock_guard<std::mutex> g(pool.m);
  pool.peak_allocated = pool.allocated;
  pool.peak_reserved = pool.reserved;
}

static uintptr_t stream_handle(int d) {
  flush_deferred();  // the caller may launch its own work on the stream
  return (uintptr_t)stream_for(d < 0 ? current_device() : d);
}

// event helpers used by timing code: create/record/elapsed on the current stream
static uintptr_t event_create(bool timing) {
  pvb2_event e = nullptr;
  OCL_CHECK(pvb2_event_create(&e, timing ? 1 : 0));
  return (uintptr_t)e;
}
static void event_record(uintptr_t e, int d) {
  DeviceScope scope(d);
  OCL_CHECK(pvb2_event_record((pvb2_event)e, stream_for(d)));
}
static double event_elapsed(uintptr_t a, uintptr_t b) {
  float ms = 0;
  OCL_CHECK(pvb2_event_synchronize((pvb2_event)b));
  OCL_CHECK(pvb2_event_elapsed_ms((pvb2_event)a, (pvb2_event)b, &ms));
  return ms;
}
static void event_destroy(uintptr_t e) { pvb2_event_destroy((pvb2_event)e); }

// ================================================================== graphs
// A training step (or any other sequence of this backend's ops on one
// stream) captured once and replayed with one launch: the host-side work of
// every op -- Python, the autograd engine, dispatch, planning, deferred
// fusion decisions -- runs once, at capture.  Memory allocated during the
// capture comes from the graph's own pool (CapturePool above).
struct HostGraph {
  pvb2_graph graph = nullptr;
  std::shared_ptr<CapturePool> pool;
  int device = 0;
};

// the pool's free blocks join the device's ordinary free lists; blocks still
// held by tensors follow when those are freed
static void retire_capture_pool(HostGraph* h) {
  Pool& pool = pools()[h->device];
  std::lock_guard<std::mutex> g(pool.m);
  for (auto& kv : h->pool->free_blocks)
    for (void* p : kv.second) pool.free_blocks[kv.first].push_back(p);
  h->pool->free_blocks.clear();
  h->pool->retired = true;
  if (pool.capturing == h->pool) pool.capturing.reset();
}

static uintptr_t graph_capture_begin(int d) {
  check_index(d);
  TORCH_CHECK(!g_no_cache, "ocl graphs: not available with the memory cache off (B200_NO_MEM_CACHE=1)");
  DeviceScope scope(d);  // launches any deferred work first: it precedes the capture
  dev_state(d);
  OCL_CHECK(pvb2_stream_synchronize(stream_for(d)));
  auto h = std::make_unique<HostGraph>();
  h->device = d;
  h->pool = std::make_shared<CapturePool>();
  Pool& pool = pools()[d];
  {
    std::lock_guard<std::mutex> g(pool.m);
    TORCH_CHECK(!pool.capturing, "ocl graphs: a capture is already in progress on device ", d);
    process_pending(pool);  // event queries may not run once the capture has begun
    pool.capturing = h->pool;
  }
  const int s = pvb2_graph_capture_begin(stream_for(d));
  if (s != PVB2_OK) {
    const std::string msg = pvb2_last_error();
    retire_capture_pool(h.get());
    TORCH_CHECK(false, "ocl graphs: ", msg);
  }
  return reinterpret_cast<uintptr_t>(h.release());
}

static void graph_capture_end(uintptr_t handle) {
  HostGraph* h = reinterpret_cast<HostGraph*>(handle);
  TORCH_CHECK(h && !h->graph, "ocl graphs: no capture in progress for this handle");
  pvb2_graph g = nullptr;
  int s;
  std::string msg;
  {
    DeviceScope scope(h->device, /*flush=*/false);
    // deferred work belongs to the capture; if launching it fails (a capture
    // already invalidated), the capture is still ended and the pool cleared
    try {
      flush_deferred();
    } catch (const std::exception& e) {
      msg = e.what();
    }
    s = pvb2_graph_capture_end(stream_for(h->device), &g);
  }
  if (s != PVB2_OK) msg = std::string(pvb2_last_error()) + (msg.empty() ? "" : "; " + msg);
  if (s == PVB2_OK && !msg.empty()) {  // captured, but without the deferred work
    pvb2_graph_destroy(g);
    s = PVB2_ERR_CUDA;
  }
  {
    Pool& pool = pools()[h->device];
    std::lock_guard<std::mutex> lk(pool.m);
    pool.capturing.reset();
  }
  if (s != PVB2_OK) {
    retire_capture_pool(h);  // a failed capture ran nothing on the device
    TORCH_CHECK(false, "ocl graphs: ", msg);
  }
  h->graph = g;
}

static void graph_replay(uintptr_t handle) {
  HostGraph* h = reinterpret_cast<HostGraph*>(handle);
  TORCH_CHECK(h && h->graph, "ocl graphs: replay of a graph that was not captured");
  DeviceScope scope(h->device);
  OCL_CHECK(pvb2_graph_launch(h->graph, stream_for(h->device)));
}

static int64_t graph_kernels(uintptr_t handle) {
  HostGraph* h = reinterpret_cast<HostGraph*>(handle);
  TORCH_CHECK(h && h->graph, "ocl graphs: not a captured graph");
  int64_t n = 0;
  OCL_CHECK(pvb2_graph_kernel_count(h->graph, &n));
  return n;
}

// after every replay has finished (device synchronisation), the graph and
// its pool are released
static void graph_destroy(uintptr_t handle) {
  HostGraph* h = reinterpret_cast<HostGraph*>(handle);
  if (!h) return;
  {
    DeviceScope scope(h->device);
    OCL_CHECK(pvb2_device_synchronize());
    if (h->graph) OCL_CHECK(pvb2_graph_destroy(h->graph));
    h->graph = nullptr;
  }
  retire_capture_pool(h);
  delete h;
}

}  // namespace ocl

// defined in ops_dist.cpp
void register_dist_bindings(pybind11::module& m);

PYBIND11_MODULE(_C, m) {
  using namespace ocl;
  m.def("impl_custom_device", [](int id) { return c10::Device(kOcl, id); }, "device object for index id");
  m.def("impl_seed_all", &seed_all, "seed the Philox generator of every device");
  m.def("impl_synchronize_device", &synchronize_device, "wait for device work (-1 = all devices)");
  m.def("impl_is_bad_fork", []() { return g_bad_fork.load(); });
  m.def("impl_empty_cache", &empty_cache_all, "release cached device blocks");
  m.def("impl_staged_input_bytes", &staged_input_bytes, "bytes of convolution inputs kept for the weight gradient");
  m.def("impl_enable_profiling", &enable_profiling);
  m.def("impl_start_profiling", &start_profiling);
  m.def("impl_stop_profiling", &stop_profiling);
  m.def("impl_device_count", &device_count);
  m.def("impl_current_device", &current_device);
  m.def("impl_set_device", &set_device);
  m.def("impl_device_name", [](int d) {
    char buf[256] = {0};
    OCL_CHECK(pvb2_device_name(d, buf, sizeof(buf)));
    return std::string(buf);
  });
  m.def("impl_memory_stats", &memory_stats);
  m.def("impl_reset_peak_memory_stats", &reset_peak);
  m.def("impl_set_math_mode", &set_math_mode);
  m.def("impl_get_math_mode", &math_mode);
  m.def("impl_set_debug_mode", [](int v) { g_trace_mode = v; });
  m.def("impl_launch_count", []() { return (int64_t)pvb2_launch_count(); });
  m.def("impl_stream_handle", &stream_handle);
  m.def("impl_event_create", &event_create);
  m.def("impl_event_record", &event_record);
  m.def("impl_event_elapsed_ms", &event_elapsed);
  m.def("impl_event_destroy", &event_destroy);
  m.def("impl_graph_capture_begin", &graph_capture_begin, "begin capturing device d's current stream");
  m.def("impl_graph_capture_end", &graph_capture_end, "end the capture and instantiate the graph");
  m.def("impl_graph_replay", &graph_replay, "replay a captured graph on its device's current stream");
  m.def("impl_graph_kernels", &graph_kernels, "kernels launched by one replay");
  m.def("impl_graph_destroy", &graph_destroy, "release a graph and its memory pool");
  register_dist_bindings(m);
}
