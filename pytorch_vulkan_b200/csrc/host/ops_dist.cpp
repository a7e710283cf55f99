// Python bindings for data-parallel training on `ocl` devices: NCCL
// communicators driven on the backend's own streams, stream / event helpers
// for overlapping the gradient exchange with the backward pass, and the
// multi-tensor bucket flatten.  The reference has no multi-device code; the
// host-side rendezvous (unique-id exchange, barriers) stays in
// torch.distributed (gloo) and only the data path runs here.
#include <torch/extension.h>

#include "ocl.h"

namespace ocl {

static pvb2_stream stream_of(int dev, int64_t id) {
  // resolve through the guard so user-created streams work too
  c10::Stream s(c10::Stream::UNSAFE, c10::Device(kOcl, dev), id);
  return (pvb2_stream)c10::impl::getDeviceGuardImpl(kOcl)->getStreamNativeHandle(s);
}

static pybind11::bytes nccl_unique_id() {
  uint8_t id[PVB2_NCCL_ID_BYTES];
  OCL_CHECK(pvb2_nccl_get_unique_id(id));
  return pybind11::bytes(reinterpret_cast<const char*>(id), PVB2_NCCL_ID_BYTES);
}

static uintptr_t nccl_init(int nranks, const std::string& id, int rank, int dev) {
  TORCH_CHECK(id.size() == PVB2_NCCL_ID_BYTES, "nccl unique id must be ", PVB2_NCCL_ID_BYTES, " bytes");
  DeviceScope scope(dev);
  void* comm = nullptr;
  OCL_CHECK(pvb2_nccl_comm_init(&comm, nranks, reinterpret_cast<const uint8_t*>(id.data()), rank));
  return (uintptr_t)comm;
}

// in-place all-reduce of a contiguous tensor on stream `stream_id` of its device
static void nccl_allreduce(uintptr_t comm, const at::Tensor& t, int op, int64_t stream_id) {
  TORCH_CHECK(is_ocl(t) && t.is_contiguous(), "nccl_allreduce: contiguous ocl tensor expected");
  const int dev = t.device().index();
  DeviceScope scope(dev);
  OCL_OP("nccl_allreduce", dev);
  OCL_CHECK(pvb2_nccl_allreduce((void*)comm, t.data_ptr(), t.data_ptr(), (size_t)t.numel(), dtype_code(t.scalar_type()),
                                op, stream_of(dev, stream_id)));
}

static void nccl_broadcast(uintptr_t comm, const at::Tensor& t, int root, int64_t stream_id) {
  TORCH_CHECK(is_ocl(t) && t.is_contiguous(), "nccl_broadcast: contiguous ocl tensor expected");
  const int dev = t.device().index();
  DeviceScope scope(dev);
  OCL_CHECK(pvb2_nccl_broadcast((void*)comm, t.data_ptr(), (size_t)t.numel(), dtype_code(t.scalar_type()), root,
                                stream_of(dev, stream_id)));
}

static void nccl_destroy(uintptr_t comm) { OCL_CHECK(pvb2_nccl_comm_destroy((void*)comm)); }
static void nccl_abort(uintptr_t comm) { OCL_CHECK(pvb2_nccl_comm_abort((void*)comm)); }

// streams by id (0 = the device's backend stream)
static int64_t new_stream(int dev, int priority) {
  return c10::impl::getDeviceGuardImpl(kOcl)->getNewStream(c10::Device(kOcl, dev), priority).id();
}
static int64_t get_stream(int dev) {
  return c10::impl::getDeviceGuardImpl(kOcl)->getStream(c10::Device(kOcl, dev)).id();
}
static void set_stream(int dev, int64_t id) {
  c10::impl::getDeviceGuardImpl(kOcl)->exchangeStream(c10::Stream(c10::Stream::UNSAFE, c10::Device(kOcl, dev), id));
}
// make `waiter` wait for all work queued so far on `waitee`
static void stream_wait_stream(int dev, int64_t waiter, int64_t waitee) {
  DeviceScope scope(dev);
  pvb2_event e = nullptr;
  OCL_CHECK(pvb2_event_create(&e, 0));
  OCL_CHECK(pvb2_event_record(e, stream_of(dev, waitee)));
  OCL_CHECK(pvb2_stream_wait_event(stream_of(dev, waiter), e));
  OCL_CHECK(pvb2_event_destroy(e));  // destruction is deferred by CUDA until the wait resolves
}
static void stream_synchronize(int dev, int64_t id) { OCL_CHECK(pvb2_stream_synchronize(stream_of(dev, id))); }
// record a (timing) event of impl_event_create on stream `id` of device `dev`
static void event_record_stream(uintptr_t e, int dev, int64_t id) {
  DeviceScope scope(dev);
  OCL_CHECK(pvb2_event_record((pvb2_event)e, stream_of(dev, id)));
}
static void record_stream(const at::Tensor& t, int64_t id) {
  allocator_record_stream(t.storage().data_ptr(), stream_of(t.device().index(), id));
}

// flat <- tensors (direction 0) or tensors <- flat (direction 1), scaled
static void flatten_multi(const std::vector<at::Tensor>& ts, const at::Tensor& flat, int direction, double scale) {
  if (ts.empty()) return;
  const int dev = flat.device().index();
  DeviceScope scope(dev);
  OCL_OP("bucket_flatten", dev);
  TORCH_CHECK(flat.is_contiguous() && flat.scalar_type() == at::kFloat, "flatten: flat buffer must be contiguous fp32");
  std::vector<float*> p(ts.size());
  std::vector<int64_t> n(ts.size());
  int64_t total = 0;
  for (size_t i = 0; i < ts.size(); ++i) {
    TORCH_CHECK(is_ocl(ts[i]) && ts[i].is_contiguous() && ts[i].scalar_type() == at::kFloat,
                "flatten: contiguous fp32 ocl tensors expected");
    p[i] = ts[i].numel() ? ts[i].data_ptr<float>() : nullptr;
    n[i] = ts[i].numel();
    total += n[i];
  }
  TORCH_CHECK(total <= flat.numel(), "flatten: flat buffer too small");
  OCL_CHECK(pvb2_flatten_multi((int)ts.size(), p.data(), n.data(), flat.data_ptr<float>(), direction, scale,
                               stream_for(dev)));
}

}  // namespace ocl

void register_dist_bindings(pybind11::module& m) {
  using namespace ocl;
  m.def("impl_nccl_unique_id", &nccl_unique_id);
  m.def("impl_nccl_init", &nccl_init);
  m.def("impl_nccl_allreduce", &nccl_allreduce);
  m.def("impl_nccl_broadcast", &nccl_broadcast);
  m.def("impl_nccl_destroy", &nccl_destroy);
  m.def("impl_nccl_abort", &nccl_abort);
  m.def("impl_new_stream", &new_stream);
  m.def("impl_get_stream", &get_stream);
  m.def("impl_set_stream", &set_stream);
  m.def("impl_stream_wait_stream", &stream_wait_stream);
  m.def("impl_stream_synchronize", &stream_synchronize);
  m.def("impl_event_record_stream", &event_record_stream);
  m.def("impl_record_stream", &record_stream);
  m.def("impl_flatten_multi", &flatten_multi);
}
