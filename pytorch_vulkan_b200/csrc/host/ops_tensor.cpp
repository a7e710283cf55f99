// Tensor plumbing for the `ocl` device: factories, views, copies between
// host and device, fill, scalar read-back, resize and set_.
// Mirrors the registrations of src/tensor_ops.cpp:433-452 (the reference's
// boxed CPU fallback, tensor_ops.cpp:423-429,454-456, is deliberately not
// provided: an op without a device kernel raises).
#include <ATen/EmptyTensor.h>
#include <ATen/native/Resize.h>
#include <ATen/native/TensorFactories.h>
#include <ATen/ops/as_strided_native.h>
#include <ATen/ops/view_native.h>
#include <ATen/ops/_reshape_alias_native.h>
#include <c10/core/CPUAllocator.h>

#include "ocl.h"

namespace ocl {

int dtype_code(c10::ScalarType t) {
  switch (t) {
    case at::kFloat: return PVB2_F32;
    case at::kDouble: return PVB2_F64;
    case at::kHalf: return PVB2_F16;
    case at::kBFloat16: return PVB2_BF16;
    case at::kLong: return PVB2_I64;
    case at::kInt: return PVB2_I32;
    case at::kShort: return PVB2_I16;
    case at::kChar: return PVB2_I8;
    case at::kByte: return PVB2_U8;
    case at::kBool: return PVB2_BOOL;
    default: TORCH_CHECK(false, "ocl: unsupported dtype ", t);
  }
}

int compute_code(c10::ScalarType t) {
  switch (t) {
    case at::kFloat:
    case at::kHalf:
    case at::kBFloat16: return PVB2_F32;
    case at::kDouble: return PVB2_F64;
    case at::kBool: return PVB2_BOOL;
    default: return PVB2_I64;
  }
}

pvb2_tensor desc(const at::Tensor& t) {
  pvb2_tensor d;
  memset(&d, 0, sizeof(d));
  TORCH_CHECK(t.dim() <= PVB2_MAX_DIMS, "ocl: tensors with more than ", PVB2_MAX_DIMS, " dims are not supported");
  d.data = t.numel() ? t.data_ptr() : nullptr;
  d.ndim = (int32_t)t.dim();
  d.dtype = dtype_code(t.scalar_type());
  for (int i = 0; i < t.dim(); ++i) {
    d.sizes[i] = t.size(i);
    d.strides[i] = t.stride(i);
  }
  return d;
}

pvb2_tensor desc_expanded(const at::Tensor& t, c10::IntArrayRef sizes) {
  if (t.sizes().equals(sizes)) return desc(t);
  // broadcast without building a view: align trailing dims, stride 0 where t has size 1
  const int64_t nd = (int64_t)sizes.size(), td = t.dim();
  TORCH_CHECK(td <= nd && nd <= PVB2_MAX_DIMS, "ocl: cannot broadcast ", t.sizes(), " to ", sizes);
  pvb2_tensor d;
  memset(&d, 0, sizeof(d));
  d.data = t.numel() ? t.data_ptr() : nullptr;
  d.ndim = (int32_t)nd;
  d.dtype = dtype_code(t.scalar_type());
  for (int64_t i = 0; i < nd; ++i) {
    const int64_t j = i - (nd - td);
    d.sizes[i] = sizes[i];
    if (j < 0) {
      d.strides[i] = 0;
    } else {
      TORCH_CHECK(t.size(j) == sizes[i] || t.size(j) == 1, "ocl: cannot broadcast ", t.sizes(), " to ", sizes);
      d.strides[i] = t.size(j) == sizes[i] ? t.stride(j) : 0;
    }
  }
  return d;
}

at::Tensor empty(c10::IntArrayRef sizes, c10::ScalarType dtype, int device, c10::MemoryFormat mf) {
  DeviceScope scope(device, /*flush=*/false);
  c10::DispatchKeySet ks(c10::DispatchKey::PrivateUse1);
  return at::detail::empty_generic(sizes, allocator(), ks, dtype, mf);
}

at::Tensor empty_like_dev(const at::Tensor& t) { return empty(t.sizes(), t.scalar_type(), t.device().index()); }

at::Tensor empty_strided_dev(c10::IntArrayRef sizes, c10::IntArrayRef strides, c10::ScalarType dtype, int device) {
  DeviceScope scope(device, /*flush=*/false);
  c10::DispatchKeySet ks(c10::DispatchKey::PrivateUse1);
  return at::detail::empty_strided_generic(sizes, strides, allocator(), ks, dtype);
}

at::Tensor contiguous(const at::Tensor& t) {
  if (t.is_contiguous()) return t;
  at::Tensor out = empty(t.sizes(), t.scalar_type(), t.device().index());
  pvb2_tensor d = desc(out), s = desc(t);
  OCL_CHECK(pvb2_copy(&d, &s, stream_for(t.device().index())));
  return out;
}

at::Tensor& write_back(at::Tensor& out, const at::Tensor& tmp) {
  if (out.is_same(tmp)) return out;
  pvb2_tensor d = desc(out), s = desc(tmp);
  OCL_CHECK(pvb2_copy(&d, &s, stream_for(out.device().index())));
  return out;
}

// ------------------------------------------------------------- factories
// empty.memory_format, tensor_ops.cpp:23-37
static at::Tensor empty_memory_format(c10::IntArrayRef size, std::optional<at::ScalarType> dtype,
                                      std::optional<at::Layout> layout, std::optional<at::Device> device,
                                      std::optional<bool> pin_memory, std::optional<at::MemoryFormat> memory_format) {
  const int d = device.has_value() && device->index() >= 0 ? device->index() : current_device();
  return empty(size, dtype.value_or(at::get_default_dtype_as_scalartype()), d,
               memory_format.value_or(at::MemoryFormat::Contiguous));
}

// empty_strided, tensor_ops.cpp:49-54
static at::Tensor empty_strided(c10::IntArrayRef size, c10::IntArrayRef stride, std::optional<at::ScalarType> dtype,
                                std::optional<at::Layout> layout, std::optional<at::Device> device,
                                std::optional<bool> pin_memory) {
  const int d = device.has_value() && device->index() >= 0 ? device->index() : current_device();
  return empty_strided_dev(size, stride, dtype.value_or(at::get_default_dtype_as_scalartype()), d);
}

// ------------------------------------------------------------------- views
static at::Tensor as_strided(const at::Tensor& self, c10::IntArrayRef size, c10::IntArrayRef stride,
                             std::optional<int64_t> storage_offset) {
  return at::native::as_strided_tensorimpl(self, size, stride, storage_offset);
}
static at::Tensor view(const at::Tensor& self, c10::IntArrayRef size) { return at::native::view(self, size); }
static at::Tensor reshape_alias(const at::Tensor& self, c10::IntArrayRef size, c10::IntArrayRef stride) {
  return at::native::_reshape_alias(self, size, stride);
}

// -------------------------------------------------------------------- copy
// _copy_from, tensor_ops.cpp:118-186: host<->device and device<->device,
// any strides, any dtypes (conversion runs on the device).
static void h2d(const at::Tensor& dst, const at::Tensor& src_cpu, bool non_blocking) {
  const int dev = dst.device().index();
  DeviceScope scope(dev);
  OCL_OP("copy_h2d", dev);
  at::Tensor s = src_cpu.is_contiguous() ? src_cpu : src_cpu.contiguous();
  pvb2_stream st = stream_for(dev);
  if (s.scalar_type() == dst.scalar_type() && dst.is_contiguous()) {
    OCL_CHECK(pvb2_memcpy_async(dst.data_ptr(), s.data_ptr(), s.nbytes(), 0, st));
    if (!non_blocking || !s.is_pinned()) OCL_CHECK(pvb2_stream_synchronize(st));
    return;
  }
  at::Tensor tmp = empty(s.sizes(), s.scalar_type(), dev);
  OCL_CHECK(pvb2_memcpy_async(tmp.data_ptr(), s.data_ptr(), s.nbytes(), 0, st));
  pvb2_tensor d = desc(dst), t = desc(tmp);
  OCL_CHECK(pvb2_copy(&d, &t, st));
  if (!non_blocking || !s.is_pinned()) OCL_CHECK(pvb2_stream_synchronize(st));
}

static void d2h(const at::Tensor& dst_cpu, const at::Tensor& src, bool non_blocking) {
  const int dev = src.device().index();
  DeviceScope scope(dev);
  OCL_OP("copy_d2h", dev);
  pvb2_stream st = stream_for(dev);
  at::Tensor s = src;
  if (s.scalar_type() != dst_cpu.scalar_type() || !s.is_contiguous()) {
    at::Tensor tmp = empty(s.sizes(), dst_cpu.scalar_type(), dev);
    pvb2_tensor d = desc(tmp), t = desc(s);
    OCL_CHECK(pvb2_copy(&d, &t, st));
    s = tmp;
  }
  if (dst_cpu.is_contiguous()) {
    OCL_CHECK(pvb2_memcpy_async(dst_cpu.data_ptr(), s.data_ptr(), s.nbytes(), 1, st));
    if (!non_blocking || !dst_cpu.is_pinned()) OCL_CHECK(pvb2_stream_synchronize(st));
    return;
  }
  at::Tensor host = at::empty(s.sizes(), dst_cpu.options().memory_format(at::MemoryFormat::Contiguous));
  OCL_CHECK(pvb2_memcpy_async(host.data_ptr(), s.data_ptr(), s.nbytes(), 1, st));
  OCL_CHECK(pvb2_stream_synchronize(st));
  dst_cpu.copy_(host);
}

void copy_into(const at::Tensor& dst, const at::Tensor& src, bool non_blocking) {
  if (dst.numel() == 0) return;
  const bool src_dev = is_ocl(src), dst_dev = is_ocl(dst);
  if (dst_dev && src.device().is_cpu()) {
    h2d(dst, src, non_blocking);
  } else if (src_dev && dst.device().is_cpu()) {
    d2h(dst, src, non_blocking);
  } else if (src_dev && dst_dev) {
    const int dd = dst.device().index(), sd = src.device().index();
    if (dd == sd) {
      if (fuse_deferred_copy(dst, src)) return;  // joined a pending batch-norm pass
      DeviceScope scope(dd);
      OCL_OP("copy_d2d", dd);
      pvb2_tensor d = desc(dst), s = desc(src);
      OCL_CHECK(pvb2_copy(&d, &s, stream_for(dd)));
    } else {
      // different devices: make the source contiguous on its device, move the
      // bytes with a peer copy, then lay them out on the destination device
      at::Tensor sc;
      {
        DeviceScope scope(sd);
        sc = contiguous(src);
        OCL_CHECK(pvb2_stream_synchronize(stream_for(sd)));
      }
      DeviceScope scope(dd);
      OCL_OP("copy_p2p", dd);
      at::Tensor tmp = empty(sc.sizes(), sc.scalar_type(), dd);
      OCL_CHECK(pvb2_memcpy_async(tmp.data_ptr(), sc.data_ptr(), sc.nbytes(), 3, stream_for(dd)));
      pvb2_tensor d = desc(dst), s = desc(tmp);
      OCL_CHECK(pvb2_copy(&d, &s, stream_for(dd)));
      OCL_CHECK(pvb2_stream_synchronize(stream_for(dd)));
    }
  } else {
    TORCH_CHECK(false, "ocl: copy between ", src.device(), " and ", dst.device(), " is not supported");
  }
}

static at::Tensor copy_from(const at::Tensor& self, const at::Tensor& dst, bool non_blocking) {
  TORCH_CHECK(self.sizes().equals(dst.sizes()) || self.numel() == dst.numel() || self.dim() == 0,
              "ocl: _copy_from size mismatch ", self.sizes(), " vs ", dst.sizes());
  if (self.sizes().equals(dst.sizes())) {
    copy_into(dst, self, non_blocking);
  } else {
    // broadcast copy (dst.copy_(scalar-like src))
    at::Tensor s = self;
    if (is_ocl(self)) {
      s = self.expand(dst.sizes());
      copy_into(dst, s, non_blocking);
    } else {
      copy_into(dst, self.expand(dst.sizes()).contiguous(), non_blocking);
    }
  }
  return dst;
}

static at::Tensor copy_from_and_resize(const at::Tensor& self, const at::Tensor& dst) {
  if (!dst.sizes().equals(self.sizes())) dst.resize_(self.sizes());
  copy_into(dst, self, false);
  return dst;
}

// ------------------------------------------------------------------- fill
// fill_ / zero_, tensor_ops.cpp:204-225
static at::Tensor& fill_scalar(at::Tensor& self, const at::Scalar& value) {
  if (self.numel() == 0) return self;
  const int dev = self.device().index();
  DeviceScope scope(dev);
  OCL_OP("fill_", dev);
  pvb2_tensor d = desc(self);
  double v = value.isBoolean() ? (value.toBool() ? 1.0 : 0.0) : value.toDouble();
  OCL_CHECK(pvb2_fill(&d, v, stream_for(dev)));
  return self;
}

static at::Tensor& fill_tensor(at::Tensor& self, const at::Tensor& value) {
  TORCH_CHECK(value.dim() == 0, "fill_ only supports 0-dimension value tensor");
  if (!is_ocl(value)) return fill_scalar(self, value.item());
  if (self.numel() == 0) return self;
  const int dev = self.device().index();
  DeviceScope scope(dev);
  OCL_OP("fill_", dev);
  pvb2_tensor d = desc(self), s = desc(value.expand(self.sizes()));
  OCL_CHECK(pvb2_copy(&d, &s, stream_for(dev)));
  return self;
}

static at::Tensor& zero_(at::Tensor& self) { return fill_scalar(self, 0); }

// _local_scalar_dense, tensor_ops.cpp:239-272: one element back to the host
static at::Scalar local_scalar_dense(const at::Tensor& self) {
  const int dev = self.device().index();
  DeviceScope scope(dev);
  OCL_OP("_local_scalar_dense", dev);
  at::Tensor host = at::empty({}, self.options().device(at::kCPU));
  pvb2_stream st = stream_for(dev);
  OCL_CHECK(pvb2_memcpy_async(host.data_ptr(), self.data_ptr(), self.element_size(), 1, st));
  OCL_CHECK(pvb2_stream_synchronize(st));
  return host.item();
}

// ------------------------------------------------------------ resize / set
// resize_, tensor_ops.cpp:382-420
static const at::Tensor& resize_(const at::Tensor& self, c10::IntArrayRef size,
                                 std::optional<at::MemoryFormat> memory_format) {
  auto* impl = self.unsafeGetTensorImpl();
  impl->set_sizes_contiguous(size);
  const int64_t numel = impl->numel();
  const size_t need = (size_t)(impl->storage_offset() + numel) * self.element_size();
  if (numel > 0 && need > impl->storage().nbytes()) {
    at::detail::getPrivateUse1Hooks().resizePrivateUse1Bytes(impl->storage(), need);
  }
  if (memory_format.has_value() && *memory_format != at::MemoryFormat::Preserve)
    impl->empty_tensor_restride(*memory_format);
  return self;
}

static void set_sizes_strides(at::Tensor& self, int64_t offset, c10::IntArrayRef size, c10::IntArrayRef stride) {
  auto* impl = self.unsafeGetTensorImpl();
  if (stride.data() == nullptr || stride.empty() && !size.empty()) impl->set_sizes_contiguous(size);
  else impl->set_sizes_and_strides(size, stride);
  impl->set_storage_offset(offset);
  int64_t extent = 1;
  bool empty_t = false;
  for (size_t i = 0; i < size.size(); ++i) {
    if (size[i] == 0) empty_t = true;
    extent += (size[i] - 1) * self.stride(i);
  }
  if (!empty_t) {
    const size_t need = (size_t)(offset + extent) * self.element_size();
    if (need > impl->storage().nbytes())
      at::detail::getPrivateUse1Hooks().resizePrivateUse1Bytes(impl->storage(), need);
  }
}

static at::Tensor& set_storage_offset(at::Tensor& self, c10::Storage source, int64_t storage_offset,
                                      c10::IntArrayRef size, c10::IntArrayRef stride) {
  self.unsafeGetTensorImpl()->set_storage_keep_dtype(std::move(source));
  set_sizes_strides(self, storage_offset, size, stride);
  return self;
}

static at::Tensor& set_storage(at::Tensor& self, c10::Storage source) {
  const int64_t n = (int64_t)(source.nbytes() / self.element_size());
  std::vector<int64_t> size{n}, stride{1};
  return set_storage_offset(self, std::move(source), 0, size, stride);
}

static at::Tensor& set_tensor(at::Tensor& self, const at::Tensor& src) {
  if (self.is_same(src)) return self;
  return set_storage_offset(self, src.storage(), src.storage_offset(), src.sizes(), src.strides());
}

static at::Tensor& set_empty(at::Tensor& self) {
  c10::Storage st(c10::Storage::use_byte_size_t(), 0, allocator(), true);
  self.unsafeGetTensorImpl()->set_storage_keep_dtype(std::move(st));
  self.unsafeGetTensorImpl()->set_sizes_contiguous({0});
  return self;
}

}  // namespace ocl

TORCH_LIBRARY_IMPL(aten, PrivateUse1, m) {
  m.impl("empty.memory_format", &ocl::empty_memory_format);
  m.impl("empty_strided", &ocl::empty_strided);
  m.impl("as_strided", &ocl::as_strided);
  m.impl("view", &ocl::view);
  m.impl("_reshape_alias", &ocl::reshape_alias);
  m.impl("_copy_from", &ocl::copy_from);
  m.impl("_copy_from_and_resize", &ocl::copy_from_and_resize);
  m.impl("fill_.Scalar", &ocl::fill_scalar);
  m.impl("fill_.Tensor", &ocl::fill_tensor);
  m.impl("zero_", &ocl::zero_);
  m.impl("_local_scalar_dense", &ocl::local_scalar_dense);
  m.impl("resize_", &ocl::resize_);
  m.impl("set_.source_Storage", &ocl::set_storage);
  m.impl("set_.source_Storage_storage_offset", &ocl::set_storage_offset);
  m.impl("set_.source_Tensor", &ocl::set_tensor);
  m.impl("set_", &ocl::set_empty);
}
