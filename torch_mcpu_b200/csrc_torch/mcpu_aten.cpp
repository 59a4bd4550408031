// Dispatcher registrations of the mcpu (PrivateUse1) device on B200.
//
// The minimal tensor set of the reference (csrc/aten/OpenRegMinimal.cpp:
// 150-167) plus the hot-path aten ops (mm/addmm: csrc/aten/ops/mm.cpp:115-120;
// sigmoid/silu: unary_out.cpp:817-836; add/sub/mul/div: binary_out.cpp:
// 757-828; sum/mean/max/min: reduction_scatter.cpp:557-578; topk:
// topk.cpp:43-45; _softmax: softmax_random_argmax.cpp:140-144; gather,
// scatter, masked_fill, pow, rsqrt, bitwise_not), which let the reference's
// router function and vLLM's native ops run op by op on mcpu tensors, and the
// mcpu:: custom ops of the router / MLP path.  Every op enqueues on the
// current mcpu stream and returns, as the reference's ops do.
#include <ATen/ATen.h>
#include <ATen/EmptyTensor.h>
#include <ATen/native/Resize.h>
#include <ATen/ops/_reshape_alias_native.h>
#include <ATen/ops/as_strided_native.h>
#include <ATen/ops/view_native.h>
#include <c10/core/ScalarType.h>
#include <torch/library.h>

#include <algorithm>
#include <cstring>
#include <vector>

#include "mcpu_torch.h"

namespace mcpu_torch {
namespace {

#define MCPU_OK(expr, what)                                                          \
  do {                                                                               \
    orError_t _e = (expr);                                                           \
    TORCH_CHECK(_e == orSuccess, what, " failed: ", mcpuGetLastErrorString());       \
  } while (0)

const c10::DispatchKeySet kKeys(c10::DispatchKey::PrivateUse1);

int dtype_code(at::ScalarType t) {
  switch (t) {
    case at::kFloat: return MCPU_FLOAT32;
    case at::kBFloat16: return MCPU_BFLOAT16;
    case at::kHalf: return MCPU_FLOAT16;
    case at::kInt: return MCPU_INT32;
    case at::kLong: return MCPU_INT64;
    case at::kByte: return MCPU_UINT8;
    case at::kBool: return MCPU_BOOL;
    case at::kDouble: return MCPU_FLOAT64;
    case at::kChar: return MCPU_INT8;
    case at::kShort: return MCPU_INT16;
    default: TORCH_CHECK(false, "mcpu: unsupported dtype ", t);
  }
}

bool is_mcpu(const at::Tensor& t) { return t.device().type() == c10::DeviceType::PrivateUse1; }

orStream_t stream_of(const at::Tensor& t) { return current_stream_handle(t.device().index()); }

// ---------------------------------------------------------------- creation / views
at::Tensor empty_memory_format(c10::IntArrayRef size, std::optional<at::ScalarType> dtype,
                               std::optional<at::Layout> layout, std::optional<at::Device> device,
                               std::optional<bool> pin_memory,
                               std::optional<at::MemoryFormat> memory_format) {
  const auto dev = device.value_or(at::Device(c10::DeviceType::PrivateUse1, current_device()));
  TORCH_CHECK(!layout || *layout == at::kStrided, "mcpu: only strided tensors");
  const int prev = current_device();
  if (dev.has_index() && dev.index() != prev) orSetDevice(dev.index());
  auto t = at::detail::empty_generic(size, allocator(), kKeys, c10::dtype_or_default(dtype),
                                     memory_format);
  if (dev.has_index() && dev.index() != prev) orSetDevice(prev);
  return t;
}

at::Tensor empty_strided(c10::IntArrayRef size, c10::IntArrayRef stride,
                         std::optional<at::ScalarType> dtype, std::optional<at::Layout> layout,
                         std::optional<at::Device> device, std::optional<bool> pin_memory) {
  const auto dev = device.value_or(at::Device(c10::DeviceType::PrivateUse1, current_device()));
  const int prev = current_device();
  if (dev.has_index() && dev.index() != prev) orSetDevice(dev.index());
  auto t = at::detail::empty_strided_generic(size, stride, allocator(), kKeys,
                                             c10::dtype_or_default(dtype));
  if (dev.has_index() && dev.index() != prev) orSetDevice(prev);
  return t;
}

const at::Tensor& resize_(const at::Tensor& self, c10::IntArrayRef size,
                          std::optional<at::MemoryFormat> memory_format) {
  int64_t numel = 1;
  for (auto s : size) numel *= s;
  const int64_t need = (self.storage_offset() + numel) * static_cast<int64_t>(self.itemsize());
  if (need > static_cast<int64_t>(self.storage().nbytes())) {
    // grow the storage: new block, old bytes copied on the current stream;
    // the old block goes back to the stream-ordered allocator after the copy
    c10::StorageImpl* st = self.storage().unsafeGetStorageImpl();
    TORCH_CHECK(st->resizable(), "mcpu resize_: the tensor's storage is not resizable");
    c10::DataPtr fresh = allocator()->allocate(static_cast<size_t>(need));
    const size_t old = st->nbytes();
    if (old > 0)
      MCPU_OK(orMemcpyAsync(fresh.get(), st->data(), old, orMemcpyDeviceToDevice, stream_of(self)),
              "resize_ copy");
    st->set_data_ptr_noswap(std::move(fresh));
    st->set_nbytes(static_cast<size_t>(need));
  }
  self.unsafeGetTensorImpl()->set_sizes_contiguous(size);
  return self;
}

// ---------------------------------------------------------------- copies
void strided_copy(const at::Tensor& src, const at::Tensor& dst) {
  TORCH_CHECK(src.dim() <= 8, "mcpu copy: at most 8 dimensions");
  std::vector<int64_t> sizes(dst.sizes().begin(), dst.sizes().end());
  std::vector<int64_t> ss(src.strides().begin(), src.strides().end());
  std::vector<int64_t> ds(dst.strides().begin(), dst.strides().end());
  MCPU_OK(mcpu_copy_strided(src.const_data_ptr(), dtype_code(src.scalar_type()), dst.data_ptr(),
                            dtype_code(dst.scalar_type()), static_cast<int>(sizes.size()),
                            sizes.data(), ss.data(), ds.data(), stream_of(dst)),
          "mcpu copy");
}

bool same_dense(const at::Tensor& a, const at::Tensor& b) {
  return a.scalar_type() == b.scalar_type() && a.is_contiguous() && b.is_contiguous() &&
         a.sizes() == b.sizes();
}

at::Tensor copy_from(const at::Tensor& self, const at::Tensor& dst, bool non_blocking) {
  at::Tensor src = self;
  if (src.sizes() != dst.sizes()) src = src.expand(dst.sizes());
  if (dst.numel() == 0) return dst;
  if (is_mcpu(src) && is_mcpu(dst)) {
    if (same_dense(src, dst)) {
      MCPU_OK(orMemcpyAsync(dst.data_ptr(), src.const_data_ptr(), dst.nbytes(),
                            orMemcpyDeviceToDevice, stream_of(dst)),
              "mcpu device copy");
    } else {
      strided_copy(src, dst);
    }
    return dst;
  }
  if (!is_mcpu(src) && is_mcpu(dst)) {  // host -> device
    at::Tensor h = src.to(dst.scalar_type()).contiguous();
    at::Tensor d = dst.is_contiguous() ? dst : at::empty(dst.sizes(), dst.options());
    orStream_t st = stream_of(dst);
    MCPU_OK(orMemcpyAsync(d.data_ptr(), h.const_data_ptr(), d.nbytes(), orMemcpyHostToDevice, st),
            "mcpu host-to-device copy");
    if (!d.is_same(dst)) strided_copy(d, dst);
    if (!(non_blocking && h.is_pinned() && h.is_same(src))) MCPU_OK(orStreamSynchronize(st), "mcpu sync");
    return dst;
  }
  if (is_mcpu(src) && !is_mcpu(dst)) {  // device -> host
    at::Tensor d = src;
    if (!(src.is_contiguous() && src.scalar_type() == dst.scalar_type())) {
      d = at::empty(src.sizes(), src.options().dtype(dst.scalar_type()));
      strided_copy(src, d);
    }
    const bool direct = dst.is_contiguous() && dst.scalar_type() == d.scalar_type();
    at::Tensor h = direct ? dst : at::empty(dst.sizes(), dst.options());
    orStream_t st = stream_of(src);
    MCPU_OK(orMemcpyAsync(h.data_ptr(), d.const_data_ptr(), h.nbytes(), orMemcpyDeviceToHost, st),
            "mcpu device-to-host copy");
    if (!(non_blocking && direct && dst.is_pinned())) MCPU_OK(orStreamSynchronize(st), "mcpu sync");
    if (!direct) dst.copy_(h);
    return dst;
  }
  TORCH_CHECK(false, "mcpu copy: unsupported devices ", src.device(), " -> ", dst.device());
}

at::Tensor copy_from_and_resize(const at::Tensor& self, const at::Tensor& dst) {
  dst.resize_(self.sizes());
  return copy_from(self, dst, false);
}

at::Scalar local_scalar_dense(const at::Tensor& self) {
  TORCH_CHECK(self.numel() == 1, "a Tensor with ", self.numel(), " elements cannot be converted to Scalar");
  at::Tensor h = at::empty({1}, self.options().device(at::kCPU));
  copy_from(self.reshape({1}), h, false);
  return h.item();
}

at::Tensor& fill_scalar(at::Tensor& self, const at::Scalar& value) {
  if (self.numel() == 0) return self;
  std::vector<int64_t> sizes(self.sizes().begin(), self.sizes().end());
  std::vector<int64_t> strides(self.strides().begin(), self.strides().end());
  const bool fp = value.isFloatingPoint();
  MCPU_OK(mcpu_fill(self.data_ptr(), dtype_code(self.scalar_type()), static_cast<int>(sizes.size()),
                    sizes.data(), strides.data(), fp ? value.toDouble() : 0.0,
                    fp ? 0 : (value.isBoolean() ? static_cast<int64_t>(value.toBool()) : value.toLong()),
                    fp ? 1 : 0, stream_of(self)),
          "mcpu fill");
  return self;
}

at::Tensor& zero_(at::Tensor& self) { return fill_scalar(self, 0); }

void record_stream_op(at::Tensor& self, c10::Stream s) { record_stream(self.storage().data_ptr(), s); }

// ---------------------------------------------------------------- hot aten ops
// [M, K] x [K, N] with mat2 = w.t() of a row-major [N, K] weight (the MLP's
// layout); any other mat2 layout is first made K-contiguous on the device.
at::Tensor k_major_weight(const at::Tensor& mat2) {
  at::Tensor w = mat2.t();
  return w.is_contiguous() ? w : w.contiguous();
}

at::Tensor& mm_out(const at::Tensor& self, const at::Tensor& mat2, at::Tensor& out) {
  TORCH_CHECK(self.dim() == 2 && mat2.dim() == 2, "mm: expected 2-D tensors");
  TORCH_CHECK(self.size(1) == mat2.size(0), "mm: self.size(1) must match mat2.size(0)");
  TORCH_CHECK(self.scalar_type() == at::kBFloat16 && mat2.scalar_type() == at::kBFloat16,
              "mm on mcpu (B200): bfloat16 operands only, got ", self.scalar_type(), " and ",
              mat2.scalar_type());
  TORCH_CHECK(out.sizes() == c10::IntArrayRef({self.size(0), mat2.size(1)}) && out.is_contiguous() &&
                  out.scalar_type() == at::kBFloat16,
              "mm.out: out must be a contiguous bfloat16 [", self.size(0), ", ", mat2.size(1), "] tensor");
  const at::Tensor a = self.contiguous();
  const at::Tensor b = k_major_weight(mat2);
  MCPU_OK(mcpu_mm(a.const_data_ptr(), b.const_data_ptr(), out.data_ptr(), a.size(0), b.size(0), a.size(1),
                  MCPU_BFLOAT16, stream_of(out)),
          "mm");
  return out;
}

at::Tensor mm(const at::Tensor& self, const at::Tensor& mat2) {
  at::Tensor out = at::empty({self.size(0), mat2.size(1)}, self.options());
  return mm_out(self, mat2, out);
}

at::Tensor& addmm_out(const at::Tensor& bias, const at::Tensor& self, const at::Tensor& mat2,
                      const at::Scalar& beta, const at::Scalar& alpha, at::Tensor& out) {
  TORCH_CHECK(beta.toDouble() == 1.0 && alpha.toDouble() == 1.0,
              "addmm on mcpu (B200): beta = alpha = 1 only");
  TORCH_CHECK(bias.numel() == mat2.size(1) && bias.scalar_type() == at::kBFloat16,
              "addmm on mcpu (B200): bias must be a bfloat16 vector of size N");
  TORCH_CHECK(self.scalar_type() == at::kBFloat16 && mat2.scalar_type() == at::kBFloat16,
              "addmm on mcpu (B200): bfloat16 operands only");
  TORCH_CHECK(out.sizes() == c10::IntArrayRef({self.size(0), mat2.size(1)}) && out.is_contiguous(),
              "addmm.out: out must be contiguous [M, N]");
  const at::Tensor a = self.contiguous();
  const at::Tensor b = k_major_weight(mat2);
  const at::Tensor c = bias.contiguous();
  MCPU_OK(mcpu_addmm(c.const_data_ptr(), a.const_data_ptr(), b.const_data_ptr(), out.data_ptr(), a.size(0),
                     b.size(0), a.size(1), MCPU_BFLOAT16, stream_of(out)),
          "addmm");
  return out;
}

at::Tensor addmm(const at::Tensor& bias, const at::Tensor& self, const at::Tensor& mat2,
                 const at::Scalar& beta, const at::Scalar& alpha) {
  at::Tensor out = at::empty({self.size(0), mat2.size(1)}, self.options());
  return addmm_out(bias, self, mat2, beta, alpha, out);
}

template <orError_t (*Fn)(void*, const void*, int64_t, int, orStream_t)>
at::Tensor& unary_out(const at::Tensor& self, at::Tensor& out, const char* name) {
  TORCH_CHECK(self.scalar_type() == at::kFloat || self.scalar_type() == at::kBFloat16, name,
              " on mcpu (B200): float32 or bfloat16 only");
  TORCH_CHECK(out.scalar_type() == self.scalar_type() && out.sizes() == self.sizes(), name,
              ".out: out must match self");
  const at::Tensor x = self.contiguous();
  at::Tensor o = out.is_contiguous() ? out : at::empty(out.sizes(), out.options());
  MCPU_OK(Fn(o.data_ptr(), x.const_data_ptr(), x.numel(), dtype_code(x.scalar_type()), stream_of(o)), name);
  if (!o.is_same(out)) strided_copy(o, out);
  return out;
}

at::Tensor& sigmoid_out(const at::Tensor& self, at::Tensor& out) { return unary_out<mcpu_sigmoid>(self, out, "sigmoid"); }
at::Tensor sigmoid(const at::Tensor& self) {
  at::Tensor out = at::empty(self.sizes(), self.options());
  return sigmoid_out(self, out);
}
at::Tensor& silu_out(const at::Tensor& self, at::Tensor& out) { return unary_out<mcpu_silu>(self, out, "silu"); }
at::Tensor silu(const at::Tensor& self) {
  at::Tensor out = at::empty(self.sizes(), self.options());
  return silu_out(self, out);
}

// ---------------------------------------------------------------- generic ops
// Shapes and strides of a tensor as int64 vectors (element strides).
std::vector<int64_t> vec(c10::IntArrayRef r) { return std::vector<int64_t>(r.begin(), r.end()); }

// A scalar operand (a wrapped number or a 0-dim CPU tensor) as a 0-dim mcpu tensor.
at::Tensor on_device(const at::Tensor& t, const at::Tensor& like) {
  if (is_mcpu(t)) return t;
  TORCH_CHECK(t.dim() == 0, "mcpu: a CPU operand must be a scalar (0-dim), got shape ", t.sizes());
  at::Tensor d = at::empty({}, like.options().dtype(t.scalar_type()));
  d.fill_(t.item());
  return d;
}

at::Tensor& binary_into(int op, const at::Tensor& self_, const at::Tensor& other_, const at::Scalar& alpha,
                        at::Tensor& out) {
  const at::Tensor self = on_device(self_, is_mcpu(self_) ? self_ : other_);
  const at::Tensor other = on_device(other_, self);
  const auto shape = at::infer_size(self.sizes(), other.sizes());
  TORCH_CHECK(out.sizes() == c10::IntArrayRef(shape), "mcpu binary op: out has shape ", out.sizes(),
              ", expected ", c10::IntArrayRef(shape));
  const at::Tensor a = self.expand(shape), b = other.expand(shape);
  const auto sz = vec(out.sizes()), sa = vec(a.strides()), sb = vec(b.strides()), so = vec(out.strides());
  MCPU_OK(mcpu_binary(op, a.const_data_ptr(), dtype_code(a.scalar_type()), sa.data(), b.const_data_ptr(),
                      dtype_code(b.scalar_type()), sb.data(), out.data_ptr(), dtype_code(out.scalar_type()),
                      so.data(), static_cast<int>(out.dim()), sz.data(), alpha.toDouble(), stream_of(out)),
          "binary op");
  return out;
}

at::ScalarType binary_result(const at::Tensor& a, const at::Tensor& b, bool true_div) {
  at::ScalarType t = at::result_type(a, b);
  if (true_div && at::isIntegralType(t, /*includeBool=*/true)) t = c10::typeMetaToScalarType(c10::get_default_dtype());
  return t;
}

at::Tensor binary_new(int op, const at::Tensor& self, const at::Tensor& other, const at::Scalar& alpha) {
  const auto shape = at::infer_size(self.sizes(), other.sizes());
  const at::Tensor& dev = is_mcpu(self) ? self : other;
  at::Tensor out = at::empty(shape, dev.options().dtype(binary_result(self, other, op == MCPU_BINARY_DIV)));
  return binary_into(op, self, other, alpha, out);
}

at::Tensor add(const at::Tensor& s, const at::Tensor& o, const at::Scalar& alpha) { return binary_new(MCPU_BINARY_ADD, s, o, alpha); }
at::Tensor& add_out(const at::Tensor& s, const at::Tensor& o, const at::Scalar& alpha, at::Tensor& out) { return binary_into(MCPU_BINARY_ADD, s, o, alpha, out); }
at::Tensor& add_(at::Tensor& s, const at::Tensor& o, const at::Scalar& alpha) { return binary_into(MCPU_BINARY_ADD, s, o, alpha, s); }
at::Tensor sub(const at::Tensor& s, const at::Tensor& o, const at::Scalar& alpha) { return binary_new(MCPU_BINARY_SUB, s, o, alpha); }
at::Tensor& sub_out(const at::Tensor& s, const at::Tensor& o, const at::Scalar& alpha, at::Tensor& out) { return binary_into(MCPU_BINARY_SUB, s, o, alpha, out); }
at::Tensor mul(const at::Tensor& s, const at::Tensor& o) { return binary_new(MCPU_BINARY_MUL, s, o, 1); }
at::Tensor& mul_out(const at::Tensor& s, const at::Tensor& o, at::Tensor& out) { return binary_into(MCPU_BINARY_MUL, s, o, 1, out); }
at::Tensor& mul_(at::Tensor& s, const at::Tensor& o) { return binary_into(MCPU_BINARY_MUL, s, o, 1, s); }
at::Tensor div_tensor(const at::Tensor& s, const at::Tensor& o) { return binary_new(MCPU_BINARY_DIV, s, o, 1); }
at::Tensor& div_out(const at::Tensor& s, const at::Tensor& o, at::Tensor& out) { return binary_into(MCPU_BINARY_DIV, s, o, 1, out); }
at::Tensor& div_(at::Tensor& s, const at::Tensor& o) { return binary_into(MCPU_BINARY_DIV, s, o, 1, s); }

at::Tensor& unary_into(int op, const at::Tensor& self, double scalar, at::Tensor& out) {
  TORCH_CHECK(out.sizes() == self.sizes(), "mcpu unary op: out must have the input's shape");
  const auto sz = vec(self.sizes()), sx = vec(self.strides()), so = vec(out.strides());
  MCPU_OK(mcpu_unary(op, self.const_data_ptr(), dtype_code(self.scalar_type()), sx.data(), out.data_ptr(),
                     dtype_code(out.scalar_type()), so.data(), static_cast<int>(self.dim()), sz.data(), scalar,
                     stream_of(out)),
          "unary op");
  return out;
}

at::ScalarType float_result(const at::Tensor& t) {
  return at::isFloatingType(t.scalar_type()) ? t.scalar_type() : c10::typeMetaToScalarType(c10::get_default_dtype());
}

at::Tensor neg(const at::Tensor& s) { at::Tensor o = at::empty(s.sizes(), s.options()); return unary_into(MCPU_UNARY_NEG, s, 0, o); }
at::Tensor& neg_out(const at::Tensor& s, at::Tensor& o) { return unary_into(MCPU_UNARY_NEG, s, 0, o); }
at::Tensor abs_tensor(const at::Tensor& s) { at::Tensor o = at::empty(s.sizes(), s.options()); return unary_into(MCPU_UNARY_ABS, s, 0, o); }
at::Tensor& abs_out(const at::Tensor& s, at::Tensor& o) { return unary_into(MCPU_UNARY_ABS, s, 0, o); }
at::Tensor rsqrt(const at::Tensor& s) { at::Tensor o = at::empty(s.sizes(), s.options().dtype(float_result(s))); return unary_into(MCPU_UNARY_RSQRT, s, 0, o); }
at::Tensor& rsqrt_out(const at::Tensor& s, at::Tensor& o) { return unary_into(MCPU_UNARY_RSQRT, s, 0, o); }
at::Tensor sqrt_tensor(const at::Tensor& s) { at::Tensor o = at::empty(s.sizes(), s.options().dtype(float_result(s))); return unary_into(MCPU_UNARY_SQRT, s, 0, o); }
at::Tensor& sqrt_out(const at::Tensor& s, at::Tensor& o) { return unary_into(MCPU_UNARY_SQRT, s, 0, o); }
at::Tensor bitwise_not(const at::Tensor& s) {
  TORCH_CHECK(at::isIntegralType(s.scalar_type(), true), "bitwise_not: integer or bool tensors only");
  at::Tensor o = at::empty(s.sizes(), s.options());
  return unary_into(MCPU_UNARY_BITWISE_NOT, s, 0, o);
}
at::Tensor& bitwise_not_out(const at::Tensor& s, at::Tensor& o) { return unary_into(MCPU_UNARY_BITWISE_NOT, s, 0, o); }
at::Tensor pow_scalar(const at::Tensor& s, const at::Scalar& e) {
  const at::ScalarType t = e.isFloatingPoint() ? float_result(s) : s.scalar_type();
  at::Tensor o = at::empty(s.sizes(), s.options().dtype(t));
  return unary_into(MCPU_UNARY_POW_SCALAR, s, e.toDouble(), o);
}
at::Tensor& pow_scalar_out(const at::Tensor& s, const at::Scalar& e, at::Tensor& o) {
  return unary_into(MCPU_UNARY_POW_SCALAR, s, e.toDouble(), o);
}

at::Tensor& masked_fill_(at::Tensor& self, const at::Tensor& mask_, const at::Scalar& value) {
  TORCH_CHECK(mask_.scalar_type() == at::kBool, "masked_fill_: the mask must be a bool tensor");
  const at::Tensor mask = on_device(mask_, self).expand(self.sizes());
  const auto sz = vec(self.sizes()), ss = vec(self.strides()), sm = vec(mask.strides());
  MCPU_OK(mcpu_masked_fill(self.data_ptr(), dtype_code(self.scalar_type()), ss.data(), mask.const_data_ptr(),
                           sm.data(), static_cast<int>(self.dim()), sz.data(), value.toDouble(),
                           value.isFloatingPoint() ? 0 : value.toLong(), value.isFloatingPoint() ? 1 : 0,
                           stream_of(self)),
          "masked_fill_");
  return self;
}
at::Tensor& masked_fill_tensor_(at::Tensor& self, const at::Tensor& mask, const at::Tensor& value) {
  TORCH_CHECK(value.dim() == 0, "masked_fill_: value must be a 0-dim tensor");
  return masked_fill_(self, mask, value.item());
}

// Reductions and selections run over the last dimension of a contiguous
// tensor; another dimension is moved last first.
at::Tensor dim_last(const at::Tensor& t, int64_t dim) {
  return (dim == t.dim() - 1 ? t : t.movedim(dim, -1)).contiguous();
}

at::Tensor& reduce_into(int op, const at::Tensor& self, int64_t dim, bool keepdim, at::Tensor& values,
                        at::Tensor* indices) {
  dim = c10::maybe_wrap_dim(dim, self.dim());
  const at::Tensor x = dim_last(self, dim);
  const int64_t n = self.dim() == 0 ? 1 : self.size(dim);
  const int64_t rows = n == 0 ? x.numel() : x.numel() / n;
  std::vector<int64_t> shape = vec(self.sizes());
  if (self.dim() > 0) {
    if (keepdim) shape[dim] = 1;
    else shape.erase(shape.begin() + dim);
  }
  at::Tensor v = at::empty({rows}, values.options());
  at::Tensor ix;
  if (indices) ix = at::empty({rows}, values.options().dtype(at::kLong));
  MCPU_OK(mcpu_reduce_lastdim(op, x.const_data_ptr(), dtype_code(x.scalar_type()), rows, n, v.data_ptr(),
                              dtype_code(v.scalar_type()), indices ? ix.data_ptr<int64_t>() : nullptr,
                              stream_of(x)),
          "reduction");
  values.resize_(shape);
  values.copy_(v.view(shape));
  if (indices) {
    indices->resize_(shape);
    indices->copy_(ix.view(shape));
  }
  return values;
}

at::Tensor sum_dim(const at::Tensor& self, at::OptionalIntArrayRef dims, bool keepdim, std::optional<at::ScalarType> dtype) {
  at::ScalarType t = dtype.value_or(at::isIntegralType(self.scalar_type(), true) ? at::kLong : self.scalar_type());
  if (!dims || dims->empty()) {
    at::Tensor flat = self.reshape({1, self.numel()});
    at::Tensor out = at::empty({1}, self.options().dtype(t));
    reduce_into(MCPU_REDUCE_SUM, flat, 1, false, out, nullptr);
    return keepdim ? out.view(std::vector<int64_t>(self.dim(), 1)) : out.view({});
  }
  TORCH_CHECK(dims->size() == 1, "sum on mcpu: one dimension at a time");
  at::Tensor out = at::empty({0}, self.options().dtype(t));
  return reduce_into(MCPU_REDUCE_SUM, self, (*dims)[0], keepdim, out, nullptr);
}
at::Tensor& sum_dim_out(const at::Tensor& self, at::OptionalIntArrayRef dims, bool keepdim,
                        std::optional<at::ScalarType> dtype, at::Tensor& out) {
  TORCH_CHECK(dims && dims->size() == 1, "sum.out on mcpu: one dimension");
  return reduce_into(MCPU_REDUCE_SUM, self, (*dims)[0], keepdim, out, nullptr);
}
at::Tensor mean_dim(const at::Tensor& self, at::OptionalIntArrayRef dims, bool keepdim, std::optional<at::ScalarType> dtype) {
  TORCH_CHECK(dims && dims->size() == 1, "mean on mcpu: one dimension at a time");
  at::Tensor out = at::empty({0}, self.options().dtype(dtype.value_or(self.scalar_type())));
  return reduce_into(MCPU_REDUCE_MEAN, self, (*dims)[0], keepdim, out, nullptr);
}
std::tuple<at::Tensor, at::Tensor> max_dim(const at::Tensor& self, int64_t dim, bool keepdim) {
  at::Tensor v = at::empty({0}, self.options());
  at::Tensor i = at::empty({0}, self.options().dtype(at::kLong));
  reduce_into(MCPU_REDUCE_MAX, self, dim, keepdim, v, &i);
  return {v, i};
}
std::tuple<at::Tensor, at::Tensor> min_dim(const at::Tensor& self, int64_t dim, bool keepdim) {
  at::Tensor v = at::empty({0}, self.options());
  at::Tensor i = at::empty({0}, self.options().dtype(at::kLong));
  reduce_into(MCPU_REDUCE_MIN, self, dim, keepdim, v, &i);
  return {v, i};
}

std::tuple<at::Tensor&, at::Tensor&> topk_out(const at::Tensor& self, int64_t k, int64_t dim, bool largest,
                                              bool sorted, at::Tensor& values, at::Tensor& indices) {
  dim = c10::maybe_wrap_dim(dim, self.dim());
  const int64_t n = self.dim() == 0 ? 1 : self.size(dim);
  TORCH_CHECK(k >= 0 && k <= n, "selected index k out of range");
  const at::Tensor x = dim_last(self, dim);
  const int64_t rows = n == 0 ? 0 : x.numel() / n;
  std::vector<int64_t> last_shape = vec(x.sizes());
  if (!last_shape.empty()) last_shape.back() = k;
  at::Tensor v = at::empty(last_shape, self.options());
  at::Tensor ix = at::empty(last_shape, self.options().dtype(at::kLong));
  MCPU_OK(mcpu_topk_lastdim(x.const_data_ptr(), dtype_code(x.scalar_type()), rows, n, k, largest ? 1 : 0,
                            v.data_ptr(), ix.data_ptr<int64_t>(), stream_of(x)),
          "topk");
  // (sorted or not, the values come in order, ties to the lower index)
  at::Tensor vv = dim == self.dim() - 1 ? v : v.movedim(-1, dim);
  at::Tensor ii = dim == self.dim() - 1 ? ix : ix.movedim(-1, dim);
  values.resize_(vv.sizes());
  indices.resize_(ii.sizes());
  values.copy_(vv);
  indices.copy_(ii);
  return {values, indices};
}
std::tuple<at::Tensor, at::Tensor> topk(const at::Tensor& self, int64_t k, int64_t dim, bool largest, bool sorted) {
  at::Tensor v = at::empty({0}, self.options());
  at::Tensor i = at::empty({0}, self.options().dtype(at::kLong));
  topk_out(self, k, dim, largest, sorted, v, i);
  return {v, i};
}

at::Tensor& softmax_into(const at::Tensor& self, int64_t dim, bool log, at::Tensor& out) {
  dim = c10::maybe_wrap_dim(dim, self.dim());
  const at::Tensor x = dim_last(self, dim);
  const int64_t n = self.dim() == 0 ? 1 : self.size(dim);
  const int64_t rows = n == 0 ? 0 : x.numel() / n;
  at::Tensor o = at::empty(x.sizes(), out.options());
  MCPU_OK(mcpu_softmax_lastdim(x.const_data_ptr(), dtype_code(x.scalar_type()), rows, n, o.data_ptr(),
                               dtype_code(o.scalar_type()), log ? 1 : 0, stream_of(x)),
          "softmax");
  at::Tensor oo = dim == self.dim() - 1 ? o : o.movedim(-1, dim);
  out.resize_(oo.sizes());
  out.copy_(oo);
  return out;
}
at::Tensor softmax_(const at::Tensor& self, int64_t dim, bool half_to_float) {
  at::Tensor out = at::empty({0}, self.options().dtype(half_to_float ? at::kFloat : self.scalar_type()));
  return softmax_into(self, dim, false, out);
}
at::Tensor& softmax_out(const at::Tensor& self, int64_t dim, bool half_to_float, at::Tensor& out) {
  return softmax_into(self, dim, false, out);
}
at::Tensor log_softmax_(const at::Tensor& self, int64_t dim, bool half_to_float) {
  at::Tensor out = at::empty({0}, self.options().dtype(half_to_float ? at::kFloat : self.scalar_type()));
  return softmax_into(self, dim, true, out);
}

at::Tensor& gather_out(const at::Tensor& self, int64_t dim, const at::Tensor& index, bool sparse_grad, at::Tensor& out) {
  dim = c10::maybe_wrap_dim(dim, self.dim());
  TORCH_CHECK(index.scalar_type() == at::kLong, "gather: index must be int64");
  TORCH_CHECK(index.dim() == self.dim(), "gather: index and self must have the same number of dimensions");
  out.resize_(index.sizes());
  const auto ss = vec(self.sizes()), st = vec(self.strides()), is = vec(index.sizes()), it = vec(index.strides()),
             ot = vec(out.strides());
  MCPU_OK(mcpu_gather(self.const_data_ptr(), dtype_code(self.scalar_type()), static_cast<int>(self.dim()), ss.data(),
                      st.data(), dim, index.const_data_ptr<int64_t>(), is.data(), it.data(), out.data_ptr(), ot.data(),
                      stream_of(self)),
          "gather");
  return out;
}
at::Tensor gather(const at::Tensor& self, int64_t dim, const at::Tensor& index, bool sparse_grad) {
  at::Tensor out = at::empty(index.sizes(), self.options());
  return gather_out(self, dim, index, sparse_grad, out);
}

at::Tensor& scatter_value_(at::Tensor& self, int64_t dim, const at::Tensor& index, const at::Scalar& value) {
  dim = c10::maybe_wrap_dim(dim, self.dim());
  TORCH_CHECK(index.scalar_type() == at::kLong, "scatter_: index must be int64");
  TORCH_CHECK(index.dim() == self.dim(), "scatter_: index and self must have the same number of dimensions");
  const auto ss = vec(self.sizes()), st = vec(self.strides()), is = vec(index.sizes()), it = vec(index.strides());
  MCPU_OK(mcpu_scatter_value(self.data_ptr(), dtype_code(self.scalar_type()), static_cast<int>(self.dim()), ss.data(),
                             st.data(), dim, index.const_data_ptr<int64_t>(), is.data(), it.data(), value.toDouble(),
                             value.isFloatingPoint() ? 0 : value.toLong(), value.isFloatingPoint() ? 1 : 0,
                             stream_of(self)),
          "scatter_");
  return self;
}
at::Tensor& scatter_value_out(const at::Tensor& self, int64_t dim, const at::Tensor& index, const at::Scalar& value,
                              at::Tensor& out) {
  if (!out.is_same(self)) {
    out.resize_(self.sizes());
    out.copy_(self);
  }
  return scatter_value_(out, dim, index, value);
}
at::Tensor scatter_value(const at::Tensor& self, int64_t dim, const at::Tensor& index, const at::Scalar& value) {
  at::Tensor out = self.clone();
  return scatter_value_(out, dim, index, value);
}

// ---------------------------------------------------------------- custom ops
std::tuple<at::Tensor, at::Tensor> grouped_topk(const at::Tensor& gating, int64_t num_expert_group,
                                                int64_t topk_group, int64_t topk, bool renormalize,
                                                double routed_scaling_factor,
                                                const std::optional<at::Tensor>& bias,
                                                c10::string_view scoring_func) {
  TORCH_CHECK(gating.dim() == 2, "grouped_topk: gating_output must be [num_tokens, num_experts]");
  TORCH_CHECK(scoring_func == "softmax" || scoring_func == "sigmoid", "Unsupported scoring function: ",
              scoring_func);
  const at::Tensor g = gating.contiguous();
  at::Tensor b;
  if (bias.has_value() && bias->defined()) b = bias->to(at::kFloat).contiguous();
  at::Tensor w = at::empty({g.size(0), topk}, g.options().dtype(at::kFloat));
  at::Tensor ids = at::empty({g.size(0), topk}, g.options().dtype(at::kInt));
  MCPU_OK(mcpu_grouped_topk(g.const_data_ptr(), dtype_code(g.scalar_type()), g.size(0), g.size(1),
                            num_expert_group, topk_group, topk, renormalize ? 1 : 0,
                            static_cast<float>(routed_scaling_factor),
                            b.defined() ? static_cast<const float*>(b.const_data_ptr()) : nullptr,
                            scoring_func == "sigmoid" ? MCPU_SCORING_SIGMOID : MCPU_SCORING_SOFTMAX,
                            w.data_ptr<float>(), ids.data_ptr<int32_t>(), stream_of(g)),
          "grouped_topk");
  return {w, ids};
}

void silu_and_mul(at::Tensor& out, const at::Tensor& x) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && out.scalar_type() == at::kBFloat16,
              "silu_and_mul: bfloat16 tensors expected");
  TORCH_CHECK(x.is_contiguous() && out.is_contiguous(), "silu_and_mul: contiguous tensors expected");
  const int64_t d = x.size(-1) / 2;
  TORCH_CHECK(out.size(-1) == d && out.numel() * 2 == x.numel(), "silu_and_mul: out must be [..., d]");
  MCPU_OK(mcpu_silu_and_mul(out.data_ptr(), x.const_data_ptr(), x.numel() / (2 * d > 0 ? 2 * d : 1), d,
                            MCPU_BFLOAT16, stream_of(x)),
          "silu_and_mul");
}

void rms_norm(at::Tensor& out, const at::Tensor& x, const at::Tensor& weight, double eps) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && out.scalar_type() == at::kBFloat16 &&
                  weight.scalar_type() == at::kBFloat16,
              "rms_norm: bfloat16 tensors expected");
  TORCH_CHECK(x.is_contiguous() && out.is_contiguous() && weight.is_contiguous(),
              "rms_norm: contiguous tensors expected");
  const int64_t H = x.size(-1);
  TORCH_CHECK(weight.numel() == H && out.sizes() == x.sizes(), "rms_norm: shape mismatch");
  MCPU_OK(mcpu_rms_norm(out.data_ptr(), x.const_data_ptr(), weight.const_data_ptr(), x.numel() / H, H,
                        static_cast<float>(eps), MCPU_BFLOAT16, stream_of(x)),
          "rms_norm");
}

at::Tensor& gemm_swiglu_out(const at::Tensor& x, const at::Tensor& w_gate_up, at::Tensor& out) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w_gate_up.scalar_type() == at::kBFloat16 &&
                  out.scalar_type() == at::kBFloat16,
              "gemm_swiglu: bfloat16 tensors expected");
  TORCH_CHECK(x.is_contiguous() && w_gate_up.is_contiguous() && out.is_contiguous(),
              "gemm_swiglu.out: contiguous tensors expected");
  TORCH_CHECK(out.dim() == 2 && out.size(0) == x.size(0) && out.size(1) == w_gate_up.size(0) / 2,
              "gemm_swiglu.out: out must be [M, I]");
  MCPU_OK(mcpu_gemm_swiglu(x.const_data_ptr(), w_gate_up.const_data_ptr(), out.data_ptr(), x.size(0),
                           w_gate_up.size(0) / 2, x.size(1), MCPU_BFLOAT16, stream_of(x)),
          "gemm_swiglu");
  return out;
}

at::Tensor gemm_swiglu(const at::Tensor& x, const at::Tensor& w_gate_up) {
  const at::Tensor a = x.contiguous(), w = w_gate_up.contiguous();
  at::Tensor out = at::empty({a.size(0), w.size(0) / 2}, a.options());
  return gemm_swiglu_out(a, w, out);
}

// MoE expert dispatch after the router, vLLM's moe_align_block_size schema
// (vllm/_custom_ops.py:2247-2264); the workspace comes from the device's
// stream-ordered allocator.
void moe_align_block_size(const at::Tensor& topk_ids, int64_t num_experts, int64_t block_size,
                          at::Tensor& sorted_token_ids, at::Tensor& experts_ids, at::Tensor& num_tokens_post_pad) {
  TORCH_CHECK(topk_ids.scalar_type() == at::kInt || topk_ids.scalar_type() == at::kLong,
              "moe_align_block_size: topk_ids must be int32 or int64");
  for (const at::Tensor* t : {&sorted_token_ids, &experts_ids, &num_tokens_post_pad}) {
    TORCH_CHECK(t->scalar_type() == at::kInt && t->is_contiguous() && t->device() == topk_ids.device(),
                "moe_align_block_size: outputs must be contiguous int32 tensors on the ids' device");
  }
  TORCH_CHECK(num_tokens_post_pad.numel() >= 1, "moe_align_block_size: num_tokens_post_pad needs one element");
  const at::Tensor ids = topk_ids.to(at::kInt).contiguous();
  uint64_t ws = 0;
  MCPU_OK(mcpu_moe_align_workspace_bytes(ids.numel(), static_cast<int>(num_experts), &ws),
          "moe_align_block_size");
  at::Tensor work = at::empty({static_cast<int64_t>(ws)}, ids.options().dtype(at::kByte));
  MCPU_OK(mcpu_moe_align_block_size(ids.const_data_ptr<int32_t>(), ids.numel(), static_cast<int>(num_experts),
                                    static_cast<int>(block_size), sorted_token_ids.data_ptr<int32_t>(),
                                    sorted_token_ids.numel(), experts_ids.data_ptr<int32_t>(), experts_ids.numel(),
                                    num_tokens_post_pad.data_ptr<int32_t>(), work.data_ptr(), ws, stream_of(ids)),
          "moe_align_block_size");
}

// vLLM sampler kernels with the reference's own schemas
// (csrc/aten/vllm_kernels/min_p.cpp:113-124, logprob.cpp:188-208).
int sampler_dtype(const at::Tensor& t, const char* name) {
  switch (t.scalar_type()) {
    case at::kFloat: return MCPU_FLOAT32;
    case at::kHalf: return MCPU_FLOAT16;
    case at::kBFloat16: return MCPU_BFLOAT16;
    default: TORCH_CHECK(false, name, " must be float32, float16, or bfloat16, got ", t.scalar_type());
  }
}

void vllm_min_p_kernel(at::Tensor& logits, const at::Tensor& expanded_idx_mapping, const at::Tensor& min_p,
                       int64_t vocab_size) {
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1, "logits must be 2-D with unit column stride");
  TORCH_CHECK(expanded_idx_mapping.dim() == 1 && expanded_idx_mapping.scalar_type() == at::kInt,
              "expanded_idx_mapping must be 1-D int32");
  TORCH_CHECK(min_p.dim() == 1 && min_p.scalar_type() == at::kFloat, "min_p must be 1-D float32");
  TORCH_CHECK(vocab_size > 0 && vocab_size <= logits.size(1), "vocab_size ", vocab_size, " out of range [1, ",
              logits.size(1), "]");
  TORCH_CHECK(expanded_idx_mapping.numel() >= logits.size(0), "expanded_idx_mapping shorter than the tokens");
  const int dt = sampler_dtype(logits, "logits");
  const at::Tensor idx = expanded_idx_mapping.contiguous(), mp = min_p.contiguous();
  MCPU_OK(mcpu_vllm_min_p(logits.data_ptr(), dt, logits.size(0), logits.stride(0), idx.const_data_ptr<int32_t>(),
                          mp.const_data_ptr<float>(), vocab_size, stream_of(logits)),
          "vllm_min_p_kernel");
}

void vllm_topk_log_softmax_kernel(at::Tensor& output, const at::Tensor& logits, const at::Tensor& topk_ids,
                                  int64_t topk, int64_t vocab_size) {
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1, "logits must be 2-D with unit column stride");
  const int dt = sampler_dtype(logits, "logits");
  TORCH_CHECK(output.dim() == 2 && output.scalar_type() == at::kFloat && output.is_contiguous(),
              "output must be a contiguous 2-D float32 tensor");
  TORCH_CHECK(topk_ids.dim() == 2 && topk_ids.scalar_type() == at::kLong && topk_ids.stride(1) == 1,
              "topk_ids must be 2-D int64 with unit column stride");
  TORCH_CHECK(vocab_size > 0 && vocab_size <= logits.size(1), "vocab_size out of range");
  TORCH_CHECK(output.size(0) == logits.size(0) && output.size(1) == topk && topk_ids.size(1) >= topk &&
                  topk_ids.size(0) >= logits.size(0),
              "vllm_topk_log_softmax_kernel: shape mismatch");
  MCPU_OK(mcpu_vllm_topk_log_softmax(output.data_ptr<float>(), logits.const_data_ptr(), dt, logits.size(0),
                                     logits.stride(0), topk_ids.const_data_ptr<int64_t>(), topk_ids.stride(0), topk,
                                     vocab_size, stream_of(logits)),
          "vllm_topk_log_softmax_kernel");
}

void vllm_ranks_kernel(at::Tensor& output, const at::Tensor& logits, const at::Tensor& token_ids,
                       int64_t vocab_size) {
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1, "logits must be 2-D with unit column stride");
  const int dt = sampler_dtype(logits, "logits");
  TORCH_CHECK(output.dim() == 1 && output.scalar_type() == at::kLong && output.is_contiguous(),
              "output must be a contiguous 1-D int64 tensor");
  TORCH_CHECK(token_ids.dim() == 1 && token_ids.scalar_type() == at::kLong, "token_ids must be 1-D int64");
  TORCH_CHECK(vocab_size > 0 && vocab_size <= logits.size(1), "vocab_size out of range");
  TORCH_CHECK(output.numel() == logits.size(0) && token_ids.numel() >= logits.size(0),
              "vllm_ranks_kernel: shape mismatch");
  const at::Tensor ids = token_ids.contiguous();
  MCPU_OK(mcpu_vllm_ranks(output.data_ptr<int64_t>(), logits.const_data_ptr(), dt, logits.size(0),
                          logits.stride(0), ids.const_data_ptr<int64_t>(), vocab_size, stream_of(logits)),
          "vllm_ranks_kernel");
}

// csrc/aten/vllm_kernels/penalties.cpp:87-118 (checks) and 248-272 (schemas)
void vllm_penalties_kernel(at::Tensor& logits, const at::Tensor& expanded_idx_mapping,
                           const at::Tensor& token_ids, const at::Tensor& expanded_local_pos,
                           const at::Tensor& repetition_penalty, const at::Tensor& frequency_penalty,
                           const at::Tensor& presence_penalty, const at::Tensor& prompt_bin_mask,
                           const at::Tensor& output_bin_counts, int64_t vocab_size, int64_t max_spec_len) {
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1, "logits must be 2-D with unit column stride");
  const int dt = sampler_dtype(logits, "logits");
  auto int1d = [](const at::Tensor& t, const char* name) {
    TORCH_CHECK(t.dim() == 1 && t.scalar_type() == at::kInt, name, " must be 1-D int32");
    return t.contiguous();
  };
  auto float1d = [](const at::Tensor& t, const char* name) {
    TORCH_CHECK(t.dim() == 1 && t.scalar_type() == at::kFloat, name, " must be 1-D float32");
    return t.contiguous();
  };
  const at::Tensor idx = int1d(expanded_idx_mapping, "expanded_idx_mapping");
  const at::Tensor tids = int1d(token_ids, "token_ids");
  const at::Tensor lpos = int1d(expanded_local_pos, "expanded_local_pos");
  const at::Tensor rep = float1d(repetition_penalty, "repetition_penalty");
  const at::Tensor freq = float1d(frequency_penalty, "frequency_penalty");
  const at::Tensor pres = float1d(presence_penalty, "presence_penalty");
  TORCH_CHECK(prompt_bin_mask.dim() == 2 && prompt_bin_mask.scalar_type() == at::kInt &&
                  prompt_bin_mask.stride(1) == 1,
              "prompt_bin_mask must be 2-D int32 with unit column stride");
  TORCH_CHECK(output_bin_counts.dim() == 2 && output_bin_counts.scalar_type() == at::kInt &&
                  output_bin_counts.stride(1) == 1,
              "output_bin_counts must be 2-D int32 with unit column stride");
  TORCH_CHECK(vocab_size > 0 && vocab_size <= logits.size(1) && vocab_size <= output_bin_counts.size(1) &&
                  (vocab_size + 31) / 32 <= prompt_bin_mask.size(1),
              "vllm_penalties_kernel: vocab_size ", vocab_size, " out of range");
  const int64_t n = logits.size(0);
  TORCH_CHECK(idx.numel() >= n && tids.numel() >= n && lpos.numel() >= n,
              "vllm_penalties_kernel: per-token tensors shorter than the logits rows");
  const int64_t reqs = std::min({rep.numel(), freq.numel(), pres.numel(), prompt_bin_mask.size(0),
                                 output_bin_counts.size(0)});
  MCPU_OK(mcpu_vllm_penalties(logits.data_ptr(), dt, n, logits.stride(0), idx.const_data_ptr<int32_t>(),
                              tids.const_data_ptr<int32_t>(), lpos.const_data_ptr<int32_t>(),
                              rep.const_data_ptr<float>(), freq.const_data_ptr<float>(),
                              pres.const_data_ptr<float>(), reqs, prompt_bin_mask.const_data_ptr<int32_t>(),
                              prompt_bin_mask.stride(0), output_bin_counts.const_data_ptr<int32_t>(),
                              output_bin_counts.stride(0), vocab_size, max_spec_len, stream_of(logits)),
          "vllm_penalties_kernel");
}

void vllm_bincount_kernel(const at::Tensor& expanded_idx_mapping, const at::Tensor& all_token_ids,
                          const at::Tensor& prompt_len, const at::Tensor& prefill_len, at::Tensor& prompt_bin_mask,
                          at::Tensor& output_bin_counts) {
  auto int1d = [](const at::Tensor& t, const char* name) {
    TORCH_CHECK(t.dim() == 1 && t.scalar_type() == at::kInt, name, " must be 1-D int32");
    return t.contiguous();
  };
  auto int2d = [](const at::Tensor& t, const char* name) {
    TORCH_CHECK(t.dim() == 2 && t.scalar_type() == at::kInt && t.stride(1) == 1, name,
                " must be 2-D int32 with unit column stride");
  };
  const at::Tensor idx = int1d(expanded_idx_mapping, "expanded_idx_mapping");
  const at::Tensor plen = int1d(prompt_len, "prompt_len");
  const at::Tensor flen = int1d(prefill_len, "prefill_len");
  int2d(all_token_ids, "all_token_ids");
  int2d(prompt_bin_mask, "prompt_bin_mask");
  int2d(output_bin_counts, "output_bin_counts");
  const int64_t reqs = std::min({plen.numel(), flen.numel(), all_token_ids.size(0), prompt_bin_mask.size(0),
                                 output_bin_counts.size(0)});
  MCPU_OK(mcpu_vllm_bincount(idx.const_data_ptr<int32_t>(), idx.numel(), all_token_ids.const_data_ptr<int32_t>(),
                             all_token_ids.stride(0), all_token_ids.size(1), plen.const_data_ptr<int32_t>(),
                             flen.const_data_ptr<int32_t>(), reqs, prompt_bin_mask.data_ptr<int32_t>(),
                             prompt_bin_mask.size(1), prompt_bin_mask.stride(0), output_bin_counts.data_ptr<int32_t>(),
                             output_bin_counts.size(1), output_bin_counts.stride(0), stream_of(all_token_ids)),
          "vllm_bincount_kernel");
}

// csrc/aten/vllm_kernels/logit_bias.cpp:98-191 (checks) and 195-211 (schema)
void vllm_bias_kernel(at::Tensor& logits, int64_t vocab_size, const at::Tensor& expanded_idx_mapping,
                      const at::Tensor& num_allowed_token_ids, const at::Tensor& allowed_token_ids,
                      const at::Tensor& num_logit_bias, const at::Tensor& bias_token_ids, const at::Tensor& bias,
                      const at::Tensor& pos, const at::Tensor& min_lens, const at::Tensor& num_stop_token_ids,
                      const at::Tensor& stop_token_ids) {
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1, "logits must be 2-D with unit column stride");
  const int dt = sampler_dtype(logits, "logits");
  TORCH_CHECK(vocab_size > 0 && vocab_size <= logits.size(1), "vllm_bias_kernel: vocab_size ", vocab_size,
              " out of range");
  auto int1d = [](const at::Tensor& t, const char* name) {
    TORCH_CHECK(t.dim() == 1 && t.scalar_type() == at::kInt, name, " must be 1-D int32");
    return t.contiguous();
  };
  auto list2d = [](const at::Tensor& t, at::ScalarType dt2, const char* name) {
    TORCH_CHECK(t.dim() == 2 && t.scalar_type() == dt2 && t.stride(1) == 1, name,
                " must be 2-D with unit column stride and dtype ", dt2);
  };
  const at::Tensor idx = int1d(expanded_idx_mapping, "expanded_idx_mapping");
  const at::Tensor na = int1d(num_allowed_token_ids, "num_allowed_token_ids");
  const at::Tensor nb = int1d(num_logit_bias, "num_logit_bias");
  const at::Tensor ml = int1d(min_lens, "min_lens");
  const at::Tensor ns = int1d(num_stop_token_ids, "num_stop_token_ids");
  TORCH_CHECK(pos.dim() == 1 && pos.scalar_type() == at::kLong, "pos must be 1-D int64");
  const at::Tensor ps = pos.contiguous();
  list2d(allowed_token_ids, at::kInt, "allowed_token_ids");
  list2d(bias_token_ids, at::kInt, "bias_token_ids");
  list2d(bias, at::kFloat, "bias");
  list2d(stop_token_ids, at::kInt, "stop_token_ids");
  TORCH_CHECK(bias.size(1) == bias_token_ids.size(1), "bias and bias_token_ids differ in width");
  const int64_t n = logits.size(0);
  TORCH_CHECK(idx.numel() >= n && ps.numel() >= n, "vllm_bias_kernel: per-token tensors shorter than the rows");
  const int64_t reqs = std::min({na.numel(), nb.numel(), ml.numel(), ns.numel(), allowed_token_ids.size(0),
                                 bias_token_ids.size(0), bias.size(0), stop_token_ids.size(0)});
  MCPU_OK(mcpu_vllm_bias(logits.data_ptr(), dt, n, logits.stride(0), vocab_size, idx.const_data_ptr<int32_t>(), reqs,
                         na.const_data_ptr<int32_t>(), allowed_token_ids.const_data_ptr<int32_t>(),
                         allowed_token_ids.stride(0), allowed_token_ids.size(1), nb.const_data_ptr<int32_t>(),
                         bias_token_ids.const_data_ptr<int32_t>(), bias_token_ids.stride(0),
                         bias.const_data_ptr<float>(), bias.stride(0), bias.size(1), ps.const_data_ptr<int64_t>(),
                         ml.const_data_ptr<int32_t>(), ns.const_data_ptr<int32_t>(),
                         stop_token_ids.const_data_ptr<int32_t>(), stop_token_ids.stride(0), stop_token_ids.size(1),
                         stream_of(logits)),
          "vllm_bias_kernel");
}

// csrc/aten/vllm_kernels/bad_words.cpp:84-180 (checks) and 184-198 (schema)
void vllm_bad_words_kernel(at::Tensor& logits, const at::Tensor& expanded_idx_mapping,
                           const at::Tensor& bad_word_token_ids, const at::Tensor& bad_word_offsets,
                           const at::Tensor& num_bad_words, const at::Tensor& all_token_ids,
                           const at::Tensor& prompt_len, const at::Tensor& total_len, const at::Tensor& input_ids,
                           const at::Tensor& expanded_local_pos) {
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1, "logits must be 2-D with unit column stride");
  const int dt = sampler_dtype(logits, "logits");
  auto int1d = [](const at::Tensor& t, const char* name) {
    TORCH_CHECK(t.dim() == 1 && t.scalar_type() == at::kInt, name, " must be 1-D int32");
    return t.contiguous();
  };
  auto int2d = [](const at::Tensor& t, const char* name) {
    TORCH_CHECK(t.dim() == 2 && t.scalar_type() == at::kInt && t.stride(1) == 1, name,
                " must be 2-D int32 with unit column stride");
  };
  const at::Tensor idx = int1d(expanded_idx_mapping, "expanded_idx_mapping");
  const at::Tensor nbw = int1d(num_bad_words, "num_bad_words");
  const at::Tensor pl = int1d(prompt_len, "prompt_len");
  const at::Tensor tl = int1d(total_len, "total_len");
  const at::Tensor inp = int1d(input_ids, "input_ids");
  const at::Tensor lpos = int1d(expanded_local_pos, "expanded_local_pos");
  int2d(bad_word_token_ids, "bad_word_token_ids");
  int2d(bad_word_offsets, "bad_word_offsets");
  int2d(all_token_ids, "all_token_ids");
  const int64_t n = logits.size(0);
  TORCH_CHECK(idx.numel() >= n && inp.numel() >= n && lpos.numel() >= n,
              "vllm_bad_words_kernel: per-token tensors shorter than the rows");
  const int64_t reqs = std::min({nbw.numel(), pl.numel(), tl.numel(), bad_word_token_ids.size(0),
                                 bad_word_offsets.size(0), all_token_ids.size(0)});
  MCPU_OK(mcpu_vllm_bad_words(logits.data_ptr(), dt, n, logits.stride(0), logits.size(1),
                              idx.const_data_ptr<int32_t>(), reqs, bad_word_token_ids.const_data_ptr<int32_t>(),
                              bad_word_token_ids.stride(0), bad_word_token_ids.size(1),
                              bad_word_offsets.const_data_ptr<int32_t>(), bad_word_offsets.stride(0),
                              bad_word_offsets.size(1), nbw.const_data_ptr<int32_t>(),
                              all_token_ids.const_data_ptr<int32_t>(), all_token_ids.stride(0),
                              all_token_ids.size(1), pl.const_data_ptr<int32_t>(), tl.const_data_ptr<int32_t>(),
                              inp.const_data_ptr<int32_t>(), lpos.const_data_ptr<int32_t>(), stream_of(logits)),
          "vllm_bad_words_kernel");
}

// Row-parallel down projection + SUM all-reduce of the partials in one kernel
// (mm, csrc/aten/ops/mm.cpp:13-51, then McpuBackend::allreduce,
// torch_mcpu/csrc/Distributed.cpp:403-413).  `window` is the address of the
// mcpuSymmWindow a torch_mcpu_b200.symm.SymmetricWindow holds; the result is
// a view of this rank's window, valid until the next call on that window.
at::Tensor mm_allreduce(const at::Tensor& a, const at::Tensor& b, int64_t window) {
  TORCH_CHECK(a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16,
              "mm_allreduce: bfloat16 tensors expected");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && a.size(1) == b.size(1),
              "mm_allreduce: a [M, K] and b [N, K] expected");
  TORCH_CHECK(a.device() == b.device(), "mm_allreduce: a and b must be on one device");
  TORCH_CHECK(window != 0, "mm_allreduce: NULL window");
  const at::Tensor ac = a.contiguous(), bc = b.contiguous();
  void* out = nullptr;
  MCPU_OK(mcpu_mm_allreduce(ac.const_data_ptr(), bc.const_data_ptr(), ac.size(0), bc.size(0), ac.size(1),
                            MCPU_BFLOAT16, reinterpret_cast<const mcpuSymmWindow*>(window), &out,
                            stream_of(ac)),
          "mm_allreduce");
  return at::from_blob(out, {ac.size(0), bc.size(0)}, [](void*) {}, ac.options());
}

}  // namespace
}  // namespace mcpu_torch

TORCH_LIBRARY_IMPL(aten, PrivateUse1, m) {
  using namespace mcpu_torch;
  m.impl("empty.memory_format", empty_memory_format);
  m.impl("empty_strided", empty_strided);
  m.impl("as_strided", at::native::as_strided_tensorimpl);
  m.impl("view", at::native::view);
  m.impl("_reshape_alias", at::native::_reshape_alias);
  m.impl("resize_", resize_);
  m.impl("_copy_from", copy_from);
  m.impl("_copy_from_and_resize", copy_from_and_resize);
  m.impl("_local_scalar_dense", local_scalar_dense);
  m.impl("fill_.Scalar", fill_scalar);
  m.impl("zero_", zero_);
  m.impl("record_stream", record_stream_op);
  m.impl("mm", mm);
  m.impl("mm.out", mm_out);
  m.impl("addmm", addmm);
  m.impl("addmm.out", addmm_out);
  m.impl("sigmoid", sigmoid);
  m.impl("sigmoid.out", sigmoid_out);
  m.impl("silu", silu);
  m.impl("silu.out", silu_out);
  m.impl("add.Tensor", add);
  m.impl("add.out", add_out);
  m.impl("add_.Tensor", add_);
  m.impl("sub.Tensor", sub);
  m.impl("sub.out", sub_out);
  m.impl("mul.Tensor", mul);
  m.impl("mul.out", mul_out);
  m.impl("mul_.Tensor", mul_);
  m.impl("div.Tensor", div_tensor);
  m.impl("div.out", div_out);
  m.impl("div_.Tensor", div_);
  m.impl("neg", neg);
  m.impl("neg.out", neg_out);
  m.impl("abs", abs_tensor);
  m.impl("abs.out", abs_out);
  m.impl("rsqrt", rsqrt);
  m.impl("rsqrt.out", rsqrt_out);
  m.impl("sqrt", sqrt_tensor);
  m.impl("sqrt.out", sqrt_out);
  m.impl("bitwise_not", bitwise_not);
  m.impl("bitwise_not.out", bitwise_not_out);
  m.impl("pow.Tensor_Scalar", pow_scalar);
  m.impl("pow.Tensor_Scalar_out", pow_scalar_out);
  m.impl("masked_fill_.Scalar", masked_fill_);
  m.impl("masked_fill_.Tensor", masked_fill_tensor_);
  m.impl("sum.dim_IntList", sum_dim);
  m.impl("sum.IntList_out", sum_dim_out);
  m.impl("mean.dim", mean_dim);
  m.impl("max.dim", max_dim);
  m.impl("min.dim", min_dim);
  m.impl("topk", topk);
  m.impl("topk.values", topk_out);
  m.impl("_softmax", softmax_);
  m.impl("_softmax.out", softmax_out);
  m.impl("_log_softmax", log_softmax_);
  m.impl("gather", gather);
  m.impl("gather.out", gather_out);
  m.impl("scatter_.value", scatter_value_);
  m.impl("scatter.value", scatter_value);
  m.impl("scatter.value_out", scatter_value_out);
}

// The reference's TORCH_LIBRARY(mcpu) block (csrc/aten/OpenRegExtra.cpp:
// 147-162, registered in mcpu_extra.cpp) owns the namespace; the hot-path
// ops join it as a fragment.
TORCH_LIBRARY_FRAGMENT(mcpu, m) {
  m.def("grouped_topk(Tensor gating_output, int num_expert_group, int topk_group, int topk, "
        "bool renormalize, float routed_scaling_factor, Tensor? e_score_correction_bias, "
        "str scoring_func) -> (Tensor, Tensor)");
  m.def("silu_and_mul(Tensor(a!) out, Tensor x) -> ()");
  m.def("rms_norm(Tensor(a!) out, Tensor x, Tensor weight, float eps) -> ()");
  m.def("gemm_swiglu(Tensor x, Tensor w_gate_up_interleaved) -> Tensor");
  m.def("gemm_swiglu.out(Tensor x, Tensor w_gate_up_interleaved, *, Tensor(a!) out) -> Tensor(a!)");
  m.def("mm_allreduce(Tensor a, Tensor b, int window) -> Tensor");
  m.def("vllm_min_p_kernel(Tensor(a!) logits, Tensor expanded_idx_mapping, Tensor min_p, int vocab_size) -> ()");
  m.def("vllm_topk_log_softmax_kernel(Tensor(a!) output, Tensor logits, Tensor topk_ids, int topk, "
        "int vocab_size) -> ()");
  m.def("vllm_ranks_kernel(Tensor(a!) output, Tensor logits, Tensor token_ids, int vocab_size) -> ()");
  m.def("vllm_penalties_kernel(Tensor(a!) logits, Tensor expanded_idx_mapping, Tensor token_ids, "
        "Tensor expanded_local_pos, Tensor repetition_penalty, Tensor frequency_penalty, "
        "Tensor presence_penalty, Tensor prompt_bin_mask, Tensor output_bin_counts, int vocab_size, "
        "int max_spec_len) -> ()");
  m.def("vllm_bias_kernel(Tensor(a!) logits, int vocab_size, Tensor expanded_idx_mapping, "
        "Tensor num_allowed_token_ids, Tensor allowed_token_ids, Tensor num_logit_bias, Tensor bias_token_ids, "
        "Tensor bias, Tensor pos, Tensor min_lens, Tensor num_stop_token_ids, Tensor stop_token_ids) -> ()");
  m.def("vllm_bad_words_kernel(Tensor(a!) logits, Tensor expanded_idx_mapping, Tensor bad_word_token_ids, "
        "Tensor bad_word_offsets, Tensor num_bad_words, Tensor all_token_ids, Tensor prompt_len, "
        "Tensor total_len, Tensor input_ids, Tensor expanded_local_pos) -> ()");
  m.def("vllm_bincount_kernel(Tensor expanded_idx_mapping, Tensor all_token_ids, Tensor prompt_len, "
        "Tensor prefill_len, Tensor(a!) prompt_bin_mask, Tensor(b!) output_bin_counts) -> ()");
  m.def("moe_align_block_size(Tensor topk_ids, int num_experts, int block_size, Tensor(a!) sorted_token_ids, "
        "Tensor(b!) experts_ids, Tensor(c!) num_tokens_post_pad) -> ()");
}

TORCH_LIBRARY_IMPL(mcpu, PrivateUse1, m) {
  using namespace mcpu_torch;
  m.impl("grouped_topk", grouped_topk);
  m.impl("silu_and_mul", silu_and_mul);
  m.impl("rms_norm", rms_norm);
  m.impl("gemm_swiglu", gemm_swiglu);
  m.impl("gemm_swiglu.out", gemm_swiglu_out);
  m.impl("mm_allreduce", mm_allreduce);
  m.impl("vllm_min_p_kernel", vllm_min_p_kernel);
  m.impl("vllm_topk_log_softmax_kernel", vllm_topk_log_softmax_kernel);
  m.impl("vllm_ranks_kernel", vllm_ranks_kernel);
  m.impl("vllm_penalties_kernel", vllm_penalties_kernel);
  m.impl("vllm_bincount_kernel", vllm_bincount_kernel);
  m.impl("vllm_bias_kernel", vllm_bias_kernel);
  m.impl("vllm_bad_words_kernel", vllm_bad_words_kernel);
  m.impl("moe_align_block_size", moe_align_block_size);
}
