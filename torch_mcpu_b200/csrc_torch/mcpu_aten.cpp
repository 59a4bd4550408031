// Dispatcher registrations of the mcpu (PrivateUse1) device on B200.
//
// The minimal tensor set of the reference (csrc/aten/OpenRegMinimal.cpp:
// 150-167) plus the hot-path aten ops (mm/addmm: csrc/aten/ops/mm.cpp:115-120;
// sigmoid/silu: unary_out.cpp:817-836; mul: binary_out.cpp:757-828) and the
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

at::Tensor& mul_out(const at::Tensor& self, const at::Tensor& other, at::Tensor& out) {
  TORCH_CHECK(self.sizes() == other.sizes() && self.scalar_type() == other.scalar_type(),
              "mul on mcpu (B200): same-shape, same-dtype operands only");
  TORCH_CHECK(self.scalar_type() == at::kFloat || self.scalar_type() == at::kBFloat16,
              "mul on mcpu (B200): float32 or bfloat16 only");
  TORCH_CHECK(out.sizes() == self.sizes() && out.scalar_type() == self.scalar_type(), "mul.out: out must match");
  const at::Tensor a = self.contiguous(), b = other.contiguous();
  at::Tensor o = out.is_contiguous() ? out : at::empty(out.sizes(), out.options());
  MCPU_OK(mcpu_mul(o.data_ptr(), a.const_data_ptr(), b.const_data_ptr(), a.numel(),
                   dtype_code(a.scalar_type()), stream_of(o)),
          "mul");
  if (!o.is_same(out)) strided_copy(o, out);
  return out;
}
at::Tensor mul(const at::Tensor& self, const at::Tensor& other) {
  at::Tensor out = at::empty(self.sizes(), self.options());
  return mul_out(self, other, out);
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

at::Tensor gemm_swiglu(const at::Tensor& x, const at::Tensor& w_gate_up) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w_gate_up.scalar_type() == at::kBFloat16,
              "gemm_swiglu: bfloat16 tensors expected");
  const at::Tensor a = x.contiguous(), w = w_gate_up.contiguous();
  at::Tensor out = at::empty({a.size(0), w.size(0) / 2}, a.options());
  MCPU_OK(mcpu_gemm_swiglu(a.const_data_ptr(), w.const_data_ptr(), out.data_ptr(), a.size(0), w.size(0) / 2,
                           a.size(1), MCPU_BFLOAT16, stream_of(a)),
          "gemm_swiglu");
  return out;
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
  m.impl("mul.Tensor", mul);
  m.impl("mul.out", mul_out);
}

// The reference's TORCH_LIBRARY(mcpu) block (csrc/aten/OpenRegExtra.cpp:
// 147-162) owns the namespace; the hot-path ops join it as a fragment.
TORCH_LIBRARY_FRAGMENT(mcpu, m) {
  m.def("grouped_topk(Tensor gating_output, int num_expert_group, int topk_group, int topk, "
        "bool renormalize, float routed_scaling_factor, Tensor? e_score_correction_bias, "
        "str scoring_func) -> (Tensor, Tensor)");
  m.def("silu_and_mul(Tensor(a!) out, Tensor x) -> ()");
  m.def("rms_norm(Tensor(a!) out, Tensor x, Tensor weight, float eps) -> ()");
  m.def("gemm_swiglu(Tensor x, Tensor w_gate_up_interleaved) -> Tensor");
}

TORCH_LIBRARY_IMPL(mcpu, PrivateUse1, m) {
  using namespace mcpu_torch;
  m.impl("grouped_topk", grouped_topk);
  m.impl("silu_and_mul", silu_and_mul);
  m.impl("rms_norm", rms_norm);
  m.impl("gemm_swiglu", gemm_swiglu);
}
