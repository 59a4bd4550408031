// c10d Backend "mcpu" over NCCL (NVLink / NVSwitch on a B200 box).
//
// Replaces McpuBackend of the reference (torch_mcpu/csrc/Distributed.cpp:
// 248-751), which stages mcpu tensors to the CPU and runs Gloo on a detached
// host thread.  Here every collective is one NCCL call enqueued on the current
// mcpu stream of the tensor's device; Work records an event behind it.
//   creator      _create_process_group_mcpu(store, rank, size, timeout)
//                (Distributed.cpp:759-788)
//   Work::wait   with a timeout, polls the event and throws "Operation timed
//                out!" after the deadline, aborting the communicator
//                (Distributed.cpp:191-224); without one, the caller's current
//                stream waits on the event (no host block)
// Collectives: allreduce (sum/avg/min/max/product), broadcast,
// allgather_into_tensor (_allgather_base), reduce_scatter_tensor
// (_reduce_scatter_base), barrier.  Others raise, as unsupported.
#include <torch/csrc/distributed/c10d/Backend.hpp>
#include <torch/csrc/distributed/c10d/Store.hpp>
#include <torch/csrc/distributed/c10d/Types.hpp>
#include <torch/csrc/distributed/c10d/Work.hpp>
#include <torch/csrc/utils/pybind.h>

#include <pybind11/chrono.h>

#include <ATen/ATen.h>
#include <c10/util/Exception.h>

#include <nccl.h>

#include <chrono>
#include <mutex>
#include <thread>
#include <vector>

#include "mcpu_torch.h"

namespace mcpu_torch {

#define NCCL_OK(expr)                                                                     \
  do {                                                                                    \
    ncclResult_t _r = (expr);                                                             \
    TORCH_CHECK(_r == ncclSuccess, "NCCL error ", ncclGetErrorString(_r), " in ", #expr); \
  } while (0)

static ncclDataType_t nccl_dtype(at::ScalarType t) {
  switch (t) {
    case at::kFloat: return ncclFloat32;
    case at::kBFloat16: return ncclBfloat16;
    case at::kHalf: return ncclFloat16;
    case at::kDouble: return ncclFloat64;
    case at::kInt: return ncclInt32;
    case at::kLong: return ncclInt64;
    case at::kByte:
    case at::kBool: return ncclUint8;
    case at::kChar: return ncclInt8;
    default: TORCH_CHECK(false, "mcpu ProcessGroup: unsupported dtype ", t);
  }
}

static ncclRedOp_t nccl_op(const c10d::ReduceOp& op) {
  switch (op) {
    case c10d::ReduceOp::SUM: return ncclSum;
    case c10d::ReduceOp::AVG: return ncclAvg;
    case c10d::ReduceOp::MIN: return ncclMin;
    case c10d::ReduceOp::MAX: return ncclMax;
    case c10d::ReduceOp::PRODUCT: return ncclProd;
    default: TORCH_CHECK(false, "mcpu ProcessGroup: unsupported reduce op");
  }
}

class McpuWork : public c10d::Work {
 public:
  McpuWork(int rank, c10d::OpType type, orEvent_t ev, ncclComm_t comm, std::vector<at::Tensor> outputs,
           std::chrono::milliseconds default_timeout)
      : c10d::Work(rank, type), ev_(ev), comm_(comm), outputs_(std::move(outputs)),
        default_timeout_(default_timeout) {}
  ~McpuWork() override {
    if (ev_) orEventDestroy(ev_);
  }
  bool isCompleted() override { return orEventQuery(ev_) == orSuccess; }
  bool isSuccess() const override { return !failed_; }
  std::exception_ptr exception() const override { return exc_; }
  std::vector<at::Tensor> result() override { return outputs_; }
  void synchronize() override { orEventSynchronize(ev_); }
  bool wait(std::chrono::milliseconds timeout) override {
    if (timeout == kNoTimeout) {
      // like NCCL in PyTorch: the caller's current stream waits on the work
      const c10::DeviceIndex dev = outputs_.empty() ? current_device() : outputs_[0].device().index();
      TORCH_CHECK(orStreamWaitEvent(current_stream_handle(dev), ev_, 0) == orSuccess,
                  "mcpu Work::wait: ", mcpuGetLastErrorString());
      return true;
    }
    const auto deadline = std::chrono::steady_clock::now() + timeout;
    while (orEventQuery(ev_) == orErrorNotReady) {
      if (std::chrono::steady_clock::now() > deadline) {
        failed_ = true;
        ncclCommAbort(comm_);
        exc_ = std::make_exception_ptr(std::runtime_error("Operation timed out!"));
        TORCH_CHECK(false, "Operation timed out!");
      }
      std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
    return true;
  }
  void abort() override { ncclCommAbort(comm_); }

 private:
  orEvent_t ev_;
  ncclComm_t comm_;
  std::vector<at::Tensor> outputs_;
  std::chrono::milliseconds default_timeout_;
  bool failed_ = false;
  std::exception_ptr exc_;
};

class McpuNcclBackend : public c10d::Backend {
 public:
  McpuNcclBackend(const c10::intrusive_ptr<c10d::Store>& store, int rank, int size,
                  std::chrono::milliseconds timeout)
      : c10d::Backend(rank, size), store_(store), timeout_(timeout) {
    device_ = current_device();
    ncclUniqueId id;
    const std::string key = "mcpu_nccl_unique_id";
    if (rank == 0) {
      NCCL_OK(ncclGetUniqueId(&id));
      const auto* b = reinterpret_cast<const uint8_t*>(&id);
      store_->set(key, std::vector<uint8_t>(b, b + sizeof(id)));
    } else {
      const std::vector<uint8_t> v = store_->get(key);
      TORCH_CHECK(v.size() == sizeof(id), "mcpu ProcessGroup: bad NCCL id from the store");
      std::memcpy(&id, v.data(), sizeof(id));
    }
    NCCL_OK(ncclCommInitRank(&comm_, size, id, rank));
  }
  ~McpuNcclBackend() override {
    if (comm_) ncclCommDestroy(comm_);
  }
  const std::string getBackendName() const override { return "mcpu"; }

  c10::intrusive_ptr<c10d::Work> allreduce(std::vector<at::Tensor>& tensors,
                                           const c10d::AllreduceOptions& opts) override {
    TORCH_CHECK(tensors.size() == 1, "mcpu ProcessGroup: one tensor per collective");
    at::Tensor& t = tensors[0];
    check(t);
    orStream_t st = stream_for(t);
    NCCL_OK(ncclAllReduce(t.data_ptr(), t.data_ptr(), t.numel(), nccl_dtype(t.scalar_type()),
                          nccl_op(opts.reduceOp), comm_, reinterpret_cast<cudaStream_t>(st)));
    return finish(c10d::OpType::ALLREDUCE, st, tensors);
  }

  c10::intrusive_ptr<c10d::Work> broadcast(std::vector<at::Tensor>& tensors,
                                           const c10d::BroadcastOptions& opts) override {
    TORCH_CHECK(tensors.size() == 1, "mcpu ProcessGroup: one tensor per collective");
    at::Tensor& t = tensors[0];
    check(t);
    orStream_t st = stream_for(t);
    NCCL_OK(ncclBroadcast(t.data_ptr(), t.data_ptr(), t.numel(), nccl_dtype(t.scalar_type()),
                          static_cast<int>(opts.rootRank), comm_, reinterpret_cast<cudaStream_t>(st)));
    return finish(c10d::OpType::BROADCAST, st, tensors);
  }

  c10::intrusive_ptr<c10d::Work> _allgather_base(at::Tensor& output, at::Tensor& input,
                                                 const c10d::AllgatherOptions&) override {
    check(input);
    check(output);
    TORCH_CHECK(output.numel() == input.numel() * getSize(), "allgather_into_tensor: size mismatch");
    orStream_t st = stream_for(input);
    NCCL_OK(ncclAllGather(input.data_ptr(), output.data_ptr(), input.numel(), nccl_dtype(input.scalar_type()),
                          comm_, reinterpret_cast<cudaStream_t>(st)));
    std::vector<at::Tensor> outs{output};
    return finish(c10d::OpType::_ALLGATHER_BASE, st, outs);
  }

  c10::intrusive_ptr<c10d::Work> _reduce_scatter_base(at::Tensor& output, at::Tensor& input,
                                                      const c10d::ReduceScatterOptions& opts) override {
    check(input);
    check(output);
    TORCH_CHECK(input.numel() == output.numel() * getSize(), "reduce_scatter_tensor: size mismatch");
    orStream_t st = stream_for(input);
    NCCL_OK(ncclReduceScatter(input.data_ptr(), output.data_ptr(), output.numel(),
                              nccl_dtype(input.scalar_type()), nccl_op(opts.reduceOp), comm_,
                              reinterpret_cast<cudaStream_t>(st)));
    std::vector<at::Tensor> outs{output};
    return finish(c10d::OpType::_REDUCE_SCATTER_BASE, st, outs);
  }

  c10::intrusive_ptr<c10d::Work> barrier(const c10d::BarrierOptions&) override {
    at::Tensor t = at::zeros({1}, at::TensorOptions().dtype(at::kFloat)).to(
        at::Device(c10::DeviceType::PrivateUse1, device_));
    std::vector<at::Tensor> v{t};
    auto w = allreduce(v, c10d::AllreduceOptions());
    TORCH_CHECK(orEventSynchronize(last_event_) == orSuccess, "barrier: ", mcpuGetLastErrorString());
    return w;
  }

 private:
  void check(const at::Tensor& t) const {
    TORCH_CHECK(t.device().type() == c10::DeviceType::PrivateUse1,
                "mcpu ProcessGroup: tensors must be on the mcpu device, got ", t.device());
    TORCH_CHECK(t.is_contiguous(), "mcpu ProcessGroup: contiguous tensors only");
  }
  orStream_t stream_for(const at::Tensor& t) const { return current_stream_handle(t.device().index()); }
  c10::intrusive_ptr<c10d::Work> finish(c10d::OpType type, orStream_t st, std::vector<at::Tensor>& outs) {
    orEvent_t ev = nullptr;
    TORCH_CHECK(orEventCreateWithFlags(&ev, orEventDisableTiming) == orSuccess && orEventRecord(ev, st) == orSuccess,
                "mcpu ProcessGroup: ", mcpuGetLastErrorString());
    last_event_ = ev;
    return c10::make_intrusive<McpuWork>(getRank(), type, ev, comm_, outs, timeout_);
  }

  c10::intrusive_ptr<c10d::Store> store_;
  std::chrono::milliseconds timeout_;
  c10::DeviceIndex device_ = 0;
  ncclComm_t comm_ = nullptr;
  orEvent_t last_event_ = nullptr;
};

void bind_distributed(pybind11::module& m) {
  namespace py = pybind11;
  py::class_<McpuNcclBackend, c10d::Backend, c10::intrusive_ptr<McpuNcclBackend>>(m, "McpuBackend");
  // dist.Backend.register_backend("mcpu", create_process_group_mcpu,
  // devices=["mcpu"]) calls this with (store, rank, size, timeout)
  m.def(
      "create_process_group_mcpu",
      [](const c10::intrusive_ptr<c10d::Store>& store, int rank, int size, std::chrono::milliseconds timeout) {
        return c10::make_intrusive<McpuNcclBackend>(store, rank, size, timeout);
      },
      py::arg("store"), py::arg("rank"), py::arg("size"), py::arg("timeout"),
      py::call_guard<py::gil_scoped_release>());
}

}  // namespace mcpu_torch
