// ProcessGroupLowBit: the `lowbit` torch.distributed backend.
//
// Reference counterpart: cpp/include/process_group_lowbit.h:20-120 and
// cpp/src/process_group_lowbit.cc (a c10d::Backend that owns a
// ProcessGroupNCCL and runs an ATen pack -> NCCL alltoall -> ATen reduce ->
// NCCL allgather chain with a blocking post-hook).
//
// Here:
//   * CUDA low-bit collectives (all-reduce, and — unlike the reference, which
//     forwards them — reduce-scatter and all-gather) run as ONE fused sm_100a
//     kernel each over NVLink peer memory (LowBitComm), on a dedicated
//     high-priority communication stream ordered after the caller's stream;
//   * the returned Work completes through a CUDA-aware Future that is marked
//     complete in stream order right after the kernel, so DDP and
//     get_future().then(...) observe the finished output (the reference
//     returned the NCCL phase-1 future, process_group_lowbit.cc:42-44, so the
//     post-hook never ran through futures);
//   * CPU tensors (gloo inner backend) and CUDA groups without peer access use
//     a staged path with the reference's per-shard-scale semantics;
//   * every other collective is forwarded to the inner backend of the
//     tensor's device (gloo for CPU, NCCL for CUDA), including the ones the
//     reference left unimplemented (barrier, reduce, gather, scatter,
//     send/recv, coalesced variants).
#pragma once

#include <ATen/cuda/CUDAEvent.h>
#include <c10/cuda/CUDAStream.h>
#include <pybind11/pybind11.h>
#include <torch/csrc/distributed/c10d/Backend.hpp>
#include <torch/csrc/distributed/c10d/Store.hpp>
#include <torch/csrc/distributed/c10d/Types.hpp>
#include <torch/csrc/distributed/c10d/Work.hpp>

#include <chrono>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "../runtime/comm.h"

namespace bitscom_b200 {

struct LowBitOptions {
  // Reference options (cpp/include/process_group_lowbit.h:20-24).
  int bitwidth = 4;
  bool error_feedback = false;
  std::chrono::milliseconds timeout{600000};
  // Additions.
  bool stochastic_rounding = false;  // SR of the first quantisation
  bool fp8 = false;                  // 8-bit collectives use block-scaled E4M3
  bool force_lowbit = false;         // compress at 8/12/16 bits too (the reference forwards >=8 bits)
  int algo = 0;                      // 0 auto, 1 two-shot, 2 one-shot
  int64_t workspace_bytes = 256ll << 20;
  int max_ctas = 0;                  // 0 = one CTA per SM
  uint64_t seed = 0x5eed;
  bool blocking_wait = false;        // Work.wait() blocks the host and checks the kernel status
  int64_t oneshot_max_bytes = 512ll << 10;  // automatic algorithm: one-shot up to this packed size
  // Tuning-table entries for this world size: {bits, fmt, oneshot_max_bytes, ws_min_bytes}.
  std::vector<std::vector<int64_t>> tuning;
};

class WorkLowBit : public c10d::Work {
 public:
  // CUDA work: completes when `event` (recorded after the kernel) completes.
  WorkLowBit(int rank, c10d::OpType op, std::vector<at::Tensor> outputs, c10::Device device,
             std::shared_ptr<LowBitComm> comm, bool blocking_wait);
  // CPU / already-finished work.
  WorkLowBit(int rank, c10d::OpType op, std::vector<at::Tensor> outputs);

  bool isCompleted() override;
  bool isSuccess() const override;
  bool wait(std::chrono::milliseconds timeout = c10d::kUnsetTimeout) override;
  void synchronize() override;
  std::vector<at::Tensor> result() override { return outputs_; }
  c10::intrusive_ptr<c10::ivalue::Future> getFuture() override { return future_; }

  at::cuda::CUDAEvent& event() { return *event_; }
  void finish_cuda(c10::cuda::CUDAStream stream);  // record the event + complete the future

 private:
  std::vector<at::Tensor> outputs_;
  c10::Device device_;
  bool cuda_;
  std::shared_ptr<LowBitComm> comm_;
  std::shared_ptr<at::cuda::CUDAEvent> event_;
  c10::intrusive_ptr<c10::ivalue::Future> future_;
  bool blocking_wait_ = false;
};

class ProcessGroupLowBit : public c10d::Backend {
 public:
  ProcessGroupLowBit(const c10::intrusive_ptr<c10d::Store>& store, int rank, int size,
                     c10::intrusive_ptr<c10d::Backend> cpu_inner,
                     c10::intrusive_ptr<c10d::Backend> cuda_inner, LowBitOptions options);
  ~ProcessGroupLowBit() override;

  const std::string getBackendName() const override { return "lowbit"; }
  const LowBitOptions& options() const { return options_; }

  c10::intrusive_ptr<c10d::Work> allreduce(std::vector<at::Tensor>& tensors,
                                          const c10d::AllreduceOptions& opts = c10d::AllreduceOptions()) override;
  c10::intrusive_ptr<c10d::Work> allreduce_coalesced(
      std::vector<at::Tensor>& tensors,
      const c10d::AllreduceCoalescedOptions& opts = c10d::AllreduceCoalescedOptions()) override;
  c10::intrusive_ptr<c10d::Work> allgather(std::vector<std::vector<at::Tensor>>& outputs,
                                          std::vector<at::Tensor>& inputs,
                                          const c10d::AllgatherOptions& opts = c10d::AllgatherOptions()) override;
  c10::intrusive_ptr<c10d::Work> _allgather_base(at::Tensor& output, at::Tensor& input,
                                                const c10d::AllgatherOptions& opts = c10d::AllgatherOptions()) override;
  c10::intrusive_ptr<c10d::Work> allgather_coalesced(
      std::vector<std::vector<at::Tensor>>& outputs, std::vector<at::Tensor>& inputs,
      const c10d::AllgatherOptions& opts = c10d::AllgatherOptions()) override;
  c10::intrusive_ptr<c10d::Work> allgather_into_tensor_coalesced(
      std::vector<at::Tensor>& outputs, std::vector<at::Tensor>& inputs,
      const c10d::AllgatherOptions& opts = c10d::AllgatherOptions()) override;
  c10::intrusive_ptr<c10d::Work> reduce_scatter(
      std::vector<at::Tensor>& outputs, std::vector<std::vector<at::Tensor>>& inputs,
      const c10d::ReduceScatterOptions& opts = c10d::ReduceScatterOptions()) override;
  c10::intrusive_ptr<c10d::Work> _reduce_scatter_base(
      at::Tensor& output, at::Tensor& input,
      const c10d::ReduceScatterOptions& opts = c10d::ReduceScatterOptions()) override;
  c10::intrusive_ptr<c10d::Work> reduce_scatter_tensor_coalesced(
      std::vector<at::Tensor>& outputs, std::vector<at::Tensor>& inputs,
      const c10d::ReduceScatterOptions& opts = c10d::ReduceScatterOptions()) override;
  c10::intrusive_ptr<c10d::Work> broadcast(std::vector<at::Tensor>& tensors,
                                          const c10d::BroadcastOptions& opts = c10d::BroadcastOptions()) override;
  c10::intrusive_ptr<c10d::Work> reduce(std::vector<at::Tensor>& tensors,
                                       const c10d::ReduceOptions& opts = c10d::ReduceOptions()) override;
  c10::intrusive_ptr<c10d::Work> gather(std::vector<std::vector<at::Tensor>>& outputs,
                                       std::vector<at::Tensor>& inputs,
                                       const c10d::GatherOptions& opts = c10d::GatherOptions()) override;
  c10::intrusive_ptr<c10d::Work> scatter(std::vector<at::Tensor>& outputs,
                                        std::vector<std::vector<at::Tensor>>& inputs,
                                        const c10d::ScatterOptions& opts = c10d::ScatterOptions()) override;
  c10::intrusive_ptr<c10d::Work> alltoall(std::vector<at::Tensor>& outputs, std::vector<at::Tensor>& inputs,
                                         const c10d::AllToAllOptions& opts = c10d::AllToAllOptions()) override;
  c10::intrusive_ptr<c10d::Work> alltoall_base(at::Tensor& output, at::Tensor& input,
                                              std::vector<int64_t>& output_split_sizes,
                                              std::vector<int64_t>& input_split_sizes,
                                              const c10d::AllToAllOptions& opts = c10d::AllToAllOptions()) override;
  c10::intrusive_ptr<c10d::Work> send(std::vector<at::Tensor>& tensors, int dst, int tag) override;
  c10::intrusive_ptr<c10d::Work> recv(std::vector<at::Tensor>& tensors, int src, int tag) override;
  c10::intrusive_ptr<c10d::Work> recvAnysource(std::vector<at::Tensor>& tensors, int tag) override;
  c10::intrusive_ptr<c10d::Work> barrier(const c10d::BarrierOptions& opts = c10d::BarrierOptions()) override;
  void setSequenceNumberForGroup() override;
  uint64_t getSequenceNumberForGroup() override;
  void setTimeout(std::chrono::milliseconds timeout) override { options_.timeout = timeout; }
  // destroy_process_group(): shut the inner backends down and release the
  // fused-path workspaces now, not whenever the last Python reference to this
  // backend goes away (by then the peers may have exited).
  void shutdown() override;
  void abort() override;

  // Introspection (exposed to Python).
  std::map<std::string, int64_t> stats() const;
  int64_t residual_count() const;
  void clear_residuals();
  // Fused-path communicator of `device` (created on first use; collective).
  std::shared_ptr<LowBitComm> comm(int device);
  bool p2p_available(int device);

 private:
  bool use_lowbit_reduce(c10d::ReduceOp op) const;
  bool use_lowbit_gather() const;
  int wire_bits() const { return options_.bitwidth; }
  int wire_fmt() const { return (options_.fp8 && options_.bitwidth == 8) ? 1 : 0; }
  c10::intrusive_ptr<c10d::Backend> inner(const at::Tensor& t) const;
  c10::intrusive_ptr<c10d::Backend> inner_any() const;
  c10::cuda::CUDAStream comm_stream(int device);
  enum class ResidualKind : int { kAllReduce = 0, kReduceScatter = 1, kAllGather = 2 };
  at::Tensor residual_for(const at::Tensor& key, int64_t numel, c10::Device dev, ResidualKind kind);
  void surface_errors();

  c10::intrusive_ptr<c10d::Work> allreduce_fused(std::vector<at::Tensor>& tensors);
  c10::intrusive_ptr<c10d::Work> allreduce_staged(std::vector<at::Tensor>& tensors);
  c10::intrusive_ptr<c10d::Work> reduce_scatter_fused(at::Tensor& output, at::Tensor& input, float post_scale);
  c10::intrusive_ptr<c10d::Work> allgather_fused(at::Tensor& output, at::Tensor& input);

  c10::intrusive_ptr<c10d::Store> store_;
  c10::intrusive_ptr<c10d::Backend> cpu_inner_, cuda_inner_;
  LowBitOptions options_;
  std::mutex mu_;
  std::unordered_map<int, std::shared_ptr<LowBitComm>> comms_;
  std::unordered_map<int, bool> p2p_ok_;
  std::unordered_map<int, c10::cuda::CUDAStream> streams_;
  // Error-feedback residuals with their last use (see residual_for for the
  // keys); at most kMaxResiduals, least recently used dropped first.
  static constexpr size_t kMaxResiduals = 1024;
  std::unordered_map<int64_t, std::pair<at::Tensor, uint64_t>> residuals_;
  uint64_t residual_clock_ = 0;
  std::vector<c10::intrusive_ptr<WorkLowBit>> recent_;  // for early error surfacing
  uint64_t sr_calls_ = 0;
  int comm_generation_ = 0;
  int64_t fused_calls_ = 0, staged_calls_ = 0, forwarded_calls_ = 0;
};

c10::intrusive_ptr<c10d::Backend> createProcessGroupLowBit(
    const c10::intrusive_ptr<c10d::Store>& store, int rank, int size,
    c10::intrusive_ptr<c10d::Backend> cpu_inner, c10::intrusive_ptr<c10d::Backend> cuda_inner,
    const LowBitOptions& options);

void register_backend_bindings(pybind11::module& m);

}  // namespace bitscom_b200
