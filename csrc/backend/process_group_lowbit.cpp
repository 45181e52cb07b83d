// ProcessGroupLowBit implementation (see process_group_lowbit.h).
#include "process_group_lowbit.h"

#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <ATen/record_function.h>
#include <c10/cuda/CUDACachingAllocator.h>
#include <c10/cuda/CUDAGuard.h>
#include <pybind11/chrono.h>
#include <pybind11/stl.h>
#include <torch/csrc/distributed/c10d/PrefixStore.hpp>
#include <torch/extension.h>
#include <unistd.h>

#include <cstdlib>
#include <stdexcept>

namespace bitscom_b200 {
namespace {

std::pair<int, int> quant_bounds(int bits) {
  if (bits == 1) return {0, 1};
  return {-(1 << (bits - 1)), (1 << (bits - 1)) - 1};
}

DType dt_of(at::ScalarType t) {
  switch (t) {
    case at::kFloat: return kF32;
    case at::kBFloat16: return kBF16;
    case at::kHalf: return kF16;
    default: TORCH_CHECK(false, "bitscom: unsupported dtype ", t);
  }
}

bool fused_dtype(const at::Tensor& t) {
  const auto s = t.scalar_type();
  return s == at::kFloat || s == at::kBFloat16 || s == at::kHalf;
}

// Reference-layout byte packing with ATen ops (staged path; bits in {1,2,4,8}).
// codes: [rows, m] int32 offsets in [0, 2^bits).  Returns [rows, bytes] uint8.
at::Tensor pack_rows(const at::Tensor& codes, int bits) {
  const int per = 8 / bits;
  const int64_t rows = codes.size(0), m = codes.size(1);
  const int64_t pad = (per - m % per) % per;
  at::Tensor c = pad ? at::cat({codes, at::zeros({rows, pad}, codes.options())}, 1) : codes;
  c = c.view({rows, -1, per});
  auto shifts = at::arange(per, codes.options()) * bits;
  return at::bitwise_left_shift(c, shifts).sum(-1).to(at::kByte);
}

at::Tensor unpack_rows(const at::Tensor& packed, int bits, int64_t m) {
  const int per = 8 / bits;
  auto p = packed.to(at::kInt).unsqueeze(-1);
  auto shifts = at::arange(per, p.options()) * bits;
  auto v = at::bitwise_and(at::bitwise_right_shift(p, shifts), (1 << bits) - 1);
  return v.reshape({packed.size(0), -1}).narrow(1, 0, m);
}

std::string hostname() {
  char buf[256] = {0};
  gethostname(buf, sizeof(buf) - 1);
  return std::string(buf);
}

std::vector<uint8_t> to_bytes(const std::string& s) { return std::vector<uint8_t>(s.begin(), s.end()); }
std::string to_string(const std::vector<uint8_t>& v) { return std::string(v.begin(), v.end()); }

}  // namespace

// ============================================================================
// WorkLowBit
// ============================================================================
WorkLowBit::WorkLowBit(int rank, c10d::OpType op, std::vector<at::Tensor> outputs, c10::Device device,
                       std::shared_ptr<LowBitComm> comm, bool blocking_wait)
    : c10d::Work(rank, op),
      outputs_(std::move(outputs)),
      device_(device),
      cuda_(true),
      comm_(std::move(comm)),
      event_(std::make_shared<at::cuda::CUDAEvent>(cudaEventDisableTiming)),
      blocking_wait_(blocking_wait) {
  future_ = c10::make_intrusive<c10::ivalue::Future>(c10::ListType::create(c10::TensorType::get()),
                                                     std::vector<c10::Device>{device_});
}

WorkLowBit::WorkLowBit(int rank, c10d::OpType op, std::vector<at::Tensor> outputs)
    : c10d::Work(rank, op), outputs_(std::move(outputs)), device_(c10::kCPU), cuda_(false) {
  future_ = c10::make_intrusive<c10::ivalue::Future>(c10::ListType::create(c10::TensorType::get()));
  future_->markCompleted(c10::IValue(outputs_));
}

void WorkLowBit::finish_cuda(c10::cuda::CUDAStream stream) {
  event_->record(stream);
  c10::cuda::CUDAStreamGuard g(stream);
  future_->markCompleted(c10::IValue(outputs_));
}

bool WorkLowBit::isCompleted() { return !cuda_ || event_->query(); }

bool WorkLowBit::isSuccess() const {
  if (!cuda_) return true;
  if (!event_->query()) return false;
  return comm_ == nullptr || comm_->status() == kStatusOk;
}

void WorkLowBit::synchronize() {
  if (!cuda_) return;
  event_->block(c10::cuda::getCurrentCUDAStream(device_.index()));
}

bool WorkLowBit::wait(std::chrono::milliseconds timeout) {
  if (!cuda_) return true;
  synchronize();
  // kNoTimeout (0) and kUnsetTimeout (-1) both mean "no host-side limit".
  const bool bounded = timeout.count() > 0;
  if (blocking_wait_ || bounded) {
    const auto t0 = std::chrono::steady_clock::now();
    while (!event_->query()) {
      if (bounded && std::chrono::steady_clock::now() - t0 > timeout)
        TORCH_CHECK(false, "bitscom: Work.wait timed out after ", timeout.count(), " ms");
      std::this_thread::yield();
    }
    if (comm_) comm_->check();
  }
  return true;
}

// ============================================================================
// ProcessGroupLowBit
// ============================================================================
ProcessGroupLowBit::ProcessGroupLowBit(const c10::intrusive_ptr<c10d::Store>& store, int rank, int size,
                                       c10::intrusive_ptr<c10d::Backend> cpu_inner,
                                       c10::intrusive_ptr<c10d::Backend> cuda_inner, LowBitOptions options)
    : c10d::Backend(rank, size),
      store_(store),
      cpu_inner_(std::move(cpu_inner)),
      cuda_inner_(std::move(cuda_inner)),
      options_(std::move(options)) {
  TORCH_CHECK(options_.bitwidth == 1 || options_.bitwidth == 2 || options_.bitwidth == 4 ||
                  options_.bitwidth == 8 || options_.bitwidth == 12 || options_.bitwidth == 16,
              "bitscom: bitwidth must be one of (1, 2, 4, 8, 12, 16), got ", options_.bitwidth);
  TORCH_CHECK(cpu_inner_ || cuda_inner_, "bitscom: ProcessGroupLowBit needs an inner backend");
  if (const char* lvl = std::getenv("BITSCOM_LOG_LEVEL")) {
    if (std::string(lvl) == "INFO" || std::string(lvl) == "DEBUG")
      LOG(INFO) << "[bitscom] ProcessGroupLowBit rank=" << rank << " size=" << size
                << " bitwidth=" << options_.bitwidth << " error_feedback=" << options_.error_feedback;
  }
}

ProcessGroupLowBit::~ProcessGroupLowBit() = default;

void ProcessGroupLowBit::shutdown() {
  {
    std::lock_guard<std::mutex> lk(mu_);
    recent_.clear();
    comms_.clear();
    p2p_ok_.clear();
    residuals_.clear();
  }
  if (cuda_inner_) cuda_inner_->shutdown();
  if (cpu_inner_) cpu_inner_->shutdown();
  cuda_inner_.reset();
  cpu_inner_.reset();
}

void ProcessGroupLowBit::abort() {
  if (cuda_inner_) cuda_inner_->abort();
  if (cpu_inner_) cpu_inner_->abort();
  shutdown();
}

c10::intrusive_ptr<c10d::Backend> ProcessGroupLowBit::inner(const at::Tensor& t) const {
  if (t.is_cuda()) {
    TORCH_CHECK(cuda_inner_, "bitscom: no CUDA inner backend for a CUDA tensor");
    return cuda_inner_;
  }
  TORCH_CHECK(cpu_inner_, "bitscom: no CPU inner backend for a CPU tensor");
  return cpu_inner_;
}

c10::intrusive_ptr<c10d::Backend> ProcessGroupLowBit::inner_any() const { return cuda_inner_ ? cuda_inner_ : cpu_inner_; }

bool ProcessGroupLowBit::use_lowbit_reduce(c10d::ReduceOp op) const {
  const bool sum_like = op == c10d::ReduceOp::SUM || op == c10d::ReduceOp::AVG;
  if (!sum_like) return false;
  return options_.bitwidth < 8 || options_.force_lowbit || (options_.fp8 && options_.bitwidth == 8);
}

bool ProcessGroupLowBit::use_lowbit_gather() const {
  return options_.bitwidth < 8 || options_.force_lowbit || (options_.fp8 && options_.bitwidth == 8);
}

c10::cuda::CUDAStream ProcessGroupLowBit::comm_stream(int device) {
  std::lock_guard<std::mutex> lk(mu_);
  auto it = streams_.find(device);
  if (it == streams_.end())
    it = streams_.emplace(device, c10::cuda::getStreamFromPool(/*isHighPriority=*/true, device)).first;
  return it->second;
}

bool ProcessGroupLowBit::p2p_available(int device) {
  comm(device);
  std::lock_guard<std::mutex> lk(mu_);
  return p2p_ok_[device];
}

std::shared_ptr<LowBitComm> ProcessGroupLowBit::comm(int device) {
  {
    std::lock_guard<std::mutex> lk(mu_);
    auto it = p2p_ok_.find(device);
    if (it != p2p_ok_.end()) return it->second ? comms_[device] : nullptr;
  }
  // Collective rendezvous over the store: publish host / device / IPC handle,
  // try to map every peer, then agree on the outcome (all or nothing).
  const int W = getSize(), R = getRank();
  // Keyed by how many communicators this backend created so far (identical on
  // every rank), not by the device index (which differs between ranks).
  const std::string gen = "bitscom_lowbit/" + std::to_string(comm_generation_++);
  std::shared_ptr<LowBitComm> c;
  std::string err;
  try {
    int64_t ws = options_.workspace_bytes;
    if (const char* mb = std::getenv("BITSCOM_WORKSPACE_MB")) ws = std::atoll(mb) << 20;
    c = std::make_shared<LowBitComm>(R, W, device, ws);
    c->set_timeout_ms(static_cast<double>(options_.timeout.count()));
    c->set_oneshot_max_bytes(options_.oneshot_max_bytes);
    for (const auto& e : options_.tuning)
      if (e.size() == 4) c->set_tuning(static_cast<int>(e[0]), static_cast<int>(e[1]), e[2], e[3]);
    if (const char* t = std::getenv("BITSCOM_TIMEOUT_MS")) c->set_timeout_ms(std::atof(t));
  } catch (const std::exception& e) {
    err = e.what();
  }
  std::string info = hostname() + "|" + std::to_string(device) + "|";
  if (c) {
    auto h = c->ipc_handle();
    info += std::string(h.begin(), h.end());
  }
  store_->set(gen + "/info/" + std::to_string(R), to_bytes(info));
  bool ok = c != nullptr;
  std::vector<std::vector<uint8_t>> handles(W);
  const std::string host = hostname();
  for (int r = 0; r < W && ok; ++r) {
    const std::string s = to_string(store_->get(gen + "/info/" + std::to_string(r)));
    const auto p1 = s.find('|');
    const auto p2 = s.find('|', p1 + 1);
    if (p1 == std::string::npos || p2 == std::string::npos) { ok = false; break; }
    const std::string h = s.substr(0, p1);
    const int pdev = std::atoi(s.substr(p1 + 1, p2 - p1 - 1).c_str());
    const std::string handle = s.substr(p2 + 1);
    if (h != host || handle.size() != sizeof(cudaIpcMemHandle_t)) { ok = false; break; }
    if (r != R) {
      int can = 0;
      if (pdev == device) { ok = false; break; }  // two ranks on one GPU: never spin across them
      cudaDeviceCanAccessPeer(&can, device, pdev);
      if (!can) { ok = false; break; }
    }
    handles[r] = std::vector<uint8_t>(handle.begin(), handle.end());
  }
  if (ok) {
    try {
      c->open_peers(handles);
    } catch (const std::exception& e) {
      ok = false;
      err = e.what();
    }
  }
  store_->set(gen + "/ok/" + std::to_string(R), to_bytes(ok ? "1" : "0"));
  bool all_ok = true;
  for (int r = 0; r < W; ++r) all_ok = all_ok && to_string(store_->get(gen + "/ok/" + std::to_string(r))) == "1";
  if (!all_ok && W > 1 && std::getenv("BITSCOM_LOG_LEVEL"))
    LOG(WARNING) << "[bitscom] peer-to-peer workspace unavailable on rank " << R
                 << " (" << (err.empty() ? "a peer is unreachable" : err) << "); using the staged path";
  std::lock_guard<std::mutex> lk(mu_);
  p2p_ok_[device] = all_ok;
  if (all_ok) comms_[device] = c;
  return all_ok ? c : nullptr;
}

at::Tensor ProcessGroupLowBit::residual_for(const at::Tensor& key, int64_t numel, c10::Device dev, ResidualKind kind) {
  // All-reduce: keyed by the tensor (TensorImpl address), as the reference's
  // residual cache (cpp/include/process_group_lowbit.h:117-119) keys it.
  // Reduce-scatter / all-gather: keyed by (kind, buffer address), since
  // sharded data parallel (e.g. FSDP2) passes a freshly created flat tensor
  // over the same, allocator-reused buffer every step.
  const int64_t k = kind == ResidualKind::kAllReduce
                        ? static_cast<int64_t>(reinterpret_cast<uintptr_t>(key.unsafeGetTensorImpl()))
                        : static_cast<int64_t>(reinterpret_cast<uintptr_t>(key.data_ptr()) ^
                                               (static_cast<uint64_t>(kind) << 56));
  std::lock_guard<std::mutex> lk(mu_);
  const uint64_t now = ++residual_clock_;
  auto it = residuals_.find(k);
  if (it == residuals_.end() || it->second.first.numel() != numel || it->second.first.device() != dev) {
    if (it == residuals_.end() && residuals_.size() >= kMaxResiduals) {
      // Bound the cache: drop the least recently used residual.
      auto victim = residuals_.begin();
      for (auto jt = residuals_.begin(); jt != residuals_.end(); ++jt)
        if (jt->second.second < victim->second.second) victim = jt;
      residuals_.erase(victim);
    }
    auto r = at::zeros({numel}, at::TensorOptions().dtype(at::kFloat).device(dev));
    residuals_[k] = {r, now};
    return r;
  }
  it->second.second = now;
  return it->second.first;
}

int64_t ProcessGroupLowBit::residual_count() const { return static_cast<int64_t>(residuals_.size()); }

void ProcessGroupLowBit::clear_residuals() {
  std::lock_guard<std::mutex> lk(mu_);
  residuals_.clear();
}

std::map<std::string, int64_t> ProcessGroupLowBit::stats() const {
  std::map<std::string, int64_t> m;
  m["fused_calls"] = fused_calls_;
  m["staged_calls"] = staged_calls_;
  m["forwarded_calls"] = forwarded_calls_;
  m["residuals"] = static_cast<int64_t>(residuals_.size());
  for (const auto& kv : comms_) {
    const auto& s = kv.second->stats();
    const std::string p = "cuda" + std::to_string(kv.first) + ".";
    m[p + "launches"] = static_cast<int64_t>(s.launches);
    m[p + "wire_bytes"] = static_cast<int64_t>(s.wire_bytes);
    m[p + "elements"] = static_cast<int64_t>(s.elements);
    m[p + "oneshot"] = static_cast<int64_t>(s.oneshot);
    m[p + "twoshot"] = static_cast<int64_t>(s.twoshot);
  }
  return m;
}

void ProcessGroupLowBit::surface_errors() {
  // Raise, at the next call, a timeout reported by an earlier fused launch.
  std::vector<c10::intrusive_ptr<WorkLowBit>> keep;
  for (auto& w : recent_) {
    if (w->isCompleted()) {
      if (!w->isSuccess()) {
        recent_.clear();
        for (auto& kv : comms_) kv.second->check();
      }
    } else {
      keep.push_back(w);
    }
  }
  recent_.swap(keep);
}

// ---------------------------------------------------------------------------
// all-reduce
// ---------------------------------------------------------------------------
c10::intrusive_ptr<c10d::Work> ProcessGroupLowBit::allreduce(std::vector<at::Tensor>& tensors,
                                                            const c10d::AllreduceOptions& opts) {
  RECORD_FUNCTION("lowbit:allreduce", std::vector<c10::IValue>());
  if (tensors.empty() || !use_lowbit_reduce(opts.reduceOp) ||
      (getSize() == 1 && !options_.error_feedback && !options_.force_lowbit)) {
    ++forwarded_calls_;
    if (tensors.empty()) return inner_any()->allreduce(tensors, opts);
    return inner(tensors[0])->allreduce(tensors, opts);
  }
  for (const auto& t : tensors)
    if (!t.is_floating_point()) {
      ++forwarded_calls_;
      return inner(tensors[0])->allreduce(tensors, opts);
    }
  const bool avg = opts.reduceOp == c10d::ReduceOp::AVG;
  if (tensors[0].is_cuda()) {
    surface_errors();
    bool all_fused = true;
    for (const auto& t : tensors) all_fused = all_fused && fused_dtype(t) && t.device() == tensors[0].device();
    if (all_fused && comm(tensors[0].device().index()) != nullptr) {
      auto w = allreduce_fused(tensors);
      if (avg) {
        // AVG: scale in stream order after the fused kernel (the fused path
        // folds it into the kernel when called through LowBitGroup / hooks).
        c10::cuda::CUDAStreamGuard g(comm_stream(tensors[0].device().index()));
        for (auto& t : tensors) t.div_(getSize());
      }
      return w;
    }
  }
  auto w = allreduce_staged(tensors);
  if (avg)
    for (auto& t : tensors) t.div_(getSize());
  return w;
}

c10::intrusive_ptr<c10d::Work> ProcessGroupLowBit::allreduce_fused(std::vector<at::Tensor>& tensors) {
  const int dev = tensors[0].device().index();
  auto c = comm(dev);
  auto cur = c10::cuda::getCurrentCUDAStream(dev);
  auto cs = comm_stream(dev);
  at::cuda::CUDAEvent ready;
  ready.record(cur);
  ready.block(cs);
  c10::cuda::CUDAGuard dg(dev);
  c10::cuda::CUDAStreamGuard sg(cs);
  for (auto& t : tensors) {
    at::Tensor buf = t.is_contiguous() ? t : t.contiguous();
    at::Tensor res;
    if (options_.error_feedback) res = residual_for(t, buf.numel(), buf.device(), ResidualKind::kAllReduce);
    const uint64_t offset = sr_calls_++;
    c->allreduce(buf.data_ptr(), buf.data_ptr(), res.defined() ? res.data_ptr<float>() : nullptr, buf.numel(),
                 dt_of(buf.scalar_type()), wire_bits(), wire_fmt(), options_.algo, options_.stochastic_rounding,
                 false, options_.seed, offset, 1.0f, cs.stream(), options_.max_ctas);
    if (!buf.is_same(t)) t.copy_(buf);
    c10::cuda::CUDACachingAllocator::recordStream(t.storage().data_ptr(), cs);
    if (res.defined()) c10::cuda::CUDACachingAllocator::recordStream(res.storage().data_ptr(), cs);
  }
  ++fused_calls_;
  auto work = c10::make_intrusive<WorkLowBit>(getRank(), c10d::OpType::ALLREDUCE, tensors, tensors[0].device(), c,
                                              options_.blocking_wait);
  work->finish_cuda(cs);
  recent_.push_back(work);
  return work;
}

// Staged path with the reference's per-shard scales (process_group_lowbit.cc:
// 153-328): CPU tensors over gloo, or CUDA groups without peer access.
c10::intrusive_ptr<c10d::Work> ProcessGroupLowBit::allreduce_staged(std::vector<at::Tensor>& tensors) {
  int bits = options_.bitwidth;
  if (bits > 8) bits = 8;  // the staged byte layout covers 1/2/4/8 bits
  const auto [qmin, qmax] = quant_bounds(bits);
  const int W = getSize();
  auto be = inner(tensors[0]);
  for (auto& t : tensors) {
    const int64_t n = t.numel();
    if (n == 0) continue;
    auto flat = t.reshape({-1}).to(at::kFloat);
    at::Tensor res;
    if (options_.error_feedback) {
      res = residual_for(t, n, t.device(), ResidualKind::kAllReduce);
      flat = flat + res;
    }
    const int64_t pad = (W - n % W) % W;
    auto xp = pad ? at::cat({flat, at::zeros({pad}, flat.options())}) : flat;
    const int64_t shard = xp.numel() / W;
    auto xs = xp.view({W, shard});
    auto amax = xs.abs().amax({1});
    auto scale = at::where(amax == 0, at::ones_like(amax), amax / static_cast<float>(qmax));
    auto v = xs / scale.unsqueeze(1);
    at::Tensor q;
    if (options_.stochastic_rounding) {
      auto lo = v.floor();
      q = at::where(at::rand_like(v) < (v - lo), lo + 1, lo);
    } else {
      q = v.round();
    }
    q = q.clamp(qmin, qmax);
    if (res.defined()) res.copy_((xp - (q * scale.unsqueeze(1)).view({-1})).narrow(0, 0, n));
    auto send = pack_rows((q - qmin).to(at::kInt), bits).contiguous();
    const int64_t S = send.size(1);
    auto recv = at::empty_like(send);
    std::vector<int64_t> splits;
    auto send_flat = send.view({-1});
    auto recv_flat = recv.view({-1});
    be->alltoall_base(recv_flat, send_flat, splits, splits)->wait();
    auto scale_recv = at::empty_like(scale);
    auto scale_send = scale.contiguous();
    be->alltoall_base(scale_recv, scale_send, splits, splits)->wait();
    auto parts = (unpack_rows(recv, bits, shard) + qmin).to(at::kFloat) * scale_recv.unsqueeze(1);
    auto local = parts.sum(0);
    const float lamax = local.abs().max().item<float>();
    const float rs = lamax == 0.0f ? 1.0f : lamax / static_cast<float>(qmax);
    auto qr = (local / rs).round().clamp(qmin, qmax);
    auto packed_r = pack_rows((qr - qmin).to(at::kInt).unsqueeze(0), bits).view({-1});
    std::vector<std::vector<at::Tensor>> gathered(1);
    for (int r = 0; r < W; ++r) gathered[0].push_back(at::empty_like(packed_r));
    std::vector<at::Tensor> in1{packed_r};
    be->allgather(gathered, in1)->wait();
    auto rs_t = at::full({1}, rs, flat.options());
    std::vector<std::vector<at::Tensor>> gscales(1);
    for (int r = 0; r < W; ++r) gscales[0].push_back(at::empty_like(rs_t));
    std::vector<at::Tensor> in2{rs_t};
    be->allgather(gscales, in2)->wait();
    auto allp = at::stack(gathered[0]).view({W, S});
    auto sc = at::cat(gscales[0]);
    auto out = ((unpack_rows(allp, bits, shard) + qmin).to(at::kFloat) * sc.unsqueeze(1)).view({-1}).narrow(0, 0, n);
    t.copy_(out.view(t.sizes()).to(t.scalar_type()));
  }
  ++staged_calls_;
  return c10::make_intrusive<WorkLowBit>(getRank(), c10d::OpType::ALLREDUCE, tensors);
}

c10::intrusive_ptr<c10d::Work> ProcessGroupLowBit::allreduce_coalesced(std::vector<at::Tensor>& tensors,
                                                                      const c10d::AllreduceCoalescedOptions& opts) {
  c10d::AllreduceOptions o;
  o.reduceOp = opts.reduceOp;
  o.timeout = opts.timeout;
  if (tensors.empty() || !use_lowbit_reduce(opts.reduceOp)) {
    ++forwarded_calls_;
    return (tensors.empty() ? inner_any() : inner(tensors[0]))->allreduce_coalesced(tensors, opts);
  }
  return allreduce(tensors, o);
}

// ---------------------------------------------------------------------------
// reduce-scatter / all-gather
// ---------------------------------------------------------------------------
c10::intrusive_ptr<c10d::Work> ProcessGroupLowBit::reduce_scatter_fused(at::Tensor& output, at::Tensor& input,
                                                                       float post_scale) {
  const int dev = input.device().index();
  auto c = comm(dev);
  auto cur = c10::cuda::getCurrentCUDAStream(dev);
  auto cs = comm_stream(dev);
  at::cuda::CUDAEvent ready;
  ready.record(cur);
  ready.block(cs);
  c10::cuda::CUDAGuard dg(dev);
  c10::cuda::CUDAStreamGuard sg(cs);
  at::Tensor in = input.contiguous();
  at::Tensor out = output.is_contiguous() ? output : at::empty_like(output, at::MemoryFormat::Contiguous);
  at::Tensor res;
  if (options_.error_feedback) res = residual_for(in, in.numel(), in.device(), ResidualKind::kReduceScatter);
  c->reduce_scatter(in.data_ptr(), out.data_ptr(), res.defined() ? res.data_ptr<float>() : nullptr, out.numel(),
                    dt_of(in.scalar_type()), wire_bits(), wire_fmt(), options_.stochastic_rounding, options_.seed,
                    sr_calls_++, post_scale, cs.stream(), options_.max_ctas);
  if (!out.is_same(output)) output.copy_(out);
  c10::cuda::CUDACachingAllocator::recordStream(in.storage().data_ptr(), cs);
  c10::cuda::CUDACachingAllocator::recordStream(output.storage().data_ptr(), cs);
  ++fused_calls_;
  auto work = c10::make_intrusive<WorkLowBit>(getRank(), c10d::OpType::_REDUCE_SCATTER_BASE,
                                              std::vector<at::Tensor>{output}, output.device(), c,
                                              options_.blocking_wait);
  work->finish_cuda(cs);
  recent_.push_back(work);
  return work;
}

c10::intrusive_ptr<c10d::Work> ProcessGroupLowBit::allgather_fused(at::Tensor& output, at::Tensor& input) {
  const int dev = input.device().index();
  auto c = comm(dev);
  auto cur = c10::cuda::getCurrentCUDAStream(dev);
  auto cs = comm_stream(dev);
  at::cuda::CUDAEvent ready;
  ready.record(cur);
  ready.block(cs);
  c10::cuda::CUDAGuard dg(dev);
  c10::cuda::CUDAStreamGuard sg(cs);
  at::Tensor in = input.contiguous();
  at::Tensor out = output.is_contiguous() ? output : at::empty_like(output, at::MemoryFormat::Contiguous);
  at::Tensor res;
  if (options_.error_feedback) res = residual_for(in, in.numel(), in.device(), ResidualKind::kAllGather);
  c->all_gather(in.data_ptr(), out.data_ptr(), res.defined() ? res.data_ptr<float>() : nullptr, in.numel(),
                dt_of(in.scalar_type()), wire_bits(), wire_fmt(), options_.stochastic_rounding, options_.seed,
                sr_calls_++, cs.stream(), options_.max_ctas);
  if (!out.is_same(output)) output.copy_(out);
  c10::cuda::CUDACachingAllocator::recordStream(in.storage().data_ptr(), cs);
  c10::cuda::CUDACachingAllocator::recordStream(output.storage().data_ptr(), cs);
  ++fused_calls_;
  auto work = c10::make_intrusive<WorkLowBit>(getRank(), c10d::OpType::_ALLGATHER_BASE,
                                              std::vector<at::Tensor>{output}, output.device(), c,
                                              options_.blocking_wait);
  work->finish_cuda(cs);
  recent_.push_back(work);
  return work;
}

c10::intrusive_ptr<c10d::Work> ProcessGroupLowBit::_reduce_scatter_base(at::Tensor& output, at::Tensor& input,
                                                                       const c10d::ReduceScatterOptions& opts) {
  RECORD_FUNCTION("lowbit:reduce_scatter", std::vector<c10::IValue>());
  const bool sum_like = opts.reduceOp == c10d::ReduceOp::SUM || opts.reduceOp == c10d::ReduceOp::AVG;
  if (sum_like && use_lowbit_gather() && input.is_cuda() && fused_dtype(input) &&
      input.numel() == output.numel() * getSize() && comm(input.device().index()) != nullptr) {
    surface_errors();
    // AVG: the kernel scales its fp32 sums by 1/W before the output store, so
    // the Work completes after the averaged values are written.
    const float post = opts.reduceOp == c10d::ReduceOp::AVG ? 1.0f / static_cast<float>(getSize()) : 1.0f;
    return reduce_scatter_fused(output, input, post);
  }
  ++forwarded_calls_;
  return inner(input)->_reduce_scatter_base(output, input, opts);
}

c10::intrusive_ptr<c10d::Work> ProcessGroupLowBit::reduce_scatter(std::vector<at::Tensor>& outputs,
                                                                 std::vector<std::vector<at::Tensor>>& inputs,
                                                                 const c10d::ReduceScatterOptions& opts) {
  if (outputs.size() == 1 && inputs.size() == 1 && outputs[0].is_cuda() && use_lowbit_gather() &&
      fused_dtype(outputs[0]) && static_cast<int>(inputs[0].size()) == getSize() &&
      comm(outputs[0].device().index()) != nullptr) {
    bool same = true;
    for (const auto& t : inputs[0]) same = same && t.numel() == outputs[0].numel() && t.scalar_type() == outputs[0].scalar_type();
    if (same) {
      at::Tensor flat = at::cat(inputs[0]).view({-1});
      return _reduce_scatter_base(outputs[0], flat, opts);
    }
  }
  ++forwarded_calls_;
  return inner(outputs[0])->reduce_scatter(outputs, inputs, opts);
}

c10::intrusive_ptr<c10d::Work> ProcessGroupLowBit::reduce_scatter_tensor_coalesced(
    std::vector<at::Tensor>& outputs, std::vector<at::Tensor>& inputs, const c10d::ReduceScatterOptions& opts) {
  c10::intrusive_ptr<c10d::Work> last;
  for (size_t i = 0; i < outputs.size(); ++i) last = _reduce_scatter_base(outputs[i], inputs[i], opts);
  return last;
}

c10::intrusive_ptr<c10d::Work> ProcessGroupLowBit::_allgather_base(at::Tensor& output, at::Tensor& input,
                                                                  const c10d::AllgatherOptions& opts) {
  RECORD_FUNCTION("lowbit:all_gather", std::vector<c10::IValue>());
  if (use_lowbit_gather() && input.is_cuda() && fused_dtype(input) && output.numel() == input.numel() * getSize() &&
      comm(input.device().index()) != nullptr) {
    surface_errors();
    return allgather_fused(output, input);
  }
  ++forwarded_calls_;
  return inner(input)->_allgather_base(output, input, opts);
}

c10::intrusive_ptr<c10d::Work> ProcessGroupLowBit::allgather(std::vector<std::vector<at::Tensor>>& outputs,
                                                            std::vector<at::Tensor>& inputs,
                                                            const c10d::AllgatherOptions& opts) {
  if (inputs.size() == 1 && inputs[0].is_cuda() && use_lowbit_gather() && fused_dtype(inputs[0]) &&
      static_cast<int>(outputs[0].size()) == getSize() && comm(inputs[0].device().index()) != nullptr) {
    at::Tensor flat = at::empty({inputs[0].numel() * getSize()}, inputs[0].options());
    at::Tensor in = inputs[0].reshape({-1});
    auto w = _allgather_base(flat, in, opts);
    c10::cuda::CUDAStreamGuard g(comm_stream(inputs[0].device().index()));
    auto chunks = flat.chunk(getSize());
    for (int r = 0; r < getSize(); ++r) outputs[0][r].copy_(chunks[r].view(outputs[0][r].sizes()));
    auto work = c10::make_intrusive<WorkLowBit>(getRank(), c10d::OpType::ALLGATHER, outputs[0], inputs[0].device(),
                                                comm(inputs[0].device().index()), options_.blocking_wait);
    work->finish_cuda(comm_stream(inputs[0].device().index()));
    return work;
  }
  ++forwarded_calls_;
  return inner(inputs[0])->allgather(outputs, inputs, opts);
}

c10::intrusive_ptr<c10d::Work> ProcessGroupLowBit::allgather_coalesced(std::vector<std::vector<at::Tensor>>& outputs,
                                                                      std::vector<at::Tensor>& inputs,
                                                                      const c10d::AllgatherOptions& opts) {
  ++forwarded_calls_;
  return inner(inputs[0])->allgather_coalesced(outputs, inputs, opts);
}

c10::intrusive_ptr<c10d::Work> ProcessGroupLowBit::allgather_into_tensor_coalesced(std::vector<at::Tensor>& outputs,
                                                                                  std::vector<at::Tensor>& inputs,
                                                                                  const c10d::AllgatherOptions& opts) {
  c10::intrusive_ptr<c10d::Work> last;
  for (size_t i = 0; i < outputs.size(); ++i) last = _allgather_base(outputs[i], inputs[i], opts);
  return last;
}

// ---------------------------------------------------------------------------
// forwarded collectives
// ---------------------------------------------------------------------------
c10::intrusive_ptr<c10d::Work> ProcessGroupLowBit::broadcast(std::vector<at::Tensor>& tensors,
                                                            const c10d::BroadcastOptions& opts) {
  ++forwarded_calls_;
  return inner(tensors.at(0))->broadcast(tensors, opts);
}
c10::intrusive_ptr<c10d::Work> ProcessGroupLowBit::reduce(std::vector<at::Tensor>& tensors,
                                                         const c10d::ReduceOptions& opts) {
  ++forwarded_calls_;
  return inner(tensors.at(0))->reduce(tensors, opts);
}
c10::intrusive_ptr<c10d::Work> ProcessGroupLowBit::gather(std::vector<std::vector<at::Tensor>>& outputs,
                                                         std::vector<at::Tensor>& inputs,
                                                         const c10d::GatherOptions& opts) {
  ++forwarded_calls_;
  return inner(inputs.at(0))->gather(outputs, inputs, opts);
}
c10::intrusive_ptr<c10d::Work> ProcessGroupLowBit::scatter(std::vector<at::Tensor>& outputs,
                                                          std::vector<std::vector<at::Tensor>>& inputs,
                                                          const c10d::ScatterOptions& opts) {
  ++forwarded_calls_;
  return inner(outputs.at(0))->scatter(outputs, inputs, opts);
}
c10::intrusive_ptr<c10d::Work> ProcessGroupLowBit::alltoall(std::vector<at::Tensor>& outputs,
                                                           std::vector<at::Tensor>& inputs,
                                                           const c10d::AllToAllOptions& opts) {
  ++forwarded_calls_;
  return inner(inputs.at(0))->alltoall(outputs, inputs, opts);
}
c10::intrusive_ptr<c10d::Work> ProcessGroupLowBit::alltoall_base(at::Tensor& output, at::Tensor& input,
                                                                std::vector<int64_t>& output_split_sizes,
                                                                std::vector<int64_t>& input_split_sizes,
                                                                const c10d::AllToAllOptions& opts) {
  ++forwarded_calls_;
  return inner(input)->alltoall_base(output, input, output_split_sizes, input_split_sizes, opts);
}
c10::intrusive_ptr<c10d::Work> ProcessGroupLowBit::send(std::vector<at::Tensor>& tensors, int dst, int tag) {
  ++forwarded_calls_;
  return inner(tensors.at(0))->send(tensors, dst, tag);
}
c10::intrusive_ptr<c10d::Work> ProcessGroupLowBit::recv(std::vector<at::Tensor>& tensors, int src, int tag) {
  ++forwarded_calls_;
  return inner(tensors.at(0))->recv(tensors, src, tag);
}
c10::intrusive_ptr<c10d::Work> ProcessGroupLowBit::recvAnysource(std::vector<at::Tensor>& tensors, int tag) {
  ++forwarded_calls_;
  return inner(tensors.at(0))->recvAnysource(tensors, tag);
}
c10::intrusive_ptr<c10d::Work> ProcessGroupLowBit::barrier(const c10d::BarrierOptions& opts) {
  ++forwarded_calls_;
  return inner_any()->barrier(opts);
}
void ProcessGroupLowBit::setSequenceNumberForGroup() {
  if (cuda_inner_) cuda_inner_->setSequenceNumberForGroup();
  if (cpu_inner_) cpu_inner_->setSequenceNumberForGroup();
}
uint64_t ProcessGroupLowBit::getSequenceNumberForGroup() { return inner_any()->getSequenceNumberForGroup(); }

c10::intrusive_ptr<c10d::Backend> createProcessGroupLowBit(const c10::intrusive_ptr<c10d::Store>& store, int rank,
                                                          int size, c10::intrusive_ptr<c10d::Backend> cpu_inner,
                                                          c10::intrusive_ptr<c10d::Backend> cuda_inner,
                                                          const LowBitOptions& options) {
  return c10::make_intrusive<ProcessGroupLowBit>(store, rank, size, std::move(cpu_inner), std::move(cuda_inner),
                                                 options);
}

// ---------------------------------------------------------------------------
// Python bindings
// ---------------------------------------------------------------------------
void register_backend_bindings(pybind11::module& m) {
  namespace py = pybind11;
  py::module::import("torch.distributed");
  // The C++ namespace (bitscom_b200) keeps these types distinct from the
  // reference's same-named classes when both extensions share a process.
  py::class_<LowBitOptions>(m, "LowBitOptions")
      .def(py::init<>())
      .def_readwrite("bitwidth", &LowBitOptions::bitwidth)
      .def_readwrite("error_feedback", &LowBitOptions::error_feedback)
      .def_readwrite("timeout", &LowBitOptions::timeout)
      .def_readwrite("stochastic_rounding", &LowBitOptions::stochastic_rounding)
      .def_readwrite("fp8", &LowBitOptions::fp8)
      .def_readwrite("force_lowbit", &LowBitOptions::force_lowbit)
      .def_readwrite("algo", &LowBitOptions::algo)
      .def_readwrite("workspace_bytes", &LowBitOptions::workspace_bytes)
      .def_readwrite("max_ctas", &LowBitOptions::max_ctas)
      .def_readwrite("oneshot_max_bytes", &LowBitOptions::oneshot_max_bytes)
      .def_readwrite("tuning", &LowBitOptions::tuning)
      .def_readwrite("seed", &LowBitOptions::seed)
      .def_readwrite("blocking_wait", &LowBitOptions::blocking_wait);

  py::class_<ProcessGroupLowBit, c10d::Backend, c10::intrusive_ptr<ProcessGroupLowBit>>(m, "ProcessGroupLowBit")
      .def(py::init([](const c10::intrusive_ptr<c10d::Store>& store, int rank, int size,
                       c10::intrusive_ptr<c10d::Backend> cpu_inner, c10::intrusive_ptr<c10d::Backend> cuda_inner,
                       LowBitOptions options) {
             return c10::make_intrusive<ProcessGroupLowBit>(store, rank, size, std::move(cpu_inner),
                                                            std::move(cuda_inner), std::move(options));
           }),
           py::arg("store"), py::arg("rank"), py::arg("size"), py::arg("cpu_inner"), py::arg("cuda_inner"),
           py::arg("options") = LowBitOptions(), py::call_guard<py::gil_scoped_release>())
      .def_property_readonly("options", &ProcessGroupLowBit::options)
      .def("stats", &ProcessGroupLowBit::stats)
      .def("residual_count", &ProcessGroupLowBit::residual_count)
      .def("clear_residuals", &ProcessGroupLowBit::clear_residuals)
      .def("p2p_available", &ProcessGroupLowBit::p2p_available, py::call_guard<py::gil_scoped_release>())
      .def("communicator", &ProcessGroupLowBit::comm, py::call_guard<py::gil_scoped_release>());
}

}  // namespace bitscom_b200
