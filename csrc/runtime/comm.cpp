// LowBitComm implementation (see comm.h).
//
// Workspace layout (bytes, per rank):
//   [0, 4096)                   local counters (ticket, done, abort, fault-skip)
//   [flag_off, data_off)        4 flag arrays: rs/ag x parity 0/1, flag_cap words each
//   [data_off, end)             4 data regions of half_bytes: rs0, ag0, rs1, ag1
// A data region holds `world` slots; a slot holds `slot_subs` packed
// sub-chunks of the current bitwidth, so capacity adapts per call.
// Double-buffering by epoch parity makes back-to-back launches safe without a
// barrier: finishing launch e on any rank requires every peer's data of launch
// e, which every peer sends only after finishing launch e-1.
#include "comm.h"

#include <algorithm>
#include <cstring>
#include <stdexcept>
#include <string>

namespace bitscom_b200 {
namespace {

void ck(cudaError_t e, const char* what) {
  if (e != cudaSuccess)
    throw std::runtime_error(std::string("bitscom LowBitComm: ") + what + ": " + cudaGetErrorString(e));
}

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) ck(cudaSetDevice(dev), "cudaSetDevice");
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

constexpr int64_t kCounterBytes = 4096;
constexpr int64_t kMinSubBytes = kHeaderBytes + kSubBlocks * 128 * 1;  // 1-bit sub-chunk
constexpr int kTicket = 0, kDone = 32, kAbort = 64, kFaultSkip = 96, kEpoch = 128;  // word indices (128 B apart)
constexpr int64_t kCanaryBytes = 256;
constexpr int kCanaryByte = 0xA5;

int64_t div_up(int64_t a, int64_t b) { return (a + b - 1) / b; }

}  // namespace

LowBitComm::LowBitComm(int rank, int world, int device, int64_t workspace_bytes)
    : rank_(rank), world_(world), device_(device) {
  if (world < 1 || world > kMaxRanks) throw std::runtime_error("bitscom: world size must be in 1..8");
  if (rank < 0 || rank >= world) throw std::runtime_error("bitscom: rank out of range");
  DeviceGuard g(device_);
  ck(cudaDeviceGetAttribute(&sm_count_, cudaDevAttrMultiProcessorCount, device_), "sm count");
  // Data: 4 regions; flags: 4 arrays sized for the smallest (1-bit) sub-chunk.
  const int64_t min_ws = 64ll << 20;
  workspace_bytes = std::max(workspace_bytes, min_ws);
  half_bytes_ = ((workspace_bytes - kCounterBytes) * 95 / 100 / 4) & ~int64_t(4095);
  flag_cap_ = half_bytes_ / kMinSubBytes + 1;
  flag_off_ = kCounterBytes;
  data_off_ = flag_off_ + ((4 * flag_cap_ * 4 + kCanaryBytes + 4095) & ~int64_t(4095));
  ws_bytes_ = data_off_ + 4 * half_bytes_;
  ck(cudaMalloc(&ws_, ws_bytes_), "cudaMalloc(workspace)");
  ck(cudaMemset(ws_, 0, data_off_), "cudaMemset(flags)");
  // Guard bytes after the flag arrays and at the end of every data region
  // (never addressed by a slot); check_canaries() reports any overwrite.
  for (int64_t off : canary_offsets()) ck(cudaMemset(ws_ + off, kCanaryByte, kCanaryBytes), "cudaMemset(canary)");
  counters_ = reinterpret_cast<uint32_t*>(ws_);
  ck(cudaHostAlloc(&status_host_, 64, cudaHostAllocMapped | cudaHostAllocPortable), "cudaHostAlloc(status)");
  std::memset(status_host_, 0, 64);
  ck(cudaHostGetDevicePointer(reinterpret_cast<void**>(&status_dev_), status_host_, 0),
     "cudaHostGetDevicePointer(status)");
  ck(cudaDeviceSynchronize(), "init sync");
  peers_[rank_] = ws_;
  opened_[rank_] = true;
  if (world_ == 1) ready_ = true;
  if (const char* t = std::getenv("BITSCOM_TIMEOUT_MS")) set_timeout_ms(std::atof(t));
  if (const char* t = std::getenv("BITSCOM_SCHED_LAG")) sched_lag_ = std::atoll(t);
  if (const char* t = std::getenv("BITSCOM_SUB_PER_ITEM")) spi_override_ = std::atoi(t);
  if (const char* t = std::getenv("BITSCOM_KERNEL")) {
    const std::string k(t);
    if (k == "reg") kernel_variant_ = kKernelRegister, kernel_forced_ = true;
    else if (k == "ws") kernel_variant_ = kKernelWarpSpecialised, kernel_forced_ = true;
    else if (k.empty() || k == "auto") kernel_forced_ = false;
    else throw std::runtime_error("bitscom: BITSCOM_KERNEL must be auto, ws or reg");
  }
  if (const char* t = std::getenv("BITSCOM_WS_SMEM_KB")) ws_smem_budget_ = std::max<int64_t>(32, std::atoll(t)) << 10;
  if (const char* t = std::getenv("BITSCOM_ALGO")) {
    const std::string a(t);
    if (a == "oneshot") algo_override_ = kAlgoOneShot;
    else if (a == "twoshot") algo_override_ = kAlgoTwoShot;
    else if (a != "auto" && !a.empty()) throw std::runtime_error("bitscom: BITSCOM_ALGO must be auto, oneshot or twoshot");
  }
}

LowBitComm::~LowBitComm() {
  int cur = -1;
  cudaGetDevice(&cur);
  cudaSetDevice(device_);
  cudaDeviceSynchronize();
  for (auto& pr : timed_) {
    cudaEventDestroy(pr.first);
    cudaEventDestroy(pr.second);
  }
  for (cudaEvent_t e : event_pool_) cudaEventDestroy(e);
  if (order_ev_) cudaEventDestroy(order_ev_);
  for (int r = 0; r < world_; ++r)
    if (r != rank_ && opened_[r] && peers_[r]) cudaIpcCloseMemHandle(peers_[r]);
  if (ws_) cudaFree(ws_);
  if (status_host_) cudaFreeHost(status_host_);
  if (cur >= 0) cudaSetDevice(cur);
}

std::vector<uint8_t> LowBitComm::ipc_handle() const {
  DeviceGuard g(device_);
  cudaIpcMemHandle_t h;
  ck(cudaIpcGetMemHandle(&h, ws_), "cudaIpcGetMemHandle");
  std::vector<uint8_t> out(sizeof(h));
  std::memcpy(out.data(), &h, sizeof(h));
  return out;
}

void LowBitComm::open_peers(const std::vector<std::vector<uint8_t>>& handles) {
  if (static_cast<int>(handles.size()) != world_) throw std::runtime_error("bitscom: need one IPC handle per rank");
  DeviceGuard g(device_);
  for (int r = 0; r < world_; ++r) {
    if (r == rank_ || opened_[r]) continue;
    if (handles[r].size() != sizeof(cudaIpcMemHandle_t)) throw std::runtime_error("bitscom: bad IPC handle size");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handles[r].data(), sizeof(h));
    void* p = nullptr;
    ck(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
    peers_[r] = static_cast<uint8_t*>(p);
    opened_[r] = true;
  }
  ready_ = true;
}

cudaEvent_t LowBitComm::take_event() {
  if (!event_pool_.empty()) {
    cudaEvent_t e = event_pool_.back();
    event_pool_.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  ck(cudaEventCreate(&e), "cudaEventCreate");
  return e;
}

void LowBitComm::collect_timings(bool wait) {
  DeviceGuard g(device_);
  size_t keep = 0;
  for (size_t i = 0; i < timed_.size(); ++i) {
    auto pr = timed_[i];
    if (wait) cudaEventSynchronize(pr.second);
    if (cudaEventQuery(pr.second) == cudaSuccess) {
      float ms = 0.0f;
      if (cudaEventElapsedTime(&ms, pr.first, pr.second) == cudaSuccess) {
        stats_.kernel_ms += ms;
        stats_.timed_launches += 1;
      }
      event_pool_.push_back(pr.first);
      event_pool_.push_back(pr.second);
    } else {
      timed_[keep++] = pr;
    }
  }
  timed_.resize(keep);
  cudaGetLastError();  // a not-ready query leaves cudaErrorNotReady behind
}

CollStats LowBitComm::stats() {
  collect_timings(false);
  return stats_;
}

void LowBitComm::reset_stats() {
  collect_timings(true);
  stats_ = CollStats();
}

std::vector<int64_t> LowBitComm::canary_offsets() const {
  std::vector<int64_t> v;
  v.push_back(flag_off_ + 4 * flag_cap_ * 4);
  for (int r = 0; r < 4; ++r) v.push_back(data_off_ + (r + 1) * half_bytes_ - kCanaryBytes);
  return v;
}

int LowBitComm::check_canaries() const {
  DeviceGuard g(device_);
  ck(cudaDeviceSynchronize(), "canary sync");
  std::vector<uint8_t> buf(kCanaryBytes);
  int bad = 0;
  for (int64_t off : canary_offsets()) {
    ck(cudaMemcpy(buf.data(), ws_ + off, kCanaryBytes, cudaMemcpyDeviceToHost), "canary read");
    for (uint8_t b : buf) {
      if (b != static_cast<uint8_t>(kCanaryByte)) {
        ++bad;
        break;
      }
    }
  }
  return bad;
}

LowBitComm::Layout LowBitComm::layout(int bits) const {
  Layout L;
  L.sub_bytes = launch::coll_sub_bytes(bits);
  L.slot_subs = (half_bytes_ - kCanaryBytes) / (world_ * L.sub_bytes);
  L.slot_items = L.slot_subs;  // at most one flag per sub-chunk
  if (world_ * L.slot_items > flag_cap_) L.slot_items = flag_cap_ / world_;
  for (int p = 0; p < 2; ++p) {
    L.rs_data[p] = data_off_ + (2 * p) * half_bytes_;
    L.ag_data[p] = data_off_ + (2 * p + 1) * half_bytes_;
    L.rs_flag[p] = flag_off_ + (2 * p) * flag_cap_ * 4;
    L.ag_flag[p] = flag_off_ + (2 * p + 1) * flag_cap_ * 4;
  }
  return L;
}

int64_t LowBitComm::max_elems_per_launch(int op, int bits) const {
  const Layout L = layout(bits);
  if (op == kAllReduceOneShot) return L.slot_subs * kSubElems;
  if (op == kAllGather) return L.slot_subs * kSubElems;  // per-rank shard
  return L.slot_subs * kSubElems * world_;               // full tensor (two-shot / reduce-scatter)
}

uint32_t LowBitComm::status() const { return *reinterpret_cast<volatile uint32_t*>(status_host_); }

void LowBitComm::ensure_usable() const {
  if (broken_) throw std::runtime_error("bitscom: communicator is broken by an earlier timeout; re-create it");
  if (!ready_) throw std::runtime_error("bitscom: peers are not mapped yet (open_peers not called)");
}

void LowBitComm::check() const {
  const uint32_t st = status();
  if (st != kStatusOk) {
    broken_ = true;
    throw std::runtime_error(std::string("bitscom: low-bit collective failed: ") +
                             ((st & kStatusTimeout) ? "a peer did not signal within the timeout" : "aborted") +
                             " (rank " + std::to_string(rank_) + ", epoch " + std::to_string(epoch_) + ")");
  }
  if (broken_) throw std::runtime_error("bitscom: communicator is broken by an earlier timeout; re-create it");
}

uint32_t LowBitComm::device_epoch() const {
  DeviceGuard g(device_);
  uint32_t v = 0;
  ck(cudaMemcpy(&v, counters_ + kEpoch, 4, cudaMemcpyDeviceToHost), "device epoch");
  return v;
}

void LowBitComm::set_fault_skip_signal(bool on) {
  DeviceGuard g(device_);
  const uint32_t v = on ? 1u : 0u;
  ck(cudaMemcpy(counters_ + kFaultSkip, &v, 4, cudaMemcpyHostToDevice), "fault skip");
}

void LowBitComm::launch(int op, const void* in, void* out, ResidualBuf residual, int64_t n,
                        int64_t shard_len, int64_t in_stride, int64_t shard_valid, int64_t n_sub, DType dt, int bits, int fmt, bool sr,
                        bool sr2, uint64_t seed, uint64_t offset, float post_scale, cudaStream_t s,
                        int max_ctas, int64_t out_stride) {
  const Layout L = layout(bits);
  CollParams p;
  std::memset(&p, 0, sizeof(p));
  p.op = op;
  p.fmt = fmt;
  p.world = world_;
  p.rank = rank_;
  p.epoch = ++epoch_;
  if (p.epoch == 0) p.epoch = ++epoch_;  // 0 is the "never written" flag value
  p.parity = static_cast<int>(p.epoch & 1u);
  p.n = n;
  p.shard_len = shard_len;
  p.in_stride = in_stride;
  p.shard_valid = shard_valid;
  p.out_stride = out_stride > 0 ? out_stride : n;
  p.n_sub = n_sub;
  // Warp-specialised kernel: one 288-thread CTA per SM (its stage ring takes
  // most of the shared memory).  Register kernel: two 256-thread CTAs per SM
  // (bounded to 128 registers).
  const int64_t packed_bytes = n * bits / 8;
  const bool ws = kernel_for(bits, fmt, packed_bytes) == kKernelWarpSpecialised;
  const int resident = ws ? sm_count_ : 2 * sm_count_;
  const int grid_cap = std::max(1, max_ctas > 0 ? std::min(max_ctas, resident) : resident);
  const int64_t phase1_units = (op == kAllReduceTwoShot || op == kReduceScatter) ? world_ * n_sub : n_sub;
  // Each item ends with one system-scope release (a fence that waits for the
  // item's NVLink stores): aim for about three phase-1 items per CTA so the
  // fence is amortised over several sub-chunks, while small messages keep
  // one sub-chunk per item for parallelism.  At most 8 sub-chunks per item
  // across GPUs unless overridden: measured at 256 MB, 4-bit EF, bf16
  // residual, 8 beat the uncapped 10 by 2.6 % at W=4 (0.201 vs 0.206 ms) and
  // 2 % at W=8 (0.218 vs 0.2225 ms), 2 and 4 were slower; at world size 1 the
  // cap cost 1-4 % (64M elements, two-shot), so it is not applied there.
  int64_t spi = div_up(phase1_units, 3 * static_cast<int64_t>(grid_cap));
  if (world_ > 1) spi = std::min<int64_t>(8, spi);
  if (spi_override_ > 0) spi = spi_override_;
  spi = std::max<int64_t>(1, std::min<int64_t>(16, spi));
  p.sub_per_item = static_cast<int>(spi);
  p.n_items_slot = div_up(n_sub, spi);
  if (p.n_items_slot > L.slot_items) throw std::runtime_error("bitscom: flag capacity exceeded");
  p.in = in;
  p.out = out;
  p.residual = residual.ptr;
  p.res_dtype = residual.dt;
  p.post_scale = post_scale;
  p.stochastic = sr ? 1 : 0;
  p.stochastic2 = sr2 ? 1 : 0;
  p.seed = seed;
  p.offset = offset;
  for (int r = 0; r < world_; ++r) p.peer_base[r] = peers_[r];
  p.sub_bytes = L.sub_bytes;
  p.slot_subs = L.slot_subs;
  p.slot_items = L.slot_items;
  for (int q = 0; q < 2; ++q) {
    p.rs_data_off[q] = L.rs_data[q];
    p.ag_data_off[q] = L.ag_data[q];
    p.rs_flag_off[q] = L.rs_flag[q];
    p.ag_flag_off[q] = L.ag_flag[q];
  }
  p.ticket = counters_ + kTicket;
  p.done = counters_ + kDone;
  p.abort_flag = counters_ + kAbort;
  p.fault_skip = counters_ + kFaultSkip;
  // The launch epoch lives on the device, so a launch captured into a CUDA
  // graph gets a fresh epoch (and, under capture, fresh stochastic-rounding
  // draws) on every replay.
  p.epoch_ctr = counters_ + kEpoch;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(s, &cap) == cudaSuccess && cap == cudaStreamCaptureStatusActive) p.offset_from_epoch = 1;
  p.status = status_dev_;
  p.timeout_ns = timeout_ns_;
  if (ws) {
    // Stage = the largest unit staged at once: an encode sub-chunk (8192
    // inputs + residuals), a decode sub-chunk (one packed sub-chunk) and, when
    // it fits in 64 KB, the owner's W packed source sub-chunks.
    const int64_t esz = dt == kF32 ? 4 : 2;
    const int64_t rsz = residual ? (residual.dt == kF32 ? 4 : 2) : 0;
    int64_t sb = std::max<int64_t>(kSubElems * (esz + rsz), L.sub_bytes);
    const int64_t p2 = world_ * L.sub_bytes;
    const bool p2_bulk = p2 <= std::max<int64_t>(sb, 64ll << 10);
    if (p2_bulk) sb = std::max(sb, p2);
    sb = (sb + 127) & ~int64_t(127);
    const int64_t stages = std::min<int64_t>(kWsMaxStages, ws_smem_budget_ / sb);
    if (stages >= 2) {
      p.stages = static_cast<int>(stages);
      p.stage_bytes = sb;
      p.p2_bulk = p2_bulk ? 1 : 0;
    }
  }

  int a1, a2, a3;
  coll_phase_items(op, world_, &a1, &a2, &a3);
  const int64_t IS = p.n_items_slot;
  const int64_t total = (a1 + a2 + a3) * IS;
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(grid_cap, total)));
  // Schedule lag: phase 2 of a chunk is handed out `lag` groups after its
  // phase 1 (0 = phase-major).  Measured on B200 (4-bit EF, 16-512 MB): at
  // W=1 and W=2 phase-major is fastest (a lag of two CTA waves is 3-9 %
  // slower at W=2, a lag of 32 groups 60 % slower at W=1: owners then spin on
  // chunks still being encoded), so automatic means phase-major.
  p.lag = sched_lag_ >= 0 ? sched_lag_ : 0;
  DeviceGuard g(device_);
  const bool capturing = p.offset_from_epoch != 0;
  // Launches share the workspace, counters and epoch parity: one launch must
  // finish before the next starts.  Launches on one stream are ordered by the
  // stream; a launch on another stream (e.g. a DDP hook's comm stream and a
  // LowBitGroup call on the caller's stream) first waits for the previous
  // launch's completion event.  Captured launches are ordered by their graph.
  if (!capturing && have_last_ && last_stream_ != s) ck(cudaStreamWaitEvent(s, order_ev_, 0), "cudaStreamWaitEvent");
  const bool timed = timing_ && !capturing;  // never under capture
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  if (timed) {
    e0 = take_event();
    e1 = take_event();
    ck(cudaEventRecord(e0, s), "cudaEventRecord");
  }
  launch::lowbit_coll(p, dt, bits, grid, s);
  if (timed) {
    ck(cudaEventRecord(e1, s), "cudaEventRecord");
    timed_.emplace_back(e0, e1);
    if (timed_.size() > 4096) collect_timings(true);  // bound the in-flight list
  }
  if (!capturing) {
    if (order_ev_ == nullptr) ck(cudaEventCreateWithFlags(&order_ev_, cudaEventDisableTiming), "cudaEventCreate");
    ck(cudaEventRecord(order_ev_, s), "cudaEventRecord");
    last_stream_ = s;
    have_last_ = true;
  }
  stats_.launches += 1;
  const int64_t sub_b = L.sub_bytes;
  if (op == kAllReduceTwoShot) stats_.wire_bytes += 2ull * (world_ - 1) * n_sub * sub_b;
  else if (op == kReduceScatter) stats_.wire_bytes += static_cast<uint64_t>(world_ - 1) * n_sub * sub_b;
  else stats_.wire_bytes += static_cast<uint64_t>(world_ - 1) * n_sub * sub_b;
}

int LowBitComm::kernel_for(int bits, int fmt, int64_t packed_bytes) const {
  if (kernel_forced_) return kernel_variant_;
  const int64_t t = (bits >= 1 && bits <= 16 && fmt >= 0 && fmt <= 2) ? tune_ws_min_[fmt][bits] : -1;
  if (t >= 0) return packed_bytes >= t ? kKernelWarpSpecialised : kKernelRegister;
  return kernel_variant_;
}

void LowBitComm::allreduce(const void* in, void* out, ResidualBuf residual, int64_t n, DType dt, int bits,
                           int fmt, int algo, bool sr, bool sr_requant, uint64_t seed, uint64_t offset,
                           float post_scale, cudaStream_t s, int max_ctas) {
  ensure_usable();
  if (n <= 0) return;
  const int esz = dt == kF32 ? 4 : 2;
  stats_.calls += 1;
  stats_.elements += static_cast<uint64_t>(n);
  int a = algo == kAlgoAuto ? algo_override_ : algo;
  if (a == kAlgoAuto) {
    // Small messages are latency bound: one launch-wide broadcast beats two
    // dependent phases.  Measured crossover on B200 (4-bit, W=2 and W=8):
    // one-shot wins up to 512 KB packed (4 MB fp32), two-shot from 1 MB.
    const int64_t packed = n * bits / 8;
    const int64_t t = (bits >= 1 && bits <= 16 && fmt >= 0 && fmt <= 2) ? tune_oneshot_[fmt][bits] : -1;
    a = (world_ == 1 || packed <= (t >= 0 ? t : oneshot_max_bytes_)) ? kAlgoOneShot : kAlgoTwoShot;
  }
  const int op = (a == kAlgoOneShot) ? kAllReduceOneShot : kAllReduceTwoShot;
  const int64_t cap = max_elems_per_launch(op, bits);
  if (cap <= 0) throw std::runtime_error("bitscom: workspace too small for this bitwidth");
  const int64_t seg = (op == kAllReduceOneShot) ? cap : cap;  // elements per launch
  for (int64_t off = 0; off < n; off += seg) {
    const int64_t m = std::min(seg, n - off);
    const char* ip = static_cast<const char*>(in) + off * esz;
    char* op_ = static_cast<char*>(out) + off * esz;
    const ResidualBuf rp = residual.at(off);
    if (op == kAllReduceOneShot) {
      stats_.oneshot += 1;
      const int64_t n_sub = div_up(m, kSubElems);
      launch(op, ip, op_, rp, m, n_sub * kSubElems, 0, m, n_sub, dt, bits, fmt, sr, sr_requant, seed,
             offset + static_cast<uint64_t>(off), post_scale, s, max_ctas, 0);
    } else {
      stats_.twoshot += 1;
      const int64_t shard = div_up(div_up(m, world_), kSubElems) * kSubElems;
      const int64_t n_sub = shard / kSubElems;
      launch(op, ip, op_, rp, m, shard, shard, shard, n_sub, dt, bits, fmt, sr, sr_requant, seed,
             offset + static_cast<uint64_t>(off), post_scale, s, max_ctas, 0);
    }
  }
}

void LowBitComm::reduce_scatter(const void* in, void* out, ResidualBuf residual, int64_t shard, DType dt,
                                int bits, int fmt, bool sr, uint64_t seed, uint64_t offset,
                                float post_scale, cudaStream_t s, int max_ctas) {
  ensure_usable();
  if (shard <= 0) return;
  stats_.calls += 1;
  stats_.elements += static_cast<uint64_t>(shard) * world_;
  const int esz = dt == kF32 ? 4 : 2;
  // Shards larger than one launch's slot capacity are processed as column
  // segments [a, a+m) of every rank's shard (input stride stays `shard`).
  const int64_t cap = (max_elems_per_launch(kReduceScatter, bits) / world_) / kSubElems * kSubElems;
  if (cap <= 0) throw std::runtime_error("bitscom: workspace too small for this bitwidth");
  for (int64_t a = 0; a < shard; a += cap) {
    const int64_t m = std::min(cap, shard - a);
    const int64_t m_pad = div_up(m, kSubElems) * kSubElems;
    launch(kReduceScatter, static_cast<const char*>(in) + a * esz, static_cast<char*>(out) + a * esz,
           residual.at(a), static_cast<int64_t>(world_ - 1) * shard + m, m_pad, shard, m,
           m_pad / kSubElems, dt, bits, fmt, sr, false, seed, offset + static_cast<uint64_t>(a), post_scale, s,
           max_ctas, 0);
  }
}

void LowBitComm::all_gather(const void* in, void* out, ResidualBuf residual, int64_t shard, DType dt, int bits,
                            int fmt, bool sr, uint64_t seed, uint64_t offset, cudaStream_t s,
                            int max_ctas) {
  ensure_usable();
  if (shard <= 0) return;
  stats_.calls += 1;
  stats_.elements += static_cast<uint64_t>(shard) * world_;
  const int esz = dt == kF32 ? 4 : 2;
  // Large shards: segments [a, a+m) of every rank's slice; the output keeps
  // the rank-major layout through out_stride = shard.
  const int64_t cap = max_elems_per_launch(kAllGather, bits) / kSubElems * kSubElems;
  if (cap <= 0) throw std::runtime_error("bitscom: workspace too small for this bitwidth");
  for (int64_t a = 0; a < shard; a += cap) {
    const int64_t m = std::min(cap, shard - a);
    const int64_t n_sub = div_up(m, kSubElems);
    launch(kAllGather, static_cast<const char*>(in) + a * esz, static_cast<char*>(out) + a * esz,
           residual.at(a), m, n_sub * kSubElems, 0, m, n_sub, dt, bits, fmt, sr, false, seed,
           offset + static_cast<uint64_t>(a), 1.0f, s, max_ctas, shard);
  }
}

}  // namespace bitscom_b200
