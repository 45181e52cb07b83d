// LowBitComm: the native runtime behind every fused low-bit collective.
//
// It owns one symmetric workspace per rank (a cudaMalloc'd buffer whose IPC
// handle is exchanged with the peers of the group, so every rank can store
// straight into every other rank's buffer over NVLink/NVSwitch), the per-rank
// work/exit counters, a host-mapped status word for bounded-wait errors, and
// the epoch counter that versions every flag.
//
// The reference has no transport of its own: every transfer is an NCCL call
// made through an owned ProcessGroupNCCL (reference
// cpp/src/process_group_lowbit.cc:67-70, :254-255, :292, :304).
//
// Every rank must issue the same sequence of collectives on one LowBitComm
// (like an NCCL communicator).  Launches from the host may use different
// streams: a launch on a stream other than the previous launch's waits for
// the previous launch's completion event first, so two streams never run
// launches of one communicator at the same time.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <stdexcept>
#include <string>
#include <vector>

#include "../kernels/coll_params.h"
#include "../kernels/launchers.h"

namespace bitscom_b200 {

enum Algo : int { kAlgoAuto = 0, kAlgoTwoShot = 1, kAlgoOneShot = 2 };

// Kernel organisation: the register kernel (default: every warp loads,
// computes and waits itself, two CTAs per SM) or the warp-specialised kernel
// with a bulk-copy stage ring (one CTA per SM).  Measured on B200 at world
// size 1 (64M fp32, 4-bit EF, two-shot): 0.226 ms register, 0.289 ms
// warp-specialised.
enum KernelVariant : int { kKernelWarpSpecialised = 0, kKernelRegister = 1 };

// Error-feedback residual: fp32 or bf16 elements (null = no error feedback).
// A bf16 residual halves the residual's HBM traffic (read + write per
// element); it rounds the stored error to 8 significant bits, i.e. to about
// 1/500 of a quantisation step.
struct ResidualBuf {
  void* ptr = nullptr;
  DType dt = kF32;
  ResidualBuf() = default;
  ResidualBuf(float* p) : ptr(p), dt(kF32) {}  // NOLINT: fp32 residuals convert implicitly
  ResidualBuf(void* p, DType d) : ptr(p), dt(d) {}
  explicit operator bool() const { return ptr != nullptr; }
  ResidualBuf at(int64_t elems) const {
    if (ptr == nullptr) return {};
    return {static_cast<char*>(ptr) + elems * (dt == kF32 ? 4 : 2), dt};
  }
};

struct CollStats {
  uint64_t calls = 0;
  uint64_t launches = 0;
  uint64_t elements = 0;
  uint64_t wire_bytes = 0;  // packed bytes this rank stored to peers
  uint64_t oneshot = 0;
  uint64_t twoshot = 0;
  uint64_t timed_launches = 0;  // launches whose device time is in kernel_ms
  double kernel_ms = 0.0;       // summed device time of timed launches (set_timing)
};

class LowBitComm {
 public:
  LowBitComm(int rank, int world, int device, int64_t workspace_bytes);
  ~LowBitComm();
  LowBitComm(const LowBitComm&) = delete;
  LowBitComm& operator=(const LowBitComm&) = delete;

  int rank() const { return rank_; }
  int world() const { return world_; }
  int device() const { return device_; }
  int64_t workspace_bytes() const { return ws_bytes_; }

  // 64-byte cudaIpcMemHandle of this rank's workspace.
  std::vector<uint8_t> ipc_handle() const;
  // Maps every peer's workspace (handles indexed by rank; own entry ignored).
  void open_peers(const std::vector<std::vector<uint8_t>>& handles);
  bool ready() const { return ready_; }

  // All-reduce (SUM) of n elements: out = post_scale * sum_r dequant(quant(in_r + residual_r)).
  // `residual` (fp32 or bf16, n elements) is updated in place when non-null.
  void allreduce(const void* in, void* out, ResidualBuf residual, int64_t n, DType dt, int bits, int fmt,
                 int algo, bool sr, bool sr_requant, uint64_t seed, uint64_t offset,
                 float post_scale, cudaStream_t s, int max_ctas);
  // Reduce-scatter: `in` holds world*shard elements; this rank receives shard `rank` in `out`.
  void reduce_scatter(const void* in, void* out, ResidualBuf residual, int64_t shard, DType dt, int bits,
                      int fmt, bool sr, uint64_t seed, uint64_t offset, float post_scale,
                      cudaStream_t s, int max_ctas);
  // All-gather: `in` holds `shard` elements; `out` receives world*shard elements.
  void all_gather(const void* in, void* out, ResidualBuf residual, int64_t shard, DType dt, int bits,
                  int fmt, bool sr, uint64_t seed, uint64_t offset, cudaStream_t s, int max_ctas);

  // Host-mapped status of the launches so far (0 = ok).  Only meaningful once
  // the launches have completed (stream / event synchronised).
  uint32_t status() const;
  // Throws std::runtime_error if a launch reported an error; the communicator
  // then stays broken (every later call throws) until it is re-created.
  void check() const;
  bool broken() const { return broken_; }

  void set_timeout_ms(double ms) { timeout_ns_ = static_cast<uint64_t>(ms * 1e6); }
  double timeout_ms() const { return static_cast<double>(timeout_ns_) / 1e6; }
  // Chunk-group lag of the work schedule: -1 = automatic (phase-major), 0 =
  // phase-major (every encode before any reduce), k > 0 = reduce chunk c
  // after encoding chunk c + k.  Env BITSCOM_SCHED_LAG sets the initial value.
  void set_schedule_lag(int64_t lag) { sched_lag_ = lag < -1 ? -1 : lag; }
  int64_t schedule_lag() const { return sched_lag_; }
  // Sub-chunks (8192 elements) per work item, i.e. per completion flag:
  // 0 = automatic (about three phase-1 items per CTA), 1..16 = fixed.
  // Env BITSCOM_SUB_PER_ITEM sets the initial value.
  void set_sub_per_item(int spi) { spi_override_ = spi < 0 ? 0 : (spi > 16 ? 16 : spi); }
  int sub_per_item() const { return spi_override_; }
  // Automatic algorithm choice: one-shot up to this many packed bytes per
  // rank, two-shot above (tuning table; default 512 KB, the B200 crossover
  // measured at W=2 and W=8).  Env BITSCOM_ALGO=oneshot|twoshot replaces the
  // automatic choice.
  void set_oneshot_max_bytes(int64_t b) { oneshot_max_bytes_ = b < 0 ? 0 : b; }
  int64_t oneshot_max_bytes() const { return oneshot_max_bytes_; }
  // Per wire format (bits, fmt) entries of the tuning table: the one-shot
  // threshold, and the packed size from which the warp-specialised kernel
  // runs (-1: no entry, the defaults above apply).
  void set_tuning(int bits, int fmt, int64_t oneshot_max_bytes, int64_t ws_min_bytes) {
    if (bits < 1 || bits > 16 || fmt < 0 || fmt > 2) throw std::runtime_error("bitscom: tuning entry needs bits 1..16, fmt 0..2");
    tune_oneshot_[fmt][bits] = oneshot_max_bytes;
    tune_ws_min_[fmt][bits] = ws_min_bytes;
  }
  // Kernel organisation (KernelVariant); env BITSCOM_KERNEL=ws|reg sets the
  // initial value.  Both variants produce identical bytes.
  void set_kernel_variant(int v) {
    if (v != kKernelWarpSpecialised && v != kKernelRegister) throw std::runtime_error("bitscom: kernel variant must be 0 (ws) or 1 (reg)");
    kernel_variant_ = v;
    kernel_forced_ = true;
  }
  int kernel_variant() const { return kernel_variant_; }
  // Shared memory of the warp-specialised kernel's stage ring (bytes; env
  // BITSCOM_WS_SMEM_KB).  At least two stages must fit, else the register
  // kernel runs.
  void set_ws_smem_budget(int64_t bytes) { ws_smem_budget_ = bytes < (32 << 10) ? (32 << 10) : bytes; }
  int64_t ws_smem_budget() const { return ws_smem_budget_; }
  // Number of workspace guard regions whose bytes changed since creation
  // (0 = none).  Synchronises the device.
  int check_canaries() const;
  // Test hook: this rank stops storing its completion flags, so waiting peers time out.
  void set_fault_skip_signal(bool on);
  // Launches issued from the host (replays of a captured launch advance only
  // the device-side epoch).
  uint32_t epoch() const { return epoch_; }
  // Epoch of the last completed launch as the device sees it (synchronising read).
  uint32_t device_epoch() const;
  // Counters; folds in the device time of every timed launch that has
  // completed (launches still running are added by a later call).
  CollStats stats();
  void reset_stats();
  // Time every launch with a pair of CUDA events on its stream (off by
  // default; launches under stream capture are never timed).
  void set_timing(bool on) { timing_ = on; }
  bool timing() const { return timing_; }

  // Segment capacity in elements for an op (for tests and planning).
  int64_t max_elems_per_launch(int op, int bits) const;

 private:
  struct Layout {
    int64_t sub_bytes, slot_subs, slot_items;
    int64_t rs_data[2], ag_data[2], rs_flag[2], ag_flag[2];
  };
  Layout layout(int bits) const;
  void launch(int op, const void* in, void* out, ResidualBuf residual, int64_t n, int64_t shard_len,
              int64_t in_stride, int64_t shard_valid, int64_t n_sub, DType dt, int bits, int fmt, bool sr, bool sr2, uint64_t seed,
              uint64_t offset, float post_scale, cudaStream_t s, int max_ctas, int64_t out_stride);
  void ensure_usable() const;

  int rank_, world_, device_;
  int64_t ws_bytes_;
  uint8_t* ws_ = nullptr;               // own workspace
  uint8_t* peers_[kMaxRanks] = {};      // mapped peer workspaces (own at [rank_])
  bool opened_[kMaxRanks] = {};
  uint32_t* counters_ = nullptr;        // device: ticket, done, abort, fault_skip (each 128 B apart)
  uint32_t* status_host_ = nullptr;     // pinned host-mapped
  uint32_t* status_dev_ = nullptr;
  int64_t data_off_ = 0, flag_off_ = 0, half_bytes_ = 0, flag_cap_ = 0;
  uint32_t epoch_ = 0;
  uint64_t timeout_ns_ = 100ull * 1000ull * 1000ull * 1000ull;  // 100 s default
  int64_t sched_lag_ = -1;
  int spi_override_ = 0;
  int64_t oneshot_max_bytes_ = 512ll << 10;
  int algo_override_ = kAlgoAuto;
  int kernel_variant_ = kKernelRegister;
  bool kernel_forced_ = false;  // set_kernel_variant / BITSCOM_KERNEL override the tuning table
  int64_t tune_oneshot_[3][17] = {{-1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1},
                                  {-1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1},
                                  {-1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1}};
  int64_t tune_ws_min_[3][17] = {{-1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1},
                                 {-1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1},
                                 {-1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1}};
  int kernel_for(int bits, int fmt, int64_t packed_bytes) const;
  int64_t ws_smem_budget_ = 200ll << 10;
  std::vector<int64_t> canary_offsets() const;
  int sm_count_ = 148;
  bool ready_ = false;
  mutable bool broken_ = false;
  CollStats stats_;
  bool timing_ = false;
  std::vector<std::pair<cudaEvent_t, cudaEvent_t>> timed_;  // in flight
  std::vector<cudaEvent_t> event_pool_;
  cudaEvent_t take_event();
  void collect_timings(bool wait);
  // Completion event of the last host-issued (not captured) launch and its stream.
  cudaEvent_t order_ev_ = nullptr;
  cudaStream_t last_stream_ = nullptr;
  bool have_last_ = false;
};

}  // namespace bitscom_b200
