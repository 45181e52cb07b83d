// Allocation-free entry point of the fused low-bit reduction (see noalloc.h).
//
// This entry point has no counterpart in the reference implementation.
//
// It launches the same kernel as LowBitComm::allreduce on a one-rank
// communicator (lowbit_coll_kernel, two-shot variant), but the kernel's
// scratch comes from the file-scope array below instead of a cudaMalloc'd
// workspace.  Layout of the scratch (bytes):
//   [0, 4096)            counters: ticket @0, done @128, abort @256,
//                        fault-skip @384, status @512
//   [4096, 4096+kFlags)  4 flag arrays (rs/ag x parity), kMaxSubs words each
//   [kDataOff, end)      4 data regions (rs/ag x parity) of kMaxSubs packed
//                        sub-chunks at the widest (16-bit) sub-chunk size
#include <cuda_runtime.h>

#include <atomic>
#include <cstring>
#include <mutex>

#include "coll_params.h"
#include "launchers.h"
#include "noalloc.h"

namespace {

constexpr long long kMaxElems = 1ll << 20;                    // 1,048,576 elements
constexpr long long kMaxSubs = kMaxElems / bitscom_b200::kSubElems;  // 128 sub-chunks
constexpr long long kMaxSubBytes = bitscom_b200::kHeaderBytes + bitscom_b200::kSubBlocks * 128ll * 16;  // 16-bit
constexpr long long kCounterBytes = 4096;
constexpr long long kFlagBytes = 4 * kMaxSubs * 4;
constexpr long long kDataOff = kCounterBytes + ((kFlagBytes + 255) / 256) * 256;
constexpr long long kRegionBytes = kMaxSubs * kMaxSubBytes;
constexpr long long kScratchBytes = kDataOff + 4 * kRegionBytes;  // about 8.4 MB

// The scratch.  In host code `g_noalloc_scratch` names a host-side stand-in,
// not a device address: its device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
constexpr int kStatusWord = 128;  // word index of the status word in the counter page
std::mutex g_setup_mu;
// Per-device scratch address, published with release ordering after the
// other per-device fields, so a reader that sees a non-null pointer (acquire)
// also sees the SM count and the epoch reset.
std::atomic<unsigned char*> g_dev_ptr[kMaxDevices] = {};
int g_sm_count[kMaxDevices] = {};
std::atomic<uint32_t> g_epoch[kMaxDevices];

// One-time set-up of `dev` (current device): device address of the scratch,
// SM count, and cleared counters/flags.  Returns false on a CUDA error.
bool setup(int dev, cudaStream_t stream) {
  std::lock_guard<std::mutex> lk(g_setup_mu);
  if (g_dev_ptr[dev].load(std::memory_order_acquire) != nullptr) return true;
  void* ptr = nullptr;
  if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || ptr == nullptr) return false;
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return false;
  if (cudaMemsetAsync(ptr, 0, static_cast<size_t>(kDataOff), stream) != cudaSuccess) return false;
  g_sm_count[dev] = sms > 0 ? sms : 148;
  g_epoch[dev].store(0);
  g_dev_ptr[dev].store(static_cast<unsigned char*>(ptr), std::memory_order_release);
  return true;
}

}  // namespace

extern "C" {

__attribute__((visibility("default"))) long long bitscom_noalloc_max_elems(void) { return kMaxElems; }

__attribute__((visibility("default"))) long long bitscom_noalloc_scratch_bytes(void) { return kScratchBytes; }

__attribute__((visibility("default"))) const char* bitscom_noalloc_strerror(int code) {
  switch (code) {
    case BITSCOM_NOALLOC_OK: return "ok";
    case BITSCOM_NOALLOC_EINVAL: return "invalid argument (dtype, bitwidth, null pointer or negative n)";
    case BITSCOM_NOALLOC_ETOOBIG: return "n exceeds the static scratch capacity of 1048576 elements";
    case BITSCOM_NOALLOC_ECUDA: return "CUDA set-up or launch failed (see cudaGetLastError)";
    default: return "unknown error";
  }
}

__attribute__((visibility("default"))) int bitscom_lowbit_allreduce_local_noalloc(
    const void* in, void* out, float* residual, long long n, int dtype, int bits, float post_scale,
    void* stream_ptr) {
  using namespace bitscom_b200;
  if (n < 0 || in == nullptr || out == nullptr) return BITSCOM_NOALLOC_EINVAL;
  if (dtype < 0 || dtype > 2) return BITSCOM_NOALLOC_EINVAL;
  if (bits != 1 && bits != 2 && bits != 4 && bits != 8 && bits != 12 && bits != 16) return BITSCOM_NOALLOC_EINVAL;
  if (n > kMaxElems) return BITSCOM_NOALLOC_ETOOBIG;
  if (n == 0) return BITSCOM_NOALLOC_OK;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return BITSCOM_NOALLOC_ECUDA;
  unsigned char* base = g_dev_ptr[dev].load(std::memory_order_acquire);
  if (base == nullptr) {
    if (!setup(dev, stream)) return BITSCOM_NOALLOC_ECUDA;
    base = g_dev_ptr[dev].load(std::memory_order_acquire);
  }

  CollParams p;
  std::memset(&p, 0, sizeof(p));
  p.op = kAllReduceTwoShot;
  p.fmt = kFmtInt;
  p.world = 1;
  p.rank = 0;
  uint32_t e = g_epoch[dev].fetch_add(1) + 1;
  if (e == 0) e = g_epoch[dev].fetch_add(1) + 1;  // 0 means "never written"
  p.epoch = e;
  p.parity = static_cast<int>(e & 1u);
  p.n = n;
  const long long n_sub = (n + kSubElems - 1) / kSubElems;
  p.shard_len = n_sub * kSubElems;
  p.in_stride = p.shard_len;
  p.shard_valid = p.shard_len;
  p.n_sub = n_sub;
  p.sub_per_item = 1;
  p.n_items_slot = n_sub;
  p.in = in;
  p.out = out;
  p.residual = residual;
  p.post_scale = post_scale;
  p.stochastic = 0;
  p.stochastic2 = 0;
  p.peer_base[0] = base;
  p.sub_bytes = launch::coll_sub_bytes(bits);
  p.slot_subs = kMaxSubs;
  p.slot_items = kMaxSubs;
  for (int q = 0; q < 2; ++q) {
    p.rs_data_off[q] = kDataOff + (2 * q) * kRegionBytes;
    p.ag_data_off[q] = kDataOff + (2 * q + 1) * kRegionBytes;
    p.rs_flag_off[q] = kCounterBytes + (2 * q) * kMaxSubs * 4;
    p.ag_flag_off[q] = kCounterBytes + (2 * q + 1) * kMaxSubs * 4;
  }
  uint32_t* counters = reinterpret_cast<uint32_t*>(base);
  p.ticket = counters + 0;
  p.done = counters + 32;
  p.abort_flag = counters + 64;
  p.fault_skip = counters + 96;
  p.status = counters + kStatusWord;
  p.timeout_ns = 10ull * 1000ull * 1000ull * 1000ull;  // world size 1 only waits on its own flags

  const long long items = 2 * n_sub;  // phase 1 + phase 2 at world size 1
  const int grid = static_cast<int>(items < g_sm_count[dev] ? items : g_sm_count[dev]);
  if (launch::lowbit_coll_nothrow(p, static_cast<DType>(dtype), bits, grid, stream) != cudaSuccess)
    return BITSCOM_NOALLOC_ECUDA;
  return BITSCOM_NOALLOC_OK;
}

__attribute__((visibility("default"))) int bitscom_noalloc_status(int reset) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return BITSCOM_NOALLOC_ECUDA;
  if (g_dev_ptr[dev].load(std::memory_order_acquire) == nullptr) return 0;  // no call yet on this device
  // Synchronous copies from and to the scratch's status word (the status
  // lives in device memory; these copies allocate nothing).
  uint32_t v = 0;
  const size_t off = static_cast<size_t>(kStatusWord) * sizeof(uint32_t);
  if (cudaMemcpyFromSymbol(&v, g_noalloc_scratch, sizeof(v), off, cudaMemcpyDeviceToHost) != cudaSuccess)
    return BITSCOM_NOALLOC_ECUDA;
  if (reset && v != 0u) {
    const uint32_t zero = 0u;
    if (cudaMemcpyToSymbol(g_noalloc_scratch, &zero, sizeof(zero), off, cudaMemcpyHostToDevice) != cudaSuccess)
      return BITSCOM_NOALLOC_ECUDA;
  }
  return static_cast<int>(v);
}

}  // extern "C"
