// Launch parameters of the fused low-bit collective kernels (shared by the
// .cu kernel file and the host runtime).
#pragma once

#include <stdint.h>

#ifdef __CUDACC__
#define BITSCOM_HD __host__ __device__
#else
#define BITSCOM_HD
#endif

namespace bitscom_b200 {

constexpr int kMaxRanks = 8;          // one NVSwitch node
constexpr int kBlockElems = 1024;     // elements per quantisation block (one warp)
constexpr int kSubBlocks = 8;         // blocks per sub-chunk (one 256-thread CTA pass)
constexpr int kSubElems = kBlockElems * kSubBlocks;  // 8192
constexpr int kHeaderBytes = kSubBlocks * 4;         // fp32 scale per block

// Collective kinds.
enum CollOp : int {
  kAllReduceTwoShot = 0,  // reduce-scatter of packed shards, owner requantises, packed all-gather
  kAllReduceOneShot = 1,  // every rank pushes its whole packed tensor to every peer
  kReduceScatter = 2,     // packed reduce-scatter, fp output shard
  kAllGather = 3,         // packed all-gather of each rank's shard
};

// Wire formats.
enum WireFmt : int {
  kFmtInt = 0,   // signed integer codes (1-bit: unsigned {0,1}), per-block absmax scale
  kFmtE4M3 = 1,  // fp8 E4M3 codes with a per-block fp32 scale (absmax / 448)
  kFmtSign = 2,  // 1-bit sign codes (1: x >= 0 -> +scale, 0: -scale), scale = mean |x| of the block
};

// Status bits written to the host-mapped status word.
enum CollStatus : uint32_t {
  kStatusOk = 0u,
  kStatusTimeout = 1u,   // a peer flag did not arrive within timeout_ns
  kStatusAborted = 2u,   // another CTA of the launch timed out first
};

struct CollParams {
  int op;
  int fmt;
  int world;
  int rank;
  uint32_t epoch;
  int parity;

  // Problem.  For all-reduce / reduce-scatter `n` is the element count of the
  // full input; for all-gather it is the element count of this rank's shard.
  int64_t n;
  int64_t shard_len;   // elements per shard on the wire, a multiple of kSubElems
  int64_t in_stride;   // distance between shard starts in the input (all-reduce / reduce-scatter)
  int64_t shard_valid; // elements of each shard that exist in the input
  int64_t out_stride;  // all-gather: distance between source slices in the output
  int64_t n_sub;       // sub-chunks per slot (per shard; per tensor for one-shot)
  int sub_per_item;    // sub-chunks handled by one work item (one flag each)
  int64_t n_items_slot;  // items per slot = ceil(n_sub / sub_per_item)
  int64_t lag;           // schedule lag in chunk groups (<= 0 or >= n_items_slot: phase-major order)

  const void* in;
  void* out;
  void* residual;      // error-feedback residual (same length as the quantised input) or null
  int res_dtype;       // residual element type: 0 = fp32, 1 = bf16 (DType values)
  float post_scale;    // outputs are multiplied by this (1/W for averaging)
  int stochastic;      // stochastic rounding of the first quantisation
  int stochastic2;     // stochastic rounding of the owner's requantisation
  uint64_t seed;
  uint64_t offset;

  // Symmetric workspace (peer_base[rank] is this rank's own mapping).
  uint8_t* peer_base[kMaxRanks];
  int64_t sub_bytes;             // bytes of one packed sub-chunk (header + payload)
  int64_t rs_data_off[2];        // per parity
  int64_t ag_data_off[2];
  int64_t rs_flag_off[2];
  int64_t ag_flag_off[2];
  int64_t slot_subs;             // capacity of one slot in sub-chunks
  int64_t slot_items;            // capacity of one slot's flag array

  // Local bookkeeping.
  uint32_t* ticket;     // work counter (zero between launches)
  uint32_t* done;       // exit counter (zero between launches)
  uint32_t* abort_flag; // set when a CTA gives up
  uint32_t* status;     // host-mapped status word
  uint32_t* fault_skip; // test hook: when non-null and *fault_skip != 0 this rank skips its signals
  uint64_t timeout_ns;
  // Device-side epoch.  When non-null the launch epoch is *epoch_ctr + 1
  // (read by every CTA at start, stored back by the last CTA out) and
  // `epoch` / `parity` above are ignored, so a launch replayed from a CUDA
  // graph still gets a fresh epoch.  With offset_from_epoch the Philox call
  // offset is `offset + epoch`, so replays draw fresh stochastic rounding.
  uint32_t* epoch_ctr;
  int offset_from_epoch;

  // Warp-specialised kernel (lowbit_coll_ws_kernel): shared-memory ring of
  // `stages` stages of `stage_bytes` each, filled by bulk async copies.  Zero
  // stages selects the register-only kernel.  p2_bulk: the owner phase's W
  // packed source sub-chunks fit in one stage and are staged too.
  int stages;
  int p2_bulk;
  int64_t stage_bytes;
};

// Warp-specialised kernel geometry: 8 consumer warps (one 1024-element block
// each per sub-chunk) and one producer warp; a fixed header (mbarriers, work
// descriptors) precedes the stage ring in dynamic shared memory.
constexpr int kWsConsumerWarps = 8;
constexpr int kWsThreads = (kWsConsumerWarps + 1) * 32;
constexpr int kWsDescSlots = 4;
constexpr int kWsMaxStages = 8;
constexpr int kWsHeaderBytes = 1024;

// Work items per chunk in each phase of a collective (phase 1: encode and
// push; phase 2: owner reduce; phase 3: decode a peer's reduced chunk).
BITSCOM_HD inline void coll_phase_items(int op, int world, int* a1, int* a2, int* a3) {
  switch (op) {
    case kAllReduceTwoShot: *a1 = world; *a2 = 1; *a3 = world - 1; break;
    case kReduceScatter:    *a1 = world; *a2 = 1; *a3 = 0; break;
    case kAllReduceOneShot: *a1 = 1; *a2 = 1; *a3 = 0; break;
    default:                *a1 = 1; *a2 = 0; *a3 = world - 1; break;  // all-gather
  }
}

// Ticket -> work item.  Items are numbered phase-major: phase-1 item of chunk
// c and destination k is c*a1 + k, phase-2 item of chunk c is n1 + c,
// phase-3 item of chunk c and source k is n1 + n2 + c*a3 + k.  Tickets are
// handed out in "groups": group g holds phase 1 of chunk g, phase 2 of chunk
// g - lag and phase 3 of chunk g - 2*lag (g - lag when there is no phase 2),
// so owners reduce and peers decode while later chunks are still being
// encoded instead of after the whole phase 1.
//
// Deadlock freedom: every item waits only for items of a strictly earlier
// group (phase 2 of chunk c for phase 1 of chunk c on every rank, phase 3
// for phase 2 of chunk c on the owner), and every rank hands out tickets in
// the same order.  The earliest unfinished ticket over all ranks therefore
// waits for nothing unfinished, and it is claimed as soon as its rank has a
// free CTA, which it has because every ticket that rank claimed before it is
// finished.  This holds for any number of resident CTAs, so the kernel can
// share the GPU with other work.
BITSCOM_HD inline int64_t coll_schedule_item(int op, int world, int64_t IS, int64_t lag, int64_t t) {
  int a1, a2, a3;
  coll_phase_items(op, world, &a1, &a2, &a3);
  const int64_t n1 = a1 * IS, n2 = a2 * IS, total = n1 + n2 + a3 * IS;
  if (t >= total) return total;
  if (lag <= 0 || lag >= IS) return t;
  const int64_t L2 = lag;
  const int64_t L3 = a2 ? 2 * lag : lag;
  // Items handed out before group g.
  auto before = [&](int64_t g) -> int64_t {
    const int64_t p1 = g < IS ? g : IS;
    const int64_t p2 = g - L2 < 0 ? 0 : (g - L2 < IS ? g - L2 : IS);
    const int64_t p3 = g - L3 < 0 ? 0 : (g - L3 < IS ? g - L3 : IS);
    return a1 * p1 + a2 * p2 + a3 * p3;
  };
  int64_t lo = 0, hi = IS + L3;  // before(lo) <= t < before(hi) == total
  while (hi - lo > 1) {
    const int64_t mid = (lo + hi) >> 1;
    if (before(mid) <= t) lo = mid; else hi = mid;
  }
  const int64_t g = lo;
  int64_t r = t - before(g);
  if (g < IS) {
    if (r < a1) return g * a1 + r;
    r -= a1;
  }
  if (a2 != 0 && g >= L2 && g < IS + L2) {
    if (r < a2) return n1 + (g - L2);
    r -= a2;
  }
  return n1 + n2 + (g - L3) * a3 + r;
}

}  // namespace bitscom_b200
