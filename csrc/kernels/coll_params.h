// Launch parameters of the fused low-bit collective kernels (shared by the
// .cu kernel file and the host runtime).
#pragma once

#include <stdint.h>

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

  const void* in;
  void* out;
  float* residual;     // error-feedback residual (fp32, same length as the quantised input) or null
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
};

}  // namespace bitscom_b200
