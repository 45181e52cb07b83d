// Fused low-bit collectives over NVLink-5 / NVSwitch peer memory (sm_100a).
//
// One kernel launch performs an entire collective:
//
//   two-shot all-reduce  (replaces reference python/bitscom/api.py:179-257 and
//                         cpp/src/process_group_lowbit.cc:153-328 with their
//                         4 NCCL calls, >=2W+1 host syncs and ~6W ATen launches)
//     phase 1  for every destination shard d: read g (fp32|bf16), add the
//              error-feedback residual, block absmax, quantise (Philox SR),
//              pack, STORE the packed sub-chunk straight into rank d's
//              receive slot over NVLink, write the new residual, signal d.
//     phase 2  (owner) wait for all W packed contributions of one chunk of its
//              shard, dequantise + sum in fp32 in rank order, requantise,
//              pack, STORE the packed result into every rank's gather slot,
//              write its own output, signal every rank.
//     phase 3  wait for each owner's packed chunk, unpack + dequantise into
//              the output.
//   one-shot all-reduce  phase 1 broadcasts the whole packed tensor; phase 2
//                        dequantise-sums all W contributions (no requantisation).
//   reduce-scatter       phases 1+2, fp output shard.
//   all-gather           quantise own shard once, broadcast, unpack all shards.
//
// Work distribution is a per-launch ticket counter mapped to items by
// coll_schedule_item (coll_params.h): phase order by default (all phase-1
// items are handed out before any phase-2 item, ...), or phases interleaved
// with a lag.  Every item waits only for items handed out earlier on every
// rank, so every wait depends on items already claimed by running CTAs; the
// kernel therefore cannot deadlock even when only part of its grid is
// resident (e.g. sharing SMs with backward kernels), which a static
// CTA->chunk mapping would not guarantee.
//
// Every wait is bounded by %globaltimer: on expiry the CTA records
// kStatusTimeout in a host-mapped status word, raises a launch-local abort
// flag that makes the other CTAs drain, and returns normally (no trap).
//
// Wire format (internal; compress() keeps the reference layout): 1024-element
// blocks with one fp32 scale each; lane l of a warp owns elements
// (k*32+l)*4+m (k<8, m<4) of the block, so input loads are fully coalesced
// 128-bit loads and each lane emits exactly `bits` 32-bit words with no
// shared-memory transpose.  Eight blocks form a sub-chunk:
//   [8 x fp32 scales][8 x 128*bits bytes payload].
// Payload words are interleaved across lanes in 16-byte vectors so every
// store/load instruction of a warp covers a contiguous span.
#include "bulk_async.cuh"
#include "coll_params.h"
#include "common.cuh"
#include "launchers.h"

#include <cuda_fp8.h>

#include <atomic>
#include <stdexcept>
#include <string>

namespace bitscom_b200 {
namespace {

constexpr int kThreads = 256;  // 8 warps = one sub-chunk per CTA pass

// ---------------------------------------------------------------------------
// Element access in the interleaved block mapping.
// ---------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ void load_block(const T* __restrict__ p, int64_t blk_base, int64_t n,
                                           bool vec, int lane, float (&v)[32]) {
  if (vec && blk_base + kBlockElems <= n) {
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float t[4];
      ElemIO<T>::load4(p + blk_base + (k * 32 + lane) * 4, t);
#pragma unroll
      for (int m = 0; m < 4; ++m) v[k * 4 + m] = t[m];
    }
  } else {
#pragma unroll
    for (int k = 0; k < 8; ++k)
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const int64_t e = blk_base + (k * 32 + lane) * 4 + m;
        v[k * 4 + m] = (e < n) ? ElemIO<T>::load(p + e) : 0.0f;
      }
  }
}

template <typename T>
__device__ __forceinline__ void store_block(T* __restrict__ p, int64_t blk_base, int64_t n,
                                            bool vec, int lane, const float (&v)[32]) {
  if (vec && blk_base + kBlockElems <= n) {
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float t[4] = {v[k * 4], v[k * 4 + 1], v[k * 4 + 2], v[k * 4 + 3]};
      ElemIO<T>::store4(p + blk_base + (k * 32 + lane) * 4, t);
    }
  } else {
#pragma unroll
    for (int k = 0; k < 8; ++k)
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const int64_t e = blk_base + (k * 32 + lane) * 4 + m;
        if (e < n) ElemIO<T>::store(p + e, v[k * 4 + m]);
      }
  }
}

// ---------------------------------------------------------------------------
// Packed sub-chunk I/O.  Lane-interleaved payload: vector r of lane l sits at
// vector index r*32 + l.
// ---------------------------------------------------------------------------
template <int B>
__device__ __forceinline__ void put_words(uint8_t* sub, int blk, int lane, const uint32_t (&w)[B]) {
  uint8_t* pay = sub + kHeaderBytes + blk * 128 * B;
  if constexpr (B % 4 == 0) {
#pragma unroll
    for (int r = 0; r < B / 4; ++r)
      *reinterpret_cast<uint4*>(pay + (r * 32 + lane) * 16) =
          make_uint4(w[4 * r], w[4 * r + 1], w[4 * r + 2], w[4 * r + 3]);
  } else if constexpr (B == 2) {
    *reinterpret_cast<uint2*>(pay + lane * 8) = make_uint2(w[0], w[1]);
  } else {
    *reinterpret_cast<uint32_t*>(pay + lane * 4) = w[0];
  }
}

template <int B>
__device__ __forceinline__ void get_words(const uint8_t* sub, int blk, int lane, uint32_t (&w)[B]) {
  const uint8_t* pay = sub + kHeaderBytes + blk * 128 * B;
  if constexpr (B % 4 == 0) {
#pragma unroll
    for (int r = 0; r < B / 4; ++r) {
      const uint4 t = __ldcg(reinterpret_cast<const uint4*>(pay + (r * 32 + lane) * 16));
      w[4 * r] = t.x; w[4 * r + 1] = t.y; w[4 * r + 2] = t.z; w[4 * r + 3] = t.w;
    }
  } else if constexpr (B == 2) {
    const uint2 t = __ldcg(reinterpret_cast<const uint2*>(pay + lane * 8));
    w[0] = t.x; w[1] = t.y;
  } else {
    w[0] = __ldcg(reinterpret_cast<const uint32_t*>(pay + lane * 4));
  }
}

__device__ __forceinline__ float get_scale(const uint8_t* sub, int blk) {
  return __ldcg(reinterpret_cast<const float*>(sub) + blk);
}

__device__ __forceinline__ void put_scale(uint8_t* sub, int blk, float s) {
  reinterpret_cast<float*>(sub)[blk] = s;
}

// ---------------------------------------------------------------------------
// Workspace addressing.
// ---------------------------------------------------------------------------
// `par` is the launch's epoch parity: consecutive launches alternate
// between two sets of data regions and flag arrays.
__device__ __forceinline__ uint8_t* rs_sub(const CollParams& p, int par, int rank_base, int slot, int64_t sub) {
  return p.peer_base[rank_base] + p.rs_data_off[par] + (slot * p.slot_subs + sub) * p.sub_bytes;
}
__device__ __forceinline__ uint8_t* ag_sub(const CollParams& p, int par, int rank_base, int slot, int64_t sub) {
  return p.peer_base[rank_base] + p.ag_data_off[par] + (slot * p.slot_subs + sub) * p.sub_bytes;
}
__device__ __forceinline__ uint32_t* rs_flag(const CollParams& p, int par, int rank_base, int slot, int64_t item) {
  return reinterpret_cast<uint32_t*>(p.peer_base[rank_base] + p.rs_flag_off[par]) + slot * p.slot_items + item;
}
__device__ __forceinline__ uint32_t* ag_flag(const CollParams& p, int par, int rank_base, int slot, int64_t item) {
  return reinterpret_cast<uint32_t*>(p.peer_base[rank_base] + p.ag_flag_off[par]) + slot * p.slot_items + item;
}

// ---------------------------------------------------------------------------
// Bounded wait (one thread).  Returns false on timeout or launch abort.
// ---------------------------------------------------------------------------
__device__ bool wait_epoch(const CollParams& p, uint32_t epoch, const uint32_t* flag) {
  if (ld_acquire_sys(flag) == epoch) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t spins = 0;
  while (true) {
    if (ld_acquire_sys(flag) == epoch) return true;
    if ((++spins & 63u) == 0u) {
      if (*reinterpret_cast<volatile uint32_t*>(p.abort_flag) != 0u) return false;
      if (globaltimer_ns() - t0 > p.timeout_ns) {
        // Host-mapped status: a plain system-scope store (device atomics on
        // host memory are not available on every platform).
        *reinterpret_cast<volatile uint32_t*>(p.status) = kStatusTimeout;
        atomicExch(p.abort_flag, 1u);
        return false;
      }
    }
    __nanosleep(64);
  }
}

// ---------------------------------------------------------------------------
// Codes <-> words, one element at a time (j is a compile-time constant inside
// the unrolled loops, so every shift and word index folds away).
// ---------------------------------------------------------------------------
template <int B>
__device__ __forceinline__ void put_code(uint32_t (&w)[B], int j, uint32_t code) {
  const int bit = j * B, wi = bit >> 5, off = bit & 31;
  w[wi] |= code << off;
  if (off + B > 32) w[wi + 1] |= code >> (32 - off);
}

template <int B>
__device__ __forceinline__ uint32_t get_code(const uint32_t (&w)[B], int j) {
  const int bit = j * B, wi = bit >> 5, off = bit & 31;
  uint32_t x = w[wi] >> off;
  if (off + B > 32) x |= w[wi + 1] << (32 - off);
  return x & QBounds<B>::mask;
}

// ---------------------------------------------------------------------------
// Codecs: block scale, per-element encode (value -> code, dequantised value)
// and decode.  Products use __fmul_rn so no FMA contraction can change a
// decoded value between the encoder, the reducer and the decoders.
// ---------------------------------------------------------------------------
template <int B, int FMT>
struct Codec;

template <int B>
struct Codec<B, kFmtInt> {
  static constexpr int qmin = QBounds<B>::qmin;
  static constexpr int qmax = QBounds<B>::qmax;
  __device__ __forceinline__ static float scale_of(float amax) {
    return amax > 0.0f ? amax / static_cast<float>(qmax) : 1.0f;
  }
  // x = value * (1/scale); r = random bits (used when sr).
  __device__ __forceinline__ static uint32_t encode(float x, bool sr, uint32_t r, float scale, float& deq) {
    float q = sr ? sr_round(x, r) : rintf(x);
    q = fminf(fmaxf(q, static_cast<float>(qmin)), static_cast<float>(qmax));
    deq = __fmul_rn(q, scale);
    return static_cast<uint32_t>(static_cast<int>(q) - qmin);
  }
  __device__ __forceinline__ static float decode(uint32_t code, float scale) {
    return __fmul_rn(static_cast<float>(static_cast<int>(code) + qmin), scale);
  }
};

// Sign-magnitude 1 bit (error-feedback signSGD: Seide et al., Interspeech
// 2014; Karimireddy et al., ICML 2019): code = (x >= 0), value = +-scale with
// scale = mean |x| over the 1024-element block (see encode_block).  The
// reference's 1-bit codes are unsigned {0, 1} and lose every negative value;
// this format is the opt-in alternative for 1-bit gradients.
template <int B>
struct Codec<B, kFmtSign> {
  static_assert(B == 1, "sign codes are 1 bit");
  __device__ __forceinline__ static uint32_t encode(float x, bool, uint32_t, float scale, float& deq) {
    const uint32_t c = (x >= 0.0f) ? 1u : 0u;
    deq = c ? scale : -scale;
    return c;
  }
  __device__ __forceinline__ static float decode(uint32_t code, float scale) { return code ? scale : -scale; }
};

template <int B>
struct Codec<B, kFmtE4M3> {
  static_assert(B == 8, "E4M3 codes are 8 bits");
  __device__ __forceinline__ static float scale_of(float amax) {
    return amax > 0.0f ? amax / 448.0f : 1.0f;
  }
  __device__ __forceinline__ static uint32_t encode(float x, bool, uint32_t, float scale, float& deq) {
    const __nv_fp8_storage_t c = __nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3);
    deq = decode(c, scale);
    return c;
  }
  __device__ __forceinline__ static float decode(uint32_t code, float scale) {
    const __half_raw h = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(code), __NV_E4M3);
    return __fmul_rn(__half2float(__half(h)), scale);
  }
};

// Philox draws of the float4 group `grp` (counter {grp, stream, offset}).
__device__ __forceinline__ Philox4 sr_draws(uint64_t grp, uint32_t stream, uint64_t seed, uint64_t offset) {
  Philox4 c;
  c.x = static_cast<uint32_t>(grp);
  c.y = static_cast<uint32_t>(grp >> 32) ^ (stream << 20);
  c.z = static_cast<uint32_t>(offset);
  c.w = static_cast<uint32_t>(offset >> 32);
  return philox4x32_10(c, static_cast<uint32_t>(seed), static_cast<uint32_t>(seed >> 32));
}

__device__ __forceinline__ uint32_t lane_of(const Philox4& r, int m) {
  return m == 0 ? r.x : (m == 1 ? r.y : (m == 2 ? r.z : r.w));
}

// What encode_block leaves in v.
enum EncodeKeep : int { kKeepInput = 0, kKeepResidual = 1, kKeepDequant = 2 };

// Quantises the 32 values of this lane with the warp-wide block scale:
// packs the codes into w, returns the scale, and replaces v[j] with
// (v[j] - dequantised), the new error-feedback residual (kKeepResidual), or
// with the dequantised value itself (kKeepDequant, bit-identical to decoding
// the packed code).
template <int B, int FMT, int KEEP>
__device__ __forceinline__ float encode_block(float (&v)[32], bool sr, uint64_t grp0, uint32_t stream,
                                              uint64_t seed, uint64_t offset, uint32_t (&w)[B]) {
  using C = Codec<B, FMT>;
  float scale, inv;
  if constexpr (FMT == kFmtSign) {
    // mean |x| of the block: per-lane sums in element order, then an xor
    // butterfly (every lane ends with the same total: each pairwise sum is
    // commutative), times 2^-10 (exact).
    float s = 0.0f;
#pragma unroll
    for (int j = 0; j < 32; ++j) s = __fadd_rn(s, fabsf(v[j]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
    scale = __fmul_rn(s, 1.0f / static_cast<float>(kBlockElems));
    inv = 1.0f;  // the sign codec reads only the sign of x * inv
  } else {
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(v[j]));
    amax = warp_max(amax);
    scale = C::scale_of(amax);
    inv = 1.0f / scale;
  }
#pragma unroll
  for (int i = 0; i < B; ++i) w[i] = 0u;
  // Stochastic rounding draws 16 bits per element: one Philox call (128
  // bits) serves two float4 groups (k even: low halves, k odd: high halves),
  // keyed by the even group's index.  16-bit uniforms bias a rounding by at
  // most 2^-16 of a quantisation step and halve the generator's cost, which
  // is the largest compute item of the encode.
  Philox4 r{0u, 0u, 0u, 0u};
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    if (FMT == kFmtInt && sr && (k & 1) == 0) r = sr_draws(grp0 + k * 32, stream, seed, offset);
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const int j = k * 4 + m;
      float deq;
      const uint32_t bits32 = lane_of(r, m);
      const uint32_t draw = (k & 1) ? (bits32 & 0xFFFF0000u) : (bits32 << 16);  // 16 random bits on top
      const uint32_t code = C::encode(__fmul_rn(v[j], inv), sr, draw, scale, deq);
      put_code<B>(w, j, code);
      if (KEEP == kKeepResidual) v[j] = __fsub_rn(v[j], deq);
      if (KEEP == kKeepDequant) v[j] = deq;
    }
  }
  return scale;
}

// Sources decoded per batch in the owner's reduce: about 16 payload words
// per lane in flight (4 sources at 4 bits, 2 at 8 bits, 1 at 12/16 bits).
template <int B>
constexpr int kSrcBatch = (B <= 2) ? 8 : (16 / B > 0 ? 16 / B : 1);

// ---------------------------------------------------------------------------
// The kernel.
// ---------------------------------------------------------------------------
template <typename T, typename R, int B, int FMT>
__global__ void __launch_bounds__(kThreads, 2) lowbit_coll_kernel(const __grid_constant__ CollParams p) {
  using C = Codec<B, FMT>;
  // Double-buffered by item parity: thread 0 writes the next slot while the
  // CTA still reads the current one; every item has at least one CTA barrier
  // after that write, which publishes it.
  __shared__ int64_t s_item[2];
  __shared__ int s_ok[2];
  __shared__ uint32_t s_epoch;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int W = p.world;
  const int me = p.rank;
  const int64_t IS = p.n_items_slot;
  const bool vec_in = (reinterpret_cast<uintptr_t>(p.in) & 15u) == 0;
  const bool vec_out = (reinterpret_cast<uintptr_t>(p.out) & 15u) == 0;
  const bool vec_res = (reinterpret_cast<uintptr_t>(p.residual) & 15u) == 0;
  const bool has_res = p.residual != nullptr;
  const T* in = static_cast<const T*>(p.in);
  R* residual = static_cast<R*>(p.residual);
  T* out = static_cast<T*>(p.out);
  const bool skip_signals = p.fault_skip != nullptr && *p.fault_skip != 0u;  // test hook

  int a1, a2, a3;
  coll_phase_items(p.op, W, &a1, &a2, &a3);
  const int64_t n1 = a1 * IS, n2 = a2 * IS, n3 = a3 * IS;
  const int64_t total = n1 + n2 + n3;
  const bool bcast1 = (p.op == kAllReduceOneShot || p.op == kAllGather);  // phase 1 stores to every rank

  // Elements of input shard d that exist.
  auto shard_lim = [&](int d) -> int64_t {
    const int64_t rest = p.n - static_cast<int64_t>(d) * p.in_stride;
    return rest < p.shard_valid ? rest : p.shard_valid;
  };
  auto grab = [&]() -> int64_t {
    const uint32_t t = atomicAdd(p.ticket, 1u);
    if (*reinterpret_cast<volatile uint32_t*>(p.abort_flag) != 0u) return total;
    return coll_schedule_item(p.op, W, IS, p.lag, static_cast<int64_t>(t));
  };

  if (threadIdx.x == 0) {
    uint32_t e = p.epoch;
    if (p.epoch_ctr != nullptr) {
      // Every CTA reads the counter before the last CTA out advances it.
      e = *reinterpret_cast<volatile uint32_t*>(p.epoch_ctr) + 1u;
      if (e == 0u) e = 1u;  // 0 is the "never written" flag value
    }
    s_epoch = e;
    s_item[0] = grab();
  }
  __syncthreads();
  const uint32_t epoch = s_epoch;
  const int par = p.epoch_ctr != nullptr ? static_cast<int>(epoch & 1u) : p.parity;
  const uint64_t offset = p.offset + (p.offset_from_epoch ? static_cast<uint64_t>(epoch) : 0ull);
  int cur = 0;
  while (true) {
    const int64_t item = s_item[cur];
    if (item >= total) break;
    // Prefetch the next ticket; its latency hides behind this item's work.
    if (threadIdx.x == 0) s_item[cur ^ 1] = grab();

    if (item < n1) {
      // ------------------------------------------------------------ phase 1
      const int64_t c = bcast1 ? item : item / W;
      const int dst = bcast1 ? me : (me + 1 + static_cast<int>(item % W)) % W;
      const int64_t base = bcast1 ? 0 : static_cast<int64_t>(dst) * p.in_stride;
      const int64_t lim = bcast1 ? p.n : shard_lim(dst);
      const bool vx = vec_in && ((base * static_cast<int64_t>(sizeof(T))) & 15) == 0;
      const bool vr = vec_res && ((base * static_cast<int64_t>(sizeof(R))) & 15) == 0;
      for (int g = 0; g < p.sub_per_item; ++g) {
        const int64_t sub = c * p.sub_per_item + g;
        if (sub >= p.n_sub) break;
        const int64_t off = sub * kSubElems + warp * kBlockElems;
        // Bulk-prefetch this warp's block of the next sub-chunk into L2 (TMA
        // engine, no registers held): its loads then wait on L2, not DRAM.
        if (lane == 0 && g + 1 < p.sub_per_item && off + kSubElems + kBlockElems <= lim) {
          if (vx) bulk_prefetch_l2(in + base + off + kSubElems, kBlockElems * static_cast<uint32_t>(sizeof(T)));
          if (has_res && vr) bulk_prefetch_l2(residual + base + off + kSubElems, kBlockElems * static_cast<uint32_t>(sizeof(R)));
        }
        float v[32];
        load_block<T>(in, base + off, base + lim, vx, lane, v);
        if (has_res) {
          float r[32];
          load_block<R>(residual, base + off, base + lim, vr, lane, r);
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __fadd_rn(v[j], r[j]);
        }
        uint32_t w[B];
        float scale;
        if (has_res) {
          scale = encode_block<B, FMT, kKeepResidual>(v, p.stochastic != 0, static_cast<uint64_t>((base + off) >> 2) + lane,
                                                      1u + 4u * me, p.seed, offset, w);
          store_block<R>(residual, base + off, base + lim, vr, lane, v);
        } else {
          scale = encode_block<B, FMT, kKeepInput>(v, p.stochastic != 0, static_cast<uint64_t>((base + off) >> 2) + lane,
                                                   1u + 4u * me, p.seed, offset, w);
        }
        if (!bcast1) {
          uint8_t* d = rs_sub(p, par, dst, me, sub);
          put_words<B>(d, warp, lane, w);
          if (lane == 0) put_scale(d, warp, scale);
        } else {
          for (int k = 0; k < W; ++k) {
            const int d = (me + 1 + k) % W;
            uint8_t* dp = (p.op == kAllGather) ? ag_sub(p, par, d, me, sub) : rs_sub(p, par, d, me, sub);
            put_words<B>(dp, warp, lane, w);
            if (lane == 0) put_scale(dp, warp, scale);
          }
          if (p.op == kAllGather) {  // own slice = decoded own codes (identical on every rank)
            float o[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) o[j] = C::decode(get_code<B>(w, j), scale);
            const bool va = vec_out && ((static_cast<int64_t>(me) * p.out_stride * static_cast<int64_t>(sizeof(T))) & 15) == 0;
            store_block<T>(out + static_cast<int64_t>(me) * p.out_stride, off, p.n, va, lane, o);
          }
        }
      }
      __syncthreads();
      // Completion flags, released by the last warp while the others move on.
      if (warp == kThreads / 32 - 1 && !skip_signals) {
        if (!bcast1) {
          if (lane == 0) st_release_sys(rs_flag(p, par, dst, me, c), epoch);
        } else if (lane < W) {
          const int d = (me + 1 + lane) % W;
          st_release_sys((p.op == kAllGather) ? ag_flag(p, par, d, me, c) : rs_flag(p, par, d, me, c), epoch);
        }
      }
    } else if (item < n1 + n2) {
      // ------------------------------------------------------------ phase 2
      const int64_t c = item - n1;
      if (warp == 0) {
        // Lane s waits for source s: the W flag round trips overlap instead
        // of running one after another.
        const bool ok = lane < W ? wait_epoch(p, epoch, rs_flag(p, par, me, lane, c)) : true;
        __syncwarp();
        const bool all = __all_sync(0xffffffffu, ok);
        if (lane == 0) s_ok[cur] = all ? 1 : 0;
      }
      __syncthreads();
      if (!s_ok[cur]) break;
      for (int g = 0; g < p.sub_per_item; ++g) {
        const int64_t sub = c * p.sub_per_item + g;
        if (sub >= p.n_sub) break;
        float acc[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[j] = 0.0f;
        // Sources in batches of G: all G loads are in flight before the
        // first decode, so a chunk costs ceil(W/G) memory latencies instead
        // of W.  Sums stay in rank order (bit-identical on every rank).
        constexpr int G = kSrcBatch<B>;
        for (int s0 = 0; s0 < W; s0 += G) {
          uint32_t wv[G][B];
          float sc[G];
#pragma unroll
          for (int u = 0; u < G; ++u) {
            if (s0 + u < W) {
              const uint8_t* src = rs_sub(p, par, me, s0 + u, sub);
              get_words<B>(src, warp, lane, wv[u]);
              sc[u] = get_scale(src, warp);
            }
          }
#pragma unroll
          for (int u = 0; u < G; ++u) {
            if (s0 + u < W) {
#pragma unroll
              for (int j = 0; j < 32; ++j) acc[j] = __fadd_rn(acc[j], C::decode(get_code<B>(wv[u], j), sc[u]));
            }
          }
        }
        const int64_t off = sub * kSubElems + warp * kBlockElems;
        if (p.op == kAllReduceTwoShot) {
          const int64_t elem_base = static_cast<int64_t>(me) * p.shard_len + off;
          uint32_t w[B];
          const float scale = encode_block<B, FMT, kKeepDequant>(acc, p.stochastic2 != 0,
                                                                 static_cast<uint64_t>(elem_base >> 2) + lane,
                                                                 2u + 4u * me, p.seed, offset, w);
          for (int k = 0; k < W; ++k) {
            const int d = (me + 1 + k) % W;
            uint8_t* dp = ag_sub(p, par, d, me, sub);
            put_words<B>(dp, warp, lane, w);
            if (lane == 0) put_scale(dp, warp, scale);
          }
          // Own output: acc now holds the dequantised codes, bit-identical to
          // what the other ranks decode from the packed bytes.
#pragma unroll
          for (int j = 0; j < 32; ++j) acc[j] = __fmul_rn(acc[j], p.post_scale);
          store_block<T>(out, elem_base, p.n, vec_out, lane, acc);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) acc[j] = __fmul_rn(acc[j], p.post_scale);
          store_block<T>(out, off, p.op == kReduceScatter ? shard_lim(me) : p.n, vec_out, lane, acc);
        }
      }
      if (p.op == kAllReduceTwoShot) {
        __syncthreads();
        if (warp == kThreads / 32 - 1 && lane < W && !skip_signals) {
          const int d = (me + 1 + lane) % W;
          st_release_sys(ag_flag(p, par, d, me, c), epoch);
        }
      }
    } else {
      // ------------------------------------------------------------ phase 3
      const int64_t k3 = item - n1 - n2;
      const int64_t c = k3 / (W - 1);
      const int src = (me + 1 + static_cast<int>(k3 % (W - 1))) % W;
      if (threadIdx.x == 0) s_ok[cur] = wait_epoch(p, epoch, ag_flag(p, par, me, src, c)) ? 1 : 0;
      __syncthreads();
      if (!s_ok[cur]) break;
      const bool ag = p.op == kAllGather;
      const int64_t obase = ag ? static_cast<int64_t>(src) * p.out_stride : static_cast<int64_t>(src) * p.shard_len;
      const bool vo = vec_out && ((ag ? obase * static_cast<int64_t>(sizeof(T)) : 0) & 15) == 0;
      // One sub-chunk of prefetch: the next sub-chunk's words are loaded
      // before this one is decoded and stored.
      const int64_t sub0 = c * p.sub_per_item;
      uint32_t wn[B];
      float scn = 0.0f;
      if (sub0 < p.n_sub) {
        const uint8_t* sp = ag_sub(p, par, me, src, sub0);
        get_words<B>(sp, warp, lane, wn);
        scn = get_scale(sp, warp);
      }
      for (int g = 0; g < p.sub_per_item; ++g) {
        const int64_t sub = sub0 + g;
        if (sub >= p.n_sub) break;
        uint32_t w[B];
#pragma unroll
        for (int q = 0; q < B; ++q) w[q] = wn[q];
        const float sc = scn;
        if (g + 1 < p.sub_per_item && sub + 1 < p.n_sub) {
          const uint8_t* sp = ag_sub(p, par, me, src, sub + 1);
          get_words<B>(sp, warp, lane, wn);
          scn = get_scale(sp, warp);
        }
        float o[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) o[j] = __fmul_rn(C::decode(get_code<B>(w, j), sc), p.post_scale);
        const int64_t off = sub * kSubElems + warp * kBlockElems;
        if (ag) store_block<T>(out + obase, off, p.n, vo, lane, o);
        else store_block<T>(out, obase + off, p.n, vec_out, lane, o);
      }
    }
    cur ^= 1;
  }

  // Exit bookkeeping: the last CTA out resets the launch-local counters.
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t prev = atomicAdd(p.done, 1u);
    if (prev == gridDim.x - 1) {
      if (p.epoch_ctr != nullptr) *p.epoch_ctr = epoch;
      *p.ticket = 0u;
      *p.done = 0u;
      *p.abort_flag = 0u;
      __threadfence();
    }
  }
}


// ---------------------------------------------------------------------------
// Warp-specialised kernel.
//
// Same work items, schedule, wire format and arithmetic as lowbit_coll_kernel
// (so both produce identical bytes), reorganised so no warp that computes
// ever waits on a peer or on a CTA-wide barrier:
//
//   producer warp (one elected lane): claims tickets, performs the bounded
//     waits on peer completion flags (owner-reduce and decode items), then
//     stages each sub-chunk's data into a ring of shared-memory stages with
//     1-D bulk async copies from this GPU's own memory (cp.async.bulk, TMA
//     engine) -- the gradient and residual sub-chunks of encode items, the W
//     packed source sub-chunks of owner-reduce items (when they fit a stage),
//     the packed sub-chunk of decode items -- and hands the item to the
//     consumers through a small ring of work descriptors;
//   8 consumer warps (one 1024-element block each per sub-chunk): take the
//     next descriptor, read each stage from shared memory (or, for a partial
//     or unaligned sub-chunk, straight from global memory), release the stage
//     and compute/store as before.  The last warp to finish an item (counted
//     with a CTA-scope acquire-release atomic instead of a CTA barrier)
//     releases the item's completion flag(s) over NVLink.
//
// Stages and descriptors are tracked with mbarriers (full: producer arrival
// plus transaction bytes; empty: one arrival per consumer warp).  The
// producer runs up to `stages` sub-chunks ahead, so HBM reads stay in flight
// while the consumers encode, and peer-flag latency hides behind the
// consumers' work on earlier items.
//
// Deadlock freedom is the ticket argument of the register kernel: the only
// waits on other CTAs or ranks are the producer's flag waits, each on items
// of strictly earlier tickets; consumers wait only on their own producer,
// which never waits on its own consumers except for ring space, which they
// free without waiting on anything else.
//
// Every wait (flags, mbarriers) is bounded by %globaltimer; on expiry the
// thread records kStatusTimeout, raises the launch's abort flag, and the CTA
// drains: consumers stop, the producer waits (bounded) for the bulk copies it
// issued and every thread returns normally.
// ---------------------------------------------------------------------------
template <typename T>
struct SmemIO;

template <>
struct SmemIO<float> {
  __device__ __forceinline__ static void load4(const float* p, float (&o)[4]) {
    const uint4 v = lds_v4(p);
    o[0] = __uint_as_float(v.x); o[1] = __uint_as_float(v.y); o[2] = __uint_as_float(v.z); o[3] = __uint_as_float(v.w);
  }
};

template <>
struct SmemIO<__nv_bfloat16> {
  __device__ __forceinline__ static void load4(const __nv_bfloat16* p, float (&o)[4]) {
    const uint2 t = lds_v2(p);
    const float2 fa = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&t.x));
    const float2 fb = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&t.y));
    o[0] = fa.x; o[1] = fa.y; o[2] = fb.x; o[3] = fb.y;
  }
};

template <>
struct SmemIO<__half> {
  __device__ __forceinline__ static void load4(const __half* p, float (&o)[4]) {
    const uint2 t = lds_v2(p);
    const float2 fa = __half22float2(*reinterpret_cast<const __half2*>(&t.x));
    const float2 fb = __half22float2(*reinterpret_cast<const __half2*>(&t.y));
    o[0] = fa.x; o[1] = fa.y; o[2] = fb.x; o[3] = fb.y;
  }
};

template <typename T>
__device__ __forceinline__ void load_block_smem(const T* blk, int lane, float (&v)[32]) {
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    float t[4];
    SmemIO<T>::load4(blk + (k * 32 + lane) * 4, t);
#pragma unroll
    for (int m = 0; m < 4; ++m) v[k * 4 + m] = t[m];
  }
}

template <int B>
__device__ __forceinline__ void get_words_smem(const uint8_t* sub, int blk, int lane, uint32_t (&w)[B]) {
  const uint8_t* pay = sub + kHeaderBytes + blk * 128 * B;
  if constexpr (B % 4 == 0) {
#pragma unroll
    for (int r = 0; r < B / 4; ++r) {
      const uint4 t = lds_v4(pay + (r * 32 + lane) * 16);
      w[4 * r] = t.x; w[4 * r + 1] = t.y; w[4 * r + 2] = t.z; w[4 * r + 3] = t.w;
    }
  } else if constexpr (B == 2) {
    const uint2 t = lds_v2(pay + lane * 8);
    w[0] = t.x; w[1] = t.y;
  } else {
    w[0] = lds_u32(pay + lane * 4);
  }
}

__device__ __forceinline__ float get_scale_smem(const uint8_t* sub, int blk) {
  return __uint_as_float(lds_u32(sub + blk * 4));
}

// Bounded mbarrier wait (one thread).  Returns false on timeout (after
// recording it and raising the abort flag) or when the launch was aborted.
__device__ bool ws_wait(const CollParams& p, uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t spins = 0;
  while (!mbar_try_wait(bar, parity)) {
    if ((++spins & 15u) == 0u) {
      if (*reinterpret_cast<volatile uint32_t*>(p.abort_flag) != 0u) return false;
      if (globaltimer_ns() - t0 > limit_ns) {
        *reinterpret_cast<volatile uint32_t*>(p.status) = kStatusTimeout;
        atomicExch(p.abort_flag, 1u);
        return false;
      }
    }
  }
  return true;
}

// Warp-wide form: lane 0 waits, the result is broadcast, and __syncwarp
// orders the other lanes' later reads after lane 0's acquire.
__device__ __forceinline__ bool ws_warp_wait(const CollParams& p, uint64_t* bar, uint32_t parity, uint64_t limit_ns,
                                             int lane) {
  int ok = 1;
  if (lane == 0) ok = ws_wait(p, bar, parity, limit_ns) ? 1 : 0;
  ok = __shfl_sync(0xffffffffu, ok, 0);
  __syncwarp();
  return ok != 0;
}

template <typename T, typename R, int B, int FMT>
__global__ void __launch_bounds__(kWsThreads, 1) lowbit_coll_ws_kernel(const __grid_constant__ CollParams p) {
  using C = Codec<B, FMT>;
  extern __shared__ __align__(128) uint8_t ws_smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(ws_smem);
  uint64_t* empty = full + kWsMaxStages;
  uint64_t* dfull = empty + kWsMaxStages;
  uint64_t* dempty = dfull + kWsDescSlots;
  int64_t* d_item = reinterpret_cast<int64_t*>(dempty + kWsDescSlots);
  int* d_ok = reinterpret_cast<int*>(d_item + kWsDescSlots);
  uint32_t* d_cnt = reinterpret_cast<uint32_t*>(d_ok + kWsDescSlots);
  uint32_t* s_epoch = d_cnt + kWsDescSlots;
  uint8_t* stage_base = ws_smem + kWsHeaderBytes;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int W = p.world;
  const int me = p.rank;
  const int64_t IS = p.n_items_slot;
  const int spi = p.sub_per_item;
  const bool vec_in = (reinterpret_cast<uintptr_t>(p.in) & 15u) == 0;
  const bool vec_out = (reinterpret_cast<uintptr_t>(p.out) & 15u) == 0;
  const bool vec_res = (reinterpret_cast<uintptr_t>(p.residual) & 15u) == 0;
  const bool has_res = p.residual != nullptr;
  const T* in = static_cast<const T*>(p.in);
  R* residual = static_cast<R*>(p.residual);
  T* out = static_cast<T*>(p.out);
  const bool skip_signals = p.fault_skip != nullptr && *p.fault_skip != 0u;  // test hook
  const int S = p.stages;
  const int64_t SB = p.stage_bytes;
  const int64_t SUBB = p.sub_bytes;
  const uint64_t wait_ns = p.timeout_ns;

  int a1, a2, a3;
  coll_phase_items(p.op, W, &a1, &a2, &a3);
  const int64_t n1 = a1 * IS, n2 = a2 * IS, n3 = a3 * IS;
  const int64_t total = n1 + n2 + n3;
  const bool bcast1 = (p.op == kAllReduceOneShot || p.op == kAllGather);

  auto shard_lim = [&](int d) -> int64_t {
    const int64_t rest = p.n - static_cast<int64_t>(d) * p.in_stride;
    return rest < p.shard_valid ? rest : p.shard_valid;
  };
  // Encode items: destination rank, input base and valid length.
  auto enc_geom = [&](int64_t item, int64_t& c, int& dst, int64_t& base, int64_t& lim) {
    c = bcast1 ? item : item / W;
    dst = bcast1 ? me : (me + 1 + static_cast<int>(item % W)) % W;
    base = bcast1 ? 0 : static_cast<int64_t>(dst) * p.in_stride;
    lim = bcast1 ? p.n : shard_lim(dst);
  };
  // Whether an encode sub-chunk is staged by bulk copy (identical decision in
  // producer and consumers): aligned input (and residual) and a full sub-chunk.
  auto bulk1 = [&](int64_t base, int64_t lim, int64_t sub) -> bool {
    if (!vec_in || ((base * static_cast<int64_t>(sizeof(T))) & 15) != 0) return false;
    if (has_res && (!vec_res || ((base * static_cast<int64_t>(sizeof(R))) & 15) != 0)) return false;
    return (sub + 1) * kSubElems <= lim;
  };
  auto nsub_of = [&](int64_t c) -> int {
    const int64_t r = p.n_sub - c * spi;
    return static_cast<int>(r < spi ? r : spi);
  };

  if (threadIdx.x == 0) {
    uint32_t e = p.epoch;
    if (p.epoch_ctr != nullptr) {
      e = *reinterpret_cast<volatile uint32_t*>(p.epoch_ctr) + 1u;
      if (e == 0u) e = 1u;
    }
    *s_epoch = e;
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kWsConsumerWarps);
    }
    for (int i = 0; i < kWsDescSlots; ++i) {
      mbar_init(&dfull[i], 1);
      mbar_init(&dempty[i], kWsConsumerWarps);
      d_cnt[i] = 0u;
    }
    mbar_init_fence();
  }
  __syncthreads();
  const uint32_t epoch = *s_epoch;
  const int par = p.epoch_ctr != nullptr ? static_cast<int>(epoch & 1u) : p.parity;
  const uint64_t offset = p.offset + (p.offset_from_epoch ? static_cast<uint64_t>(epoch) : 0ull);

  if (warp == kWsConsumerWarps) {
    // ============================================================ producer
    // The whole warp runs the loop in step (every branch below is uniform);
    // lane 0 claims tickets and issues the mbarrier operations and bulk
    // copies, lanes 0..W-1 wait on the W source flags of an owner item in
    // parallel.
    uint32_t dseq = 0, sseq = 0;
    while (true) {
      int64_t item = 0;
      if (lane == 0) {
        const uint32_t t = atomicAdd(p.ticket, 1u);
        item = coll_schedule_item(p.op, W, IS, p.lag, static_cast<int64_t>(t));
        if (*reinterpret_cast<volatile uint32_t*>(p.abort_flag) != 0u) item = total;
      }
      item = __shfl_sync(0xffffffffu, item, 0);
      const int slot = static_cast<int>(dseq % kWsDescSlots);
      int free_ok = 1;
      if (lane == 0) free_ok = ws_wait(p, &dempty[slot], ((dseq / kWsDescSlots) & 1u) ^ 1u, wait_ns) ? 1 : 0;
      if (!__shfl_sync(0xffffffffu, free_ok, 0)) break;
      bool ok = true;
      int kind = 0, src = 0;
      int64_t c = 0;
      if (item < total) {
        if (item < n1) {
          kind = 1;
          c = bcast1 ? item : item / W;
        } else if (item < n1 + n2) {
          kind = 2;
          c = item - n1;
          ok = lane < W ? wait_epoch(p, epoch, rs_flag(p, par, me, lane, c)) : true;
          __syncwarp();
          ok = __all_sync(0xffffffffu, ok);
        } else {
          kind = 3;
          const int64_t k3 = item - n1 - n2;
          c = k3 / (W - 1);
          src = (me + 1 + static_cast<int>(k3 % (W - 1))) % W;
          int okl = 1;
          if (lane == 0) okl = wait_epoch(p, epoch, ag_flag(p, par, me, src, c)) ? 1 : 0;
          ok = __shfl_sync(0xffffffffu, okl, 0) != 0;
        }
        // Peers' stores, acquired through the flags, are read next by bulk
        // copies (async proxy).
        if (kind >= 2 && ok) fence_proxy_async_global();
      }
      if (lane == 0) {
        d_item[slot] = item;
        d_ok[slot] = ok ? 1 : 0;
        mbar_arrive(&dfull[slot]);
      }
      ++dseq;
      if (item >= total || !ok) break;

      int64_t base = 0, lim = 0, c1 = 0;
      int dst = 0;
      if (kind == 1) enc_geom(item, c1, dst, base, lim);
      const int64_t sub0 = c * spi;
      const int nsub = nsub_of(c);
      bool alive = true;
      for (int g = 0; g < nsub; ++g) {
        const int64_t sub = sub0 + g;
        const int st = static_cast<int>(sseq % S);
        int room = 1;
        if (lane == 0) {
          room = ws_wait(p, &empty[st], ((sseq / S) & 1u) ^ 1u, wait_ns) ? 1 : 0;
          if (room) {
            uint8_t* sbuf = stage_base + st * SB;
            if (kind == 1) {
              if (bulk1(base, lim, sub)) {
                const uint32_t xb = kSubElems * static_cast<uint32_t>(sizeof(T));
                const uint32_t rb = has_res ? kSubElems * static_cast<uint32_t>(sizeof(R)) : 0u;
                mbar_arrive_expect_tx(&full[st], xb + rb);
                bulk_g2s(sbuf, in + base + sub * kSubElems, xb, &full[st]);
                if (has_res) bulk_g2s(sbuf + xb, residual + base + sub * kSubElems, rb, &full[st]);
              } else {
                mbar_arrive(&full[st]);
              }
            } else if (kind == 2) {
              if (p.p2_bulk) {
                mbar_arrive_expect_tx(&full[st], static_cast<uint32_t>(W * SUBB));
                for (int s = 0; s < W; ++s)
                  bulk_g2s(sbuf + s * SUBB, rs_sub(p, par, me, s, sub), static_cast<uint32_t>(SUBB), &full[st]);
              } else {
                mbar_arrive(&full[st]);
              }
            } else {
              mbar_arrive_expect_tx(&full[st], static_cast<uint32_t>(SUBB));
              bulk_g2s(sbuf, ag_sub(p, par, me, src, sub), static_cast<uint32_t>(SUBB), &full[st]);
            }
          }
        }
        if (!__shfl_sync(0xffffffffu, room, 0)) {
          alive = false;
          break;
        }
        ++sseq;
      }
      if (!alive) break;
    }
    // Drain: every bulk copy this CTA issued has landed before it exits
    // (bounded; the copies read local memory and complete in microseconds).
    if (lane == 0) {
      const uint32_t armed = sseq < static_cast<uint32_t>(S) ? sseq : static_cast<uint32_t>(S);
      for (uint32_t i = sseq - armed; i < sseq; ++i) {
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(&full[i % S], (i / S) & 1u)) {
          if (globaltimer_ns() - t0 > wait_ns) break;
        }
      }
    }
    __syncwarp();
  } else {
    // ============================================================ consumers
    uint32_t dseq = 0, sseq = 0;
    while (true) {
      const int slot = static_cast<int>(dseq % kWsDescSlots);
      if (!ws_warp_wait(p, &dfull[slot], (dseq / kWsDescSlots) & 1u, 2 * wait_ns, lane)) break;
      const int64_t item = d_item[slot];
      const int ok = d_ok[slot];
      if (item >= total || !ok) break;
      bool alive = true;
      int kind, dst = 0;
      int64_t c;
      if (item < n1) {
        // ---------------------------------------------------------- encode
        kind = 1;
        int64_t base, lim;
        enc_geom(item, c, dst, base, lim);
        const bool vx = vec_in && ((base * static_cast<int64_t>(sizeof(T))) & 15) == 0;
        const bool vr = vec_res && ((base * static_cast<int64_t>(sizeof(R))) & 15) == 0;
        const int nsub = nsub_of(c);
        for (int g = 0; g < nsub; ++g) {
          const int64_t sub = c * spi + g;
          const int st = static_cast<int>(sseq % S);
          if (!ws_warp_wait(p, &full[st], (sseq / S) & 1u, 2 * wait_ns, lane)) {
            alive = false;
            break;
          }
          const int64_t off = sub * kSubElems + warp * kBlockElems;
          const uint8_t* sbuf = stage_base + st * SB;
          float v[32];
          if (bulk1(base, lim, sub)) {
            load_block_smem<T>(reinterpret_cast<const T*>(sbuf) + warp * kBlockElems, lane, v);
            if (has_res) {
              float r[32];
              load_block_smem<R>(reinterpret_cast<const R*>(sbuf + kSubElems * sizeof(T)) + warp * kBlockElems, lane, r);
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = __fadd_rn(v[j], r[j]);
            }
          } else {
            load_block<T>(in, base + off, base + lim, vx, lane, v);
            if (has_res) {
              float r[32];
              load_block<R>(residual, base + off, base + lim, vr, lane, r);
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = __fadd_rn(v[j], r[j]);
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[st]);
          ++sseq;
          uint32_t w[B];
          float scale;
          if (has_res) {
            scale = encode_block<B, FMT, kKeepResidual>(v, p.stochastic != 0, static_cast<uint64_t>((base + off) >> 2) + lane,
                                                        1u + 4u * me, p.seed, offset, w);
            store_block<R>(residual, base + off, base + lim, vr, lane, v);
          } else {
            scale = encode_block<B, FMT, kKeepInput>(v, p.stochastic != 0, static_cast<uint64_t>((base + off) >> 2) + lane,
                                                     1u + 4u * me, p.seed, offset, w);
          }
          if (!bcast1) {
            uint8_t* d = rs_sub(p, par, dst, me, sub);
            put_words<B>(d, warp, lane, w);
            if (lane == 0) put_scale(d, warp, scale);
          } else {
            for (int k = 0; k < W; ++k) {
              const int d = (me + 1 + k) % W;
              uint8_t* dp = (p.op == kAllGather) ? ag_sub(p, par, d, me, sub) : rs_sub(p, par, d, me, sub);
              put_words<B>(dp, warp, lane, w);
              if (lane == 0) put_scale(dp, warp, scale);
            }
            if (p.op == kAllGather) {
              float o[32];
#pragma unroll
              for (int j = 0; j < 32; ++j) o[j] = C::decode(get_code<B>(w, j), scale);
              const bool va = vec_out && ((static_cast<int64_t>(me) * p.out_stride * static_cast<int64_t>(sizeof(T))) & 15) == 0;
              store_block<T>(out + static_cast<int64_t>(me) * p.out_stride, off, p.n, va, lane, o);
            }
          }
        }
      } else if (item < n1 + n2) {
        // ---------------------------------------------------- owner reduce
        kind = 2;
        c = item - n1;
        const int nsub = nsub_of(c);
        for (int g = 0; g < nsub; ++g) {
          const int64_t sub = c * spi + g;
          const int st = static_cast<int>(sseq % S);
          if (!ws_warp_wait(p, &full[st], (sseq / S) & 1u, 2 * wait_ns, lane)) {
            alive = false;
            break;
          }
          const uint8_t* sbuf = stage_base + st * SB;
          float acc[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) acc[j] = 0.0f;
          constexpr int G = kSrcBatch<B>;
          for (int s0 = 0; s0 < W; s0 += G) {
            uint32_t wv[G][B];
            float sc[G];
#pragma unroll
            for (int u = 0; u < G; ++u) {
              if (s0 + u < W) {
                if (p.p2_bulk) {
                  const uint8_t* src = sbuf + (s0 + u) * SUBB;
                  get_words_smem<B>(src, warp, lane, wv[u]);
                  sc[u] = get_scale_smem(src, warp);
                } else {
                  const uint8_t* src = rs_sub(p, par, me, s0 + u, sub);
                  get_words<B>(src, warp, lane, wv[u]);
                  sc[u] = get_scale(src, warp);
                }
              }
            }
#pragma unroll
            for (int u = 0; u < G; ++u) {
              if (s0 + u < W) {
#pragma unroll
                for (int j = 0; j < 32; ++j) acc[j] = __fadd_rn(acc[j], C::decode(get_code<B>(wv[u], j), sc[u]));
              }
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[st]);
          ++sseq;
          const int64_t off = sub * kSubElems + warp * kBlockElems;
          if (p.op == kAllReduceTwoShot) {
            const int64_t elem_base = static_cast<int64_t>(me) * p.shard_len + off;
            uint32_t w[B];
            const float scale = encode_block<B, FMT, kKeepDequant>(acc, p.stochastic2 != 0,
                                                                   static_cast<uint64_t>(elem_base >> 2) + lane,
                                                                   2u + 4u * me, p.seed, offset, w);
            for (int k = 0; k < W; ++k) {
              const int d = (me + 1 + k) % W;
              uint8_t* dp = ag_sub(p, par, d, me, sub);
              put_words<B>(dp, warp, lane, w);
              if (lane == 0) put_scale(dp, warp, scale);
            }
#pragma unroll
            for (int j = 0; j < 32; ++j) acc[j] = __fmul_rn(acc[j], p.post_scale);
            store_block<T>(out, elem_base, p.n, vec_out, lane, acc);
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) acc[j] = __fmul_rn(acc[j], p.post_scale);
            store_block<T>(out, off, p.op == kReduceScatter ? shard_lim(me) : p.n, vec_out, lane, acc);
          }
        }
      } else {
        // ---------------------------------------------------------- decode
        kind = 3;
        const int64_t k3 = item - n1 - n2;
        c = k3 / (W - 1);
        const int src = (me + 1 + static_cast<int>(k3 % (W - 1))) % W;
        const bool ag = p.op == kAllGather;
        const int64_t obase = ag ? static_cast<int64_t>(src) * p.out_stride : static_cast<int64_t>(src) * p.shard_len;
        const bool vo = vec_out && ((ag ? obase * static_cast<int64_t>(sizeof(T)) : 0) & 15) == 0;
        const int nsub = nsub_of(c);
        for (int g = 0; g < nsub; ++g) {
          const int64_t sub = c * spi + g;
          const int st = static_cast<int>(sseq % S);
          if (!ws_warp_wait(p, &full[st], (sseq / S) & 1u, 2 * wait_ns, lane)) {
            alive = false;
            break;
          }
          const uint8_t* sbuf = stage_base + st * SB;
          uint32_t w[B];
          get_words_smem<B>(sbuf, warp, lane, w);
          const float sc = get_scale_smem(sbuf, warp);
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[st]);
          ++sseq;
          float o[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) o[j] = __fmul_rn(C::decode(get_code<B>(w, j), sc), p.post_scale);
          const int64_t off = sub * kSubElems + warp * kBlockElems;
          if (ag) store_block<T>(out + obase, off, p.n, vo, lane, o);
          else store_block<T>(out, obase + off, p.n, vec_out, lane, o);
        }
      }
      if (!alive) break;
      // Item done in this warp; the last of the 8 warps releases its flags.
      // Every lane first fences its own peer stores at system scope, so the
      // release below never depends on another warp's stores still being in
      // flight over NVLink.
      if ((kind == 1 || (kind == 2 && p.op == kAllReduceTwoShot)) && !skip_signals) __threadfence_system();
      __syncwarp();
      int last = 0;
      if (lane == 0) last = (atom_add_acq_rel_cta(&d_cnt[slot], 1u) == kWsConsumerWarps - 1) ? 1 : 0;
      last = __shfl_sync(0xffffffffu, last, 0);
      __syncwarp();
      if (last) {
        if (lane == 0) d_cnt[slot] = 0u;
        if (!skip_signals) {
          if (kind == 1) {
            if (!bcast1) {
              if (lane == 0) st_release_sys(rs_flag(p, par, dst, me, c), epoch);
            } else if (lane < W) {
              const int d = (me + 1 + lane) % W;
              st_release_sys((p.op == kAllGather) ? ag_flag(p, par, d, me, c) : rs_flag(p, par, d, me, c), epoch);
            }
          } else if (kind == 2 && p.op == kAllReduceTwoShot && lane < W) {
            const int d = (me + 1 + lane) % W;
            st_release_sys(ag_flag(p, par, d, me, c), epoch);
          }
        }
        __syncwarp();
      }
      if (lane == 0) mbar_arrive(&dempty[slot]);
      ++dseq;
    }
  }

  // Exit bookkeeping: the last CTA out resets the launch-local counters.
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t prev = atomicAdd(p.done, 1u);
    if (prev == gridDim.x - 1) {
      if (p.epoch_ctr != nullptr) *p.epoch_ctr = epoch;
      *p.ticket = 0u;
      *p.done = 0u;
      *p.abort_flag = 0u;
      __threadfence();
    }
  }
}

template <typename F>
void dispatch_bits_fmt(int bits, int fmt, F&& f) {
  if (fmt == kFmtE4M3) {
    if (bits != 8) throw std::runtime_error("bitscom: the E4M3 wire format needs bitwidth 8");
    f(std::integral_constant<int, 8>{}, std::integral_constant<int, kFmtE4M3>{});
    return;
  }
  if (fmt == kFmtSign) {
    if (bits != 1) throw std::runtime_error("bitscom: the sign wire format needs bitwidth 1");
    f(std::integral_constant<int, 1>{}, std::integral_constant<int, kFmtSign>{});
    return;
  }
  if (fmt != kFmtInt) throw std::runtime_error("bitscom: unknown wire format");
  switch (bits) {
    case 1: f(std::integral_constant<int, 1>{}, std::integral_constant<int, kFmtInt>{}); break;
    case 2: f(std::integral_constant<int, 2>{}, std::integral_constant<int, kFmtInt>{}); break;
    case 4: f(std::integral_constant<int, 4>{}, std::integral_constant<int, kFmtInt>{}); break;
    case 8: f(std::integral_constant<int, 8>{}, std::integral_constant<int, kFmtInt>{}); break;
    case 12: f(std::integral_constant<int, 12>{}, std::integral_constant<int, kFmtInt>{}); break;
    case 16: f(std::integral_constant<int, 16>{}, std::integral_constant<int, kFmtInt>{}); break;
    default: throw std::runtime_error("bitscom: bitwidth must be one of 1,2,4,8,12,16");
  }
}

// Opt-in to the dynamic shared memory of the warp-specialised kernel, once
// per instantiation and device (the template parameters make the static
// per kernel instantiation).
template <typename T, typename R, int B, int F>
cudaError_t ws_prepare(int bytes) {
  auto kernel = lowbit_coll_ws_kernel<T, R, B, F>;
  static std::atomic<uint64_t> done_mask{0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = 1ull << (dev & 63);
  if (done_mask.load(std::memory_order_acquire) & bit) return cudaSuccess;
  int optin = 0;
  e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (e != cudaSuccess) return e;
  if (bytes > optin) return cudaErrorInvalidValue;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, optin);
  if (e == cudaSuccess) done_mask.fetch_or(bit, std::memory_order_acq_rel);
  return e;
}

template <typename T, typename R, int B, int F>
cudaError_t launch_one(const CollParams& p, int grid, cudaStream_t s) {
  if (p.stages > 0) {
    if (p.stages > kWsMaxStages || p.stage_bytes <= 0 || (p.stage_bytes & 127) != 0) return cudaErrorInvalidValue;
    const int smem = kWsHeaderBytes + static_cast<int>(p.stages * p.stage_bytes);
    const cudaError_t e = ws_prepare<T, R, B, F>(smem);
    if (e != cudaSuccess) return e;
    lowbit_coll_ws_kernel<T, R, B, F><<<grid, kWsThreads, smem, s>>>(p);
  } else {
    lowbit_coll_kernel<T, R, B, F><<<grid, kThreads, 0, s>>>(p);
  }
  return cudaGetLastError();
}

template <int B, int F, typename T>
cudaError_t launch_res(const CollParams& p, int grid, cudaStream_t s) {
  if (p.res_dtype == kBF16) return launch_one<T, __nv_bfloat16, B, F>(p, grid, s);
  return launch_one<T, float, B, F>(p, grid, s);
}

template <int B, int F>
cudaError_t launch_typed(const CollParams& p, DType dt, int grid, cudaStream_t s) {
  if (dt == kF32) return launch_res<B, F, float>(p, grid, s);
  if (dt == kBF16) return launch_res<B, F, __nv_bfloat16>(p, grid, s);
  return launch_res<B, F, __half>(p, grid, s);
}

}  // namespace

namespace launch {

int64_t coll_sub_bytes(int bits) { return kHeaderBytes + static_cast<int64_t>(kSubBlocks) * 128 * bits; }

void lowbit_coll(const CollParams& p, DType dt, int bits, int grid, cudaStream_t s) {
  if (p.world < 1 || p.world > kMaxRanks) throw std::runtime_error("bitscom: world size must be 1..8");
  if (p.res_dtype != kF32 && p.res_dtype != kBF16) throw std::runtime_error("bitscom: residual must be fp32 or bf16");
  if (dt != kF32 && dt != kBF16 && dt != kF16) throw std::runtime_error("bitscom: unsupported dtype");
  cudaError_t e = cudaSuccess;
  dispatch_bits_fmt(bits, p.fmt, [&](auto bc, auto fc) { e = launch_typed<decltype(bc)::value, decltype(fc)::value>(p, dt, grid, s); });
  if (e != cudaSuccess) throw std::runtime_error(std::string("lowbit_coll_kernel: ") + cudaGetErrorString(e));
}

// Same launch without exceptions or host allocations (used by the
// allocation-free entry point); returns cudaErrorInvalidValue for an
// unsupported configuration.
cudaError_t lowbit_coll_nothrow(const CollParams& p, DType dt, int bits, int grid, cudaStream_t s) {
  if (p.world < 1 || p.world > kMaxRanks || grid < 1) return cudaErrorInvalidValue;
  if (p.fmt == kFmtE4M3 && bits != 8) return cudaErrorInvalidValue;
  if (p.fmt == kFmtSign && bits != 1) return cudaErrorInvalidValue;
  if (p.fmt != kFmtInt && p.fmt != kFmtE4M3 && p.fmt != kFmtSign) return cudaErrorInvalidValue;
  if (bits != 1 && bits != 2 && bits != 4 && bits != 8 && bits != 12 && bits != 16) return cudaErrorInvalidValue;
  if (dt != kF32 && dt != kBF16 && dt != kF16) return cudaErrorInvalidValue;
  if (p.res_dtype != kF32 && p.res_dtype != kBF16) return cudaErrorInvalidValue;
  cudaError_t e = cudaSuccess;
  dispatch_bits_fmt(bits, p.fmt, [&](auto bc, auto fc) { e = launch_typed<decltype(bc)::value, decltype(fc)::value>(p, dt, grid, s); });
  return e;
}

}  // namespace launch
}  // namespace bitscom_b200
