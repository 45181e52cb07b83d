// Standalone sm_100a quantisation kernels with the reference's semantics and
// byte layout (reference: cpp/src/lowbit_cuda_kernels.cu:28-132 for the four
// SIMT kernels; python/bitscom/quantization.py:60-196 for the exact CPU
// semantics these kernels reproduce bit-for-bit).
//
// Design (B200): the reference runs one thread per element/byte, an ATen
// absmax with a blocking .item() host sync, and launches on the legacy default
// stream.  Here:
//   * the absmax is a device-side reduction (128-bit loads, warp shuffles, one
//     atomicMax per CTA) that feeds the quantiser through device memory — no
//     host round trip;
//   * quantise+pack is ONE pass: each warp owns a 1024-element tile, loads it
//     with coalesced 128-bit loads, transposes it through a bank-conflict-free
//     33-float-pitch shared-memory tile so every lane owns 32 consecutive
//     elements, and each lane emits exactly `bits` 32-bit words of the
//     LSB-first bit stream with vector stores (no int16 intermediate);
//   * 12- and 16-bit widths (torch fallbacks in the reference) are native;
//   * stochastic rounding uses Philox-4x32-10 keyed by (seed, offset) so runs
//     are reproducible, instead of wall-clock ^ pointer (reference .cu:161-163).
#include "common.cuh"
#include "launchers.h"

#include <stdexcept>
#include <string>

namespace bitscom_b200 {
namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kTile = 1024;  // elements per warp tile: 32 lanes x 32 codes
constexpr int kPitch = 33;   // padded shared-memory row for the 32x32 transpose

__device__ __forceinline__ int sidx(int i) { return (i >> 5) * kPitch + (i & 31); }

template <typename T>
struct TileIO;

template <typename T>
struct TileIO {
  // Coalesced load of tile elements [base, base+1024) into the transpose tile;
  // positions at or beyond n read as zero.
  __device__ __forceinline__ static void load(const T* __restrict__ x, int64_t base, int64_t n,
                                              bool vec, float* sm, int lane) {
    if (vec && base + kTile <= n) {
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int i = (k * 32 + lane) * 4;
        float v[4];
        ElemIO<T>::load4(x + base + i, v);
#pragma unroll
        for (int m = 0; m < 4; ++m) sm[sidx(i + m)] = v[m];
      }
    } else {
      for (int i = lane; i < kTile; i += 32) {
        const int64_t e = base + i;
        sm[sidx(i)] = (e < n) ? ElemIO<T>::load(x + e) : 0.0f;
      }
    }
    __syncwarp();
  }
};

template <>
struct TileIO<int16_t> {
  __device__ __forceinline__ static void load(const int16_t* __restrict__ x, int64_t base,
                                              int64_t n, bool vec, float* sm, int lane) {
    if (vec && base + kTile <= n) {
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        const int i = (k * 32 + lane) * 2;
        const uint32_t w = __ldg(reinterpret_cast<const uint32_t*>(x + base + i));
        sm[sidx(i)] = static_cast<float>(static_cast<int16_t>(w & 0xffffu));
        sm[sidx(i + 1)] = static_cast<float>(static_cast<int16_t>(w >> 16));
      }
    } else {
      for (int i = lane; i < kTile; i += 32) {
        const int64_t e = base + i;
        sm[sidx(i)] = (e < n) ? static_cast<float>(x[e]) : 0.0f;
      }
    }
    __syncwarp();
  }
};

// Coalesced store of a transposed tile of int16 codes (held exactly as floats).
__device__ __forceinline__ void store_tile_i16(int16_t* __restrict__ q16, int64_t base, int64_t n,
                                               bool vec, const float* sm, int lane) {
  if (vec && base + kTile <= n) {
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const int i = (k * 32 + lane) * 2;
      const uint32_t lo = static_cast<uint16_t>(static_cast<int16_t>(sm[sidx(i)]));
      const uint32_t hi = static_cast<uint16_t>(static_cast<int16_t>(sm[sidx(i + 1)]));
      *reinterpret_cast<uint32_t*>(q16 + base + i) = lo | (hi << 16);
    }
  } else {
    for (int i = lane; i < kTile; i += 32) {
      const int64_t e = base + i;
      if (e < n) q16[e] = static_cast<int16_t>(sm[sidx(i)]);
    }
  }
}

template <typename T>
__device__ __forceinline__ void store_tile(T* __restrict__ out, int64_t base, int64_t n, bool vec,
                                           const float* sm, int lane) {
  if (vec && base + kTile <= n) {
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int i = (k * 32 + lane) * 4;
      float v[4];
#pragma unroll
      for (int m = 0; m < 4; ++m) v[m] = sm[sidx(i + m)];
      ElemIO<T>::store4(out + base + i, v);
    }
  } else {
    for (int i = lane; i < kTile; i += 32) {
      const int64_t e = base + i;
      if (e < n) ElemIO<T>::store(out + e, sm[sidx(i)]);
    }
  }
}

// Writes this lane's B words at word offset `woff` of `packed`, clipped to
// `packed_len` bytes; vector stores when the whole run is in bounds.
template <int B>
__device__ __forceinline__ void store_words(uint8_t* __restrict__ packed, int64_t woff,
                                            int64_t packed_len, const uint32_t (&w)[B]) {
  const int64_t byte0 = woff * 4;
  if (byte0 + 4 * B <= packed_len) {
    uint32_t* p = reinterpret_cast<uint32_t*>(packed) + woff;
    if constexpr (B % 4 == 0) {
#pragma unroll
      for (int i = 0; i < B; i += 4)
        *reinterpret_cast<uint4*>(p + i) = make_uint4(w[i], w[i + 1], w[i + 2], w[i + 3]);
    } else if constexpr (B == 2) {
      *reinterpret_cast<uint2*>(p) = make_uint2(w[0], w[1]);
    } else {
#pragma unroll
      for (int i = 0; i < B; ++i) p[i] = w[i];
    }
  } else {
#pragma unroll
    for (int i = 0; i < B; ++i) {
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const int64_t pos = byte0 + 4 * i + b;
        if (pos < packed_len) packed[pos] = static_cast<uint8_t>(w[i] >> (8 * b));
      }
    }
  }
}

template <int B>
__device__ __forceinline__ void load_words(const uint8_t* __restrict__ packed, int64_t woff,
                                           int64_t packed_len, bool vec, uint32_t (&w)[B]) {
  const int64_t byte0 = woff * 4;
  if (vec && byte0 + 4 * B <= packed_len) {
    const uint32_t* p = reinterpret_cast<const uint32_t*>(packed) + woff;
    if constexpr (B % 4 == 0) {
#pragma unroll
      for (int i = 0; i < B; i += 4) {
        const uint4 t = __ldg(reinterpret_cast<const uint4*>(p + i));
        w[i] = t.x; w[i + 1] = t.y; w[i + 2] = t.z; w[i + 3] = t.w;
      }
    } else if constexpr (B == 2) {
      const uint2 t = __ldg(reinterpret_cast<const uint2*>(p));
      w[0] = t.x; w[1] = t.y;
    } else {
#pragma unroll
      for (int i = 0; i < B; ++i) w[i] = __ldg(p + i);
    }
  } else {
#pragma unroll
    for (int i = 0; i < B; ++i) {
      uint32_t x = 0;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const int64_t pos = byte0 + 4 * i + b;
        if (pos < packed_len) x |= static_cast<uint32_t>(packed[pos]) << (8 * b);
      }
      w[i] = x;
    }
  }
}

__device__ __forceinline__ float scale_from_amax(uint32_t bits, int qmax, double* sd) {
  const float amax = __uint_as_float(bits);
  const double d = (amax == 0.0f) ? 1.0 : static_cast<double>(amax) / static_cast<double>(qmax);
  if (sd) *sd = d;
  return static_cast<float>(d);
}

__device__ __forceinline__ uint32_t pick(const Philox4& r, int j) {
  const int s = j & 3;
  return s == 0 ? r.x : (s == 1 ? r.y : (s == 2 ? r.z : r.w));
}

__device__ __forceinline__ Philox4 philox_at(uint64_t group, uint64_t seed, uint64_t offset) {
  Philox4 c;
  c.x = static_cast<uint32_t>(group);
  c.y = static_cast<uint32_t>(group >> 32);
  c.z = static_cast<uint32_t>(offset);
  c.w = static_cast<uint32_t>(offset >> 32);
  return philox4x32_10(c, static_cast<uint32_t>(seed), static_cast<uint32_t>(seed >> 32));
}

// ---------------------------------------------------------------------------
// absmax
// ---------------------------------------------------------------------------
template <typename T, bool WITH_RES>
__global__ void __launch_bounds__(kThreads)
    absmax_kernel(const T* __restrict__ x, const float* __restrict__ res, int64_t n, bool vec,
                  uint32_t* amax_bits) {
  float m = 0.0f;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t nthr = static_cast<int64_t>(gridDim.x) * blockDim.x;
  if (vec) {
    const int64_t n4 = n / 4;
    for (int64_t i = tid; i < n4; i += nthr) {
      float v[4];
      ElemIO<T>::load4(x + 4 * i, v);
      if constexpr (WITH_RES) {
        float r[4];
        ElemIO<float>::load4(res + 4 * i, r);
#pragma unroll
        for (int k = 0; k < 4; ++k) v[k] += r[k];
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) m = fmaxf(m, fabsf(v[k]));
    }
    for (int64_t i = 4 * n4 + tid; i < n; i += nthr) {
      float v = ElemIO<T>::load(x + i);
      if constexpr (WITH_RES) v += res[i];
      m = fmaxf(m, fabsf(v));
    }
  } else {
    for (int64_t i = tid; i < n; i += nthr) {
      float v = ElemIO<T>::load(x + i);
      if constexpr (WITH_RES) v += res[i];
      m = fmaxf(m, fabsf(v));
    }
  }
  m = warp_max(m);
  __shared__ float red[kWarps];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = m;
  __syncthreads();
  if (warp == 0) {
    m = lane < kWarps ? red[lane] : 0.0f;
    m = warp_max(m);
    if (lane == 0 && m > 0.0f) atomicMax(amax_bits, __float_as_uint(m));
  }
}

// ---------------------------------------------------------------------------
// quantise (+ pack) in the reference layout
// ---------------------------------------------------------------------------
template <typename T, int B, bool SR>
__global__ void __launch_bounds__(kThreads, 3)
    quantize_ref_kernel(const T* __restrict__ x, int64_t n, const uint32_t* __restrict__ amax_bits,
                        uint64_t seed, uint64_t offset, uint8_t* __restrict__ packed,
                        int16_t* __restrict__ q16, double* __restrict__ scale_out, bool vec_in,
                        bool vec_q, int64_t packed_len) {
  __shared__ float sm_all[kWarps][32 * kPitch];
  constexpr int qmin = QBounds<B>::qmin, qmax = QBounds<B>::qmax;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* sm = sm_all[warp];
  double sd;
  const float scale = scale_from_amax(*amax_bits, qmax, &sd);
  if (scale_out && blockIdx.x == 0 && threadIdx.x == 0) *scale_out = sd;
  const int64_t ntiles = (n + kTile - 1) / kTile;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * kWarps + warp; t < ntiles;
       t += static_cast<int64_t>(gridDim.x) * kWarps) {
    const int64_t base = t * kTile;
    TileIO<T>::load(x, base, n, vec_in, sm, lane);
    const int64_t e0 = base + lane * 32;
    uint32_t codes[32];
    Philox4 rnd{0u, 0u, 0u, 0u};
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const float v = __fdiv_rn(sm[lane * kPitch + j], scale);
      float r;
      if constexpr (SR) {
        if ((j & 3) == 0) rnd = philox_at(static_cast<uint64_t>(e0 + j) >> 2, seed, offset);
        r = sr_round(v, pick(rnd, j));
      } else {
        r = rintf(v);
      }
      r = fminf(fmaxf(r, static_cast<float>(qmin)), static_cast<float>(qmax));
      const int q = static_cast<int>(r);
      codes[j] = (e0 + j < n) ? static_cast<uint32_t>(q - qmin) : 0u;
      if (q16) sm[lane * kPitch + j] = static_cast<float>(q);
    }
    if (packed) {
      uint32_t w[B];
      pack32<B>(codes, w);
      store_words<B>(packed, t * 32 * B + lane * B, packed_len, w);
    }
    if (q16) {
      __syncwarp();
      store_tile_i16(q16, base, n, vec_q, sm, lane);
    }
    __syncwarp();
  }
}

// int16 codes -> packed reference layout
template <int B>
__global__ void __launch_bounds__(kThreads)
    pack_ref_kernel(const int16_t* __restrict__ q16, int64_t n, bool vec_in,
                    uint8_t* __restrict__ packed, int64_t packed_len) {
  __shared__ float sm_all[kWarps][32 * kPitch];
  constexpr int qmin = QBounds<B>::qmin;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* sm = sm_all[warp];
  const int64_t ntiles = (n + kTile - 1) / kTile;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * kWarps + warp; t < ntiles;
       t += static_cast<int64_t>(gridDim.x) * kWarps) {
    const int64_t base = t * kTile;
    TileIO<int16_t>::load(q16, base, n, vec_in, sm, lane);
    const int64_t e0 = base + lane * 32;
    uint32_t codes[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      int v = static_cast<int>(sm[lane * kPitch + j]) - qmin;
      v = v < 0 ? 0 : (v > static_cast<int>(QBounds<B>::mask) ? static_cast<int>(QBounds<B>::mask) : v);
      codes[j] = (e0 + j < n) ? static_cast<uint32_t>(v) : 0u;
    }
    uint32_t w[B];
    pack32<B>(codes, w);
    store_words<B>(packed, t * 32 * B + lane * B, packed_len, w);
    __syncwarp();
  }
}

// packed reference layout -> int16 codes and/or dequantised values
template <int B, typename OutT>
__global__ void __launch_bounds__(kThreads)
    unpack_ref_kernel(const uint8_t* __restrict__ packed, int64_t n, int64_t packed_len,
                      bool vec_in, int16_t* __restrict__ q16, bool vec_q, OutT* __restrict__ out,
                      bool vec_out, float scale, const float* __restrict__ scale_ptr) {
  __shared__ float sm_all[kWarps][32 * kPitch];
  constexpr int qmin = QBounds<B>::qmin;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* sm = sm_all[warp];
  const float sc = scale_ptr ? *scale_ptr : scale;
  const int64_t ntiles = (n + kTile - 1) / kTile;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * kWarps + warp; t < ntiles;
       t += static_cast<int64_t>(gridDim.x) * kWarps) {
    const int64_t base = t * kTile;
    uint32_t w[B];
    load_words<B>(packed, t * 32 * B + lane * B, packed_len, vec_in, w);
    uint32_t codes[32];
    unpack32<B>(w, codes);
#pragma unroll
    for (int j = 0; j < 32; ++j)
      sm[lane * kPitch + j] = static_cast<float>(static_cast<int>(codes[j]) + qmin);
    __syncwarp();
    if (q16) store_tile_i16(q16, base, n, vec_q, sm, lane);
    if (out) {
      if (q16) __syncwarp();
#pragma unroll
      for (int j = 0; j < 32; ++j) sm[lane * kPitch + j] = __fmul_rn(sm[lane * kPitch + j], sc);
      __syncwarp();
      store_tile<OutT>(out, base, n, vec_out, sm, lane);
    }
    __syncwarp();
  }
}

template <typename OutT>
__global__ void __launch_bounds__(kThreads)
    dequant_i16_kernel(const int16_t* __restrict__ q16, int64_t n, bool vec, OutT* __restrict__ out,
                       float scale, const float* __restrict__ scale_ptr) {
  const float sc = scale_ptr ? *scale_ptr : scale;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t nthr = static_cast<int64_t>(gridDim.x) * blockDim.x;
  if (vec) {
    const int64_t n4 = n / 4;
    for (int64_t i = tid; i < n4; i += nthr) {
      const uint2 t = __ldg(reinterpret_cast<const uint2*>(q16 + 4 * i));
      float v[4] = {static_cast<float>(static_cast<int16_t>(t.x & 0xffffu)) * sc,
                    static_cast<float>(static_cast<int16_t>(t.x >> 16)) * sc,
                    static_cast<float>(static_cast<int16_t>(t.y & 0xffffu)) * sc,
                    static_cast<float>(static_cast<int16_t>(t.y >> 16)) * sc};
      ElemIO<OutT>::store4(out + 4 * i, v);
    }
    for (int64_t i = 4 * n4 + tid; i < n; i += nthr)
      ElemIO<OutT>::store(out + i, static_cast<float>(q16[i]) * sc);
  } else {
    for (int64_t i = tid; i < n; i += nthr) ElemIO<OutT>::store(out + i, static_cast<float>(q16[i]) * sc);
  }
}

// corrected = x + residual ; y = dequant(quant(corrected)) ; residual = corrected - y
template <typename T, int B, bool SR>
__global__ void __launch_bounds__(kThreads)
    ef_roundtrip_kernel(const T* __restrict__ x, int64_t n, bool vec, float* __restrict__ residual,
                        const uint32_t* __restrict__ amax_bits, uint64_t seed, uint64_t offset,
                        T* __restrict__ y) {
  constexpr int qmin = QBounds<B>::qmin, qmax = QBounds<B>::qmax;
  const float scale = scale_from_amax(*amax_bits, qmax, nullptr);
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t nthr = static_cast<int64_t>(gridDim.x) * blockDim.x;
  auto one = [&](float c, int64_t e, uint32_t r) -> float {
    const float v = __fdiv_rn(c, scale);
    float q = SR ? sr_round(v, r) : rintf(v);
    q = fminf(fmaxf(q, static_cast<float>(qmin)), static_cast<float>(qmax));
    (void)e;
    return __fmul_rn(q, scale);  // not contracted with the residual subtraction
  };
  const int64_t n4 = vec ? n / 4 : 0;
  for (int64_t i = tid; i < n4; i += nthr) {
    float v[4], r[4] = {0.f, 0.f, 0.f, 0.f};
    ElemIO<T>::load4(x + 4 * i, v);
    if (residual) ElemIO<float>::load4(residual + 4 * i, r);
    Philox4 rnd{0u, 0u, 0u, 0u};
    if constexpr (SR) rnd = philox_at(static_cast<uint64_t>(i), seed, offset);
    float o[4], nr[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float c = __fadd_rn(v[k], r[k]);
      o[k] = one(c, 4 * i + k, pick(rnd, k));
      nr[k] = __fsub_rn(c, o[k]);
    }
    ElemIO<T>::store4(y + 4 * i, o);
    if (residual) ElemIO<float>::store4(residual + 4 * i, nr);
  }
  for (int64_t i = 4 * n4 + tid; i < n; i += nthr) {
    const float c = __fadd_rn(ElemIO<T>::load(x + i), residual ? residual[i] : 0.0f);
    Philox4 rnd{0u, 0u, 0u, 0u};
    if constexpr (SR) rnd = philox_at(static_cast<uint64_t>(i) >> 2, seed, offset);
    const float o = one(c, i, pick(rnd, static_cast<int>(i & 3)));
    ElemIO<T>::store(y + i, o);
    if (residual) residual[i] = __fsub_rn(c, o);
  }
}

// ---------------------------------------------------------------------------
// launch helpers
// ---------------------------------------------------------------------------
inline void check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

inline int sm_count() {
  static int cached = 0;
  if (cached == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&cached, cudaDevAttrMultiProcessorCount, dev);
    if (cached <= 0) cached = 148;
  }
  return cached;
}

inline int grid_for(int64_t work_items, int per_block, int waves = 4) {
  const int64_t need = (work_items + per_block - 1) / per_block;
  const int64_t cap = static_cast<int64_t>(sm_count()) * waves;
  const int64_t g = need < cap ? need : cap;
  return static_cast<int>(g < 1 ? 1 : g);
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <typename F>
void dispatch_dtype(DType dt, F&& f) {
  switch (dt) {
    case kF32: f(static_cast<float*>(nullptr)); break;
    case kBF16: f(static_cast<__nv_bfloat16*>(nullptr)); break;
    case kF16: f(static_cast<__half*>(nullptr)); break;
    default: throw std::runtime_error("bitscom: unsupported dtype");
  }
}

template <typename F>
void dispatch_bits(int bits, F&& f) {
  switch (bits) {
    case 1: f(std::integral_constant<int, 1>{}); break;
    case 2: f(std::integral_constant<int, 2>{}); break;
    case 4: f(std::integral_constant<int, 4>{}); break;
    case 8: f(std::integral_constant<int, 8>{}); break;
    case 12: f(std::integral_constant<int, 12>{}); break;
    case 16: f(std::integral_constant<int, 16>{}); break;
    default: throw std::runtime_error("bitscom: bitwidth must be one of 1,2,4,8,12,16");
  }
}

}  // namespace

namespace launch {

void absmax(const void* x, DType dt, int64_t n, uint32_t* amax_bits, cudaStream_t s) {
  if (n <= 0) return;
  dispatch_dtype(dt, [&](auto tag) {
    using T = std::remove_pointer_t<decltype(tag)>;
    const int g = grid_for(n / 4 + 1, kThreads, 8);
    absmax_kernel<T, false><<<g, kThreads, 0, s>>>(static_cast<const T*>(x), nullptr, n,
                                                   aligned16(x), amax_bits);
  });
  check_launch("absmax_kernel");
}

void absmax_sum(const void* x, DType dt, const float* residual, int64_t n, uint32_t* amax_bits,
                cudaStream_t s) {
  if (n <= 0) return;
  dispatch_dtype(dt, [&](auto tag) {
    using T = std::remove_pointer_t<decltype(tag)>;
    const int g = grid_for(n / 4 + 1, kThreads, 8);
    absmax_kernel<T, true><<<g, kThreads, 0, s>>>(static_cast<const T*>(x), residual, n,
                                                  aligned16(x) && aligned16(residual), amax_bits);
  });
  check_launch("absmax_kernel(x+residual)");
}

void quantize_ref(const void* x, DType dt, int64_t n, int bits, const uint32_t* amax_bits,
                  bool stochastic, uint64_t seed, uint64_t offset, uint8_t* packed, int16_t* q16,
                  double* scale_out, cudaStream_t s) {
  if (n <= 0) return;
  const int64_t plen = packed_bytes_ref(n, bits);
  // Three CTAs per SM (the kernel is bounded to 85 registers): the grid is
  // exactly one resident wave.
  const int g = grid_for((n + kTile - 1) / kTile, kWarps, 3);
  dispatch_dtype(dt, [&](auto tag) {
    using T = std::remove_pointer_t<decltype(tag)>;
    dispatch_bits(bits, [&](auto bc) {
      constexpr int B = decltype(bc)::value;
      if (packed && !aligned16(packed)) throw std::runtime_error("quantize_ref: packed output must be 16-byte aligned");
      if (stochastic)
        quantize_ref_kernel<T, B, true><<<g, kThreads, 0, s>>>(
            static_cast<const T*>(x), n, amax_bits, seed, offset, packed, q16, scale_out,
            aligned16(x), q16 && aligned16(q16), plen);
      else
        quantize_ref_kernel<T, B, false><<<g, kThreads, 0, s>>>(
            static_cast<const T*>(x), n, amax_bits, seed, offset, packed, q16, scale_out,
            aligned16(x), q16 && aligned16(q16), plen);
    });
  });
  check_launch("quantize_ref_kernel");
}

void pack_ref(const int16_t* q16, int64_t n, int bits, uint8_t* packed, cudaStream_t s) {
  if (n <= 0) return;
  if (!aligned16(packed)) throw std::runtime_error("pack_ref: packed output must be 16-byte aligned");
  const int64_t plen = packed_bytes_ref(n, bits);
  const int g = grid_for((n + kTile - 1) / kTile, kWarps, 4);
  dispatch_bits(bits, [&](auto bc) {
    constexpr int B = decltype(bc)::value;
    pack_ref_kernel<B><<<g, kThreads, 0, s>>>(q16, n, aligned16(q16), packed, plen);
  });
  check_launch("pack_ref_kernel");
}

void unpack_ref(const uint8_t* packed, int64_t n, int bits, int16_t* q16, void* out, DType out_dt,
                float scale, const float* scale_ptr, cudaStream_t s) {
  if (n <= 0) return;
  const int64_t plen = packed_bytes_ref(n, bits);
  const int g = grid_for((n + kTile - 1) / kTile, kWarps, 4);
  dispatch_dtype(out_dt, [&](auto tag) {
    using T = std::remove_pointer_t<decltype(tag)>;
    dispatch_bits(bits, [&](auto bc) {
      constexpr int B = decltype(bc)::value;
      unpack_ref_kernel<B, T><<<g, kThreads, 0, s>>>(
          packed, n, plen, aligned16(packed), q16, q16 && aligned16(q16), static_cast<T*>(out),
          out && aligned16(out), scale, scale_ptr);
    });
  });
  check_launch("unpack_ref_kernel");
}

void dequantize_i16(const int16_t* q16, int64_t n, void* out, DType out_dt, float scale,
                    const float* scale_ptr, cudaStream_t s) {
  if (n <= 0) return;
  dispatch_dtype(out_dt, [&](auto tag) {
    using T = std::remove_pointer_t<decltype(tag)>;
    const int g = grid_for(n / 4 + 1, kThreads, 8);
    dequant_i16_kernel<T><<<g, kThreads, 0, s>>>(q16, n, aligned16(q16) && aligned16(out),
                                                 static_cast<T*>(out), scale, scale_ptr);
  });
  check_launch("dequant_i16_kernel");
}

void ef_roundtrip_ref(const void* x, DType dt, int64_t n, int bits, float* residual,
                      const uint32_t* amax_bits, bool stochastic, uint64_t seed, uint64_t offset,
                      void* y, cudaStream_t s) {
  if (n <= 0) return;
  dispatch_dtype(dt, [&](auto tag) {
    using T = std::remove_pointer_t<decltype(tag)>;
    dispatch_bits(bits, [&](auto bc) {
      constexpr int B = decltype(bc)::value;
      const int g = grid_for(n / 4 + 1, kThreads, 8);
      const bool vec = aligned16(x) && aligned16(y) && (residual == nullptr || aligned16(residual));
      if (stochastic)
        ef_roundtrip_kernel<T, B, true><<<g, kThreads, 0, s>>>(
            static_cast<const T*>(x), n, vec, residual, amax_bits, seed, offset, static_cast<T*>(y));
      else
        ef_roundtrip_kernel<T, B, false><<<g, kThreads, 0, s>>>(
            static_cast<const T*>(x), n, vec, residual, amax_bits, seed, offset, static_cast<T*>(y));
    });
  });
  check_launch("ef_roundtrip_kernel");
}

}  // namespace launch
}  // namespace bitscom_b200
