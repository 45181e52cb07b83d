// Shared device helpers for the bitscom_b200 sm_100a kernels.
//
// Contents:
//   * quantisation bounds for the supported bitwidths {1,2,4,8,12,16}
//     (reference semantics: python/bitscom/quantization.py:37-43 — 1-bit is
//     the unsigned pair {0,1}, every other width is signed two's-complement);
//   * a Philox-4x32-10 counter RNG written from Salmon, Moraes, Dror & Shaw,
//     "Parallel random numbers: as easy as 1, 2, 3" (SC'11), used for
//     stochastic rounding;
//   * bit-stream packing of 32 b-bit codes into exactly b 32-bit words.  All
//     six reference layouts (quantization.py:118-196) are the same
//     little-endian LSB-first b-bit stream of the offset code (q - qmin), so a
//     single compile-time-unrolled routine covers 1/2/4/8/12/16 bits;
//   * load/convert helpers for fp32 / bf16 / fp16 inputs;
//   * system-scope release/acquire flag operations and %globaltimer for the
//     bounded peer waits used by the fused collectives.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace bitscom_b200 {

// ---------------------------------------------------------------------------
// Quantisation bounds
// ---------------------------------------------------------------------------
template <int B>
struct QBounds {
  static constexpr int qmin = (B == 1) ? 0 : -(1 << (B - 1));
  static constexpr int qmax = (B == 1) ? 1 : (1 << (B - 1)) - 1;
  static constexpr uint32_t mask = (B >= 32) ? 0xffffffffu : ((1u << B) - 1u);
};

// ---------------------------------------------------------------------------
// Philox-4x32-10 (Salmon et al., SC'11, section 5: multipliers 0xD2511F53 and
// 0xCD9E8D57, Weyl key increments 0x9E3779B9 (golden ratio) and 0xBB67AE85
// (sqrt(3)-1)).  One call turns a 128-bit counter into four 32-bit outputs.
// ---------------------------------------------------------------------------
struct Philox4 {
  uint32_t x, y, z, w;
};

__device__ __forceinline__ Philox4 philox4x32_10(Philox4 c, uint32_t k0, uint32_t k1) {
  constexpr uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u;
  constexpr uint32_t W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(M0, c.x), lo0 = M0 * c.x;
    const uint32_t hi1 = __umulhi(M1, c.z), lo1 = M1 * c.z;
    Philox4 n;
    n.x = hi1 ^ c.y ^ k0;
    n.y = lo1;
    n.z = hi0 ^ c.w ^ k1;
    n.w = lo0;
    c = n;
    k0 += W0;
    k1 += W1;
  }
  return c;
}

// Uniform float in [0, 1) with 24 random bits (exactly representable).
__device__ __forceinline__ float u01(uint32_t r) {
  return static_cast<float>(r >> 8) * (1.0f / 16777216.0f);
}

// Stochastic rounding of v: floor(v) + 1 with probability frac(v).
__device__ __forceinline__ float sr_round(float v, uint32_t r) {
  const float lo = floorf(v);
  return lo + ((u01(r) < (v - lo)) ? 1.0f : 0.0f);
}

// ---------------------------------------------------------------------------
// Bit packing: 32 codes of B bits <-> B words, element j at stream bit j*B.
// ---------------------------------------------------------------------------
template <int B>
__device__ __forceinline__ void pack32(const uint32_t (&v)[32], uint32_t (&w)[B]) {
#pragma unroll
  for (int i = 0; i < B; ++i) w[i] = 0u;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const int bit = j * B;
    const int wi = bit >> 5;
    const int off = bit & 31;
    w[wi] |= v[j] << off;
    if (off + B > 32) w[wi + 1] |= v[j] >> (32 - off);
  }
}

template <int B>
__device__ __forceinline__ void unpack32(const uint32_t (&w)[B], uint32_t (&v)[32]) {
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const int bit = j * B;
    const int wi = bit >> 5;
    const int off = bit & 31;
    uint32_t x = w[wi] >> off;
    if (off + B > 32) x |= w[wi + 1] << (32 - off);
    v[j] = x & QBounds<B>::mask;
  }
}

// ---------------------------------------------------------------------------
// Element load / store helpers
// ---------------------------------------------------------------------------
template <typename T>
struct ElemIO;

template <>
struct ElemIO<float> {
  __device__ __forceinline__ static float load(const float* p) { return *p; }
  __device__ __forceinline__ static void store(float* p, float v) { *p = v; }
  // Loads 4 consecutive elements from a 16-byte aligned address.
  __device__ __forceinline__ static void load4(const float* p, float (&o)[4]) {
    const float4 t = __ldg(reinterpret_cast<const float4*>(p));
    o[0] = t.x; o[1] = t.y; o[2] = t.z; o[3] = t.w;
  }
  __device__ __forceinline__ static void store4(float* p, const float (&o)[4]) {
    *reinterpret_cast<float4*>(p) = make_float4(o[0], o[1], o[2], o[3]);
  }
  static constexpr int kAlign = 16;
};

template <>
struct ElemIO<__nv_bfloat16> {
  __device__ __forceinline__ static float load(const __nv_bfloat16* p) { return __bfloat162float(*p); }
  __device__ __forceinline__ static void store(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }
  __device__ __forceinline__ static void load4(const __nv_bfloat16* p, float (&o)[4]) {
    const uint2 t = __ldg(reinterpret_cast<const uint2*>(p));
    const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&t.x);
    const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&t.y);
    const float2 fa = __bfloat1622float2(a), fb = __bfloat1622float2(b);
    o[0] = fa.x; o[1] = fa.y; o[2] = fb.x; o[3] = fb.y;
  }
  __device__ __forceinline__ static void store4(__nv_bfloat16* p, const float (&o)[4]) {
    __nv_bfloat162 a = __floats2bfloat162_rn(o[0], o[1]);
    __nv_bfloat162 b = __floats2bfloat162_rn(o[2], o[3]);
    uint2 t;
    t.x = *reinterpret_cast<uint32_t*>(&a);
    t.y = *reinterpret_cast<uint32_t*>(&b);
    *reinterpret_cast<uint2*>(p) = t;
  }
  static constexpr int kAlign = 8;
};

template <>
struct ElemIO<__half> {
  __device__ __forceinline__ static float load(const __half* p) { return __half2float(*p); }
  __device__ __forceinline__ static void store(__half* p, float v) { *p = __float2half_rn(v); }
  __device__ __forceinline__ static void load4(const __half* p, float (&o)[4]) {
    const uint2 t = __ldg(reinterpret_cast<const uint2*>(p));
    const __half2 a = *reinterpret_cast<const __half2*>(&t.x);
    const __half2 b = *reinterpret_cast<const __half2*>(&t.y);
    const float2 fa = __half22float2(a), fb = __half22float2(b);
    o[0] = fa.x; o[1] = fa.y; o[2] = fb.x; o[3] = fb.y;
  }
  __device__ __forceinline__ static void store4(__half* p, const float (&o)[4]) {
    __half2 a = __floats2half2_rn(o[0], o[1]);
    __half2 b = __floats2half2_rn(o[2], o[3]);
    uint2 t;
    t.x = *reinterpret_cast<uint32_t*>(&a);
    t.y = *reinterpret_cast<uint32_t*>(&b);
    *reinterpret_cast<uint2*>(p) = t;
  }
  static constexpr int kAlign = 8;
};

// ---------------------------------------------------------------------------
// Warp reductions
// ---------------------------------------------------------------------------
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ---------------------------------------------------------------------------
// System-scope flags (NVLink peers) and the global nanosecond timer.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint32_t ld_relaxed_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// L2-only (L1-bypassing) 16-byte load, used for buffers that peers write.
__device__ __forceinline__ uint4 ld_cg_v4(const void* p) {
  return __ldcg(reinterpret_cast<const uint4*>(p));
}

}  // namespace bitscom_b200
