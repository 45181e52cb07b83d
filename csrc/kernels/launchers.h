// Host-side launch interface of the bitscom_b200 CUDA kernels.
//
// Every launcher takes raw device pointers, element counts and the CUDA stream
// to run on (always the caller's current stream — the reference launched on the
// legacy default stream, lowbit_cuda_kernels.cu:159).  Nothing here allocates:
// scratch (the absmax word, the scale output) is passed in by the caller.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace bitscom_b200 {

enum DType : int { kF32 = 0, kBF16 = 1, kF16 = 2 };

// Packed size in bytes of `numel` codes in the reference layout: whole bytes
// for 1/2/4/8 bits, whole 3-byte pairs for 12 bits, 2 bytes per code for 16
// (reference python/bitscom/quantization.py:118-164).
inline int64_t packed_bytes_ref(int64_t numel, int b) {
  if (b <= 8) {
    const int per = 8 / b;
    return (numel + per - 1) / per;
  }
  if (b == 12) return ((numel + 1) / 2) * 3;
  return numel * 2;
}

namespace launch {

// |x|_max of n elements, accumulated with atomicMax into *amax_bits (the float
// bit pattern; non-negative floats order like unsigned ints).  *amax_bits must
// be zero (or a previous partial result) on entry.
void absmax(const void* x, DType dt, int64_t n, uint32_t* amax_bits, cudaStream_t s);

// Reference-compatible per-tensor quantisation + packing.
//   scale = amax == 0 ? 1 : amax / qmax  (computed in double, used as float)
//   q     = clamp(round_half_even(x / scale), qmin, qmax)     [deterministic]
//   q     = clamp(floor(x/scale) + (u < frac), qmin, qmax)    [stochastic]
// Writes the packed reference layout to `packed` (may be null) and the int16
// codes to `q16` (may be null); thread 0 writes the double scale to
// `scale_out` (may be null).  SR uses Philox(seed, offset).
void quantize_ref(const void* x, DType dt, int64_t n, int bits, const uint32_t* amax_bits,
                  bool stochastic, uint64_t seed, uint64_t offset, uint8_t* packed,
                  int16_t* q16, double* scale_out, cudaStream_t s);

// int16 codes -> packed reference layout (codes are clamped to the range).
void pack_ref(const int16_t* q16, int64_t n, int bits, uint8_t* packed, cudaStream_t s);

// packed reference layout -> int16 codes (q16 non-null) and/or dequantised
// values out = float(q) * scale written as `out_dt` (out non-null).  The scale
// is read from *scale_ptr when non-null, otherwise `scale` is used.
void unpack_ref(const uint8_t* packed, int64_t n, int bits, int16_t* q16, void* out,
                DType out_dt, float scale, const float* scale_ptr, cudaStream_t s);

// int16 codes -> out = float(q) * scale.
void dequantize_i16(const int16_t* q16, int64_t n, void* out, DType out_dt, float scale,
                    const float* scale_ptr, cudaStream_t s);

// Error-feedback roundtrip used by simulate_quantization and the EF
// benchmarks: corrected = x + residual; y = dequant(quant(corrected)) with a
// per-tensor scale from *amax_bits (the absmax of `corrected`); residual is
// overwritten with corrected - y when non-null.
void ef_roundtrip_ref(const void* x, DType dt, int64_t n, int bits, float* residual,
                      const uint32_t* amax_bits, bool stochastic, uint64_t seed,
                      uint64_t offset, void* y, cudaStream_t s);

// absmax of (x + residual) for the EF roundtrip.
void absmax_sum(const void* x, DType dt, const float* residual, int64_t n, uint32_t* amax_bits,
                cudaStream_t s);

}  // namespace launch
}  // namespace bitscom_b200

#include "coll_params.h"

namespace bitscom_b200 {
namespace launch {

// Bytes of one packed sub-chunk (8 x 1024 elements) at `bits` per element.
int64_t coll_sub_bytes(int bits);

// Launches one fused low-bit collective (see lowbit_coll.cu).
void lowbit_coll(const CollParams& p, DType dt, int bits, int grid, cudaStream_t s);

// The same launch reporting errors through the return value instead of
// exceptions (no host allocation on any path).
cudaError_t lowbit_coll_nothrow(const CollParams& p, DType dt, int bits, int grid, cudaStream_t s);

}  // namespace launch
}  // namespace bitscom_b200
