// Allocation-free C entry point of the fused low-bit reduction.
//
// This entry point has no counterpart in the reference implementation.
//
// bitscom_lowbit_allreduce_local_noalloc() runs the fused low-bit
// collective kernel (lowbit_coll.cu) at world size 1 — quantise (in +
// residual) with 1024-element block scales, update the error-feedback
// residual, dequantise-reduce, requantise and decode into `out`, exactly what
// LowBitComm::allreduce does on a one-rank communicator — without allocating
// any memory.  It is meant for callers that cannot call cudaMalloc: code that
// owns all device memory through its own arena or pool (an inference server,
// an embedding runtime, a foreign-function caller that hands over
// pre-allocated buffers) and code running where an allocation would stall or
// is not allowed (a latency-critical step, a region where the caching
// allocator must not grow).  The caller passes the input, output and residual
// buffers; the kernel's scratch (work counters, completion flags, packed
// intermediate sub-chunks, status word) lives in one file-scope
// `static __device__ __align__(256)` array of kNoAllocScratchBytes bytes,
// which every GPU that loads the library holds until the process exits.
//
// Limits and rules:
//   * n <= bitscom_noalloc_max_elems() (1,048,576 elements); larger n is
//     rejected with BITSCOM_NOALLOC_ETOOBIG and nothing is launched;
//   * dtype: 0 = float32, 1 = bfloat16, 2 = float16; bits in {1,2,4,8,12,16};
//     residual is float32 with n elements, or null for no error feedback;
//   * the first call on a device performs a one-time set-up with that device
//     current (it looks up the device address of the scratch array with
//     cudaGetSymbolAddress and clears the scratch's counters and flags with
//     cudaMemsetAsync on the given stream), so make the first call on a
//     device before any stream capture begins on that device;
//   * every call on a device shares the same scratch, which keeps the last
//     call's contents: calls must be ordered on the GPU (one stream, or
//     explicit dependencies).  Calls that overlap on the GPU race and produce
//     wrong results.
//   * a call returns as soon as its kernel is enqueued, so its return code
//     covers argument checks, set-up and the launch only; a kernel that gave
//     up waiting reports through bitscom_noalloc_status();
//   * no cudaMalloc, cudaFree, host allocation or allocating library routine
//     is called.
#pragma once

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BITSCOM_NOALLOC_OK 0
#define BITSCOM_NOALLOC_EINVAL (-1)   /* bad dtype, bitwidth, pointer or negative n */
#define BITSCOM_NOALLOC_ETOOBIG (-2)  /* n exceeds bitscom_noalloc_max_elems() */
#define BITSCOM_NOALLOC_ECUDA (-3)    /* set-up or launch failed (see cudaGetLastError) */

// Returns BITSCOM_NOALLOC_OK or one of the error codes above.  `stream` is a
// cudaStream_t (0 = legacy default stream).
int bitscom_lowbit_allreduce_local_noalloc(const void* in, void* out, float* residual, long long n, int dtype,
                                           int bits, float post_scale, void* stream);

// Largest n accepted.
long long bitscom_noalloc_max_elems(void);

// Bytes of the static scratch array.
long long bitscom_noalloc_scratch_bytes(void);

// Status of the calls completed so far on the current device: 0 when every
// kernel finished normally, otherwise the kernel's status bits (1 = a wait on
// a completion flag gave up after its time limit; the output and residual of
// that call are then incomplete).  A kernel writes the word only on failure,
// so read it after synchronising with the calls it should cover; `reset` != 0
// clears it.  Returns BITSCOM_NOALLOC_ECUDA if the read fails.  Synchronous.
int bitscom_noalloc_status(int reset);

// Human-readable message of an error code.
const char* bitscom_noalloc_strerror(int code);

#ifdef __cplusplus
}
#endif
