// Allocation-free codec entry point.
//
// Declaration: this entry point has no counterpart in the reference
// (monopodium/results); it is an addition of this library.
//
// Some callers cannot call cudaMalloc at the moment they need to compress:
// a serving process that reserved all of its HBM for weights and KV cache at
// start-up and may not grow its footprint afterwards, or a latency-critical
// path that must not hit cudaMalloc's implicit device synchronisation. For
// them, lz_codec_encode_noalloc() compresses into a caller-provided output
// using a scratch area that lives in a fixed-size file-scope __device__ array
// of the library, so the call itself allocates nothing.
//
// Limits and contract:
//   * Scratch is LZ_NOALLOC_SCRATCH_BYTES (32 MiB) per GPU that loads the
//     library, held until the process exits. Inputs whose scratch need
//     (lz_codec_scratch_bytes) exceeds it are rejected with LZE_ARG and a
//     message naming the limit; lz_codec_noalloc_max_elems() gives the largest
//     accepted element count per dtype (16,744,448 for bf16 and fp16,
//     8,355,840 for fp32, 33,488,896 for 8-bit data).
//   * The first call on a device looks up the array's device address
//     (cudaGetSymbolAddress, once per device, with that device current). Make
//     that first call before any stream capture on the device.
//   * Every call on a device shares the one array and it keeps the previous
//     call's contents; the encoder overwrites everything it reads, so nothing
//     has to start at zero. Calls whose executions overlap on the GPU (e.g. on
//     two streams without ordering between them) race on the array: order
//     them on one stream or serialise them.
//   * Every dtype of lz_codec_encode() is accepted (fp32, fp16, bf16, bytes
//     and the packed fp8 pair containers e4m3 / e5m2, whose element count is
//     the number of pairs), with the encoder level in the same argument
//     (dtype | level << 8); output is byte-identical to lz_codec_encode()
//     with caller scratch.
#pragma once
#include <stddef.h>
#include <cuda_runtime.h>

#define LZ_NOALLOC_SCRATCH_BYTES (32u << 20)
#define LZ_NOALLOC_MAX_DEVICES 64

#ifdef __cplusplus
extern "C" {
#endif

// Compact LZC1 stream of `n` elements of `dtype` from `in` into `out`
// (capacity lz_codec_max_bytes(n, dtype)); the stream size is written to the
// device word *d_total. Stream-ordered on `stream`; returns 0 or an LZE_* code.
int lz_codec_encode_noalloc(const void* in, size_t n, int dtype, void* out, size_t out_cap,
                            unsigned long long* d_total, cudaStream_t stream);

// Largest element count lz_codec_encode_noalloc accepts for `dtype`.
size_t lz_codec_noalloc_max_elems(int dtype);

#ifdef __cplusplus
}
#endif
