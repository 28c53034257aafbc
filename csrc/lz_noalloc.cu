// Allocation-free variant of the codec encoder (contract in lz_noalloc.h).
// The scratch the compact encoder needs (table-group slots, record sizes and
// offsets) is a file-scope __device__ array instead of caller or runtime
// allocated memory. This entry point has no counterpart in the reference.
#include <mutex>

#include "lz_codec_format.h"
#include "lz_internal.h"
#include "lz_noalloc.h"

extern "C" size_t lz_codec_scratch_bytes(size_t n, int dtype);
extern "C" int lz_codec_encode(const void* in, size_t n, int dtype, void* scratch,
                               size_t scratch_bytes, void* out, size_t out_cap,
                               unsigned long long* d_total, int nblocks, cudaStream_t s);

static __device__ __align__(256) unsigned char g_noalloc_scratch[LZ_NOALLOC_SCRATCH_BYTES];

namespace {
std::mutex g_mu;
void* g_scratch_addr[LZ_NOALLOC_MAX_DEVICES] = {nullptr};

// Device address of the array for the current device, looked up once per
// device. In host code `g_noalloc_scratch` names a host-side stand-in, so
// it is never passed to a kernel directly.
int scratch_for_current_device(void** out) {
  int dev = -1;
  LZ_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= LZ_NOALLOC_MAX_DEVICES) {
    lz_set_error("noalloc encoder: device %d out of range", dev);
    return LZE_ARG;
  }
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      lz_set_error("noalloc encoder: cudaGetSymbolAddress failed on device %d: %s", dev,
                   cudaGetErrorString(e));
      return LZE_CUDA;
    }
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return LZE_OK;
}
}  // namespace

extern "C" size_t lz_codec_noalloc_max_elems(int dtype) {
  dtype = lzc::codec_dtype(dtype);
  if (!lzc::valid_dtype(dtype)) return 0;
  // largest table-group count whose scratch fits, times the group size
  size_t lo = 0, hi = (size_t)LZ_NOALLOC_SCRATCH_BYTES / 16 + 1;
  while (hi - lo > 1) {
    const size_t mid = (lo + hi) / 2;
    if (lz_codec_scratch_bytes(mid * lzc::TG_ELEMS, dtype) <= LZ_NOALLOC_SCRATCH_BYTES) lo = mid;
    else hi = mid;
  }
  return lo * lzc::TG_ELEMS;
}

extern "C" int lz_codec_encode_noalloc(const void* in, size_t n, int dtype, void* out,
                                       size_t out_cap, unsigned long long* d_total,
                                       cudaStream_t stream) {
  if (!lzc::valid_dtype(lzc::codec_dtype(dtype)) || !lzc::valid_level(lzc::codec_level(dtype))) {
    lz_set_error("noalloc encoder: unsupported dtype/level argument %d", dtype);
    return LZE_ARG;
  }
  const size_t need = lz_codec_scratch_bytes(n, dtype);
  if (need > LZ_NOALLOC_SCRATCH_BYTES) {
    lz_set_error(
        "noalloc encoder: %zu elements need %zu bytes of scratch, above the fixed %u-byte "
        "array (at most %zu elements for this dtype); use lz_codec_encode with caller scratch",
        n, need, (unsigned)LZ_NOALLOC_SCRATCH_BYTES, lz_codec_noalloc_max_elems(dtype));
    return LZE_ARG;
  }
  void* scratch = nullptr;
  int rc = scratch_for_current_device(&scratch);
  if (rc) return rc;
  return lz_codec_encode(in, n, dtype, scratch, LZ_NOALLOC_SCRATCH_BYTES, out, out_cap, d_total, 0,
                         stream);
}
