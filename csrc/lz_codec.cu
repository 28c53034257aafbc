// Standalone LZC1 codec kernels (GPU). Whole-tensor compact streams are
// produced in three stream-ordered launches: every CTA encodes table groups
// into fixed-capacity slots of a scratch buffer (recording each record's
// size), one CTA scans the sizes into offsets, and a gather kernel packs the
// records behind the stream header. Decoding validates every record and
// reports corruption through a status word instead of trapping (the
// reference's codec asserted on a bad header, raw/a.txt:290-320 of the
// reference).
#include <stdlib.h>

#include <cub/block/block_scan.cuh>

#include "lz_codec_dev.cuh"
#include "lz_internal.h"

using namespace lzc;
using namespace lzg;

namespace {

template <int DT, int LEVEL>
__global__ void __launch_bounds__(LZC_THREADS, LZC_MIN_BLOCKS) encode_slotted_kernel(const char* __restrict__ in,
                                                                      uint64_t n, char* slots,
                                                                      uint32_t slot_cap,
                                                                      uint32_t* sizes, int stop_after) {
  extern __shared__ __align__(16) char smem_raw[];
  EncSmem& sm = *reinterpret_cast<EncSmem*>(smem_raw);
  constexpr int ES = DT == DT_F32 ? 4 : (DT == DT_U8 ? 1 : 2);
  const uint64_t ntg = num_tgs(n);
  for (uint64_t t = blockIdx.x; t < ntg; t += gridDim.x) {
    const uint32_t tn = (uint32_t)min((uint64_t)TG_ELEMS, n - t * TG_ELEMS);
    const uint32_t bytes =
        encode_tg<DT>(in + t * (uint64_t)TG_ELEMS * ES, tn, slots + t * (uint64_t)slot_cap, sm, LEVEL, stop_after);
    if (threadIdx.x == 0) sizes[t] = bytes;
  }
}

// Exclusive scan of record sizes -> offsets (stream positions), one CTA.
__global__ void __launch_bounds__(1024) scan_sizes_kernel(const uint32_t* sizes, uint64_t ntg,
                                                          uint64_t* offsets, uint64_t base,
                                                          unsigned long long* total) {
  using Scan = cub::BlockScan<unsigned long long, 1024>;
  __shared__ typename Scan::TempStorage tmp;
  __shared__ unsigned long long carry;
  if (threadIdx.x == 0) carry = base;
  __syncthreads();
  for (uint64_t b0 = 0; b0 < ntg; b0 += 1024) {
    const uint64_t i = b0 + threadIdx.x;
    unsigned long long v = i < ntg ? sizes[i] : 0ull, ex, agg;
    Scan(tmp).ExclusiveSum(v, ex, agg);
    if (i < ntg) offsets[i] = carry + ex;
    __syncthreads();
    if (threadIdx.x == 0) carry += agg;
    __syncthreads();
  }
  if (threadIdx.x == 0) *total = carry;
}

__global__ void gather_records_kernel(const char* __restrict__ slots, uint32_t slot_cap,
                                      const uint32_t* __restrict__ sizes,
                                      const uint64_t* __restrict__ offsets, uint64_t ntg,
                                      char* __restrict__ out, uint64_t n, int dt,
                                      const unsigned long long* total) {
  // header + offset table by block 0
  if (blockIdx.x == 0) {
    const uint64_t tab = sizeof(StreamHeader);
    for (uint64_t i = threadIdx.x; i < ntg; i += blockDim.x)
      reinterpret_cast<uint64_t*>(out + tab)[i] = offsets[i];
    const uint64_t tab_end = tab + 8 * ntg, tab_pad = pad16_64(tab_end);
    if (threadIdx.x < tab_pad - tab_end) out[tab_end + threadIdx.x] = 0;
    if (threadIdx.x == 0) {
      StreamHeader h;
      memset(&h, 0, sizeof(h));
      h.magic = STREAM_MAGIC;
      h.version = VERSION;
      h.dtype = (uint8_t)dt;
      h.tg_elems = TG_ELEMS;
      h.n_tg = (uint32_t)ntg;
      h.n_elems = n;
      h.total_bytes = *total;
      memcpy(out, &h, sizeof(h));
    }
  }
  for (uint64_t t = blockIdx.x; t < ntg; t += gridDim.x) {
    const char* src = slots + t * (uint64_t)slot_cap;
    char* dst = out + offsets[t];
    const uint32_t bytes = sizes[t];
    for (uint32_t o = threadIdx.x * 16; o < bytes; o += blockDim.x * 16)
      *reinterpret_cast<uint4*>(dst + o) = *reinterpret_cast<const uint4*>(src + o);
  }
}

template <int DT>
__global__ void __launch_bounds__(LZC_THREADS, LZC_MIN_BLOCKS) decode_stream_kernel(const char* __restrict__ st,
                                                                     uint64_t stream_bytes,
                                                                     char* __restrict__ out,
                                                                     uint64_t n, int* status) {
  extern __shared__ __align__(16) char smem_raw[];
  DecSmem& sm = *reinterpret_cast<DecSmem*>(smem_raw);
  constexpr int ES = DT == DT_F32 ? 4 : (DT == DT_U8 ? 1 : 2);
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    const StreamHeader* h = reinterpret_cast<const StreamHeader*>(st);
    s_ok = stream_bytes >= sizeof(StreamHeader) && h->magic == STREAM_MAGIC &&
           h->version == VERSION && h->dtype == DT && h->n_elems == n && h->tg_elems == TG_ELEMS &&
           h->n_tg == num_tgs(n) && h->total_bytes <= stream_bytes;
    if (!s_ok) atomicCAS(status, 0, 1);
  }
  __syncthreads();
  if (!s_ok) return;
  const uint64_t total = reinterpret_cast<const StreamHeader*>(st)->total_bytes;
  const uint64_t* offs = reinterpret_cast<const uint64_t*>(st + sizeof(StreamHeader));
  const uint64_t ntg = num_tgs(n);
  for (uint64_t t = blockIdx.x; t < ntg; t += gridDim.x) {
    const uint64_t off = offs[t];
    const uint32_t tn = (uint32_t)min((uint64_t)TG_ELEMS, n - t * TG_ELEMS);
    bool ok = off % 16 == 0 && off < total;
    if (ok) ok = decode_tg<DT>(st + off, (uint32_t)((total - off) < 0xffffffffull ? (total - off) : 0xffffffffull), tn,
                               out + t * (uint64_t)TG_ELEMS * ES, sm);
    if (!ok) {
      if (threadIdx.x == 0) atomicCAS(status, 0, (int)(2 + (t < (1u << 28) ? t : (1u << 28))));
      return;
    }
  }
}

template <int DT>
__global__ void __launch_bounds__(LZC_THREADS, LZC_MIN_BLOCKS) decode_slotted_kernel(const char* __restrict__ slots,
                                                                      uint32_t slot_cap,
                                                                      char* __restrict__ out,
                                                                      uint64_t n, int* status) {
  extern __shared__ __align__(16) char smem_raw[];
  DecSmem& sm = *reinterpret_cast<DecSmem*>(smem_raw);
  constexpr int ES = DT == DT_F32 ? 4 : (DT == DT_U8 ? 1 : 2);
  const uint64_t ntg = num_tgs(n);
  for (uint64_t t = blockIdx.x; t < ntg; t += gridDim.x) {
    const uint32_t tn = (uint32_t)min((uint64_t)TG_ELEMS, n - t * TG_ELEMS);
    if (!decode_tg<DT>(slots + t * (uint64_t)slot_cap, slot_cap, tn, out + t * (uint64_t)TG_ELEMS * ES, sm)) {
      if (threadIdx.x == 0) atomicCAS(status, 0, (int)(2 + (t < (1u << 28) ? t : (1u << 28))));
      return;
    }
  }
}

template <typename K>
int prep_smem(K kernel, size_t bytes) {
  static thread_local int done_dev[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  (void)done_dev;
  LZ_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
  return LZE_OK;
}

int grid_for(uint64_t ntg, int nblocks) {
  int sms = 148;
  int dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  long long g = nblocks > 0 ? nblocks : (long long)sms * 3;
  if ((uint64_t)g > ntg) g = (long long)ntg;
  return (int)(g < 1 ? 1 : g);
}

#define LZ_DT_DISPATCH(dt, FN, ...)                 \
  switch (dt) {                                     \
    case DT_BF16:                                   \
      return FN<DT_BF16>(__VA_ARGS__);              \
    case DT_F16:                                    \
      return FN<DT_F16>(__VA_ARGS__);               \
    case DT_F32:                                    \
      return FN<DT_F32>(__VA_ARGS__);               \
    case DT_U8:                                     \
      return FN<DT_U8>(__VA_ARGS__);                \
    case DT_E4M3P:                                  \
      return FN<DT_E4M3P>(__VA_ARGS__);             \
    case DT_E5M2P:                                  \
      return FN<DT_E5M2P>(__VA_ARGS__);             \
    default:                                        \
      lz_set_error("codec: unsupported dtype %d", dt); \
      return LZE_ARG;                               \
  }

template <int DT>
int launch_encode_slotted(const void* in, uint64_t n, void* slots, uint32_t* sizes, int level,
                          int nblocks, cudaStream_t s) {
  const uint64_t ntg = num_tgs(n);
  if (ntg == 0) return LZE_OK;
  if ((uintptr_t)in % 16 || (uintptr_t)slots % 16) {
    lz_set_error("codec: buffers must be 16-byte aligned");
    return LZE_ARG;
  }
  auto kernel = level == LEVEL_PACK ? encode_slotted_kernel<DT, LEVEL_PACK> : encode_slotted_kernel<DT, LEVEL_ANS>;
  int rc = prep_smem(kernel, sizeof(EncSmem));
  if (rc) return rc;
  static const int stop_after = getenv("LZ_CODEC_STOP_AFTER") ? atoi(getenv("LZ_CODEC_STOP_AFTER")) : 0;
  kernel<<<grid_for(ntg, nblocks), LZC_THREADS, sizeof(EncSmem), s>>>(
      static_cast<const char*>(in), n, static_cast<char*>(slots), tg_capacity(DT), sizes, stop_after);
  LZ_CUDA_TRY(cudaGetLastError());
  return LZE_OK;
}

template <int DT>
int launch_decode_slotted(const void* slots, void* out, uint64_t n, int* status, int nblocks,
                          cudaStream_t s) {
  const uint64_t ntg = num_tgs(n);
  if (ntg == 0) return LZE_OK;
  int rc = prep_smem(decode_slotted_kernel<DT>, sizeof(DecSmem));
  if (rc) return rc;
  decode_slotted_kernel<DT><<<grid_for(ntg, nblocks), LZC_THREADS, sizeof(DecSmem), s>>>(
      static_cast<const char*>(slots), tg_capacity(DT), static_cast<char*>(out), n, status);
  LZ_CUDA_TRY(cudaGetLastError());
  return LZE_OK;
}

template <int DT>
int launch_decode_stream(const void* st, uint64_t bytes, void* out, uint64_t n, int* status,
                         int nblocks, cudaStream_t s) {
  const uint64_t ntg = num_tgs(n);
  if (ntg == 0) return LZE_OK;
  int rc = prep_smem(decode_stream_kernel<DT>, sizeof(DecSmem));
  if (rc) return rc;
  decode_stream_kernel<DT><<<grid_for(ntg, nblocks), LZC_THREADS, sizeof(DecSmem), s>>>(
      static_cast<const char*>(st), bytes, static_cast<char*>(out), n, status);
  LZ_CUDA_TRY(cudaGetLastError());
  return LZE_OK;
}

}  // namespace

extern "C" {

size_t lz_codec_tg_elems(void) { return TG_ELEMS; }
// `dtype` arguments of the entry points below: the dtype code, optionally
// | level << CODEC_LEVEL_SHIFT (encoders; LEVEL_PACK = fast, lower ratio).
size_t lz_codec_tg_capacity(int dtype) { return tg_capacity(codec_dtype(dtype)); }
size_t lz_codec_max_bytes(size_t n, int dtype) { return max_stream_bytes(n, codec_dtype(dtype)); }

// Scratch of the compact encoder: slots + sizes + offsets (+ total).
size_t lz_codec_scratch_bytes(size_t n, int dtype) {
  dtype = codec_dtype(dtype);
  const uint64_t ntg = num_tgs(n);
  return ntg * tg_capacity(dtype) + pad16_64(4 * ntg) + pad16_64(8 * ntg) + 16;
}

int lz_codec_encode_slotted(const void* in, size_t n, int dtype, void* slots, uint32_t* d_sizes,
                            int nblocks, cudaStream_t s) {
  const int level = codec_level(dtype);
  if (!valid_level(level)) {
    lz_set_error("codec: unknown level %d", level);
    return LZE_ARG;
  }
  LZ_DT_DISPATCH(codec_dtype(dtype), launch_encode_slotted, in, n, slots, d_sizes, level, nblocks, s);
}

int lz_codec_decode_slotted(const void* slots, void* out, size_t n, int dtype, int* d_status,
                            int nblocks, cudaStream_t s) {
  LZ_DT_DISPATCH(codec_dtype(dtype), launch_decode_slotted, slots, out, n, d_status, nblocks, s);
}

// Compact stream: writes the total stream size to *d_total (device memory).
int lz_codec_encode(const void* in, size_t n, int dtype, void* scratch, size_t scratch_bytes,
                    void* out, size_t out_cap, unsigned long long* d_total, int nblocks,
                    cudaStream_t s) {
  const uint64_t ntg = num_tgs(n);
  const int dt = codec_dtype(dtype);
  if (scratch_bytes < lz_codec_scratch_bytes(n, dt) || out_cap < max_stream_bytes(n, dt)) {
    lz_set_error("codec: scratch (%zu) or output (%zu) too small", scratch_bytes, out_cap);
    return LZE_ARG;
  }
  if ((uintptr_t)out % 16 || (uintptr_t)scratch % 16) {
    lz_set_error("codec: buffers must be 16-byte aligned");
    return LZE_ARG;
  }
  char* slots = static_cast<char*>(scratch);
  uint32_t* sizes = reinterpret_cast<uint32_t*>(slots + ntg * tg_capacity(dt));
  uint64_t* offsets = reinterpret_cast<uint64_t*>(reinterpret_cast<char*>(sizes) + pad16_64(4 * ntg));
  int rc = lz_codec_encode_slotted(in, n, dtype, slots, sizes, nblocks, s);
  if (rc) return rc;
  const uint64_t base = sizeof(StreamHeader) + pad16_64(8 * ntg);
  scan_sizes_kernel<<<1, 1024, 0, s>>>(sizes, ntg, offsets, base, d_total);
  LZ_CUDA_TRY(cudaGetLastError());
  gather_records_kernel<<<grid_for(ntg ? ntg : 1, nblocks), 256, 0, s>>>(
      slots, tg_capacity(dt), sizes, offsets, ntg, static_cast<char*>(out), n, dt, d_total);
  LZ_CUDA_TRY(cudaGetLastError());
  return LZE_OK;
}

int lz_codec_decode(const void* stream, size_t stream_bytes, void* out, size_t n, int dtype,
                    int* d_status, int nblocks, cudaStream_t s) {
  if ((uintptr_t)stream % 16 || (uintptr_t)out % 16) {
    lz_set_error("codec: buffers must be 16-byte aligned");
    return LZE_ARG;
  }
  LZ_DT_DISPATCH(codec_dtype(dtype), launch_decode_stream, stream, stream_bytes, out, n, d_status, nblocks, s);
}

}  // extern "C"
