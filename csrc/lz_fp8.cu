// fp8 pair packing kernels: two fp8 values -> one 16-bit container whose
// bits 14..7 (the bf16 exponent byte) carry exponent bits of both values, so
// the bf16 split codec compresses fp8 data with one symbol per pair.
// e4m3 uses the reference's container layout
// (back_up/fp8_e4m3fn_pack_benchmark.cu:21-93: grid-stride byte loads, one pair
// per thread); these kernels move 16 bytes per load/store and are also fused
// into the codec's split/merge (DT_E4M3P / DT_E5M2P table groups).
#include "lz_codec_format.h"
#include "lz_common.cuh"
#include "lz_internal.h"

using namespace lzc;

namespace {

template <bool kE4M3>
__global__ void __launch_bounds__(256) pack_kernel(const uint8_t* __restrict__ in,
                                                   uint16_t* __restrict__ out, size_t npairs) {
  const size_t nvec = npairs / 8;  // 16 input bytes -> 8 containers (16 output bytes)
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t v = (size_t)blockIdx.x * blockDim.x + threadIdx.x; v < nvec; v += stride) {
    const uint4 x = ld_nc_v4(in + 16 * v);
    const uint8_t* b = reinterpret_cast<const uint8_t*>(&x);
    uint4 y;
    uint16_t* w = reinterpret_cast<uint16_t*>(&y);
#pragma unroll
    for (int k = 0; k < 8; ++k) w[k] = kE4M3 ? pack_e4m3(b[2 * k], b[2 * k + 1]) : pack_e5m2(b[2 * k], b[2 * k + 1]);
    st_cs_v4(out + 8 * v, y);
  }
  if (blockIdx.x == 0 && threadIdx.x < npairs - nvec * 8) {
    const size_t i = nvec * 8 + threadIdx.x;
    out[i] = kE4M3 ? pack_e4m3(in[2 * i], in[2 * i + 1]) : pack_e5m2(in[2 * i], in[2 * i + 1]);
  }
}

template <bool kE4M3>
__global__ void __launch_bounds__(256) unpack_kernel(const uint16_t* __restrict__ in,
                                                     uint8_t* __restrict__ out, size_t npairs) {
  const size_t nvec = npairs / 8;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t v = (size_t)blockIdx.x * blockDim.x + threadIdx.x; v < nvec; v += stride) {
    const uint4 x = ld_nc_v4(in + 8 * v);
    const uint16_t* w = reinterpret_cast<const uint16_t*>(&x);
    uint4 y;
    uint8_t* b = reinterpret_cast<uint8_t*>(&y);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if (kE4M3) unpack_e4m3(w[k], &b[2 * k], &b[2 * k + 1]);
      else unpack_e5m2(w[k], &b[2 * k], &b[2 * k + 1]);
    }
    st_cs_v4(out + 16 * v, y);
  }
  if (blockIdx.x == 0 && threadIdx.x < npairs - nvec * 8) {
    const size_t i = nvec * 8 + threadIdx.x;
    if (kE4M3) unpack_e4m3(in[i], &out[2 * i], &out[2 * i + 1]);
    else unpack_e5m2(in[i], &out[2 * i], &out[2 * i + 1]);
  }
}

int grid_for(size_t nvec) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  size_t g = (nvec + 255) / 256;
  const size_t cap = (size_t)sms * 8;  // grid-stride beyond 8 CTAs per SM
  if (g > cap) g = cap;
  return (int)(g < 1 ? 1 : g);
}

}  // namespace

// kind: 0 = e4m3 (reference container), 1 = e5m2 container.
extern "C" int lz_fp8_pack(const void* in, void* out, size_t npairs, int kind, cudaStream_t s) {
  if ((uintptr_t)in % 16 || (uintptr_t)out % 16) {
    lz_set_error("fp8 pack: 16-byte aligned buffers required");
    return LZE_ARG;
  }
  const int g = grid_for(npairs / 8);
  if (kind == 0)
    pack_kernel<true><<<g, 256, 0, s>>>(static_cast<const uint8_t*>(in), static_cast<uint16_t*>(out), npairs);
  else
    pack_kernel<false><<<g, 256, 0, s>>>(static_cast<const uint8_t*>(in), static_cast<uint16_t*>(out), npairs);
  LZ_CUDA_TRY(cudaGetLastError());
  return LZE_OK;
}

extern "C" int lz_fp8_unpack(const void* in, void* out, size_t npairs, int kind, cudaStream_t s) {
  if ((uintptr_t)in % 16 || (uintptr_t)out % 16) {
    lz_set_error("fp8 unpack: 16-byte aligned buffers required");
    return LZE_ARG;
  }
  const int g = grid_for(npairs / 8);
  if (kind == 0)
    unpack_kernel<true><<<g, 256, 0, s>>>(static_cast<const uint16_t*>(in), static_cast<uint8_t*>(out), npairs);
  else
    unpack_kernel<false><<<g, 256, 0, s>>>(static_cast<const uint16_t*>(in), static_cast<uint8_t*>(out), npairs);
  LZ_CUDA_TRY(cudaGetLastError());
  return LZE_OK;
}
