// Copy-engine two-shot allreduce: the peer reads of both phases are done by
// the DMA copy engines (cudaMemcpyAsync from peer-mapped heap addresses), so
// the only SM work is the local fp32 accumulation; a non-SM alternative for
// when SMs are budgeted to compute. Phases are separated by the device-side
// barrier kernel (bounded waits). Work is cut into `pipes` pieces on two
// streams so copies of piece k+1 overlap the accumulation of piece k.
//
// Reference behaviour being re-designed:
// single_node_nccl_allreduce_benchmark/memcpy_p2p_allreduce_kernel.cu:176-346 (D2D
// and host-staged pipelines, bf16 __hadd2 accumulation rounding at every
// step); here accumulation is fp32 in rank order, rounded once.
#include "lz_common.cuh"
#include "lz_internal.h"

namespace {

template <int DT>
__global__ void __launch_bounds__(256) accum_kernel(const char* __restrict__ own,
                                                    const char* __restrict__ tmp, size_t tmp_stride,
                                                    int world, int me, char* __restrict__ out,
                                                    char* __restrict__ out2, size_t nvec) {
  using V = Vec<DT>;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += stride) {
    float acc[V::N];
    bool first = true;
    for (int r = 0; r < world; ++r) {
      const uint4 v = (r == me) ? reinterpret_cast<const uint4*>(own)[i]
                                : reinterpret_cast<const uint4*>(tmp + (size_t)r * tmp_stride)[i];
      if (first) V::load(acc, v);
      else V::add(acc, v);
      first = false;
    }
    const uint4 res = V::pack(acc);
    reinterpret_cast<uint4*>(out)[i] = res;
    reinterpret_cast<uint4*>(out2)[i] = res;
  }
}

}  // namespace

extern "C" int lz_barrier(LzComm* c, cudaStream_t s);

// in/out: any device buffers of count elements. Uses the communicator stage:
// [W slots of my input slices for peers | my result slice | W temp slices].
extern "C" int lz_ce_allreduce(LzComm* c, const void* in, void* out, size_t count, int dtype,
                               int pipes, cudaStream_t s, cudaStream_t s2) {
  const int W = c->dev.world, me = c->dev.rank;
  const size_t es = dtype == LZ_F32 ? 4 : 2;
  const size_t bytes = count * es;
  if (bytes % (16 * (size_t)W)) {
    lz_set_error("copy-engine allreduce: size must be a multiple of 16 * world bytes");
    return LZE_ARG;
  }
  if (W == 1) {
    if (in != out) LZ_CUDA_TRY(cudaMemcpyAsync(out, in, bytes, cudaMemcpyDeviceToDevice, s));
    return LZE_OK;
  }
  const size_t slice = bytes / W;
  const size_t need = bytes + slice + (size_t)W * slice;
  if (need > c->stage_bytes) {
    lz_set_error("copy-engine allreduce: stage needs %zu bytes, have %zu", need, c->stage_bytes);
    return LZE_ARG;
  }
  if (pipes < 1) pipes = 1;
  while (pipes > 1 && (slice / pipes) % 16) --pipes;
  char* my = c->dev.heap[me];
  const size_t in_off = c->stage_off;                // full copy of my input
  const size_t res_off = in_off + bytes;             // my reduced slice
  const size_t tmp_off = res_off + slice;            // W temp slices (peer copies)
  LZ_CUDA_TRY(cudaMemcpyAsync(my + in_off, in, bytes, cudaMemcpyDeviceToDevice, s));
  int rc = lz_barrier(c, s);
  if (rc) return rc;
  cudaEvent_t ev[64];
  const int np = pipes > 64 ? 64 : pipes;
  const size_t piece = slice / np;
  for (int k = 0; k < np; ++k) LZ_CUDA_TRY(cudaEventCreateWithFlags(&ev[k], cudaEventDisableTiming));
  cudaEvent_t start;
  LZ_CUDA_TRY(cudaEventCreateWithFlags(&start, cudaEventDisableTiming));
  LZ_CUDA_TRY(cudaEventRecord(start, s));
  LZ_CUDA_TRY(cudaStreamWaitEvent(s2, start, 0));
  // RS: copy engines fetch my slice from every peer (pipelined), SMs accumulate
  for (int k = 0; k < np; ++k) {
    const size_t off = (size_t)me * slice + (size_t)k * piece;
    const size_t len = (k == np - 1) ? slice - (size_t)k * piece : piece;
    for (int j = 1; j < W; ++j) {
      const int p = (me + j) % W;
      LZ_CUDA_TRY(cudaMemcpyAsync(my + tmp_off + (size_t)p * slice + (size_t)k * piece,
                                  c->dev.heap[p] + in_off + off, len, cudaMemcpyDeviceToDevice, s2));
    }
    LZ_CUDA_TRY(cudaEventRecord(ev[k], s2));
    LZ_CUDA_TRY(cudaStreamWaitEvent(s, ev[k], 0));
    const size_t nvec = len / 16;
    const int G = (int)((nvec + 255) / 256 < 1184 ? (nvec + 255) / 256 : 1184);
    const char* own = static_cast<const char*>(in) + off;
    char* o1 = static_cast<char*>(out) + off;
    char* o2 = my + res_off + (size_t)k * piece;
    const char* tmp = my + tmp_off + (size_t)k * piece;
    switch (dtype) {
      case LZ_F32:
        accum_kernel<LZ_F32><<<G > 0 ? G : 1, 256, 0, s>>>(own, tmp, slice, W, me, o1, o2, nvec);
        break;
      case LZ_F16:
        accum_kernel<LZ_F16><<<G > 0 ? G : 1, 256, 0, s>>>(own, tmp, slice, W, me, o1, o2, nvec);
        break;
      default:
        accum_kernel<LZ_BF16><<<G > 0 ? G : 1, 256, 0, s>>>(own, tmp, slice, W, me, o1, o2, nvec);
    }
    LZ_CUDA_TRY(cudaGetLastError());
  }
  rc = lz_barrier(c, s);
  if (rc) return rc;
  // AG: copy engines fetch every peer's reduced slice into my output
  LZ_CUDA_TRY(cudaEventRecord(start, s));
  LZ_CUDA_TRY(cudaStreamWaitEvent(s2, start, 0));
  for (int j = 1; j < W; ++j) {
    const int p = (me + j) % W;
    LZ_CUDA_TRY(cudaMemcpyAsync(static_cast<char*>(out) + (size_t)p * slice, c->dev.heap[p] + res_off, slice,
                                cudaMemcpyDeviceToDevice, s2));
  }
  LZ_CUDA_TRY(cudaEventRecord(ev[0], s2));
  LZ_CUDA_TRY(cudaStreamWaitEvent(s, ev[0], 0));
  // nobody may overwrite a result slice before every peer has copied it
  rc = lz_barrier(c, s);
  for (int k = 0; k < np; ++k) cudaEventDestroy(ev[k]);
  cudaEventDestroy(start);
  return rc;
}
