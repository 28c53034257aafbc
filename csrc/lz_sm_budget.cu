// SM budgets. A green context owns a fixed subset of the GPU's SMs; kernels
// launched on its stream run only there, so the collective/codec kernels can
// be limited to 16/32/64/96/128 of the 148 SMs while the rest compute
// (reference: back_up/green_context_example.cu:15-79, SM counts in multiples of
// 8 on sm_90; the UCCL engine's "[GreenContext] Created: 16/132 SMs" logs).
// The %smid probe records which SM every block ran on, to check a budget.
#include "lz_common.cuh"
#include "lz_internal.h"

struct LzSmBudget {
  CUgreenCtx gctx;
  CUstream stream;
  int sm_count;
};

namespace {
__global__ void smid_probe_kernel(int* out, int nblocks) {
  if (threadIdx.x == 0 && blockIdx.x < (unsigned)nblocks) {
    unsigned smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    out[blockIdx.x] = (int)smid;
    // keep the block resident for a moment so blocks spread over the partition
    const unsigned long long t0 = globaltimer();
    while (globaltimer() - t0 < 20000ull) {
    }
  }
}
}  // namespace

// Creates a green context with at least `sm_count` SMs (rounded up to the
// hardware's split granularity) on `device` and a non-blocking stream in it.
extern "C" int lz_sm_budget_create(int device, int sm_count, LzSmBudget** out, void** stream,
                                   int* granted) {
  LzDriver& d = lz_driver();
  if (!d.ok || !d.cuGreenCtxCreate || !d.cuDevSmResourceSplitByCount) {
    lz_set_error("green contexts unavailable in this driver");
    return LZE_UNSUPPORTED;
  }
  LZ_CUDA_TRY(cudaSetDevice(device));
  cudaFree(0);
  CUdevice dev;
  CUresult r = d.cuDeviceGet(&dev, device);
  if (r != CUDA_SUCCESS) {
    lz_set_error("cuDeviceGet: %s", lz_cu_errstr(r));
    return LZE_DRIVER;
  }
  CUdevResource all;
  memset(&all, 0, sizeof(all));
  r = d.cuDeviceGetDevResource(dev, &all, CU_DEV_RESOURCE_TYPE_SM);
  if (r != CUDA_SUCCESS) {
    lz_set_error("cuDeviceGetDevResource: %s", lz_cu_errstr(r));
    return LZE_DRIVER;
  }
  CUdevResource part[1], rest;
  unsigned int nb = 1;
  memset(part, 0, sizeof(part));
  memset(&rest, 0, sizeof(rest));
  r = d.cuDevSmResourceSplitByCount(part, &nb, &all, &rest, 0, (unsigned)sm_count);
  if (r != CUDA_SUCCESS || nb < 1) {
    lz_set_error("cuDevSmResourceSplitByCount(%d): %s", sm_count, lz_cu_errstr(r));
    return LZE_DRIVER;
  }
  CUdevResourceDesc desc;
  r = d.cuDevResourceGenerateDesc(&desc, part, 1);
  if (r != CUDA_SUCCESS) {
    lz_set_error("cuDevResourceGenerateDesc: %s", lz_cu_errstr(r));
    return LZE_DRIVER;
  }
  LzSmBudget* b = new LzSmBudget();
  r = d.cuGreenCtxCreate(&b->gctx, desc, dev, CU_GREEN_CTX_DEFAULT_STREAM);
  if (r != CUDA_SUCCESS) {
    delete b;
    lz_set_error("cuGreenCtxCreate: %s", lz_cu_errstr(r));
    return LZE_DRIVER;
  }
  r = d.cuGreenCtxStreamCreate(&b->stream, b->gctx, CU_STREAM_NON_BLOCKING, 0);
  if (r != CUDA_SUCCESS) {
    d.cuGreenCtxDestroy(b->gctx);
    delete b;
    lz_set_error("cuGreenCtxStreamCreate: %s", lz_cu_errstr(r));
    return LZE_DRIVER;
  }
  b->sm_count = (int)part[0].sm.smCount;
  *out = b;
  *stream = (void*)b->stream;
  *granted = b->sm_count;
  return LZE_OK;
}

extern "C" int lz_sm_budget_destroy(LzSmBudget* b) {
  if (!b) return LZE_OK;
  LzDriver& d = lz_driver();
  cudaStreamSynchronize((cudaStream_t)b->stream);
  d.cuStreamDestroy(b->stream);
  d.cuGreenCtxDestroy(b->gctx);
  delete b;
  return LZE_OK;
}

// Launches `nblocks` blocks on `stream` and records each block's SM id.
extern "C" int lz_smid_probe(void* stream, int* d_out, int nblocks) {
  smid_probe_kernel<<<nblocks, 32, 0, (cudaStream_t)stream>>>(d_out, nblocks);
  LZ_CUDA_TRY(cudaGetLastError());
  return LZE_OK;
}
