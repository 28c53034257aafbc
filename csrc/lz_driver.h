// Driver-API entry points resolved at runtime through the CUDA runtime
// (cudaGetDriverEntryPointByVersion), so the library has no link-time
// dependency on libcuda and can be loaded on a machine without a GPU.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#define LZ_DRIVER_FNS(X)                  \
  X(cuGetErrorString)                     \
  X(cuDeviceGet)                          \
  X(cuDeviceGetAttribute)                 \
  X(cuCtxGetCurrent)                      \
  X(cuMemGetAllocationGranularity)        \
  X(cuMemCreate)                          \
  X(cuMemRelease)                         \
  X(cuMemExportToShareableHandle)         \
  X(cuMemImportFromShareableHandle)       \
  X(cuMemAddressReserve)                  \
  X(cuMemAddressFree)                     \
  X(cuMemMap)                             \
  X(cuMemUnmap)                           \
  X(cuMemSetAccess)                       \
  X(cuMulticastCreate)                    \
  X(cuMulticastAddDevice)                 \
  X(cuMulticastBindMem)                   \
  X(cuMulticastUnbind)                    \
  X(cuMulticastGetGranularity)            \
  X(cuDeviceGetDevResource)               \
  X(cuDevSmResourceSplitByCount)          \
  X(cuDevResourceGenerateDesc)            \
  X(cuGreenCtxCreate)                     \
  X(cuGreenCtxDestroy)                    \
  X(cuGreenCtxStreamCreate)               \
  X(cuStreamDestroy)

struct LzDriver {
#define LZ_DECL(name) decltype(&::name) name = nullptr;
  LZ_DRIVER_FNS(LZ_DECL)
#undef LZ_DECL
  bool loaded = false;
  bool ok = false;
};

// Returns the resolved table; `ok` is false when no driver is present.
LzDriver& lz_driver();

// Formats the last driver error into a thread-local message buffer.
const char* lz_cu_errstr(CUresult r);
