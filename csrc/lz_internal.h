// Host-side internals shared by the native translation units.
#pragma once
#include <stdarg.h>
#include <stdio.h>

#include "lz_api.h"
#include "lz_types.h"
#include "lz_driver.h"

void lz_set_error(const char* fmt, ...);
int lz_heap_device(LzHeap* h);
int lz_heap_rank(LzHeap* h);
int lz_heap_world(LzHeap* h);

#define LZ_CUDA_TRY(call)                                                              \
  do {                                                                                 \
    cudaError_t e__ = (call);                                                          \
    if (e__ != cudaSuccess) {                                                          \
      lz_set_error("%s failed: %s (%s:%d)", #call, cudaGetErrorString(e__), __FILE__, \
                   __LINE__);                                                          \
      return LZE_CUDA;                                                                 \
    }                                                                                  \
  } while (0)

// Communicator: device-visible state plus the heap layout.
//
// Flag area at the start of every rank's heap (kLzFlagsBytes, zeroed at
// creation; every protocol writes monotonic values, so nothing is reset):
//   [0, 32K)        block barriers [LZ_MAX_BLOCKS][LZ_MAX_RANKS]      lz_common.cuh
//   [32K, 40K)      ring ready / credit [LZ_MAX_BLOCKS]               lz_allreduce.cu
//   [64K, 128K)     weight-transfer ready flags, p2p / broadcast        lz_weights.cu
//   [128K, 192K)    weight-transfer credits, p2p / broadcast            lz_weights.cu
//   [192K, 448K)    relay-broadcast barriers, one 32K region per sender lz_weights.cu
//   [448K, 480K)    relay-broadcast chunk-ready flags, 4K per sender    lz_weights.cu
//   [480K, 480K+128) copy-engine ready / clear-to-send                  lz_weights.cu
//   [512K]          failure-test flag that nothing sets                 lz_allreduce.cu
//   [544K, 562K)    copy-engine two-shot: started / done / chunk flags   lz_copy_engine.cu
//   [576K, 608K)    compressed allreduce chunk progress [block][rank]   lz_compressed.cu
// (static_asserts next to each region keep neighbours from overlapping.)
static constexpr size_t kLzFlagsBytes = 1 << 20;
static constexpr size_t kLzLlMaxBytes = 256u << 10;  // largest low-latency one-shot message

struct LzComm {
  LzHeap* heap;           // nullptr for emulated ranks
  size_t heap_bytes;
  int device;
  LzDevComm dev;          // copied by value into every launch
  size_t oneshot_off;     // two stages of oneshot_bytes each (double buffered)
  size_t oneshot_bytes;
  size_t ll_off;          // low-latency one-shot receive areas (two parities)
  size_t ll_bytes;        // bytes per parity: world x 2 x kLzLlMaxBytes
  size_t stage_off;       // general staging region
  size_t stage_bytes;
  size_t user_off;        // start of the user-allocatable region
  int sm_count;
  int* status_host;       // host view of dev.status
  // copy-engine allreduce (lz_copy_engine.cu): call counter and finished-block
  // counter in device memory, plus side streams and events created on first use
  unsigned long long* ce_seq;
  unsigned int* ce_done;
  cudaStream_t ce_stream[3];
  cudaEvent_t* ce_events;
  int ce_nevents;
};

// Releases the copy-engine streams and events of a communicator (if created).
void lz_ce_release(LzComm* c);

// Returns the heap offset of [p, p+bytes) when it lies in this rank's heap, or
// (size_t)-1.
size_t lz_comm_heap_offset(const LzComm* c, const void* p, size_t bytes);

// Single-GPU emulation internals shared between translation units.
typedef struct LzEmu LzEmu;
LzComm* lz_emu_comm(LzEmu* e, int r);
LzDevComm* lz_emu_dev_comms(LzEmu* e);
int lz_emu_world(LzEmu* e);
void* lz_emu_param_buffer(LzEmu* e);  // 4 KB device buffer for per-rank params
