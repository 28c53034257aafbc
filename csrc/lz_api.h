// C ABI of the native runtime (loaded from Python with ctypes).
// Every function returns 0 on success or a negative error code; the last
// error message of the calling thread is available through lz_last_error().
#pragma once
#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct LzHeap LzHeap;
typedef struct LzComm LzComm;

// Error codes returned by the C ABI.
#define LZE_OK 0
#define LZE_CUDA -1
#define LZE_DRIVER -2
#define LZE_ARG -3
#define LZE_SOCKET -4
#define LZE_UNSUPPORTED -5
#define LZE_STATE -6
#define LZE_TIMEOUT -7

const char* lz_last_error(void);
int lz_version(void);

// ---- topology / device probes -------------------------------------------
int lz_device_info(int device, int* sm_count, int* multicast_supported, int* cc_major,
                   int* cc_minor, size_t* total_mem);
int lz_can_access_peer(int device, int peer, int* can);
int lz_nvlink_p2p_attr(int device, int peer, int* perf_rank, int* native_atomics);

// ---- symmetric heap (cuMem VMM, POSIX fd exchange, NVLS multicast) --------
// Phase 1: allocate and export (local only).
int lz_heap_create(int device, int rank, int world, size_t bytes, int want_multicast,
                   const char* tag, LzHeap** out);
// Phase 2: serve this rank's fds to peers (background thread).
int lz_heap_serve(LzHeap* h);
// Phase 3 (after a barrier): fetch every peer's fd and map its memory.
int lz_heap_connect(LzHeap* h);
// Multicast steps, each separated by a barrier on the host:
//   rank 0: lz_mc_create -> barrier -> all: lz_mc_attach (others fetch fd, add device)
//   -> barrier -> all: lz_mc_bind -> barrier -> all: lz_mc_map
int lz_mc_create(LzHeap* h);
int lz_mc_attach(LzHeap* h);
int lz_mc_bind(LzHeap* h);
int lz_mc_map(LzHeap* h);
int lz_heap_stop_serving(LzHeap* h);
int lz_heap_destroy(LzHeap* h);
size_t lz_heap_size(LzHeap* h);
void* lz_heap_ptr(LzHeap* h, int rank);  // device VA of `rank`'s heap here
void* lz_heap_mc_ptr(LzHeap* h);         // multicast VA or NULL
int lz_heap_has_mc(LzHeap* h);

// ---- communicator ------------------------------------------------------------
// Layout inside the heap: [flags | oneshot stage x2 | general stage | user region].
int lz_comm_create(LzHeap* h, size_t oneshot_bytes, size_t stage_bytes, double timeout_s,
                   LzComm** out);
int lz_comm_destroy(LzComm* c);
size_t lz_comm_user_offset(LzComm* c);  // first byte of the user region
int lz_comm_status(LzComm* c);          // host-mapped status word (0 = ok)
int lz_comm_clear_status(LzComm* c);
int lz_comm_epoch(LzComm* c, unsigned long long* epoch, cudaStream_t s);

// Algorithms of lz_allreduce.
#define LZ_ALGO_ONESHOT 0
#define LZ_ALGO_TWOSHOT 1
#define LZ_ALGO_NVLS 2
#define LZ_ALGO_RING 3
#define LZ_ALGO_RHD 4
#define LZ_ALGO_NVLS_ONESHOT 5
#define LZ_ALGO_LL 6  /* low-latency one-shot (flag-in-data words), <= 256 KB */

// Sum-allreduce of `count` elements. `in`/`out` may alias; when they lie in
// the heap's user region the zero-copy symmetric path is used.
int lz_allreduce(LzComm* c, const void* in, void* out, size_t count, int dtype, int algo,
                 int nblocks, int nthreads, cudaStream_t stream);

// Device-side barrier (all ranks, one block).
int lz_barrier(LzComm* c, cudaStream_t stream);

// ---- single-GPU emulation of R ranks (tests) ---------------------------------
typedef struct LzEmu LzEmu;
int lz_emu_create(int R, size_t heap_bytes, size_t oneshot_bytes, size_t stage_bytes,
                  double timeout_s, LzEmu** out);
int lz_emu_destroy(LzEmu* e);
void* lz_emu_heap_ptr(LzEmu* e, int r);
size_t lz_emu_user_offset(LzEmu* e);
int lz_emu_status(LzEmu* e, int r);
int lz_emu_allreduce(LzEmu* e, const void* const* ins, void* const* outs, size_t count, int dtype,
                     int algo, int nblocks, int nthreads, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
