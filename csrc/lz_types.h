// Types and constants shared by host and device code.
#pragma once
#include <stddef.h>
#include <stdint.h>

#define LZ_MAX_RANKS 8
#define LZ_MAX_BLOCKS 512

// Status word codes (host mirror in lz_api.h).
#define LZ_OK 0
#define LZ_ERR_TIMEOUT 1
#define LZ_ERR_ABORTED 2
#define LZ_ERR_BOUNDS 3
#define LZ_ERR_CORRUPT 4

enum LzDtype : int { LZ_F32 = 0, LZ_F16 = 1, LZ_BF16 = 2, LZ_U8 = 3 };

// Everything a collective kernel needs to reach its peers. Passed by value so
// launches are CUDA-graph replayable (no per-call host arguments besides
// buffer pointers and sizes).
struct LzDevComm {
  int rank;
  int world;
  char* heap[LZ_MAX_RANKS];       // base of every rank's symmetric heap, mapped here
  char* heap_mc;                  // multicast (NVLS) mapping of the heap, or nullptr
  unsigned long long* flags;      // local flag array [LZ_MAX_BLOCKS][LZ_MAX_RANKS]
  size_t flags_off;               // byte offset of the flag array inside the heap
  unsigned long long* epoch;      // local call counter (incremented by the last block)
  unsigned int* done;             // blocks-finished counter for the epoch bump
  int* abort_flag;                // local: set when any block gave up waiting
  int* status;                    // host-mapped: first error (code | where)
  unsigned long long timeout_ns;  // bound of every flag wait
  int fence_all;                  // 1: every thread fences its peer stores before a signal
  size_t heap_bytes;              // bytes of every rank's heap (bounds checks)
  int poll_relaxed;               // 1: flag polls are relaxed loads + one fence (default: ld.acquire)
};

