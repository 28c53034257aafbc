// Shared device-side primitives for every sm_100a kernel of the library.
//
// Memory-model discipline (replaces the unbounded atomicExch/atomicAdd spin
// flags of single_node_nccl_allreduce_benchmark/cuda_p2p_allreduce_kernel.cu:184-192):
//   * signals are monotonic 64-bit values ((epoch+1) << 3 | phase) stored with
//     st.release.sys, so a flag never needs a reset;
//   * waits are ld.acquire.sys loops bounded by %globaltimer and by an
//     iteration cap; on expiry the kernel records an error in a host-mapped
//     status word, raises the communicator's abort flag and returns.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "lz_types.h"
#define LZ_DEV __device__ __forceinline__

// ----------------------------------------------------------------------------
// Raw PTX wrappers
// ----------------------------------------------------------------------------
LZ_DEV unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

LZ_DEV unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

LZ_DEV void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

LZ_DEV unsigned long long ld_relaxed_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

LZ_DEV void st_relaxed_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

LZ_DEV int ld_volatile_i32(const int* p) {
  int v;
  asm volatile("ld.volatile.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

LZ_DEV void fence_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
LZ_DEV void fence_proxy_alias() { asm volatile("fence.proxy.alias;" ::: "memory"); }

// ----------------------------------------------------------------------------
// Bulk asynchronous copy global -> this CTA's shared memory (the TMA engine,
// no multicast) completing on an mbarrier. Addresses and size must be
// multiples of 16 bytes; callers check and fall back to vector loads.
// ----------------------------------------------------------------------------
LZ_DEV uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

LZ_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
LZ_DEV void mbar_inval(uint64_t* bar) {
  asm volatile("mbarrier.inval.shared::cta.b64 [%0];" ::"r"(smem_addr(bar)) : "memory");
}
// Generic-proxy shared-memory writes made so far are ordered before later
// async-proxy (bulk copy) accesses of the same memory.
LZ_DEV void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
LZ_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

// One thread: announce `bytes` of transaction on `bar` and start the copy.
LZ_DEV void bulk_g2s(void* dst_smem, const void* src_global, uint32_t bytes, uint64_t* bar) {
  uint64_t state;
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 %0, [%1], %2;"
               : "=l"(state)
               : "r"(smem_addr(bar)), "r"(bytes)
               : "memory");
  (void)state;
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst_smem)),
      "l"(src_global), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// Bounded wait for phase `parity` of `bar`; false after max_iters polls.
LZ_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t max_iters) {
  for (uint32_t it = 0; it < max_iters; ++it) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}

// 16-byte global loads/stores. `cg` bypasses L1 for data another GPU wrote.
// These are compiler intrinsics, not volatile asm, so loads of later loop
// iterations can be scheduled early; ordering against flag waits is kept
// because those are volatile asm with memory clobbers.
LZ_DEV uint4 ld_cg_v4(const void* p) { return __ldcg(reinterpret_cast<const uint4*>(p)); }
LZ_DEV uint4 ld_nc_v4(const void* p) {  // read-only for the kernel's lifetime, streamed
  return __ldcs(reinterpret_cast<const uint4*>(p));
}
LZ_DEV uint8_t ld_cg_u8(const void* p) {
  return (uint8_t)__ldcg(reinterpret_cast<const unsigned char*>(p));
}
LZ_DEV uint32_t ld_cg_u32(const void* p) { return __ldcg(reinterpret_cast<const unsigned int*>(p)); }
LZ_DEV void st_v4(void* p, uint4 v) { *reinterpret_cast<uint4*>(p) = v; }
LZ_DEV void st_cs_v4(void* p, uint4 v) {  // streaming store (evict-first)
  __stcs(reinterpret_cast<uint4*>(p), v);
}

// ----------------------------------------------------------------------------
// NVLS multimem (NVSwitch in-fabric reduce / broadcast). Only ever used on the
// multicast mapping of the symmetric heap.
// ----------------------------------------------------------------------------
template <int DT>
LZ_DEV uint4 multimem_ld_reduce_v4(const void* mc);

template <>
LZ_DEV uint4 multimem_ld_reduce_v4<LZ_BF16>(const void* mc) {
  uint4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(mc)
               : "memory");
  return v;
}
template <>
LZ_DEV uint4 multimem_ld_reduce_v4<LZ_F16>(const void* mc) {
  uint4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.f16x2 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(mc)
               : "memory");
  return v;
}
template <>
LZ_DEV uint4 multimem_ld_reduce_v4<LZ_F32>(const void* mc) {
  uint4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(mc)
               : "memory");
  return v;
}

// bf16 reduction accumulated in bf16 by the switch (no .acc::f32): lower
// precision, offered only as an explicit option.
LZ_DEV uint4 multimem_ld_reduce_bf16_noacc(const void* mc) {
  uint4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.bf16x2 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(mc)
               : "memory");
  return v;
}

LZ_DEV void multimem_st_v4(void* mc, uint4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(mc),
               "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

LZ_DEV void multimem_st_release_u64(unsigned long long* mc, unsigned long long v) {
  asm volatile("multimem.st.release.sys.global.u64 [%0], %1;" ::"l"(mc), "l"(v) : "memory");
}

// ----------------------------------------------------------------------------
// Element conversion helpers: 16 bytes <-> 8 (or 4) fp32 accumulators.
// ----------------------------------------------------------------------------
template <int DT>
struct Vec;  // elements per 16-byte vector

template <>
struct Vec<LZ_BF16> {
  static constexpr int N = 8;
  LZ_DEV static void add(float* acc, uint4 v) {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f = __bfloat1622float2(h[i]);
      acc[2 * i] += f.x;
      acc[2 * i + 1] += f.y;
    }
  }
  LZ_DEV static void load(float* acc, uint4 v) {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f = __bfloat1622float2(h[i]);
      acc[2 * i] = f.x;
      acc[2 * i + 1] = f.y;
    }
  }
  LZ_DEV static uint4 pack(const float* acc) {
    uint4 v;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
    return v;
  }
};

template <>
struct Vec<LZ_F16> {
  static constexpr int N = 8;
  LZ_DEV static void add(float* acc, uint4 v) {
    const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f = __half22float2(h[i]);
      acc[2 * i] += f.x;
      acc[2 * i + 1] += f.y;
    }
  }
  LZ_DEV static void load(float* acc, uint4 v) {
    const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f = __half22float2(h[i]);
      acc[2 * i] = f.x;
      acc[2 * i + 1] = f.y;
    }
  }
  LZ_DEV static uint4 pack(const float* acc) {
    uint4 v;
    __half2* h = reinterpret_cast<__half2*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(acc[2 * i], acc[2 * i + 1]);
    return v;
  }
};

template <>
struct Vec<LZ_F32> {
  static constexpr int N = 4;
  LZ_DEV static void add(float* acc, uint4 v) {
    acc[0] += __uint_as_float(v.x);
    acc[1] += __uint_as_float(v.y);
    acc[2] += __uint_as_float(v.z);
    acc[3] += __uint_as_float(v.w);
  }
  LZ_DEV static void load(float* acc, uint4 v) {
    acc[0] = __uint_as_float(v.x);
    acc[1] = __uint_as_float(v.y);
    acc[2] = __uint_as_float(v.z);
    acc[3] = __uint_as_float(v.w);
  }
  LZ_DEV static uint4 pack(const float* acc) {
    return make_uint4(__float_as_uint(acc[0]), __float_as_uint(acc[1]), __float_as_uint(acc[2]),
                      __float_as_uint(acc[3]));
  }
};

// ----------------------------------------------------------------------------
// Error reporting and bounded waits.
// ----------------------------------------------------------------------------
// Status layout: bits 0..7 code, 8..15 phase, 16..23 peer, 24..31 block.
LZ_DEV void lz_report(const LzDevComm& c, int code, int phase, int peer) {
  int word = (code & 0xff) | ((phase & 0xff) << 8) | ((peer & 0xff) << 16) |
             ((int)(blockIdx.x & 0xff) << 24);
  atomicCAS(c.status, 0, word);
  atomicExch(c.abort_flag, 1);
  __threadfence_system();
}

// Waits until *flag >= target. Returns false after a timeout or an abort
// raised by another block; never traps.
// Polling uses ld.acquire.sys (measured on 2xB200: a 1-block barrier kernel
// 5.3 us vs 6.6 us for relaxed polls + one fence.acq_rel.sys, whose
// system-scope fence costs more than the acquiring loads); environment
// LZ_POLL=1 selects the relaxed-poll + fence form.
LZ_DEV bool lz_wait_ge(const LzDevComm& c, const unsigned long long* flag,
                       unsigned long long target, int phase, int peer) {
  const bool relaxed = c.poll_relaxed != 0;
  if ((relaxed ? ld_relaxed_sys(flag) : ld_acquire_sys(flag)) >= target) {
    if (relaxed) fence_sys();
    return true;
  }
  const unsigned long long t0 = globaltimer();
  for (unsigned int it = 1; it < (1u << 30); ++it) {
    if ((relaxed ? ld_relaxed_sys(flag) : ld_acquire_sys(flag)) >= target) {
      if (relaxed) fence_sys();
      return true;
    }
    if ((it & 255u) == 0u) {
      if (ld_volatile_i32(c.abort_flag)) {
        return false;
      }
      if (globaltimer() - t0 > c.timeout_ns) {
        lz_report(c, LZ_ERR_TIMEOUT, phase, peer);
        return false;
      }
    }
  }
  lz_report(c, LZ_ERR_TIMEOUT, phase, peer);
  return false;
}

// Waits until *flag == target exactly (bounded like lz_wait_ge). For flags
// that live inside reused data areas (slot footers), where a stale word may
// hold any bit pattern and only an exact match may count.
LZ_DEV bool lz_wait_eq(const LzDevComm& c, const unsigned long long* flag,
                       unsigned long long target, int phase, int peer) {
  if (ld_acquire_sys(flag) == target) return true;
  const unsigned long long t0 = globaltimer();
  for (unsigned int it = 1; it < (1u << 30); ++it) {
    if (ld_acquire_sys(flag) == target) return true;
    if ((it & 255u) == 0u) {
      if (ld_volatile_i32(c.abort_flag)) return false;
      if (globaltimer() - t0 > c.timeout_ns) {
        lz_report(c, LZ_ERR_TIMEOUT, phase, peer);
        return false;
      }
    }
  }
  lz_report(c, LZ_ERR_TIMEOUT, phase, peer);
  return false;
}

#ifndef LZ_BOUNDS
#define LZ_BOUNDS 0
#endif
// Debug builds (-DLZ_BOUNDS=1): a peer / multicast store range must lie in one
// mapped heap; a violation is recorded (LZ_ERR_BOUNDS, `where`) and the caller
// skips the store instead of executing it. Release builds compile this away.
LZ_DEV bool lz_range_ok(const LzDevComm& c, const void* p, size_t len, int where) {
#if LZ_BOUNDS
  const char* q = static_cast<const char*>(p);
  for (int r = 0; r < c.world; ++r)
    if (q >= c.heap[r] && q + len <= c.heap[r] + c.heap_bytes) return true;
  if (c.heap_mc && q >= c.heap_mc && q + len <= c.heap_mc + c.heap_bytes) return true;
  lz_report(c, LZ_ERR_BOUNDS, where, 0);
  return false;
#else
  (void)c;
  (void)p;
  (void)len;
  (void)where;
  return true;
#endif
}

LZ_DEV unsigned long long flag_value(unsigned long long epoch, int phase) {
  return ((epoch + 1ull) << 3) | (unsigned long long)phase;
}

// Flag slot [block][src] in the array that lives at `base`.
LZ_DEV unsigned long long* flag_slot(unsigned long long* base, int block, int src) {
  return base + (size_t)block * LZ_MAX_RANKS + src;
}

LZ_DEV unsigned long long* peer_flags(const LzDevComm& c, int peer) {
  return reinterpret_cast<unsigned long long*>(c.heap[peer] + c.flags_off);
}

// CTA barrier ahead of a release signal. The signalling thread then issues
// one st.release.sys (no separate fence): by the PTX memory model the
// bar.sync puts every thread's earlier stores in causality order before that
// release, so they are published with it. `fence_all` (environment
// LZ_FENCE_ALL=1) additionally makes every thread execute fence.acq_rel.sys
// before the barrier: a diagnostic switch for ordering questions, off by
// default (it costs a system-scope fence per warp per signal).
LZ_DEV void publish_block_writes(const LzDevComm& c) {
  if (c.fence_all) fence_sys();
  __syncthreads();
}

// All-pairs barrier between block `blockIdx.x` of every rank. Threads
// 0..world-1 each own one peer. Prior stores of the whole block are released
// by bar.sync followed by each owning thread's st.release.sys to its peer
// (plus a per-thread fence first only under LZ_FENCE_ALL=1).
// Returns false (uniformly for the block) if a wait gave up.
LZ_DEV bool block_barrier(const LzDevComm& c, unsigned long long epoch, int phase) {
  __shared__ int s_fail;
  if (threadIdx.x == 0) s_fail = 0;
  publish_block_writes(c);
  const int t = threadIdx.x;
  if (t < c.world && t != c.rank) {
    const unsigned long long v = flag_value(epoch, phase);
    st_release_sys(flag_slot(peer_flags(c, t), blockIdx.x, c.rank), v);
    if (!lz_wait_ge(c, flag_slot(c.flags, blockIdx.x, t), v, phase, t)) s_fail = 1;
  }
  __syncthreads();
  return s_fail == 0;
}

// Same as block_barrier but only with one partner rank (recursive halving).
LZ_DEV bool pair_barrier(const LzDevComm& c, unsigned long long epoch, int phase, int partner) {
  __shared__ int s_fail2;
  if (threadIdx.x == 0) s_fail2 = 0;
  publish_block_writes(c);
  if (threadIdx.x == 0) {
    const unsigned long long v = flag_value(epoch, phase);
    st_release_sys(flag_slot(peer_flags(c, partner), blockIdx.x, c.rank), v);
    if (!lz_wait_ge(c, flag_slot(c.flags, blockIdx.x, partner), v, phase, partner)) s_fail2 = 1;
  }
  __syncthreads();
  return s_fail2 == 0;
}

// NVLS barrier: one multimem store publishes this rank's flag in every GPU's
// copy of the flag array; the block then waits on its local copies.
LZ_DEV bool block_barrier_mc(const LzDevComm& c, unsigned long long epoch, int phase) {
  __shared__ int s_fail3;
  if (threadIdx.x == 0) s_fail3 = 0;
  publish_block_writes(c);
  const unsigned long long v = flag_value(epoch, phase);
  if (threadIdx.x == 0) {
    fence_sys();
    unsigned long long* mcf =
        reinterpret_cast<unsigned long long*>(c.heap_mc + c.flags_off);
    multimem_st_release_u64(flag_slot(mcf, blockIdx.x, c.rank), v);
  }
  const int t = threadIdx.x;
  if (t < c.world && t != c.rank) {
    if (!lz_wait_ge(c, flag_slot(c.flags, blockIdx.x, t), v, phase, t)) s_fail3 = 1;
  }
  __syncthreads();
  if (threadIdx.x == 0) fence_proxy_alias();
  __syncthreads();
  return s_fail3 == 0;
}

// Every block calls this once at its very end; the last one to finish bumps
// the communicator epoch so the next launch (stream-ordered) sees it.
LZ_DEV void epoch_advance(const LzDevComm& c) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    unsigned int prev = atomicAdd(c.done, 1u);
    if (prev == gridDim.x - 1) {
      *c.done = 0;
      *c.epoch = *c.epoch + 1ull;
      __threadfence();
    }
  }
}

LZ_DEV unsigned long long epoch_read(const LzDevComm& c) {
  return *reinterpret_cast<volatile unsigned long long*>(c.epoch);
}

// Work split helpers: [begin, end) of part `i` out of `parts` over `n` units.
LZ_DEV size_t part_begin(size_t n, int parts, int i) {
  return (n / parts) * i + min((size_t)i, n % parts);
}
