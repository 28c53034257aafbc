// Allreduce kernels over the symmetric heap (NVLink 5 peer loads/stores and
// NVLS multimem). One persistent launch per call; every cross-GPU dependency
// is an in-kernel flag with a bounded wait.
//
// Reference behaviour being re-designed (see the call-site notes there):
//   * two-shot P2P: single_node_nccl_allreduce_benchmark/cuda_p2p_allreduce_kernel.cu:196-285
//     (2(ws-1)+2 launches, staggered pull-RS, pull-AG, unbounded spin barrier);
//   * ring P2P: single_node_nccl_allreduce_benchmark/ring_p2p_allreduce_kernel.cu:125-248
//     (one launch per step, no back-pressure from the right neighbour);
//   * fused all-source fp32 reduction: single_node_nccl_allreduce_benchmark/compressed_p2p_kernel.cu:238-288;
//   * recursive halving-doubling: single_node_nccl_allreduce_benchmark/recursive_halving_allreduce.py:20-113.
//
// Numerics: one-shot and two-shot accumulate every element in fp32 in rank
// order 0..W-1 and round once, so all ranks produce bit-identical results
// equal to a sequential fp32 reference. Ring and RHD round to the storage
// dtype after every hop (as NCCL does); NVLS accumulates in fp32 inside the
// switch in a hardware-defined order.
#include <stdlib.h>

#include "lz_common.cuh"
#include "lz_internal.h"

namespace {

constexpr int kUnroll = 4;

// Per-launch arguments of every allreduce body (meaning of a..d per algo).
struct ArParams {
  const char* in;
  char* out;
  size_t bytes;
  size_t a, b, c, d;
  int i0, i1;
};

// ----------------------------------------------------------------------------
// building blocks
// ----------------------------------------------------------------------------
// Copies vectors [0, n) from src to dst (16 B each) with kUnroll loads in
// flight per thread.
template <bool kRemoteSrc>
__device__ __forceinline__ void copy_vecs(uint4* __restrict__ dst, const uint4* __restrict__ src,
                                          size_t n) {
  const size_t stride = (size_t)blockDim.x * kUnroll;
  size_t i = threadIdx.x;
  for (; i + (kUnroll - 1) * blockDim.x < n; i += stride) {
    uint4 v[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u)
      v[u] = kRemoteSrc ? ld_cg_v4(src + i + u * blockDim.x) : src[i + u * blockDim.x];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) st_v4(dst + i + u * blockDim.x, v[u]);
  }
  for (; i < n; i += blockDim.x) {
    uint4 v = kRemoteSrc ? ld_cg_v4(src + i) : src[i];
    st_v4(dst + i, v);
  }
}

// Slice `p` of a vector of nv 16-byte units split into W near-equal slices,
// then the block's piece of it.
struct Range {
  size_t begin, len;
};
__device__ __forceinline__ Range slice_piece(size_t nv, int W, int p, int G, int b) {
  size_t s0 = part_begin(nv, W, p), s1 = part_begin(nv, W, p + 1);
  size_t len = s1 - s0;
  size_t b0 = part_begin(len, G, b), b1 = part_begin(len, G, b + 1);
  return {s0 + b0, b1 - b0};
}
__device__ __forceinline__ size_t piece_offset_in_slice(size_t nv, int W, int p, int G, int b) {
  size_t s0 = part_begin(nv, W, p), s1 = part_begin(nv, W, p + 1);
  return part_begin(s1 - s0, G, b);
}

// ----------------------------------------------------------------------------
// one-shot: copy-in to the (double-buffered) stage, all-pairs barrier, every
// rank reads every peer and reduces the whole vector locally.
// ----------------------------------------------------------------------------
template <int DT>
__device__ __forceinline__ void oneshot_body(const LzDevComm& c, const ArParams& P) {
  const char* __restrict__ in = P.in;
  char* __restrict__ out = P.out;
  const size_t bytes = P.bytes, os_off = P.a, os_bytes = P.b;
  using V = Vec<DT>;
  constexpr int ES = (DT == LZ_F32) ? 4 : 2;
  const unsigned long long epoch = epoch_read(c);
  const size_t st_off = os_off + (epoch & 1ull) * os_bytes;
  const size_t nv = bytes / 16;
  const size_t tail = bytes - nv * 16;
  const int G = gridDim.x, b = blockIdx.x;
  const size_t v0 = part_begin(nv, G, b), v1 = part_begin(nv, G, b + 1);

  // copy-in (local)
  copy_vecs<false>(reinterpret_cast<uint4*>(c.heap[c.rank] + st_off) + v0,
                   reinterpret_cast<const uint4*>(in) + v0, v1 - v0);
  if (b == G - 1 && threadIdx.x < tail / ES) {
    size_t e = nv * 16 / ES + threadIdx.x;
    if (ES == 2)
      reinterpret_cast<uint16_t*>(c.heap[c.rank] + st_off)[e] =
          reinterpret_cast<const uint16_t*>(in)[e];
    else
      reinterpret_cast<uint32_t*>(c.heap[c.rank] + st_off)[e] =
          reinterpret_cast<const uint32_t*>(in)[e];
  }
  if (!block_barrier(c, epoch, 1)) return;

  const int W = c.world;
  for (size_t i = v0 + threadIdx.x; i < v1; i += blockDim.x) {
    uint4 v[LZ_MAX_RANKS];
#pragma unroll
    for (int r = 0; r < LZ_MAX_RANKS; ++r)
      if (r < W) v[r] = ld_cg_v4(reinterpret_cast<const uint4*>(c.heap[r] + st_off) + i);
    float acc[V::N];
    V::load(acc, v[0]);
#pragma unroll
    for (int r = 1; r < LZ_MAX_RANKS; ++r)
      if (r < W) V::add(acc, v[r]);
    st_v4(reinterpret_cast<uint4*>(out) + i, V::pack(acc));
  }
  if (b == G - 1 && threadIdx.x < tail / ES) {
    size_t e = nv * 16 / ES + threadIdx.x;
    float acc = 0.f;
    for (int r = 0; r < W; ++r) {
      const char* src = c.heap[r] + st_off;
      if (DT == LZ_F32)
        acc += reinterpret_cast<const float*>(src)[e];
      else if (DT == LZ_BF16)
        acc += __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(src)[e]);
      else
        acc += __half2float(reinterpret_cast<const __half*>(src)[e]);
    }
    if (DT == LZ_F32)
      reinterpret_cast<float*>(out)[e] = acc;
    else if (DT == LZ_BF16)
      reinterpret_cast<__nv_bfloat16*>(out)[e] = __float2bfloat16_rn(acc);
    else
      reinterpret_cast<__half*>(out)[e] = __float2half_rn(acc);
  }
  epoch_advance(c);
}

// ----------------------------------------------------------------------------
// two-shot for arbitrary (non-symmetric) buffers:
//   RS by push: slice p of my input -> peer p's stage slot [my rank];
//   barrier; reduce my slice (rank order, fp32) -> out and my stage slot [me];
//   barrier; AG by pull of every peer's result slot.
// ----------------------------------------------------------------------------
template <int DT>
__device__ __forceinline__ void twoshot_body(const LzDevComm& c, const ArParams& P) {
  const char* __restrict__ in = P.in;
  char* __restrict__ out = P.out;
  const size_t bytes = P.bytes, stage_off = P.a;
  using V = Vec<DT>;
  const unsigned long long epoch = epoch_read(c);
  const int W = c.world, me = c.rank, G = gridDim.x, b = blockIdx.x;
  const size_t nv = bytes / 16;
  const size_t slot_vecs = (nv + W - 1) / W;
  const uint4* vin = reinterpret_cast<const uint4*>(in);
  uint4* vout = reinterpret_cast<uint4*>(out);

  // RS push (staggered peer order spreads the load over the switch ports)
  for (int k = 1; k < W; ++k) {
    const int p = (me + k) % W;
    Range rg = slice_piece(nv, W, p, G, b);
    size_t po = piece_offset_in_slice(nv, W, p, G, b);
    uint4* dst = reinterpret_cast<uint4*>(c.heap[p] + stage_off) + (size_t)me * slot_vecs + po;
    if (lz_range_ok(c, dst, rg.len * 16, 25)) copy_vecs<false>(dst, vin + rg.begin, rg.len);
  }
  if (!block_barrier(c, epoch, 1)) return;

  {
    Range rg = slice_piece(nv, W, me, G, b);
    size_t po = piece_offset_in_slice(nv, W, me, G, b);
    const uint4* stage = reinterpret_cast<const uint4*>(c.heap[me] + stage_off);
    uint4* my_slot = reinterpret_cast<uint4*>(c.heap[me] + stage_off) + (size_t)me * slot_vecs + po;
    for (size_t i = threadIdx.x; i < rg.len; i += blockDim.x) {
      uint4 v[LZ_MAX_RANKS];
#pragma unroll
      for (int r = 0; r < LZ_MAX_RANKS; ++r)
        if (r < W)
          v[r] = (r == me) ? vin[rg.begin + i] : ld_cg_v4(stage + (size_t)r * slot_vecs + po + i);
      float acc[V::N];
      V::load(acc, v[0]);
#pragma unroll
      for (int r = 1; r < LZ_MAX_RANKS; ++r)
        if (r < W) V::add(acc, v[r]);
      uint4 res = V::pack(acc);
      st_v4(vout + rg.begin + i, res);
      st_v4(my_slot + i, res);
    }
  }
  if (!block_barrier(c, epoch, 2)) return;

  for (int k = 1; k < W; ++k) {
    const int p = (me + W - k) % W;
    Range rg = slice_piece(nv, W, p, G, b);
    size_t po = piece_offset_in_slice(nv, W, p, G, b);
    const uint4* src = reinterpret_cast<const uint4*>(c.heap[p] + stage_off) + (size_t)p * slot_vecs + po;
    copy_vecs<true>(vout + rg.begin, src, rg.len);
  }
  epoch_advance(c);
}

// ----------------------------------------------------------------------------
// two-shot, zero-copy: input and output live at the same heap offsets on
// every rank. Pull-reduce my slice from all ranks, push the result to all.
// ----------------------------------------------------------------------------
template <int DT>
__device__ __forceinline__ void twoshot_sym_body(const LzDevComm& c, const ArParams& P) {
  const size_t in_off = P.a, out_off = P.b, bytes = P.bytes;
  using V = Vec<DT>;
  const unsigned long long epoch = epoch_read(c);
  const int W = c.world, me = c.rank, G = gridDim.x, b = blockIdx.x;
  const size_t nv = bytes / 16;
  if (!block_barrier(c, epoch, 1)) return;
  Range rg = slice_piece(nv, W, me, G, b);
  const size_t stride = (size_t)blockDim.x * 2;
  size_t i = threadIdx.x;
  for (; i < rg.len; i += stride) {
    const bool two = i + blockDim.x < rg.len;
    uint4 v[2][LZ_MAX_RANKS];
#pragma unroll
    for (int r = 0; r < LZ_MAX_RANKS; ++r) {
      if (r < W) {
        const uint4* src = reinterpret_cast<const uint4*>(c.heap[r] + in_off) + rg.begin;
        v[0][r] = ld_cg_v4(src + i);
        if (two) v[1][r] = ld_cg_v4(src + i + blockDim.x);
      }
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      if (u == 1 && !two) break;
      float acc[V::N];
      V::load(acc, v[u][0]);
#pragma unroll
      for (int r = 1; r < LZ_MAX_RANKS; ++r)
        if (r < W) V::add(acc, v[u][r]);
      uint4 res = V::pack(acc);
      const size_t j = rg.begin + i + u * blockDim.x;
#pragma unroll
      for (int k = 0; k < LZ_MAX_RANKS; ++k) {
        if (k < W) {
          const int p = (me + k) % W;
          st_v4(reinterpret_cast<uint4*>(c.heap[p] + out_off) + j, res);
        }
      }
    }
  }
  if (!block_barrier(c, epoch, 2)) return;
  epoch_advance(c);
}

// ----------------------------------------------------------------------------
// NVLS: the switch reads my slice from every GPU and reduces it in fp32
// (multimem.ld_reduce); one multimem.st writes the result to every GPU.
// Non-symmetric buffers are staged through the heap with local copies.
// ----------------------------------------------------------------------------
template <int DT>
__device__ __forceinline__ void nvls_body(const LzDevComm& c, const ArParams& P) {
  const char* __restrict__ in = P.in;
  char* __restrict__ out = P.out;
  const size_t in_off = P.a, out_off = P.b, bytes = P.bytes;
  const int copy_in = P.i0, copy_out = P.i1;
  const unsigned long long epoch = epoch_read(c);
  const int W = c.world, me = c.rank, G = gridDim.x, b = blockIdx.x;
  const size_t nv = bytes / 16;
  // Block b owns the vectors b*T + t (mod G*T) of every slice: grid-stride
  // interleaving measured 7 % faster than contiguous per-block pieces for the
  // multimem loop (4 x B200, 1 GiB: 2.32 vs 2.50 ms). Copy-in, reduction and
  // copy-out use the same mapping, so block b's barrier covers exactly the
  // vectors its peers' blocks b touch.
  const size_t stride = (size_t)G * blockDim.x;
  if (copy_in) {
    for (int p = 0; p < W; ++p) {
      const size_t s0 = part_begin(nv, W, p), s1 = part_begin(nv, W, p + 1);
      uint4* dst = reinterpret_cast<uint4*>(c.heap[me] + in_off);
      const uint4* src = reinterpret_cast<const uint4*>(in);
      for (size_t i = s0 + (size_t)b * blockDim.x + threadIdx.x; i < s1; i += stride) dst[i] = ld_nc_v4(src + i);
    }
  }
  if (!block_barrier_mc(c, epoch, 1)) return;
  {
    const size_t s0 = part_begin(nv, W, me), s1 = part_begin(nv, W, me + 1);
    const uint4* src = reinterpret_cast<const uint4*>(c.heap_mc + in_off);
    uint4* dst = reinterpret_cast<uint4*>(c.heap_mc + out_off);
    // P.c: loads in flight per thread (1..8); P.d bit 0: bf16 accumulation in the switch
    const int U = P.c >= 1 && P.c <= 8 ? (int)P.c : kUnroll;
    const bool noacc = (DT == LZ_BF16) && (P.d & 1);
    size_t i = s0 + (size_t)b * blockDim.x + threadIdx.x;
    for (; i + (U - 1) * stride < s1; i += U * stride) {
      uint4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (u < U)
          v[u] = noacc ? multimem_ld_reduce_bf16_noacc(src + i + u * stride)
                       : multimem_ld_reduce_v4<DT>(src + i + u * stride);
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (u < U) multimem_st_v4(dst + i + u * stride, v[u]);
    }
    for (; i < s1; i += stride) multimem_st_v4(dst + i, multimem_ld_reduce_v4<DT>(src + i));
  }
  if (!block_barrier_mc(c, epoch, 2)) return;
  if (copy_out) {
    for (int p = 0; p < W; ++p) {
      const size_t s0 = part_begin(nv, W, p), s1 = part_begin(nv, W, p + 1);
      const uint4* src = reinterpret_cast<const uint4*>(c.heap[me] + out_off);
      uint4* dst = reinterpret_cast<uint4*>(out);
      for (size_t i = s0 + (size_t)b * blockDim.x + threadIdx.x; i < s1; i += stride) dst[i] = ld_cg_v4(src + i);
    }
  }
  epoch_advance(c);
}

// NVLS one-shot (small messages): copy-in to the double-buffered stage, one
// barrier, every rank reads the whole reduced vector through the switch.
template <int DT>
__device__ __forceinline__ void nvls_oneshot_body(const LzDevComm& c, const ArParams& P) {
  const char* __restrict__ in = P.in;
  char* __restrict__ out = P.out;
  const size_t bytes = P.bytes, os_off = P.a, os_bytes = P.b;
  const unsigned long long epoch = epoch_read(c);
  const size_t st_off = os_off + (epoch & 1ull) * os_bytes;
  const size_t nv = bytes / 16;
  const int G = gridDim.x, b = blockIdx.x;
  const size_t v0 = part_begin(nv, G, b), v1 = part_begin(nv, G, b + 1);
  copy_vecs<false>(reinterpret_cast<uint4*>(c.heap[c.rank] + st_off) + v0,
                   reinterpret_cast<const uint4*>(in) + v0, v1 - v0);
  if (!block_barrier_mc(c, epoch, 1)) return;
  const uint4* src = reinterpret_cast<const uint4*>(c.heap_mc + st_off);
  for (size_t i = v0 + threadIdx.x; i < v1; i += blockDim.x)
    st_v4(reinterpret_cast<uint4*>(out) + i, multimem_ld_reduce_v4<DT>(src + i));
  epoch_advance(c);
}

// ----------------------------------------------------------------------------
// Ring: every tile makes 2(W-1) hops through NS slots in the right
// neighbour's stage, with a ready flag (left -> me) and a credit flag
// (right -> me) per block, so a sender never overruns its receiver.
// Hop k of a tile carries chunk (rank - k) mod W; hops 1..W-1 add the local
// input (reduce-scatter), hops >= W-1 also write the output (all-gather).
// Tiles are processed tile-major (all hops of tile t before tile t+1) so the
// receiver consumes slots in exactly the order they were filled; with NS >= 2
// the earliest pending hop of the whole ring can always make progress.
// ----------------------------------------------------------------------------
constexpr int kRingSlots = 4;

template <int DT>
__device__ __forceinline__ void ring_body(const LzDevComm& c, const ArParams& P) {
  const char* __restrict__ in = P.in;
  char* __restrict__ out = P.out;
  const size_t bytes = P.bytes, stage_off = P.a, tile_vecs = P.b, ready_off = P.c, credit_off = P.d;
  using V = Vec<DT>;
  const unsigned long long epoch = epoch_read(c);
  const int W = c.world, me = c.rank, G = gridDim.x, b = blockIdx.x;
  const int left = (me + W - 1) % W, right = (me + 1) % W;
  const size_t nv = bytes / 16;
  const uint4* vin = reinterpret_cast<const uint4*>(in);
  uint4* vout = reinterpret_cast<uint4*>(out);
  // every chunk piece of this block is cut into the same number of tiles
  const size_t max_piece = ((nv + W - 1) / W + G - 1) / G;
  const size_t ntiles = (max_piece + tile_vecs - 1) / tile_vecs;
  const size_t block_slots = (size_t)kRingSlots * tile_vecs;
  const int hops = 2 * W - 2;  // sends per tile
  uint4* my_slots = reinterpret_cast<uint4*>(c.heap[me] + stage_off) + (size_t)b * block_slots;
  uint4* right_slots = reinterpret_cast<uint4*>(c.heap[right] + stage_off) + (size_t)b * block_slots;
  unsigned long long* my_ready = reinterpret_cast<unsigned long long*>(c.heap[me] + ready_off) + b;
  unsigned long long* right_ready =
      reinterpret_cast<unsigned long long*>(c.heap[right] + ready_off) + b;
  unsigned long long* my_credit = reinterpret_cast<unsigned long long*>(c.heap[me] + credit_off) + b;
  unsigned long long* left_credit =
      reinterpret_cast<unsigned long long*>(c.heap[left] + credit_off) + b;
  const unsigned long long base = (epoch + 1ull) << 32;
  __shared__ int s_fail;
  if (threadIdx.x == 0) s_fail = 0;
  __syncthreads();

  for (size_t t = 0; t < ntiles; ++t) {
    for (int k = 0; k <= hops; ++k) {
      const int chunk = ((me - k) % W + W) % W;
      Range rg = slice_piece(nv, W, chunk, G, b);
      const size_t t0 = t * tile_vecs;
      const size_t tl = (t0 < rg.len) ? min(tile_vecs, rg.len - t0) : 0;
      const unsigned long long q_send = (unsigned long long)t * hops + k;  // valid if k < hops
      const unsigned long long q_recv = q_send - 1;                        // valid if k > 0
      if (threadIdx.x == 0) {
        if (k > 0 && !lz_wait_ge(c, my_ready, base + q_recv + 1, 3, left)) s_fail = 1;
        if (!s_fail && k < hops && q_send >= kRingSlots &&
            !lz_wait_ge(c, my_credit, base + q_send - kRingSlots + 1, 4, right))
          s_fail = 1;
      }
      __syncthreads();
      if (s_fail) return;
      const size_t rslot = (size_t)((q_recv + kRingSlots) % kRingSlots);
      const size_t sslot = (size_t)(q_send % kRingSlots);
      for (size_t i = threadIdx.x; i < tl; i += blockDim.x) {
        uint4 data;
        if (k == 0) {
          data = vin[rg.begin + t0 + i];
        } else {
          uint4 r = ld_cg_v4(my_slots + rslot * tile_vecs + i);
          if (k <= W - 1) {
            float acc[V::N];
            V::load(acc, r);
            V::add(acc, vin[rg.begin + t0 + i]);
            data = V::pack(acc);
          } else {
            data = r;
          }
          if (k >= W - 1) st_v4(vout + rg.begin + t0 + i, data);
        }
        if (k < hops) st_v4(right_slots + sslot * tile_vecs + i, data);
      }
      publish_block_writes(c);
      if (threadIdx.x == 0) {
        if (k > 0) st_release_sys(left_credit, base + q_recv + 1);
        if (k < hops) st_release_sys(right_ready, base + q_send + 1);
      }
    }
  }
  epoch_advance(c);
}

// ----------------------------------------------------------------------------
// Recursive halving-doubling (power-of-two W) on the stage, pairwise barriers.
// Halving round k: partner = me ^ (W >> (k+1)); keep the half selected by that
// bit and add the partner's partial sums for it. Doubling mirrors it and
// pulls the partner's finished half.
// ----------------------------------------------------------------------------
template <int DT>
__device__ __forceinline__ void rhd_body(const LzDevComm& c, const ArParams& P) {
  const char* __restrict__ in = P.in;
  char* __restrict__ out = P.out;
  const size_t bytes = P.bytes, stage_off = P.a;
  using V = Vec<DT>;
  const unsigned long long epoch = epoch_read(c);
  const int W = c.world, me = c.rank, G = gridDim.x, b = blockIdx.x;
  const size_t nv = bytes / 16;
  uint4* my = reinterpret_cast<uint4*>(c.heap[me] + stage_off);
  // copy-in my piece of every segment
  for (int p = 0; p < W; ++p) {
    Range rg = slice_piece(nv, W, p, G, b);
    copy_vecs<false>(my + rg.begin, reinterpret_cast<const uint4*>(in) + rg.begin, rg.len);
  }
  int rounds = 0;
  while ((1 << rounds) < W) ++rounds;
  int lo = 0, len = W;  // active segment range [lo, lo+len)
  for (int k = 0; k < rounds; ++k) {
    const int half = len >> 1;
    const int bit = W >> (k + 1);
    const int partner = me ^ bit;
    const int keep_lo = (me & bit) ? lo + half : lo;
    if (!pair_barrier(c, epoch, 1 + k, partner)) return;
    const uint4* ps = reinterpret_cast<const uint4*>(c.heap[partner] + stage_off);
    for (int sgm = keep_lo; sgm < keep_lo + half; ++sgm) {
      Range rg = slice_piece(nv, W, sgm, G, b);
      for (size_t i = threadIdx.x; i < rg.len; i += blockDim.x) {
        uint4 a = my[rg.begin + i];
        uint4 o = ld_cg_v4(ps + rg.begin + i);
        float acc[V::N];
        V::load(acc, a);
        V::add(acc, o);
        my[rg.begin + i] = V::pack(acc);
      }
    }
    lo = keep_lo;
    len = half;
  }
  for (int k = rounds - 1; k >= 0; --k) {
    const int bit = W >> (k + 1);
    const int partner = me ^ bit;
    // partner's finished range is the sibling of mine at this level
    const int plo = lo ^ bit;
    if (!pair_barrier(c, epoch, 4 + k, partner)) return;
    const uint4* ps = reinterpret_cast<const uint4*>(c.heap[partner] + stage_off);
    for (int sgm = plo; sgm < plo + len; ++sgm) {
      Range rg = slice_piece(nv, W, sgm, G, b);
      copy_vecs<true>(my + rg.begin, ps + rg.begin, rg.len);
    }
    lo = min(lo, plo);
    len <<= 1;
  }
  // every peer must be done reading my stage before the next call rewrites it
  if (!block_barrier(c, epoch, 7)) return;
  for (int p = 0; p < W; ++p) {
    Range rg = slice_piece(nv, W, p, G, b);
    copy_vecs<false>(reinterpret_cast<uint4*>(out) + rg.begin, my + rg.begin, rg.len);
  }
  epoch_advance(c);
}

__device__ __forceinline__ void barrier_body(const LzDevComm& c, const ArParams&) {
  const unsigned long long epoch = epoch_read(c);
  if (!block_barrier(c, epoch, 1)) return;
  epoch_advance(c);
}

// ----------------------------------------------------------------------------
// low-latency one-shot for small messages: every rank pushes its input
// straight into each peer's receive area as 8-byte words {4 payload bytes,
// 32-bit call flag}. A naturally aligned 64-bit store is single-copy atomic,
// so a word whose flag equals this call's value carries this call's payload:
// no barrier and no fence, one NVLink traversal. Receivers poll their own
// memory and reduce in rank order (fp32), bit-identical to the other
// algorithms. Areas are double-buffered by call parity: a rank reaches call
// e+2 (reusing parity e&1) only after every peer has started call e+1, i.e.
// finished reading call e. Flags are an odd-multiplier hash of the call
// number with the low bit set: never 0 (zeroed memory) and distinct across
// 2^31 uses of one parity.
// Params: a = heap offset of the areas, b = bytes per parity, c = bytes per
// source rank (2 x the largest message).
// ----------------------------------------------------------------------------
LZ_DEV uint32_t ll_flag(unsigned long long epoch) {
  return ((uint32_t)(epoch + 1ull) * 0x9E3779B1u) | 1u;
}
LZ_DEV void st_ll2(void* p, unsigned long long a, unsigned long long b) {
  asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}
LZ_DEV void ld_ll2(const void* p, unsigned long long& a, unsigned long long& b) {
  asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

// Polls the 4 words of one 16-byte payload vector until all carry `flag`.
LZ_DEV uint4 ll_recv(const LzDevComm& c, const char* p, uint32_t flag, bool& ok, int peer) {
  unsigned long long w0, w1, w2, w3;
  ld_ll2(p, w0, w1);
  ld_ll2(p + 16, w2, w3);
  const unsigned long long t0 = globaltimer();
  unsigned int it = 0;
  while (ok && ((uint32_t)(w0 >> 32) != flag || (uint32_t)(w1 >> 32) != flag ||
                (uint32_t)(w2 >> 32) != flag || (uint32_t)(w3 >> 32) != flag)) {
    if ((++it & 1023u) == 0u) {
      if (ld_volatile_i32(c.abort_flag)) {
        ok = false;
        break;
      }
      if (globaltimer() - t0 > c.timeout_ns) {
        lz_report(c, LZ_ERR_TIMEOUT, 9, peer);
        ok = false;
        break;
      }
    }
    ld_ll2(p, w0, w1);
    ld_ll2(p + 16, w2, w3);
  }
  return make_uint4((uint32_t)w0, (uint32_t)w1, (uint32_t)w2, (uint32_t)w3);
}

template <int DT>
__device__ __forceinline__ void ll_oneshot_body(const LzDevComm& c, const ArParams& P) {
  using V = Vec<DT>;
  const unsigned long long epoch = epoch_read(c);
  const uint32_t flag = ll_flag(epoch);
  const unsigned long long fhi = (unsigned long long)flag << 32;
  const size_t area = P.a + (epoch & 1ull) * P.b, slot = P.c;
  const int W = c.world, me = c.rank;
  const size_t nv = P.bytes / 16;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  const size_t i0 = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const uint4* in = reinterpret_cast<const uint4*>(P.in);
  for (size_t i = i0; i < nv; i += stride) {
    const uint4 v = in[i];
    const unsigned long long w0 = fhi | v.x, w1 = fhi | v.y, w2 = fhi | v.z, w3 = fhi | v.w;
#pragma unroll
    for (int r = 0; r < LZ_MAX_RANKS; ++r) {
      if (r >= W || r == me) continue;
      char* dst = c.heap[r] + area + (size_t)me * slot + i * 32;
      if (!lz_range_ok(c, dst, 32, 24)) continue;
      st_ll2(dst, w0, w1);
      st_ll2(dst + 16, w2, w3);
    }
  }
  bool ok = true;
  for (size_t i = i0; i < nv; i += stride) {
    const uint4 mine = in[i];
    float acc[V::N];
#pragma unroll
    for (int r = 0; r < LZ_MAX_RANKS; ++r) {
      if (r >= W) continue;
      const uint4 v = r == me ? mine : ll_recv(c, c.heap[me] + area + (size_t)r * slot + i * 32, flag, ok, r);
      if (r == 0) V::load(acc, v);
      else V::add(acc, v);
    }
    st_v4(reinterpret_cast<uint4*>(P.out) + i, V::pack(acc));
  }
  epoch_advance(c);
}

enum ArKind { K_ONESHOT, K_TWOSHOT, K_TWOSHOT_SYM, K_NVLS, K_NVLS_ONESHOT, K_RING, K_RHD, K_BARRIER, K_LL };

template <int DT, int K>
__device__ __forceinline__ void ar_body(const LzDevComm& c, const ArParams& p) {
  if constexpr (K == K_ONESHOT) oneshot_body<DT>(c, p);
  else if constexpr (K == K_TWOSHOT) twoshot_body<DT>(c, p);
  else if constexpr (K == K_TWOSHOT_SYM) twoshot_sym_body<DT>(c, p);
  else if constexpr (K == K_NVLS) nvls_body<DT>(c, p);
  else if constexpr (K == K_NVLS_ONESHOT) nvls_oneshot_body<DT>(c, p);
  else if constexpr (K == K_RING) ring_body<DT>(c, p);
  else if constexpr (K == K_RHD) rhd_body<DT>(c, p);
  else if constexpr (K == K_LL) ll_oneshot_body<DT>(c, p);
  else barrier_body(c, p);
}

// Real multi-GPU launch: one rank per GPU.
template <int DT, int K>
__global__ void __launch_bounds__(512) ar_kernel(LzDevComm c, ArParams p) {
  ar_body<DT, K>(c, p);
}

// Single-GPU emulation of gridDim.y ranks in ONE cooperative launch (all
// blocks co-resident): block (x, y) runs block x of virtual rank y.
template <int DT, int K>
__global__ void __launch_bounds__(512) ar_emu_kernel(const LzDevComm* cs, const ArParams* ps) {
  ar_body<DT, K>(cs[blockIdx.y], ps[blockIdx.y]);
}

__global__ void read_epoch_kernel(LzDevComm c, unsigned long long* out) { *out = *c.epoch; }

// World size 1: the allreduce is the identity; out-of-place calls copy with
// 16-byte vectors (tail bytes by the first threads).
__global__ void __launch_bounds__(512) local_copy_kernel(const char* __restrict__ in,
                                                         char* __restrict__ out, size_t bytes) {
  const size_t nv = bytes / 16;
  const uint4* src = reinterpret_cast<const uint4*>(in);
  uint4* dst = reinterpret_cast<uint4*>(out);
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (; i + 3 * stride < nv; i += 4 * stride) {
    uint4 a = ld_nc_v4(src + i), b = ld_nc_v4(src + i + stride), c = ld_nc_v4(src + i + 2 * stride),
          d = ld_nc_v4(src + i + 3 * stride);
    st_cs_v4(dst + i, a);
    st_cs_v4(dst + i + stride, b);
    st_cs_v4(dst + i + 2 * stride, c);
    st_cs_v4(dst + i + 3 * stride, d);
  }
  for (; i < nv; i += stride) st_cs_v4(dst + i, ld_nc_v4(src + i));
  if (blockIdx.x == 0 && threadIdx.x < bytes - nv * 16) out[nv * 16 + threadIdx.x] = in[nv * 16 + threadIdx.x];
}

// ----------------------------------------------------------------------------
// host side
// ----------------------------------------------------------------------------
inline int clamp_int(long long v, int lo, int hi) {
  return (int)(v < lo ? lo : (v > hi ? hi : v));
}

}  // namespace

// Flag-area layout inside the heap (offsets from the heap base):
//   [0, 32K)       barrier flags [LZ_MAX_BLOCKS][LZ_MAX_RANKS]
//   [32K, 36K)     ring ready flags [LZ_MAX_BLOCKS]
//   [36K, 40K)     ring credit flags [LZ_MAX_BLOCKS]
//   [64K, 1M)      other protocols (weight transfer)
static constexpr size_t kRingReadyOff = 32768;
static constexpr size_t kRingCreditOff = 36864;

static int init_comm_state(LzComm* c, int dev, size_t oneshot_bytes, size_t stage_bytes,
                           double timeout_s) {
  c->oneshot_bytes = (oneshot_bytes + 4095) / 4096 * 4096;
  c->oneshot_off = kLzFlagsBytes;
  c->ll_off = c->oneshot_off + 2 * c->oneshot_bytes;
  c->ll_bytes = (size_t)c->dev.world * 2 * kLzLlMaxBytes;  // per parity
  c->stage_off = c->ll_off + 2 * c->ll_bytes;
  c->stage_bytes = (stage_bytes + 4095) / 4096 * 4096;
  c->user_off = c->stage_off + c->stage_bytes;
  c->user_off = (c->user_off + (2u << 20) - 1) / (2u << 20) * (2u << 20);
  if (c->user_off > c->heap_bytes) {
    lz_set_error("heap too small: need %zu bytes for flags+stages, have %zu", c->user_off,
                 c->heap_bytes);
    return LZE_ARG;
  }
  char* dstate = nullptr;
  LZ_CUDA_TRY(cudaMalloc(&dstate, 256));
  LZ_CUDA_TRY(cudaMemset(dstate, 0, 256));
  c->dev.epoch = reinterpret_cast<unsigned long long*>(dstate);
  c->dev.done = reinterpret_cast<unsigned int*>(dstate + 64);
  c->dev.abort_flag = reinterpret_cast<int*>(dstate + 128);
  c->ce_seq = reinterpret_cast<unsigned long long*>(dstate + 192);
  c->ce_done = reinterpret_cast<unsigned int*>(dstate + 224);
  int* st_host = nullptr;
  LZ_CUDA_TRY(cudaHostAlloc(&st_host, 64, cudaHostAllocMapped));
  memset(st_host, 0, 64);
  int* st_dev = nullptr;
  LZ_CUDA_TRY(cudaHostGetDevicePointer(&st_dev, st_host, 0));
  c->status_host = st_host;
  c->dev.status = st_dev;
  c->dev.timeout_ns = (unsigned long long)(timeout_s * 1e9);
  c->dev.heap_bytes = c->heap_bytes;
  {
    const char* fa = getenv("LZ_FENCE_ALL");
    c->dev.fence_all = (fa && atoi(fa) != 0) ? 1 : 0;
    const char* pr = getenv("LZ_POLL");
    c->dev.poll_relaxed = (pr && atoi(pr) == 1) ? 1 : 0;
  }
  c->dev.flags_off = 0;
  c->dev.flags = reinterpret_cast<unsigned long long*>(c->dev.heap[c->dev.rank]);
  LZ_CUDA_TRY(cudaMemset(c->dev.heap[c->dev.rank], 0, kLzFlagsBytes));
  LZ_CUDA_TRY(cudaMemset(c->dev.heap[c->dev.rank] + c->ll_off, 0, 2 * c->ll_bytes));
  LZ_CUDA_TRY(cudaDeviceSynchronize());  // zeroed before any peer can push (callers barrier next)
  int sms = 0;
  LZ_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  c->sm_count = sms;
  c->device = dev;
  return LZE_OK;
}

extern "C" int lz_comm_create(LzHeap* h, size_t oneshot_bytes, size_t stage_bytes,
                              double timeout_s, LzComm** out) {
  const int dev = lz_heap_device(h);
  LZ_CUDA_TRY(cudaSetDevice(dev));
  LzComm* c = new LzComm();
  c->heap = h;
  c->heap_bytes = lz_heap_size(h);
  memset(&c->dev, 0, sizeof(c->dev));
  c->dev.rank = lz_heap_rank(h);
  c->dev.world = lz_heap_world(h);
  for (int r = 0; r < c->dev.world; ++r) c->dev.heap[r] = (char*)lz_heap_ptr(h, r);
  c->dev.heap_mc = (char*)lz_heap_mc_ptr(h);
  int rc = init_comm_state(c, dev, oneshot_bytes, stage_bytes, timeout_s);
  if (rc) {
    delete c;
    return rc;
  }
  LZ_CUDA_TRY(cudaDeviceSynchronize());
  *out = c;
  return LZE_OK;
}

static void free_comm_state(LzComm* c) {
  lz_ce_release(c);
  cudaFree(c->dev.epoch);
  cudaFreeHost(c->status_host);
}

extern "C" int lz_comm_destroy(LzComm* c) {
  if (!c) return LZE_OK;
  cudaSetDevice(c->device);
  cudaDeviceSynchronize();
  free_comm_state(c);
  delete c;
  return LZE_OK;
}

extern "C" size_t lz_comm_user_offset(LzComm* c) { return c->user_off; }
extern "C" int lz_comm_status(LzComm* c) {
  return *reinterpret_cast<volatile int*>(c->status_host);
}
extern "C" int lz_comm_clear_status(LzComm* c) {
  *reinterpret_cast<volatile int*>(c->status_host) = 0;
  cudaMemset(c->dev.abort_flag, 0, sizeof(int));
  return LZE_OK;
}

extern "C" int lz_comm_epoch(LzComm* c, unsigned long long* epoch, cudaStream_t s) {
  LZ_CUDA_TRY(cudaMemcpyAsync(epoch, c->dev.epoch, 8, cudaMemcpyDeviceToHost, s));
  LZ_CUDA_TRY(cudaStreamSynchronize(s));
  return LZE_OK;
}

size_t lz_comm_heap_offset(const LzComm* c, const void* p, size_t bytes) {
  const char* base = c->dev.heap[c->dev.rank];
  const char* q = static_cast<const char*>(p);
  if (q >= base + c->user_off && q + bytes <= base + c->heap_bytes) return (size_t)(q - base);
  return (size_t)-1;
}

// A fully resolved launch: kernel kind, grid and arguments.
struct ArPlan {
  int kind;
  int G;
  int nthreads;
  ArParams p;
};

template <int DT>
static int plan_allreduce(const LzComm* c, const void* in, void* out, size_t count, int algo,
                          int nblocks, int nthreads, ArPlan* plan) {
  const int W = c->dev.world;
  const size_t es = (DT == LZ_F32) ? 4 : 2;
  const size_t bytes = count * es;
  const size_t nv = bytes / 16;
  // Launch shape measured on 8xB200 (1 GiB: NVLS 256 threads x 4 loads in
  // flight = 809 GB/s busbw; 64 MB: 512 threads x 8 in flight): used when the
  // caller does not force one (nthreads <= 0).
  const bool auto_shape = nthreads <= 0;
  int nvls_unroll = 8;
  if (auto_shape) {
    nthreads = 512;
    if (algo == LZ_ALGO_NVLS && bytes >= (128u << 20)) {
      nthreads = 256;
      nvls_unroll = 4;
    }
  } else {
    nvls_unroll = kUnroll;
  }
  nthreads = clamp_int(nthreads, 32, 512) / 32 * 32;
  const int smax = c->sm_count < LZ_MAX_BLOCKS ? c->sm_count : LZ_MAX_BLOCKS;
  ArPlan P;
  memset(&P, 0, sizeof(P));
  P.nthreads = nthreads;
  P.p.in = static_cast<const char*>(in);
  P.p.out = static_cast<char*>(out);
  P.p.bytes = bytes;
  const bool aligned =
      (bytes % 16 == 0) && ((uintptr_t)in % 16 == 0) && ((uintptr_t)out % 16 == 0);
  if (algo != LZ_ALGO_ONESHOT && !aligned) {
    lz_set_error("algo %d needs 16-byte aligned pointers and a size multiple of 16 bytes", algo);
    return LZE_ARG;
  }
  if (algo != LZ_ALGO_ONESHOT && algo != LZ_ALGO_NVLS_ONESHOT && (size_t)W > nv)
    algo = LZ_ALGO_ONESHOT;  // tiny vector: less than one 16-byte unit per rank
  // Explicit grids may exceed one CTA per SM, up to what stays co-resident.
  const int gmax = nblocks > 0 ? (c->sm_count * (2048 / nthreads) < LZ_MAX_BLOCKS
                                      ? c->sm_count * (2048 / nthreads)
                                      : LZ_MAX_BLOCKS)
                               : smax;
  auto grid = [&](size_t units_per_block) {
    int G = nblocks > 0 ? nblocks
                        : clamp_int((long long)((nv / W + units_per_block - 1) / units_per_block), 1, smax);
    return clamp_int(G, 1, gmax);
  };
  switch (algo) {
    case LZ_ALGO_ONESHOT:
    case LZ_ALGO_NVLS_ONESHOT: {
      if (bytes > c->oneshot_bytes) {
        lz_set_error("one-shot limited to %zu bytes (got %zu)", c->oneshot_bytes, bytes);
        return LZE_ARG;
      }
      if ((uintptr_t)in % 16 || (uintptr_t)out % 16) {
        lz_set_error("one-shot needs 16-byte aligned pointers");
        return LZE_ARG;
      }
      int G = nblocks > 0 ? nblocks
                          : clamp_int((long long)((nv + nthreads * 2 - 1) / (nthreads * 2)), 1, smax);
      P.G = clamp_int(G, 1, smax);
      P.p.a = c->oneshot_off;
      P.p.b = c->oneshot_bytes;
      if (algo == LZ_ALGO_NVLS_ONESHOT) {
        if (!c->dev.heap_mc || bytes % 16) {
          lz_set_error("NVLS one-shot needs multicast support and 16-byte multiple sizes");
          return LZE_UNSUPPORTED;
        }
        P.kind = K_NVLS_ONESHOT;
      } else {
        P.kind = K_ONESHOT;
      }
      break;
    }
    case LZ_ALGO_LL: {
      if (bytes > kLzLlMaxBytes || !aligned) {
        lz_set_error("low-latency one-shot needs 16-byte aligned pointers and sizes up to %zu bytes (got %zu)",
                     (size_t)kLzLlMaxBytes, bytes);
        return LZE_ARG;
      }
      if (auto_shape) nthreads = nv >= 512 * 8 ? 512 : (nv >= 128 ? 256 : 128);
      P.nthreads = nthreads;
      // every block waits only on the same-index blocks of its peers; G never
      // exceeds one block per SM so all of them are resident
      P.G = nblocks > 0 ? clamp_int(nblocks, 1, smax)
                        : clamp_int((long long)((nv + nthreads - 1) / nthreads), 1, smax);
      P.p.a = c->ll_off;
      P.p.b = c->ll_bytes;
      P.p.c = 2 * kLzLlMaxBytes;
      P.kind = K_LL;
      break;
    }
    case LZ_ALGO_TWOSHOT: {
      const size_t in_off = lz_comm_heap_offset(c, in, bytes);
      const size_t out_off = lz_comm_heap_offset(c, out, bytes);
      P.G = grid((size_t)nthreads * 2);
      if (in_off != (size_t)-1 && out_off != (size_t)-1) {
        P.kind = K_TWOSHOT_SYM;
        P.p.a = in_off;
        P.p.b = out_off;
      } else {
        const size_t slot = (nv + W - 1) / W * 16;
        if (slot * W > c->stage_bytes) {
          lz_set_error("two-shot stage too small (%zu needed, %zu available)", slot * W,
                       c->stage_bytes);
          return LZE_ARG;
        }
        P.kind = K_TWOSHOT;
        P.p.a = c->stage_off;
      }
      break;
    }
    case LZ_ALGO_NVLS: {
      if (!c->dev.heap_mc) {
        lz_set_error("NVLS requested but the heap has no multicast mapping");
        return LZE_UNSUPPORTED;
      }
      size_t in_off = lz_comm_heap_offset(c, in, bytes);
      size_t out_off = lz_comm_heap_offset(c, out, bytes);
      int copy_in = 0, copy_out = 0;
      if (in_off == (size_t)-1 || out_off == (size_t)-1) {
        if (bytes > c->stage_bytes) {
          lz_set_error("NVLS stage too small (%zu > %zu)", bytes, c->stage_bytes);
          return LZE_ARG;
        }
        if (in_off == (size_t)-1) {
          copy_in = 1;
          in_off = c->stage_off;
        }
        out_off = c->stage_off;  // reduce into the stage, then copy to the caller's buffer
        copy_out = 1;
      }
      P.kind = K_NVLS;
      {
        const char* u = getenv("LZ_NVLS_UNROLL");
        const char* a = getenv("LZ_NVLS_BF16_ACC");
        P.p.c = u ? (size_t)atoi(u) : (size_t)nvls_unroll;
        P.p.d = (a && atoi(a) == 0) ? 1 : 0;
      }
      P.G = grid((size_t)nthreads * kUnroll);
      P.p.a = in_off;
      P.p.b = out_off;
      P.p.i0 = copy_in;
      P.p.i1 = copy_out;
      break;
    }
    case LZ_ALGO_RING: {
      const size_t tile_vecs = (size_t)nthreads * 4;
      P.G = grid(tile_vecs);
      const size_t need = (size_t)P.G * kRingSlots * tile_vecs * 16;
      if (need > c->stage_bytes) {
        lz_set_error("ring stage too small (%zu > %zu)", need, c->stage_bytes);
        return LZE_ARG;
      }
      P.kind = K_RING;
      P.p.a = c->stage_off;
      P.p.b = tile_vecs;
      P.p.c = kRingReadyOff;
      P.p.d = kRingCreditOff;
      break;
    }
    case LZ_ALGO_RHD: {
      if (W & (W - 1)) {
        lz_set_error("recursive halving-doubling needs a power-of-two world size (got %d)", W);
        return LZE_ARG;
      }
      if (bytes > c->stage_bytes) {
        lz_set_error("RHD stage too small (%zu > %zu)", bytes, c->stage_bytes);
        return LZE_ARG;
      }
      P.kind = K_RHD;
      P.G = grid((size_t)nthreads);
      P.p.a = c->stage_off;
      break;
    }
    default:
      lz_set_error("unknown algo %d", algo);
      return LZE_ARG;
  }
  *plan = P;
  return LZE_OK;
}

template <int DT, int K>
static void* emu_fn() {
  return reinterpret_cast<void*>(&ar_emu_kernel<DT, K>);
}

template <int DT>
static void* kernel_ptr(int kind, bool emu) {
  switch (kind) {
#define LZ_K(k) \
  case k:       \
    return emu ? emu_fn<DT, k>() : reinterpret_cast<void*>(&ar_kernel<DT, k>);
    LZ_K(K_ONESHOT)
    LZ_K(K_TWOSHOT)
    LZ_K(K_TWOSHOT_SYM)
    LZ_K(K_NVLS)
    LZ_K(K_NVLS_ONESHOT)
    LZ_K(K_RING)
    LZ_K(K_RHD)
    LZ_K(K_BARRIER)
    LZ_K(K_LL)
#undef LZ_K
  }
  return nullptr;
}

static void* kernel_for(int dtype, int kind, bool emu) {
  switch (dtype) {
    case LZ_F32:
      return kernel_ptr<LZ_F32>(kind, emu);
    case LZ_F16:
      return kernel_ptr<LZ_F16>(kind, emu);
    default:
      return kernel_ptr<LZ_BF16>(kind, emu);
  }
}

static int plan_for(int dtype, const LzComm* c, const void* in, void* out, size_t count, int algo,
                    int nblocks, int nthreads, ArPlan* plan) {
  switch (dtype) {
    case LZ_F32:
      return plan_allreduce<LZ_F32>(c, in, out, count, algo, nblocks, nthreads, plan);
    case LZ_F16:
      return plan_allreduce<LZ_F16>(c, in, out, count, algo, nblocks, nthreads, plan);
    case LZ_BF16:
      return plan_allreduce<LZ_BF16>(c, in, out, count, algo, nblocks, nthreads, plan);
    default:
      lz_set_error("unsupported dtype %d", dtype);
      return LZE_ARG;
  }
}

extern "C" int lz_allreduce(LzComm* c, const void* in, void* out, size_t count, int dtype,
                            int algo, int nblocks, int nthreads, cudaStream_t s) {
  if (c->dev.world == 1) {
    const size_t es = dtype == LZ_F32 ? 4 : 2;
    const size_t bytes = count * es;
    if (in != out && bytes) {
      const bool al = ((uintptr_t)in % 16 == 0) && ((uintptr_t)out % 16 == 0);
      if (!al) {
        LZ_CUDA_TRY(cudaMemcpyAsync(out, in, bytes, cudaMemcpyDeviceToDevice, s));
      } else {
        int G = clamp_int((long long)((bytes / 16 + 2047) / 2048), 1, c->sm_count * 4);
        local_copy_kernel<<<G, 512, 0, s>>>(static_cast<const char*>(in), static_cast<char*>(out), bytes);
        LZ_CUDA_TRY(cudaGetLastError());
      }
    }
    return LZE_OK;
  }
  ArPlan P;
  int rc = plan_for(dtype, c, in, out, count, algo, nblocks, nthreads, &P);
  if (rc) return rc;
  void* fn = kernel_for(dtype, P.kind, false);
  void* args[] = {&c->dev, &P.p};
  LZ_CUDA_TRY(cudaLaunchKernel(fn, dim3(P.G), dim3(P.nthreads), args, 0, s));
  return LZE_OK;
}

extern "C" int lz_barrier(LzComm* c, cudaStream_t s) {
  if (c->dev.world == 1) return LZE_OK;
  ArParams p;
  memset(&p, 0, sizeof(p));
  void* args[] = {&c->dev, &p};
  LZ_CUDA_TRY(cudaLaunchKernel(kernel_for(LZ_BF16, K_BARRIER, false), dim3(1), dim3(32), args, 0, s));
  return LZE_OK;
}

// ----------------------------------------------------------------------------
// Single-GPU emulation of R ranks (testing only): R heaps in one device, one
// cooperative launch of grid (G, R).
// ----------------------------------------------------------------------------
struct LzEmu {
  int R;
  size_t heap_bytes;
  char* heaps[LZ_MAX_RANKS];
  LzComm comms[LZ_MAX_RANKS];
  LzDevComm* d_comms;
  ArParams* d_params;
};

extern "C" int lz_emu_create(int R, size_t heap_bytes, size_t oneshot_bytes, size_t stage_bytes,
                             double timeout_s, LzEmu** out) {
  if (R < 1 || R > LZ_MAX_RANKS) {
    lz_set_error("emulated world size must be 1..%d", LZ_MAX_RANKS);
    return LZE_ARG;
  }
  int dev = 0;
  LZ_CUDA_TRY(cudaGetDevice(&dev));
  LzEmu* e = new LzEmu();
  e->R = R;
  e->heap_bytes = heap_bytes;
  for (int r = 0; r < R; ++r) {
    LZ_CUDA_TRY(cudaMalloc(&e->heaps[r], heap_bytes));
    LZ_CUDA_TRY(cudaMemset(e->heaps[r], 0, heap_bytes));
  }
  for (int r = 0; r < R; ++r) {
    LzComm* c = &e->comms[r];
    c->heap = nullptr;
    c->heap_bytes = heap_bytes;
    memset(&c->dev, 0, sizeof(c->dev));
    c->dev.rank = r;
    c->dev.world = R;
    for (int q = 0; q < R; ++q) c->dev.heap[q] = e->heaps[q];
    c->dev.heap_mc = nullptr;
    int rc = init_comm_state(c, dev, oneshot_bytes, stage_bytes, timeout_s);
    if (rc) return rc;
  }
  LZ_CUDA_TRY(cudaMalloc(&e->d_comms, sizeof(LzDevComm) * LZ_MAX_RANKS));
  LZ_CUDA_TRY(cudaMalloc(&e->d_params, 4096));  // also used by other emulated kernels
  LzDevComm hc[LZ_MAX_RANKS];
  for (int r = 0; r < R; ++r) hc[r] = e->comms[r].dev;
  LZ_CUDA_TRY(cudaMemcpy(e->d_comms, hc, sizeof(LzDevComm) * R, cudaMemcpyHostToDevice));
  LZ_CUDA_TRY(cudaDeviceSynchronize());
  *out = e;
  return LZE_OK;
}

extern "C" int lz_emu_destroy(LzEmu* e) {
  if (!e) return LZE_OK;
  cudaDeviceSynchronize();
  for (int r = 0; r < e->R; ++r) {
    free_comm_state(&e->comms[r]);
    cudaFree(e->heaps[r]);
  }
  cudaFree(e->d_comms);
  cudaFree(e->d_params);
  delete e;
  return LZE_OK;
}

extern "C" void* lz_emu_heap_ptr(LzEmu* e, int r) { return e->heaps[r]; }
extern "C" size_t lz_emu_user_offset(LzEmu* e) { return e->comms[0].user_off; }
extern "C" int lz_emu_status(LzEmu* e, int r) {
  return *reinterpret_cast<volatile int*>(e->comms[r].status_host);
}
LzComm* lz_emu_comm(LzEmu* e, int r) { return &e->comms[r]; }
LzDevComm* lz_emu_dev_comms(LzEmu* e) { return e->d_comms; }
int lz_emu_world(LzEmu* e) { return e->R; }
void* lz_emu_param_buffer(LzEmu* e) { return e->d_params; }

extern "C" int lz_emu_allreduce(LzEmu* e, const void* const* ins, void* const* outs, size_t count,
                                int dtype, int algo, int nblocks, int nthreads, cudaStream_t s) {
  const int R = e->R;
  ArPlan plans[LZ_MAX_RANKS];
  ArParams hp[LZ_MAX_RANKS];
  for (int r = 0; r < R; ++r) {
    int rc = plan_for(dtype, &e->comms[r], ins[r], outs[r], count, algo, nblocks, nthreads, &plans[r]);
    if (rc) return rc;
    if (plans[r].kind != plans[0].kind || plans[r].G != plans[0].G) {
      lz_set_error("emulated ranks planned different launches");
      return LZE_STATE;
    }
    hp[r] = plans[r].p;
  }
  void* fn = kernel_for(dtype, plans[0].kind, true);
  int per_sm = 0;
  LZ_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, plans[0].nthreads, 0));
  const long long cap = (long long)per_sm * e->comms[0].sm_count;
  if ((long long)plans[0].G * R > cap) {
    lz_set_error("emulation grid %d x %d exceeds co-residency (%lld blocks); pass fewer blocks",
                 plans[0].G, R, cap);
    return LZE_ARG;
  }
  LZ_CUDA_TRY(cudaMemcpyAsync(e->d_params, hp, sizeof(ArParams) * R, cudaMemcpyHostToDevice, s));
  void* args[] = {&e->d_comms, &e->d_params};
  LZ_CUDA_TRY(cudaLaunchCooperativeKernel(fn, dim3(plans[0].G, R), dim3(plans[0].nthreads), args, 0, s));
  LZ_CUDA_TRY(cudaStreamSynchronize(s));  // hp lives on this stack frame
  return LZE_OK;
}

// ----------------------------------------------------------------------------
// Test hook: one block waits on a local flag word that nothing sets, with the
// communicator's bounded wait. The kernel must give up after timeout_ns and
// report LZ_ERR_TIMEOUT through the host-mapped status word; the context
// stays usable. No other rank is involved.
// ----------------------------------------------------------------------------
namespace {
__global__ void wait_never_set_kernel(LzDevComm c, unsigned long long* flag) {
  if (threadIdx.x == 0) lz_wait_ge(c, flag, 1ull, 9, c.rank);
}
}  // namespace

extern "C" int lz_test_wait_timeout(LzComm* c, double timeout_s, cudaStream_t s) {
  LzDevComm d = c->dev;
  d.timeout_ns = (unsigned long long)(timeout_s * 1e9);
  // a flag word in the reserved part of this rank's flag area, zeroed here
  unsigned long long* flag = reinterpret_cast<unsigned long long*>(c->dev.heap[c->dev.rank] + (512u << 10));
  LZ_CUDA_TRY(cudaMemsetAsync(flag, 0, 8, s));
  wait_never_set_kernel<<<1, 32, 0, s>>>(d, flag);
  LZ_CUDA_TRY(cudaGetLastError());
  return LZE_OK;
}
