// RL weight-update transfer: one sender (the trainer rank) to one or more
// receivers (inference ranks), tensor by tensor, split+rANS encoded or raw.
//
// One persistent launch per bucket on every participating rank. The bucket is
// a table of table-group (TG) descriptors; CTA b handles TGs b, b+G, ...
// Receivers hold K slots per CTA; the sender waits for a slot's credit from
// every receiver, encodes the TG (or takes it raw), publishes the record and
// raises the receivers' ready flag; receivers decode into their destination
// tensors and return the credit. When every rank receives, records and ready
// flags go out with NVLS multimem.st (one store reaches all GPUs through the
// switch); otherwise with peer stores. Flags carry (sequence << 32 | item+1)
// with a sequence number per (sender, receiver) pair (or per sender for
// all-rank broadcasts), so different calls never satisfy each other's waits.
//
// Reference behaviour being re-designed: the per-tensor NCCL broadcast of
// back_up/update_weight_from_distributed.py:422-449 and the UCCL-P2P
// split/encode sends whose logs and CSVs the reference keeps
// (raw/bf16_split_sm16_split_encode_time_count.txt, csv/weight_update_rl_GLM4_9B.csv).
#include <stdlib.h>

#include "lz_codec_dev.cuh"
#include "lz_internal.h"

using namespace lzc;
using namespace lzg;

namespace {

constexpr size_t kReadyP = 65536;    // [src][block] ready flags, point-to-point calls
constexpr size_t kReadyB = 98304;    // [src][block] ready flags, all-rank broadcasts
constexpr size_t kCreditP = 131072;  // [block][receiver] credits, point-to-point calls
constexpr size_t kCreditB = 163840;  // [block][receiver] credits, all-rank broadcasts

struct WxDesc {
  char* ptr;        // sender: source bytes; receiver: destination bytes
  uint32_t n;       // elements
  uint8_t dtype;    // LZ dtype code
  uint8_t encode;   // 0: raw bytes; 1: split + rANS record; 2: split + PACK record
  uint16_t pad;
};
static_assert(sizeof(WxDesc) == 16, "descriptor layout");

struct WxParams {
  const WxDesc* descs;
  uint32_t ntg;
  int role;          // 0 sender, 1 receiver
  int src;
  uint32_t recv_mask;
  int use_mc;
  int kslots;
  int group;         // table groups per work item (one flag round trip per item)
  int stage_local;   // encode records locally and push them, even to a single receiver
  uint32_t cap;
  size_t slots_off;
  size_t ready_off;
  size_t credit_off;
  unsigned long long seq[LZ_MAX_RANKS];  // sender: per receiver; receiver: seq[0]
};

union WxSmem {
  EncSmem enc;
  DecSmem dec;
};

LZ_DEV int es_of(int dt) { return dt == LZ_F32 ? 4 : (dt == LZ_U8 ? 1 : 2); }  // pairs: 2

// Byte copy of `bytes` from src to dst (16-B aligned both); the tail < 16 B is
// assembled in a register and stored as one vector (dst capacity allows it).
template <bool kMc>
LZ_DEV void push_bytes(const LzDevComm& c, char* dst, const char* src, uint32_t bytes) {
  if (!lz_range_ok(c, dst, (bytes + 15u) & ~15u, 20)) return;
  const uint32_t full = bytes & ~15u;
  constexpr int U = 8;  // loads in flight per thread
  uint32_t o = threadIdx.x * 16;
  for (; o + (U - 1) * blockDim.x * 16 < full; o += U * blockDim.x * 16) {
    uint4 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) v[u] = ld_cg_v4(src + o + u * blockDim.x * 16);
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (kMc) multimem_st_v4(dst + o + u * blockDim.x * 16, v[u]);
      else st_v4(dst + o + u * blockDim.x * 16, v[u]);
    }
  }
  for (; o < full; o += blockDim.x * 16) {
    const uint4 v = ld_cg_v4(src + o);
    if (kMc) multimem_st_v4(dst + o, v);
    else st_v4(dst + o, v);
  }
  if (threadIdx.x == 0 && full < bytes) {
    uint4 v = make_uint4(0, 0, 0, 0);
    uint8_t* vb = reinterpret_cast<uint8_t*>(&v);
    for (uint32_t k = 0; k < bytes - full; ++k) vb[k] = ld_cg_u8(src + full + k);
    if (kMc) multimem_st_v4(dst + full, v);
    else st_v4(dst + full, v);
  }
}

// Records are encoded at the kernel's level LV (one instantiation per level,
// chosen by the host from the engine's mode).
template <int LV>
LZ_DEV uint32_t encode_dispatch(int dt, const char* in, uint32_t n, char* dst, EncSmem& sm) {
  switch (dt) {
    case LZ_F32:
      return encode_tg<DT_F32>(in, n, dst, sm, LV);
    case LZ_F16:
      return encode_tg<DT_F16>(in, n, dst, sm, LV);
    case LZ_BF16:
      return encode_tg<DT_BF16>(in, n, dst, sm, LV);
    case DT_E4M3P:
      return encode_tg<DT_E4M3P>(in, n, dst, sm, LV);
    case DT_E5M2P:
      return encode_tg<DT_E5M2P>(in, n, dst, sm, LV);
    default:
      return encode_tg<DT_U8>(in, n, dst, sm, LV);
  }
}

LZ_DEV bool decode_dispatch(int dt, const char* rec, uint32_t cap, uint32_t n, char* out, DecSmem& sm) {
  switch (dt) {
    case LZ_F32:
      return decode_tg<DT_F32>(rec, cap, n, out, sm);
    case LZ_F16:
      return decode_tg<DT_F16>(rec, cap, n, out, sm);
    case LZ_BF16:
      return decode_tg<DT_BF16>(rec, cap, n, out, sm);
    case DT_E4M3P:
      return decode_tg<DT_E4M3P>(rec, cap, n, out, sm);
    case DT_E5M2P:
      return decode_tg<DT_E5M2P>(rec, cap, n, out, sm);
    default:
      return decode_tg<DT_U8>(rec, cap, n, out, sm);
  }
}

template <int LV>
__device__ __forceinline__ void wx_body(const LzDevComm& c, const WxParams& p) {
  extern __shared__ __align__(16) char smem_raw[];
  WxSmem& sm = *reinterpret_cast<WxSmem*>(smem_raw);
  const int W = c.world, me = c.rank, G = gridDim.x, b = blockIdx.x;
  const int K = p.kslots;
  __shared__ int s_fail;
  if (threadIdx.x == 0) s_fail = 0;
  __syncthreads();
  int nrecv = 0, only = -1;
  for (int r = 0; r < W; ++r)
    if ((p.recv_mask >> r) & 1u) {
      ++nrecv;
      only = r;
    }

  if (p.role == 0) {
    // ---------------------------------------------------------------- sender
    // item i of CTA b = table groups [(b + i*G) * g, (b + i*G) * g + g)
    const uint32_t g = (uint32_t)p.group;
    const uint32_t nitems = (p.ntg + g - 1) / g;
    for (uint32_t i = 0; b + (uint64_t)i * G < nitems; ++i) {
      const uint32_t item = b + i * G;
      const uint32_t k = i % K;
      const int t_r = threadIdx.x;
      // first K items: the receiver's CTA b has started this transfer (so its
      // previous transfer, stream-ordered before it, no longer reads any
      // slot); later items: slot k was drained K items ago
      if (t_r < W && ((p.recv_mask >> t_r) & 1u)) {
        const unsigned long long* cr = reinterpret_cast<const unsigned long long*>(
            c.heap[me] + p.credit_off) + (size_t)b * LZ_MAX_RANKS + t_r;
        const unsigned long long need = p.seq[t_r] | (i >= (uint32_t)K ? (unsigned long long)(i - K + 1) : 0ull);
        if (!lz_wait_ge(c, cr, need, 5, t_r)) s_fail = 1;
      }
      __syncthreads();
      if (s_fail) return;
      for (uint32_t j = 0; j < g && item * g + j < p.ntg; ++j) {
        const WxDesc d = p.descs[item * g + j];
        const size_t slot_off = p.slots_off + (((size_t)b * K + k) * g + j) * p.cap;
        char* local = c.heap[me] + slot_off;
        const int es = es_of(d.dtype);
        if (d.encode) {
          // one receiver: encode straight into its slot, unless the records are
          // staged locally and pushed as 16-byte vectors (p.stage_local)
          const bool direct = !p.use_mc && nrecv == 1 && !p.stage_local;
          char* dst = direct ? c.heap[only] + slot_off : local;
          if (!lz_range_ok(c, dst, p.cap, 21)) return;
          const uint32_t bytes = encode_dispatch<LV>(d.dtype, d.ptr, d.n, dst, sm.enc);
          if (p.use_mc) {
            push_bytes<true>(c, c.heap_mc + slot_off, local, pad16(bytes));
          } else if (!direct) {
            for (int r = 0; r < W; ++r)
              if ((p.recv_mask >> r) & 1u) push_bytes<false>(c, c.heap[r] + slot_off, local, pad16(bytes));
          }
        } else {
          const uint32_t bytes = d.n * (uint32_t)es;
          if (p.use_mc) {
            push_bytes<true>(c, c.heap_mc + slot_off, d.ptr, bytes);
          } else {
            for (int r = 0; r < W; ++r)
              if ((p.recv_mask >> r) & 1u) push_bytes<false>(c, c.heap[r] + slot_off, d.ptr, bytes);
          }
        }
      }
      publish_block_writes(c);
      if (p.use_mc) {
        if (threadIdx.x == 0) {
          fence_sys();
          unsigned long long* f = reinterpret_cast<unsigned long long*>(c.heap_mc + p.ready_off) +
                                  (size_t)p.src * LZ_MAX_BLOCKS + b;
          multimem_st_release_u64(f, p.seq[0] | (unsigned long long)(i + 1));
        }
      } else if (t_r < W && ((p.recv_mask >> t_r) & 1u)) {
        unsigned long long* f = reinterpret_cast<unsigned long long*>(c.heap[t_r] + p.ready_off) +
                                (size_t)p.src * LZ_MAX_BLOCKS + b;
        st_release_sys(f, p.seq[t_r] | (unsigned long long)(i + 1));
      }
    }
  } else {
    // -------------------------------------------------------------- receiver
    const unsigned long long* ready = reinterpret_cast<const unsigned long long*>(
        c.heap[me] + p.ready_off) + (size_t)p.src * LZ_MAX_BLOCKS + b;
    unsigned long long* credit = reinterpret_cast<unsigned long long*>(c.heap[p.src] + p.credit_off) +
                                 (size_t)b * LZ_MAX_RANKS + me;
    const uint32_t g = (uint32_t)p.group;
    const uint32_t nitems = (p.ntg + g - 1) / g;
    if (threadIdx.x == 0 && b < nitems) {
      st_release_sys(credit, p.seq[0]);  // started: the sender may fill the slots
    }
    for (uint32_t i = 0; b + (uint64_t)i * G < nitems; ++i) {
      const uint32_t item = b + i * G;
      const uint32_t k = i % K;
      if (threadIdx.x == 0 && !lz_wait_ge(c, ready, p.seq[0] | (unsigned long long)(i + 1), 6, p.src))
        s_fail = 1;
      __syncthreads();
      if (s_fail) return;
      if (threadIdx.x == 0 && p.use_mc) fence_proxy_alias();
      __syncthreads();
      for (uint32_t j = 0; j < g && item * g + j < p.ntg; ++j) {
        const WxDesc d = p.descs[item * g + j];
        const char* slot = c.heap[me] + p.slots_off + (((size_t)b * K + k) * g + j) * p.cap;
        if (d.encode) {
          if (!decode_dispatch(d.dtype, slot, p.cap, d.n, d.ptr, sm.dec)) {
            if (threadIdx.x == 0) lz_report(c, LZ_ERR_CORRUPT, 7, p.src);
            return;
          }
        } else {
          const uint32_t bytes = d.n * (uint32_t)es_of(d.dtype);
          const uint32_t full = bytes & ~15u;
          uint32_t o = threadIdx.x * 16;
          for (; o + 3 * blockDim.x * 16 < full; o += 4 * blockDim.x * 16) {
            uint4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) v[u] = ld_cg_v4(slot + o + u * blockDim.x * 16);
#pragma unroll
            for (int u = 0; u < 4; ++u) st_v4(d.ptr + o + u * blockDim.x * 16, v[u]);
          }
          for (; o < full; o += blockDim.x * 16) st_v4(d.ptr + o, ld_cg_v4(slot + o));
          if (threadIdx.x < bytes - full) d.ptr[full + threadIdx.x] = (char)ld_cg_u8(slot + full + threadIdx.x);
        }
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        st_release_sys(credit, p.seq[0] | (unsigned long long)(i + 1));
      }
    }
  }
}

template <int LV>
__global__ void __launch_bounds__(LZC_THREADS, LZC_MIN_BLOCKS) wx_kernel(LzDevComm c, WxParams p) {
  wx_body<LV>(c, p);
}
// flags bit 1: records at the PACK level
void* wx_fn(int flags) {
  return (flags & 2) ? reinterpret_cast<void*>(&wx_kernel<LEVEL_PACK>) : reinterpret_cast<void*>(&wx_kernel<LEVEL_ANS>);
}

}  // namespace

extern "C" size_t lz_wx_slot_capacity(void) { return tg_capacity(LZ_F32); }
extern "C" size_t lz_wx_tg_elems(void) { return TG_ELEMS; }

// Stage bytes needed for `nblocks` CTAs with `kslots` slots each.
extern "C" size_t lz_wx_stage_bytes(int nblocks, int kslots) {
  return (size_t)nblocks * kslots * tg_capacity(LZ_F32);
}

// Table groups per work item used by lz_weight_transfer (env LZ_WX_GROUP, default 4).
static int wx_group() {
  const char* e = getenv("LZ_WX_GROUP");
  const int g = e ? atoi(e) : 4;
  return g < 1 ? 1 : (g > 16 ? 16 : g);
}
extern "C" int lz_wx_group(void) { return wx_group(); }

// role 0 = sender (seq[r] per receiver r), 1 = receiver (seq[0]).
// descs: device array of 16-byte descriptors (ptr, n, dtype, encode).
static int wx_plan(const LzComm* c, int role, int src, unsigned int recv_mask, const void* descs,
                   unsigned int ntg, int nblocks, int kslots, int broadcast_all,
                   const unsigned long long* seqs, WxParams* out, int* grid) {
  const int W = c->dev.world;
  if (src < 0 || src >= W || (recv_mask >> src) & 1u || recv_mask == 0 ||
      (recv_mask >> W) != 0u) {
    lz_set_error("weight transfer: bad src %d / receiver mask 0x%x", src, recv_mask);
    return LZE_ARG;
  }
  int G = nblocks > 0 ? nblocks : c->sm_count * 3;
  if (G > LZ_MAX_BLOCKS) G = LZ_MAX_BLOCKS;
  if (kslots < 2) kslots = 2;
  WxParams p;
  memset(&p, 0, sizeof(p));
  p.descs = static_cast<const WxDesc*>(descs);
  p.ntg = ntg;
  p.role = role;
  p.src = src;
  p.recv_mask = recv_mask;
  const bool all = (broadcast_all & 1) && recv_mask == (((1u << W) - 1u) & ~(1u << src));
  // one receiver: direct peer stores beat a multicast write that also lands locally
  p.use_mc = (all && W > 2 && c->dev.heap_mc) ? 1 : 0;
  p.kslots = kslots;
  p.cap = tg_capacity(LZ_F32);
  p.slots_off = c->stage_off;
  p.group = wx_group();
  {
    // diagnostic: LZ_WX_STAGE_LOCAL=1 encodes a single receiver's records
    // locally and pushes them as vectors instead of encoding into its slot
    static const char* e = getenv("LZ_WX_STAGE_LOCAL");
    p.stage_local = e ? atoi(e) : 0;
  }
  if (lz_wx_stage_bytes(G, kslots) * p.group > c->stage_bytes) {
    lz_set_error("weight transfer: %d blocks x %d slots x %d groups need %zu stage bytes, have %zu", G,
                 kslots, p.group, lz_wx_stage_bytes(G, kslots) * p.group, c->stage_bytes);
    return LZE_ARG;
  }
  p.ready_off = all ? kReadyB : kReadyP;
  p.credit_off = all ? kCreditB : kCreditP;
  for (int r = 0; r < LZ_MAX_RANKS; ++r) p.seq[r] = seqs[r] << 32;
  *out = p;
  *grid = G;
  return LZE_OK;
}

// broadcast_all: bit 0 every rank but src receives (multicast when possible),
// bit 1 encoded records use the codec's PACK level (else rANS).
extern "C" int lz_weight_transfer(LzComm* c, int role, int src, unsigned int recv_mask,
                                  const void* descs, unsigned int ntg, int nblocks, int kslots,
                                  int broadcast_all, const unsigned long long* seqs, cudaStream_t s) {
  if (c->dev.world == 1 || ntg == 0) return LZE_OK;
  WxParams p;
  int G = 0;
  int rc = wx_plan(c, role, src, recv_mask, descs, ntg, nblocks, kslots, broadcast_all, seqs, &p, &G);
  if (rc) return rc;
  const size_t smem = sizeof(WxSmem);
  void* fn = wx_fn(broadcast_all);
  LZ_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  void* args[] = {&c->dev, &p};
  LZ_CUDA_TRY(cudaLaunchKernel(fn, dim3(G), dim3(LZC_THREADS), args, smem, s));
  return LZE_OK;
}

// Single-GPU emulation of one transfer: block (x, y) is CTA x of emulated
// rank y, all in ONE cooperative launch; ranks that neither send nor receive
// idle. descs[r]: device descriptor table of rank r; seqs: R x 8 values.
namespace {
template <int LV>
__global__ void __launch_bounds__(LZC_THREADS, 2) wx_emu_kernel(const LzDevComm* cs, const WxParams* ps) {
  const WxParams& p = ps[blockIdx.y];
  if (p.role > 1) return;
  wx_body<LV>(cs[blockIdx.y], p);
}
}  // namespace

extern "C" int lz_emu_weight_transfer(LzEmu* e, int src, unsigned int recv_mask, const void* const* descs,
                                      unsigned int ntg, int nblocks, int kslots, int broadcast_all,
                                      const unsigned long long* seqs, cudaStream_t s) {
  const int R = lz_emu_world(e);
  WxParams hp[LZ_MAX_RANKS];
  int G = 0;
  for (int r = 0; r < R; ++r) {
    const int role = r == src ? 0 : (((recv_mask >> r) & 1u) ? 1 : 2);
    int rc = wx_plan(lz_emu_comm(e, r), role < 2 ? role : 1, src, recv_mask, descs[r], ntg, nblocks, kslots,
                     broadcast_all, seqs + 8 * r, &hp[r], &G);
    if (rc) return rc;
    hp[r].role = role;
  }
  const size_t smem = sizeof(WxSmem);
  void* fn = (broadcast_all & 2) ? reinterpret_cast<void*>(&wx_emu_kernel<LEVEL_PACK>)
                                 : reinterpret_cast<void*>(&wx_emu_kernel<LEVEL_ANS>);
  LZ_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  int per_sm = 0;
  LZ_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, LZC_THREADS, smem));
  if ((long long)G * R > (long long)per_sm * lz_emu_comm(e, 0)->sm_count) {
    lz_set_error("emulated weight transfer: %d x %d blocks exceed co-residency", G, R);
    return LZE_ARG;
  }
  static_assert(sizeof(WxParams) * LZ_MAX_RANKS <= 4096, "param buffer");
  void* dparams = lz_emu_param_buffer(e);
  LZ_CUDA_TRY(cudaMemcpyAsync(dparams, hp, sizeof(WxParams) * R, cudaMemcpyHostToDevice, s));
  LzDevComm* dcomms = lz_emu_dev_comms(e);
  void* args[] = {&dcomms, &dparams};
  LZ_CUDA_TRY(cudaLaunchCooperativeKernel(fn, dim3(G, R), dim3(LZC_THREADS), args, smem, s));
  LZ_CUDA_TRY(cudaStreamSynchronize(s));
  return LZE_OK;
}

// ----------------------------------------------------------------------------
// Zero-copy raw transfer into symmetric destinations. Receivers' tensors live
// in the symmetric heap at the same offsets on every rank, so the sender
// writes each table group straight into every receiver's tensor: one
// multimem.st per 16 bytes through the switch when every other rank receives,
// peer stores otherwise. No slots, credits or receiver copies; each sender
// CTA raises one completion flag per receiver at the end, and receiver CTA b
// waits for the flag of sender CTA b.
// ----------------------------------------------------------------------------
namespace {

struct WxDirectDesc {
  const char* src;  // sender: source bytes (unused on receivers)
  uint64_t dst_off; // heap offset of the destination bytes (same on every rank)
  uint64_t bytes;
  uint64_t pad;
};
static_assert(sizeof(WxDirectDesc) == 32, "direct descriptor layout");

struct WxDirectParams {
  const WxDirectDesc* descs;
  uint32_t ndesc;
  int role;
  int src;
  uint32_t recv_mask;
  int use_mc;
  size_t ready_off;
  size_t credit_off;
  unsigned long long seq[LZ_MAX_RANKS];
};

constexpr uint64_t kDirectChunk = 256u << 10;  // bytes per work item

__global__ void __launch_bounds__(256) wx_direct_kernel(LzDevComm c, WxDirectParams p) {
  const int W = c.world, G = gridDim.x, b = blockIdx.x;
  if (p.role == 0) {
    // every receiver's CTA b must have started (its earlier work on the
    // destination tensors is done, stream order) before CTA b writes
    __shared__ int s_fail;
    if (threadIdx.x == 0) s_fail = 0;
    __syncthreads();
    if (threadIdx.x < W && ((p.recv_mask >> threadIdx.x) & 1u)) {
      const unsigned long long* cr = reinterpret_cast<const unsigned long long*>(c.heap[c.rank] + p.credit_off) +
                                     (size_t)b * LZ_MAX_RANKS + threadIdx.x;
      if (!lz_wait_ge(c, cr, p.seq[threadIdx.x] | 1ull, 10, threadIdx.x)) s_fail = 1;
    }
    __syncthreads();
    if (s_fail) return;
    // work items: 256 KB chunks of every descriptor, dealt round-robin to CTAs
    uint64_t item = 0;
    for (uint32_t k = 0; k < p.ndesc; ++k) {
      const WxDirectDesc d = p.descs[k];
      const uint64_t nchunks = (d.bytes + kDirectChunk - 1) / kDirectChunk;
      for (uint64_t ch = 0; ch < nchunks; ++ch, ++item) {
        if (item % G != (uint64_t)b) continue;
        const uint64_t off = ch * kDirectChunk;
        const uint32_t len = (uint32_t)min(kDirectChunk, d.bytes - off);
        if (p.use_mc) {
          push_bytes<true>(c, c.heap_mc + d.dst_off + off, d.src + off, len);  // every rank, sender included
        } else {
          for (int r = 0; r < W; ++r)
            if (((p.recv_mask >> r) & 1u) || r == c.rank)
              push_bytes<false>(c, c.heap[r] + d.dst_off + off, d.src + off, len);
        }
      }
    }
    publish_block_writes(c);
    const int t = threadIdx.x;
    if (t < W && ((p.recv_mask >> t) & 1u)) {
      unsigned long long* f = reinterpret_cast<unsigned long long*>(c.heap[t] + p.ready_off) +
                              (size_t)p.src * LZ_MAX_BLOCKS + b;
      st_release_sys(f, p.seq[t] | 1ull);
    }
  } else {
    if (threadIdx.x == 0) {
      unsigned long long* cr = reinterpret_cast<unsigned long long*>(c.heap[p.src] + p.credit_off) +
                               (size_t)b * LZ_MAX_RANKS + c.rank;
      st_release_sys(cr, p.seq[0] | 1ull);  // clear to send
      const unsigned long long* f = reinterpret_cast<const unsigned long long*>(c.heap[c.rank] + p.ready_off) +
                                    (size_t)p.src * LZ_MAX_BLOCKS + b;
      lz_wait_ge(c, f, p.seq[0] | 1ull, 8, p.src);
      fence_proxy_alias();
    }
  }
}

}  // namespace

extern "C" int lz_weight_transfer_direct(LzComm* c, int role, int src, unsigned int recv_mask,
                                         const void* descs, unsigned int ndesc, int nblocks,
                                         int broadcast_all, const unsigned long long* seqs,
                                         cudaStream_t s) {
  const int W = c->dev.world;
  if (W == 1 || ndesc == 0) return LZE_OK;
  if (src < 0 || src >= W || (recv_mask >> src) & 1u || recv_mask == 0 || (recv_mask >> W) != 0u) {
    lz_set_error("direct weight transfer: bad src %d / receiver mask 0x%x", src, recv_mask);
    return LZE_ARG;
  }
  int G = nblocks > 0 ? nblocks : c->sm_count * 2;
  if (G > LZ_MAX_BLOCKS) G = LZ_MAX_BLOCKS;
  WxDirectParams p;
  memset(&p, 0, sizeof(p));
  p.descs = static_cast<const WxDirectDesc*>(descs);
  p.ndesc = ndesc;
  p.role = role;
  p.src = src;
  p.recv_mask = recv_mask;
  const bool all = broadcast_all && recv_mask == (((1u << W) - 1u) & ~(1u << src));
  p.use_mc = (all && W > 2 && c->dev.heap_mc) ? 1 : 0;
  p.ready_off = all ? kReadyB : kReadyP;
  p.credit_off = all ? kCreditB : kCreditP;
  for (int r = 0; r < LZ_MAX_RANKS; ++r) p.seq[r] = seqs[r] << 32;
  wx_direct_kernel<<<G, 256, 0, s>>>(c->dev, p);
  LZ_CUDA_TRY(cudaGetLastError());
  return LZE_OK;
}

// ----------------------------------------------------------------------------
// Relay broadcast into symmetric destinations (every other rank receives).
// A broadcast is bound by each receiver's NVLink ingress (every receiver must
// take in all the bytes), not by the sender's egress, so the sender should not
// be the only GPU that sends. The bytes are cut into 256 KB chunks, dealt to
// CTAs round-robin; round t of CTA b is owned by rank (b + t) % W. The sender
// multicasts the chunks it owns itself; a chunk owned by rank o goes to o
// alone with peer stores, and o then forwards it from its own copy to every
// other rank (one multimem.st through the switch, or peer stores). Every
// rank's egress is then ~1/W of the bytes (the sender's ~all of them once),
// and every receiver takes in each byte once.
// CTA b of all ranks meets in an all-pairs barrier before its first store
// (every rank has started, so earlier stream work on the destinations is
// done) and after its last one (every chunk of CTA b has landed everywhere).
// Flags live in per-sender regions so calls from different senders never mix.
// ----------------------------------------------------------------------------
namespace {

constexpr size_t kRelayBar = 196608;           // [src] x [block][rank] u64 barrier flags
constexpr size_t kRelayBarStride = 32768;
constexpr size_t kRelayReady = 458752;          // [src] x [block] u64 chunk-ready flags (owner's heap)
constexpr size_t kRelayReadyStride = 4096;
static_assert(kRelayBar + LZ_MAX_RANKS * kRelayBarStride <= kRelayReady, "relay flag regions overlap");
static_assert(kRelayReady + LZ_MAX_RANKS * kRelayReadyStride <= (512u << 10), "relay flags reach the test word");

struct WxRelayParams {
  const WxDirectDesc* descs;
  uint32_t ndesc;
  int src;
  int use_mc;
  unsigned long long seq;  // sequence << 32
};

// All-pairs meeting of CTA b of every rank at value v (per-sender region).
LZ_DEV bool relay_barrier(const LzDevComm& c, size_t bar_off, unsigned long long v, int phase) {
  __shared__ int s_fail_rb;
  if (threadIdx.x == 0) s_fail_rb = 0;
  publish_block_writes(c);
  const int t = threadIdx.x;
  if (t < c.world && t != c.rank) {
    unsigned long long* mine = reinterpret_cast<unsigned long long*>(c.heap[t] + bar_off) +
                               (size_t)blockIdx.x * LZ_MAX_RANKS + c.rank;
    st_release_sys(mine, v);
    const unsigned long long* theirs = reinterpret_cast<const unsigned long long*>(c.heap[c.rank] + bar_off) +
                                       (size_t)blockIdx.x * LZ_MAX_RANKS + t;
    if (!lz_wait_ge(c, theirs, v, phase, t)) s_fail_rb = 1;
  }
  __syncthreads();
  return s_fail_rb == 0;
}

// Peer stores of `len` bytes at heap offset `off` to every rank but `skip`
// (and but this rank when `src` is this rank's own copy).
LZ_DEV void relay_push_p2p(const LzDevComm& c, uint64_t off, const char* src, uint32_t len, int skip) {
  for (int r = 0; r < c.world; ++r) {
    if (r == skip) continue;
    char* dst = c.heap[r] + off;
    if (dst == src) continue;
    push_bytes<false>(c, dst, src, len);
  }
}

__device__ __forceinline__ void wx_relay_body(const LzDevComm& c, const WxRelayParams& p) {
  const int W = c.world, me = c.rank, G = gridDim.x, b = blockIdx.x;
  const size_t bar_off = kRelayBar + (size_t)p.src * kRelayBarStride;
  const size_t rdy_off = kRelayReady + (size_t)p.src * kRelayReadyStride;
  if (!relay_barrier(c, bar_off, p.seq | 1ull, 11)) return;
  __shared__ int s_fail;
  if (threadIdx.x == 0) s_fail = 0;
  __syncthreads();
  uint64_t item = 0;
  uint32_t t = 0;  // round of this CTA
  for (uint32_t k = 0; k < p.ndesc; ++k) {
    const WxDirectDesc d = p.descs[k];
    const uint64_t nchunks = (d.bytes + kDirectChunk - 1) / kDirectChunk;
    for (uint64_t ch = 0; ch < nchunks; ++ch, ++item) {
      if (item % G != (uint64_t)b) continue;
      const uint32_t round = t++;
      const int owner = (int)((b + round) % (uint32_t)W);
      const uint64_t off = ch * kDirectChunk;
      const uint32_t len = (uint32_t)min(kDirectChunk, d.bytes - off);
      const uint64_t hoff = d.dst_off + off;
      if (me == p.src) {
        if (owner == me) {
          if (p.use_mc) push_bytes<true>(c, c.heap_mc + hoff, d.src + off, len);
          else relay_push_p2p(c, hoff, d.src + off, len, -1);
        } else {
          push_bytes<false>(c, c.heap[owner] + hoff, d.src + off, len);
          publish_block_writes(c);
          if (threadIdx.x == 0) {
            unsigned long long* f = reinterpret_cast<unsigned long long*>(c.heap[owner] + rdy_off) + b;
            st_release_sys(f, p.seq | (unsigned long long)(round + 1));
          }
        }
      } else if (owner == me) {
        if (threadIdx.x == 0) {
          const unsigned long long* f = reinterpret_cast<const unsigned long long*>(c.heap[me] + rdy_off) + b;
          if (!lz_wait_ge(c, f, p.seq | (unsigned long long)(round + 1), 12, p.src)) s_fail = 1;
        }
        __syncthreads();
        if (s_fail) return;
        const char* mine = c.heap[me] + hoff;
        if (p.use_mc) push_bytes<true>(c, c.heap_mc + hoff, mine, len);
        else relay_push_p2p(c, hoff, mine, len, me);
      }
    }
  }
  relay_barrier(c, bar_off, p.seq | 2ull, 13);
  if (p.use_mc && threadIdx.x == 0) fence_proxy_alias();
}

__global__ void __launch_bounds__(256) wx_relay_kernel(LzDevComm c, WxRelayParams p) { wx_relay_body(c, p); }

// Emulation: grid (G, R), blockIdx.y = rank; the body sees blockIdx.x only.
__global__ void __launch_bounds__(256) wx_relay_emu_kernel(const LzDevComm* cs, const WxRelayParams* ps) {
  wx_relay_body(cs[blockIdx.y], ps[blockIdx.y]);
}

int relay_plan(const LzComm* c, int src, const void* descs, unsigned int ndesc, int use_mc,
               unsigned long long seq, WxRelayParams* p) {
  const int W = c->dev.world;
  if (src < 0 || src >= W) {
    lz_set_error("relay broadcast: bad src %d", src);
    return LZE_ARG;
  }
  if (use_mc && !c->dev.heap_mc) {
    lz_set_error("relay broadcast: multicast requested but unavailable");
    return LZE_UNSUPPORTED;
  }
  memset(p, 0, sizeof(*p));
  p->descs = static_cast<const WxDirectDesc*>(descs);
  p->ndesc = ndesc;
  p->src = src;
  p->use_mc = use_mc;
  p->seq = seq << 32;
  return LZE_OK;
}

}  // namespace

// Every rank calls with the same descriptors' destination offsets (sender's
// carry the source pointers); use_mc = forward with multimem.st.
extern "C" int lz_weight_broadcast_relay(LzComm* c, int src, const void* descs, unsigned int ndesc,
                                         int nblocks, int use_mc, unsigned long long seq, cudaStream_t s) {
  if (c->dev.world == 1 || ndesc == 0) return LZE_OK;
  WxRelayParams p;
  int rc = relay_plan(c, src, descs, ndesc, use_mc, seq, &p);
  if (rc) return rc;
  int G = nblocks > 0 ? nblocks : c->sm_count * 2;
  if (G > LZ_MAX_BLOCKS) G = LZ_MAX_BLOCKS;
  wx_relay_kernel<<<G, 256, 0, s>>>(c->dev, p);
  LZ_CUDA_TRY(cudaGetLastError());
  return LZE_OK;
}

// Single-GPU emulation of the relay broadcast (peer stores only; descs[r] is
// rank r's descriptor array). Synchronous.
extern "C" int lz_emu_weight_broadcast_relay(LzEmu* e, int src, const void* const* descs, unsigned int ndesc,
                                             int nblocks, unsigned long long seq, cudaStream_t s) {
  const int R = lz_emu_world(e);
  WxRelayParams hp[LZ_MAX_RANKS];
  for (int r = 0; r < R; ++r) {
    int rc = relay_plan(lz_emu_comm(e, r), src, descs[r], ndesc, 0, seq, &hp[r]);
    if (rc) return rc;
  }
  int G = nblocks > 0 ? nblocks : 8;
  void* fn = reinterpret_cast<void*>(&wx_relay_emu_kernel);
  int per_sm = 0;
  LZ_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, 256, 0));
  if ((long long)G * R > (long long)per_sm * lz_emu_comm(e, 0)->sm_count) {
    lz_set_error("emulated relay broadcast: %d x %d blocks exceed co-residency", G, R);
    return LZE_ARG;
  }
  static_assert(sizeof(WxRelayParams) * LZ_MAX_RANKS <= 4096, "param buffer");
  void* dparams = lz_emu_param_buffer(e);
  LZ_CUDA_TRY(cudaMemcpyAsync(dparams, hp, sizeof(WxRelayParams) * R, cudaMemcpyHostToDevice, s));
  LzDevComm* dcomms = lz_emu_dev_comms(e);
  void* args[] = {&dcomms, &dparams};
  LZ_CUDA_TRY(cudaLaunchCooperativeKernel(fn, dim3(G, R), dim3(256), args, 0, s));
  LZ_CUDA_TRY(cudaStreamSynchronize(s));
  return LZE_OK;
}

// ----------------------------------------------------------------------------
// Copy-engine point-to-point transfer into a receiver's symmetric tensors.
// The bytes move by DMA (cudaMemcpyAsync into the peer's heap mapping), so no
// SM is used for the data; two one-thread kernels carry the protocol:
//   receiver: post "clear to send" (its earlier stream work on the
//             destinations is done), then wait until the sender's "ready";
//   sender:   wait for "clear to send", issue one copy per tensor on the same
//             stream, then post "ready" (stream order puts it after the copies'
//             completion, so the receiver's acquire sees the bytes).
// Flags: per (sender, receiver) pair, value = sequence number of the pair.
// ----------------------------------------------------------------------------
namespace {

constexpr size_t kCeReady = 491520;        // [src] u64 in the receiver's heap
constexpr size_t kCeCredit = 491520 + 64;  // [receiver] u64 in the sender's heap
static_assert(kCeCredit + 64 <= (512u << 10), "copy-engine flags reach the test word");
static_assert(kRelayReady + LZ_MAX_RANKS * kRelayReadyStride <= kCeReady, "copy-engine flags overlap relay flags");

__global__ void ce_signal_kernel(unsigned long long* flag, unsigned long long v) {
  st_release_sys(flag, v);
}

__global__ void ce_wait_kernel(LzDevComm c, const unsigned long long* flag, unsigned long long v, int peer) {
  lz_wait_ge(c, flag, v, 14, peer);
}

}  // namespace

// role 0: sender to `peer`; role 1: receiver from `peer`. Sender arrays (host
// memory): source pointers, destination heap offsets and sizes of n tensors.
extern "C" int lz_weight_transfer_ce(LzComm* c, int role, int peer, const unsigned long long* src_ptrs,
                                     const unsigned long long* dst_offs, const unsigned long long* sizes,
                                     unsigned int n, unsigned long long seq, cudaStream_t s) {
  const int W = c->dev.world, me = c->dev.rank;
  if (peer < 0 || peer >= W || peer == me) {
    lz_set_error("copy-engine transfer: bad peer %d", peer);
    return LZE_ARG;
  }
  if (role == 0) {
    for (unsigned int i = 0; i < n; ++i) {
      if (dst_offs[i] + sizes[i] > c->heap_bytes) {
        lz_set_error("copy-engine transfer: destination %u outside the heap", i);
        return LZE_ARG;
      }
    }
    const unsigned long long* credit =
        reinterpret_cast<const unsigned long long*>(c->dev.heap[me] + kCeCredit) + peer;
    ce_wait_kernel<<<1, 1, 0, s>>>(c->dev, credit, seq, peer);
    LZ_CUDA_TRY(cudaGetLastError());
    for (unsigned int i = 0; i < n; ++i) {
      if (!sizes[i]) continue;
      LZ_CUDA_TRY(cudaMemcpyAsync(c->dev.heap[peer] + dst_offs[i], reinterpret_cast<const void*>(src_ptrs[i]),
                                  sizes[i], cudaMemcpyDeviceToDevice, s));
    }
    unsigned long long* ready = reinterpret_cast<unsigned long long*>(c->dev.heap[peer] + kCeReady) + me;
    ce_signal_kernel<<<1, 1, 0, s>>>(ready, seq);
    LZ_CUDA_TRY(cudaGetLastError());
  } else {
    unsigned long long* credit = reinterpret_cast<unsigned long long*>(c->dev.heap[peer] + kCeCredit) + me;
    ce_signal_kernel<<<1, 1, 0, s>>>(credit, seq);
    LZ_CUDA_TRY(cudaGetLastError());
    const unsigned long long* ready = reinterpret_cast<const unsigned long long*>(c->dev.heap[me] + kCeReady) + peer;
    ce_wait_kernel<<<1, 1, 0, s>>>(c->dev, ready, seq, peer);
    LZ_CUDA_TRY(cudaGetLastError());
  }
  return LZE_OK;
}
