// Lossless compressed allreduce, fused with the NVLink transfer.
//
// One persistent launch per call: one start barrier between same-index CTAs
// of all ranks, then three phases linked by per-record flags (no barrier
// between phases, so a CTA decodes and reduces its table groups while other
// CTAs are still encoding theirs; bounded waits):
//   1. RS encode+push: every table group (TG) of every peer's slice is
//      split + encoded (rANS or PACK level) by this GPU and the record is written straight
//      into the peer's receive slot (peer stores over NVLink): only the
//      compressed bytes cross the link, no staging copy, no size exchange.
//   2. decode+reduce: the owner decodes the W-1 incoming records of each of
//      its TGs and accumulates them with its own input in fp32 in rank order
//      0..W-1 (bit-identical to an fp32 sequential reference), rounds once,
//      stores its output slice, re-encodes the reduced TG once and publishes
//      the record to every peer (NVLS multimem.st when a multicast object
//      exists: one store reaches all GPUs; else peer stores).
//   3. AG decode: every rank decodes the W-1 published records of the other
//      slices straight into its output.
// Records are never truncated: a TG that does not compress is stored RAW.
// Every slot is followed by a 16-byte footer whose first word is the slot's
// ready flag: the call epoch and chunk index mixed with a 64-bit constant, stored with release
// semantics after the CTA's record stores and matched exactly (the stage is
// shared with other algorithms, so a footer may hold stale data of any
// value; a small integer or all-zero word can never match).
// Chunks: every slice is processed in chunks of C table groups (C = all of
// them unless the caller asks for chunks); table group t (slice-local index)
// is handled by CTA t mod G on every rank in every chunk, so consecutive
// chunks smaller than the grid still spread over all CTAs; a chunked call keeps
// two chunks' slots (a ring), so its stage is bounded by the chunk size. A
// CTA starts chunk k + 2 only after the CTA that used its ring slots in chunk
// k has finished that chunk on every rank (progress words in the flag area),
// so chunks k and k + 1 are in flight together. The start
// barrier of CTA b (every rank's CTA b has finished the previous call) keeps
// a new call from overwriting slots the previous one still reads.
//
// Reference behaviour being re-designed: the compressed two-shot all-to-all
// ("LZip two-shot", single_node_nccl_allreduce_benchmark/compressed_twoshot_allreduce.py:126-247),
// which compresses with dietgpu, sends a fixed 0.65-ratio prefix with NCCL
// (silently truncating streams that do not fit, :177-178) and decompresses in
// separate launches; the compressed P2P hybrid
// (single_node_nccl_allreduce_benchmark/compressed_p2p_allreduce.py:54-188);
// and the double-buffered chunk pipeline of the compressed send/recv
// allreduce (single_node_nccl_allreduce_benchmark/compressed_sendrecv_allreduce.py:41-231),
// here a ring of two chunks' slots inside one launch.
#include "lz_codec_dev.cuh"
#include "lz_internal.h"

using namespace lzc;
using namespace lzg;

namespace {

struct CzParams {
  const char* in;
  char* out;
  uint64_t n;          // elements
  uint64_t slice;      // elements per slice (multiple of 16); slice p = [p*slice, ...)
  uint32_t ntg_max;    // TGs per slice (max)
  uint32_t cap;        // TG record capacity
  uint32_t sstride;    // slot stride: cap + 16-byte flag footer
  size_t rs_off;       // heap offset: RS slots [src][tg]
  size_t ag_off;       // heap offset: AG slots [owner][tg]
  float* acc;          // local fp32 scratch, TG_ELEMS per CTA
  int use_mc;          // publish AG records with multimem.st
  int hybrid;          // reduce-scatter moves raw bytes; only the all-gather is compressed
  int stage_local;     // RS records are encoded into local memory, then pushed as 16-byte vectors
  unsigned long long* trace;  // optional: per-CTA nanoseconds per phase [G][kCzTraceSlots]
  uint32_t chunk_tgs;  // TGs per slice per chunk (C); every slice is processed in chunks of C TGs
  uint32_t nchunks;    // ceil(ntg_max / C)
  uint32_t nslots;     // slots per source: ntg_max (one chunk) or 2 C (a ring of two chunks)
};

// Phase tracer: with a trace buffer, thread 0 of every CTA adds the
// %globaltimer nanoseconds spent in each phase to its row (added across calls).
enum CzPhase {
  CZ_T_TOTAL = 0,    // kernel start to end of the CTA
  CZ_T_BARRIER,      // start barrier
  CZ_T_RS_ENCODE,    // reduce-scatter: encode (or copy) + push of records to peers
  CZ_T_RS_WAIT,      // owner: waiting for peers' records
  CZ_T_RS_DECODE,    // owner: decoding records' symbols
  CZ_T_REDUCE,       // owner: rank-order fp32 reduction passes
  CZ_T_AG_ENCODE,    // owner: encoding the reduced table group
  CZ_T_AG_PUSH,      // owner: publishing it (peer stores or multimem) + flags
  CZ_T_AG_WAIT,      // waiting for the other owners' records
  CZ_T_AG_DECODE,    // decoding them into the output
  CZ_T_CHUNK_WAIT,   // waiting for ring slots (chunked calls)
  CZ_T_TGS,          // table groups reduced by this CTA (a count)
  kCzTraceSlots = 12
};

// Chunk progress words [LZ_MAX_BLOCKS][LZ_MAX_RANKS] in the flag area (a
// region of its own, written with monotonic values only).
constexpr size_t kCzProgOff = 576u << 10;
static_assert(kCzProgOff + (size_t)LZ_MAX_BLOCKS * LZ_MAX_RANKS * 8 <= kLzFlagsBytes,
              "compressed-allreduce progress words exceed the flag area");

union CzSmem {
  EncSmem enc;
  DecSmem dec;
};

LZ_DEV uint64_t slice_begin(const CzParams& p, int s) {
  const uint64_t b = (uint64_t)s * p.slice;
  return b < p.n ? b : p.n;
}
LZ_DEV uint64_t slice_len(const CzParams& p, int s) {
  const uint64_t b = slice_begin(p, s), e = slice_begin(p, s + 1);
  return e - b;
}
LZ_DEV uint32_t ntg_of(const CzParams& p, int s) { return (uint32_t)num_tgs(slice_len(p, s)); }

// Copies `padded` bytes (multiple of 16, both 16-B aligned) with the whole CTA,
// eight 16-byte loads in flight per thread (peer destinations).
LZ_DEV void cta_push16(char* dst, const char* src, uint32_t padded) {
  constexpr int U = 8;
  const uint32_t step = blockDim.x * 16;
  uint32_t o = threadIdx.x * 16;
  for (; o + (U - 1) * step < padded; o += U * step) {
    uint4 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) v[u] = ld_cg_v4(src + o + u * step);
#pragma unroll
    for (int u = 0; u < U; ++u) st_v4(dst + o + u * step, v[u]);
  }
  for (; o < padded; o += step) st_v4(dst + o, ld_cg_v4(src + o));
}

// Copies `bytes` from src to dst (both 16-B aligned) with the whole CTA:
// 16-byte vectors, then the last bytes one per thread (never reads past src).
LZ_DEV void cta_copy_bytes(char* dst, const char* src, uint32_t bytes) {
  const uint32_t v = bytes / 16 * 16;
  for (uint32_t o = threadIdx.x * 16; o < v; o += blockDim.x * 16) st_v4(dst + o, ld_cg_v4(src + o));
  if (threadIdx.x < bytes - v) dst[v + threadIdx.x] = src[v + threadIdx.x];
}

// Values of unit u (16 elements, guarded against n) of a reduction source:
// the caller's plain input, or a decoded record (raw plane + symbols in sm).
template <int DT>
LZ_DEV void unit_plain(const char* __restrict__ in, uint32_t u, uint32_t n, float (&v)[16]) {
  constexpr int ES = DT == DT_F32 ? 4 : 2;
  const uint32_t i0 = u * 16;
  if (i0 + 16 <= n) {
    uint4 raw[ES];
#pragma unroll
    for (int q = 0; q < ES; ++q) raw[q] = ld_cg_v4(in + (size_t)i0 * ES + 16 * q);
    if (DT == DT_F32) {
      const float* f = reinterpret_cast<const float*>(raw);
#pragma unroll
      for (int k = 0; k < 16; ++k) v[k] = f[k];
    } else if (DT == DT_BF16) {
      const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(raw);
#pragma unroll
      for (int k = 0; k < 16; ++k) v[k] = __bfloat162float(h[k]);
    } else {
      const __half* h = reinterpret_cast<const __half*>(raw);
#pragma unroll
      for (int k = 0; k < 16; ++k) v[k] = __half2float(h[k]);
    }
  } else {
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const uint32_t i = i0 + k;
      float x = 0.f;
      if (i < n) {
        if (DT == DT_F32) x = reinterpret_cast<const float*>(in)[i];
        else if (DT == DT_BF16) x = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(in)[i]);
        else x = __half2float(reinterpret_cast<const __half*>(in)[i]);
      }
      v[k] = x;
    }
  }
}

template <int DT>
LZ_DEV void unit_rec(const char* __restrict__ raw, const DecSmem& sm, uint32_t u, uint32_t n, float (&v)[16]) {
  using S = Split16<DT>;
  constexpr int RB = DT == DT_F32 ? 3 : 1;
  const bool full = (u + 1) * 16 <= n;
  if (DT != DT_F32) {
    // 16 symbols and 16 raw bytes as four words each; element k is byte k % 4 of word k / 4
    uint4 sv, rv;
    if (full) {
      rv = ld_cg_v4(raw + (size_t)u * 16);
      sv = *reinterpret_cast<const uint4*>(&sm.syms[u * 16]);
    } else {
      uint32_t sw[4] = {0, 0, 0, 0}, rwd[4] = {0, 0, 0, 0};
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        const uint32_t i = u * 16 + k;
        if (i < n) {
          sw[k / 4] |= (uint32_t)sm.syms[i] << (8 * (k % 4));
          rwd[k / 4] |= (uint32_t)ld_cg_u8(raw + i) << (8 * (k % 4));
        }
      }
      sv = make_uint4(sw[0], sw[1], sw[2], sw[3]);
      rv = make_uint4(rwd[0], rwd[1], rwd[2], rwd[3]);
    }
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const uint32_t sb = (word_of(sv, k / 4) >> (8 * (k % 4))) & 0xFFu;
      const uint32_t rb = (word_of(rv, k / 4) >> (8 * (k % 4))) & 0xFFu;
      if (DT == DT_BF16)
        v[k] = __uint_as_float((((rb & 0x80u) << 8) | (sb << 7) | (rb & 0x7Fu)) << 16);
      else
        v[k] = __half2float(__ushort_as_half((unsigned short)((sb << 8) | rb)));
    }
    return;
  }
  alignas(16) uint8_t rw[S::RAW_BYTES];
  uint8_t sy[16];
  if (full) {
#pragma unroll
    for (int q = 0; q < S::RAW_BYTES / 16; ++q)
      reinterpret_cast<uint4*>(rw)[q] = ld_cg_v4(raw + (size_t)u * S::RAW_BYTES + 16 * q);
    *reinterpret_cast<uint4*>(sy) = *reinterpret_cast<const uint4*>(&sm.syms[u * 16]);
  } else {
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const uint32_t i = u * 16 + k;
      sy[k] = i < n ? sm.syms[i] : 0;
#pragma unroll
      for (int q = 0; q < RB; ++q) rw[k * RB + q] = i < n ? ld_cg_u8(raw + (size_t)i * RB + q) : 0;
    }
  }
#pragma unroll
  for (int k = 0; k < 16; ++k) v[k] = elem_to_f32<DT>(sy[k], rw + k * RB);
}

// One source of a TG reduction: plain input elements, or a record whose
// symbols are decoded in sm (raw plane at `raw`).
struct RedSrc {
  const char* plain;
  const char* raw;
};

// One pass of the rank-order fp32 reduction of a TG of n elements: v = value
// of source a (+ value of source b, the next rank, when b is given); then
// sum = v (first pass) or acc + v, in that order, so the result equals the
// sequential fp32 sum. Intermediate passes keep the sum in `acc` (fp32
// scratch); the last pass stores it rounded once to the element type at
// `out` (no separate rounding pass).
template <int DT>
LZ_DEV void reduce_pass(RedSrc a, const RedSrc* b, const DecSmem& sm, uint32_t n, float* __restrict__ acc,
                        bool first, char* __restrict__ out) {
  constexpr int ES = DT == DT_F32 ? 4 : 2;
  const uint32_t units = (n + 15) / 16;
  for (uint32_t u = threadIdx.x; u < units; u += blockDim.x) {
    float v[16];
    if (a.plain) unit_plain<DT>(a.plain, u, n, v);
    else unit_rec<DT>(a.raw, sm, u, n, v);
    if (b) {
      float w[16];
      if (b->plain) unit_plain<DT>(b->plain, u, n, w);
      else unit_rec<DT>(b->raw, sm, u, n, w);
#pragma unroll
      for (int k = 0; k < 16; ++k) v[k] = v[k] + w[k];
    }
    float4* a4 = reinterpret_cast<float4*>(acc + (size_t)u * 16);
    if (!first) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 o = a4[q];
        v[4 * q] = o.x + v[4 * q];
        v[4 * q + 1] = o.y + v[4 * q + 1];
        v[4 * q + 2] = o.z + v[4 * q + 2];
        v[4 * q + 3] = o.w + v[4 * q + 3];
      }
    }
    if (!out) {
#pragma unroll
      for (int q = 0; q < 4; ++q) a4[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
      continue;
    }
    const uint32_t i0 = u * 16;
    if (i0 + 16 <= n) {
      uint4 o[ES];
      if (DT == DT_F32) {
        float* f = reinterpret_cast<float*>(o);
#pragma unroll
        for (int k = 0; k < 16; ++k) f[k] = v[k];
      } else if (DT == DT_BF16) {
        __nv_bfloat16* h = reinterpret_cast<__nv_bfloat16*>(o);
#pragma unroll
        for (int k = 0; k < 16; ++k) h[k] = __float2bfloat16_rn(v[k]);
      } else {
        __half* h = reinterpret_cast<__half*>(o);
#pragma unroll
        for (int k = 0; k < 16; ++k) h[k] = __float2half_rn(v[k]);
      }
#pragma unroll
      for (int q = 0; q < ES; ++q) st_v4(out + (size_t)i0 * ES + 16 * q, o[q]);
    } else {
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        const uint32_t i = i0 + k;
        if (i >= n) break;
        if (DT == DT_F32) reinterpret_cast<float*>(out)[i] = v[k];
        else if (DT == DT_BF16) reinterpret_cast<__nv_bfloat16*>(out)[i] = __float2bfloat16_rn(v[k]);
        else reinterpret_cast<__half*>(out)[i] = __float2half_rn(v[k]);
      }
    }
  }
}

template <int DT, int LV>
__device__ __forceinline__ void cz_allreduce_body(const LzDevComm& c, const CzParams& p) {
  extern __shared__ __align__(16) char smem_raw[];
  CzSmem& sm = *reinterpret_cast<CzSmem*>(smem_raw);
  constexpr int ES = DT == DT_F32 ? 4 : 2;
  const unsigned long long epoch = epoch_read(c);
  const int W = c.world, me = c.rank, G = gridDim.x, b = blockIdx.x;
  // slot of slice-local TG t in chunk k: its own slot (one chunk) or ring
  // position (k & 1) * C + (t - k * C) (two chunks in flight)
  const uint32_t C = p.chunk_tgs;
  auto ring = [&](uint32_t t, uint32_t k) { return p.nchunks > 1 ? (k & 1u) * C + (t - k * C) : t; };
  auto rs_slot = [&](int rank_heap, int src, uint32_t t, uint32_t k) {
    return c.heap[rank_heap] + p.rs_off + ((size_t)src * p.nslots + ring(t, k)) * p.sstride;
  };
  auto ag_slot = [&](char* base, int owner, uint32_t t, uint32_t k) {
    return base + p.ag_off + ((size_t)owner * p.nslots + ring(t, k)) * p.sstride;
  };
  auto flag_of = [&](char* slot) { return reinterpret_cast<unsigned long long*>(slot + p.cap); };
  // ready value of a slot: distinct for every (call, chunk), mixed with a
  // constant so that stale data of other algorithms never matches
  auto ready_of = [&](uint32_t k) {
    return (((epoch + 1ull) << 24) + (unsigned long long)k) ^ 0x9E3779B97F4A7C15ull;
  };
  unsigned long long ready = ready_of(0);
  __shared__ int s_wfail;
  // chunk progress: prog(r, blk, src) on rank r's heap = last chunk CTA blk of
  // rank src finished, as ((epoch + 1) << 24) + chunk + 1 (monotonic across
  // calls, so nothing is ever reset)
  auto prog = [&](int rank_heap, uint32_t blk, int src) {
    return reinterpret_cast<unsigned long long*>(c.heap[rank_heap] + kCzProgOff) + (size_t)blk * LZ_MAX_RANKS + src;
  };
  auto done_value = [&](uint32_t k) { return ((epoch + 1ull) << 24) + (unsigned long long)k + 1ull; };
  // CTA-wide bounded wait for a slot flag (thread 0 polls)
  auto wait_slot = [&](char* slot, int phase, int peer) {
    if (threadIdx.x == 0) s_wfail = lz_wait_eq(c, flag_of(slot), ready, phase, peer) ? 0 : 1;
    __syncthreads();
    return s_wfail == 0;
  };
  // phase tracer: thread 0 keeps the running sums in shared memory
  // (s_tr[kCzTraceSlots] = last mark, s_tr[kCzTraceSlots + 1] = start)
  __shared__ unsigned long long s_tr[kCzTraceSlots + 2];
  const bool tr = p.trace != nullptr && threadIdx.x == 0;
  if (tr) {
    for (int k = 0; k < kCzTraceSlots; ++k) s_tr[k] = 0ull;
    s_tr[kCzTraceSlots] = s_tr[kCzTraceSlots + 1] = globaltimer();
  }
  auto lap = [&](int slot) {  // time since the last mark goes to `slot`
    if (tr) {
      const unsigned long long now = globaltimer();
      s_tr[slot] += now - s_tr[kCzTraceSlots];
      s_tr[kCzTraceSlots] = now;
    }
  };
  // every rank's CTA b has finished the previous call
  if (!block_barrier(c, epoch, 1)) return;
  lap(CZ_T_BARRIER);

  for (uint32_t ck = 0; ck < p.nchunks; ++ck) {
  ready = ready_of(ck);
  const uint32_t t0 = ck * C, t1 = t0 + C;  // slice-local TG range of the chunk
  // TG t is handled by CTA t mod G: this CTA's first TG of the chunk
  const uint32_t first = (uint32_t)((b + G - (int)(((uint64_t)ck * C) % G)) % G);
  // The ring slots of this CTA's TGs were last used in chunk ck - 2 by CTA
  // (b - 2C) mod G of every rank (consumer of the records, and this rank's own
  // staging): wait until each of them has finished that chunk (bounded).
  if (ck >= 2) {
    __shared__ int s_pfail;
    if (threadIdx.x == 0) s_pfail = 0;
    __syncthreads();
    const uint32_t prev = (uint32_t)((b + G - (int)((2ull * C) % G)) % G);
    if (threadIdx.x < (unsigned)W && !lz_wait_ge(c, prog(me, prev, threadIdx.x), done_value(ck - 2), 4, threadIdx.x))
      s_pfail = 1;
    __syncthreads();
    if (s_pfail) return;
  }
  lap(CZ_T_CHUNK_WAIT);

  // 1. encode my input's TGs of every peer's slice into that peer's RS slots
  //    (hybrid: copy them raw; the reduce-scatter then pays no codec work)
  for (int k = 1; k < W; ++k) {
    const int dst = (me + k) % W;
    const uint64_t s0 = slice_begin(p, dst), sl = slice_len(p, dst);
    const uint32_t nt = min(ntg_of(p, dst), t1);
    for (uint32_t t = t0 + first; t < nt; t += G) {
      const uint32_t tn = (uint32_t)min((uint64_t)TG_ELEMS, sl - (uint64_t)t * TG_ELEMS);
      const char* src = p.in + (s0 + (uint64_t)t * TG_ELEMS) * ES;
      char* slot = rs_slot(dst, me, t, ck);
      if (p.hybrid) {
        cta_copy_bytes(slot, src, tn * ES);
      } else if (p.stage_local) {
        // encode next to this CTA (the slot of my own slice's TG t on my heap,
        // not yet used in this chunk), then push the record in 16-byte vectors
        char* loc = ag_slot(c.heap[me], me, t, ck);
        const uint32_t bytes = encode_tg<DT>(src, tn, loc, sm.enc, LV);
        cta_push16(slot, loc, pad16(bytes));
      } else {
        encode_tg<DT>(src, tn, slot, sm.enc, LV);
      }
      publish_block_writes(c);
      if (threadIdx.x == 0) st_release_sys(flag_of(slot), ready);
    }
  }
  lap(CZ_T_RS_ENCODE);

  // 2. decode + reduce (rank order, fp32) + store + re-encode + publish
  {
    const uint64_t s0 = slice_begin(p, me), sl = slice_len(p, me);
    const uint32_t nt = min(ntg_of(p, me), t1);
    float* acc = p.acc + (size_t)b * TG_ELEMS;
    for (uint32_t t = t0 + first; t < nt; t += G) {
      const uint32_t tn = (uint32_t)min((uint64_t)TG_ELEMS, sl - (uint64_t)t * TG_ELEMS);
      const uint64_t e0 = s0 + (uint64_t)t * TG_ELEMS;
      char* out_tg = p.out + e0 * ES;
      // Sources in rank order. The first two go in one pass when one of them
      // is this rank's own input (one decoded record at a time); the last
      // pass rounds straight into the output.
      int s = 0;
      while (s < W) {
        const bool pair = s == 0 && (me == 0 || me == 1);
        const int last = pair ? 1 : s;
        // source of rank r: own input, or its record (waited for, symbols decoded)
        auto source = [&](int r, RedSrc& out_src) -> bool {
          if (r == me) {
            out_src = RedSrc{p.in + e0 * ES, nullptr};
            return true;
          }
          if (!wait_slot(rs_slot(me, r, t, ck), 2, r)) return false;
          lap(CZ_T_RS_WAIT);
          const char* rec = rs_slot(me, r, t, ck);
          if (p.hybrid) {
            out_src = RedSrc{rec, nullptr};
            return true;
          }
          if (!decode_tg_syms<DT, kModesOfLevel<LV>>(rec, p.cap, tn, sm.dec)) {
            if (threadIdx.x == 0) lz_report(c, LZ_ERR_CORRUPT, 2, r);
            return false;
          }
          lap(CZ_T_RS_DECODE);
          out_src = RedSrc{nullptr, rec + sizeof(TgHeader)};
          return true;
        };
        RedSrc a, b2;
        if (!source(s, a)) return;
        if (pair && !source(1, b2)) return;
        reduce_pass<DT>(a, pair ? &b2 : nullptr, sm.dec, tn, acc, s == 0, last == W - 1 ? out_tg : nullptr);
        __syncthreads();
        lap(CZ_T_REDUCE);
        s = last + 1;
      }
      char* mine = ag_slot(c.heap[me], me, t, ck);
      const uint32_t bytes = encode_tg<DT>(p.out + e0 * ES, tn, mine, sm.enc, LV);
      lap(CZ_T_AG_ENCODE);
      const uint32_t padded = pad16(bytes);
      if (p.use_mc) {
        char* mc = ag_slot(c.heap_mc, me, t, ck);
        // eight 16-byte loads in flight per thread, then their multicast stores
        constexpr int U = 8;
        const uint32_t step = blockDim.x * 16;
        uint32_t o = threadIdx.x * 16;
        for (; o + (U - 1) * step < padded; o += U * step) {
          uint4 v[U];
#pragma unroll
          for (int u = 0; u < U; ++u) v[u] = ld_cg_v4(mine + o + u * step);
#pragma unroll
          for (int u = 0; u < U; ++u) multimem_st_v4(mc + o + u * step, v[u]);
        }
        for (; o < padded; o += step) multimem_st_v4(mc + o, ld_cg_v4(mine + o));
        publish_block_writes(c);
        if (threadIdx.x == 0) {
          fence_sys();
          multimem_st_release_u64(flag_of(mc), ready);
        }
      } else {
        for (int k = 1; k < W; ++k) cta_push16(ag_slot(c.heap[(me + k) % W], me, t, ck), mine, padded);
        publish_block_writes(c);
        if (threadIdx.x == 0)
          for (int k = 1; k < W; ++k) st_release_sys(flag_of(ag_slot(c.heap[(me + k) % W], me, t, ck)), ready);
      }
      __syncthreads();
      lap(CZ_T_AG_PUSH);
      if (tr) s_tr[CZ_T_TGS] += 1;
    }
  }

  // 3. decode the other owners' reduced TGs into my output
  for (int k = 1; k < W; ++k) {
    const int own = (me + W - k) % W;
    const uint64_t s0 = slice_begin(p, own), sl = slice_len(p, own);
    const uint32_t nt = min(ntg_of(p, own), t1);
    for (uint32_t t = t0 + first; t < nt; t += G) {
      const uint32_t tn = (uint32_t)min((uint64_t)TG_ELEMS, sl - (uint64_t)t * TG_ELEMS);
      if (!wait_slot(ag_slot(c.heap[me], own, t, ck), 3, own)) return;
      lap(CZ_T_AG_WAIT);
      if (p.use_mc) fence_proxy_alias();  // the record arrived through the multicast mapping
      if (!decode_tg<DT, kModesOfLevel<LV>>(ag_slot(c.heap[me], own, t, ck), p.cap, tn, p.out + (s0 + (uint64_t)t * TG_ELEMS) * ES,
                         sm.dec)) {
        if (threadIdx.x == 0) lz_report(c, LZ_ERR_CORRUPT, 3, own);
        return;
      }
      lap(CZ_T_AG_DECODE);
    }
  }
  // chunk ck done on this CTA: every rank (this one included) may refill the
  // ring slots it read or staged with chunk ck + 2
  if (ck + 2 < p.nchunks) {
    publish_block_writes(c);
    if (threadIdx.x < (unsigned)W) st_release_sys(prog(threadIdx.x, b, me), done_value(ck));
  }
  lap(CZ_T_CHUNK_WAIT);
  }  // chunks
  if (tr) {
    s_tr[CZ_T_TOTAL] = globaltimer() - s_tr[kCzTraceSlots + 1];
    unsigned long long* row = p.trace + (size_t)b * kCzTraceSlots;
    for (int k = 0; k < kCzTraceSlots; ++k) row[k] += s_tr[k];
  }
  epoch_advance(c);
}

template <int DT, int LV>
__global__ void __launch_bounds__(LZC_THREADS, LZC_MIN_BLOCKS) cz_allreduce_kernel(LzDevComm c, CzParams p) {
  cz_allreduce_body<DT, LV>(c, p);
}

// Single-GPU emulation: block (x, y) is block x of rank y (cooperative launch).
template <int DT, int LV>
__global__ void __launch_bounds__(LZC_THREADS, LZC_MIN_BLOCKS) cz_allreduce_emu_kernel(const LzDevComm* cs,
                                                                       const CzParams* ps) {
  cz_allreduce_body<DT, LV>(cs[blockIdx.y], ps[blockIdx.y]);
}

template <int DT>
void* cz_fn(bool emu, bool pack) {
  if (pack)
    return emu ? reinterpret_cast<void*>(&cz_allreduce_emu_kernel<DT, LEVEL_PACK>)
               : reinterpret_cast<void*>(&cz_allreduce_kernel<DT, LEVEL_PACK>);
  return emu ? reinterpret_cast<void*>(&cz_allreduce_emu_kernel<DT, LEVEL_ANS>)
             : reinterpret_cast<void*>(&cz_allreduce_kernel<DT, LEVEL_ANS>);
}

// flags bit 2: the codec's PACK level instead of rANS
void* cz_kernel_for(int dtype, bool emu, int flags) {
  const bool pack = (flags & 4) != 0;
  switch (dtype) {
    case LZ_F32:
      return cz_fn<DT_F32>(emu, pack);
    case LZ_F16:
      return cz_fn<DT_F16>(emu, pack);
    default:
      return cz_fn<DT_BF16>(emu, pack);
  }
}

}  // namespace

// Geometry of a call: TGs per slice, TGs per slice per chunk, chunks, slots
// per source. chunk_elems = elements of the whole vector per chunk (0 or
// >= n: one chunk, every TG its own slot); a chunked call keeps two chunks'
// slots in flight (ring), so its stage is bounded by the chunk, not by n.
struct CzGeom {
  uint64_t slice;
  uint32_t ntg, chunk_tgs, nchunks, nslots;
};
static CzGeom cz_geom(size_t n, int world, size_t chunk_elems) {
  CzGeom g;
  g.slice = ((n + world - 1) / world + 15) / 16 * 16;
  g.ntg = (uint32_t)num_tgs(g.slice);
  uint64_t per_slice = chunk_elems ? (chunk_elems + world - 1) / world : 0;
  uint32_t c = per_slice ? (uint32_t)num_tgs(per_slice) : g.ntg;
  if (c < 1) c = 1;
  if (c >= g.ntg) c = g.ntg;
  g.chunk_tgs = c;
  g.nchunks = g.ntg ? (g.ntg + c - 1) / c : 1;
  if (g.nchunks < 1) g.nchunks = 1;
  g.nslots = g.nchunks > 1 ? 2 * c : g.ntg;
  return g;
}

static size_t cz_stage_bytes(size_t n, int dtype, int world, int nblocks, size_t chunk_elems) {
  const CzGeom g = cz_geom(n, world, chunk_elems);
  const uint64_t sstride = tg_capacity(dtype) + 16;  // record capacity + flag footer
  return 2 * (size_t)world * g.nslots * sstride + (size_t)nblocks * TG_ELEMS * 4 + 256;
}

// Bytes of the compressed-allreduce staging region for n elements (one chunk).
extern "C" int lz_cz_trace_slots(void) { return kCzTraceSlots; }

extern "C" size_t lz_cz_stage_bytes(size_t n, int dtype, int world, int nblocks) {
  return cz_stage_bytes(n, dtype, world, nblocks, 0);
}
// The same for calls processed in chunks of chunk_elems elements.
extern "C" size_t lz_cz_stage_bytes_chunked(size_t n, int dtype, int world, int nblocks, size_t chunk_elems) {
  return cz_stage_bytes(n, dtype, world, nblocks, chunk_elems);
}

extern "C" int lz_cz_default_blocks(LzComm* c) { return c->sm_count * 3; }

// flags: bit 0 publish the all-gather records with NVLS multimem.st (when a
// multicast object exists), bit 1 hybrid (raw reduce-scatter), bit 2 PACK
// codec level (table codes; faster than rANS, lower ratio).
static int cz_plan(const LzComm* c, const void* in, void* out, size_t n, int dtype, int G,
                   int flags, size_t chunk_elems, CzParams* out_p) {
  const int W = c->dev.world;
  if (dtype != LZ_F32 && dtype != LZ_F16 && dtype != LZ_BF16) {
    lz_set_error("compressed allreduce: dtype %d not supported (float types only)", dtype);
    return LZE_ARG;
  }
  if ((uintptr_t)in % 16 || (uintptr_t)out % 16) {
    lz_set_error("compressed allreduce needs 16-byte aligned buffers");
    return LZE_ARG;
  }
  const CzGeom g = cz_geom(n, W, chunk_elems);
  CzParams p;
  memset(&p, 0, sizeof(p));
  p.in = static_cast<const char*>(in);
  p.out = static_cast<char*>(out);
  p.n = n;
  p.slice = g.slice;
  p.ntg_max = g.ntg;
  p.chunk_tgs = g.chunk_tgs;
  p.nchunks = g.nchunks;
  p.nslots = g.nslots;
  p.cap = tg_capacity(dtype);
  p.sstride = p.cap + 16;
  const size_t need = cz_stage_bytes(n, dtype, W, G, chunk_elems);
  if (need > c->stage_bytes) {
    lz_set_error("compressed allreduce: stage needs %zu bytes, communicator has %zu (raise stage_bytes "
                 "or process the call in chunks)",
                 need, c->stage_bytes);
    return LZE_ARG;
  }
  const size_t slots = (size_t)W * p.nslots * p.sstride;
  p.rs_off = c->stage_off;
  p.ag_off = c->stage_off + slots;
  const size_t acc_off = p.ag_off + slots;
  p.acc = reinterpret_cast<float*>(c->dev.heap[c->dev.rank] + acc_off);
  // multicast publish only pays with more than one receiver: at 2 ranks a
  // peer store writes the record once, a multimem.st also writes it locally
  // (traced on 2 x B200, 1 GiB: the multicast publish took 1.08 of 3.05 ms)
  p.use_mc = ((flags & 1) && c->dev.heap_mc && W > 2) ? 1 : 0;
  p.hybrid = (flags & 2) ? 1 : 0;
  p.stage_local = (flags & 8) ? 1 : 0;
  *out_p = p;
  return LZE_OK;
}

// flags: bit 0 multicast all-gather, bit 1 hybrid (raw reduce-scatter, the
// compressed P2P hybrid of the reference's compressed_p2p_allreduce.py:54-188),
// bit 2 PACK codec level, bit 3 encode reduce-scatter records locally and push
// them as 16-byte vectors (instead of encoding straight into the peer's slot).
// chunk_elems: see cz_geom (0: one chunk).
// trace: optional device buffer of nblocks x lz_cz_trace_slots() u64 (phase
// nanoseconds per CTA, added to; phases in CzPhase), or nullptr.
extern "C" int lz_compressed_allreduce_traced(LzComm* c, const void* in, void* out, size_t n, int dtype,
                                              int nblocks, int flags, size_t chunk_elems,
                                              unsigned long long* trace, cudaStream_t s);
extern "C" int lz_compressed_allreduce_chunked(LzComm* c, const void* in, void* out, size_t n, int dtype,
                                               int nblocks, int flags, size_t chunk_elems, cudaStream_t s) {
  return lz_compressed_allreduce_traced(c, in, out, n, dtype, nblocks, flags, chunk_elems, nullptr, s);
}

extern "C" int lz_compressed_allreduce_traced(LzComm* c, const void* in, void* out, size_t n, int dtype,
                                              int nblocks, int flags, size_t chunk_elems,
                                              unsigned long long* trace, cudaStream_t s) {
  const int W = c->dev.world;
  const size_t es = dtype == LZ_F32 ? 4 : 2;
  if (W == 1) {
    if (in != out) LZ_CUDA_TRY(cudaMemcpyAsync(out, in, n * es, cudaMemcpyDeviceToDevice, s));
    return LZE_OK;
  }
  int G = nblocks > 0 ? nblocks : lz_cz_default_blocks(c);
  if (G > LZ_MAX_BLOCKS) G = LZ_MAX_BLOCKS;
  CzParams p;
  int rc = cz_plan(c, in, out, n, dtype, G, flags, chunk_elems, &p);
  if (rc) return rc;
  p.trace = trace;
  void* fn = cz_kernel_for(dtype, false, flags);
  const size_t smem = sizeof(CzSmem);
  LZ_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  void* args[] = {&c->dev, &p};
  LZ_CUDA_TRY(cudaLaunchKernel(fn, dim3(G), dim3(LZC_THREADS), args, smem, s));
  return LZE_OK;
}

extern "C" int lz_compressed_allreduce(LzComm* c, const void* in, void* out, size_t n, int dtype,
                                       int nblocks, int flags, cudaStream_t s) {
  return lz_compressed_allreduce_chunked(c, in, out, n, dtype, nblocks, flags, 0, s);
}

// Single-GPU emulation of the compressed allreduce over the R emulated ranks.
// trace: optional device buffer of R x G x lz_cz_trace_slots() u64 (rank r's
// CTA rows at r * G), or nullptr.
extern "C" int lz_emu_compressed_allreduce_traced(LzEmu* e, const void* const* ins, void* const* outs,
                                                  size_t n, int dtype, int nblocks, int flags,
                                                  size_t chunk_elems, unsigned long long* trace,
                                                  cudaStream_t s);
extern "C" int lz_emu_compressed_allreduce_chunked(LzEmu* e, const void* const* ins, void* const* outs,
                                                   size_t n, int dtype, int nblocks, int flags,
                                                   size_t chunk_elems, cudaStream_t s) {
  return lz_emu_compressed_allreduce_traced(e, ins, outs, n, dtype, nblocks, flags, chunk_elems, nullptr, s);
}

extern "C" int lz_emu_compressed_allreduce_traced(LzEmu* e, const void* const* ins, void* const* outs,
                                                  size_t n, int dtype, int nblocks, int flags,
                                                  size_t chunk_elems, unsigned long long* trace,
                                                  cudaStream_t s) {
  const int R = lz_emu_world(e);
  void* fn = cz_kernel_for(dtype, true, flags);
  const size_t smem = sizeof(CzSmem);
  LZ_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  int per_sm = 0;
  LZ_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, LZC_THREADS, smem));
  const int cap = per_sm * lz_emu_comm(e, 0)->sm_count;
  int G = nblocks > 0 ? nblocks : cap / R;
  if (G * R > cap || G < 1) {
    lz_set_error("emulated compressed allreduce: %d x %d blocks exceed co-residency %d", G, R, cap);
    return LZE_ARG;
  }
  CzParams hp[LZ_MAX_RANKS];
  for (int r = 0; r < R; ++r) {
    int rc = cz_plan(lz_emu_comm(e, r), ins[r], outs[r], n, dtype, G, flags & (2 | 8), chunk_elems, &hp[r]);
    if (rc) return rc;
    hp[r].trace = trace ? trace + (size_t)r * G * kCzTraceSlots : nullptr;
  }
  static_assert(sizeof(CzParams) * LZ_MAX_RANKS <= 4096, "param buffer");
  void* dparams = lz_emu_param_buffer(e);
  LZ_CUDA_TRY(cudaMemcpyAsync(dparams, hp, sizeof(CzParams) * R, cudaMemcpyHostToDevice, s));
  LzDevComm* dcomms = lz_emu_dev_comms(e);
  void* args[] = {&dcomms, &dparams};
  LZ_CUDA_TRY(cudaLaunchCooperativeKernel(fn, dim3(G, R), dim3(LZC_THREADS), args, smem, s));
  LZ_CUDA_TRY(cudaStreamSynchronize(s));
  return LZE_OK;
}

extern "C" int lz_emu_compressed_allreduce(LzEmu* e, const void* const* ins, void* const* outs,
                                           size_t n, int dtype, int nblocks, int flags, cudaStream_t s) {
  return lz_emu_compressed_allreduce_chunked(e, ins, outs, n, dtype, nblocks, flags, 0, s);
}
