// All-to-all over NVLink peer memory, raw or split+rANS compressed.
//
// Input on every rank: W chunks of `chunk` elements; chunk j goes to rank j,
// which stores it as its chunk `src`. One persistent launch per call:
//   barrier 1  every rank has entered the call (its previous use of the
//              receive slots / output is over, stream order);
//   send       raw: peer stores of each chunk straight into the destination
//              rank's output when that output is symmetric (zero copy), else
//              into its receive slot; compressed: every table group (TG) is
//              encoded by this GPU and the record written straight into the
//              destination's slot (only compressed bytes cross NVLink);
//   barrier 2  every chunk has landed;
//   receive    copy (raw, non-symmetric output) or decode (compressed) the
//              W-1 incoming chunks into the output.
// The own chunk is copied locally. Records are never truncated (a TG that
// does not compress is stored RAW).
//
// Reference behaviour: the LZip-NCCL compressed all-to-all whose numbers the
// reference plots (plot/cccl_alltoall.py:7-16) and the all-to-all exchange of
// its compressed two-shot (single_node_nccl_allreduce_benchmark/compressed_twoshot_allreduce.py:148-163).
#include "lz_codec_dev.cuh"
#include "lz_internal.h"

using namespace lzc;
using namespace lzg;

namespace {

struct A2aParams {
  const char* in;
  char* out;
  uint64_t chunk;        // elements per chunk
  uint64_t chunk_bytes;  // multiple of 16
  size_t slot_off;       // heap offset of the receive slots [src]
  size_t out_off;        // heap offset of `out` when symmetric (raw zero copy), else ~0
  uint32_t ntg;          // TGs per chunk (compressed)
  uint32_t cap;          // TG record capacity (compressed)
};

union A2aSmem {
  EncSmem enc;
  DecSmem dec;
};

// CTA b's share [v0, v1) of nv 16-byte vectors, copied with 4 loads in flight.
LZ_DEV void cta_share_copy(char* __restrict__ dst, const char* __restrict__ src, uint64_t bytes) {
  const uint64_t nv = bytes / 16;
  const uint64_t v0 = part_begin(nv, gridDim.x, blockIdx.x), v1 = part_begin(nv, gridDim.x, blockIdx.x + 1);
  const uint4* s = reinterpret_cast<const uint4*>(src);
  uint4* d = reinterpret_cast<uint4*>(dst);
  uint64_t i = v0 + threadIdx.x;
  for (; i + 3 * blockDim.x < v1; i += 4 * blockDim.x) {
    uint4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) v[u] = ld_cg_v4(s + i + u * blockDim.x);
#pragma unroll
    for (int u = 0; u < 4; ++u) st_v4(d + i + u * blockDim.x, v[u]);
  }
  for (; i < v1; i += blockDim.x) st_v4(d + i, ld_cg_v4(s + i));
}

// KENC: 0 raw bytes, 1 split + rANS records, 2 split + PACK records
template <int DT, int KENC>
__device__ __forceinline__ void a2a_body(const LzDevComm& c, const A2aParams& p) {
  constexpr bool kEnc = KENC != 0;
  constexpr int kLevel = KENC == 2 ? LEVEL_PACK : LEVEL_ANS;
  extern __shared__ __align__(16) char smem_raw[];
  constexpr int ES = DT == DT_F32 ? 4 : (DT == DT_U8 ? 1 : 2);
  const unsigned long long epoch = epoch_read(c);
  const int W = c.world, me = c.rank, G = gridDim.x, b = blockIdx.x;
  const bool zero_copy = !kEnc && p.out_off != ~(size_t)0;
  if (!block_barrier(c, epoch, 1)) return;
  // send, starting with the next rank so that destinations are spread
  for (int k = 0; k < W; ++k) {
    const int dst = (me + k) % W;
    const char* src = p.in + (uint64_t)dst * p.chunk_bytes;
    if (dst == me) {
      cta_share_copy(p.out + (uint64_t)me * p.chunk_bytes, src, p.chunk_bytes);
    } else if (!kEnc) {
      char* tgt = zero_copy ? c.heap[dst] + p.out_off + (uint64_t)me * p.chunk_bytes
                            : c.heap[dst] + p.slot_off + (uint64_t)me * p.chunk_bytes;
      if (lz_range_ok(c, tgt, p.chunk_bytes, 22)) cta_share_copy(tgt, src, p.chunk_bytes);
    } else {
      A2aSmem& sm = *reinterpret_cast<A2aSmem*>(smem_raw);
      for (uint32_t t = b; t < p.ntg; t += G) {
        const uint32_t tn = (uint32_t)min((uint64_t)TG_ELEMS, p.chunk - (uint64_t)t * TG_ELEMS);
        char* rec = c.heap[dst] + p.slot_off + ((size_t)me * p.ntg + t) * p.cap;
        if (lz_range_ok(c, rec, p.cap, 23)) encode_tg<DT>(src + (uint64_t)t * TG_ELEMS * ES, tn, rec, sm.enc, kLevel);
      }
    }
  }
  if (!block_barrier(c, epoch, 2)) return;
  if (!zero_copy) {
    for (int k = 1; k < W; ++k) {
      const int from = (me + W - k) % W;
      char* dst = p.out + (uint64_t)from * p.chunk_bytes;
      if (!kEnc) {
        cta_share_copy(dst, c.heap[me] + p.slot_off + (uint64_t)from * p.chunk_bytes, p.chunk_bytes);
      } else {
        A2aSmem& sm = *reinterpret_cast<A2aSmem*>(smem_raw);
        for (uint32_t t = b; t < p.ntg; t += G) {
          const uint32_t tn = (uint32_t)min((uint64_t)TG_ELEMS, p.chunk - (uint64_t)t * TG_ELEMS);
          const char* rec = c.heap[me] + p.slot_off + ((size_t)from * p.ntg + t) * p.cap;
          if (!decode_tg<DT>(rec, p.cap, tn, dst + (uint64_t)t * TG_ELEMS * ES, sm.dec)) {
            if (threadIdx.x == 0) lz_report(c, LZ_ERR_CORRUPT, 4, from);
            return;
          }
        }
      }
    }
  }
  epoch_advance(c);
}

template <int DT, int KENC>
__global__ void __launch_bounds__(LZC_THREADS) a2a_kernel(LzDevComm c, A2aParams p) {
  a2a_body<DT, KENC>(c, p);
}

// Single-GPU emulation: block (x, y) is block x of rank y (cooperative launch).
template <int DT, int KENC>
__global__ void __launch_bounds__(LZC_THREADS) a2a_emu_kernel(const LzDevComm* cs, const A2aParams* ps) {
  a2a_body<DT, KENC>(cs[blockIdx.y], ps[blockIdx.y]);
}

// enc: 0 raw, 1 rANS records, 2 PACK records
void* a2a_fn(int dtype, int enc, bool emu) {
#define LZ_A2A(D)                                                                            \
  if (enc == 2) return emu ? reinterpret_cast<void*>(&a2a_emu_kernel<D, 2>)                  \
                           : reinterpret_cast<void*>(&a2a_kernel<D, 2>);                     \
  if (enc) return emu ? reinterpret_cast<void*>(&a2a_emu_kernel<D, 1>)                       \
                      : reinterpret_cast<void*>(&a2a_kernel<D, 1>);                          \
  return emu ? reinterpret_cast<void*>(&a2a_emu_kernel<D, 0>)                                \
             : reinterpret_cast<void*>(&a2a_kernel<D, 0>);
  switch (dtype) {
    case LZ_F32: { LZ_A2A(DT_F32) }
    case LZ_F16: { LZ_A2A(DT_F16) }
    case LZ_BF16: { LZ_A2A(DT_BF16) }
    default: {
      if (enc) return nullptr;
      return emu ? reinterpret_cast<void*>(&a2a_emu_kernel<DT_U8, 0>)
                 : reinterpret_cast<void*>(&a2a_kernel<DT_U8, 0>);
    }
  }
#undef LZ_A2A
}

int es_of_dtype(int dtype) { return dtype == LZ_F32 ? 4 : (dtype == LZ_U8 ? 1 : 2); }

int a2a_plan(const LzComm* c, const void* in, void* out, size_t chunk, int dtype, int encode, A2aParams* out_p) {
  const int W = c->dev.world;
  const size_t es = (size_t)es_of_dtype(dtype);
  if (encode && dtype != LZ_F32 && dtype != LZ_F16 && dtype != LZ_BF16) {
    lz_set_error("compressed all-to-all: float dtypes only (got %d)", dtype);
    return LZE_ARG;
  }
  if ((uintptr_t)in % 16 || (uintptr_t)out % 16 || (chunk * es) % 16) {
    lz_set_error("all-to-all needs 16-byte aligned buffers and chunks of a multiple of 16 bytes");
    return LZE_ARG;
  }
  if (in == out) {
    lz_set_error("all-to-all cannot run in place");
    return LZE_ARG;
  }
  A2aParams p;
  memset(&p, 0, sizeof(p));
  p.in = static_cast<const char*>(in);
  p.out = static_cast<char*>(out);
  p.chunk = chunk;
  p.chunk_bytes = chunk * es;
  p.slot_off = c->stage_off;
  p.out_off = ~(size_t)0;
  size_t need = 0;
  if (encode) {
    p.ntg = (uint32_t)num_tgs(chunk);
    p.cap = tg_capacity(dtype);
    need = (size_t)W * p.ntg * p.cap;
  } else {
    const size_t off = lz_comm_heap_offset(c, out, (size_t)W * p.chunk_bytes);
    if (off != (size_t)-1) p.out_off = off;
    else need = (size_t)W * p.chunk_bytes;
  }
  if (need > c->stage_bytes) {
    lz_set_error("all-to-all: stage needs %zu bytes, communicator has %zu (raise stage_bytes)", need,
                 c->stage_bytes);
    return LZE_ARG;
  }
  *out_p = p;
  return LZE_OK;
}

}  // namespace

// Stage bytes a call needs (0 for raw into a symmetric output).
extern "C" size_t lz_all_to_all_stage_bytes(size_t chunk, int dtype, int world, int encode) {
  if (encode) return (size_t)world * num_tgs(chunk) * tg_capacity(dtype);
  return (size_t)world * chunk * (size_t)es_of_dtype(dtype);
}

extern "C" int lz_all_to_all(LzComm* c, const void* in, void* out, size_t chunk, int dtype, int encode,
                             int nblocks, cudaStream_t s) {
  const int W = c->dev.world;
  const size_t es = (size_t)es_of_dtype(dtype);
  if (W == 1) {
    if (in != out) LZ_CUDA_TRY(cudaMemcpyAsync(out, in, chunk * es, cudaMemcpyDeviceToDevice, s));
    return LZE_OK;
  }
  A2aParams p;
  int rc = a2a_plan(c, in, out, chunk, dtype, encode, &p);
  if (rc) return rc;
  // Every CTA pays two flag barriers, so small calls use few CTAs: raw, one
  // CTA per 64 KB sent (16 .. one per SM); compressed, one per table group of
  // a chunk (up to 3 per SM, the encoder's occupancy).
  int G = nblocks;
  if (G <= 0) {
    if (encode) {
      G = (int)p.ntg;
      if (G > c->sm_count * 3) G = c->sm_count * 3;
    } else {
      const uint64_t per = (uint64_t)W * p.chunk_bytes / (64u << 10);
      G = per < 16 ? 16 : (per > (uint64_t)c->sm_count ? c->sm_count : (int)per);
    }
  }
  if (G > LZ_MAX_BLOCKS) G = LZ_MAX_BLOCKS;
  void* fn = a2a_fn(dtype, encode, false);
  const size_t smem = encode ? sizeof(A2aSmem) : 0;
  if (encode) LZ_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  void* args[] = {&c->dev, &p};
  LZ_CUDA_TRY(cudaLaunchKernel(fn, dim3(G), dim3(LZC_THREADS), args, smem, s));
  return LZE_OK;
}

// Single-GPU emulation over the R emulated ranks (ins[r], outs[r] per rank). Synchronous.
extern "C" int lz_emu_all_to_all(LzEmu* e, const void* const* ins, void* const* outs, size_t chunk, int dtype,
                                 int encode, int nblocks, cudaStream_t s) {
  const int R = lz_emu_world(e);
  void* fn = a2a_fn(dtype, encode, true);
  if (!fn) {
    lz_set_error("emulated all-to-all: unsupported dtype %d", dtype);
    return LZE_ARG;
  }
  const size_t smem = encode ? sizeof(A2aSmem) : 0;
  if (encode) LZ_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  int per_sm = 0;
  LZ_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, LZC_THREADS, smem));
  const int cap = per_sm * lz_emu_comm(e, 0)->sm_count;
  const int G = nblocks > 0 ? nblocks : cap / R;
  if (G * R > cap || G < 1) {
    lz_set_error("emulated all-to-all: %d x %d blocks exceed co-residency %d", G, R, cap);
    return LZE_ARG;
  }
  A2aParams hp[LZ_MAX_RANKS];
  for (int r = 0; r < R; ++r) {
    int rc = a2a_plan(lz_emu_comm(e, r), ins[r], outs[r], chunk, dtype, encode, &hp[r]);
    if (rc) return rc;
  }
  static_assert(sizeof(A2aParams) * LZ_MAX_RANKS <= 4096, "param buffer");
  void* dparams = lz_emu_param_buffer(e);
  LZ_CUDA_TRY(cudaMemcpyAsync(dparams, hp, sizeof(A2aParams) * R, cudaMemcpyHostToDevice, s));
  LzDevComm* dcomms = lz_emu_dev_comms(e);
  void* args[] = {&dcomms, &dparams};
  LZ_CUDA_TRY(cudaLaunchCooperativeKernel(fn, dim3(G, R), dim3(LZC_THREADS), args, smem, s));
  LZ_CUDA_TRY(cudaStreamSynchronize(s));
  return LZE_OK;
}
