// Copy-engine allreduce: the bytes cross NVLink by DMA (cudaMemcpyAsync into a
// peer's heap mapping) while the SMs only do the fp32 accumulation.
//
// Measured on 2 x B200 with both directions loaded (1 GiB, CUDA events): the
// copy engines push 768 GB/s per direction, SM peer stores 699 GB/s, SM peer
// loads 657 GB/s, and the pull-reduce-push two-shot kernel reaches 596 GB/s.
// Moving the data with the copy engines and keeping the SMs for the reduce is
// the fastest large-message allreduce at two ranks.
//
// Two entry points share lz_ce_allreduce():
//
// * zero-copy pipelined two-shot (input and output in the symmetric heap,
//   distinct): the slice of rank q is cut into `pipes` chunks.
//     start (caller's stream): post "started" to every peer and wait for
//          every peer's "started" (its earlier work on its output is done);
//     RS   (side stream 0, copies only): push chunk k of my copy of slice q
//          into q's OUTPUT buffer, then an 8-byte copy of the call number into
//          q's chunk flag [me][k] (stream order puts it after the data copy's
//          completion);
//     reduce (caller's stream): per chunk, wait for every peer's chunk flag,
//          sum in fp32 in rank order, write my output slice;
//     AG   (side stream 1): push my reduced chunk into every peer's output,
//          finally an 8-byte "done" copy; the caller's stream waits for every
//          peer's "done".
//   The output doubles as the receive area: the contribution of rank
//   (q + 1) mod W lands in q's own output slice (reduced in place), every
//   other sender r uses q's output slice r, which r overwrites in its AG only
//   after q has posted "chunk reduced" (never needed at W = 2).
// * staged (any buffers): copy-in to the stage, barrier, copy engines fetch my
//   slice from every peer in `pipes` pieces overlapped with the accumulation,
//   barrier, copy engines fetch every peer's result.
//
// Flag values are the communicator's copy-engine call number (a device
// counter bumped by the first kernel of every call), so flags are never
// reset. Every wait is bounded (lz_wait_ge).
//
// Reference behaviour being re-designed:
// single_node_nccl_allreduce_benchmark/memcpy_p2p_allreduce_kernel.cu:176-346 (D2D
// and host-staged pipelines, bf16 __hadd2 accumulation rounding at every
// step); here accumulation is fp32 in rank order, rounded once, so the result
// is bit-identical to the other allreduce paths.
#include <stdlib.h>
#include <string.h>

#include "lz_common.cuh"
#include "lz_internal.h"

extern "C" int lz_barrier(LzComm* c, cudaStream_t s);

namespace {

constexpr int kCeMaxChunks = 64;
constexpr size_t kCeArBase = 544u << 10;
constexpr size_t kCeArStarted = kCeArBase;        // [src] u64
constexpr size_t kCeArDone = kCeArBase + 64;      // [src] u64
constexpr size_t kCeArRs = kCeArBase + 128;       // [src][chunk] u64
constexpr size_t kCeArRed = kCeArRs + (size_t)LZ_MAX_RANKS * kCeMaxChunks * 8;  // [src][chunk]
constexpr size_t kCeArEnd = kCeArRed + (size_t)LZ_MAX_RANKS * kCeMaxChunks * 8;
static_assert(kCeArBase >= (512u << 10) + 64, "copy-engine allreduce flags overlap the test word");
static_assert(kCeArEnd <= kLzFlagsBytes, "copy-engine allreduce flags exceed the flag area");
// events: [0] begin, [1..kCeMaxChunks] chunk reduced, RS end, AG end, flag
// stream end, then [kCeMaxChunks] chunk copied (RS data stream -> flag stream)
constexpr int kCeEvBegin = 0, kCeEvRed = 1, kCeEvRsEnd = 1 + kCeMaxChunks, kCeEvAgEnd = 2 + kCeMaxChunks;
constexpr int kCeEvFlagEnd = 3 + kCeMaxChunks, kCeEvCopied = 4 + kCeMaxChunks;
constexpr int kCeNumEvents = 4 + 2 * kCeMaxChunks;
constexpr int kCeStreams = 3;  // RS data, AG data, RS flags

LZ_DEV unsigned long long* hflag(const LzDevComm& c, int rank, size_t off) {
  return reinterpret_cast<unsigned long long*>(c.heap[rank] + off);
}

LZ_DEV unsigned long long read_seq(const unsigned long long* seq) {
  return *reinterpret_cast<const volatile unsigned long long*>(seq);
}

// Bumps the call counter and posts "started" to every peer. One thread.
__global__ void ce_begin_kernel(LzDevComm c, unsigned long long* seq_ctr) {
  if (threadIdx.x != 0) return;
  const unsigned long long seq = read_seq(seq_ctr) + 1ull;
  *seq_ctr = seq;
  __threadfence();
  for (int q = 0; q < c.world; ++q)
    if (q != c.rank) st_release_sys(hflag(c, q, kCeArStarted + 8u * c.rank), seq);
}

// Thread t < world waits until this rank's flag t * stride + chunk (u64 words
// from `base`) reaches the current call number, for every t set in `mask`.
// Per-source flags use stride 1, per-(source, chunk) flags kCeMaxChunks.
__global__ void ce_wait_kernel(LzDevComm c, size_t base, int stride, int chunk,
                               const unsigned long long* seq_ctr, unsigned int mask, int phase) {
  const int t = threadIdx.x;
  if (t >= c.world || !((mask >> t) & 1u)) return;
  const unsigned long long seq = read_seq(seq_ctr);
  lz_wait_ge(c, hflag(c, c.rank, base + 8u * ((size_t)t * stride + chunk)), seq, phase, t);
}

struct CeRedParams {
  const char* in;       // my input (whole vector)
  char* out;            // my output (whole vector, also the receive area)
  size_t slice;         // bytes per rank slice
  size_t coff, clen;    // chunk range inside the slice (bytes, multiples of 16)
  int chunk;
  unsigned int red_mask;  // peers to tell "chunk reduced"
  const unsigned long long* seq_ctr;
  unsigned int* done;
  char* peer_out;         // SM all-gather (W = 2): the peer's output, else nullptr
  int last;               // SM all-gather: last chunk, post "done" to the peer
};

// Sender r's contribution to receiver q's slice lands in q's output slice
// dslot(r, q): q's own slice for r = (q + 1) mod W, else slice r.
LZ_DEV int dslot(int r, int q, int W) { return r == (q + 1) % W ? q : r; }

// MAXW: compile-time bound of the world size (2, 4 or 8) so the per-rank
// load arrays take registers for the ranks that exist (W = 2: 40 registers).
template <int DT, int MAXW>
__global__ void __launch_bounds__(512) ce_reduce_kernel(LzDevComm c, CeRedParams p) {
  using V = Vec<DT>;
  __shared__ int s_fail;
  const int W = c.world, me = c.rank;
  const unsigned long long seq = read_seq(p.seq_ctr);
  if (threadIdx.x == 0) s_fail = 0;
  __syncthreads();
  if (threadIdx.x < W && threadIdx.x != me) {
    const unsigned long long* f = hflag(c, me, kCeArRs + 8u * ((size_t)threadIdx.x * kCeMaxChunks + p.chunk));
    if (!lz_wait_ge(c, f, seq, 20, threadIdx.x)) s_fail = 1;
  }
  __syncthreads();
  if (s_fail) return;
  const uint4* src[MAXW];
#pragma unroll
  for (int r = 0; r < MAXW; ++r) {
    const char* base = (r == me) ? p.in + (size_t)me * p.slice
                                 : p.out + (size_t)dslot(r, me, W) * p.slice;
    src[r] = reinterpret_cast<const uint4*>(base + p.coff);
  }
  uint4* dst = reinterpret_cast<uint4*>(p.out + (size_t)me * p.slice + p.coff);
  uint4* pdst = p.peer_out ? reinterpret_cast<uint4*>(p.peer_out + (size_t)me * p.slice + p.coff) : nullptr;
  const size_t nv = p.clen / 16;
  const size_t v0 = part_begin(nv, gridDim.x, blockIdx.x), v1 = part_begin(nv, gridDim.x, blockIdx.x + 1);
  constexpr int U = 2;
  size_t i = v0 + threadIdx.x;
  for (; i + (U - 1) * blockDim.x < v1; i += U * blockDim.x) {
    uint4 v[U][MAXW];
#pragma unroll
    for (int r = 0; r < MAXW; ++r)
      if (r < W)
#pragma unroll
        for (int u = 0; u < U; ++u) v[u][r] = ld_cg_v4(src[r] + i + u * blockDim.x);
#pragma unroll
    for (int u = 0; u < U; ++u) {
      float acc[V::N];
      V::load(acc, v[u][0]);
#pragma unroll
      for (int r = 1; r < MAXW; ++r)
        if (r < W) V::add(acc, v[u][r]);
      const uint4 res = V::pack(acc);
      dst[i + u * blockDim.x] = res;
      if (pdst) pdst[i + u * blockDim.x] = res;
    }
  }
  for (; i < v1; i += blockDim.x) {
    float acc[V::N];
    V::load(acc, ld_cg_v4(src[0] + i));
#pragma unroll
    for (int r = 1; r < MAXW; ++r)
      if (r < W) V::add(acc, ld_cg_v4(src[r] + i));
    const uint4 res = V::pack(acc);
    dst[i] = res;
    if (pdst) pdst[i] = res;
  }
  if (pdst) {
    // every block fences its peer stores (system scope) before counting
    // itself finished; the last block of the last chunk posts "done"
    __syncthreads();
    if (threadIdx.x == 0) {
      fence_sys();
      if (p.last) {
        const unsigned int prev = atomicAdd(p.done, 1u);
        if (prev == gridDim.x - 1) {
          *p.done = 0;
          fence_sys();
          st_release_sys(hflag(c, 1 - me, kCeArDone + 8u * me), seq);
        }
      }
    }
    return;
  }
  if (!p.red_mask) return;
  // the last block to finish tells the senders whose receive slot it read
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned int prev = atomicAdd(p.done, 1u);
    if (prev == gridDim.x - 1) {
      *p.done = 0;
      __threadfence();
      for (int q = 0; q < W; ++q)
        if ((p.red_mask >> q) & 1u)
          st_release_sys(hflag(c, q, kCeArRed + 8u * ((size_t)me * kCeMaxChunks + p.chunk)), seq);
    }
  }
}

// Staged path: out (and my result slot) = sum over ranks of my slice.
template <int DT>
__global__ void __launch_bounds__(256) accum_kernel(const char* __restrict__ own,
                                                    const char* __restrict__ tmp, size_t tmp_stride,
                                                    int world, int me, char* __restrict__ out,
                                                    char* __restrict__ out2, size_t nvec) {
  using V = Vec<DT>;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += stride) {
    float acc[V::N];
    bool first = true;
    for (int r = 0; r < world; ++r) {
      const uint4 v = (r == me) ? reinterpret_cast<const uint4*>(own)[i]
                                : reinterpret_cast<const uint4*>(tmp + (size_t)r * tmp_stride)[i];
      if (first) V::load(acc, v);
      else V::add(acc, v);
      first = false;
    }
    const uint4 res = V::pack(acc);
    reinterpret_cast<uint4*>(out)[i] = res;
    reinterpret_cast<uint4*>(out2)[i] = res;
  }
}

template <int DT>
int launch_reduce(const LzComm* c, const CeRedParams& p, int G, cudaStream_t s) {
  const int W = c->dev.world;
  if (W <= 2) ce_reduce_kernel<DT, 2><<<G, 512, 0, s>>>(c->dev, p);
  else if (W <= 4) ce_reduce_kernel<DT, 4><<<G, 512, 0, s>>>(c->dev, p);
  else ce_reduce_kernel<DT, LZ_MAX_RANKS><<<G, 512, 0, s>>>(c->dev, p);
  LZ_CUDA_TRY(cudaGetLastError());
  return LZE_OK;
}

int launch_accum(int dtype, int G, cudaStream_t s, const char* own, const char* tmp, size_t stride, int W,
                 int me, char* o1, char* o2, size_t nvec) {
  switch (dtype) {
    case LZ_F32:
      accum_kernel<LZ_F32><<<G, 256, 0, s>>>(own, tmp, stride, W, me, o1, o2, nvec);
      break;
    case LZ_F16:
      accum_kernel<LZ_F16><<<G, 256, 0, s>>>(own, tmp, stride, W, me, o1, o2, nvec);
      break;
    default:
      accum_kernel<LZ_BF16><<<G, 256, 0, s>>>(own, tmp, stride, W, me, o1, o2, nvec);
  }
  LZ_CUDA_TRY(cudaGetLastError());
  return LZE_OK;
}

int ce_setup(LzComm* c) {
  if (c->ce_events) return LZE_OK;
  for (int i = 0; i < kCeStreams; ++i)
    LZ_CUDA_TRY(cudaStreamCreateWithFlags(&c->ce_stream[i], cudaStreamNonBlocking));
  cudaEvent_t* ev = new cudaEvent_t[kCeNumEvents];
  for (int i = 0; i < kCeNumEvents; ++i) {
    cudaError_t e = cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming);
    if (e != cudaSuccess) {
      for (int j = 0; j < i; ++j) cudaEventDestroy(ev[j]);
      delete[] ev;
      lz_set_error("cudaEventCreateWithFlags failed: %s", cudaGetErrorString(e));
      return LZE_CUDA;
    }
  }
  c->ce_events = ev;
  c->ce_nevents = kCeNumEvents;
  return LZE_OK;
}

// Zero-copy schedule knobs (environment, read per call). Default: two chunks
// per slice. Every chunk costs a fixed ~20 us (measured on 2 x B200, 1 GiB:
// 16 chunks 1.729 ms, 8 chunks 1.579 ms, 4 chunks 1.493 ms, 2 chunks
// 1.450 ms, 1 chunk 1.735 ms without any overlap), so the fewest chunks that
// still overlap the all-gather of the first chunk with the reduce-scatter of
// the second win.
//   LZ_CE_CHUNK_MB  chunk size in MiB (default: slice / 2);
//   LZ_CE_TAPER     1: the first and last chunks ramp (1/8, 1/4, 1/2 of a
//                   chunk), shortening the pipeline's fill and drain;
//   LZ_CE_FLAGS     1: chunk flags go out on their own stream (after an event
//                   per data copy) so the data copies run back to back;
//   LZ_CE_AG        "sm": at W = 2 the reduce kernel also stores the result
//                   into the peer's output (all-gather by SM peer stores).
struct CeOpts {
  size_t chunk;
  int taper, flag_stream, sm_ag;
};

CeOpts ce_opts() {
  CeOpts o;
  const char* v = getenv("LZ_CE_CHUNK_MB");
  const long long mb = v ? atoll(v) : 0;
  o.chunk = mb > 0 ? (size_t)mb << 20 : 0;  // 0: two chunks per slice
  v = getenv("LZ_CE_TAPER");
  o.taper = v ? atoi(v) : 0;
  v = getenv("LZ_CE_FLAGS");
  o.flag_stream = v ? atoi(v) : 0;
  v = getenv("LZ_CE_AG");
  o.sm_ag = (v && strcmp(v, "sm") == 0) ? 1 : 0;
  return o;
}

// Chunk boundaries of one slice (16-byte multiples, at most kCeMaxChunks):
// `pipes` equal chunks when pipes > 0, else chunks of opt.chunk bytes, with
// optional ramps of 1/8, 1/4, 1/2 chunk at both ends.
int ce_plan(size_t slice, int pipes, const CeOpts& opt, size_t* off, size_t* len) {
  size_t sizes[kCeMaxChunks];
  int n = 0;
  if (pipes > 0) {
    int k = pipes > kCeMaxChunks ? kCeMaxChunks : pipes;
    if ((size_t)k > slice / 16) k = (int)(slice / 16 > 0 ? slice / 16 : 1);
    const size_t cp = (slice / k + 15) / 16 * 16;
    for (size_t o = 0; o < slice && n < kCeMaxChunks; o += cp) sizes[n++] = cp;
  } else {
    size_t cp = opt.chunk ? (opt.chunk + 15) / 16 * 16 : ((slice + 1) / 2 + 15) / 16 * 16;
    if (cp < 16) cp = 16;
    while ((slice + cp - 1) / cp > (size_t)kCeMaxChunks - 6) cp *= 2;
    const size_t ramp[3] = {cp / 8, cp / 4, cp / 2};
    size_t rest = slice;
    int head = 0;
    if (opt.taper && slice >= 4 * cp) {
      for (int i = 0; i < 3; ++i) {
        sizes[n++] = (ramp[i] + 15) / 16 * 16;
        rest -= sizes[n - 1];
      }
      head = 3;
      // the tail ramp is reserved now and appended below
      for (int i = 0; i < 3; ++i) rest -= (ramp[2 - i] + 15) / 16 * 16;
    }
    while (rest > 0) {
      const size_t take = rest < cp ? rest : cp;
      sizes[n++] = take;
      rest -= take;
    }
    if (head)
      for (int i = 0; i < 3; ++i) sizes[n++] = (ramp[2 - i] + 15) / 16 * 16;
  }
  size_t o = 0;
  int m = 0;
  for (int i = 0; i < n && o < slice; ++i) {
    const size_t l = o + sizes[i] <= slice ? sizes[i] : slice - o;
    off[m] = o;
    len[m] = l;
    ++m;
    o += l;
  }
  return m;
}

int ce_twoshot_sym(LzComm* c, const char* in, char* out, size_t bytes, int dtype, int pipes, cudaStream_t s) {
  const int W = c->dev.world, me = c->dev.rank;
  const size_t slice = bytes / W;
  const size_t out_off = lz_comm_heap_offset(c, out, bytes);
  const CeOpts opt = ce_opts();
  size_t coffs[kCeMaxChunks], clens[kCeMaxChunks];
  const int C = ce_plan(slice, pipes, opt, coffs, clens);
  const bool sm_ag = opt.sm_ag && W == 2;
  cudaStream_t rs = c->ce_stream[0], ag = c->ce_stream[1], fs = opt.flag_stream ? c->ce_stream[2] : rs;
  cudaEvent_t* ev = c->ce_events;
  const size_t seq_bytes = sizeof(unsigned long long);
  // peers whose AG lands on a slot holding their own contribution here
  unsigned int red_mask = 0, ag_wait_mask = 0, peers = 0;
  for (int q = 0; q < W; ++q) {
    if (q == me) continue;
    peers |= 1u << q;
    if (q != (me + 1) % W) red_mask |= 1u << q;     // I tell q: "chunk reduced"
    if (me != (q + 1) % W) ag_wait_mask |= 1u << q;  // I wait for q before my AG into q
  }
  // Handshake on the caller's stream: every peer has started this call (its
  // earlier work on its output is done). Waiting here, before any reduce
  // kernel is queued, keeps kernels off the copy streams: the reduce kernels
  // spin on flags that only copy engines set, so they can never hold the SMs
  // that a wait kernel feeding those copies would need.
  ce_begin_kernel<<<1, 32, 0, s>>>(c->dev, c->ce_seq);
  LZ_CUDA_TRY(cudaGetLastError());
  ce_wait_kernel<<<1, 32, 0, s>>>(c->dev, kCeArStarted, 1, 0, c->ce_seq, peers, 21);
  LZ_CUDA_TRY(cudaGetLastError());
  LZ_CUDA_TRY(cudaEventRecord(ev[kCeEvBegin], s));
  // RS: data copies on side stream 0, chunk flags after them (same stream, or
  // the flag stream after a per-chunk event)
  LZ_CUDA_TRY(cudaStreamWaitEvent(rs, ev[kCeEvBegin], 0));
  if (fs != rs) LZ_CUDA_TRY(cudaStreamWaitEvent(fs, ev[kCeEvBegin], 0));
  for (int k = 0; k < C; ++k) {
    for (int j = 1; j < W; ++j) {
      const int q = (me + j) % W;
      char* dst = c->dev.heap[q] + out_off + (size_t)(me == (q + 1) % W ? q : me) * slice + coffs[k];
      LZ_CUDA_TRY(cudaMemcpyAsync(dst, in + (size_t)q * slice + coffs[k], clens[k], cudaMemcpyDeviceToDevice, rs));
    }
    if (fs != rs) {
      LZ_CUDA_TRY(cudaEventRecord(ev[kCeEvCopied + k], rs));
      LZ_CUDA_TRY(cudaStreamWaitEvent(fs, ev[kCeEvCopied + k], 0));
    }
    for (int j = 1; j < W; ++j) {
      const int q = (me + j) % W;
      char* f = c->dev.heap[q] + kCeArRs + 8u * ((size_t)me * kCeMaxChunks + k);
      LZ_CUDA_TRY(cudaMemcpyAsync(f, c->ce_seq, seq_bytes, cudaMemcpyDeviceToDevice, fs));
    }
  }
  LZ_CUDA_TRY(cudaEventRecord(ev[kCeEvRsEnd], rs));
  if (fs != rs) LZ_CUDA_TRY(cudaEventRecord(ev[kCeEvFlagEnd], fs));
  // reduce on the caller's stream; AG by copies on side stream 1 (or by the
  // reduce kernel's own peer stores)
  const int G = c->sm_count > 0 ? c->sm_count : 148;
  for (int k = 0; k < C; ++k) {
    CeRedParams p;
    p.in = in;
    p.out = out;
    p.slice = slice;
    p.coff = coffs[k];
    p.clen = clens[k];
    p.chunk = k;
    p.red_mask = red_mask;
    p.seq_ctr = c->ce_seq;
    p.done = c->ce_done;
    p.peer_out = sm_ag ? c->dev.heap[1 - me] + out_off : nullptr;
    p.last = k == C - 1;
    int rc;
    switch (dtype) {
      case LZ_F32: rc = launch_reduce<LZ_F32>(c, p, G, s); break;
      case LZ_F16: rc = launch_reduce<LZ_F16>(c, p, G, s); break;
      default: rc = launch_reduce<LZ_BF16>(c, p, G, s);
    }
    if (rc) return rc;
    if (sm_ag) continue;
    LZ_CUDA_TRY(cudaEventRecord(ev[kCeEvRed + k], s));
    LZ_CUDA_TRY(cudaStreamWaitEvent(ag, ev[kCeEvRed + k], 0));
    if (ag_wait_mask) {
      ce_wait_kernel<<<1, 32, 0, ag>>>(c->dev, kCeArRed, kCeMaxChunks, k, c->ce_seq, ag_wait_mask, 22);
      LZ_CUDA_TRY(cudaGetLastError());
    }
    for (int j = 1; j < W; ++j) {
      const int q = (me + j) % W;
      const size_t o = (size_t)me * slice + coffs[k];
      LZ_CUDA_TRY(cudaMemcpyAsync(c->dev.heap[q] + out_off + o, out + o, clens[k], cudaMemcpyDeviceToDevice, ag));
    }
  }
  if (!sm_ag) {
    for (int j = 1; j < W; ++j) {
      const int q = (me + j) % W;
      LZ_CUDA_TRY(cudaMemcpyAsync(c->dev.heap[q] + kCeArDone + 8u * me, c->ce_seq, seq_bytes,
                                  cudaMemcpyDeviceToDevice, ag));
    }
    LZ_CUDA_TRY(cudaEventRecord(ev[kCeEvAgEnd], ag));
    LZ_CUDA_TRY(cudaStreamWaitEvent(s, ev[kCeEvAgEnd], 0));
  }
  LZ_CUDA_TRY(cudaStreamWaitEvent(s, ev[kCeEvRsEnd], 0));
  if (fs != rs) LZ_CUDA_TRY(cudaStreamWaitEvent(s, ev[kCeEvFlagEnd], 0));
  // every peer's AG into my output has landed
  ce_wait_kernel<<<1, 32, 0, s>>>(c->dev, kCeArDone, 1, 0, c->ce_seq, peers, 23);
  LZ_CUDA_TRY(cudaGetLastError());
  return LZE_OK;
}

int ce_staged(LzComm* c, const void* in, void* out, size_t bytes, int dtype, int pipes, cudaStream_t s) {
  const int W = c->dev.world, me = c->dev.rank;
  const size_t slice = bytes / W;
  const size_t need = bytes + slice + (size_t)W * slice;
  if (need > c->stage_bytes) {
    lz_set_error("copy-engine allreduce: stage needs %zu bytes, have %zu", need, c->stage_bytes);
    return LZE_ARG;
  }
  // at most one event per piece; every piece a multiple of 16 bytes
  if (pipes < 1) pipes = 1;
  if (pipes > kCeMaxChunks) pipes = kCeMaxChunks;
  while (pipes > 1 && (slice / pipes) % 16) --pipes;
  const int np = pipes;
  const size_t piece = slice / np;
  cudaStream_t s2 = c->ce_stream[0];
  cudaEvent_t* ev = c->ce_events;
  char* my = c->dev.heap[me];
  const size_t in_off = c->stage_off;     // full copy of my input
  const size_t res_off = in_off + bytes;  // my reduced slice
  const size_t tmp_off = res_off + slice;  // W temp slices (peer copies)
  LZ_CUDA_TRY(cudaMemcpyAsync(my + in_off, in, bytes, cudaMemcpyDeviceToDevice, s));
  int rc = lz_barrier(c, s);
  if (rc) return rc;
  LZ_CUDA_TRY(cudaEventRecord(ev[kCeEvBegin], s));
  LZ_CUDA_TRY(cudaStreamWaitEvent(s2, ev[kCeEvBegin], 0));
  // RS: copy engines fetch my slice from every peer (pipelined), SMs accumulate
  for (int k = 0; k < np; ++k) {
    const size_t off = (size_t)me * slice + (size_t)k * piece;
    const size_t len = (k == np - 1) ? slice - (size_t)k * piece : piece;
    for (int j = 1; j < W; ++j) {
      const int p = (me + j) % W;
      LZ_CUDA_TRY(cudaMemcpyAsync(my + tmp_off + (size_t)p * slice + (size_t)k * piece,
                                  c->dev.heap[p] + in_off + off, len, cudaMemcpyDeviceToDevice, s2));
    }
    LZ_CUDA_TRY(cudaEventRecord(ev[kCeEvRed + k], s2));
    LZ_CUDA_TRY(cudaStreamWaitEvent(s, ev[kCeEvRed + k], 0));
    const size_t nvec = len / 16;
    const int G = (int)((nvec + 255) / 256 < 1184 ? (nvec + 255) / 256 : 1184);
    rc = launch_accum(dtype, G > 0 ? G : 1, s, static_cast<const char*>(in) + off, my + tmp_off + (size_t)k * piece,
                      slice, W, me, static_cast<char*>(out) + off, my + res_off + (size_t)k * piece, nvec);
    if (rc) return rc;
  }
  rc = lz_barrier(c, s);
  if (rc) return rc;
  // AG: copy engines fetch every peer's reduced slice into my output
  LZ_CUDA_TRY(cudaEventRecord(ev[kCeEvBegin], s));
  LZ_CUDA_TRY(cudaStreamWaitEvent(s2, ev[kCeEvBegin], 0));
  for (int j = 1; j < W; ++j) {
    const int p = (me + j) % W;
    LZ_CUDA_TRY(cudaMemcpyAsync(static_cast<char*>(out) + (size_t)p * slice, c->dev.heap[p] + res_off, slice,
                                cudaMemcpyDeviceToDevice, s2));
  }
  LZ_CUDA_TRY(cudaEventRecord(ev[kCeEvAgEnd], s2));
  LZ_CUDA_TRY(cudaStreamWaitEvent(s, ev[kCeEvAgEnd], 0));
  // nobody may overwrite a result slice before every peer has copied it
  return lz_barrier(c, s);
}

}  // namespace

void lz_ce_release(LzComm* c) {
  if (c->ce_events) {
    for (int i = 0; i < c->ce_nevents; ++i) cudaEventDestroy(c->ce_events[i]);
    delete[] c->ce_events;
    c->ce_events = nullptr;
  }
  for (int i = 0; i < kCeStreams; ++i) {
    if (c->ce_stream[i]) cudaStreamDestroy(c->ce_stream[i]);
    c->ce_stream[i] = nullptr;
  }
}

// Returns 1 when (in, out) take the zero-copy pipelined path.
extern "C" int lz_ce_allreduce_is_zero_copy(LzComm* c, const void* in, const void* out, size_t count, int dtype) {
  const int W = c->dev.world;
  const size_t bytes = count * (dtype == LZ_F32 ? 4 : 2);
  if (W < 2 || bytes == 0 || bytes % (16 * (size_t)W)) return 0;
  if (lz_comm_heap_offset(c, in, bytes) == (size_t)-1 || lz_comm_heap_offset(c, out, bytes) == (size_t)-1)
    return 0;
  const char* a = static_cast<const char*>(in);
  const char* b = static_cast<const char*>(out);
  return (a + bytes <= b || b + bytes <= a) ? 1 : 0;
}

// in/out: device buffers of count elements. Symmetric, distinct in/out take
// the zero-copy pipelined path (pipes = chunks per slice, 0 = automatic);
// anything else the staged path through the communicator stage
// ([my input | my result slice | W temp slices]). The caller's stream `s` is
// ordered after all of the call's work when this returns.
extern "C" int lz_ce_allreduce(LzComm* c, const void* in, void* out, size_t count, int dtype, int pipes,
                               cudaStream_t s) {
  const int W = c->dev.world;
  if (dtype != LZ_F32 && dtype != LZ_F16 && dtype != LZ_BF16) {
    lz_set_error("copy-engine allreduce: unsupported dtype %d", dtype);
    return LZE_ARG;
  }
  if (pipes < 0) {
    lz_set_error("copy-engine allreduce: pipes must be >= 0 (got %d)", pipes);
    return LZE_ARG;
  }
  const size_t es = dtype == LZ_F32 ? 4 : 2;
  const size_t bytes = count * es;
  if (W == 1) {
    if (in != out) LZ_CUDA_TRY(cudaMemcpyAsync(out, in, bytes, cudaMemcpyDeviceToDevice, s));
    return LZE_OK;
  }
  if (bytes % (16 * (size_t)W) || (uintptr_t)in % 16 || (uintptr_t)out % 16) {
    lz_set_error("copy-engine allreduce: size must be a multiple of 16 * world bytes and pointers 16-byte aligned");
    return LZE_ARG;
  }
  int rc = ce_setup(c);
  if (rc) return rc;
  if (lz_ce_allreduce_is_zero_copy(c, in, out, count, dtype))
    return ce_twoshot_sym(c, static_cast<const char*>(in), static_cast<char*>(out), bytes, dtype, pipes, s);
  return ce_staged(c, in, out, bytes, dtype, pipes > 0 ? pipes : 4, s);
}
