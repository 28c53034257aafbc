// Device-side LZC1 table-group (TG) encoder and decoder, used by the
// standalone codec kernels (lz_codec.cu) and by the fused transfer kernels
// (compressed allreduce, weight transfer), which write/read records directly
// in peer or multicast memory.
//
// One CTA of LZC_THREADS = 8 warps handles one TG (8 sub-blocks of 4096
// symbols, one warp per sub-block). Output is bit-identical to the CPU oracle
// (csrc/cpu/lz_cpu.cpp).
//
// Reference behaviour being re-designed: the dietgpu float codec the
// reference calls as a closed library (exponent byte ANS-coded with local
// tables, sign/mantissa raw; ratios and GB/s in raw/dietgpu_walltime_*.csv,
// local vs global tables in plot/local_frequency_compression_ratio.py:9-19).
#pragma once
#include "lz_codec_format.h"
#include "lz_common.cuh"

namespace lzg {

using namespace lzc;
constexpr int LZC_THREADS = 256;  // one warp per sub-block
constexpr int LZC_MIN_BLOCKS = 3;  // 3 CTAs (24 warps) per SM: caps registers at 85
constexpr int HREP = 4;            // histogram replicas per warp (lane & 3)
constexpr int HSTRIDE = 256 + 8;   // replica stride in words: bin s of replica r sits in bank (s + 8r) % 32
static_assert(LZC_THREADS / 32 == NSUB, "one warp per sub-block");

struct EncSmem {
  uint8_t syms[TG_ELEMS];  // symbol plane of the TG
  union {
    uint8_t streams[NSUB][SUB_ELEMS];     // per-warp rANS output (states + words)
    uint32_t counts[NSUB][HREP][HSTRIDE];  // per-warp histograms, HREP replicas (before encoding)
  } u;
  uint32_t hist[256];                     // reduced histogram
  EncSym tab[256];
  uint32_t table[256];
  uint32_t sub_len[NSUB];
  uint32_t nnz;
  uint32_t total;
  // PACK level
  uint8_t codemap[256];  // symbol -> code
  alignas(16) uint8_t ptab[16];  // code -> symbol (table section), read as one 16-byte vector
  uint32_t topc[16];     // counts of the table candidates
  int pk_bits;           // chosen code width, -1 = RAW
  uint32_t pk_nnz, pk_nesc, pk_bytes;
  unsigned long long esc_part[NSUB];  // per-warp sums of the escape scan
};

static_assert(offsetof(EncSmem, ptab) % 16 == 0 && offsetof(EncSmem, syms) % 16 == 0,
              "vector accesses of the PACK encoder");

struct DecSmem {
  uint32_t dtab[PROB_SCALE];
  uint8_t syms[TG_ELEMS];
  uint8_t sec[TG_ELEMS];  // staged ANS symbol section (table, sizes, sub-streams)
  uint32_t cum[257];      // cumulative frequencies of the table entries
  uint32_t ent[256];      // table entries (sym << 16 | freq)
  TgHeader h;
  int ok;
  alignas(8) uint64_t bar;  // mbarrier of the bulk copy that stages `sec`
  unsigned long long esc_part[NSUB];  // per-warp sums of the PACK escape scan
};
static_assert(offsetof(DecSmem, syms) % 16 == 0, "vector accesses of the decoders");

LZ_DEV uint32_t lane_id() { return threadIdx.x & 31; }
LZ_DEV uint32_t lanemask_lt() {
  uint32_t m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

// ---------------------------------------------------------------------------
// split of 16 elements (one "unit") into 16 symbol bytes and the raw plane,
// as 32-bit words: symbol k is byte k % 4 of sw[k / 4]; the raw bytes of the
// unit (RAW_BYTES of them, in element order) are rw[0 .. RAW_BYTES / 4).
// Two 16-bit elements are processed per word operation (bf16, fp16).
// ---------------------------------------------------------------------------
// two 2-byte lanes (bytes 0 and 2 of a and b) -> one word of 4 bytes
LZ_DEV uint32_t pick_even_bytes(uint32_t a, uint32_t b) { return __byte_perm(a, b, 0x6420); }
// bytes 0, 1 (or 2, 3) of x -> bytes 0 and 2 of the result, zero elsewhere
LZ_DEV uint32_t spread_lo(uint32_t x) { return __byte_perm(x, 0u, 0x4140); }
LZ_DEV uint32_t spread_hi(uint32_t x) { return __byte_perm(x, 0u, 0x4342); }
LZ_DEV uint32_t word_of(const uint4& v, int i) { return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w)); }

template <int DT>
struct Split16;

template <>
struct Split16<DT_BF16> {
  static constexpr int IN_VECS = 2, RAW_BYTES = 16, RW = 4;
  // symbol = bits 14..7; raw = sign (bit 15) << 7 | mantissa (bits 6..0), per 16-bit lane
  LZ_DEV static void split(const uint4 (&v)[IN_VECS], uint32_t (&sw)[4], uint32_t (&rw)[RW]) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t a = word_of(v[j / 2], 2 * (j % 2)), b = word_of(v[j / 2], 2 * (j % 2) + 1);
      const uint32_t sa = (a >> 7) & 0x00FF00FFu, sb = (b >> 7) & 0x00FF00FFu;
      const uint32_t ra = ((a >> 8) & 0x00800080u) | (a & 0x007F007Fu);
      const uint32_t rb = ((b >> 8) & 0x00800080u) | (b & 0x007F007Fu);
      sw[j] = pick_even_bytes(sa, sb);
      rw[j] = pick_even_bytes(ra, rb);
    }
  }
  LZ_DEV static uint32_t merge2(uint32_t s2, uint32_t r2) {
    return ((r2 & 0x00800080u) << 8) | (s2 << 7) | (r2 & 0x007F007Fu);
  }
  LZ_DEV static void merge(const uint32_t (&sw)[4], const uint32_t (&rw)[RW], uint4 (&v)[IN_VECS]) {
    uint32_t o[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      o[2 * j] = merge2(spread_lo(sw[j]), spread_lo(rw[j]));
      o[2 * j + 1] = merge2(spread_hi(sw[j]), spread_hi(rw[j]));
    }
    v[0] = make_uint4(o[0], o[1], o[2], o[3]);
    v[1] = make_uint4(o[4], o[5], o[6], o[7]);
  }
};
template <>
struct Split16<DT_F16> {
  static constexpr int IN_VECS = 2, RAW_BYTES = 16, RW = 4;
  // symbol = high byte (sign, exponent, 2 mantissa bits); raw = low byte
  LZ_DEV static void split(const uint4 (&v)[IN_VECS], uint32_t (&sw)[4], uint32_t (&rw)[RW]) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t a = word_of(v[j / 2], 2 * (j % 2)), b = word_of(v[j / 2], 2 * (j % 2) + 1);
      sw[j] = __byte_perm(a, b, 0x7531);
      rw[j] = __byte_perm(a, b, 0x6420);
    }
  }
  LZ_DEV static void merge(const uint32_t (&sw)[4], const uint32_t (&rw)[RW], uint4 (&v)[IN_VECS]) {
    uint32_t o[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      o[2 * j] = __byte_perm(rw[j], sw[j], 0x5140);
      o[2 * j + 1] = __byte_perm(rw[j], sw[j], 0x7362);
    }
    v[0] = make_uint4(o[0], o[1], o[2], o[3]);
    v[1] = make_uint4(o[4], o[5], o[6], o[7]);
  }
};
template <>
struct Split16<DT_F32> {
  // raw plane: 3 little-endian bytes per element; four elements' 24-bit raws
  // fill three 32-bit words exactly (r0 | r1 << 24, r1 >> 8 | r2 << 16,
  // r2 >> 16 | r3 << 8), so the packing is done with word shifts
  static constexpr int IN_VECS = 4, RAW_BYTES = 48, RW = 12;
  LZ_DEV static void split(const uint4 (&v)[IN_VECS], uint32_t (&sw)[4], uint32_t (&rw)[RW]) {
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const uint32_t w0 = v[g].x, w1 = v[g].y, w2 = v[g].z, w3 = v[g].w;
      sw[g] = (uint32_t)sym_f32(w0) | ((uint32_t)sym_f32(w1) << 8) | ((uint32_t)sym_f32(w2) << 16) |
              ((uint32_t)sym_f32(w3) << 24);
      const uint32_t r0 = raw_f32(w0), r1 = raw_f32(w1), r2 = raw_f32(w2), r3 = raw_f32(w3);
      rw[3 * g] = r0 | (r1 << 24);
      rw[3 * g + 1] = (r1 >> 8) | (r2 << 16);
      rw[3 * g + 2] = (r2 >> 16) | (r3 << 8);
    }
  }
  LZ_DEV static void merge(const uint32_t (&sw)[4], const uint32_t (&rw)[RW], uint4 (&v)[IN_VECS]) {
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const uint32_t a = rw[3 * g], b = rw[3 * g + 1], c = rw[3 * g + 2], s = sw[g];
      v[g].x = merge_f32((uint8_t)s, a & 0xFFFFFFu);
      v[g].y = merge_f32((uint8_t)(s >> 8), (a >> 24) | ((b & 0xFFFFu) << 8));
      v[g].z = merge_f32((uint8_t)(s >> 16), (b >> 16) | ((c & 0xFFu) << 16));
      v[g].w = merge_f32((uint8_t)(s >> 24), c >> 8);
    }
  }
};
template <>
struct Split16<DT_U8> {
  static constexpr int IN_VECS = 1, RAW_BYTES = 0, RW = 1;
  LZ_DEV static void split(const uint4 (&v)[IN_VECS], uint32_t (&sw)[4], uint32_t (&rw)[RW]) {
    sw[0] = v[0].x, sw[1] = v[0].y, sw[2] = v[0].z, sw[3] = v[0].w;
    rw[0] = 0;
  }
  LZ_DEV static void merge(const uint32_t (&sw)[4], const uint32_t (&)[RW], uint4 (&v)[IN_VECS]) {
    v[0] = make_uint4(sw[0], sw[1], sw[2], sw[3]);
  }
};

template <int DT>
struct SplitPair16 {  // 16 fp8 pairs (32 bytes) <-> 16 container elements
  static constexpr int IN_VECS = 2, RAW_BYTES = 16, RW = 4;
  LZ_DEV static void split(const uint4 (&v)[IN_VECS], uint32_t (&sw)[4], uint32_t (&rw)[RW]) {
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const uint32_t w = word_of(v[k / 8], (k % 8) / 2);
      const uint8_t a = (uint8_t)(w >> (16 * (k % 2))), b = (uint8_t)(w >> (16 * (k % 2) + 8));
      const uint16_t u = DT == DT_E4M3P ? pack_e4m3(a, b) : pack_e5m2(a, b);
      if (k % 4 == 0) sw[k / 4] = 0, rw[k / 4] = 0;
      sw[k / 4] |= (uint32_t)sym_bf16(u) << (8 * (k % 4));
      rw[k / 4] |= (uint32_t)raw_bf16(u) << (8 * (k % 4));
    }
  }
  LZ_DEV static void merge(const uint32_t (&sw)[4], const uint32_t (&rw)[RW], uint4 (&v)[IN_VECS]) {
    uint32_t o[8];
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const uint16_t u = merge_bf16((uint8_t)(sw[k / 4] >> (8 * (k % 4))), (uint8_t)(rw[k / 4] >> (8 * (k % 4))));
      uint8_t a, b;
      if (DT == DT_E4M3P) unpack_e4m3(u, &a, &b);
      else unpack_e5m2(u, &a, &b);
      const uint32_t pair = (uint32_t)a | ((uint32_t)b << 8);
      if (k % 2 == 0) o[k / 2] = pair;
      else o[k / 2] |= pair << 16;
    }
    v[0] = make_uint4(o[0], o[1], o[2], o[3]);
    v[1] = make_uint4(o[4], o[5], o[6], o[7]);
  }
};
template <>
struct Split16<DT_E4M3P> : SplitPair16<DT_E4M3P> {};
template <>
struct Split16<DT_E5M2P> : SplitPair16<DT_E5M2P> {};

// Scalar split/merge of element i (tails).
template <int DT>
LZ_DEV void split1(const char* in, uint32_t i, uint8_t* sym, uint8_t* raw) {
  if (DT == DT_BF16) {
    uint16_t u = reinterpret_cast<const uint16_t*>(in)[i];
    *sym = sym_bf16(u);
    raw[0] = raw_bf16(u);
  } else if (DT == DT_F16) {
    uint16_t u = reinterpret_cast<const uint16_t*>(in)[i];
    *sym = sym_f16(u);
    raw[0] = raw_f16(u);
  } else if (DT == DT_F32) {
    uint32_t u = reinterpret_cast<const uint32_t*>(in)[i];
    *sym = sym_f32(u);
    uint32_t r = raw_f32(u);
    raw[0] = (uint8_t)r;
    raw[1] = (uint8_t)(r >> 8);
    raw[2] = (uint8_t)(r >> 16);
  } else if (DT == DT_E4M3P || DT == DT_E5M2P) {
    const uint8_t a = reinterpret_cast<const uint8_t*>(in)[2 * i];
    const uint8_t b = reinterpret_cast<const uint8_t*>(in)[2 * i + 1];
    const uint16_t u = DT == DT_E4M3P ? pack_e4m3(a, b) : pack_e5m2(a, b);
    *sym = sym_bf16(u);
    raw[0] = raw_bf16(u);
  } else {
    *sym = reinterpret_cast<const uint8_t*>(in)[i];
  }
}

template <int DT>
LZ_DEV void merge1(char* out, uint32_t i, uint8_t sym, const uint8_t* raw) {
  if (DT == DT_BF16) {
    reinterpret_cast<uint16_t*>(out)[i] = merge_bf16(sym, raw[0]);
  } else if (DT == DT_F16) {
    reinterpret_cast<uint16_t*>(out)[i] = merge_f16(sym, raw[0]);
  } else if (DT == DT_F32) {
    uint32_t r = raw[0] | ((uint32_t)raw[1] << 8) | ((uint32_t)raw[2] << 16);
    reinterpret_cast<uint32_t*>(out)[i] = merge_f32(sym, r);
  } else if (DT == DT_E4M3P || DT == DT_E5M2P) {
    uint8_t* o = reinterpret_cast<uint8_t*>(out);
    const uint16_t u = merge_bf16(sym, raw[0]);
    if (DT == DT_E4M3P) unpack_e4m3(u, &o[2 * i], &o[2 * i + 1]);
    else unpack_e5m2(u, &o[2 * i], &o[2 * i + 1]);
  } else {
    reinterpret_cast<uint8_t*>(out)[i] = sym;
  }
}

// Copies `bytes` (multiple of 16, both 16-B aligned) with the whole CTA.
LZ_DEV void cta_copy16(char* dst, const char* src, uint32_t bytes) {
  for (uint32_t o = threadIdx.x * 16; o < bytes; o += blockDim.x * 16)
    st_v4(dst + o, *reinterpret_cast<const uint4*>(src + o));
}

// ---------------------------------------------------------------------------
// Frequency table (warp 0): counts -> freq -> cumulative -> encoder table and
// the compact list of (sym << 16 | freq). Same result as normalize_freqs().
// ---------------------------------------------------------------------------
// Reciprocals of every frequency 1..PROB_SCALE, built at compile time with
// the same formula as make_enc_sym (so the entries are identical): the table
// build then loads them instead of running a 64-bit division per symbol.
struct RcpTable {
  uint32_t m_lo[PROB_SCALE + 1];
  uint8_t shift[PROB_SCALE + 1];
};
constexpr RcpTable make_rcp_table() {
  RcpTable t{};
  for (uint32_t f = 1; f <= PROB_SCALE; ++f) {
    uint32_t l = 0;
    while ((1u << l) < f) ++l;
    t.shift[f] = (uint8_t)l;
    t.m_lo[f] = (uint32_t)((((uint64_t)1 << (32 + l)) + f - 1) / f - ((uint64_t)1 << 32));
  }
  return t;
}
__device__ constexpr RcpTable kRcp = make_rcp_table();

LZ_DEV EncSym enc_sym_from_table(uint32_t f, uint32_t cum) {
  EncSym e;
  e.freq = f;
  e.cum = cum;
  e.shift = kRcp.shift[f];
  e.m_lo = kRcp.m_lo[f];
  return e;
}

LZ_DEV void build_tables_warp0(EncSmem& sm, uint32_t n) {
  const uint32_t lane = lane_id();
  uint32_t c[8], f[8];
  uint32_t sum = 0, maxc = 0;
  int argmax = 256;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int s = lane * 8 + k;
    c[k] = sm.hist[s];
    f[k] = 0;
    if (c[k]) {
      // c <= n <= 32768: the product fits 32 bits; a full TG divides by 2^15
      f[k] = (n & (n - 1)) == 0 ? (c[k] * PROB_SCALE) >> (31 - __clz(n)) : (c[k] * PROB_SCALE) / n;
      if (f[k] == 0) f[k] = 1;
      if (c[k] > maxc) {
        maxc = c[k];
        argmax = s;
      }
    }
    sum += f[k];
  }
  // warp reductions: total, and (max count, smallest symbol)
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    uint32_t oc = __shfl_xor_sync(0xffffffffu, maxc, o);
    int oa = __shfl_xor_sync(0xffffffffu, argmax, o);
    if (oc > maxc || (oc == maxc && oa < argmax)) {
      maxc = oc;
      argmax = oa;
    }
  }
  if (maxc > 0) {
    if (sum < PROB_SCALE) {
      if (argmax / 8 == (int)lane) f[argmax % 8] += PROB_SCALE - sum;
    } else {
      while (sum > PROB_SCALE) {  // rare: take the excess from the largest frequency
        uint32_t bf = 1;
        int best = 256;
#pragma unroll
        for (int k = 0; k < 8; ++k)
          if (f[k] > bf) {
            bf = f[k];
            best = lane * 8 + k;
          }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          uint32_t ob = __shfl_xor_sync(0xffffffffu, bf, o);
          int os = __shfl_xor_sync(0xffffffffu, best, o);
          if (ob > bf || (ob == bf && os < best)) {
            bf = ob;
            best = os;
          }
        }
        uint32_t d = sum - PROB_SCALE;
        if (d > bf - 1) d = bf - 1;
        if (best / 8 == (int)lane) f[best % 8] -= d;
        sum -= d;
      }
    }
  }
  // exclusive prefix over symbols (8 per lane, lanes in order)
  uint32_t lsum = 0, lnz = 0;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    lsum += f[k];
    lnz += f[k] ? 1u : 0u;
  }
  uint32_t incl = lsum, inz = lnz;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    uint32_t a = __shfl_up_sync(0xffffffffu, incl, o);
    uint32_t b = __shfl_up_sync(0xffffffffu, inz, o);
    if (lane >= (uint32_t)o) {
      incl += a;
      inz += b;
    }
  }
  uint32_t cum = incl - lsum, pos = inz - lnz;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int s = lane * 8 + k;
    if (f[k]) {
      sm.tab[s] = enc_sym_from_table(f[k], cum);
      sm.table[pos++] = ((uint32_t)s << 16) | f[k];
    }
    cum += f[k];
  }
  if (lane == 31) sm.nnz = inz;
}

// ---------------------------------------------------------------------------
// Interleaved rANS of one sub-block (sn <= SUB_ELEMS symbols at sm.syms[base])
// by one warp, backward over the steps: lane l owns symbols l, l+32, ...;
// renormalisation words of a step are written in lane order after the 128-byte
// state area. Returns false when the words would not beat the raw bytes.
// kFull: sn == SUB_ELEMS, so every step has all 32 lanes active.
// ---------------------------------------------------------------------------
template <bool kFull>
LZ_DEV bool rans_encode_sub(EncSmem& sm, uint32_t base, uint32_t sn, uint32_t warp, uint32_t lane,
                            uint32_t& x_out, uint32_t& pos_out) {
  if (sn < 128u) return false;  // the 32 states alone do not beat the raw bytes
  uint16_t* words = reinterpret_cast<uint16_t*>(sm.u.streams[warp] + 128);
  const uint32_t lim = (sn - 128u) / 2u;  // words that still beat the raw bytes
  uint32_t x = RANS_L;
  uint32_t pos = 0;  // words emitted (warp-uniform)
  const int jmax = (int)((sn + LANES - 1) / LANES) - 1;
  const uint32_t lt = lanemask_lt();
  const uint8_t* syms = sm.syms + base + lane;
  // software-pipelined: the table entry of step j-1 is fetched while step j runs
  EncSym e_next;
  if (kFull || (uint32_t)jmax * LANES + lane < sn) e_next = sm.tab[syms[(uint32_t)jmax * LANES]];
  for (int j = jmax; j >= 0; --j) {
    const bool act = kFull || (uint32_t)j * LANES + lane < sn;
    const EncSym e = e_next;
    if (j > 0) e_next = sm.tab[syms[(uint32_t)(j - 1) * LANES]];
    const bool need = act && enc_needs_word(x, e.freq);
    const uint32_t m = __ballot_sync(0xffffffffu, need);
    const uint32_t cnt = __popc(m);
    if (pos + cnt > lim) return false;
    if (need) {
      words[pos + __popc(m & lt)] = (uint16_t)(x & 0xFFFF);
      x >>= 16;
    }
    pos += cnt;
    if (act) x = enc_update(x, e);
  }
  x_out = x;
  pos_out = pos;
  return true;
}

// ---------------------------------------------------------------------------
// PACK level (layout in lz_codec_format.h): a table of the <= 15 most frequent
// symbols, b-bit codes in groups of 32 elements, escaped symbols in order.
// A few integer operations per element on both sides, no serial state.
// ---------------------------------------------------------------------------
LZ_DEV void write_tg_header(char* dst, uint8_t mode, uint8_t dt, uint32_t n, uint32_t sym_bytes,
                            uint32_t raw_bytes, uint32_t nnz, uint32_t nsub, uint32_t reserved) {
  TgHeader h;
  h.magic = TG_MAGIC;
  h.version = VERSION;
  h.mode = mode;
  h.dtype = dt;
  h.n = n;
  h.sym_bytes = sym_bytes;
  h.raw_bytes = raw_bytes;
  h.nnz = (uint16_t)nnz;
  h.nsub = (uint16_t)nsub;
  h.total = (uint32_t)sizeof(TgHeader) + raw_bytes + sym_bytes;
  h.reserved = reserved;
  const uint4* hv = reinterpret_cast<const uint4*>(&h);
  st_v4(dst, hv[0]);
  st_v4(dst + 16, hv[1]);
}

// Warp 0: the table (count descending, then symbol ascending: the key
// count << 8 | (255 - sym) orders both at once), the code width, and the
// symbol -> code map.
LZ_DEV void pack_tables_warp0(EncSmem& sm, uint32_t n) {
  const uint32_t lane = lane_id();
  uint32_t key[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const uint32_t s = lane * 8 + k, c = sm.hist[s];
    key[k] = c ? (c << 8) | (255u - s) : 0u;
  }
  uint32_t ntop = 0;
  for (uint32_t r = 0; r < 15; ++r) {
    uint32_t m = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) m = max(m, key[k]);
    m = __reduce_max_sync(0xffffffffu, m);
    if (m == 0) break;  // warp-uniform
    const uint32_t s = 255u - (m & 0xFFu);
#pragma unroll
    for (int k = 0; k < 8; ++k)
      if (lane * 8 + k == s) key[k] = 0;
    if (lane == 0) {
      sm.ptab[r] = (uint8_t)s;
      sm.topc[r] = m >> 8;
    }
    ntop = r + 1;
  }
  __syncwarp();
  if (lane == 0) {
    const PackChoice pc = pack_choose(sm.topc, ntop, n);
    sm.pk_bits = pc.bits;
    sm.pk_nnz = pc.nnz;
    sm.pk_nesc = pc.nesc;
    sm.pk_bytes = pc.bytes;
  }
  __syncwarp();
  const int bits = sm.pk_bits;
  const uint32_t nnz = sm.pk_nnz;
  const uint8_t esc = bits > 0 ? (uint8_t)((1u << bits) - 1u) : 0;
#pragma unroll
  for (int k = 0; k < 8; ++k) sm.codemap[lane * 8 + k] = esc;
  uint8_t t = 0;
  if (lane < 16) t = lane < nnz ? sm.ptab[lane] : 0;
  __syncwarp();
  if (lane < 16) sm.ptab[lane] = t;
  if (lane < nnz) sm.codemap[t] = (uint8_t)lane;
}

// Exclusive block scan of per-thread escape counts of up to 4 groups, packed
// as 16-bit lanes of a u64 (a TG has <= 1024 groups, so a lane sums to at
// most 8192). *tot receives the block totals (same lanes).
LZ_DEV unsigned long long esc_scan(unsigned long long v, unsigned long long* part,
                                   unsigned long long* tot) {
  const uint32_t lane = lane_id(), warp = threadIdx.x >> 5;
  unsigned long long incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= (uint32_t)o) incl += t;
  }
  if (lane == 31) part[warp] = incl;
  __syncthreads();
  unsigned long long before = 0, all = 0;
  const uint32_t nw = blockDim.x >> 5;
  for (uint32_t w = 0; w < nw; ++w) {
    const unsigned long long p = part[w];
    if (w < warp) before += p;
    all += p;
  }
  *tot = all;
  return before + incl - v;
}
LZ_DEV uint32_t lane16(unsigned long long v, int i) { return (uint32_t)(v >> (16 * i)) & 0xFFFFu; }

// Codes of group g (32 symbols in shared memory) -> w[0..B); returns the
// escape mask (bit k: element k of the group is escaped).
template <int B>
LZ_DEV uint32_t pack_group(const EncSmem& sm, uint32_t g, uint32_t n, uint32_t (&w)[4]) {
  constexpr uint32_t ESC = (1u << B) - 1u;
  uint4 sv[2];
  sv[0] = *reinterpret_cast<const uint4*>(&sm.syms[g * PACK_GROUP]);
  sv[1] = *reinterpret_cast<const uint4*>(&sm.syms[g * PACK_GROUP + 16]);
  const uint8_t* sy = reinterpret_cast<const uint8_t*>(sv);
  const uint32_t lim = n - g * PACK_GROUP;  // >= 1; elements past n take code 0
#pragma unroll
  for (int q = 0; q < 4; ++q) w[q] = 0;
  uint32_t em = 0;
#pragma unroll
  for (int k = 0; k < 32; ++k) {
    const uint32_t c = (uint32_t)k < lim ? (uint32_t)sm.codemap[sy[k]] : 0u;
    em |= (c == ESC ? 1u : 0u) << k;
    const int bit = k * B, wi = bit >> 5, sh = bit & 31;
    w[wi] |= c << sh;
    if (sh + B > 32) w[wi + 1] |= c >> (32 - sh);
  }
  return em;
}

template <int B>
LZ_DEV void pack_emit_codes(EncSmem& sm, uint32_t n, char* symsec) {
  const uint32_t tid = threadIdx.x;
  const uint32_t G = pack_groups(n);
  char* codes = symsec + PACK_TABLE_BYTES;
  char* escs = codes + pad16(G * 4u * B);
  uint32_t em[4] = {0, 0, 0, 0};
  unsigned long long cnt = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t g = tid + (uint32_t)i * blockDim.x;
    if (g < G) {
      uint32_t w[4];
      em[i] = pack_group<B>(sm, g, n, w);
      char* o = codes + (size_t)g * 4u * B;
      if (B == 4) {
        st_v4(o, make_uint4(w[0], w[1], w[2], w[3]));
      } else if (B == 2) {
        *reinterpret_cast<uint2*>(o) = make_uint2(w[0], w[1]);
      } else {
#pragma unroll
        for (int q = 0; q < B; ++q) reinterpret_cast<uint32_t*>(o)[q] = w[q];
      }
      cnt |= (unsigned long long)__popc(em[i]) << (16 * i);
    }
  }
  // zero padding of the code and escape sections
  const uint32_t cb = G * 4u * B, cpad = pad16(cb);
  if (tid < (cpad - cb) / 4) reinterpret_cast<uint32_t*>(codes + cb)[tid] = 0u;
  const uint32_t nesc = sm.pk_nesc;
  if (tid < pad16(nesc) - nesc) escs[nesc + tid] = 0;
  if (nesc == 0) return;  // block-uniform
  unsigned long long tot;
  const unsigned long long ex = esc_scan(cnt, sm.esc_part, &tot);
  uint32_t base = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t g = tid + (uint32_t)i * blockDim.x;
    uint32_t pos = base + lane16(ex, i);
    uint32_t m = em[i];
    while (m) {
      const int k = __ffs(m) - 1;
      m &= m - 1;
      escs[pos++] = (char)sm.syms[g * PACK_GROUP + k];
    }
    base += lane16(tot, i);
  }
}

// Symbol section and header of a PACK-level record (after the split and the
// histogram). Returns the record size (uniform over the CTA).
template <int DT>
LZ_DEV uint32_t encode_pack_tail(EncSmem& sm, uint32_t n, char* dst, uint32_t raw_bytes) {
  const uint32_t tid = threadIdx.x;
  if ((tid >> 5) == 0) pack_tables_warp0(sm, n);
  __syncthreads();
  const int bits = sm.pk_bits;
  char* symsec = dst + sizeof(TgHeader) + raw_bytes;
  uint32_t sym_bytes;
  if (bits < 0) {
    sym_bytes = pad16(n);
    if (tid < sym_bytes - n) sm.syms[n + tid] = 0;
    __syncthreads();
    cta_copy16(symsec, reinterpret_cast<const char*>(sm.syms), sym_bytes);
    if (tid == 0) write_tg_header(dst, MODE_RAW, (uint8_t)DT, n, sym_bytes, raw_bytes, 0, 0, 0);
  } else {
    sym_bytes = sm.pk_bytes;
    if (tid == 0) st_v4(symsec, *reinterpret_cast<const uint4*>(sm.ptab));
    switch (bits) {
      case 1: pack_emit_codes<1>(sm, n, symsec); break;
      case 2: pack_emit_codes<2>(sm, n, symsec); break;
      case 3: pack_emit_codes<3>(sm, n, symsec); break;
      case 4: pack_emit_codes<4>(sm, n, symsec); break;
      default: break;  // b = 0: the table alone
    }
    if (tid == 0)
      write_tg_header(dst, MODE_PACK, (uint8_t)DT, n, sym_bytes, raw_bytes, sm.pk_nnz, (uint32_t)bits,
                      sm.pk_nesc);
  }
  __syncthreads();  // shared memory is reused by the CTA's next table group
  return (uint32_t)sizeof(TgHeader) + raw_bytes + sym_bytes;
}

// Decoder: 4 codes of quad qd of a group as nibbles (code j at bits 4j).
template <int B>
LZ_DEV uint32_t quad_codes(const uint32_t (&w)[4], int qd) {
  const int bit = 4 * B * qd, wi = bit >> 5, sh = bit & 31;
  uint32_t f = (sh + 4 * B > 32) ? __funnelshift_r(w[wi], w[wi + 1], sh) : (w[wi] >> sh);
  if (B == 4) return f & 0xFFFFu;
  uint32_t q = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) q |= ((f >> (j * B)) & ((1u << B) - 1u)) << (4 * j);
  return q;
}
// 4 symbols (one byte each) of the nibble codes q from the 16-byte table.
template <int B>
LZ_DEV uint32_t quad_syms(uint32_t q, const uint4& tv) {
  if (B < 4) return __byte_perm(tv.x, tv.y, q);  // codes <= 7: bit 3 of every nibble is 0
  const uint32_t sel = q & 0x7777u;
  const uint32_t lo = __byte_perm(tv.x, tv.y, sel), hi = __byte_perm(tv.z, tv.w, sel);
  const uint32_t msk = __byte_perm(0x0000FF00u, 0u, (q >> 3) & 0x1111u);  // 0xFF where code >= 8
  return (lo & ~msk) | (hi & msk);
}
// Escape bits (4) of the nibble codes q.
template <int B>
LZ_DEV uint32_t quad_esc(uint32_t q) {
  uint32_t e = q;
#pragma unroll
  for (int j = 1; j < B; ++j) e &= q >> j;
  e &= 0x1111u;
  return (e | (e >> 3) | (e >> 6) | (e >> 9)) & 0xFu;
}

template <int B>
LZ_DEV bool pack_decode_b(const char* __restrict__ symsec, uint32_t n, DecSmem& sm) {
  constexpr uint32_t ESC = (1u << B) - 1u;
  const uint32_t tid = threadIdx.x;
  const uint32_t G = pack_groups(n), nnz = sm.h.nnz, nesc = sm.h.reserved;
  const uint4 tv = ld_cg_v4(symsec);
  const char* codes = symsec + PACK_TABLE_BYTES;
  const char* escs = codes + pad16(G * 4u * B);
  uint32_t em[4] = {0, 0, 0, 0};
  unsigned long long cnt = 0;
  int bad = 0;
  // all code loads of the thread's (<= 4) groups are issued before any is used
  uint32_t wv[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t g = tid + (uint32_t)i * blockDim.x;
#pragma unroll
    for (int q = 0; q < 4; ++q) wv[i][q] = 0;
    if (g < G) {
      const char* o = codes + (size_t)g * 4u * B;
      if (B == 4) {
        const uint4 v = ld_cg_v4(o);
        wv[i][0] = v.x, wv[i][1] = v.y, wv[i][2] = v.z, wv[i][3] = v.w;
      } else if (B == 2) {
        const uint2 v = __ldcg(reinterpret_cast<const uint2*>(o));
        wv[i][0] = v.x, wv[i][1] = v.y;
      } else {
#pragma unroll
        for (int q = 0; q < B; ++q) wv[i][q] = __ldcg(reinterpret_cast<const uint32_t*>(o) + q);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t g = tid + (uint32_t)i * blockDim.x;
    if (g < G) {
      const uint32_t(&w)[4] = wv[i];
      uint32_t sy[8];
#pragma unroll
      for (int qd = 0; qd < 8; ++qd) {
        const uint32_t q = quad_codes<B>(w, qd);
        sy[qd] = quad_syms<B>(q, tv);
        em[i] |= quad_esc<B>(q) << (4 * qd);
      }
      const uint32_t lim = n - g * PACK_GROUP;
      if (lim < PACK_GROUP) em[i] &= (1u << lim) - 1u;
      if (nnz < ESC) {  // a partial table: codes nnz .. ESC-1 are invalid
#pragma unroll
        for (int qd = 0; qd < 8; ++qd) {
          const uint32_t q = quad_codes<B>(w, qd);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t c = (q >> (4 * j)) & 0xFu;
            if ((uint32_t)(4 * qd + j) < lim && c >= nnz && c != ESC) bad = 1;
          }
        }
      }
      uint4* dst = reinterpret_cast<uint4*>(&sm.syms[g * PACK_GROUP]);
      dst[0] = make_uint4(sy[0], sy[1], sy[2], sy[3]);
      dst[1] = make_uint4(sy[4], sy[5], sy[6], sy[7]);
      cnt |= (unsigned long long)__popc(em[i]) << (16 * i);
    }
  }
  if (nesc == 0) return !__syncthreads_or(bad || cnt != 0);  // block-uniform branch
  unsigned long long tot;
  const unsigned long long ex = esc_scan(cnt, sm.esc_part, &tot);
  if (lane16(tot, 0) + lane16(tot, 1) + lane16(tot, 2) + lane16(tot, 3) != nesc) bad = 1;
  uint32_t base = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t g = tid + (uint32_t)i * blockDim.x;
    uint32_t pos = base + lane16(ex, i);
    uint32_t m = em[i];
    while (m) {
      const int k = __ffs(m) - 1;
      m &= m - 1;
      if (pos < nesc) sm.syms[g * PACK_GROUP + k] = ld_cg_u8(escs + pos);
      ++pos;
    }
    base += lane16(tot, i);
  }
  return !__syncthreads_or(bad);
}

// Symbol plane of a PACK record into sm.syms. Block-uniform result.
LZ_DEV bool pack_decode_syms(const char* __restrict__ symsec, uint32_t n, DecSmem& sm) {
  switch (sm.h.nsub) {
    case 0: {
      const uint32_t t = (uint32_t)ld_cg_u8(symsec) * 0x01010101u;
      for (uint32_t o = threadIdx.x * 16; o < pad16(n); o += blockDim.x * 16)
        *reinterpret_cast<uint4*>(&sm.syms[o]) = make_uint4(t, t, t, t);
      return true;
    }
    case 1: return pack_decode_b<1>(symsec, n, sm);
    case 2: return pack_decode_b<2>(symsec, n, sm);
    case 3: return pack_decode_b<3>(symsec, n, sm);
    default: return pack_decode_b<4>(symsec, n, sm);
  }
}

// ---------------------------------------------------------------------------
// Encode one TG of n elements from `in` (16-B aligned) into the record at
// `dst` (16-B aligned; any memory the CTA can store to: local, peer).
// Returns the record size (uniform over the CTA).
// ---------------------------------------------------------------------------
// `stop_after` (profiling only): 1 = split + histogram, 2 = + tables,
// 3 = + rANS, 0 = complete record.
template <int DT>
LZ_DEV uint32_t encode_tg(const char* __restrict__ in, uint32_t n, char* __restrict__ dst,
                          EncSmem& sm, int level = LEVEL_ANS, int stop_after = 0) {
  using S = Split16<DT>;
  constexpr int RB = DT == DT_F32 ? 3 : (DT == DT_U8 ? 0 : 1);
  constexpr int ES = DT == DT_F32 ? 4 : (DT == DT_U8 ? 1 : 2);
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t raw_bytes = pad16(n * RB);
  char* raw_dst = dst + sizeof(TgHeader);

  for (uint32_t k = tid; k < NSUB * HREP * HSTRIDE; k += blockDim.x) (&sm.u.counts[0][0][0])[k] = 0;
  __syncthreads();
  // 1. split + histogram (+ raw plane straight to the destination)
  const uint32_t units = n / 16;
  // software-pipelined: the vectors of the next unit are loaded before the
  // current one is split and counted
  uint4 nxt[S::IN_VECS];
  if (tid < units) {
#pragma unroll
    for (int q = 0; q < S::IN_VECS; ++q) nxt[q] = ld_cg_v4(in + (size_t)tid * 16 * ES + 16 * q);
  }
  for (uint32_t u0 = 0; u0 < units; u0 += blockDim.x) {  // block-uniform trip count
    const uint32_t u = u0 + tid;
    const bool act = u < units;
    uint32_t sw[4];
    if (act) {
      uint4 v[S::IN_VECS];
#pragma unroll
      for (int q = 0; q < S::IN_VECS; ++q) v[q] = nxt[q];
      const uint32_t un = u + blockDim.x;
      if (un < units) {
#pragma unroll
        for (int q = 0; q < S::IN_VECS; ++q) nxt[q] = ld_cg_v4(in + (size_t)un * 16 * ES + 16 * q);
      }
      uint32_t rw[S::RW];
      S::split(v, sw, rw);
      *reinterpret_cast<uint4*>(&sm.syms[u * 16]) = make_uint4(sw[0], sw[1], sw[2], sw[3]);
      if (RB > 0) {
#pragma unroll
        for (int q = 0; q < S::RAW_BYTES / 16; ++q)
          st_v4(raw_dst + (size_t)u * S::RAW_BYTES + 16 * q,
                make_uint4(rw[4 * q], rw[4 * q + 1], rw[4 * q + 2], rw[4 * q + 3]));
      }
    }
    // replicated per-warp histograms: one shared atomic per symbol, lanes
    // spread over HREP copies (padded apart by 8 banks) to cut same-address
    // and same-bank serialisation
    if (act) {
      uint32_t* h = sm.u.counts[warp][lane & (HREP - 1)];
#pragma unroll
      for (int k = 0; k < 16; ++k) atomicAdd(&h[(sw[k / 4] >> (8 * (k % 4))) & 0xFFu], 1u);
    }
  }
  // tail elements (n % 16) and the zero padding of the raw plane
  if (tid < n - units * 16) {
    const uint32_t i = units * 16 + tid;
    uint8_t s1, r1[4];
    split1<DT>(in, i, &s1, r1);
    sm.syms[i] = s1;
    atomicAdd(&sm.u.counts[0][0][s1], 1u);
    for (int q = 0; q < RB; ++q) raw_dst[(size_t)i * RB + q] = (char)r1[q];
  }
  if (RB > 0 && tid < raw_bytes - n * RB) raw_dst[n * RB + tid] = 0;
  __syncthreads();
  if (stop_after == 1) return 0;
  // 2. frequency tables: reduce the replicas (one bin per thread), then warp 0
  for (uint32_t sbin = tid; sbin < 256; sbin += blockDim.x) {
    uint32_t c = 0;
#pragma unroll
    for (int w = 0; w < NSUB; ++w)
#pragma unroll
      for (int r = 0; r < HREP; ++r) c += sm.u.counts[w][r][sbin];
    sm.hist[sbin] = c;
  }
  __syncthreads();
  if (level == LEVEL_PACK) return encode_pack_tail<DT>(sm, n, dst, raw_bytes);
  if (warp == 0) build_tables_warp0(sm, n);
  __syncthreads();
  if (stop_after == 2) return 0;
  // 3. one warp per sub-block: interleaved rANS, backward over the steps
  const uint32_t nsub = (n + SUB_ELEMS - 1) / SUB_ELEMS;
  if (warp < nsub) {
    const uint32_t base = warp * SUB_ELEMS;
    const uint32_t sn = min(SUB_ELEMS, n - base);
    uint32_t x, pos;
    // full sub-blocks (every step has 32 symbols) take the branch-free loop
    const bool ok = sn == SUB_ELEMS ? rans_encode_sub<true>(sm, base, sn, warp, lane, x, pos)
                                    : rans_encode_sub<false>(sm, base, sn, warp, lane, x, pos);
    uint8_t* out = sm.u.streams[warp];
    if (ok) {
      reinterpret_cast<uint32_t*>(out)[lane] = x;
      // zero the padding words so records are deterministic
      const uint32_t len = 128u + 2u * pos;
      if (lane < (pad16(len) - len) / 2) *reinterpret_cast<uint16_t*>(out + len + 2 * lane) = 0;
    }
    if (lane == 0) sm.sub_len[warp] = ok ? 128u + 2u * pos : 0u;
  }
  __syncthreads();
  if (stop_after == 3) return 0;
  // 4. mode decision and record emission
  __shared__ uint32_t s_mode, s_symbytes, s_tabbytes;
  if (tid == 0) {
    bool ans = n > 0;
    uint32_t bytes = pad16(4 * sm.nnz) + pad16(4 * nsub);
    for (uint32_t b = 0; b < nsub; ++b) {
      if (sm.sub_len[b] == 0) ans = false;
      bytes += pad16(sm.sub_len[b]);
    }
    if (bytes >= pad16(n)) ans = false;
    s_mode = ans ? MODE_ANS : MODE_RAW;
    s_symbytes = ans ? bytes : pad16(n);
    s_tabbytes = pad16(4 * sm.nnz);
    TgHeader h;
    h.magic = TG_MAGIC;
    h.version = VERSION;
    h.mode = (uint8_t)s_mode;
    h.dtype = (uint8_t)DT;
    h.n = n;
    h.sym_bytes = s_symbytes;
    h.raw_bytes = raw_bytes;
    h.nnz = ans ? (uint16_t)sm.nnz : 0;
    h.nsub = ans ? (uint16_t)nsub : 0;
    h.total = (uint32_t)sizeof(TgHeader) + raw_bytes + s_symbytes;
    h.reserved = 0;
    const uint4* hv = reinterpret_cast<const uint4*>(&h);
    st_v4(dst, hv[0]);
    st_v4(dst + 16, hv[1]);
    sm.total = h.total;
  }
  __syncthreads();
  char* symsec = raw_dst + raw_bytes;
  if (s_mode == MODE_RAW) {
    // zero the padding of the symbol plane, then copy it
    if (tid < pad16(n) - n) sm.syms[n + tid] = 0;
    __syncthreads();
    cta_copy16(symsec, reinterpret_cast<const char*>(sm.syms), pad16(n));
  } else {
    const uint32_t tb = s_tabbytes;
    for (uint32_t k = tid; k < tb / 4; k += blockDim.x)
      reinterpret_cast<uint32_t*>(symsec)[k] = k < sm.nnz ? sm.table[k] : 0u;
    const uint32_t sb = pad16(4 * nsub);
    if (tid < sb / 4) reinterpret_cast<uint32_t*>(symsec + tb)[tid] = tid < nsub ? sm.sub_len[tid] : 0u;
    uint32_t off = tb + sb;
    for (uint32_t b = 0; b < nsub; ++b) {
      const uint32_t len = pad16(sm.sub_len[b]);
      cta_copy16(symsec + off, reinterpret_cast<const char*>(sm.u.streams[b]), len);
      off += len;
    }
  }
  const uint32_t total = sm.total;
  __syncthreads();
  return total;
}

// ---------------------------------------------------------------------------
// Interleaved rANS decode of one sub-stream (`len` bytes at `st`: 32 states,
// then 16-bit words) into sm.syms[base, base + sn) by one warp, forward over
// the steps (the encoder's words are consumed in reverse). Returns true when
// every word was consumed and every lane ended in the initial state.
// kFull: sn == SUB_ELEMS, so every step has all 32 lanes active.
// ---------------------------------------------------------------------------
template <bool kFull>
LZ_DEV bool rans_decode_sub(DecSmem& sm, const char* st, uint32_t len, uint32_t base, uint32_t sn,
                            uint32_t lane) {
  uint32_t x = *reinterpret_cast<const uint32_t*>(st + 4 * lane);
  const uint16_t* words = reinterpret_cast<const uint16_t*>(st + 128);
  int E = (int)((len - 128) / 2);
  const uint32_t lt = lanemask_lt();
  const int jn = (int)((sn + LANES - 1) / LANES);
  uint8_t* syms = sm.syms + base + lane;
  bool wok = true;
  for (int j = 0; j < jn; ++j) {
    const bool act = kFull || (uint32_t)j * LANES + lane < sn;
    bool need = false;
    if (act) {
      const uint32_t ent = sm.dtab[x & (PROB_SCALE - 1)];
      syms[(uint32_t)j * LANES] = (uint8_t)(ent & 0xFF);
      x = dec_update(x, ent);
      need = x < RANS_L;
    }
    const uint32_t m = __ballot_sync(0xffffffffu, need);
    const int k = __popc(m);
    if (k > E) {
      wok = false;
      break;
    }
    if (need) x = (x << 16) | words[E - k + __popc(m & lt)];
    E -= k;
  }
  return wok && E == 0 && x == RANS_L;
}

// ---------------------------------------------------------------------------
// Decode the symbol plane of the TG record at `src` (n elements expected)
// into sm.syms. Returns true on success (uniform over the CTA); the raw plane
// starts at src + sizeof(TgHeader). A corrupt record returns false.
// MODES: record modes compiled in (bit 1 << MODE_x); a record of another mode
// is rejected as corrupt. Fused kernels that decode only their own level's
// records drop the other decoder from their code.
// ---------------------------------------------------------------------------
constexpr int MODES_ALL = (1 << MODE_RAW) | (1 << MODE_ANS) | (1 << MODE_PACK);
template <int LV>
constexpr int kModesOfLevel =
    LV == LEVEL_PACK ? ((1 << MODE_RAW) | (1 << MODE_PACK)) : ((1 << MODE_RAW) | (1 << MODE_ANS));

template <int DT, int MODES = MODES_ALL>
LZ_DEV bool decode_tg_syms(const char* __restrict__ src, uint32_t cap, uint32_t n, DecSmem& sm) {
  constexpr int RB = DT == DT_F32 ? 3 : (DT == DT_U8 ? 0 : 1);
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    TgHeader h;
    uint4* hv = reinterpret_cast<uint4*>(&h);
    hv[0] = ld_cg_v4(src);
    hv[1] = ld_cg_v4(src + 16);
    int ok = h.magic == TG_MAGIC && h.version == VERSION && h.dtype == DT && h.n == n &&
             h.raw_bytes == pad16(n * RB) && h.total <= cap &&
             h.total == sizeof(TgHeader) + h.raw_bytes + h.sym_bytes;
    if (ok && h.mode == MODE_RAW) ok = h.sym_bytes == pad16(n);
    else if (ok && ((MODES >> MODE_PACK) & 1) && h.mode == MODE_PACK)
      ok = h.nsub <= PACK_MAX_BITS && h.nnz >= 1 && h.reserved <= n &&
           (h.nsub == 0 ? (h.nnz == 1 && h.reserved == 0) : h.nnz <= (1u << h.nsub) - 1u) &&
           h.sym_bytes == pack_sym_bytes(n, h.nsub, h.reserved) && h.sym_bytes < pad16(n);
    else if (ok && ((MODES >> MODE_ANS) & 1) && h.mode == MODE_ANS)
      ok = h.nsub == (n + SUB_ELEMS - 1) / SUB_ELEMS && h.nnz >= 1 && h.nnz <= 256 &&
           h.sym_bytes < pad16(n) &&
           pad16(4u * h.nnz) + pad16(4u * h.nsub) <= h.sym_bytes;
    else ok = 0;
    sm.h = h;
    sm.ok = ok;
  }
  __syncthreads();
  if (!sm.ok) return false;
  const char* raw = src + sizeof(TgHeader);
  const char* symsec = raw + sm.h.raw_bytes;  // re-pointed at the staged copy for ANS
  if (sm.h.mode == MODE_RAW) {
    for (uint32_t o = tid * 16; o < pad16(n); o += blockDim.x * 16)
      *reinterpret_cast<uint4*>(&sm.syms[o]) = ld_cg_v4(symsec + o);
  } else if (sm.h.mode == MODE_PACK) {
    if constexpr (((MODES >> MODE_PACK) & 1) != 0) {
      if (!pack_decode_syms(symsec, n, sm)) return false;
    }
  } else if constexpr (((MODES >> MODE_ANS) & 1) != 0) {
    const uint32_t nnz = sm.h.nnz, nsub = sm.h.nsub;
    // stage the whole ANS section (<= pad16(n) bytes) so every word fetch of
    // the rANS loop is a shared-memory load, off the global-latency path: one
    // bulk copy by the TMA engine (vector loads if it is not 16-byte aligned)
    {
      const uint32_t sb = sm.h.sym_bytes;
      const bool bulk = ((reinterpret_cast<uintptr_t>(symsec) | smem_addr(sm.sec) | sb) & 15u) == 0 && sb > 0;
      if (bulk) {
        if (tid == 0) mbar_init(&sm.bar, 1);
        fence_proxy_async_smem();  // earlier generic writes to this shared memory come first
        __syncthreads();
        if (tid == 0) {
          fence_mbar_init();
          bulk_g2s(sm.sec, symsec, sb, &sm.bar);
        }
        // a global -> shared bulk copy always completes; the bound only keeps
        // a broken environment from spinning forever
        if (!mbar_wait(&sm.bar, 0, 1u << 26) && tid == 0) sm.ok = 0;
        __syncthreads();
        if (tid == 0) mbar_inval(&sm.bar);
      } else {
        const uint32_t step = blockDim.x * 16;
        uint32_t o = tid * 16;
        for (; o + 3 * step < sb; o += 4 * step) {
          uint4 v[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) v[u] = ld_cg_v4(symsec + o + u * step);
#pragma unroll
          for (int u = 0; u < 4; ++u) *reinterpret_cast<uint4*>(&sm.sec[o + u * step]) = v[u];
        }
        for (; o < sb; o += step) *reinterpret_cast<uint4*>(&sm.sec[o]) = ld_cg_v4(symsec + o);
      }
    }
    __syncthreads();
    if (!sm.ok) return false;
    symsec = reinterpret_cast<const char*>(sm.sec);
    // decode table: slot -> entry, by binary search over the cumulative table
    uint32_t* s_cum = sm.cum;
    uint32_t* s_ent = sm.ent;
    if (warp == 0) {
      uint32_t e[8], f[8], lsum = 0;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const uint32_t idx = lane * 8 + k;
        e[k] = idx < nnz ? *reinterpret_cast<const uint32_t*>(symsec + 4 * idx) : 0u;
        f[k] = e[k] & 0xFFFF;
        lsum += f[k];
      }
      uint32_t incl = lsum;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        uint32_t a = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= (uint32_t)o) incl += a;
      }
      uint32_t cum = incl - lsum;
      int bad = 0;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const uint32_t idx = lane * 8 + k;
        if (idx < nnz) {
          s_cum[idx] = cum;
          s_ent[idx] = e[k];
          if (f[k] == 0 || (e[k] >> 16) > 255) bad = 1;
        }
        cum += f[k];
      }
      const uint32_t total = __shfl_sync(0xffffffffu, incl, 31);
      bad = __any_sync(0xffffffffu, bad);
      if (lane == 0) {
        s_cum[nnz] = PROB_SCALE;
        if (bad || total != PROB_SCALE) sm.ok = 0;
      }
    }
    __syncthreads();
    if (!sm.ok) return false;
    for (uint32_t slot = tid; slot < PROB_SCALE; slot += blockDim.x) {
      uint32_t lo = 0, hi = nnz;  // find k with cum[k] <= slot < cum[k+1]
      while (hi - lo > 1) {
        const uint32_t mid = (lo + hi) >> 1;
        if (s_cum[mid] <= slot) lo = mid;
        else hi = mid;
      }
      const uint32_t ent = s_ent[lo];
      sm.dtab[slot] = dec_entry(ent >> 16, ent & 0xFFFF, slot - s_cum[lo]);
    }
    __syncthreads();
    // one warp per sub-stream
    const char* sizes = symsec + pad16(4 * nnz);
    uint32_t off = pad16(4 * nnz) + pad16(4 * nsub);
    bool good = true;
    for (uint32_t b = 0; b < nsub; ++b) {
      const uint32_t len = *reinterpret_cast<const uint32_t*>(sizes + 4 * b);
      if (len < 128 || (len & 1) || off + pad16(len) > sm.h.sym_bytes) {
        good = false;
        break;
      }
      if (b == warp) {
        const char* st = symsec + off;
        const uint32_t base = b * SUB_ELEMS;
        const uint32_t sn = min(SUB_ELEMS, n - base);
        // full sub-streams (every step has 32 symbols) take the branch-free loop
        bool wok = sn == SUB_ELEMS ? rans_decode_sub<true>(sm, st, len, base, sn, lane)
                                   : rans_decode_sub<false>(sm, st, len, base, sn, lane);
        wok = __all_sync(0xffffffffu, wok);
        if (!wok && lane == 0) sm.ok = 0;
      }
      off += pad16(len);
    }
    if (!good && tid == 0) sm.ok = 0;
    __syncthreads();
    if (!sm.ok) return false;
  }
  __syncthreads();
  return true;
}

// Merge decoded symbols with the raw plane and store the elements.
template <int DT>
LZ_DEV void merge_store(const char* __restrict__ raw, const DecSmem& sm, uint32_t n,
                        char* __restrict__ out) {
  using S = Split16<DT>;
  constexpr int RB = DT == DT_F32 ? 3 : (DT == DT_U8 ? 0 : 1);
  constexpr int ES = DT == DT_F32 ? 4 : (DT == DT_U8 ? 1 : 2);
  constexpr int RV = S::RAW_BYTES / 16;            // raw vectors per unit
  constexpr int NB = S::RAW_BYTES > 16 ? 2 : 4;     // units whose raw loads are in flight together
  const uint32_t tid = threadIdx.x, bd = blockDim.x;
  const uint32_t units = n / 16;
  uint32_t u = tid;
  auto merge_unit = [&](uint32_t uu, const uint32_t (&rw)[S::RW]) {
    const uint4 sv = *reinterpret_cast<const uint4*>(&sm.syms[uu * 16]);
    const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w};
    uint4 v[S::IN_VECS];
    S::merge(sw, rw, v);
#pragma unroll
    for (int q = 0; q < S::IN_VECS; ++q) st_v4(out + (size_t)uu * 16 * ES + 16 * q, v[q]);
  };
  auto load_raw = [&](uint32_t uu, uint32_t (&rw)[S::RW]) {
    rw[0] = 0;
#pragma unroll
    for (int q = 0; q < RV; ++q) {
      const uint4 x = ld_cg_v4(raw + (size_t)uu * S::RAW_BYTES + 16 * q);
      rw[4 * q] = x.x, rw[4 * q + 1] = x.y, rw[4 * q + 2] = x.z, rw[4 * q + 3] = x.w;
    }
  };
  for (; u + (NB - 1) * bd < units; u += NB * bd) {
    uint32_t rw[NB][S::RW];
#pragma unroll
    for (int b = 0; b < NB; ++b) load_raw(u + b * bd, rw[b]);
#pragma unroll
    for (int b = 0; b < NB; ++b) merge_unit(u + b * bd, rw[b]);
  }
  for (; u < units; u += bd) {
    uint32_t rw[S::RW];
    load_raw(u, rw);
    merge_unit(u, rw);
  }
  if (tid < n - units * 16) {
    const uint32_t i = units * 16 + tid;
    uint8_t r1[4] = {0, 0, 0, 0};
    for (int q = 0; q < RB; ++q) r1[q] = ld_cg_u8(raw + (size_t)i * RB + q);
    merge1<DT>(out, i, sm.syms[i], r1);
  }
  __syncthreads();
}

// Element value of decoded symbol + raw bits as fp32 (float dtypes only).
template <int DT>
LZ_DEV float elem_to_f32(uint8_t sym, const uint8_t* raw) {
  if (DT == DT_BF16) return __uint_as_float((uint32_t)merge_bf16(sym, raw[0]) << 16);
  if (DT == DT_F16) return __half2float(__ushort_as_half(merge_f16(sym, raw[0])));
  const uint32_t r = raw[0] | ((uint32_t)raw[1] << 8) | ((uint32_t)raw[2] << 16);
  return __uint_as_float(merge_f32(sym, r));
}

// Decode one TG record at `src` (n elements expected) into `out`.
// Returns true on success (uniform over the CTA).
template <int DT, int MODES = MODES_ALL>
LZ_DEV bool decode_tg(const char* __restrict__ src, uint32_t cap, uint32_t n, char* __restrict__ out,
                      DecSmem& sm) {
  if (!decode_tg_syms<DT, MODES>(src, cap, n, sm)) return false;
  merge_store<DT>(src + sizeof(TgHeader), sm, n, out);
  return true;
}

}  // namespace lzg
