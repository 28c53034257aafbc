// LZC1: lossless float codec format shared by the GPU kernels and the CPU
// oracle (which must produce bit-identical streams).
//
// Split: every element is cut into a one-byte "symbol" (the exponent byte for
// bf16/fp32, the high byte for fp16, the whole byte for 8-bit types) and a
// "raw" remainder (sign + mantissa bits) that is stored verbatim. Only the
// symbol plane is entropy coded. This is the split described by the
// reference's UCCL logs (raw/bf16_split_sm16_split_encode_time_count.txt) and
// dietgpu's float mode; the stream format and coder here are this project's own.
//
// Coder: rANS (J. Duda, "Asymmetric numeral systems", 2013) with 32-bit
// states, 16-bit renormalisation words and PROB_BITS-bit quantised
// frequencies, interleaved over the 32 lanes of a warp (the interleaving
// scheme published by F. Giesen, "Interleaved entropy coders", 2014):
// lane l codes symbols l, l+32, l+64, ... of its sub-block and all lanes share
// one word stream whose per-step order is the lane order.
//
// Layout of one table group (TG, up to TG_ELEMS elements, own frequency table):
//   TgHeader (32 B)
//   raw plane: n * raw_bytes_per_elem(dtype), zero padded to 16 B
//   symbol section, one of
//     RAW  : n symbol bytes, padded to 16 B
//     ANS  : table   nnz x u32 (sym << 16 | freq), padded to 16 B
//            sizes   nsub x u32 (bytes of each sub-stream before padding), padded to 16 B
//            nsub sub-streams, each: 32 x u32 final lane states, then the
//            16-bit words in emission order, padded to 16 B.
//     PACK : table   16 B: the nnz (<= 15) most frequent symbols, most
//                    frequent first (ties: smaller symbol first), zero padded
//            codes   one b-bit code per element (b = nsub, 0..4), in groups of
//                    32 elements: group g is b little-endian u32 words at byte
//                    4*b*g holding code k of the group at bits [k*b, k*b + b)
//                    of their 32b-bit concatenation; padded to 16 B
//            escapes `reserved` symbol bytes, in element order, padded to 16 B
//            Code c < nnz stands for table[c]; c = 2^b - 1 takes the next
//            escape byte; other codes are invalid. b = 0 (no code section)
//            means every element's symbol is table[0].
// The encoder has two levels. LEVEL_ANS codes a TG ANS only if no sub-stream
// exceeds its sub-block's symbol count in bytes (before padding) and the ANS
// section is smaller than the RAW section; otherwise RAW. LEVEL_PACK picks,
// among the b in 0..4 that escape at most n / 16 symbols, the one with the
// smallest PACK section (ties: smaller b) and uses it when it is smaller than
// the RAW section; otherwise RAW. PACK trades ratio (about
// 3.3 code bits per bf16 exponent of N(0, s) data against ~2.7 for ANS) for
// an encoder and decoder with a few integer operations per element. Decoding
// accepts every mode and validates the magic, the sizes, that every word was
// consumed and every lane state returned to RANS_L (ANS), and the code range
// and escape count (PACK).
//
// Whole-tensor stream ("compact" form):
//   StreamHeader (64 B) | n_tg x u64 TG offsets (from stream start), padded to 16 B | TG records
// Slotted form (fused transfer paths): TG t lives at t * tg_capacity().
#pragma once
#include <stddef.h>
#include <stdint.h>

#ifdef __CUDACC__
#define LZC_HD __host__ __device__ __forceinline__
#else
#define LZC_HD inline
#endif

namespace lzc {

constexpr uint32_t PROB_BITS = 11;
constexpr uint32_t PROB_SCALE = 1u << PROB_BITS;
constexpr uint32_t RANS_L = 1u << 16;
constexpr int LANES = 32;
constexpr int SUB_STEPS = 128;
constexpr uint32_t SUB_ELEMS = LANES * SUB_STEPS;  // 4096
constexpr int NSUB = 8;
constexpr uint32_t TG_ELEMS = SUB_ELEMS * NSUB;    // 32768
constexpr uint32_t TG_MAGIC = 0x47545A4Cu;         // "LZTG"
constexpr uint32_t STREAM_MAGIC = 0x31435A4Cu;     // "LZC1"
constexpr uint16_t VERSION = 1;
constexpr uint8_t MODE_RAW = 0;
constexpr uint8_t MODE_ANS = 1;
constexpr uint8_t MODE_PACK = 2;

// Encoder levels. Host entry points take the level in bits 8..11 of their
// dtype argument (dtype | level << CODEC_LEVEL_SHIFT); level 0 is ANS.
constexpr int LEVEL_ANS = 0;
constexpr int LEVEL_PACK = 1;
constexpr int CODEC_LEVEL_SHIFT = 8;
constexpr uint32_t PACK_MAX_BITS = 4;
constexpr uint32_t PACK_TABLE_BYTES = 16;
constexpr uint32_t PACK_GROUP = 32;  // elements per code group
constexpr uint32_t PACK_MAX_ESC_DIV = 16;  // at most n / 16 escaped symbols per table group

// dtype codes (same values as LzDtype). The two fp8 "pair" types treat two
// consecutive fp8 bytes as one 16-bit element: the pair is packed into a
// container whose bits 14..7 carry exponent bits of both values (symbol) and
// whose other 8 bits (raw) carry signs and mantissas, so fp8 data needs one
// rANS symbol per two values.
constexpr int DT_F32 = 0, DT_F16 = 1, DT_BF16 = 2, DT_U8 = 3, DT_E4M3P = 4, DT_E5M2P = 5;

struct TgHeader {
  uint32_t magic;
  uint16_t version;
  uint8_t mode;
  uint8_t dtype;
  uint32_t n;          // elements in this TG
  uint32_t sym_bytes;  // bytes of the symbol section (padded)
  uint32_t raw_bytes;  // bytes of the raw plane (padded)
  uint16_t nnz;        // table entries (ANS)
  uint16_t nsub;       // sub-streams (ANS)
  uint32_t total;      // bytes of the whole record
  uint32_t reserved;
};
static_assert(sizeof(TgHeader) == 32, "TgHeader must be 32 bytes");

struct StreamHeader {
  uint32_t magic;
  uint16_t version;
  uint8_t dtype;
  uint8_t flags;
  uint32_t tg_elems;
  uint32_t n_tg;
  uint64_t n_elems;
  uint64_t total_bytes;
  uint64_t reserved[4];
};
static_assert(sizeof(StreamHeader) == 64, "StreamHeader must be 64 bytes");

LZC_HD uint32_t pad16(uint32_t x) { return (x + 15u) & ~15u; }
LZC_HD uint64_t pad16_64(uint64_t x) { return (x + 15u) & ~uint64_t(15); }

// dtype argument of a host entry point -> dtype code and encoder level
LZC_HD int codec_dtype(int arg) { return arg & 0xFF; }
LZC_HD int codec_level(int arg) { return (arg >> CODEC_LEVEL_SHIFT) & 0xF; }
LZC_HD bool valid_level(int level) { return level == LEVEL_ANS || level == LEVEL_PACK; }

// --- PACK section sizes and the choice of the code width ----------------------
LZC_HD uint32_t pack_groups(uint32_t n) { return (n + PACK_GROUP - 1) / PACK_GROUP; }
LZC_HD uint32_t pack_sym_bytes(uint32_t n, uint32_t bits, uint32_t nesc) {
  return PACK_TABLE_BYTES + pad16(pack_groups(n) * 4u * bits) + pad16(nesc);
}
struct PackChoice {
  int bits;       // -1: PACK does not beat RAW
  uint32_t nnz;   // table entries
  uint32_t nesc;  // escaped elements
  uint32_t bytes; // symbol section bytes
};
// top[0..ntop) are the counts of the most frequent symbols in table order
// (ntop <= 15, all nonzero) of a TG of n elements.
LZC_HD PackChoice pack_choose(const uint32_t* top, uint32_t ntop, uint32_t n) {
  PackChoice best{-1, 0, 0, pad16(n)};
  if (n == 0 || ntop == 0) return best;
  if (ntop == 1 && top[0] == n && PACK_TABLE_BYTES < best.bytes) best = PackChoice{0, 1, 0, PACK_TABLE_BYTES};
  uint32_t covered = 0, k = 0;
  for (uint32_t b = 1; b <= PACK_MAX_BITS; ++b) {
    const uint32_t K = (1u << b) - 1u;
    for (; k < K && k < ntop; ++k) covered += top[k];
    const uint32_t nesc = n - covered;
    // escapes are written one byte each: a width that escapes more than one
    // symbol in 16 is not used (such groups are coded RAW), which keeps the
    // level's cost per element bounded on data the table does not fit
    if ((uint64_t)nesc * PACK_MAX_ESC_DIV > n) continue;
    const uint32_t bytes = pack_sym_bytes(n, b, nesc);
    if (bytes < best.bytes) best = PackChoice{(int)b, k, nesc, bytes};
  }
  return best;
}

LZC_HD int elem_bytes(int dt) { return dt == DT_F32 ? 4 : (dt == DT_U8 ? 1 : 2); }
LZC_HD bool valid_dtype(int dt) { return dt >= DT_F32 && dt <= DT_E5M2P; }
LZC_HD int raw_bytes_per_elem(int dt) { return dt == DT_F32 ? 3 : (dt == DT_U8 ? 0 : 1); }

// Worst-case record size of a TG of n elements (RAW symbol section).
LZC_HD uint32_t tg_capacity_n(uint32_t n, int dt) {
  return (uint32_t)sizeof(TgHeader) + pad16(n * (uint32_t)raw_bytes_per_elem(dt)) + pad16(n);
}
LZC_HD uint32_t tg_capacity(int dt) { return tg_capacity_n(TG_ELEMS, dt); }

LZC_HD uint64_t num_tgs(uint64_t n) { return (n + TG_ELEMS - 1) / TG_ELEMS; }

LZC_HD uint64_t max_stream_bytes(uint64_t n, int dt) {
  const uint64_t ntg = num_tgs(n);
  return sizeof(StreamHeader) + pad16_64(8 * ntg) + ntg * (uint64_t)tg_capacity(dt);
}

// --- split / merge of one element -------------------------------------------
// bf16: symbol = exponent byte (bits 14..7); raw = sign << 7 | mantissa(7).
// fp16: symbol = high byte (sign, exponent, 2 mantissa bits); raw = low byte.
// fp32: symbol = exponent byte (bits 30..23); raw = sign << 23 | mantissa(23), 3 bytes LE.
// u8  : symbol = the byte; no raw plane.
LZC_HD uint8_t sym_bf16(uint16_t u) { return (uint8_t)((u >> 7) & 0xFF); }
LZC_HD uint8_t raw_bf16(uint16_t u) { return (uint8_t)(((u >> 8) & 0x80) | (u & 0x7F)); }
LZC_HD uint16_t merge_bf16(uint8_t s, uint8_t r) {
  return (uint16_t)(((uint16_t)(r & 0x80) << 8) | ((uint16_t)s << 7) | (r & 0x7F));
}
LZC_HD uint8_t sym_f16(uint16_t u) { return (uint8_t)(u >> 8); }
LZC_HD uint8_t raw_f16(uint16_t u) { return (uint8_t)(u & 0xFF); }
LZC_HD uint16_t merge_f16(uint8_t s, uint8_t r) { return (uint16_t)(((uint16_t)s << 8) | r); }
LZC_HD uint8_t sym_f32(uint32_t u) { return (uint8_t)((u >> 23) & 0xFF); }
LZC_HD uint32_t raw_f32(uint32_t u) { return (u & 0x7FFFFFu) | ((u >> 31) << 23); }
LZC_HD uint32_t merge_f32(uint8_t s, uint32_t r) {
  return ((r >> 23) << 31) | ((uint32_t)s << 23) | (r & 0x7FFFFFu);
}

// --- fp8 pair containers ------------------------------------------------------
// e4m3 (layout of the reference packer, back_up/fp8_e4m3fn_pack_benchmark.cu:21-31):
//   [15]=a.sign [14:11]=a.exp [10:7]=b.exp [6:4]=a.mant [3]=b.sign [2:0]=b.mant
LZC_HD uint16_t pack_e4m3(uint8_t a, uint8_t b) {
  return (uint16_t)(((a & 0x80u) << 8) | ((a & 0x78u) << 8) | ((b & 0x78u) << 4) |
                    ((a & 0x07u) << 4) | ((b & 0x80u) >> 4) | (b & 0x07u));
}
LZC_HD void unpack_e4m3(uint16_t w, uint8_t* a, uint8_t* b) {
  *a = (uint8_t)(((w >> 8) & 0x80u) | ((w >> 8) & 0x78u) | ((w >> 4) & 0x07u));
  *b = (uint8_t)(((w << 4) & 0x80u) | ((w >> 4) & 0x78u) | (w & 0x07u));
}
// e5m2: 5+5 exponent bits do not fit one byte; bits 14..7 carry the high four
// exponent bits of each value, the low exponent bits move to the raw byte:
//   [15]=a.sign [14:11]=a.e[4:1] [10:7]=b.e[4:1] [6]=a.e[0] [5:4]=a.mant
//   [3]=b.sign [2]=b.e[0] [1:0]=b.mant
LZC_HD uint16_t pack_e5m2(uint8_t a, uint8_t b) {
  const uint32_t ae = (a >> 2) & 0x1Fu, be = (b >> 2) & 0x1Fu;
  return (uint16_t)(((a & 0x80u) << 8) | ((ae >> 1) << 11) | ((be >> 1) << 7) | ((ae & 1u) << 6) |
                    ((a & 0x3u) << 4) | ((b & 0x80u) >> 4) | ((be & 1u) << 2) | (b & 0x3u));
}
LZC_HD void unpack_e5m2(uint16_t w, uint8_t* a, uint8_t* b) {
  const uint32_t ae = (((w >> 11) & 0xFu) << 1) | ((w >> 6) & 1u);
  const uint32_t be = (((w >> 7) & 0xFu) << 1) | ((w >> 2) & 1u);
  *a = (uint8_t)(((w >> 8) & 0x80u) | (ae << 2) | ((w >> 4) & 0x3u));
  *b = (uint8_t)(((w << 4) & 0x80u) | (be << 2) | (w & 0x3u));
}

// --- frequency normalisation (must be identical on CPU and GPU) -------------
// counts[256] of `total` symbols -> freq[256] summing to PROB_SCALE, every
// present symbol >= 1. Surplus goes to / deficit comes from the symbol with
// the largest count / frequency (ties: smallest symbol).
LZC_HD void normalize_freqs(const uint32_t* counts, uint32_t total, uint32_t* freq) {
  uint32_t sum = 0;
  int argmax_c = -1;
  uint32_t maxc = 0;
  for (int s = 0; s < 256; ++s) {
    uint32_t c = counts[s];
    uint32_t f = 0;
    if (c) {
      f = (uint32_t)(((uint64_t)c * PROB_SCALE) / total);
      if (f == 0) f = 1;
      if (c > maxc) {
        maxc = c;
        argmax_c = s;
      }
    }
    freq[s] = f;
    sum += f;
  }
  if (argmax_c < 0) return;
  if (sum < PROB_SCALE) {
    freq[argmax_c] += PROB_SCALE - sum;
    return;
  }
  while (sum > PROB_SCALE) {
    int best = -1;
    uint32_t bf = 1;
    for (int s = 0; s < 256; ++s) {
      if (freq[s] > bf) {
        bf = freq[s];
        best = s;
      }
    }
    uint32_t d = sum - PROB_SCALE;
    if (d > bf - 1) d = bf - 1;
    freq[best] -= d;
    sum -= d;
  }
}

// floor(x / f) without a divide: m = ceil(2^(32+l) / f) with l = ceil(log2 f),
// stored as m - 2^32 (< 2^32); q = (x + umulhi(x, m_lo)) >> l. Exact for all
// 32-bit x because f <= 2^l. (Granlund & Montgomery, "Division by invariant
// integers using multiplication", PLDI 1994.)
struct EncSym {
  uint32_t m_lo;
  uint32_t freq;
  uint32_t cum;
  uint32_t shift;
};

LZC_HD EncSym make_enc_sym(uint32_t f, uint32_t cum) {
  EncSym e;
  e.freq = f;
  e.cum = cum;
  uint32_t l = 0;
  while ((1u << l) < f) ++l;
  e.shift = l;
  const uint64_t m = ((uint64_t(1) << (32 + l)) + f - 1) / f;
  e.m_lo = (uint32_t)(m - (uint64_t(1) << 32));
  return e;
}

LZC_HD uint32_t umulhi32(uint32_t a, uint32_t b) {
#ifdef __CUDA_ARCH__
  return __umulhi(a, b);
#else
  return (uint32_t)(((uint64_t)a * b) >> 32);
#endif
}

// One rANS encode step: returns true (and the word) if a renormalisation word
// must be emitted before the state update.
// x >= f << (32 - PROB_BITS), evaluated in 32 bits: the shifted bound has no
// low bits, so comparing x's top PROB_BITS+1 bits with f is equivalent (and
// f = PROB_SCALE, a single-symbol table, never renormalises).
LZC_HD bool enc_needs_word(uint32_t x, uint32_t f) {
  return (x >> (32 - PROB_BITS)) >= f;
}
LZC_HD uint32_t enc_update(uint32_t x, const EncSym& e) {
  const uint32_t q = (uint32_t)(((uint64_t)x + umulhi32(x, e.m_lo)) >> e.shift);
  const uint32_t r = x - q * e.freq;
  return (q << PROB_BITS) + r + e.cum;
}

// Decode table entry for a slot: sym | (freq-1) << 8 | (slot - cum) << 20.
LZC_HD uint32_t dec_entry(uint32_t sym, uint32_t freq, uint32_t bias) {
  return sym | ((freq - 1u) << 8) | (bias << 20);
}
LZC_HD uint32_t dec_update(uint32_t x, uint32_t entry) {
  const uint32_t f = ((entry >> 8) & 0xFFFu) + 1u;
  const uint32_t bias = entry >> 20;
  return f * (x >> PROB_BITS) + bias;
}

}  // namespace lzc
