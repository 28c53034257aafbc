// CPU oracle of the LZC1 codec and of the fp8 packers. Bit-exact with the
// GPU kernels (csrc/lz_codec.cu, csrc/lz_fp8.cu); used by the CPU test suite,
// by the CPU/gloo compressed collectives and to validate GPU output.
//
// Reference counterparts: dietgpu's compress/decompress ops (a closed .so in
// the reference, loaded at single_node_nccl_allreduce_benchmark/compressed_twoshot_allreduce.py:34-47)
// and the fp8 pair packer of back_up/fp8_e4m3fn_pack_benchmark.cu:21-93.
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <atomic>
#include <thread>
#include <vector>

#include "../lz_codec_format.h"

using namespace lzc;

namespace {

inline void split_elem(const uint8_t* data, int dt, uint32_t i, uint8_t* sym, uint8_t* raw) {
  switch (dt) {
    case DT_BF16: {
      uint16_t u;
      memcpy(&u, data + 2 * (size_t)i, 2);
      *sym = sym_bf16(u);
      raw[0] = raw_bf16(u);
      break;
    }
    case DT_F16: {
      uint16_t u;
      memcpy(&u, data + 2 * (size_t)i, 2);
      *sym = sym_f16(u);
      raw[0] = raw_f16(u);
      break;
    }
    case DT_F32: {
      uint32_t u;
      memcpy(&u, data + 4 * (size_t)i, 4);
      *sym = sym_f32(u);
      uint32_t r = raw_f32(u);
      raw[0] = (uint8_t)r;
      raw[1] = (uint8_t)(r >> 8);
      raw[2] = (uint8_t)(r >> 16);
      break;
    }
    case DT_E4M3P:
    case DT_E5M2P: {
      const uint8_t a = data[2 * (size_t)i], b = data[2 * (size_t)i + 1];
      const uint16_t u = dt == DT_E4M3P ? pack_e4m3(a, b) : pack_e5m2(a, b);
      *sym = sym_bf16(u);
      raw[0] = raw_bf16(u);
      break;
    }
    default:
      *sym = data[i];
  }
}

inline void merge_elem(uint8_t* out, int dt, uint32_t i, uint8_t sym, const uint8_t* raw) {
  switch (dt) {
    case DT_BF16: {
      uint16_t u = merge_bf16(sym, raw[0]);
      memcpy(out + 2 * (size_t)i, &u, 2);
      break;
    }
    case DT_F16: {
      uint16_t u = merge_f16(sym, raw[0]);
      memcpy(out + 2 * (size_t)i, &u, 2);
      break;
    }
    case DT_F32: {
      uint32_t r = raw[0] | ((uint32_t)raw[1] << 8) | ((uint32_t)raw[2] << 16);
      uint32_t u = merge_f32(sym, r);
      memcpy(out + 4 * (size_t)i, &u, 4);
      break;
    }
    case DT_E4M3P:
    case DT_E5M2P: {
      const uint16_t u = merge_bf16(sym, raw[0]);
      if (dt == DT_E4M3P) unpack_e4m3(u, out + 2 * (size_t)i, out + 2 * (size_t)i + 1);
      else unpack_e5m2(u, out + 2 * (size_t)i, out + 2 * (size_t)i + 1);
      break;
    }
    default:
      out[i] = sym;
  }
}

// Encodes one sub-block with the warp-interleaved rANS. Returns the stream
// length in bytes before padding (states + words), or 0 on overflow of
// `cap` bytes (cap = number of symbols of the sub-block).
uint32_t encode_sub(const uint8_t* syms, uint32_t n, const EncSym* tab, uint8_t* out,
                    uint32_t cap) {
  uint32_t x[LANES];
  for (int l = 0; l < LANES; ++l) x[l] = RANS_L;
  std::vector<uint16_t> words;
  words.reserve(n);
  for (int j = SUB_STEPS - 1; j >= 0; --j) {
    for (int l = 0; l < LANES; ++l) {
      uint32_t i = (uint32_t)j * LANES + l;
      if (i >= n) continue;
      const EncSym& e = tab[syms[i]];
      if (enc_needs_word(x[l], e.freq)) {
        words.push_back((uint16_t)(x[l] & 0xFFFF));
        x[l] >>= 16;
      }
    }
    if (128u + 2u * (uint32_t)words.size() > cap) return 0;
    for (int l = 0; l < LANES; ++l) {
      uint32_t i = (uint32_t)j * LANES + l;
      if (i >= n) continue;
      x[l] = enc_update(x[l], tab[syms[i]]);
    }
  }
  memcpy(out, x, 128);
  if (!words.empty()) memcpy(out + 128, words.data(), 2 * words.size());
  return 128u + 2u * (uint32_t)words.size();
}

// Decodes one sub-block; returns false on any inconsistency.
bool decode_sub(const uint8_t* stream, uint32_t stream_bytes, const uint32_t* dec_tab, uint32_t n,
                uint8_t* syms) {
  if (stream_bytes < 128 || (stream_bytes - 128) % 2) return false;
  uint32_t x[LANES];
  memcpy(x, stream, 128);
  const uint8_t* wbase = stream + 128;
  int64_t E = (stream_bytes - 128) / 2;
  for (int j = 0; j < SUB_STEPS; ++j) {
    int need_lanes[LANES];
    int k = 0;
    for (int l = 0; l < LANES; ++l) {
      uint32_t i = (uint32_t)j * LANES + l;
      if (i >= n) continue;
      uint32_t slot = x[l] & (PROB_SCALE - 1);
      uint32_t ent = dec_tab[slot];
      syms[i] = (uint8_t)(ent & 0xFF);
      x[l] = dec_update(x[l], ent);
      if (x[l] < RANS_L) need_lanes[k++] = l;
    }
    if (k > E) return false;
    for (int q = 0; q < k; ++q) {
      int64_t idx = E - k + q;
      uint16_t w;
      memcpy(&w, wbase + 2 * idx, 2);
      x[need_lanes[q]] = (x[need_lanes[q]] << 16) | w;
    }
    E -= k;
  }
  if (E != 0) return false;
  for (int l = 0; l < LANES; ++l)
    if (x[l] != RANS_L) return false;
  return true;
}

// PACK symbol section (layout in lz_codec_format.h). Table order: count
// descending, then symbol ascending.
uint32_t pack_top(const uint32_t* counts, uint8_t* top_sym, uint32_t* top_cnt) {
  uint32_t order[256];
  for (uint32_t s = 0; s < 256; ++s) order[s] = s;
  std::stable_sort(order, order + 256, [&](uint32_t a, uint32_t b) { return counts[a] > counts[b]; });
  uint32_t k = 0;
  for (; k < 15 && counts[order[k]]; ++k) {
    top_sym[k] = (uint8_t)order[k];
    top_cnt[k] = counts[order[k]];
  }
  return k;
}

void pack_encode(const uint8_t* syms, uint32_t n, const PackChoice& pc, const uint8_t* top_sym,
                 uint8_t* symsec) {
  memset(symsec, 0, pc.bytes);
  memcpy(symsec, top_sym, pc.nnz);
  if (pc.bits == 0) return;
  const uint32_t b = (uint32_t)pc.bits, esc = (1u << b) - 1u;
  uint8_t code_of[256];
  memset(code_of, (int)esc, sizeof(code_of));
  for (uint32_t c = 0; c < pc.nnz; ++c) code_of[top_sym[c]] = (uint8_t)c;
  uint8_t* codes = symsec + PACK_TABLE_BYTES;
  uint8_t* escs = codes + pad16(pack_groups(n) * 4u * b);
  uint32_t e = 0;
  for (uint32_t i = 0; i < n; ++i) {
    const uint32_t c = code_of[syms[i]];
    if (c == esc) escs[e++] = syms[i];
    // code k of group g sits at bit k*b of the group's little-endian words
    const uint64_t bit = (uint64_t)(i / PACK_GROUP) * 32u * b + (uint64_t)(i % PACK_GROUP) * b;
    for (uint32_t q = 0; q < b; ++q)
      if ((c >> q) & 1u) codes[(bit + q) >> 3] |= (uint8_t)(1u << ((bit + q) & 7u));
  }
}

// Returns false on a corrupt section.
bool pack_decode(const uint8_t* symsec, const TgHeader& h, uint32_t n, uint8_t* syms) {
  const uint32_t b = h.nsub, nnz = h.nnz, nesc = h.reserved;
  if (b > PACK_MAX_BITS || nnz == 0 || nesc > n) return false;
  if (b == 0 ? (nnz != 1 || nesc != 0) : nnz > (1u << b) - 1u) return false;
  if (h.sym_bytes != pack_sym_bytes(n, b, nesc) || h.sym_bytes >= pad16(n)) return false;
  if (b == 0) {
    memset(syms, symsec[0], n);
    return true;
  }
  const uint32_t esc = (1u << b) - 1u;
  const uint8_t* codes = symsec + PACK_TABLE_BYTES;
  const uint8_t* escs = codes + pad16(pack_groups(n) * 4u * b);
  uint32_t e = 0;
  for (uint32_t i = 0; i < n; ++i) {
    const uint64_t bit = (uint64_t)(i / PACK_GROUP) * 32u * b + (uint64_t)(i % PACK_GROUP) * b;
    uint32_t c = 0;
    for (uint32_t q = 0; q < b; ++q) c |= (uint32_t)((codes[(bit + q) >> 3] >> ((bit + q) & 7u)) & 1u) << q;
    if (c == esc) {
      if (e >= nesc) return false;
      syms[i] = escs[e++];
    } else if (c < nnz) {
      syms[i] = symsec[c];
    } else {
      return false;
    }
  }
  return e == nesc;
}

}  // namespace

extern "C" {

uint32_t lzc_tg_capacity(uint32_t n, int dt) { return tg_capacity_n(n, codec_dtype(dt)); }
uint64_t lzc_max_stream_bytes(uint64_t n, int dt) { return max_stream_bytes(n, codec_dtype(dt)); }

// Encodes one TG of n (<= TG_ELEMS) elements into `out` (capacity
// tg_capacity_n). `dt_arg` is the dtype code | level << CODEC_LEVEL_SHIFT.
// Returns the record size.
int64_t lzc_tg_encode(const void* data, uint32_t n, int dt_arg, void* out_) {
  const int dt = codec_dtype(dt_arg), level = codec_level(dt_arg);
  if (n > TG_ELEMS || !valid_dtype(dt) || !valid_level(level)) return -1;
  uint8_t* out = static_cast<uint8_t*>(out_);
  const uint8_t* in = static_cast<const uint8_t*>(data);
  const int rb = raw_bytes_per_elem(dt);
  const uint32_t raw_bytes = pad16(n * (uint32_t)rb);
  std::vector<uint8_t> syms(n);
  uint8_t* raw = out + sizeof(TgHeader);
  memset(raw, 0, raw_bytes);
  uint32_t counts[256] = {0};
  for (uint32_t i = 0; i < n; ++i) {
    split_elem(in, dt, i, &syms[i], raw + (size_t)i * rb);
    counts[syms[i]]++;
  }
  TgHeader h;
  memset(&h, 0, sizeof(h));
  h.magic = TG_MAGIC;
  h.version = VERSION;
  h.dtype = (uint8_t)dt;
  h.n = n;
  h.raw_bytes = raw_bytes;
  uint8_t* symsec = raw + raw_bytes;
  const uint32_t raw_sym_bytes = pad16(n);
  if (level == LEVEL_PACK) {
    uint8_t top_sym[15];
    uint32_t top_cnt[15];
    const uint32_t ntop = pack_top(counts, top_sym, top_cnt);
    const PackChoice pc = pack_choose(top_cnt, ntop, n);
    if (pc.bits >= 0) {
      h.mode = MODE_PACK;
      h.nnz = (uint16_t)pc.nnz;
      h.nsub = (uint16_t)pc.bits;
      h.reserved = pc.nesc;
      h.sym_bytes = pc.bytes;
      pack_encode(syms.data(), n, pc, top_sym, symsec);
    } else {
      h.mode = MODE_RAW;
      h.sym_bytes = raw_sym_bytes;
      memset(symsec, 0, raw_sym_bytes);
      memcpy(symsec, syms.data(), n);
    }
    h.total = (uint32_t)sizeof(TgHeader) + raw_bytes + h.sym_bytes;
    memcpy(out, &h, sizeof(h));
    return h.total;
  }
  bool use_ans = n > 0;
  uint32_t ans_bytes = 0;
  std::vector<uint8_t> ans;
  if (use_ans) {
    uint32_t freq[256];
    normalize_freqs(counts, n, freq);
    EncSym tab[256];
    uint32_t cum = 0;
    std::vector<uint32_t> table;
    for (int s = 0; s < 256; ++s) {
      tab[s] = make_enc_sym(freq[s] ? freq[s] : 1, cum);
      if (freq[s]) table.push_back(((uint32_t)s << 16) | freq[s]);
      cum += freq[s];
    }
    const uint32_t nsub = (n + SUB_ELEMS - 1) / SUB_ELEMS;
    const uint32_t tab_bytes = pad16(4 * (uint32_t)table.size());
    const uint32_t sizes_bytes = pad16(4 * nsub);
    ans.assign(tab_bytes + sizes_bytes, 0);
    memcpy(ans.data(), table.data(), 4 * table.size());
    std::vector<uint32_t> sizes(nsub);
    std::vector<uint8_t> sub(SUB_ELEMS + 16);
    for (uint32_t b = 0; b < nsub && use_ans; ++b) {
      const uint32_t sn = std::min(SUB_ELEMS, n - b * SUB_ELEMS);
      memset(sub.data(), 0, sub.size());
      uint32_t len = encode_sub(syms.data() + (size_t)b * SUB_ELEMS, sn, tab, sub.data(), sn);
      if (len == 0) {
        use_ans = false;
        break;
      }
      sizes[b] = len;
      ans.insert(ans.end(), sub.begin(), sub.begin() + pad16(len));
    }
    if (use_ans) {
      memcpy(ans.data() + tab_bytes, sizes.data(), 4 * nsub);
      ans_bytes = (uint32_t)ans.size();
      if (ans_bytes >= raw_sym_bytes) use_ans = false;
      h.nnz = (uint16_t)table.size();
      h.nsub = (uint16_t)nsub;
    }
  }
  if (use_ans) {
    h.mode = MODE_ANS;
    h.sym_bytes = ans_bytes;
    memcpy(symsec, ans.data(), ans_bytes);
  } else {
    h.mode = MODE_RAW;
    h.nnz = 0;
    h.nsub = 0;
    h.sym_bytes = raw_sym_bytes;
    memset(symsec, 0, raw_sym_bytes);
    memcpy(symsec, syms.data(), n);
  }
  h.total = (uint32_t)sizeof(TgHeader) + raw_bytes + h.sym_bytes;
  memcpy(out, &h, sizeof(h));
  return h.total;
}

// Decodes one TG record. Returns 0, or a negative code on a corrupt record.
int lzc_tg_decode(const void* rec_, uint64_t rec_cap, void* out, uint32_t n, int dt) {
  dt = codec_dtype(dt);  // the decoder reads every mode; a level is ignored
  const uint8_t* rec = static_cast<const uint8_t*>(rec_);
  if (rec_cap < sizeof(TgHeader)) return -2;
  TgHeader h;
  memcpy(&h, rec, sizeof(h));
  if (!valid_dtype(dt) || h.magic != TG_MAGIC || h.version != VERSION || h.dtype != dt || h.n != n) return -3;
  const int rb = raw_bytes_per_elem(dt);
  if (h.raw_bytes != pad16(n * (uint32_t)rb) || h.total > rec_cap ||
      h.total != sizeof(TgHeader) + h.raw_bytes + h.sym_bytes)
    return -4;
  const uint8_t* raw = rec + sizeof(TgHeader);
  const uint8_t* symsec = raw + h.raw_bytes;
  std::vector<uint8_t> syms(n);
  if (h.mode == MODE_RAW) {
    if (h.sym_bytes != pad16(n)) return -5;
    memcpy(syms.data(), symsec, n);
  } else if (h.mode == MODE_ANS) {
    const uint32_t nsub = (n + SUB_ELEMS - 1) / SUB_ELEMS;
    if (h.nsub != nsub || h.nnz == 0 || h.nnz > 256 || h.sym_bytes >= pad16(n)) return -6;
    const uint32_t tab_bytes = pad16(4u * h.nnz), sizes_bytes = pad16(4 * nsub);
    if (tab_bytes + sizes_bytes > h.sym_bytes) return -7;
    uint32_t dec_tab[PROB_SCALE];
    uint32_t cum = 0;
    for (uint32_t k = 0; k < h.nnz; ++k) {
      uint32_t e;
      memcpy(&e, symsec + 4 * k, 4);
      uint32_t s = e >> 16, f = e & 0xFFFF;
      if (s > 255 || f == 0 || cum + f > PROB_SCALE) return -8;
      for (uint32_t q = 0; q < f; ++q) dec_tab[cum + q] = dec_entry(s, f, q);
      cum += f;
    }
    if (cum != PROB_SCALE) return -9;
    const uint8_t* sizes_p = symsec + tab_bytes;
    uint64_t off = tab_bytes + sizes_bytes;
    for (uint32_t b = 0; b < nsub; ++b) {
      uint32_t sz;
      memcpy(&sz, sizes_p + 4 * b, 4);
      if (off + pad16(sz) > h.sym_bytes) return -10;
      const uint32_t sn = std::min(SUB_ELEMS, n - b * SUB_ELEMS);
      if (!decode_sub(symsec + off, sz, dec_tab, sn, syms.data() + (size_t)b * SUB_ELEMS))
        return -11;
      off += pad16(sz);
    }
  } else if (h.mode == MODE_PACK) {
    if (!pack_decode(symsec, h, n, syms.data())) return -13;
  } else {
    return -12;
  }
  uint8_t* o = static_cast<uint8_t*>(out);
  for (uint32_t i = 0; i < n; ++i) merge_elem(o, dt, i, syms[i], raw + (size_t)i * rb);
  return 0;
}

}  // extern "C"

namespace {

// Worker threads for the whole-tensor calls: environment LZ_CPU_THREADS, else
// the hardware concurrency (at most 32), never more than there are TGs.
unsigned cpu_threads(uint64_t ntg) {
  const char* e = getenv("LZ_CPU_THREADS");
  unsigned t = e ? (unsigned)atoi(e) : std::thread::hardware_concurrency();
  if (t < 1) t = 1;
  if (t > 32) t = 32;
  if ((uint64_t)t > ntg) t = (unsigned)(ntg ? ntg : 1);
  return t;
}

// Runs fn(t) for t in [0, ntg) on cpu_threads(ntg) threads (dynamic split).
template <class F>
void parallel_tgs(uint64_t ntg, F fn) {
  const unsigned nt = cpu_threads(ntg);
  if (nt <= 1) {
    for (uint64_t t = 0; t < ntg; ++t) fn(t);
    return;
  }
  std::atomic<uint64_t> next{0};
  std::vector<std::thread> pool;
  pool.reserve(nt);
  for (unsigned k = 0; k < nt; ++k)
    pool.emplace_back([&]() {
      for (uint64_t t = next++; t < ntg; t = next++) fn(t);
    });
  for (auto& th : pool) th.join();
}

}  // namespace

extern "C" {

// Whole-tensor compact stream. Returns bytes written or a negative code.
// Table groups are encoded in parallel into per-TG scratch, then packed in
// order, so the stream is the same byte for byte whatever the thread count.
// `dt_arg`: dtype code | level << CODEC_LEVEL_SHIFT.
int64_t lzc_encode(const void* data, uint64_t n, int dt_arg, void* out_, uint64_t cap) {
  const int dt = codec_dtype(dt_arg);
  if (!valid_dtype(dt) || !valid_level(codec_level(dt_arg))) return -1;
  if (cap < max_stream_bytes(n, dt)) return -1;
  uint8_t* out = static_cast<uint8_t*>(out_);
  const uint64_t ntg = num_tgs(n);
  StreamHeader sh;
  memset(&sh, 0, sizeof(sh));
  sh.magic = STREAM_MAGIC;
  sh.version = VERSION;
  sh.dtype = (uint8_t)dt;
  sh.tg_elems = TG_ELEMS;
  sh.n_tg = (uint32_t)ntg;
  sh.n_elems = n;
  uint64_t off = sizeof(StreamHeader) + pad16_64(8 * ntg);
  memset(out + sizeof(StreamHeader), 0, pad16_64(8 * ntg));
  const int es = elem_bytes(dt);
  const uint64_t tcap = tg_capacity(dt);
  std::vector<uint8_t> scratch(ntg * tcap);
  std::vector<int64_t> sizes(ntg, 0);
  parallel_tgs(ntg, [&](uint64_t t) {
    const uint32_t tn = (uint32_t)std::min<uint64_t>(TG_ELEMS, n - t * TG_ELEMS);
    sizes[t] = lzc_tg_encode(static_cast<const uint8_t*>(data) + t * TG_ELEMS * es, tn, dt_arg, &scratch[t * tcap]);
  });
  std::vector<uint64_t> offs(ntg);
  for (uint64_t t = 0; t < ntg; ++t) {
    if (sizes[t] < 0) return sizes[t];
    offs[t] = off;
    memcpy(out + sizeof(StreamHeader) + 8 * t, &off, 8);
    off += (uint64_t)sizes[t];
  }
  parallel_tgs(ntg, [&](uint64_t t) { memcpy(out + offs[t], &scratch[t * tcap], (size_t)sizes[t]); });
  sh.total_bytes = off;
  memcpy(out, &sh, sizeof(sh));
  return (int64_t)off;
}

int lzc_decode(const void* stream_, uint64_t bytes, void* out, uint64_t n, int dt) {
  dt = codec_dtype(dt);
  const uint8_t* st = static_cast<const uint8_t*>(stream_);
  if (bytes < sizeof(StreamHeader)) return -2;
  StreamHeader sh;
  memcpy(&sh, st, sizeof(sh));
  if (sh.magic != STREAM_MAGIC || sh.version != VERSION || sh.dtype != dt || sh.n_elems != n ||
      sh.tg_elems != TG_ELEMS || sh.n_tg != num_tgs(n) || sh.total_bytes > bytes)
    return -3;
  const int es = elem_bytes(dt);
  std::atomic<int> first_err{0};
  parallel_tgs(sh.n_tg, [&](uint64_t t) {
    uint64_t off;
    memcpy(&off, st + sizeof(StreamHeader) + 8 * t, 8);
    int rc = -4;
    if (off < sh.total_bytes) {
      const uint32_t tn = (uint32_t)std::min<uint64_t>(TG_ELEMS, n - t * TG_ELEMS);
      rc = lzc_tg_decode(st + off, sh.total_bytes - off, static_cast<uint8_t*>(out) + t * TG_ELEMS * es, tn, dt);
    }
    if (rc) {
      int expect = 0;
      first_err.compare_exchange_strong(expect, rc);
    }
  });
  return first_err.load();
}

// Symbol histogram (for entropy reporting).
void lzc_histogram(const void* data, uint64_t n, int dt, uint64_t* counts) {
  uint8_t raw[4];
  for (int s = 0; s < 256; ++s) counts[s] = 0;
  for (uint64_t i = 0; i < n; ++i) {
    uint8_t sym;
    split_elem(static_cast<const uint8_t*>(data), dt, (uint32_t)i, &sym, raw);
    counts[sym]++;
  }
}

// ---- fp8 -------------------------------------------------------------------
// Pair containers (layouts in lz_codec_format.h).
void lz_cpu_pack_e4m3(const uint8_t* in, uint16_t* out, uint64_t npairs) {
  for (uint64_t i = 0; i < npairs; ++i) out[i] = pack_e4m3(in[2 * i], in[2 * i + 1]);
}
void lz_cpu_unpack_e4m3(const uint16_t* in, uint8_t* out, uint64_t npairs) {
  for (uint64_t i = 0; i < npairs; ++i) unpack_e4m3(in[i], out + 2 * i, out + 2 * i + 1);
}
void lz_cpu_pack_e5m2(const uint8_t* in, uint16_t* out, uint64_t npairs) {
  for (uint64_t i = 0; i < npairs; ++i) out[i] = pack_e5m2(in[2 * i], in[2 * i + 1]);
}
void lz_cpu_unpack_e5m2(const uint16_t* in, uint8_t* out, uint64_t npairs) {
  for (uint64_t i = 0; i < npairs; ++i) unpack_e5m2(in[i], out + 2 * i, out + 2 * i + 1);
}

}  // extern "C"
