// Host encoder: chooses each packet's mode with the reference rule
// (warpshift/delta.py:176-194) and codes ANS modes with this project's
// interleaved rANS format (ws_format.h).
#include "ws_encoder.h"

#include <string.h>

#include <algorithm>
#include <cmath>
#include <numeric>

namespace ws {

namespace {

inline uint32_t round_up16(uint32_t v) { return (v + (WS_PAYLOAD_ALIGN - 1)) & ~(WS_PAYLOAD_ALIGN - 1); }

// U16 representation coded by this format: y = rotr16(zigzag(d), 1) with
// d = (target - base) mod 2^16, so the sign sits in bit 15 and the magnitude in
// bits 0..14. The reference's residual is zigzag(d) itself (delta.py:32-33);
// both are bijections of d, so the applied result is the same.
inline uint16_t u16_symbol_word(uint16_t b, uint16_t t) {
  int32_t d = (int32_t)(int16_t)(uint16_t)(t - b);
  uint32_t z = ((uint32_t)(d * 2) ^ (uint32_t)(d >> 15)) & 0xFFFFu;
  return (uint16_t)((z >> 1) | ((z & 1u) << 15));
}

inline uint16_t load_u16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

struct PlaneTables {
  uint32_t freq[2][256];
  uint32_t cdf[2][256];
};

void tables_from_counts(const uint64_t counts[2][256], PlaneTables* t, uint32_t entries[512]) {
  for (int p = 0; p < 2; ++p) {
    quantize_frequencies(counts[p], t->freq[p]);
    uint32_t c = 0;
    for (int s = 0; s < 256; ++s) {
      t->cdf[p][s] = c;
      c += t->freq[p][s];
    }
    build_slot_entries(t->freq[p], entries + 256 * p);
  }
}

// Symbol schedule of one block. Byte planes: state 0 decodes the low byte and
// state 1 the high byte of each of the lane's 8 words per group, 2 words per
// check (4 checks per group). Word dictionary: state 0 decodes the lane's words
// 0, 2, 4, 6 and state 1 words 1, 3, 5, 7, one word per step, 2 steps per check
// (2 checks per group). Symbol (check c, step k) of state s for lane l is the
// one of word w = 256 g + 8 l + j; it is absent when w >= W.
struct Schedule {
  bool dict;
  uint32_t checks_per_group() const { return dict ? 2u : 4u; }
  uint32_t word(uint32_t g, uint32_t l, uint32_t c, uint32_t k, uint32_t s) const {
    const uint32_t j = dict ? (4u * c + 2u * k + s) : (2u * c + k);
    return g * WS_GROUP_WORDS + l * WS_WORDS_PER_LANE + j;
  }
};

// Encode one block in the decoder's interleaved order. At each check the
// decoder reads one word for every lane whose state-0 value fell below 2^16
// (lane order), then for every state-1 value. Encoding runs backwards, so
// words are pushed in the mirrored order and reversed at the end.
//
// Renormalisation rule (proof sketch): with M = 2^8 and I = [2^16, 2^32), the
// states x that encode the pair (a then b in decode order) into I form the
// interval [fa*fb, 2^16*fa*fb); for a single symbol, [2^8*f, 2^24*f). So the
// encoder emits one 16-bit word exactly when x >= 2^16*fa*fb (resp. 2^24*f).
// sym[s][w] is state s's symbol for word w; freq/cdf[s] its table.
void encode_ans_block(const Schedule& sc, const uint8_t* const sym[2], uint32_t W, const uint32_t* const freq[2],
                      const uint32_t* const cdf[2], std::vector<uint8_t>* payload, uint32_t* nwords) {
  uint32_t st[2][WS_LANES];
  for (int p = 0; p < 2; ++p)
    for (uint32_t l = 0; l < WS_LANES; ++l) st[p][l] = WS_RANS_L;
  std::vector<uint16_t> rev;
  rev.reserve(W + 64);
  const uint32_t groups = (W + WS_GROUP_WORDS - 1) / WS_GROUP_WORDS;
  const uint32_t cpg = sc.checks_per_group();
  const uint32_t checks = groups * cpg;
  for (uint32_t cc = checks; cc-- > 0;) {
    const uint32_t g = cc / cpg, c = cc % cpg;
    for (int p = 1; p >= 0; --p) {
      const uint8_t* sy = sym[p];
      const uint32_t* fq = freq[p];
      const uint32_t* cd = cdf[p];
      for (int l = WS_LANES - 1; l >= 0; --l) {
        const uint32_t wa = sc.word(g, (uint32_t)l, c, 0, (uint32_t)p);
        if (wa >= W) continue;
        const uint32_t wb = sc.word(g, (uint32_t)l, c, 1, (uint32_t)p);
        const bool has_b = wb < W;
        uint32_t x = st[p][l];
        const uint32_t sa = sy[wa];
        const uint32_t fa = fq[sa];
        uint64_t xmax;
        uint32_t sb = 0, fb = 0;
        if (has_b) {
          sb = sy[wb];
          fb = fq[sb];
          xmax = ((uint64_t)fa * fb) << 16;
        } else {
          xmax = (uint64_t)fa << 24;
        }
        if ((uint64_t)x >= xmax) {
          rev.push_back((uint16_t)(x & 0xFFFFu));
          x >>= 16;
        }
        if (has_b) x = ((x / fb) << WS_PROB_BITS) + (x % fb) + cd[sb];
        x = ((x / fa) << WS_PROB_BITS) + (x % fa) + cd[sa];
        st[p][l] = x;
      }
    }
  }
  const uint32_t stream = (uint32_t)rev.size();
  *nwords = WS_HEADER_HALFWORDS + stream;
  const uint32_t bytes = round_up16(2u * *nwords);
  payload->assign(bytes, 0);
  uint8_t* out = payload->data();
  for (int p = 0; p < 2; ++p)
    for (uint32_t l = 0; l < WS_LANES; ++l) {
      uint32_t v = st[p][l];
      memcpy(out + 4 * (p * WS_LANES + l), &v, 4);
    }
  uint8_t* w = out + 2 * WS_HEADER_HALFWORDS;
  for (uint32_t k = 0; k < stream; ++k) {
    uint16_t v = rev[stream - 1 - k];
    w[2 * k] = (uint8_t)(v & 0xFF);
    w[2 * k + 1] = (uint8_t)(v >> 8);
  }
}

bool all_zero_xor(const uint8_t* a, const uint8_t* b, uint64_t n) {
  uint64_t i = 0, acc = 0;
  for (; i + 8 <= n; i += 8) {
    uint64_t x, y;
    memcpy(&x, a + i, 8);
    memcpy(&y, b + i, 8);
    acc |= x ^ y;
    if (acc) return false;
  }
  for (; i < n; ++i) acc |= (uint64_t)(a[i] ^ b[i]);
  return acc == 0;
}

// Candidate encoding of one packet with the given symbol transform.
struct Candidate {
  uint64_t size = 0;
  uint32_t table[512];
  std::vector<EncodedBlock> blocks;
};

// Estimated payload bytes of a coding: ideal code length under the quantised
// frequencies plus per-block header and padding.
double estimate_bytes(const uint64_t* counts, const uint32_t* freq, int nsym, uint32_t nblocks) {
  double bits = 0;
  for (int s = 0; s < nsym; ++s)
    if (counts[s]) bits += (double)counts[s] * std::log2((double)WS_PROB_SCALE / (double)freq[s]);
  return bits / 8.0 + nblocks * (2.0 * WS_HEADER_HALFWORDS + 10.0);
}

template <bool U16>
inline uint16_t residual_word(const uint8_t* base, const uint8_t* target, uint64_t w) {
  if (U16) return u16_symbol_word(load_u16(base + 2 * w), load_u16(target + 2 * w));
  return (uint16_t)(load_u16(base + 2 * w) ^ load_u16(target + 2 * w));
}

// Builds the packet's coding for one residual transform: the byte-plane coding,
// or the word-dictionary coding when the packet's words take 2..255 distinct
// values and its estimated size is within dict_slack_pct percent of the planes'.
template <bool U16>
void build_candidate(const uint8_t* base, const uint8_t* target, uint64_t n, const std::vector<uint8_t>& nonzero,
                     const CodingOptions& co, Candidate* cand) {
  const uint64_t W = n / 2;  // coded words; an odd last byte is carried raw in the block's tail field
  uint64_t counts[2][256];
  memset(counts, 0, sizeof(counts));
  std::vector<uint32_t> word_counts(65536, 0);
  const uint32_t nblk = (uint32_t)((n + WS_BLOCK_BYTES - 1) / WS_BLOCK_BYTES);
  uint32_t coded_blocks = 0;
  for (uint32_t k = 0; k < nblk; ++k) {
    if (!nonzero[k]) continue;
    ++coded_blocks;
    const uint64_t w0 = (uint64_t)k * (WS_BLOCK_BYTES / 2);
    const uint64_t w1 = std::min<uint64_t>(W, w0 + WS_BLOCK_BYTES / 2);
    for (uint64_t w = w0; w < w1; ++w) {
      const uint16_t v = residual_word<U16>(base, target, w);
      counts[0][v & 0xFF]++;
      counts[1][v >> 8]++;
      word_counts[v]++;
    }
  }
  // Word dictionary candidates: the distinct words in increasing order, and the
  // distinct values of their high 12 bits.
  std::vector<uint16_t> words, high_words;
  std::vector<uint64_t> wcounts, high_counts;
  for (uint32_t v = 0; v < 65536; ++v)
    if (word_counts[v]) {
      words.push_back((uint16_t)v);
      wcounts.push_back(word_counts[v]);
    }
  split_words(words, wcounts, 4, &high_words, &high_counts);
  CodingTables ct;
  choose_coding(counts, words, wcounts, words.size() > 255, high_words, high_counts, high_words.size() > 255,
                coded_blocks, co, &ct);
  const bool use_dict = ct.dict;
  const uint32_t k = ct.split;
  const uint16_t keep = (uint16_t)~((1u << k) - 1u);  // the coded part of a word
  const uint8_t esc = (uint8_t)ct.words.size();  // the escape symbol (when ct.escape)
  std::vector<uint8_t> index_of;
  if (use_dict) {
    index_of.assign(65536, ct.escape ? esc : 0);
    for (size_t i = 0; i < ct.words.size(); ++i) index_of[ct.words[i]] = (uint8_t)i;
  }
  std::vector<uint32_t> lanes[WS_LANES];
  memcpy(cand->table, ct.entries, sizeof(cand->table));
  cand->size = 1024;  // compact per-packet tables (frequencies, and the dictionary words)
  const Schedule sc{use_dict};
  const uint32_t* freq[2] = {ct.freq[0], ct.freq[1]};
  const uint32_t* cdf[2] = {ct.cdf[0], ct.cdf[1]};
  std::vector<uint8_t> s0(WS_BLOCK_BYTES / 2), s1(WS_BLOCK_BYTES / 2);
  std::vector<uint16_t> vw(WS_BLOCK_BYTES / 2);
  for (uint32_t b = 0; b < nblk; ++b) {
    if (!nonzero[b]) continue;
    EncodedBlock blk;
    blk.offset = b * WS_BLOCK_BYTES;
    blk.nbytes = (uint32_t)std::min<uint64_t>(WS_BLOCK_BYTES, n - blk.offset);
    blk.tail = 0;
    blk.flags = 0;
    const uint32_t wb = blk.nbytes / 2;
    const uint8_t* bb = base + blk.offset;
    const uint8_t* tb = target + blk.offset;
    for (auto& l : lanes) l.clear();
    for (uint32_t w = 0; w < wb; ++w) {
      const uint16_t v = residual_word<U16>(bb, tb, w);
      vw[w] = v;
      if (use_dict) {
        const uint16_t h = (uint16_t)(v & keep);
        s0[w] = s1[w] = index_of[h];
        if (ct.escape && index_of[h] == esc)
          lanes[(w % WS_GROUP_WORDS) / WS_WORDS_PER_LANE].push_back(w | ((uint32_t)h << 16));
      } else {
        s0[w] = (uint8_t)(v & 0xFF);
        s1[w] = (uint8_t)(v >> 8);
      }
    }
    size_t most = 0, escaped = 0;
    for (const auto& l : lanes) {
      most = std::max(most, l.size());
      escaped += l.size();
    }
    if (blk.nbytes & 1u) {
      blk.flags |= WS_FLAG_ODD_TAIL;
      blk.tail = (uint8_t)(bb[blk.nbytes - 1] ^ tb[blk.nbytes - 1]);
    }
    const uint8_t* sym[2] = {s0.data(), s1.data()};
    encode_ans_block(sc, sym, wb, freq, cdf, &blk.payload, &blk.nwords);
    blk.kind = use_dict ? (U16 ? WS_KIND_DICT_U16 : WS_KIND_DICT_XOR) : (U16 ? WS_KIND_ANS_U16 : WS_KIND_ANS_XOR);
    if (k) {
      blk.flags |= (uint8_t)ws_split_flags(k);
      append_split_raw(vw.data(), wb, k, &blk.payload);
    }
    if (escaped) {
      blk.flags |= WS_FLAG_ESCAPES;
      append_escapes(lanes, &blk.payload);
    }
    const uint32_t raw = round_up16(blk.nbytes);
    if (blk.payload.size() >= raw || most > WS_ESCAPE_LANE_MAX) {  // incompressible, or too many escapes: raw XOR
      blk.kind = WS_KIND_RAW;
      blk.flags = 0;
      blk.tail = 0;
      blk.nwords = 0;
      blk.payload.assign(raw, 0);
      for (uint32_t i = 0; i < blk.nbytes; ++i) blk.payload[i] = (uint8_t)(bb[i] ^ tb[i]);
    }
    blk.lane_sum[0] = block_lane_sum(tb, blk.nbytes);
    blk.lane_sum[1] = block_lane_sum(bb, blk.nbytes);
    cand->size += blk.payload.size();
    cand->blocks.push_back(std::move(blk));
  }
}

}  // namespace

void quantize_frequencies(const uint64_t counts[256], uint32_t f[256]) {
  uint64_t total = 0;
  int present = 0, last = 0;
  for (int s = 0; s < 256; ++s) {
    total += counts[s];
    if (counts[s]) {
      ++present;
      last = s;
    }
    f[s] = 0;
  }
  if (present == 0) return;
  if (present == 1) {
    f[last] = WS_PROB_SCALE;
    return;
  }
  int64_t sum = 0;
  for (int s = 0; s < 256; ++s) {
    if (!counts[s]) continue;
    uint64_t v = (uint64_t)((unsigned __int128)counts[s] * WS_PROB_SCALE / total);
    f[s] = v ? (uint32_t)v : 1u;
    sum += f[s];
  }
  // Greedy fix-up: each +1/-1 step picks the symbol whose code length changes most/least.
  while (sum < (int64_t)WS_PROB_SCALE) {
    int best = -1;
    double best_gain = -1.0;
    for (int s = 0; s < 256; ++s) {
      if (!counts[s]) continue;
      double gain = (double)counts[s] * std::log2((double)(f[s] + 1) / (double)f[s]);
      if (gain > best_gain) {
        best_gain = gain;
        best = s;
      }
    }
    f[best]++;
    ++sum;
  }
  while (sum > (int64_t)WS_PROB_SCALE) {
    int best = -1;
    double best_loss = 0.0;
    for (int s = 0; s < 256; ++s) {
      if (f[s] <= 1) continue;
      double loss = (double)counts[s] * std::log2((double)f[s] / (double)(f[s] - 1));
      if (best < 0 || loss < best_loss) {
        best_loss = loss;
        best = s;
      }
    }
    f[best]--;
    --sum;
  }
}

void build_slot_entries(const uint32_t freqs[256], uint32_t entries[256]) {
  uint32_t slot = 0;
  for (uint32_t s = 0; s < 256; ++s)
    for (uint32_t k = 0; k < freqs[s]; ++k, ++slot) entries[slot] = WS_ENTRY(k, s, freqs[s]);
  for (; slot < 256; ++slot) entries[slot] = 0;  // only reachable for an empty table
}

namespace {

// Dictionary tables from symbol counts (symbol i = words[i], plus the escape
// symbol words.size() when `escape`); returns the estimated payload bytes.
double dict_tables(const std::vector<uint16_t>& words, const uint64_t* sym_counts, bool escape, uint64_t escaped,
                   uint32_t coded_blocks, CodingTables* out) {
  uint64_t dcounts[256];
  uint32_t dict_freq[256];
  memset(dcounts, 0, sizeof(dcounts));
  const size_t nsym = words.size() + (escape ? 1 : 0);
  for (size_t i = 0; i < nsym; ++i) dcounts[i] = sym_counts[i];
  quantize_frequencies(dcounts, dict_freq);
  double est = estimate_bytes(dcounts, dict_freq, 256, coded_blocks);
  if (escape) est += 4.0 * (double)escaped + (double)coded_blocks * WS_ESCAPE_HEADER_BYTES;
  if (out) {
    out->dict = true;
    out->escape = escape;
    out->words = words;
    uint32_t c = 0, slot = 0;
    for (uint32_t i = 0; i < 256; ++i) {
      out->freq[0][i] = out->freq[1][i] = dict_freq[i];
      out->cdf[0][i] = out->cdf[1][i] = c;
      c += dict_freq[i];
    }
    memset(out->entries, 0, sizeof(out->entries));
    for (size_t i = 0; i < nsym; ++i) {
      const uint16_t word = i < words.size() ? words[i] : 0;  // the escape symbol decodes as 0: no change
      for (uint32_t k = 0; k < dict_freq[i]; ++k, ++slot) out->entries[slot] = WS_DICT_ENTRY(k, word, dict_freq[i]);
    }
  }
  return est;
}

}  // namespace

namespace {

// Estimated size a split-word dictionary must save over the whole-word one.
constexpr double kSplitGainPct = 3.0;

// The best dictionary of one symbol alphabet (distinct values `words`,
// increasing, with `counts`): every value a symbol, or (escapes) the K most
// frequent ones (ties: smaller value first) plus the escape symbol. Returns the
// estimated payload bytes, with `raw_bytes` added for a split coding's raw
// sections, and the number of kept symbols in *kept (words.size() when none is
// escaped); with `out`, fills the tables.
double best_dictionary(const std::vector<uint16_t>& words, const std::vector<uint64_t>& counts, double raw_bytes,
                       uint32_t coded_blocks, const CodingOptions& co, size_t* kept, CodingTables* out) {
  double best = dict_tables(words, counts.data(), false, 0, coded_blocks, nullptr) + raw_bytes;
  size_t best_k = words.size();
  std::vector<uint32_t> order(words.size());
  std::iota(order.begin(), order.end(), 0u);
  std::stable_sort(order.begin(), order.end(), [&](uint32_t x, uint32_t y) { return counts[x] > counts[y]; });
  auto subset = [&](size_t k, std::vector<uint16_t>* kw, std::vector<uint64_t>* kc) {
    uint64_t escaped = 0;
    for (size_t r = k; r < order.size(); ++r) escaped += counts[order[r]];
    std::vector<uint32_t> keep(order.begin(), order.begin() + k);
    std::sort(keep.begin(), keep.end());
    kw->clear();
    kc->clear();
    for (uint32_t i : keep) {
      kw->push_back(words[i]);
      kc->push_back(counts[i]);
    }
    kc->push_back(escaped);
    return escaped;
  };
  if (co.escapes >= 0) {
    const uint64_t total = std::accumulate(counts.begin(), counts.end(), (uint64_t)0);
    bool first = true;
    std::vector<uint16_t> kw;
    std::vector<uint64_t> kc;
    for (size_t k : {8, 12, 16, 24, 32, 48, 64, 96, 128, 192}) {
      if (k >= words.size()) break;
      const uint64_t escaped = subset(k, &kw, &kc);
      if (escaped * 100 > total) continue;  // keep the per-lane lists short
      const double est = dict_tables(kw, kc.data(), true, escaped, coded_blocks, nullptr) + raw_bytes;
      if (est < best || (co.escapes > 0 && first)) {
        best = est;
        best_k = k;
        first = false;
      }
    }
  }
  *kept = best_k;
  if (out) {
    if (best_k == words.size()) {
      dict_tables(words, counts.data(), false, 0, coded_blocks, out);
    } else {
      std::vector<uint16_t> kw;
      std::vector<uint64_t> kc;
      const uint64_t escaped = subset(best_k, &kw, &kc);
      dict_tables(kw, kc.data(), true, escaped, coded_blocks, out);
    }
  }
  return best;
}

}  // namespace

void split_words(const std::vector<uint16_t>& words, const std::vector<uint64_t>& counts, uint32_t k,
                 std::vector<uint16_t>* out_words, std::vector<uint64_t>* out_counts) {
  const uint16_t keep = (uint16_t)~((1u << k) - 1u);
  out_words->clear();
  out_counts->clear();
  for (size_t i = 0; i < words.size(); ++i) {  // increasing words keep equal high parts adjacent
    const uint16_t h = (uint16_t)(words[i] & keep);
    if (!out_words->empty() && out_words->back() == h) {
      out_counts->back() += counts[i];
    } else {
      out_words->push_back(h);
      out_counts->push_back(counts[i]);
    }
  }
}

void choose_coding(const uint64_t counts[2][256], const std::vector<uint16_t>& words,
                   const std::vector<uint64_t>& word_counts, bool many_words,
                   const std::vector<uint16_t>& high_words, const std::vector<uint64_t>& high_counts,
                   bool many_high, uint32_t coded_blocks, const CodingOptions& co, CodingTables* out) {
  PlaneTables t;
  uint32_t plane_entries[512];
  tables_from_counts(counts, &t, plane_entries);
  const double planes_est = estimate_bytes(counts[0], t.freq[0], 256, coded_blocks) +
                            estimate_bytes(counts[1], t.freq[1], 256, 0);
  out->dict = false;
  out->escape = false;
  out->split = 0;
  out->words.clear();
  if (co.dict_slack_pct >= 0) {
    // Candidate alphabets: k = 0 (the words), 1, 2 (derived from the words) and
    // 4 (the high 12 bits, counted separately because the words may be too many).
    double best = 0;
    int best_k = -1;
    size_t best_kept = 0;
    std::vector<uint16_t> best_words;
    std::vector<uint64_t> best_counts;
    for (uint32_t k : {0u, 1u, 2u, 4u}) {
      const bool allowed = co.split > 0 ? k == (uint32_t)co.split : (k == 0 || co.split == 0);
      if (!allowed) continue;
      std::vector<uint16_t> sw;
      std::vector<uint64_t> sc;
      if (k == 4 && !many_high) {
        sw = high_words;
        sc = high_counts;
      } else if (k < 4 && !many_words) {
        split_words(words, word_counts, k, &sw, &sc);
      } else {
        continue;
      }
      if (sw.size() < 2 || sw.size() > 255) continue;
      const double raw_bytes = (double)coded_blocks * ws_split_raw_bytes(WS_BLOCK_BYTES / 2, k);
      size_t kept;
      const double est = best_dictionary(sw, sc, raw_bytes, coded_blocks, co, &kept, nullptr);
      // A split block decodes more slowly (its raw bits are a second read and
      // a table lookup per group), so unless forced a split coding must beat
      // the whole-word dictionary by kSplitGainPct of its size.
      const double bar = (best_k == 0 && co.split == 0) ? best * (1.0 - kSplitGainPct / 100.0) : best;
      const bool wins = best_k < 0 || est < bar;
      if (wins) {
        best = est;
        best_k = (int)k;
        best_kept = kept;
        best_words = std::move(sw);
        best_counts = std::move(sc);
      }
    }
    // A forced split, or forced escapes that escape something, take the dictionary
    // whatever its estimate.
    const bool forced = best_k >= 0 && (co.split > 0 || (co.escapes > 0 && best_kept < best_words.size()));
    if (best_k >= 0 && (forced || best <= planes_est * (1.0 + co.dict_slack_pct / 100.0))) {
      size_t kept;
      best_dictionary(best_words, best_counts,
                      (double)coded_blocks * ws_split_raw_bytes(WS_BLOCK_BYTES / 2, (uint32_t)best_k), coded_blocks,
                      co, &kept, out);
      out->split = (uint32_t)best_k;
      return;
    }
  }
  memcpy(out->entries, plane_entries, sizeof(out->entries));
  memcpy(out->freq, t.freq, sizeof(out->freq));
  memcpy(out->cdf, t.cdf, sizeof(out->cdf));
}

void append_split_raw(const uint16_t* v, uint32_t W, uint32_t k, std::vector<uint8_t>* payload) {
  const uint32_t bytes = ws_split_raw_bytes(W, k);
  if (!bytes) return;
  std::vector<uint32_t> raw(bytes / 4, 0);
  const uint32_t per = 4u / k, mask = (1u << k) - 1u;
  for (uint32_t w = 0; w < W; ++w) {
    const uint32_t g = w / WS_GROUP_WORDS, lane = (w % WS_GROUP_WORDS) / WS_WORDS_PER_LANE, j = w % WS_WORDS_PER_LANE;
    const uint32_t bit = (g % per) * 8u * k + j * k;
    raw[(g / per) * WS_LANES + lane] |= ((uint32_t)v[w] & mask) << bit;
  }
  const size_t at = payload->size();
  payload->resize(at + bytes);
  memcpy(payload->data() + at, raw.data(), bytes);
}

void u16_residual_reference(const uint8_t* base, const uint8_t* target, uint64_t nbytes, uint8_t* out) {
  const uint64_t W = nbytes / 2;
  for (uint64_t w = 0; w < W; ++w) {
    int32_t d = (int32_t)(int16_t)(uint16_t)(load_u16(target + 2 * w) - load_u16(base + 2 * w));
    uint32_t z = ((uint32_t)(d * 2) ^ (uint32_t)(d >> 15)) & 0xFFFFu;
    out[w] = (uint8_t)(z & 0xFF);
    out[W + w] = (uint8_t)(z >> 8);
  }
}

uint64_t block_lane_sum(const uint8_t* bytes, uint32_t n) {
  const uint32_t groups = (n + WS_GROUP_BYTES - 1) / WS_GROUP_BYTES;
  uint64_t sum = 0;
  for (uint32_t l = 0; l < WS_LANES; ++l) {
    uint32_t a = 0, b = 0;
    for (uint32_t g = 0; g < groups; ++g) {
      const uint32_t off = g * WS_GROUP_BYTES + l * 16u;
      uint8_t chunk[16];
      memset(chunk, 0, 16);
      if (off < n) memcpy(chunk, bytes + off, std::min<uint32_t>(16u, n - off));
      uint32_t w[4];
      memcpy(w, chunk, 16);
      a += w[0] + w[1] + w[2] + w[3];
      b += a;
    }
    sum += ws_lane_hash(a, b, l);
  }
  return sum;
}

void append_escapes(const std::vector<uint32_t> lanes[WS_LANES], std::vector<uint8_t>* payload) {
  size_t at = payload->size();
  size_t total = 0;
  for (uint32_t l = 0; l < WS_LANES; ++l) total += lanes[l].size();
  payload->resize(round_up16((uint32_t)(at + WS_ESCAPE_HEADER_BYTES + 4 * total)), 0);
  uint8_t* p = payload->data() + at;
  for (uint32_t l = 0; l < WS_LANES; ++l) {
    const uint16_t c = (uint16_t)lanes[l].size();
    memcpy(p + 2 * l, &c, 2);
  }
  p += WS_ESCAPE_HEADER_BYTES;
  for (uint32_t l = 0; l < WS_LANES; ++l) {
    memcpy(p, lanes[l].data(), 4 * lanes[l].size());
    p += 4 * lanes[l].size();
  }
}

void encode_packet(const uint8_t* base, const uint8_t* target, uint64_t n, bool is_bf16, int policy,
                   const CodingOptions& co, EncodedPacket* out) {
  out->nbytes = n;
  out->blocks.clear();
  out->zero_block_bytes = 0;
  out->payload_bytes = 0;
  if (n == 0 || all_zero_xor(base, target, n)) {
    out->mode = WS_MODE_SKIP;
    return;
  }
  const uint32_t nblk = (uint32_t)((n + WS_BLOCK_BYTES - 1) / WS_BLOCK_BYTES);
  std::vector<uint8_t> nonzero(nblk);
  for (uint32_t k = 0; k < nblk; ++k) {
    const uint64_t off = (uint64_t)k * WS_BLOCK_BYTES;
    const uint64_t len = std::min<uint64_t>(WS_BLOCK_BYTES, n - off);
    nonzero[k] = !all_zero_xor(base + off, target + off, len);
    if (!nonzero[k]) out->zero_block_bytes += len;
  }
  // delta.py:184: raw XOR is the default; its size is the packet size.
  int mode = WS_MODE_XOR_RAW;
  uint64_t best = n;
  Candidate chosen;
  const bool big = n >= WS_COMPRESS_MIN;  // delta.py:185
  const bool try_xor = big && !(policy == 2 && is_bf16);
  const bool try_u16 = big && is_bf16 && (n % 2 == 0) && policy != 1;
  if (try_xor) {
    Candidate c;
    build_candidate<false>(base, target, n, nonzero, co, &c);
    if (c.size < best) {  // delta.py:188-189: strictly smaller replaces raw
      best = c.size;
      mode = (n % 2 == 0) ? WS_MODE_XOR_GROUP2_ANS : WS_MODE_XOR_ANS;
      chosen = std::move(c);
    }
  }
  if (try_u16) {
    Candidate c;
    build_candidate<true>(base, target, n, nonzero, co, &c);
    if (c.size < best) {  // delta.py:192-193: strictly smaller than the current best
      best = c.size;
      mode = WS_MODE_U16_ANS;
      chosen = std::move(c);
    }
  }
  out->mode = mode;
  out->payload_bytes = best;
  if (mode == WS_MODE_XOR_RAW) {
    memset(out->table, 0, sizeof(out->table));
    for (uint32_t k = 0; k < nblk; ++k) {
      if (!nonzero[k]) continue;
      EncodedBlock blk;
      blk.offset = k * WS_BLOCK_BYTES;
      blk.nbytes = (uint32_t)std::min<uint64_t>(WS_BLOCK_BYTES, n - blk.offset);
      blk.kind = WS_KIND_RAW;
      blk.tail = 0;
      blk.flags = 0;
      blk.nwords = 0;
      blk.payload.assign(round_up16(blk.nbytes), 0);
      const uint8_t* bb = base + blk.offset;
      const uint8_t* tb = target + blk.offset;
      for (uint32_t i = 0; i < blk.nbytes; ++i) blk.payload[i] = (uint8_t)(bb[i] ^ tb[i]);
      blk.lane_sum[0] = block_lane_sum(tb, blk.nbytes);
      blk.lane_sum[1] = block_lane_sum(bb, blk.nbytes);
      out->blocks.push_back(std::move(blk));
    }
  } else {
    memcpy(out->table, chosen.table, sizeof(out->table));
    out->blocks = std::move(chosen.blocks);
  }
}

}  // namespace ws
