// Host-side encoder internals (no CUDA). See ws_format.h for the stream format.
#pragma once
#include <stdint.h>

#include <vector>

#include "ws_format.h"

namespace ws {

// One encoded block (WS_BLOCK_BYTES of weights) of a packet.
struct EncodedBlock {
  uint32_t offset;  // byte offset of the block inside its packet
  uint32_t nbytes;  // weight bytes covered
  uint16_t kind;    // ws_kind
  uint8_t tail;
  uint8_t flags;
  uint32_t nwords;  // ANS stream halfwords incl. header (0 for RAW)
  std::vector<uint8_t> payload;  // padded to WS_PAYLOAD_ALIGN
  uint32_t clen = 0;             // payload bytes when the payload is held in an arena chunk instead
  uint64_t lane_sum[2];          // checksum lane sums of the bytes written: [0] forward (B), [1] reverse (A)
};

struct EncodedPacket {
  int mode = WS_MODE_SKIP;       // ws_mode chosen by the reference rule
  uint64_t nbytes = 0;
  uint64_t payload_bytes = 0;    // size compared in the mode choice (delta.py:188, 192)
  uint64_t zero_block_bytes = 0;
  uint32_t table[512];           // slot entries, plane 0 then plane 1 (ANS modes only)
  std::vector<EncodedBlock> blocks;  // non-zero blocks in order
};

// Coding choices of a plan (ws_build_options).
struct CodingOptions {
  int dict_slack_pct = 6;  // word dictionary when within this many % of the byte planes' size; < 0: never
  int escapes = 0;         // dictionary with escapes: 0 when smaller, < 0 never, > 0 whenever eligible
  int split = 0;           // split words: 0 the k (0, 1, 2, 4) estimated smallest, < 0 never,
                           // 1, 2 or 4: that k whenever eligible (WS_FLAG_SPLIT_MASK)
};

// Tables of one packet coding: byte planes (two tables) or word dictionary
// (one table for both states, whose symbols index `words`; with `escape`, the
// extra symbol words.size() stands for every other word, decoded as word 0 and
// listed per block after the stream, see WS_FLAG_ESCAPES). A split-word
// dictionary (`split` = k > 0) codes each word with its low k bits cleared
// (`words` have them clear) and stores those bits raw.
struct CodingTables {
  bool dict = false;
  bool escape = false;
  uint32_t split = 0;
  uint32_t entries[512];          // slot entries as the kernel reads them
  uint32_t freq[2][256], cdf[2][256];
  std::vector<uint16_t> words;    // dictionary: word of each kept symbol, increasing
};

// Builds the byte-plane tables from `counts` (plane histograms over the coded
// words) and switches to a word dictionary when one is estimated within
// dict_slack_pct % of the planes' size. Dictionaries: of the words themselves
// or, split, of the words with their low k bits cleared (k = 1, 2 from `words`;
// k = 4 from `high_words`, the distinct values of word & 0xFFF0); each needs
// 2..255 distinct values (`words` increasing, `word_counts` aligned, many_words
// = more than 255 distinct words; likewise high_words / high_counts /
// many_high). A dictionary keeps all its values, or (escapes) only the most
// frequent ones when that is estimated smaller and the escaped words are at
// most 1 % of the words. The smallest estimate wins (ties: smaller k).
void choose_coding(const uint64_t counts[2][256], const std::vector<uint16_t>& words,
                   const std::vector<uint64_t>& word_counts, bool many_words,
                   const std::vector<uint16_t>& high_words, const std::vector<uint64_t>& high_counts,
                   bool many_high, uint32_t coded_blocks, const CodingOptions& co, CodingTables* out);

// Distinct values of (word & ~(2^k - 1)) with summed counts, increasing, from
// the increasing distinct `words` and their counts.
void split_words(const std::vector<uint16_t>& words, const std::vector<uint64_t>& counts, uint32_t k,
                 std::vector<uint16_t>* out_words, std::vector<uint64_t>* out_counts);

// Appends a split-word block's raw section (WS_FLAG_SPLIT_MASK layout) for its
// residual words v[0..W) and k raw bits to a payload whose stream part is
// padded to 16 bytes.
void append_split_raw(const uint16_t* v, uint32_t W, uint32_t k, std::vector<uint8_t>* payload);

// Quantise symbol counts to frequencies summing to WS_PROB_SCALE; every symbol
// with a non-zero count gets frequency >= 1. Greedy fix-up minimising code length.
void quantize_frequencies(const uint64_t counts[256], uint32_t freqs[256]);

// Expand frequencies into 256 slot entries (WS_ENTRY layout).
void build_slot_entries(const uint32_t freqs[256], uint32_t entries[256]);

// Reference residual layout of delta.py:26-34 (low plane then high plane of zigzag).
void u16_residual_reference(const uint8_t* base, const uint8_t* target, uint64_t nbytes, uint8_t* out);

// Encode one packet (<= WS_PACKET_BYTES) following delta.py:176-194 with our codec.
void encode_packet(const uint8_t* base, const uint8_t* target, uint64_t nbytes, bool is_bf16, int policy,
                   const CodingOptions& co, EncodedPacket* out);

// Appends a block's escape list (WS_FLAG_ESCAPES layout) to a payload whose
// stream part is already padded to 16 bytes. lanes[l] = lane l's entries.
void append_escapes(const std::vector<uint32_t> lanes[WS_LANES], std::vector<uint8_t>* payload);

// Checksum lane sum of `n` bytes (one block) as defined in ws_format.h.
uint64_t block_lane_sum(const uint8_t* bytes, uint32_t n);

}  // namespace ws
