// Host-side encoder internals (no CUDA). See ws_format.h for the stream format.
#pragma once
#include <stdint.h>

#include <vector>

#include "ws_format.h"

namespace ws {

// One encoded 64 KiB block of a packet.
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

// Tables of one packet coding: byte planes (two tables) or word dictionary
// (one table for both states, whose symbols index `words`).
struct CodingTables {
  bool dict = false;
  uint32_t entries[512];          // slot entries as the kernel reads them
  uint32_t freq[2][256], cdf[2][256];
  std::vector<uint16_t> words;    // dictionary: word of each symbol, increasing
};

// Builds the byte-plane tables from `counts` (plane histograms over the coded
// words) and switches to the word dictionary when the packet has 2..255
// distinct words (`words` increasing, `word_counts` aligned; many_words = more
// than 255) and its estimated size is within dict_slack_pct % of the planes'.
void choose_coding(const uint64_t counts[2][256], const std::vector<uint16_t>& words,
                   const std::vector<uint64_t>& word_counts, bool many_words, uint32_t coded_blocks, int dict_slack_pct,
                   CodingTables* out);

// Quantise symbol counts to frequencies summing to WS_PROB_SCALE; every symbol
// with a non-zero count gets frequency >= 1. Greedy fix-up minimising code length.
void quantize_frequencies(const uint64_t counts[256], uint32_t freqs[256]);

// Expand frequencies into 256 slot entries (WS_ENTRY layout).
void build_slot_entries(const uint32_t freqs[256], uint32_t entries[256]);

// Reference residual layout of delta.py:26-34 (low plane then high plane of zigzag).
void u16_residual_reference(const uint8_t* base, const uint8_t* target, uint64_t nbytes, uint8_t* out);

// Encode one packet (<= WS_PACKET_BYTES) following delta.py:176-194 with our codec.
// dict_slack_pct: use the word-dictionary coding when its estimated size is at
// most this many percent above the byte-plane coding (negative: never).
void encode_packet(const uint8_t* base, const uint8_t* target, uint64_t nbytes, bool is_bf16, int policy,
                   int dict_slack_pct, EncodedPacket* out);

// Checksum lane sum of `n` bytes (one block) as defined in ws_format.h.
uint64_t block_lane_sum(const uint8_t* bytes, uint32_t n);

}  // namespace ws
