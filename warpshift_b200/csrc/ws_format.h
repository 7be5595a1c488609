// Delta stream format shared by the host encoder (ws_encoder.cpp) and the
// sm_100a decode+apply kernel (ws_apply.cu).
//
// What the stream represents follows warpshift/delta.py of the reference:
//   * a tensor is cut into packets of at most 16 MiB (delta.py:20 _CHUNK_BYTES),
//     each with one mode chosen by delta.py:176-194 _encode_chunk:
//       0 XOR_RAW, 1 XOR_GROUP2_ANS, 2 XOR_ANS (odd size), 3 U16_ANS, or SKIP
//       when the packet's XOR is all zero (delta.py:181-182, 209-212);
//   * applying XOR modes computes dst ^= residual, U16 mode computes
//     dst = dst +/- unzigzag(residual) modulo 2^16 (delta.py:74-92).
// The entropy stage is this project's own chunked, interleaved rANS code,
// which replaces nvCOMP's ANS (delta.py:111-113, 164-174, 313-316):
//   * a packet is cut into blocks of 128 KiB of weight bytes; one warp decodes
//     one block; 32 lanes x 2 interleaved 32-bit states (plane 0 = low byte of
//     each uint16 word, plane 1 = high byte) share one 16-bit renormalisation
//     word stream;
//   * per packet there is one 256-slot (8-bit precision) frequency table per
//     plane, expanded into 32-bit slot entries;
//   * a lane owns words 8*lane .. 8*lane+7 of every 256-word (512-byte) group,
//     so after 8 decode steps it holds exactly one aligned 16-byte vector;
//   * states are checked for renormalisation after every second decode step;
//     with 8-bit precision two symbols lower a state by at most 2^16, so one
//     16-bit read per check restores it.
//   * a packet is coded either as two byte planes (above) or, when its 16-bit
//     residual words take at most 255 distinct values, as one symbol per word
//     from a per-packet word dictionary: each slot entry then carries the
//     16-bit word itself, and the lane's two states decode alternate words
//     (state A words 0, 2, 4, 6 and state B words 1, 3, 5, 7 of the lane's 8).
#pragma once
#include <stdint.h>

#define WS_PACKET_BYTES (16u << 20)  // delta.py:20
#define WS_BLOCK_BYTES 131072u       // rANS chunk; one warp per block
#define WS_COMPRESS_MIN 16384u       // delta.py:185 (compression tried only at >= 16384 B)
#define WS_GROUP_WORDS 256u          // one 512-byte group per warp step of 8 words/lane
#define WS_GROUP_BYTES 512u
#define WS_LANES 32u
#define WS_WORDS_PER_LANE 8u         // words per lane per group
#define WS_PROB_BITS 8u
#define WS_PROB_SCALE 256u
#define WS_RANS_L 65536u             // lower bound of the normalised state interval [2^16, 2^32)
#define WS_HEADER_HALFWORDS 128u     // 64 initial states (uint32) at the start of an ANS payload
#define WS_PAYLOAD_ALIGN 16u         // every payload starts and ends 16-byte aligned
#define WS_TILE_BLOCKS 16u           // blocks per CTA tile (one per warp)
#define WS_RING_BYTES 2048u          // per-warp staging ring in shared memory (2 halves)
#define WS_RING_HALF_BYTES 1024u

// Packet modes (delta.py:23 _MODES) plus SKIP.
enum ws_mode { WS_MODE_XOR_RAW = 0, WS_MODE_XOR_GROUP2_ANS = 1, WS_MODE_XOR_ANS = 2, WS_MODE_U16_ANS = 3, WS_MODE_SKIP = 4 };

// Block kinds (per 128 KiB block inside a packet). All-zero blocks are omitted.
enum ws_kind {
  WS_KIND_RAW = 0,       // payload = raw XOR bytes
  WS_KIND_ANS_XOR = 1,   // byte planes, XOR apply
  WS_KIND_ANS_U16 = 2,   // byte planes, wrapping u16 apply
  WS_KIND_DICT_XOR = 3,  // word dictionary, XOR apply
  WS_KIND_DICT_U16 = 4   // word dictionary, wrapping u16 apply
};
#define WS_FLAG_ODD_TAIL 1u  // block's last byte (odd packet size) is not coded; its XOR value is `tail`
// Word-dictionary block with escapes: the packet's dictionary keeps its most
// frequent words plus one escape symbol whose word is 0 (no change in either
// apply), and every escaped word of the block is listed after the stream. The
// list starts at byte align16(2 * nwords) of the payload: uint16 count[32] (the
// entries of each lane, lane l owning words 8l..8l+7 of every 256-word group),
// then the entries grouped by lane in lane order, each uint32 = word index in
// the block (bits 0-15) | coded residual word (bits 16-31), increasing index
// within a lane; zero-padded to 16 bytes. After decoding, each lane applies its
// own entries and corrects its checksum sums.
#define WS_FLAG_ESCAPES 2u
#define WS_ESCAPE_LANE_MAX 64u  // entries per lane at most; an encoder codes a block with more as RAW
#define WS_ESCAPE_HEADER_BYTES 64u
// Split words (word-dictionary blocks only): flags bits 2-3 hold a code c and
// the low k = {0, 1, 2, 4}[c] bits of every residual word are stored raw; the
// dictionary codes the word with those bits cleared (its entries carry the
// word with the low k bits zero, so decoding is unchanged). The raw section
// follows the stream at byte align16(2 * nwords) and precedes any escape list;
// it is read, not staged. It holds uint32 raw words: G = 4 / k groups share one
// word per lane, raw word (g / G) * 32 + lane for group g. Inside it the lane's
// 8k bits of group g are bytes (g % G) * k .. (g % G) * k + k - 1, and its word
// j (of the 8 it owns in the group) has bits [8k * (g % G) + jk, ... + k): a
// byte holds the bits of 8 / k consecutive words, so the kernel expands one
// byte through a 256-entry table. Words past the block's end have zero bits.
// The section is 4 * 32 * ceil(ceil(W / 256) / G) bytes (a multiple of 16). An
// escaped word's list entry carries the word with its low k bits cleared.
#define WS_FLAG_SPLIT_SHIFT 2u
#define WS_FLAG_SPLIT_MASK 0x0Cu

// Device-side errors reported through ws_device_result.errors.
#define WS_DEVERR_STATE 1u     // final rANS state != WS_RANS_L
#define WS_DEVERR_LENGTH 2u    // stream words consumed != nwords
#define WS_DEVERR_TIMEOUT 4u   // a bounded wait on a staging barrier gave up
#define WS_DEVERR_KIND 8u      // unknown block kind
#define WS_DEVERR_BOUNDS 16u   // a caller-written descriptor points outside the caller's arrays (checked applies)

// 32-byte block descriptor (resident in HBM for the plan's lifetime).
typedef struct ws_block_desc {
  uint64_t dst;      // absolute address of the block's first weight byte
  uint64_t src;      // byte offset of the block payload inside the plan arena
  uint32_t nbytes;   // weight bytes covered (1 .. WS_BLOCK_BYTES)
  uint32_t clen;     // payload bytes (multiple of 16)
  uint32_t nwords;   // ANS: stream halfwords incl. the 128-halfword state header; RAW: 0
  uint16_t kind;     // ws_kind
  uint8_t tail;      // XOR value of the last byte when flags & WS_FLAG_ODD_TAIL
  uint8_t flags;
} ws_block_desc;

// 16-byte tile descriptor: up to 16 blocks of one packet, one CTA.
typedef struct ws_tile_desc {
  uint32_t first_block;
  uint32_t nblocks;
  uint32_t table;  // packet table index (512 entries each), or WS_NO_TABLE
  uint32_t split;  // the packet's split code (flags bits 2-3 of its split-word blocks, shifted down), or 0
} ws_tile_desc;
#define WS_NO_TABLE 0xFFFFFFFFu

// Slot entry of a byte-plane table: bits 0-7 bias = slot - cdf[sym], bits 8-15
// sym, bits 16-24 freq (1..256). A packet table holds plane 0 then plane 1.
#define WS_ENTRY(bias, sym, freq) ((uint32_t)(bias) | ((uint32_t)(sym) << 8) | ((uint32_t)(freq) << 16))
// Slot entry of a word-dictionary table: bits 0-15 the residual word, bits
// 16-23 bias, bits 24-31 freq (1..255). Only the first 256 entries are used.
#define WS_DICT_ENTRY(bias, word, freq) ((uint32_t)(word) | ((uint32_t)(bias) << 16) | ((uint32_t)(freq) << 24))

// Accumulators written by the kernel for one apply.
typedef struct ws_device_result {
  unsigned long long checksum;  // sum of per-block hashes of the written bytes
  uint32_t errors;              // OR of WS_DEVERR_*
  uint32_t bad_block_plus1;     // 1 + index of a failing block, 0 if none
} ws_device_result;

// ---------------------------------------------------------------------------
// Checksum of written bytes. For each block and each lane l, over the block's
// 512-byte groups g in order, with w0..w3 the four little-endian uint32 words
// of bytes [512g + 16l, 512g + 16l + 16) after the write (bytes past the block
// end read as 0):  a += w0 + w1 + w2 + w3;  b += a   (mod 2^32).
// lane hash h_l = mix64(((uint64)b << 32 | a) + (l + 1) * K1),
// block hash = mix64(sum_l h_l ^ ((block_index + 1) * K2)); the plan checksum
// is the sum of block hashes (mod 2^64) over all blocks written.
// mix64 is the splitmix64 finaliser (Steele, Lea, Flood 2014).
#define WS_CK_K1 0x9E3779B97F4A7C15ull
#define WS_CK_K2 0xD1B54A32D192ED03ull
// Per-tensor content hash (ws_tensor_hashes): word position and length keys.
#define WS_TH_KPOS 0xC2B2AE3D27D4EB4Full
#define WS_TH_KLEN 0x165667B19E3779F9ull
#define WS_TH_KMUL 0x9E3779B97F4A7C15ull  // odd multiplier of the per-word mix


#ifdef __CUDACC__
#define WS_HD __host__ __device__ __forceinline__
#else
#define WS_HD static inline
#endif

// Raw low bits per word of a split-word block (0 when not split).
WS_HD uint32_t ws_split_bits(uint32_t flags) {
  const uint32_t c = (flags & WS_FLAG_SPLIT_MASK) >> WS_FLAG_SPLIT_SHIFT;
  return c == 3u ? 4u : c;
}
// Flag bits of a split of k raw bits (k in {0, 1, 2, 4}).
WS_HD uint32_t ws_split_flags(uint32_t k) { return (k == 4u ? 3u : k) << WS_FLAG_SPLIT_SHIFT; }
// Bytes of a split-word block's raw section for W coded words and k raw bits.
WS_HD uint32_t ws_split_raw_bytes(uint32_t W, uint32_t k) {
  if (k == 0u) return 0u;
  const uint32_t groups = (W + WS_GROUP_WORDS - 1u) / WS_GROUP_WORDS;
  const uint32_t per = 4u / k;  // groups per raw word
  return 4u * WS_LANES * ((groups + per - 1u) / per);
}

WS_HD uint64_t ws_mix64(uint64_t x) {
  x ^= x >> 30;
  x *= 0xBF58476D1CE4E5B9ull;
  x ^= x >> 27;
  x *= 0x94D049BB133111EBull;
  x ^= x >> 31;
  return x;
}
WS_HD uint64_t ws_lane_hash(uint32_t a, uint32_t b, uint32_t lane) {
  return ws_mix64((((uint64_t)b << 32) | a) + (uint64_t)(lane + 1) * WS_CK_K1);
}
WS_HD uint64_t ws_block_hash(uint64_t lane_sum, uint64_t block_index) {
  return ws_mix64(lane_sum ^ ((block_index + 1) * WS_CK_K2));
}
// Per-word term of the tensor hash: xmul(x) = y ^ (y >> 32) with y = x * KMUL
// (mod 2^64). Multiplying by an odd constant and folding the high half into the
// low half are both bijections, so a change of one word always changes its term.
WS_HD uint64_t ws_xmul64(uint64_t x) {
  const uint64_t y = x * WS_TH_KMUL;
  return y ^ (y >> 32);
}
