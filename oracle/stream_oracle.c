/*
 * ORACLE — test infrastructure only, never part of the product path.
 *
 * Plain-C, single-threaded-per-block restatement of this project's delta
 * stream format (chunked, interleaved rANS; constants and descriptor layouts
 * in warpshift_b200/csrc/ws_format.h), written independently of the product
 * encoder and the CUDA kernel. Used by tests/ to check (a) that the host encoder's output
 * decodes to the exact residual and (b) that the GPU applied the same bytes,
 * and by bench.py's CPU baseline leg. Parity of the entropy stage against the
 * reference is unpinned: the reference codes with nvCOMP ANS (closed source),
 * so only the residual and the applied bytes are compared with the reference
 * (delta.py:26-34, 74-92, 176-194), never the compressed bytes.
 *
 * Block layout (one weight block of at most 128 KiB, payload 16-byte padded):
 *   uint32 initial states[64]  (plane 0 lanes 0..31, then plane 1 lanes 0..31)
 *   uint16 renormalisation words in decode order
 * Word i (bytes 2i, 2i+1 of the block) belongs to lane (i % 256) / 8 and is
 * decoded at step i % 8 of group i / 256; plane 0 gives its low byte, plane 1
 * its high byte. After steps 1, 3, 5, 7 of a group every state below 2^16 reads
 * the next word (all plane-0 lanes in lane order, then all plane-1 lanes).
 * Slot entry e of a 256-slot table: bias = e & 255, sym = (e >> 8) & 255,
 * freq = e >> 16; decode x -> freq * (x >> 8) + bias.
 * U16 blocks code y = rotr16(zigzag(d), 1); d = y ^ (y & 0x8000 ? 0x7FFF : 0).
 *
 * Word-dictionary blocks (kinds 3 and 4) decode one symbol per word with one
 * shared table whose entry e gives word = e & 0xFFFF, bias = (e >> 16) & 255,
 * freq = e >> 24. Lane l's state 0 decodes its words 0, 2, 4, 6 and state 1
 * its words 1, 3, 5, 7 of each group; a check follows every second word of
 * each state (after lane words 3 and 7), with the same read order.
 *
 * Dictionary blocks with flag 2 (escapes) carry, at byte (2 * nwords + 15) & ~15
 * of the payload, uint16 count[32] and then count[0] + ... + count[31] uint32
 * entries grouped by lane: word index (bits 0-15) | residual word (16-31). The
 * listed words' residuals are the listed values (their stream symbol decodes
 * as 0); an entry outside the block or not owned by its lane is an error.
 *
 * Dictionary blocks whose flag bits 2-3 hold c != 0 split every word: its low
 * k = 1, 2, 4 (c = 1, 2, 3) bits are not in the stream but in a raw section at
 * byte (2 * nwords + 15) & ~15 (escape lists, if any, move behind it). With
 * G = 4 / k groups per uint32, group g's bits for lane l are in uint32
 * (g / G) * 32 + l, starting at bit (g % G) * 8k; the lane's word j sits at
 * bit j * k from there. The section has
 * ceil(ceil(W / 256) / G) * 128 bytes. The residual word is the decoded (or
 * listed) word ORed with its raw bits.
 */
#include <pthread.h>
#include <stdint.h>
#include <string.h>

#define O_L 65536u
#define O_BLOCK_WORDS 65536u /* 16-bit words of the largest block (128 KiB) */

typedef struct {
  uint64_t dst;
  uint64_t src;
  uint32_t nbytes;
  uint32_t clen;
  uint32_t nwords;
  uint16_t kind;
  uint8_t tail;
  uint8_t flags;
} o_block;

typedef struct {
  uint32_t first_block, nblocks, table, split;
} o_tile;

enum { O_RAW = 0, O_ANS_XOR = 1, O_ANS_U16 = 2, O_DICT_XOR = 3, O_DICT_U16 = 4 };
enum { O_ERR_STATE = 1, O_ERR_LENGTH = 2, O_ERR_KIND = 8, O_ERR_BOUNDS = 16 };

static inline uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static inline uint32_t rd32(const uint8_t* p) {
  return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

/* Decode the nbytes/2 coded words of an ANS block. Returns 0 or O_ERR_*. */
int wso_decode_words(const uint8_t* payload, uint32_t clen, uint32_t nwords, uint32_t nbytes,
                     const uint32_t* table512, uint16_t* words) {
  const uint32_t W = nbytes / 2;
  if (clen < 256 || 2ull * nwords > clen) return O_ERR_BOUNDS;
  uint32_t x[2][32];
  for (int p = 0; p < 2; ++p)
    for (int l = 0; l < 32; ++l) x[p][l] = rd32(payload + 4 * (32 * p + l));
  uint32_t pos = 128;
  const uint32_t groups = (W + 255) / 256;
  for (uint32_t g = 0; g < groups; ++g) {
    for (uint32_t c = 0; c < 4; ++c) {
      for (uint32_t l = 0; l < 32; ++l) {
        for (uint32_t j = 2 * c; j < 2 * c + 2; ++j) {
          const uint32_t i = 256 * g + 8 * l + j;
          if (i >= W) continue;
          uint16_t word = 0;
          for (int p = 0; p < 2; ++p) {
            const uint32_t e = table512[256 * p + (x[p][l] & 255u)];
            const uint32_t freq = e >> 16, sym = (e >> 8) & 255u, bias = e & 255u;
            x[p][l] = freq * (x[p][l] >> 8) + bias;
            word |= (uint16_t)(sym << (8 * p));
          }
          words[i] = word;
        }
      }
      for (int p = 0; p < 2; ++p)
        for (uint32_t l = 0; l < 32; ++l)
          if (x[p][l] < O_L) {
            const uint32_t w = (pos < nwords) ? rd16(payload + 2 * pos) : 0;
            x[p][l] = (x[p][l] << 16) | w;
            ++pos;
          }
    }
  }
  int err = 0;
  for (int p = 0; p < 2; ++p)
    for (int l = 0; l < 32; ++l)
      if (x[p][l] != O_L) err |= O_ERR_STATE;
  if (pos != nwords) err |= O_ERR_LENGTH;
  return err;
}

/* Word-dictionary variant of wso_decode_words. */
int wso_decode_dict_words(const uint8_t* payload, uint32_t clen, uint32_t nwords, uint32_t nbytes,
                          const uint32_t* table256, uint16_t* words) {
  const uint32_t W = nbytes / 2;
  if (clen < 256 || 2ull * nwords > clen) return O_ERR_BOUNDS;
  uint32_t x[2][32];
  for (int p = 0; p < 2; ++p)
    for (int l = 0; l < 32; ++l) x[p][l] = rd32(payload + 4 * (32 * p + l));
  uint32_t pos = 128;
  const uint32_t groups = (W + 255) / 256;
  for (uint32_t g = 0; g < groups; ++g) {
    for (uint32_t c = 0; c < 2; ++c) {
      for (uint32_t l = 0; l < 32; ++l) {
        for (uint32_t k = 0; k < 2; ++k) {
          for (int p = 0; p < 2; ++p) {
            const uint32_t i = 256 * g + 8 * l + 4 * c + 2 * k + (uint32_t)p;
            if (i >= W) continue;
            const uint32_t e = table256[x[p][l] & 255u];
            const uint32_t freq = e >> 24, bias = (e >> 16) & 255u;
            x[p][l] = freq * (x[p][l] >> 8) + bias;
            words[i] = (uint16_t)(e & 0xFFFFu);
          }
        }
      }
      for (int p = 0; p < 2; ++p)
        for (uint32_t l = 0; l < 32; ++l)
          if (x[p][l] < O_L) {
            const uint32_t w = (pos < nwords) ? rd16(payload + 2 * pos) : 0;
            x[p][l] = (x[p][l] << 16) | w;
            ++pos;
          }
    }
  }
  int err = 0;
  for (int p = 0; p < 2; ++p)
    for (int l = 0; l < 32; ++l)
      if (x[p][l] != O_L) err |= O_ERR_STATE;
  if (pos != nwords) err |= O_ERR_LENGTH;
  return err;
}

static inline uint16_t o_unrotate(uint16_t y) { return (uint16_t)(y ^ ((y & 0x8000u) ? 0x7FFFu : 0u)); }

/* Apply one block to dst (host memory). Returns 0 or O_ERR_*. */
int wso_apply_block(const o_block* b, const uint8_t* payload, const uint32_t* table512, uint8_t* dst, int reverse,
                    uint16_t* scratch_words /* >= 2 * O_BLOCK_WORDS: decoded words, then raw low bits */) {
  uint16_t* raw_low = scratch_words + O_BLOCK_WORDS;
  const uint32_t n = b->nbytes;
  if (b->kind == O_RAW) {
    if (b->clen < n) return O_ERR_BOUNDS;
    for (uint32_t i = 0; i < n; ++i) dst[i] ^= payload[i];
    return 0;
  }
  int err;
  if (b->kind == O_ANS_XOR || b->kind == O_ANS_U16)
    err = wso_decode_words(payload, b->clen, b->nwords, n, table512, scratch_words);
  else if (b->kind == O_DICT_XOR || b->kind == O_DICT_U16)
    err = wso_decode_dict_words(payload, b->clen, b->nwords, n, table512, scratch_words);
  else
    return O_ERR_KIND;
  const int xor_apply = b->kind == O_ANS_XOR || b->kind == O_DICT_XOR;
  const int dict = b->kind == O_DICT_XOR || b->kind == O_DICT_U16;
  const uint32_t W = n / 2;
  uint32_t side = (2u * b->nwords + 15u) & ~15u;
  const uint32_t split_code = (b->flags >> 2) & 3u;
  if (split_code && !dict) return err | O_ERR_KIND;
  if (split_code) {
    const uint32_t k = split_code == 3u ? 4u : split_code, per = 4u / k;
    const uint32_t groups = (W + 255u) / 256u;
    const uint64_t raw_bytes = 128ull * ((groups + per - 1u) / per);
    if ((uint64_t)side + raw_bytes > b->clen) return err | O_ERR_LENGTH;
    for (uint32_t i = 0; i < W; ++i) {
      const uint32_t g = i / 256u, l = (i % 256u) / 8u, j = i % 8u;
      const uint32_t rw = rd32(payload + side + 4u * ((g / per) * 32u + l));
      const uint32_t bit = (g % per) * 8u * k + j * k;
      raw_low[i] = (uint16_t)((rw >> bit) & ((1u << k) - 1u));
    }
    side += (uint32_t)raw_bytes;
  }
  if (dict && (b->flags & 2u)) {
    if ((uint64_t)side + 64 > b->clen) return err | O_ERR_LENGTH;
    uint32_t at = side + 64;
    for (uint32_t l = 0; l < 32; ++l) {
      const uint32_t count = rd16(payload + side + 2 * l);
      if ((uint64_t)at + 4ull * count > b->clen) return err | O_ERR_LENGTH;
      for (uint32_t k = 0; k < count; ++k, at += 4) {
        const uint32_t e = rd32(payload + at), i = e & 0xFFFFu;
        if (i >= W || (i % 256) / 8 != l) {
          err |= O_ERR_LENGTH;
          continue;
        }
        scratch_words[i] = (uint16_t)(e >> 16);
      }
    }
  }
  if (split_code)
    for (uint32_t i = 0; i < W; ++i) scratch_words[i] |= raw_low[i];
  for (uint32_t i = 0; i < W; ++i) {
    uint16_t old = rd16(dst + 2 * i), nw;
    if (xor_apply) {
      nw = (uint16_t)(old ^ scratch_words[i]);
    } else {
      const uint16_t d = o_unrotate(scratch_words[i]);
      nw = reverse ? (uint16_t)(old - d) : (uint16_t)(old + d);
    }
    dst[2 * i] = (uint8_t)(nw & 0xFF);
    dst[2 * i + 1] = (uint8_t)(nw >> 8);
  }
  if (b->flags & 1u) dst[n - 1] ^= b->tail;
  return err;
}

static uint64_t o_mix(uint64_t x) {
  x ^= x >> 30;
  x *= 0xBF58476D1CE4E5B9ull;
  x ^= x >> 27;
  x *= 0x94D049BB133111EBull;
  x ^= x >> 31;
  return x;
}

/* Hash of a block's bytes after the write, keyed by its index in the plan. */
uint64_t wso_block_hash(const uint8_t* bytes, uint32_t n, uint64_t block_index) {
  const uint32_t groups = (n + 511) / 512;
  uint64_t sum = 0;
  for (uint32_t l = 0; l < 32; ++l) {
    uint32_t a = 0, b = 0;
    for (uint32_t g = 0; g < groups; ++g) {
      uint8_t chunk[16];
      memset(chunk, 0, 16);
      const uint32_t off = 512 * g + 16 * l;
      for (uint32_t k = 0; k < 16; ++k)
        if (off + k < n) chunk[k] = bytes[off + k];
      for (int w = 0; w < 4; ++w) a += rd32(chunk + 4 * w);
      b += a;
    }
    sum += o_mix((((uint64_t)b << 32) | a) + (uint64_t)(l + 1) * 0x9E3779B97F4A7C15ull);
  }
  return o_mix(sum ^ ((block_index + 1) * 0xD1B54A32D192ED03ull));
}

/* Whole-plan apply on the host, blocks split over `threads` POSIX threads.
 * dst_delta is added to every block's dst address (0 when the plan was built
 * on host targets). Returns OR of block errors; *checksum receives the plan
 * checksum of the written bytes. */
typedef struct {
  const o_block* blocks;
  uint64_t nblocks;
  const o_tile* tiles;
  uint64_t ntiles;
  const uint32_t* tables;
  const uint8_t* arena;
  int64_t dst_delta;
  int reverse;
  int nthreads;
  int tid;
  int err;
  uint64_t checksum;
} o_job;

static void* o_worker(void* arg) {
  o_job* j = (o_job*)arg;
  static __thread uint16_t words[2 * O_BLOCK_WORDS];
  for (uint64_t t = (uint64_t)j->tid; t < j->ntiles; t += (uint64_t)j->nthreads) {
    const o_tile* tile = &j->tiles[t];
    const uint32_t* table = tile->table == 0xFFFFFFFFu ? 0 : j->tables + 512ull * tile->table;
    for (uint32_t k = 0; k < tile->nblocks; ++k) {
      const uint64_t bi = tile->first_block + k;
      const o_block* b = &j->blocks[bi];
      uint8_t* dst = (uint8_t*)(uintptr_t)(b->dst + (uint64_t)j->dst_delta);
      if (b->kind != O_RAW && !table) {
        j->err |= O_ERR_KIND;
        continue;
      }
      j->err |= wso_apply_block(b, j->arena + b->src, table, dst, j->reverse, words);
      j->checksum += wso_block_hash(dst, b->nbytes, bi);
    }
  }
  return 0;
}

int wso_apply_plan(const o_block* blocks, uint64_t nblocks, const o_tile* tiles, uint64_t ntiles,
                   const uint32_t* tables, const uint8_t* arena, int64_t dst_delta, int reverse, int threads,
                   uint64_t* checksum) {
  if (threads < 1) threads = 1;
  if (threads > 256) threads = 256;
  o_job jobs[256];
  pthread_t th[256];
  for (int t = 0; t < threads; ++t) {
    o_job j = {blocks, nblocks, tiles, ntiles, tables, arena, dst_delta, reverse, threads, t, 0, 0};
    jobs[t] = j;
  }
  for (int t = 1; t < threads; ++t) pthread_create(&th[t], 0, o_worker, &jobs[t]);
  o_worker(&jobs[0]);
  for (int t = 1; t < threads; ++t) pthread_join(th[t], 0);
  int err = 0;
  uint64_t sum = 0;
  for (int t = 0; t < threads; ++t) {
    err |= jobs[t].err;
    sum += jobs[t].checksum;
  }
  if (checksum) *checksum = sum;
  return err;
}
