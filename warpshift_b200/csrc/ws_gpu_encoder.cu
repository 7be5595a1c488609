// GPU encoder for prepare (replaces the host D2H + encode of delta.py:196-216,
// 164-174 when the target weights are resident on the device).
//
// Per batch of packets:
//   1. the base (A) bytes are copied host -> device;
//   2. stats_kernel: per 128 KiB block, zero detection, byte-plane histograms and
//      distinct-word tables of both residual transforms, checksum lane sums of
//      A and B, odd tail byte;
//   3. the host builds each packet's tables with the same code as the host
//      encoder (choose_coding), so the output is byte-identical;
//   4. encode_kernel: one warp per block and candidate coding, the exact mirror
//      of the decoder (checks in reverse, ballot/popc word placement, division
//      by reciprocal multiplication with one correction);
//   5. the host applies the reference's mode rule and the raw fallback;
//      compact_kernel packs the chosen payloads, which are copied back.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/syscall.h>
#include <unistd.h>

#include <stdio.h>
#include <stdlib.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "ws_encoder.h"
#include "ws_format.h"
#include "ws_gpu_encoder.h"

namespace ws {

namespace {

constexpr uint32_t kStatsThreads = 256;
constexpr uint32_t kLocalSlots = 512;     // per-CTA distinct-word table
constexpr uint32_t kPacketSlots = 1024;   // per-packet distinct-word table
constexpr uint32_t kEncWarps = 8;         // blocks per encode CTA
constexpr uint32_t kOutHalfwords = WS_HEADER_HALFWORDS + WS_BLOCK_BYTES / 2;  // header + worst-case stream
constexpr uint32_t kMaxDistinct = 255;

struct PacketStats {  // device, one per packet of the batch
  uint32_t plane[2][2][256];  // [transform xor/u16][plane][symbol]
  // Distinct words ([0]) and distinct high 12 bits (word & 0xFFF0, [1]) per transform.
  uint32_t key[2][2][kPacketSlots];  // [table][transform]: value + 1, 0 = empty
  uint32_t cnt[2][2][kPacketSlots];
  uint32_t distinct[2][2];
  uint32_t many[2][2];
};

struct BlockStats {  // device, one per block of the batch
  uint32_t nonzero;
  uint32_t tail;
  unsigned long long lane_sum[2];  // [0] target (B) bytes, [1] base (A) bytes
};

struct BlockJob {  // one block (WS_BLOCK_BYTES) of the batch
  const uint8_t* base;    // device copy of A
  const uint8_t* target;  // resident B
  uint32_t nbytes;
  uint32_t packet;        // packet index within the batch
};

struct EncodeJob {  // one block coded with one candidate
  uint32_t block;     // index into the batch's BlockJob array
  uint32_t table;     // index into the batch's encode tables
  uint32_t dict;      // 1: word dictionary, 0: byte planes
  uint32_t u16;       // 1: U16 residual words, 0: XOR words
  uint32_t esc;       // the dictionary's escape symbol, or ~0u without escapes
  uint32_t split;     // raw low bits per word of a split-word dictionary (0, 1, 2, 4)
};

struct EncTable {  // per candidate coding: per state, per symbol
  uint32_t fc[2][256];   // freq | cdf << 16
  uint32_t rcp[2][256];  // floor(2^32 / freq) (0xFFFFFFFF for freq 1)
};

struct CompactJob {
  uint32_t block;      // BlockJob index
  uint32_t encode;     // EncodeJob index (source of an ANS payload), or ~0u for raw
  uint32_t nwords;     // ANS halfwords incl. header
  uint32_t escapes;    // escape entries listed after the stream (0: no list)
  uint64_t dst;        // byte offset in the output buffer
  uint32_t split;      // raw low bits per word (0: no raw section)
  uint32_t u16;        // the raw bits are of U16 residual words
};

__device__ __forceinline__ uint16_t u16_word(uint16_t b, uint16_t t) {
  const int32_t d = (int32_t)(int16_t)(uint16_t)(t - b);
  const uint32_t z = ((uint32_t)(d * 2) ^ (uint32_t)(d >> 15)) & 0xFFFFu;
  return (uint16_t)((z >> 1) | ((z & 1u) << 15));
}

// The lane's 8 residual words starting at word w0 of the block (0 past W).
__device__ __forceinline__ void load_words(const BlockJob& blk, uint32_t w0, uint32_t W, bool aligned, bool u16,
                                           uint16_t v[8]) {
  if (w0 + 8 <= W && aligned) {
    uint4 av = *reinterpret_cast<const uint4*>(blk.base + 2 * w0);
    uint4 tv = *reinterpret_cast<const uint4*>(blk.target + 2 * w0);
    const uint16_t* a16 = reinterpret_cast<const uint16_t*>(&av);
    const uint16_t* t16 = reinterpret_cast<const uint16_t*>(&tv);
#pragma unroll
    for (uint32_t q = 0; q < 8; ++q) v[q] = u16 ? u16_word(a16[q], t16[q]) : (uint16_t)(a16[q] ^ t16[q]);
  } else {
#pragma unroll
    for (uint32_t q = 0; q < 8; ++q) {
      v[q] = 0;
      if (w0 + q < W) {
        const uint16_t a16 = (uint16_t)(blk.base[2 * (w0 + q)] | (blk.base[2 * (w0 + q) + 1] << 8));
        const uint16_t t16 = (uint16_t)(blk.target[2 * (w0 + q)] | (blk.target[2 * (w0 + q) + 1] << 8));
        v[q] = u16 ? u16_word(a16, t16) : (uint16_t)(a16 ^ t16);
      }
    }
  }
}

__device__ __forceinline__ uint32_t word_hash(uint32_t w, uint32_t bits) { return (w * 0x9E3779B1u) >> (32 - bits); }

// Insert one occurrence of word w into an open-addressing table; returns false
// when the table cannot take another distinct word.
__device__ bool table_add(uint32_t* key, uint32_t* cnt, uint32_t* distinct, uint32_t slots_log2, uint32_t w,
                          uint32_t amount) {
  const uint32_t slots = 1u << slots_log2;
  const uint32_t k = w + 1;
  uint32_t h = word_hash(w, slots_log2);
  for (uint32_t probe = 0; probe < slots; ++probe, h = (h + 1) & (slots - 1)) {
    uint32_t cur = key[h];
    if (cur == 0) {
      cur = atomicCAS(&key[h], 0u, k);
      if (cur == 0) {
        if (atomicAdd(distinct, 1u) >= kMaxDistinct) return false;
        atomicAdd(&cnt[h], amount);
        return true;
      }
    }
    if (cur == k) {
      atomicAdd(&cnt[h], amount);
      return true;
    }
  }
  return false;
}

__global__ void __launch_bounds__(kStatsThreads) stats_kernel(const BlockJob* __restrict__ jobs, PacketStats* pstats,
                                                              BlockStats* bstats) {
  __shared__ uint32_t hist[2][2][256];
  // [table][transform]: table 0 counts words, table 1 their high 12 bits.
  __shared__ uint32_t key[2][2][kLocalSlots], cnt[2][2][kLocalSlots];
  __shared__ uint32_t distinct[2][2], overflow[2][2];
  __shared__ uint32_t ck[4][kStatsThreads];  // aB, bB, aA, bA per thread
  const uint32_t t = threadIdx.x;
  for (uint32_t i = t; i < 2 * 2 * 256; i += kStatsThreads) (&hist[0][0][0])[i] = 0;
  for (uint32_t i = t; i < 2 * 2 * kLocalSlots; i += kStatsThreads) {
    (&key[0][0][0])[i] = 0;
    (&cnt[0][0][0])[i] = 0;
  }
  if (t < 4) {
    (&distinct[0][0])[t] = 0;
    (&overflow[0][0])[t] = 0;
  }
  __syncthreads();
  const BlockJob job = jobs[blockIdx.x];
  const uint32_t n = job.nbytes;
  const uint32_t W = n / 2;
  const uint32_t groups = (n + WS_GROUP_BYTES - 1) / WS_GROUP_BYTES;
  const uint32_t chunks = (n + 15) / 16;
  uint32_t nz = 0;
  uint32_t aB = 0, bB = 0, aA = 0, bA = 0;
  const bool aligned = (((uintptr_t)job.base | (uintptr_t)job.target) & 15u) == 0;
  for (uint32_t k = t; k < chunks; k += kStatsThreads) {
    const uint32_t g = k >> 5;  // 32 chunks of 16 bytes per 512-byte group; lane = k & 31 = t & 31
    uint8_t ab[16], tb[16];
    if (aligned && 16 * k + 16 <= n) {
      *reinterpret_cast<uint4*>(ab) = *reinterpret_cast<const uint4*>(job.base + 16 * k);
      *reinterpret_cast<uint4*>(tb) = *reinterpret_cast<const uint4*>(job.target + 16 * k);
    } else {
#pragma unroll
      for (uint32_t i = 0; i < 16; ++i) {
        ab[i] = 16 * k + i < n ? job.base[16 * k + i] : 0;
        tb[i] = 16 * k + i < n ? job.target[16 * k + i] : 0;
      }
    }
    const uint32_t* aw = reinterpret_cast<const uint32_t*>(ab);
    const uint32_t* tw = reinterpret_cast<const uint32_t*>(tb);
    const uint32_t sA = aw[0] + aw[1] + aw[2] + aw[3];
    const uint32_t sB = tw[0] + tw[1] + tw[2] + tw[3];
    aA += sA;
    bA += (groups - g) * sA;
    aB += sB;
    bB += (groups - g) * sB;
    nz |= (aw[0] ^ tw[0]) | (aw[1] ^ tw[1]) | (aw[2] ^ tw[2]) | (aw[3] ^ tw[3]);
#pragma unroll
    for (uint32_t j = 0; j < 8; ++j) {
      if (8 * k + j >= W) break;
      const uint16_t a16 = (uint16_t)(ab[2 * j] | (ab[2 * j + 1] << 8));
      const uint16_t t16 = (uint16_t)(tb[2 * j] | (tb[2 * j + 1] << 8));
      const uint16_t v[2] = {(uint16_t)(a16 ^ t16), u16_word(a16, t16)};
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        atomicAdd(&hist[c][0][v[c] & 0xFF], 1u);
        atomicAdd(&hist[c][1][v[c] >> 8], 1u);
        if (!overflow[0][c] && !table_add(key[0][c], cnt[0][c], &distinct[0][c], 9, v[c], 1)) overflow[0][c] = 1;
        if (!overflow[1][c] && !table_add(key[1][c], cnt[1][c], &distinct[1][c], 9, v[c] & 0xFFF0u, 1))
          overflow[1][c] = 1;
      }
    }
  }
  const bool any = __syncthreads_or(nz != 0);
  ck[0][t] = aB;
  ck[1][t] = bB;
  ck[2][t] = aA;
  ck[3][t] = bA;
  __syncthreads();
  BlockStats* out = bstats + blockIdx.x;
  if (t < 32) {
    uint32_t s[4] = {0, 0, 0, 0};
    for (uint32_t i = t; i < kStatsThreads; i += 32)
      for (int q = 0; q < 4; ++q) s[q] += ck[q][i];
    unsigned long long hB = ws_lane_hash(s[0], s[1], t), hA = ws_lane_hash(s[2], s[3], t);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      hB += __shfl_xor_sync(0xFFFFFFFFu, hB, o);
      hA += __shfl_xor_sync(0xFFFFFFFFu, hA, o);
    }
    if (t == 0) {
      uint32_t tail = 0;
      if (n & 1u) tail = (uint32_t)(job.base[n - 1] ^ job.target[n - 1]);
      out->lane_sum[0] = hB;
      out->lane_sum[1] = hA;
      out->tail = tail;
      out->nonzero = (any || tail) ? 1u : 0u;
    }
  }
  // The odd tail byte alone can make a block non-zero.
  const bool nonzero = any || ((n & 1u) && (job.base[n - 1] != job.target[n - 1]));
  if (!nonzero) return;
  PacketStats* ps = pstats + job.packet;
  for (uint32_t i = t; i < 2 * 2 * 256; i += kStatsThreads) {
    const uint32_t v = (&hist[0][0][0])[i];
    if (v) atomicAdd(&(&ps->plane[0][0][0])[i], v);
  }
  for (uint32_t h = 0; h < 2; ++h)
    for (uint32_t c = 0; c < 2; ++c) {
      if (overflow[h][c]) {
        if (t == 0) atomicExch(&ps->many[h][c], 1u);
        continue;
      }
      for (uint32_t i = t; i < kLocalSlots; i += kStatsThreads) {
        const uint32_t k = key[h][c][i];
        if (k && !ps->many[h][c] &&
            !table_add(ps->key[h][c], ps->cnt[h][c], &ps->distinct[h][c], 10, k - 1, cnt[h][c][i]))
          atomicExch(&ps->many[h][c], 1u);
      }
    }
}

// Dictionary index table of a packet: word -> symbol.
__global__ void dict_index_kernel(const uint16_t* __restrict__ words, uint32_t nwords, uint8_t* index) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < nwords) index[words[i]] = (uint8_t)i;
}

__device__ __forceinline__ uint32_t lanemask_lt() {
  uint32_t m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

// x -> E(x, s) = (x / f) * 256 + x % f + cdf, with x / f from the reciprocal.
__device__ __forceinline__ uint32_t rans_put(uint32_t x, uint32_t fc, uint32_t rcp) {
  const uint32_t f = fc & 0xFFFFu, cdf = fc >> 16;
  uint32_t q = __umulhi(x, rcp);
  uint32_t r = x - q * f;
  if (r >= f) {
    ++q;
    r -= f;
  }
  return (q << WS_PROB_BITS) + r + cdf;
}

__global__ void __launch_bounds__(kEncWarps * 32) encode_kernel(const BlockJob* __restrict__ blocks,
                                                                const EncodeJob* __restrict__ jobs, uint32_t njobs,
                                                                const EncTable* __restrict__ tables,
                                                                const uint8_t* const* __restrict__ dict_index,
                                                                uint16_t* out, uint32_t* nwords_out,
                                                                uint32_t* side_out, uint32_t* side_count) {
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  const uint32_t j = blockIdx.x * kEncWarps + warp;
  if (j >= njobs) return;
  const EncodeJob job = jobs[j];
  const BlockJob blk = blocks[job.block];
  const EncTable& tab = tables[job.table];
  const uint8_t* idx = job.dict ? dict_index[job.table] : nullptr;
  uint16_t* o = out + (uint64_t)j * kOutHalfwords;
  const uint32_t W = blk.nbytes / 2;
  const uint32_t groups = (W + WS_GROUP_WORDS - 1) / WS_GROUP_WORDS;
  const uint32_t cpg = job.dict ? 2u : 4u;
  const uint32_t ltm = lanemask_lt();
  const bool aligned = (((uintptr_t)blk.base | (uintptr_t)blk.target) & 15u) == 0;
  uint32_t x[2] = {WS_RANS_L, WS_RANS_L};
  uint32_t cursor = kOutHalfwords;
  const uint16_t keep = (uint16_t)~((1u << job.split) - 1u);  // the coded part of a split word
  if (job.esc != ~0u) {
    // Escape list of this lane: its words coded as the escape symbol, in
    // increasing word order (at most WS_ESCAPE_LANE_MAX stored; the count is exact).
    uint32_t* mine = side_out + ((uint64_t)j * WS_LANES + lane) * WS_ESCAPE_LANE_MAX;
    uint32_t count = 0;
    for (uint32_t g = 0; g < groups; ++g) {
      const uint32_t w0 = g * WS_GROUP_WORDS + lane * WS_WORDS_PER_LANE;
      uint16_t v[8];
      load_words(blk, w0, W, aligned, job.u16 != 0, v);
      for (uint32_t q = 0; q < 8; ++q) {
        const uint16_t h = (uint16_t)(v[q] & keep);
        if (w0 + q < W && idx[h] == job.esc) {
          if (count < WS_ESCAPE_LANE_MAX) mine[count] = (w0 + q) | ((uint32_t)h << 16);
          ++count;
        }
      }
    }
    side_count[(uint64_t)j * WS_LANES + lane] = count;
  }
  for (uint32_t g = groups; g-- > 0;) {
    // The lane's 8 residual words of this group and their symbols per state.
    const uint32_t w0 = g * WS_GROUP_WORDS + lane * WS_WORDS_PER_LANE;
    uint16_t v[8];
    load_words(blk, w0, W, aligned, job.u16 != 0, v);
    for (uint32_t c = cpg; c-- > 0;) {
      uint32_t sa[2], sb[2];
      bool pa[2], pb[2];
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        uint32_t ja, jb;
        if (job.dict) {
          ja = 4 * c + p;
          jb = 4 * c + 2 + p;
        } else {
          ja = 2 * c;
          jb = 2 * c + 1;
        }
        pa[p] = w0 + ja < W;
        pb[p] = w0 + jb < W;
        if (job.dict) {
          sa[p] = pa[p] ? idx[v[ja] & keep] : 0;
          sb[p] = pb[p] ? idx[v[jb] & keep] : 0;
        } else {
          sa[p] = p ? (v[ja] >> 8) : (v[ja] & 0xFFu);
          sb[p] = p ? (v[jb] >> 8) : (v[jb] & 0xFFu);
        }
      }
      // Emission (decoder reads after decoding a then b): valid pre-images of
      // the pair are [fa*fb, 2^16*fa*fb), of a single symbol [2^8 f, 2^24 f).
      bool emit[2];
      uint32_t word[2];
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        emit[p] = false;
        word[p] = 0;
        if (pa[p]) {
          const uint32_t fa = tab.fc[p][sa[p]] & 0xFFFFu;
          uint64_t xmax;
          if (pb[p])
            xmax = ((uint64_t)fa * (tab.fc[p][sb[p]] & 0xFFFFu)) << 16;
          else
            xmax = (uint64_t)fa << 24;
          if ((uint64_t)x[p] >= xmax) {
            emit[p] = true;
            word[p] = x[p] & 0xFFFFu;
            x[p] >>= 16;
          }
        }
      }
      const uint32_t e0 = __ballot_sync(0xFFFFFFFFu, emit[0]);
      const uint32_t e1 = __ballot_sync(0xFFFFFFFFu, emit[1]);
      const uint32_t n0 = __popc(e0);
      const uint32_t start = cursor - n0 - __popc(e1);
      if (emit[0]) o[start + __popc(e0 & ltm)] = (uint16_t)word[0];
      if (emit[1]) o[start + n0 + __popc(e1 & ltm)] = (uint16_t)word[1];
      cursor = start;
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        if (pb[p]) x[p] = rans_put(x[p], tab.fc[p][sb[p]], tab.rcp[p][sb[p]]);
        if (pa[p]) x[p] = rans_put(x[p], tab.fc[p][sa[p]], tab.rcp[p][sa[p]]);
      }
    }
  }
  uint32_t* hdr = reinterpret_cast<uint32_t*>(o);
  hdr[lane] = x[0];
  hdr[32 + lane] = x[1];
  if (lane == 0) nwords_out[j] = WS_HEADER_HALFWORDS + (kOutHalfwords - cursor);
}

// Packs one block's payload (ANS header + stream, or raw XOR bytes) at dst,
// zero-padded to 16 bytes.
__global__ void compact_kernel(const CompactJob* __restrict__ jobs, const BlockJob* __restrict__ blocks,
                               const uint16_t* __restrict__ enc_out, const uint32_t* __restrict__ side_out,
                               const uint32_t* __restrict__ side_count, uint8_t* out) {
  const CompactJob job = jobs[blockIdx.x];
  const BlockJob blk = blocks[job.block];
  uint8_t* d = out + job.dst;
  if (job.encode == ~0u) {
    const uint32_t n = blk.nbytes, padded = (n + 15) & ~15u;
    for (uint32_t i = threadIdx.x; i < padded; i += blockDim.x) d[i] = i < n ? (uint8_t)(blk.base[i] ^ blk.target[i]) : 0;
    return;
  }
  const uint16_t* src = enc_out + (uint64_t)job.encode * kOutHalfwords;
  const uint32_t stream = job.nwords - WS_HEADER_HALFWORDS;
  const uint32_t first = kOutHalfwords - stream;
  uint16_t* d16 = reinterpret_cast<uint16_t*>(d);
  const uint32_t padded_hw = ((2 * job.nwords + 15) & ~15u) / 2;
  for (uint32_t i = threadIdx.x; i < padded_hw; i += blockDim.x) {
    uint16_t v = 0;
    if (i < WS_HEADER_HALFWORDS)
      v = src[i];
    else if (i < job.nwords)
      v = src[first + (i - WS_HEADER_HALFWORDS)];
    d16[i] = v;
  }
  uint32_t side_off = 2 * padded_hw;
  if (job.split) {
    // Raw section (WS_FLAG_SPLIT_MASK layout): one thread per raw word.
    const uint32_t k = job.split, per = 4u / k, mask = (1u << k) - 1u;
    const uint32_t W = blk.nbytes / 2, raw_bytes = ws_split_raw_bytes(W, k);
    const bool aligned = (((uintptr_t)blk.base | (uintptr_t)blk.target) & 15u) == 0;
    uint32_t* raw = reinterpret_cast<uint32_t*>(d + side_off);
    for (uint32_t r = threadIdx.x; r < raw_bytes / 4; r += blockDim.x) {
      const uint32_t lane = r % WS_LANES, q = r / WS_LANES;
      uint32_t acc = 0;
      for (uint32_t gg = 0; gg < per; ++gg) {
        const uint32_t g = q * per + gg;
        uint16_t v[8];
        load_words(blk, g * WS_GROUP_WORDS + lane * WS_WORDS_PER_LANE, W, aligned, job.u16 != 0, v);
#pragma unroll
        for (uint32_t j = 0; j < 8; ++j)
          acc |= ((uint32_t)v[j] & mask) << (gg * 8u * k + j * k);
      }
      raw[r] = acc;
    }
    side_off += raw_bytes;
  }
  if (job.escapes == 0) return;
  // Escape list (WS_FLAG_ESCAPES layout): lane counts, entries by lane, zero padding.
  __shared__ uint32_t start[WS_LANES + 1];
  const uint32_t* cnt = side_count + (uint64_t)job.encode * WS_LANES;
  if (threadIdx.x == 0) {
    start[0] = 0;
    for (uint32_t l = 0; l < WS_LANES; ++l) start[l + 1] = start[l] + cnt[l];
  }
  __syncthreads();
  uint8_t* side = d + side_off;
  uint16_t* head = reinterpret_cast<uint16_t*>(side);
  if (threadIdx.x < WS_LANES) head[threadIdx.x] = (uint16_t)cnt[threadIdx.x];
  uint32_t* ent = reinterpret_cast<uint32_t*>(side + WS_ESCAPE_HEADER_BYTES);
  const uint32_t* lanes = side_out + (uint64_t)job.encode * WS_LANES * WS_ESCAPE_LANE_MAX;
  for (uint32_t e = threadIdx.x; e < job.escapes; e += blockDim.x) {
    uint32_t l = 0;
    while (start[l + 1] <= e) ++l;
    ent[e] = lanes[l * WS_ESCAPE_LANE_MAX + (e - start[l])];
  }
  const uint32_t used = WS_ESCAPE_HEADER_BYTES + 4 * job.escapes, padded = (used + 15) & ~15u;
  for (uint32_t i = used + threadIdx.x; i < padded; i += blockDim.x) side[i] = 0;
}

template <class T>
struct DeviceBuffer {
  T* ptr = nullptr;
  size_t count = 0;
  cudaError_t ensure(size_t n) {
    if (n <= count) return cudaSuccess;
    if (ptr) cudaFree(ptr);
    ptr = nullptr;
    count = 0;
    cudaError_t e = cudaMalloc((void**)&ptr, std::max<size_t>(n, 1) * sizeof(T));
    if (e == cudaSuccess) count = n;
    return e;
  }
  ~DeviceBuffer() {
    if (ptr) cudaFree(ptr);
  }
};

uint32_t reciprocal(uint32_t f) { return f <= 1 ? 0xFFFFFFFFu : (uint32_t)((1ull << 32) / f); }

void fill_enc_table(const CodingTables& ct, EncTable* t) {
  for (int p = 0; p < 2; ++p)
    for (int s = 0; s < 256; ++s) {
      t->fc[p][s] = ct.freq[p][s] | (ct.cdf[p][s] << 16);
      t->rcp[p][s] = reciprocal(ct.freq[p][s]);
    }
}

double seconds_since(std::chrono::steady_clock::time_point t) {
  return std::chrono::duration<double>(std::chrono::steady_clock::now() - t).count();
}

// Host -> device copies of A for one batch, issued on the uploader's own
// streams. Pinned (page-locked or registered) sources are copied by the DMA
// engine directly; pageable ones are staged by host threads, each copying into
// one of its two pinned slots while the DMA of the other slot runs. copy()
// starts after `after` (the event that releases the destination buffer);
// order_before() makes `stream` wait for the copies.
class Uploader {
 public:
  struct Piece {
    uint8_t* dst;
    const uint8_t* src;
    uint64_t bytes;
  };
  static constexpr uint64_t kSlotBytes = 16ull << 20;

  Uploader(int device, int threads) : device_(device), nworkers_(std::max(1, std::min(threads, 8))) {}
  ~Uploader() {
    cudaSetDevice(device_);
    for (Worker& w : workers_) {
      if (w.stream) cudaStreamSynchronize(w.stream);
      for (int k = 0; k < 2; ++k) {
        if (w.slot[k]) cudaFreeHost(w.slot[k]);
        if (w.ev[k]) cudaEventDestroy(w.ev[k]);
      }
      if (w.done) cudaEventDestroy(w.done);
      if (w.stream) cudaStreamDestroy(w.stream);
    }
  }

  cudaError_t copy(const std::vector<Piece>& pieces, cudaEvent_t after) {
    used_ = 0;
    cudaError_t e = cudaSetDevice(device_);
    if (e == cudaSuccess) e = ensure_workers(1);
    if (e != cudaSuccess) return e;
    std::vector<Piece> staged;
    std::vector<Piece> direct;
    for (const Piece& pc : pieces) {
      cudaPointerAttributes attr;
      e = cudaPointerGetAttributes(&attr, pc.src);
      if (e != cudaSuccess) cudaGetLastError();  // unknown host memory: treat as pageable
      if (e == cudaSuccess && attr.type == cudaMemoryTypeHost) {
        direct.push_back(pc);
      } else {
        for (uint64_t o = 0; o < pc.bytes; o += kSlotBytes)
          staged.push_back(Piece{pc.dst + o, pc.src + o, std::min(kSlotBytes, pc.bytes - o)});
      }
    }
    const size_t nw = std::max<size_t>(1, std::min<size_t>((size_t)nworkers_, staged.size()));
    e = ensure_workers(nw);
    for (size_t w = 0; w < nw && e == cudaSuccess; ++w) e = cudaStreamWaitEvent(workers_[w].stream, after, 0);
    for (const Piece& pc : direct) {
      if (e != cudaSuccess) break;
      e = cudaMemcpyAsync(pc.dst, pc.src, pc.bytes, cudaMemcpyHostToDevice, workers_[0].stream);
    }
    if (e != cudaSuccess) return e;
    std::atomic<size_t> next{0};
    std::mutex mu;
    cudaError_t first_error = cudaSuccess;
    auto body = [&](size_t w) {
      Worker& wk = workers_[w];
      cudaError_t err = cudaSetDevice(device_);
      for (size_t i = next++; i < staged.size() && err == cudaSuccess; i = next++) {
        const int k = wk.turn;
        wk.turn ^= 1;
        const auto tw = std::chrono::steady_clock::now();
        err = cudaEventSynchronize(wk.ev[k]);  // the slot's previous DMA is done
        wk.wait_seconds += seconds_since(tw);
        if (err != cudaSuccess) break;
        const auto t0 = std::chrono::steady_clock::now();
        memcpy(wk.slot[k], staged[i].src, staged[i].bytes);
        wk.memcpy_seconds += seconds_since(t0);
        err = cudaMemcpyAsync(staged[i].dst, wk.slot[k], staged[i].bytes, cudaMemcpyHostToDevice, wk.stream);
        if (err == cudaSuccess) err = cudaEventRecord(wk.ev[k], wk.stream);
      }
      if (err != cudaSuccess) {
        std::lock_guard<std::mutex> lk(mu);
        if (first_error == cudaSuccess) first_error = err;
      }
    };
    std::vector<std::thread> pool;
    for (size_t w = 1; w < nw; ++w) pool.emplace_back(body, w);
    body(0);
    for (auto& t : pool) t.join();
    if (first_error != cudaSuccess) return first_error;
    for (size_t w = 0; w < nw; ++w) {
      e = cudaEventRecord(workers_[w].done, workers_[w].stream);
      if (e != cudaSuccess) return e;
    }
    used_ = nw;
    return cudaSuccess;
  }

  // Work queued on `stream` after this call starts once the last copy() is done.
  cudaError_t order_before(cudaStream_t stream) {
    for (size_t w = 0; w < used_; ++w) {
      cudaError_t e = cudaStreamWaitEvent(stream, workers_[w].done, 0);
      if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
  }

  // Thread-seconds spent copying into slots and waiting for slots, summed over workers.
  void busy(double* memcpy_s, double* wait_s) const {
    *memcpy_s = *wait_s = 0;
    for (const Worker& w : workers_) {
      *memcpy_s += w.memcpy_seconds;
      *wait_s += w.wait_seconds;
    }
  }

 private:
  struct Worker {
    cudaStream_t stream = nullptr;
    uint8_t* slot[2] = {nullptr, nullptr};
    cudaEvent_t ev[2] = {nullptr, nullptr};
    cudaEvent_t done = nullptr;
    int turn = 0;
    double memcpy_seconds = 0, wait_seconds = 0;
  };

  cudaError_t ensure_workers(size_t n) {
    while (workers_.size() < n) {
      workers_.emplace_back();
      Worker& w = workers_.back();
      cudaError_t e = cudaStreamCreateWithFlags(&w.stream, cudaStreamNonBlocking);
      for (int k = 0; k < 2 && e == cudaSuccess; ++k) {
        e = cudaHostAlloc((void**)&w.slot[k], kSlotBytes, cudaHostAllocDefault);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&w.ev[k], cudaEventDisableTiming);
      }
      if (e == cudaSuccess) e = cudaEventCreateWithFlags(&w.done, cudaEventDisableTiming);
      if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
  }

  int device_;
  int nworkers_;
  size_t used_ = 0;
  std::vector<Worker> workers_;
};

// The device work of one batch: its packets, block jobs and A uploads.
struct BatchInput {
  size_t first = 0, last = 0;
  std::vector<BlockJob> blocks;
  std::vector<uint32_t> packet_first_block;
  std::vector<Uploader::Piece> pieces;
};

}  // namespace

int device_numa_node(int device) {
  char bus[64] = {0};
  if (cudaDeviceGetPCIBusId(bus, (int)sizeof(bus), device) != cudaSuccess) return -1;
  unsigned domain = 0, b = 0, d = 0, f = 0;
  if (sscanf(bus, "%x:%x:%x.%x", &domain, &b, &d, &f) != 4) return -1;
  char path[128];
  snprintf(path, sizeof(path), "/sys/bus/pci/devices/%04x:%02x:%02x.%x/numa_node", domain, b, d, f);
  FILE* fp = fopen(path, "r");
  if (!fp) return -1;
  int node = -1;
  if (fscanf(fp, "%d", &node) != 1) node = -1;
  fclose(fp);
  return node;
}

bool prefer_numa_node(void* p, uint64_t size, int node) {
  constexpr int kMaxNodes = 1024;
  constexpr int kBits = 8 * (int)sizeof(unsigned long);
  if (node < 0 || node >= kMaxNodes) return false;
  unsigned long mask[kMaxNodes / kBits] = {0};
  mask[node / kBits] = 1ul << (node % kBits);
  const long kMpolPreferred = 1;  // pages go to `node` while it has free memory, elsewhere otherwise
  return syscall(SYS_mbind, p, (unsigned long)size, kMpolPreferred, mask, (unsigned long)kMaxNodes, 0ul) == 0;
}

bool alloc_host_chunk(uint64_t bytes, bool pinned, int threads, ArenaChunk* out, std::string* err) {
  constexpr uint64_t kHuge = 2ull << 20;
  const uint64_t size = (std::max<uint64_t>(bytes, 1) + kHuge - 1) & ~(kHuge - 1);
  void* p = nullptr;
  if (posix_memalign(&p, kHuge, size) != 0) {
    *err = "cannot allocate " + std::to_string(bytes) + " bytes of host memory for the delta arena";
    return false;
  }
  *out = ArenaChunk{(uint8_t*)p, 0, bytes, false};
  if (!pinned) return true;
  madvise(p, size, MADV_HUGEPAGE);  // advisory: fewer, larger pages to fault and lock
  // The copy engines read the arena on every switch: place its pages on the
  // NUMA node of the device's PCIe link (advisory; WS_ARENA_NUMA=0 leaves the
  // placement to first touch).
  const char* numa = getenv("WS_ARENA_NUMA");
  int device = 0;
  if (!(numa && numa[0] == '0') && cudaGetDevice(&device) == cudaSuccess)
    prefer_numa_node(p, size, device_numa_node(device));
  const int nt = (int)std::max<uint64_t>(1, std::min<uint64_t>((uint64_t)std::max(1, std::min(threads, 8)), size / (8ull << 20)));
  const uint64_t per = (size / nt + kHuge - 1) & ~(kHuge - 1);
  std::vector<std::thread> pool;
  for (int t = 1; t < nt; ++t)
    pool.emplace_back([=] {
      const uint64_t a = std::min(size, t * per), b = std::min(size, a + per);
      memset((uint8_t*)p + a, 0, b - a);
    });
  memset(p, 0, std::min(size, per));
  for (auto& t : pool) t.join();
  const cudaError_t e = cudaHostRegister(p, size, cudaHostRegisterPortable);
  if (e != cudaSuccess) {
    free(p);
    *err = std::string("cannot page-lock the delta arena: ") + cudaGetErrorString(e);
    return false;
  }
  out->pinned = true;
  return true;
}

void free_host_chunk(const ArenaChunk& c) {
  if (!c.ptr) return;
  if (c.pinned) cudaHostUnregister(c.ptr);
  free(c.ptr);
}

#define WS_GPU_TRY(expr)                                                             \
  do {                                                                               \
    cudaError_t e_ = (expr);                                                         \
    if (e_ != cudaSuccess) {                                                         \
      if (e_ == cudaErrorMemoryAllocation) *device_oom = true;                       \
      *err = std::string("GPU encoder: ") + #expr + ": " + cudaGetErrorString(e_);   \
      return false;                                                                  \
    }                                                                                \
  } while (0)

bool gpu_encode_packets(const std::vector<GpuPacketInput>& packets, int policy, const CodingOptions& co,
                        uint64_t batch_bytes, int threads, bool pin, cudaStream_t stream,
                        std::vector<EncodedPacket>* out, std::vector<ArenaChunk>* chunks, std::string* err,
                        bool* device_oom) {
  *device_oom = false;
  out->resize(packets.size());
  int device = 0;
  WS_GPU_TRY(cudaGetDevice(&device));
  Uploader uploader(device, threads);
  uint64_t arena_off = 0;
  // WS_ENCODER_TIMING=1 prints the time spent in each phase to stderr.
  const bool timing = getenv("WS_ENCODER_TIMING") != nullptr;
  double t_upload = 0, t_stats = 0, t_tables = 0, t_encode = 0, t_pack = 0, t_alloc = 0, t_rule = 0;
  auto now = [] { return std::chrono::steady_clock::now(); };
  auto secs = [](std::chrono::steady_clock::time_point a, std::chrono::steady_clock::time_point b) {
    return std::chrono::duration<double>(b - a).count();
  };
  DeviceBuffer<uint8_t> d_base, d_payload, d_index;
  DeviceBuffer<BlockJob> d_blocks;
  DeviceBuffer<PacketStats> d_pstats;
  DeviceBuffer<BlockStats> d_bstats;
  DeviceBuffer<EncodeJob> d_jobs;
  DeviceBuffer<EncTable> d_tables;
  DeviceBuffer<const uint8_t*> d_index_ptrs;
  DeviceBuffer<uint16_t> d_enc;
  DeviceBuffer<uint32_t> d_nwords;
  DeviceBuffer<CompactJob> d_compact;
  DeviceBuffer<uint16_t> d_words;
  DeviceBuffer<uint32_t> d_side, d_side_count;
  // Batches: consecutive packets up to batch_bytes of weights; packets start
  // 256-byte aligned in the device copy of A.
  std::vector<std::pair<size_t, size_t>> ranges;
  uint64_t max_bytes = 0;
  for (size_t first = 0; first < packets.size();) {
    size_t last = first;
    uint64_t bytes = 0;
    while (last < packets.size() && (last == first || bytes + packets[last].nbytes <= batch_bytes))
      bytes += (packets[last++].nbytes + 255) & ~255ull;
    ranges.emplace_back(first, last);
    max_bytes = std::max(max_bytes, bytes);
    first = last;
  }
  if (ranges.empty()) return true;
  // One device copy of A per batch. (Uploading batch k+1 on a helper thread
  // while batch k is encoded was measured slower: the staging copies and the
  // arena's page faults and page locking contend for the host.)
  WS_GPU_TRY(d_base.ensure(max_bytes));
  struct Event {
    cudaEvent_t e = nullptr;  // the work reading d_base is done
    ~Event() {
      if (e) cudaEventDestroy(e);
    }
  } released;
  WS_GPU_TRY(cudaEventCreateWithFlags(&released.e, cudaEventDisableTiming));
  auto make_input = [&](size_t k, uint8_t* dbase) {
    BatchInput in;
    in.first = ranges[k].first;
    in.last = ranges[k].second;
    const size_t np = in.last - in.first;
    in.packet_first_block.resize(np + 1);
    uint64_t off = 0;
    for (size_t i = 0; i < np; ++i) {
      const GpuPacketInput& p = packets[in.first + i];
      if (p.nbytes) in.pieces.push_back(Uploader::Piece{dbase + off, p.base, p.nbytes});
      in.packet_first_block[i] = (uint32_t)in.blocks.size();
      for (uint64_t b = 0; b < p.nbytes; b += WS_BLOCK_BYTES)
        in.blocks.push_back(BlockJob{dbase + off + b, p.target + b,
                                     (uint32_t)std::min<uint64_t>(WS_BLOCK_BYTES, p.nbytes - b), (uint32_t)i});
      off += (p.nbytes + 255) & ~255ull;
    }
    in.packet_first_block[np] = (uint32_t)in.blocks.size();
    return in;
  };
  for (size_t k = 0; k < ranges.size(); ++k) {
    const BatchInput cur = make_input(k, d_base.ptr);
    const auto t_up = now();
    WS_GPU_TRY(cudaEventRecord(released.e, stream));
    WS_GPU_TRY(uploader.copy(cur.pieces, released.e));
    WS_GPU_TRY(uploader.order_before(stream));
    if (timing) WS_GPU_TRY(cudaStreamSynchronize(stream));
    t_upload += secs(t_up, now());
    const size_t first = cur.first, last = cur.last;
    const size_t np = last - first;
    const std::vector<BlockJob>& blocks = cur.blocks;
    const std::vector<uint32_t>& packet_first_block = cur.packet_first_block;
    auto t0 = now();
    const size_t nb = blocks.size();
    WS_GPU_TRY(d_blocks.ensure(nb));
    WS_GPU_TRY(d_pstats.ensure(np));
    WS_GPU_TRY(d_bstats.ensure(nb));
    WS_GPU_TRY(cudaMemcpyAsync(d_blocks.ptr, blocks.data(), nb * sizeof(BlockJob), cudaMemcpyHostToDevice, stream));
    WS_GPU_TRY(cudaMemsetAsync(d_pstats.ptr, 0, np * sizeof(PacketStats), stream));
    if (nb) {
      stats_kernel<<<(unsigned)nb, kStatsThreads, 0, stream>>>(d_blocks.ptr, d_pstats.ptr, d_bstats.ptr);
      WS_GPU_TRY(cudaGetLastError());
    }
    std::vector<PacketStats> pstats(np);
    std::vector<BlockStats> bstats(nb);
    WS_GPU_TRY(cudaMemcpyAsync(pstats.data(), d_pstats.ptr, np * sizeof(PacketStats), cudaMemcpyDeviceToHost, stream));
    WS_GPU_TRY(cudaMemcpyAsync(bstats.data(), d_bstats.ptr, nb * sizeof(BlockStats), cudaMemcpyDeviceToHost, stream));
    WS_GPU_TRY(cudaStreamSynchronize(stream));
    t_stats += secs(t0, now());
    t0 = now();

    // Tables per packet and candidate (host, shared code with the host encoder).
    struct Cand {
      int table = -1;
      bool dict = false;
    };
    std::vector<Cand> cand(np * 2);
    std::vector<EncTable> tables;
    std::vector<std::vector<uint16_t>> dict_words;
    std::vector<int> dict_esc;  // escape symbol of each dictionary, or -1
    bool any_escape = false;
    std::vector<int> dict_of_table;
    std::vector<EncodeJob> jobs;
    std::vector<std::vector<uint32_t>> job_of(np * 2);
    std::vector<CodingTables> coding(np * 2);
    std::vector<char> skip(np, 0);
    for (size_t i = 0; i < np; ++i) {
      const GpuPacketInput& p = packets[first + i];
      EncodedPacket& e = (*out)[first + i];
      e.nbytes = p.nbytes;
      e.blocks.clear();
      e.zero_block_bytes = 0;
      e.payload_bytes = 0;
      bool any = false;
      uint32_t coded = 0;
      for (uint32_t b = packet_first_block[i]; b < packet_first_block[i + 1]; ++b) {
        if (bstats[b].nonzero) {
          any = true;
          ++coded;
        } else {
          e.zero_block_bytes += blocks[b].nbytes;
        }
      }
      if (p.nbytes == 0 || !any) {  // delta.py:181-182: unchanged chunk
        e.mode = WS_MODE_SKIP;
        e.zero_block_bytes = 0;
        skip[i] = 1;
        continue;
      }
      const bool big = p.nbytes >= WS_COMPRESS_MIN;
      const bool try_c[2] = {big && !(policy == 2 && p.is_bf16), big && p.is_bf16 && (p.nbytes % 2 == 0) && policy != 1};
      for (int c = 0; c < 2; ++c) {
        if (!try_c[c]) continue;
        const PacketStats& ps = pstats[i];
        uint64_t counts[2][256];
        for (int q = 0; q < 2; ++q)
          for (int s = 0; s < 256; ++s) counts[q][s] = ps.plane[c][q][s];
        // Distinct words (h = 0) and distinct high 12 bits (h = 1), increasing.
        std::vector<uint16_t> words[2];
        std::vector<uint64_t> wcounts[2];
        bool many[2];
        for (int h = 0; h < 2; ++h) {
          std::vector<std::pair<uint16_t, uint64_t>> wl;
          many[h] = ps.many[h][c] != 0;
          if (!many[h])
            for (uint32_t k = 0; k < kPacketSlots; ++k)
              if (ps.key[h][c][k]) wl.emplace_back((uint16_t)(ps.key[h][c][k] - 1), ps.cnt[h][c][k]);
          std::sort(wl.begin(), wl.end());
          for (auto& pr : wl) {
            words[h].push_back(pr.first);
            wcounts[h].push_back(pr.second);
          }
        }
        CodingTables& ct = coding[2 * i + c];
        choose_coding(counts, words[0], wcounts[0], many[0] || words[0].size() > 255, words[1], wcounts[1],
                      many[1] || words[1].size() > 255, coded, co, &ct);
        Cand& cd = cand[2 * i + c];
        cd.table = (int)tables.size();
        cd.dict = ct.dict;
        EncTable et;
        fill_enc_table(ct, &et);
        tables.push_back(et);
        dict_of_table.push_back(ct.dict ? (int)dict_words.size() : -1);
        if (ct.dict) {
          dict_words.push_back(ct.words);
          dict_esc.push_back(ct.escape ? (int)ct.words.size() : -1);
        }
        const uint32_t esc = ct.escape ? (uint32_t)ct.words.size() : ~0u;
        any_escape |= ct.escape;
        for (uint32_t b = packet_first_block[i]; b < packet_first_block[i + 1]; ++b) {
          if (!bstats[b].nonzero) continue;
          job_of[2 * i + c].push_back((uint32_t)jobs.size());
          jobs.push_back(EncodeJob{b, (uint32_t)cd.table, ct.dict ? 1u : 0u, (uint32_t)c, esc, ct.dict ? ct.split : 0u});
        }
      }
    }
    t_tables += secs(t0, now());
    t0 = now();
    // Encode every candidate block.
    std::vector<uint32_t> nwords(jobs.size());
    std::vector<uint32_t> side_count;
    // Payload of job jj when coded: stream (+ escape list); `ok` is false when a
    // lane has more escapes than a list holds (the block is then coded raw).
    auto coded_size = [&](uint32_t jj, bool* ok, uint32_t* escapes) {
      uint32_t size = (2 * nwords[jj] + 15) & ~15u, total = 0, most = 0;
      size += ws_split_raw_bytes(blocks[jobs[jj].block].nbytes / 2, jobs[jj].split);
      if (jobs[jj].esc != ~0u)
        for (uint32_t l = 0; l < WS_LANES; ++l) {
          total += side_count[(size_t)jj * WS_LANES + l];
          most = std::max(most, side_count[(size_t)jj * WS_LANES + l]);
        }
      if (total) size += (WS_ESCAPE_HEADER_BYTES + 4 * total + 15) & ~15u;
      *ok = most <= WS_ESCAPE_LANE_MAX;
      *escapes = total;
      return size;
    };
    if (!jobs.empty()) {
      WS_GPU_TRY(d_tables.ensure(tables.size()));
      WS_GPU_TRY(cudaMemcpyAsync(d_tables.ptr, tables.data(), tables.size() * sizeof(EncTable), cudaMemcpyHostToDevice, stream));
      WS_GPU_TRY(d_index.ensure(std::max<size_t>(1, dict_words.size()) * 65536));
      WS_GPU_TRY(d_words.ensure(std::max<size_t>(1, dict_words.size()) * 256));
      std::vector<const uint8_t*> index_ptrs(tables.size(), nullptr);
      for (size_t t = 0; t < tables.size(); ++t) {
        const int d = dict_of_table[t];
        if (d < 0) continue;
        index_ptrs[t] = d_index.ptr + (size_t)d * 65536;
        uint16_t* dw = d_words.ptr + (size_t)d * 256;
        WS_GPU_TRY(cudaMemcpyAsync(dw, dict_words[d].data(), dict_words[d].size() * 2, cudaMemcpyHostToDevice, stream));
        // Words outside the dictionary map to its escape symbol (never looked up without escapes).
        WS_GPU_TRY(cudaMemsetAsync(d_index.ptr + (size_t)d * 65536, dict_esc[d] >= 0 ? dict_esc[d] : 0, 65536, stream));
        dict_index_kernel<<<1, 256, 0, stream>>>(dw, (uint32_t)dict_words[d].size(), d_index.ptr + (size_t)d * 65536);
        WS_GPU_TRY(cudaGetLastError());
      }
      WS_GPU_TRY(d_index_ptrs.ensure(tables.size()));
      WS_GPU_TRY(cudaMemcpyAsync(d_index_ptrs.ptr, index_ptrs.data(), tables.size() * sizeof(void*), cudaMemcpyHostToDevice, stream));
      WS_GPU_TRY(d_jobs.ensure(jobs.size()));
      WS_GPU_TRY(cudaMemcpyAsync(d_jobs.ptr, jobs.data(), jobs.size() * sizeof(EncodeJob), cudaMemcpyHostToDevice, stream));
      WS_GPU_TRY(d_enc.ensure(jobs.size() * (size_t)kOutHalfwords));
      WS_GPU_TRY(d_nwords.ensure(jobs.size()));
      WS_GPU_TRY(d_side.ensure(any_escape ? jobs.size() * WS_LANES * WS_ESCAPE_LANE_MAX : 1));
      WS_GPU_TRY(d_side_count.ensure(any_escape ? jobs.size() * WS_LANES : 1));
      const unsigned grid = (unsigned)((jobs.size() + kEncWarps - 1) / kEncWarps);
      encode_kernel<<<grid, kEncWarps * 32, 0, stream>>>(d_blocks.ptr, d_jobs.ptr, (uint32_t)jobs.size(), d_tables.ptr,
                                                         d_index_ptrs.ptr, d_enc.ptr, d_nwords.ptr, d_side.ptr,
                                                         d_side_count.ptr);
      WS_GPU_TRY(cudaGetLastError());
      WS_GPU_TRY(cudaMemcpyAsync(nwords.data(), d_nwords.ptr, jobs.size() * 4, cudaMemcpyDeviceToHost, stream));
      if (any_escape) {
        side_count.resize(jobs.size() * WS_LANES);
        WS_GPU_TRY(cudaMemcpyAsync(side_count.data(), d_side_count.ptr, side_count.size() * 4, cudaMemcpyDeviceToHost,
                                   stream));
      }
      WS_GPU_TRY(cudaStreamSynchronize(stream));
    }
    t_encode += secs(t0, now());
    t0 = now();
    // Mode rule (delta.py:184-193) and raw fallback, then pack the chosen payloads.
    std::vector<CompactJob> compact;
    uint64_t out_bytes = 0;
    for (size_t i = 0; i < np; ++i) {
      EncodedPacket& e = (*out)[first + i];
      if (skip[i]) continue;
      const uint64_t n = packets[first + i].nbytes;
      int mode = WS_MODE_XOR_RAW, best_c = -1;
      uint64_t best = n;
      for (int c = 0; c < 2; ++c) {
        if (cand[2 * i + c].table < 0) continue;
        uint64_t size = 1024;
        for (uint32_t jj : job_of[2 * i + c]) {
          bool ok;
          uint32_t esc_n;
          const uint32_t ans = coded_size(jj, &ok, &esc_n);
          const uint32_t raw = (blocks[jobs[jj].block].nbytes + 15) & ~15u;
          size += ok && ans < raw ? ans : raw;
        }
        if (size < best) {
          best = size;
          best_c = c;
          mode = c == 1 ? WS_MODE_U16_ANS : ((n % 2 == 0) ? WS_MODE_XOR_GROUP2_ANS : WS_MODE_XOR_ANS);
        }
      }
      e.mode = mode;
      e.payload_bytes = best;
      if (best_c >= 0)
        memcpy(e.table, coding[2 * i + best_c].entries, sizeof(e.table));
      else
        memset(e.table, 0, sizeof(e.table));
      size_t jpos = 0;
      for (uint32_t b = packet_first_block[i]; b < packet_first_block[i + 1]; ++b) {
        if (!bstats[b].nonzero) continue;
        EncodedBlock blk;
        blk.offset = (b - packet_first_block[i]) * WS_BLOCK_BYTES;
        blk.nbytes = blocks[b].nbytes;
        blk.tail = 0;
        blk.flags = 0;
        blk.nwords = 0;
        blk.kind = WS_KIND_RAW;
        blk.lane_sum[0] = bstats[b].lane_sum[0];
        blk.lane_sum[1] = bstats[b].lane_sum[1];
        const uint32_t raw = (blk.nbytes + 15) & ~15u;
        CompactJob cj{b, ~0u, 0, 0, out_bytes, 0, 0};
        uint32_t size = raw;
        if (best_c >= 0) {
          const uint32_t jj = job_of[2 * i + best_c][jpos];
          bool ok;
          uint32_t esc_n;
          const uint32_t ans = coded_size(jj, &ok, &esc_n);
          if (ok && ans < raw) {
            const bool dict = cand[2 * i + best_c].dict;
            blk.kind = best_c == 1 ? (dict ? WS_KIND_DICT_U16 : WS_KIND_ANS_U16)
                                   : (dict ? WS_KIND_DICT_XOR : WS_KIND_ANS_XOR);
            blk.nwords = nwords[jj];
            if (blk.nbytes & 1u) {
              blk.flags = WS_FLAG_ODD_TAIL;
              blk.tail = (uint8_t)bstats[b].tail;
            }
            if (esc_n) blk.flags |= WS_FLAG_ESCAPES;
            blk.flags |= (uint8_t)ws_split_flags(jobs[jj].split);
            cj.encode = jj;
            cj.nwords = nwords[jj];
            cj.escapes = esc_n;
            cj.split = jobs[jj].split;
            cj.u16 = jobs[jj].u16;
            size = ans;
          }
        }
        ++jpos;
        blk.clen = size;
        compact.push_back(cj);
        out_bytes += size;
        e.blocks.push_back(std::move(blk));
      }
    }
    t_rule += secs(t0, now());
    if (!compact.empty()) {
      WS_GPU_TRY(d_compact.ensure(compact.size()));
      WS_GPU_TRY(d_payload.ensure(out_bytes));
      WS_GPU_TRY(cudaMemcpyAsync(d_compact.ptr, compact.data(), compact.size() * sizeof(CompactJob), cudaMemcpyHostToDevice, stream));
      compact_kernel<<<(unsigned)compact.size(), 256, 0, stream>>>(d_compact.ptr, d_blocks.ptr, d_enc.ptr, d_side.ptr,
                                                                   d_side_count.ptr, d_payload.ptr);
      WS_GPU_TRY(cudaGetLastError());
      // The batch's payloads become one arena chunk (arena order is packet, block order).
      ArenaChunk ch;
      const auto ta = now();
      if (!alloc_host_chunk(out_bytes, pin, threads, &ch, err)) return false;
      t_alloc += secs(ta, now());
      ch.off = arena_off;
      chunks->push_back(ch);
      WS_GPU_TRY(cudaMemcpyAsync(ch.ptr, d_payload.ptr, out_bytes, cudaMemcpyDeviceToHost, stream));
      arena_off += out_bytes;
    }
    if (timing) WS_GPU_TRY(cudaStreamSynchronize(stream));
    t_pack += secs(t0, now());
  }
  WS_GPU_TRY(cudaStreamSynchronize(stream));
  if (timing) {
    double mc = 0, wt = 0;
    uploader.busy(&mc, &wt);
    fprintf(stderr,
            "gpu encoder: upload %.3f s (slot memcpy %.3f, slot wait %.3f thread-s), stats %.3f s, tables %.3f s, "
            "encode %.3f s, pack %.3f s (mode rule %.3f, chunk allocation %.3f)\n",
            t_upload, mc, wt, t_stats, t_tables, t_encode, t_pack, t_rule, t_alloc);
  }
  return true;
}

}  // namespace ws
