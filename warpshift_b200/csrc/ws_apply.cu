// Fused rANS decode + in-place XOR / wrapping-u16 apply for B200 (sm_100a).
//
// Replaces, in one kernel, nvCOMP's batched ANS decode into a scratch buffer
// (warpshift/delta.py:313-316) and the Triton read-modify-write kernel
// _restore_batch (delta.py:60-92, launched at 317-324). The decoded residual
// never touches HBM: per 128 KiB block the kernel reads the compressed payload
// once and reads + writes the destination weights once.
//
// Work decomposition: one CTA (16 warps) per tile of up to 16 blocks of one
// packet; one warp per block. The packet's two 256-slot decode tables are
// replicated 32 times in shared memory so that lane l always reads bank l
// (conflict-free random lookups). Each warp streams its compressed payload
// from HBM into a 2 x 1 KiB shared-memory ring with cp.async.bulk (TMA bulk
// copies, no multicast) completing on per-slot mbarriers; a mirror of the
// first 640 bytes of each even half sits behind the ring so that a group's
// reads never need wrapping.
//
// The inner loop (two decode steps of both planes plus the warp-cooperative
// renormalisation) is hand-written PTX: about 50 instructions per 4 decoded
// bytes per lane, balanced between the ALU and FMA pipes.
#include <cuda_runtime.h>
#include <stdint.h>

#include "ws_format.h"
#include "ws_guard.h"
#include "ws_kernels.h"

namespace ws {

namespace {

constexpr uint32_t kWarps = WS_TILE_BLOCKS;
constexpr uint32_t kThreads = kWarps * 32;
// Replicated slot tables: row `slot` (256 bytes) holds plane 0's entry for lanes
// 0..31 (bytes 4 * lane) and plane 1's (bytes 128 + 4 * lane), so lane l always
// reads bank l, and a lookup address is one PRMT of the state (its low byte
// moved into byte 1) over the lane's row offset, plus the table base.
constexpr uint32_t kRowBytes = 256;
constexpr uint32_t kTableBytes = 256 * kRowBytes;           // both planes, 64 KiB
constexpr uint32_t kRingOffset = kTableBytes;               // bytes
// Shared address at which the dynamic shared memory (and so the table region)
// of a kernel without static shared variables begins on sm_100 (after the 1 KiB
// the system reserves). The kernel checks it at run time and falls back to a
// register base if it differs.
constexpr uint32_t kFixedTableBase = 0x400;
constexpr uint32_t kMirror = 640;  // a group reads <= 512 + 128 bytes past its start position
constexpr uint32_t kRingStride = WS_RING_BYTES + kMirror;
constexpr uint32_t kBarOffset = kRingOffset + kWarps * kRingStride;
// Raw-bit expansion table of a tile whose packet splits words: entry b spreads
// raw byte b over the word pairs it covers (16, 8 or 4 bytes for k = 1, 2, 4).
constexpr uint32_t kSplitTabOffset = kBarOffset + kWarps * 2 * 8;
constexpr uint32_t kSplitTabBytes = 256 * 16;
constexpr uint32_t kSmemBytes = kSplitTabOffset + kSplitTabBytes;
constexpr uint32_t kRingHalfwords = WS_RING_BYTES / 2;      // 1024
constexpr uint32_t kHalfHalfwords = WS_RING_HALF_BYTES / 2; // 512
constexpr uint32_t kWaitLimit = 1u << 20;      // bounded spin on a staging barrier
constexpr uint32_t kDrainRounds = 16;          // bounded waits per outstanding copy before a CTA exits
constexpr uint32_t kPrefetchGroups = 3;        // destination groups requested into L2 ahead of their load

__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint32_t lds16(uint32_t addr) {
  uint16_t v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr));
  return v;
}

// Asks the TMA unit to pull `bytes` of global memory into L2 (no registers, no
// completion to wait for): hides DRAM latency of the destination loads.
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// 16-byte global load issued exactly where it appears (volatile keeps it ahead
// of the hand-written decode blocks, so it is not sunk to its first use).
__device__ __forceinline__ uint4 ldg128_early(const void* p) {
  uint4 v;
  asm volatile("ld.global.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

__device__ __forceinline__ uint32_t lanemask_lt() {
  uint32_t m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

// PRMT in its default mode: a selector nibble with bit 3 set replicates the
// sign bit of the selected byte.
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

// One expect_tx covering two bulk copies of the same source (ring slot + mirror).
__device__ __forceinline__ void bulk_load2(uint32_t dst0, uint32_t dst1, const void* src, uint32_t bytes0,
                                           uint32_t bytes1, uint32_t bar) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes0 + bytes1) : "memory");
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst0),
      "l"(src), "r"(bytes0), "r"(bar)
      : "memory");
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst1),
      "l"(src), "r"(bytes1), "r"(bar)
      : "memory");
}

// Returns true when the phase with the given parity has completed, false if
// the bounded wait gave up.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, uint32_t limit = kWaitLimit) {
  for (uint32_t it = 0; it < limit; ++it) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    if (ok) return true;
  }
  return false;
}

__device__ __forceinline__ void report(ws_device_result* res, uint32_t err, uint32_t block) {
  atomicOr(&res->errors, err);
  atomicExch(&res->bad_block_plus1, block + 1);
}

// U16 apply on two 16-bit words at once. The coded word y is the rotated
// zigzag of d = B - A, so d = y ^ (bit 15 of y ? 0x7FFF : 0) per half; the new
// word is old + d (forward) or old - d (reverse), wrapping per half. The 16x2
// SIMD add does the per-half wrap in one instruction; reverse adds the
// per-half two's complement ~d + 1.
__device__ __forceinline__ uint32_t add16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.u16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

__device__ __forceinline__ uint32_t u16_apply(uint32_t old, uint32_t y, bool reverse) {
  const uint32_t d = y ^ (prmt(y, 0, 0xBB99) & 0x7FFF7FFFu);  // prmt: 0xFFFF per half with bit 15 set
  if (!reverse) return add16x2(old, d);
  return add16x2(old, add16x2(~d, 0x00010001u));
}

struct Checksum {
  uint32_t a = 0, b = 0;
  __device__ __forceinline__ void add(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3) {
    a += w0 + w1 + w2 + w3;
    b += a;
  }
  __device__ __forceinline__ void finish(uint32_t lane, uint32_t block, ws_device_result* res) const {
    unsigned long long h = ws_lane_hash(a, b, lane);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) h += __shfl_xor_sync(0xFFFFFFFFu, h, o);
    if (lane == 0) atomicAdd(&res->checksum, (unsigned long long)ws_block_hash(h, block));
  }
};

// Slow path for one lane's 16-byte chunk of a group: partial group, odd tail,
// or a destination that is not 16-byte aligned. r[0..3] hold the lane's 8
// residual words (XOR value or rotated zigzag word); bytes below coded_bytes
// are coded words, a byte at coded_bytes is the block's uncoded odd tail.
// Fully unrolled so that r[] and out[] stay in registers.
template <bool U16, bool REVERSE>
__device__ __forceinline__ void apply_chunk_bytes(uint8_t* p, uint32_t first_byte, uint32_t nbytes,
                                                  const uint32_t (&r)[4], uint32_t coded_bytes, uint8_t tail,
                                                  uint32_t (&out)[4]) {
#pragma unroll
  for (uint32_t j = 0; j < 8; ++j) {
    const uint32_t bi = first_byte + 2 * j;
    const uint32_t rw = (r[j >> 1] >> (16 * (j & 1))) & 0xFFFFu;
    uint32_t nw = 0;
    if (bi < coded_bytes) {  // coded words come in byte pairs
      const uint32_t old = (uint32_t)p[2 * j] | ((uint32_t)p[2 * j + 1] << 8);
      if (U16)
        nw = u16_apply(old, rw, REVERSE) & 0xFFFFu;
      else
        nw = old ^ rw;
      p[2 * j] = (uint8_t)(nw & 0xFF);
      p[2 * j + 1] = (uint8_t)(nw >> 8);
    } else if (bi < nbytes) {  // the uncoded odd last byte of the block
      nw = (uint32_t)(uint8_t)(p[2 * j] ^ tail);
      p[2 * j] = (uint8_t)nw;
    }
    out[j >> 1] |= nw << (16 * (j & 1));
  }
}

__device__ void raw_block(const ws_block_desc& bd, uint32_t block, const uint8_t* __restrict__ src, uint32_t lane,
                          ws_device_result* res) {
  uint8_t* dst = reinterpret_cast<uint8_t*>(bd.dst);
  const uint32_t n = bd.nbytes;
  const uint32_t groups = (n + WS_GROUP_BYTES - 1) / WS_GROUP_BYTES;
  const bool aligned = (bd.dst & 15u) == 0;
  Checksum ck;
#pragma unroll 1
  for (uint32_t g = 0; g < groups; ++g) {
    const uint32_t off = g * WS_GROUP_BYTES + lane * 16u;
    if (aligned && (g + 1) * WS_GROUP_BYTES <= n) {
      const uint4 r = __ldg(reinterpret_cast<const uint4*>(src + off));
      uint4* d = reinterpret_cast<uint4*>(dst + off);
      uint4 v = *d;
      v.x ^= r.x;
      v.y ^= r.y;
      v.z ^= r.z;
      v.w ^= r.w;
      *d = v;
      ck.add(v.x, v.y, v.z, v.w);
    } else {
      uint32_t out[4] = {0, 0, 0, 0};
#pragma unroll
      for (uint32_t k = 0; k < 16; ++k) {
        if (off + k < n) {
          const uint8_t nv = (uint8_t)(dst[off + k] ^ src[off + k]);
          dst[off + k] = nv;
          out[k >> 2] |= (uint32_t)nv << (8 * (k & 3));
        }
      }
      ck.add(out[0], out[1], out[2], out[3]);
    }
  }
  ck.finish(lane, block, res);
}

// Generic-path decode step (partial groups, unaligned destinations): both
// planes, word = sym0 | sym1 << 8. Slot entry: bias | sym << 8 | freq << 16.
#define WS_STEP_C(ea, eb)                                      \
  {                                                            \
    ea = lds32(tb0 + ((xa & 255u) << 8));                      \
    eb = lds32(tb1 + ((xb & 255u) << 8));                      \
    xa = (ea >> 16) * (xa >> 8) + (ea & 255u);                 \
    xb = (eb >> 16) * (xb >> 8) + (eb & 255u);                 \
  }

// Generic-path renormalisation: every state below 2^16 reads one word; plane-0
// reads come first in lane order, then plane-1 reads.
#define WS_RENORM_C()                                                                         \
  {                                                                                           \
    const uint32_t base = ring_s + (pos & (kRingHalfwords - 1)) * 2u;                         \
    const bool na = xa < WS_RANS_L, nb = xb < WS_RANS_L;                                      \
    const uint32_t ba = __ballot_sync(0xFFFFFFFFu, na);                                       \
    const uint32_t bb = __ballot_sync(0xFFFFFFFFu, nb);                                       \
    const uint32_t ca = __popc(ba);                                                           \
    if (na) xa = (xa << 16) | lds16(base + 2u * __popc(ba & ltm));                            \
    if (nb) xb = (xb << 16) | lds16(base + 2u * (ca + __popc(bb & ltm)));                     \
    pos += ca + __popc(bb);                                                                   \
  }

// Row address of a slot entry: PRMT moves the state's low byte (the slot) into
// byte 1 over the lane's row offset (byte 0), and the table region's base is
// added. When the region sits at the expected shared address (FIXED_BASE) the
// base is the load's immediate offset (operand %8) and costs no instruction;
// otherwise it is added from a register.
#define WS_ROW_ADDR(ADD) \
  " prmt.b32 aa, %0, %5, 0x5504;\n prmt.b32 ab, %1, %6, 0x5504;\n" ADD
#define WS_ROW_ADDR_D(ADD) \
  " prmt.b32 aa, %0, %6, 0x5504;\n prmt.b32 ab, %1, %6, 0x5504;\n" ADD
#define WS_ADD_BASE_F " add.u32 aa, aa, %4;\n add.u32 ab, ab, %4;\n"
#define WS_ADD_BASE_D " add.u32 aa, aa, %5;\n add.u32 ab, ab, %5;\n"
#define WS_LD_ENTRIES " ld.shared.u32 ea, [aa+%8];\n ld.shared.u32 eb, [ab+%8];\n"

// Renormalisation shared by both checks: ballot, prefix counts, one 16-bit word
// per state below 2^16 (plane-0 / even-word states first in lane order, then
// the others, read from rb = rp + 2 * their count); XA, XB, RP, LTM name the
// asm operands.
#define WS_RENORM_PTX(XA, XB, RP, LTM)                                                             \
  " setp.lt.u32 pa, " XA ", 65536;\n setp.lt.u32 pb, " XB ", 65536;\n"                              \
  " vote.sync.ballot.b32 va, pa, 0xffffffff;\n vote.sync.ballot.b32 vb, pb, 0xffffffff;\n"           \
  " popc.b32 ca, va;\n"                                                                             \
  " and.b32 t, va, " LTM ";\n popc.b32 oa, t;\n mad.lo.u32 ada, oa, 2, " RP ";\n"                  \
  " mad.lo.u32 rb, ca, 2, " RP ";\n"                                                                \
  " and.b32 t, vb, " LTM ";\n popc.b32 ob, t;\n mad.lo.u32 adb, ob, 2, rb;\n"                      \
  " popc.b32 cb, vb;\n mad.lo.u32 " RP ", cb, 2, rb;\n"                                            \
  " @pa ld.shared.u16 wa, [ada];\n @pb ld.shared.u16 wb, [adb];\n"                                  \
  " @pa prmt.b32 " XA ", wa, " XA ", 0x5410;\n @pb prmt.b32 " XB ", wb, " XB ", 0x5410;\n"

// Fast-path check in hand-written PTX: two decode steps of both planes (the
// lane's words 2c and 2c+1 of the group) and one renormalisation check.
// rp is the byte address of the current stream position in the ring; the
// caller re-bases it once per group. `tbase` is the table region's shared
// address and lba / lbb the lane's row offsets of planes 0 and 1. Returns the
// two words as lo | hi << 16.
#define WS_CHECK_FAST_PTX(ADD)                                                             \
  "{\n"                                                                                    \
  " .reg .u32 aa, ab, ea, eb, qa, qb, fa, fb, ba, bb, w0, w1, va, vb, ca, cb, oa, ob, t, rb, ada, adb, wa, wb;\n" \
  " .reg .pred pa, pb;\n"                                                                  \
  WS_ROW_ADDR(ADD)                                                                         \
  WS_LD_ENTRIES                                                                            \
  " shr.u32 qa, %0, 8;\n shr.u32 qb, %1, 8;\n"                                            \
  " shr.u32 fa, ea, 16;\n shr.u32 fb, eb, 16;\n"                                          \
  " and.b32 ba, ea, 255;\n and.b32 bb, eb, 255;\n"                                        \
  " mad.lo.u32 %0, fa, qa, ba;\n mad.lo.u32 %1, fb, qb, bb;\n"                            \
  " prmt.b32 w0, ea, eb, 0x0051;\n"                                                        \
  WS_ROW_ADDR(ADD)                                                                         \
  WS_LD_ENTRIES                                                                            \
  " shr.u32 qa, %0, 8;\n shr.u32 qb, %1, 8;\n"                                            \
  " shr.u32 fa, ea, 16;\n shr.u32 fb, eb, 16;\n"                                          \
  " and.b32 ba, ea, 255;\n and.b32 bb, eb, 255;\n"                                        \
  " mad.lo.u32 %0, fa, qa, ba;\n mad.lo.u32 %1, fb, qb, bb;\n"                            \
  " prmt.b32 w1, ea, eb, 0x5100;\n"                                                        \
  " prmt.b32 %2, w0, w1, 0x7610;\n"                                                        \
  WS_RENORM_PTX("%0", "%1", "%3", "%7")                                                     \
  "}\n"

template <bool FIXED_BASE>
__device__ __forceinline__ uint32_t check_fast(uint32_t& xa, uint32_t& xb, uint32_t& rp, uint32_t tbase, uint32_t lba,
                                               uint32_t lbb, uint32_t ltm) {
  uint32_t out;
  if (FIXED_BASE)
    asm volatile(WS_CHECK_FAST_PTX("") : "+r"(xa), "+r"(xb), "=r"(out), "+r"(rp)
                 : "r"(tbase), "r"(lba), "r"(lbb), "r"(ltm), "n"(kFixedTableBase));
  else
    asm volatile(WS_CHECK_FAST_PTX(WS_ADD_BASE_F) : "+r"(xa), "+r"(xb), "=r"(out), "+r"(rp)
                 : "r"(tbase), "r"(lba), "r"(lbb), "r"(ltm), "n"(0));
  return out;
}

// Dictionary-block check in hand-written PTX: two decode steps in which state
// A decodes the lane's even word and state B the following odd word (one
// table, entry = word | bias << 16 | freq << 24, at the lane's plane-0 row
// offset lba), then one renormalisation check. out0/out1 receive words
// (2s, 2s+1) of steps s = 0, 1 as lo | hi << 16.
#define WS_CHECK_DICT_PTX(ADD)                                                             \
  "{\n"                                                                                    \
  " .reg .u32 aa, ab, ea, eb, qa, qb, fa, fb, ba, bb, va, vb, ca, cb, oa, ob, t, rb, ada, adb, wa, wb;\n" \
  " .reg .pred pa, pb;\n"                                                                  \
  WS_ROW_ADDR_D(ADD)                                                                       \
  WS_LD_ENTRIES                                                                            \
  " shr.u32 qa, %0, 8;\n shr.u32 qb, %1, 8;\n"                                            \
  " shr.u32 fa, ea, 24;\n shr.u32 fb, eb, 24;\n"                                          \
  " prmt.b32 ba, ea, 0, 0x4442;\n prmt.b32 bb, eb, 0, 0x4442;\n"                          \
  " mad.lo.u32 %0, fa, qa, ba;\n mad.lo.u32 %1, fb, qb, bb;\n"                            \
  " prmt.b32 %2, ea, eb, 0x5410;\n"                                                        \
  WS_ROW_ADDR_D(ADD)                                                                       \
  WS_LD_ENTRIES                                                                            \
  " shr.u32 qa, %0, 8;\n shr.u32 qb, %1, 8;\n"                                            \
  " shr.u32 fa, ea, 24;\n shr.u32 fb, eb, 24;\n"                                          \
  " prmt.b32 ba, ea, 0, 0x4442;\n prmt.b32 bb, eb, 0, 0x4442;\n"                          \
  " mad.lo.u32 %0, fa, qa, ba;\n mad.lo.u32 %1, fb, qb, bb;\n"                            \
  " prmt.b32 %3, ea, eb, 0x5410;\n"                                                        \
  WS_RENORM_PTX("%0", "%1", "%4", "%7")                                                     \
  "}\n"

template <bool FIXED_BASE>
__device__ __forceinline__ void check_dict(uint32_t& xa, uint32_t& xb, uint32_t& rp, uint32_t tbase, uint32_t lba,
                                           uint32_t ltm, uint32_t& out0, uint32_t& out1) {
  if (FIXED_BASE)
    asm volatile(WS_CHECK_DICT_PTX("") : "+r"(xa), "+r"(xb), "=r"(out0), "=r"(out1), "+r"(rp)
                 : "r"(tbase), "r"(lba), "r"(ltm), "n"(kFixedTableBase));
  else
    asm volatile(WS_CHECK_DICT_PTX(WS_ADD_BASE_D) : "+r"(xa), "+r"(xb), "=r"(out0), "=r"(out1), "+r"(rp)
                 : "r"(tbase), "r"(lba), "r"(ltm), "n"(0));
}

// Generic-path dictionary step: state A decodes word j, state B word j + 1.
#define WS_DICT_STEP_C(ea, eb, va, vb)                                  \
  {                                                                     \
    if (va) {                                                           \
      ea = lds32(tb0 + ((xa & 255u) << 8));                             \
      xa = (ea >> 24) * (xa >> 8) + ((ea >> 16) & 255u);                \
    }                                                                   \
    if (vb) {                                                           \
      eb = lds32(tb0 + ((xb & 255u) << 8));                             \
      xb = (eb >> 24) * (xb >> 8) + ((eb >> 16) & 255u);                \
    }                                                                   \
  }

// Escape list of a dictionary block (WS_FLAG_ESCAPES), read by the lane that
// owns the listed words (8l..8l+7 of every group). Their stream symbol decodes
// as word 0, so when the decode reaches a group that holds the lane's next
// listed word, the listed residual is ORed into the (zero) decoded half before
// the apply: the word is written once, in its group's pass, and the checksum
// covers it. `w` is the next listed word (0xFFFFFFFF when none is left).
struct EscapeCursor {
  const uint32_t* next = nullptr;
  uint32_t left = 0;
  uint32_t w = 0xFFFFFFFFu, y = 0;
  bool bad = false;

  // Reads the lane counts (global, so the latency overlaps the first ring copy)
  // and the lane's first entry; the list starts `raw_bytes` (a split-word
  // block's raw section) after the stream. A list that does not fit the payload is bad.
  __device__ __forceinline__ void open(const ws_block_desc& bd, const uint8_t* __restrict__ src, uint32_t lane,
                                       uint32_t raw_bytes) {
    const uint32_t side = ((2u * bd.nwords + 15u) & ~15u) + raw_bytes;
    bad = side + WS_ESCAPE_HEADER_BYTES > bd.clen;
    uint32_t mine = 0, incl = 0;
    if (!bad) mine = reinterpret_cast<const uint16_t*>(src + side)[lane];
    incl = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t t = __shfl_up_sync(0xFFFFFFFFu, incl, o);
      if (lane >= (uint32_t)o) incl += t;
    }
    const uint32_t total = __shfl_sync(0xFFFFFFFFu, incl, 31);
    bad = __any_sync(0xFFFFFFFFu, bad) || side + WS_ESCAPE_HEADER_BYTES + 4ull * total > bd.clen;
    if (bad) return;
    next = reinterpret_cast<const uint32_t*>(src + side + WS_ESCAPE_HEADER_BYTES) + (incl - mine);
    left = mine;
    advance();
  }
  __device__ __forceinline__ void advance() {
    if (left) {
      const uint32_t e = *next++;
      --left;
      w = e & 0xFFFFu;
      y = e >> 16;
    } else {
      w = 0xFFFFFFFFu;
    }
  }
  // ORs every listed word of group g into the lane's residual pairs r0..r3.
  __device__ __forceinline__ void patch(uint32_t g, uint32_t lane, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
    const uint32_t base = g * WS_GROUP_WORDS + lane * WS_WORDS_PER_LANE;
    while (w < (g + 1) * WS_GROUP_WORDS) {
      const uint32_t j = w - base;  // the lane's word j of this group; out of order or not owned: j >= 8
      if (j < 8) {
        const uint32_t add = y << (16u * (j & 1u));
        if (j < 2) r0 |= add; else if (j < 4) r1 |= add; else if (j < 6) r2 |= add; else r3 |= add;
      } else {
        bad = true;
      }
      advance();
    }
  }
};

// Split-word blocks (K = 1, 2, 4 raw bits per word; dictionary kinds only): the
// low bits of each word come from the raw section after the stream
// (WS_FLAG_SPLIT_MASK layout in ws_format.h), read with plain cached loads. One
// uint32 per lane covers 4 / K groups; a group's raw bits are K whole bytes, and
// each byte is expanded through the tile's 256-entry table into the bits of the
// word pairs it covers, so a group costs K byte selects (PRMT) and K shared
// loads, and the bits join the residual in the apply's existing XOR.
template <uint32_t K>
struct SplitRaw {
  uint32_t off = 0;  // byte offset of the lane's first raw word in the payload

  // The raw word holding group g's bits.
  __device__ __forceinline__ uint32_t load(const uint8_t* __restrict__ src, uint32_t g) const {
    return __ldg(reinterpret_cast<const uint32_t*>(src + off) + ((g * K) >> 2) * WS_LANES);
  }
  // The raw-bit contributions e0..e3 to the lane's word pairs of group g.
  __device__ __forceinline__ void bits(uint32_t rw, uint32_t g, uint32_t& e0, uint32_t& e1, uint32_t& e2,
                                       uint32_t& e3) const {
    extern __shared__ __align__(1024) uint8_t smem[];
    const uint8_t* tab = smem + kSplitTabOffset;
    if (K == 1) {
      const uint32_t b = prmt(rw, 0, 0x4440u | (g & 3u));
      const uint4 e = reinterpret_cast<const uint4*>(tab)[b];
      e0 = e.x, e1 = e.y, e2 = e.z, e3 = e.w;
    } else if (K == 2) {
      const uint32_t c = (g & 1u) * 2u;
      const uint2 lo = reinterpret_cast<const uint2*>(tab)[prmt(rw, 0, 0x4440u | c)];
      const uint2 hi = reinterpret_cast<const uint2*>(tab)[prmt(rw, 0, 0x4440u | (c + 1u))];
      e0 = lo.x, e1 = lo.y, e2 = hi.x, e3 = hi.y;
    } else {
      const uint32_t* t = reinterpret_cast<const uint32_t*>(tab);
      e0 = t[prmt(rw, 0, 0x4440u)];
      e1 = t[prmt(rw, 0, 0x4441u)];
      e2 = t[prmt(rw, 0, 0x4442u)];
      e3 = t[prmt(rw, 0, 0x4443u)];
    }
  }
};

// Thread t < 256 writes entry t of the expansion table for K raw bits per word.
__device__ __forceinline__ void build_split_table(uint32_t k, uint32_t t) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* tab = smem + kSplitTabOffset;
  auto pair = [&](uint32_t lo, uint32_t hi) { return lo | (hi << 16); };
  if (k == 1) {
    reinterpret_cast<uint4*>(tab)[t] = make_uint4(pair(t & 1u, (t >> 1) & 1u), pair((t >> 2) & 1u, (t >> 3) & 1u),
                                                  pair((t >> 4) & 1u, (t >> 5) & 1u), pair((t >> 6) & 1u, t >> 7));
  } else if (k == 2) {
    reinterpret_cast<uint2*>(tab)[t] = make_uint2(pair(t & 3u, (t >> 2) & 3u), pair((t >> 4) & 3u, t >> 6));
  } else {
    reinterpret_cast<uint32_t*>(tab)[t] = pair(t & 15u, t >> 4);
  }
}

template <bool U16, bool REVERSE, bool DICT, bool FIXED_BASE, uint32_t SPLITK = 0>
__device__ void ans_block(const ws_block_desc& bd, uint32_t block, const uint8_t* __restrict__ src, uint32_t tbase,
                          uint8_t* ring, uint32_t bar_base, uint32_t lane, ws_device_result* res) {
  static_assert(DICT || SPLITK == 0, "only word-dictionary blocks split words");
  constexpr bool SPLIT = SPLITK != 0;
  uint8_t* dst = reinterpret_cast<uint8_t*>(bd.dst);
  const uint32_t n = bd.nbytes;
  const uint32_t W = n / 2;
  const uint32_t coded_bytes = 2 * W;
  const uint32_t dec_groups = (W + WS_GROUP_WORDS - 1) / WS_GROUP_WORDS;
  const uint32_t groups = (n + WS_GROUP_BYTES - 1) / WS_GROUP_BYTES;
  const bool aligned = (bd.dst & 15u) == 0;
  const uint32_t stream_bytes = (2u * bd.nwords + 15u) & ~15u;
  SplitRaw<SPLIT ? SPLITK : 1u> split;
  uint32_t raw_bytes = 0;
  if (SPLIT) {
    raw_bytes = ws_split_raw_bytes(W, SPLITK);
    // The raw section must lie inside the payload; nothing is read or written otherwise.
    if ((uint64_t)stream_bytes + raw_bytes > bd.clen) {
      if (lane == 0) report(res, WS_DEVERR_LENGTH, block);
      return;
    }
    split.off = stream_bytes + 4u * lane;
  }
  // Only the stream goes through the ring; a raw section and an escape list are
  // read from global memory.
  const uint32_t staged =
      (DICT && (bd.flags & (WS_FLAG_ESCAPES | WS_FLAG_SPLIT_MASK))) ? min(bd.clen, stream_bytes) : bd.clen;
  const uint32_t total_halves = (staged + WS_RING_HALF_BYTES - 1) / WS_RING_HALF_BYTES;
  const uint32_t ring_s = smem_addr(ring);
  const uint32_t ltm = lanemask_lt();
  const uint32_t lba = lane * 4u, lbb = lane * 4u + kRowBytes / 2;  // row offsets of planes 0 and 1
  const uint32_t tb0 = tbase + lba, tb1 = tbase + lbb;

  // Half k of the payload goes to ring slot k & 1; even halves also refresh the
  // mirror behind the ring end. Both copies complete on the slot's mbarrier.
  auto issue = [&](uint32_t k) {
    if (lane == 0 && k < total_halves) {
      const uint32_t off = k * WS_RING_HALF_BYTES;
      const uint32_t bytes = min(WS_RING_HALF_BYTES, staged - off);
      const uint32_t bar = bar_base + (k & 1u) * 8u;
      if (k & 1u) {
        bulk_load(ring_s + WS_RING_HALF_BYTES, src + off, bytes, bar);
      } else {
        const uint32_t mirror = min(kMirror, bytes);
        bulk_load2(ring_s, ring_s + WS_RING_BYTES, src + off, bytes, mirror, bar);
      }
    }
  };
  uint32_t issued = min(2u, total_halves);
  issue(0);
  issue(1);
  EscapeCursor esc;
  if (DICT && (bd.flags & WS_FLAG_ESCAPES)) esc.open(bd, src, lane, raw_bytes);
  uint32_t ready = 0;
  bool ok = true;
  if (total_halves > 0) {
    ok = mbar_wait(bar_base, 0);
    ready = 1;
  }
  uint32_t xa = reinterpret_cast<const uint32_t*>(ring)[lane];
  uint32_t xb = reinterpret_cast<const uint32_t*>(ring)[32 + lane];
  uint32_t pos = WS_HEADER_HALFWORDS;
  Checksum ck;

  // Recycle the slot whose half has been consumed, then make sure every
  // halfword the next group can read ([pos, pos + 256)) has landed.
  auto stage = [&]() {
    while (issued < total_halves && pos >= kHalfHalfwords * (issued - 1)) {
      __syncwarp();
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue(issued);
      ++issued;
    }
    const uint32_t need = min(pos + 256u, bd.nwords);
    while (ready < issued && need > kHalfHalfwords * ready) {
      ok = mbar_wait(bar_base + (ready & 1u) * 8u, (ready >> 1) & 1u);
      if (!ok) return;
      ++ready;
    }
  };

  // Fast path: full 512-byte groups of a 16-byte-aligned destination. The ring
  // bookkeeping runs only when the stream position reaches `next_event`.
  uint32_t g = 0;
  const uint32_t fast_groups = aligned ? W / WS_GROUP_WORDS : 0;
  uint32_t next_event = 0;
  auto at_event = [&]() {
    stage();
    const uint32_t recycle = issued < total_halves ? kHalfHalfwords * (issued - 1) : 0xFFFFFFFFu;
    const uint32_t wait =
        (ready < issued && bd.nwords > kHalfHalfwords * ready) ? kHalfHalfwords * ready - 255u : 0xFFFFFFFFu;
    next_event = min(recycle, wait);
    return ok;
  };
  // The lane's word pairs r0..r3 of group `grp` applied to the destination
  // vector `old` (escaped words patched in first) and written back.
  // A split block's raw bits (e0..e3, from raw word rw) fill the zero low bits
  // of the decoded words, so they join with the same XOR.
  auto finish = [&](uint4* q, uint4 old, uint32_t grp, uint32_t rw, uint32_t r0, uint32_t r1, uint32_t r2,
                    uint32_t r3) {
    uint32_t e0 = 0, e1 = 0, e2 = 0, e3 = 0;
    if (SPLIT) split.bits(rw, grp, e0, e1, e2, e3);
    if (DICT && esc.w < (grp + 1) * WS_GROUP_WORDS) esc.patch(grp, lane, r0, r1, r2, r3);
    uint4 v;
    if (U16) {
      v.x = u16_apply(old.x, r0 ^ e0, REVERSE);
      v.y = u16_apply(old.y, r1 ^ e1, REVERSE);
      v.z = u16_apply(old.z, r2 ^ e2, REVERSE);
      v.w = u16_apply(old.w, r3 ^ e3, REVERSE);
    } else {
      v.x = old.x ^ r0 ^ e0;
      v.y = old.y ^ r1 ^ e1;
      v.z = old.z ^ r2 ^ e2;
      v.w = old.w ^ r3 ^ e3;
    }
    *q = v;
    ck.add(v.x, v.y, v.z, v.w);
  };
  uint4* p = reinterpret_cast<uint4*>(dst + lane * 16u);
  if (DICT) {
    // Dictionary blocks (HBM-bound at one symbol per word) run two groups per
    // iteration: both destination vectors are loaded first, so ~200
    // instructions of decode hide their latency, and lane 0 asks the TMA unit
    // to pull the groups kPrefetchGroups ahead into L2. The per-iteration
    // bookkeeping (ring events, stream position, prefetch) is paid once per
    // 1 KiB; two groups read at most 256 stream words, which the staging
    // guarantees at each event.
    if (lane == 0 && fast_groups > 2) prefetch_l2(dst + 2 * WS_GROUP_BYTES, min(kPrefetchGroups, fast_groups - 2) * WS_GROUP_BYTES);
#pragma unroll 1
    for (; g + 2 <= fast_groups; g += 2, p += 2 * WS_GROUP_BYTES / 16) {
      if (pos >= next_event && !at_event()) break;
      const uint4 old0 = ldg128_early(p);
      const uint4 old1 = ldg128_early(p + WS_GROUP_BYTES / 16);
      // g is even: for K = 1, 2 groups g and g + 1 share a raw word.
      const uint32_t rw0 = SPLIT ? split.load(src, g) : 0u;
      const uint32_t rw1 = SPLITK == 4 ? split.load(src, g + 1) : rw0;
      if (lane == 0 && g + 2 + kPrefetchGroups + 2 <= fast_groups)
        prefetch_l2(dst + (g + 2 + kPrefetchGroups) * WS_GROUP_BYTES, 2 * WS_GROUP_BYTES);
      uint32_t rp = ring_s + (pos & (kRingHalfwords - 1)) * 2u;
      const uint32_t rp0 = rp;
      uint32_t r0, r1, r2, r3;
      check_dict<FIXED_BASE>(xa, xb, rp, tbase, lba, ltm, r0, r1);
      check_dict<FIXED_BASE>(xa, xb, rp, tbase, lba, ltm, r2, r3);
      finish(p, old0, g, rw0, r0, r1, r2, r3);
      check_dict<FIXED_BASE>(xa, xb, rp, tbase, lba, ltm, r0, r1);
      check_dict<FIXED_BASE>(xa, xb, rp, tbase, lba, ltm, r2, r3);
      finish(p + WS_GROUP_BYTES / 16, old1, g + 1, rw1, r0, r1, r2, r3);
      pos += (rp - rp0) >> 1;
    }
  }
  // Byte-plane blocks (bound by instruction issue at two symbols per word)
  // run one group per iteration with a plain load: the group's four checks
  // hide its latency. A dictionary block's odd last full group also runs here.
#pragma unroll 1
  for (; ok && g < fast_groups; ++g, p += WS_GROUP_BYTES / 16) {
    if (pos >= next_event && !at_event()) break;
    const uint4 old = DICT ? ldg128_early(p) : *p;
    const uint32_t rw = SPLIT ? split.load(src, g) : 0u;
    uint32_t rp = ring_s + (pos & (kRingHalfwords - 1)) * 2u;
    const uint32_t rp0 = rp;
    uint32_t r0, r1, r2, r3;
    if (DICT) {
      check_dict<FIXED_BASE>(xa, xb, rp, tbase, lba, ltm, r0, r1);
      check_dict<FIXED_BASE>(xa, xb, rp, tbase, lba, ltm, r2, r3);
    } else {
      r0 = check_fast<FIXED_BASE>(xa, xb, rp, tbase, lba, lbb, ltm);
      r1 = check_fast<FIXED_BASE>(xa, xb, rp, tbase, lba, lbb, ltm);
      r2 = check_fast<FIXED_BASE>(xa, xb, rp, tbase, lba, lbb, ltm);
      r3 = check_fast<FIXED_BASE>(xa, xb, rp, tbase, lba, lbb, ltm);
    }
    pos += (rp - rp0) >> 1;
    finish(p, old, g, rw, r0, r1, r2, r3);
  }

  // Generic path: the partial last group, the uncoded odd tail byte, and
  // destinations that are not 16-byte aligned.
#pragma unroll 1
  for (; g < groups && ok; ++g) {
    const uint32_t off = g * WS_GROUP_BYTES + lane * 16u;
    uint32_t r[4] = {0, 0, 0, 0};
    if (g < dec_groups) {
      stage();
      if (!ok) break;
      const int first = (int)(g * WS_GROUP_WORDS + lane * WS_WORDS_PER_LANE);
      const int valid = max(0, min(8, (int)W - first));
      uint32_t ea0, eb0, ea1, eb1;
      if (DICT) {
#pragma unroll
        for (int c = 0; c < 2; ++c) {
#pragma unroll
          for (int k = 0; k < 2; ++k) {
            const int j = 4 * c + 2 * k;
            ea0 = eb0 = 0;
            WS_DICT_STEP_C(ea0, eb0, j < valid, j + 1 < valid);
            r[2 * c + k] = __byte_perm(ea0, eb0, 0x5410);
          }
          WS_RENORM_C();
        }
      } else {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          ea0 = eb0 = ea1 = eb1 = 0;
          if (2 * c < valid) WS_STEP_C(ea0, eb0);
          if (2 * c + 1 < valid) WS_STEP_C(ea1, eb1);
          r[c] = __byte_perm(__byte_perm(ea0, eb0, 0x0051), __byte_perm(ea1, eb1, 0x5100), 0x7610);
          WS_RENORM_C();
        }
      }
    }
    uint32_t out[4] = {0, 0, 0, 0};
    if (SPLIT && g < dec_groups) {
      uint32_t e[4];
      split.bits(split.load(src, g), g, e[0], e[1], e[2], e[3]);
      for (int q = 0; q < 4; ++q) r[q] |= e[q];
    }
    if (DICT && g < dec_groups) esc.patch(g, lane, r[0], r[1], r[2], r[3]);
    apply_chunk_bytes<U16, REVERSE>(dst + off, off, n, r, coded_bytes, bd.tail, out);
    ck.add(out[0], out[1], out[2], out[3]);
  }
  if (!ok) {
    if (lane == 0) report(res, WS_DEVERR_TIMEOUT, block);
  } else {
    const bool states_ok = __all_sync(0xFFFFFFFFu, xa == WS_RANS_L && xb == WS_RANS_L);
    // Every listed word must have been consumed, in order, by its owner.
    const bool escapes_ok = !DICT || !__any_sync(0xFFFFFFFFu, esc.bad || esc.w != 0xFFFFFFFFu);
    if (lane == 0) {
      if (!states_ok) report(res, WS_DEVERR_STATE, block);
      if (pos != bd.nwords || !escapes_ok) report(res, WS_DEVERR_LENGTH, block);
    }
  }
  // Never leave a bulk copy in flight into shared memory of an exiting CTA: the
  // copies still outstanding (possible only after a timeout) get up to
  // kDrainRounds further bounded waits in all. A copy from this GPU's own memory
  // that has not landed after all of them means the memory system stopped
  // answering.
  for (uint32_t round = 0; ready < issued && round < kDrainRounds;) {
    if (mbar_wait(bar_base + (ready & 1u) * 8u, (ready >> 1) & 1u)) {
      ++ready;
    } else {
      ++round;
      if (lane == 0) report(res, WS_DEVERR_TIMEOUT, block);
    }
  }
  ck.finish(lane, block, res);
}

// A word-dictionary block, by its split code (0: whole words; else the code
// the tile's raw-bit table was built for).
// Which tiles a kernel instantiation decodes: tiles without split-word blocks
// (kWholeTiles), tiles of a packet that splits words (kSplitTiles), or both
// (kAnyTiles, the allocation-free entry point, whose tiles the host cannot
// see). Keeping the split decoders out of the whole-word kernel keeps its
// register allocation free of their spills.
enum TileMode : int { kWholeTiles = 0, kSplitTiles = 1, kAnyTiles = 2 };

template <bool U16, bool REVERSE, bool FIXED_BASE, int MODE>
__device__ __forceinline__ void dict_block(const ws_block_desc& bd, uint32_t block, const uint8_t* __restrict__ src,
                                           uint32_t tbase, uint8_t* ring, uint32_t bar_base, uint32_t lane,
                                           ws_device_result* res, uint32_t tile_split) {
  const uint32_t code = (bd.flags & WS_FLAG_SPLIT_MASK) >> WS_FLAG_SPLIT_SHIFT;
  if (code != tile_split) {  // the tile's expansion table is for another k (or none)
    if (lane == 0) report(res, WS_DEVERR_KIND, block);
  } else if (code == 0) {
    if constexpr (MODE != kSplitTiles) ans_block<U16, REVERSE, true, FIXED_BASE>(bd, block, src, tbase, ring, bar_base, lane, res);
  } else if constexpr (MODE != kWholeTiles) {
    if (code == 1)
      ans_block<U16, REVERSE, true, FIXED_BASE, 1>(bd, block, src, tbase, ring, bar_base, lane, res);
    else if (code == 2)
      ans_block<U16, REVERSE, true, FIXED_BASE, 2>(bd, block, src, tbase, ring, bar_base, lane, res);
    else
      ans_block<U16, REVERSE, true, FIXED_BASE, 4>(bd, block, src, tbase, ring, bar_base, lane, res);
  }
}

// One block by its kind. FIXED_BASE: the table region starts at the shared
// address kFixedTableBase, which the lookups then take as an immediate offset.
template <bool REVERSE, bool FIXED_BASE, int MODE>
__device__ __forceinline__ void run_block(const ws_block_desc& bd, uint32_t block, const uint8_t* __restrict__ src,
                                          uint32_t tbase, uint8_t* ring, uint32_t bar_base, uint32_t lane,
                                          ws_device_result* res, uint32_t tile_split) {
  switch (bd.kind) {
    case WS_KIND_RAW:
      raw_block(bd, block, src, lane, res);
      break;
    case WS_KIND_ANS_XOR:
    case WS_KIND_ANS_U16:
      // Byte planes never split words, and a packet that splits words has none.
      if ((bd.flags & WS_FLAG_SPLIT_MASK) || tile_split != 0) {
        if (lane == 0) report(res, WS_DEVERR_KIND, block);
      } else if constexpr (MODE != kSplitTiles) {
        if (bd.kind == WS_KIND_ANS_XOR)
          ans_block<false, REVERSE, false, FIXED_BASE>(bd, block, src, tbase, ring, bar_base, lane, res);
        else
          ans_block<true, REVERSE, false, FIXED_BASE>(bd, block, src, tbase, ring, bar_base, lane, res);
      }
      break;
    case WS_KIND_DICT_XOR:
      dict_block<false, REVERSE, FIXED_BASE, MODE>(bd, block, src, tbase, ring, bar_base, lane, res, tile_split);
      break;
    case WS_KIND_DICT_U16:
      dict_block<true, REVERSE, FIXED_BASE, MODE>(bd, block, src, tbase, ring, bar_base, lane, res, tile_split);
      break;
    default:
      if (lane == 0) report(res, WS_DEVERR_KIND, block);
  }
}

// Bounds of the caller-owned arrays an allocation-free apply receives. The
// plan-based apply builds its descriptors itself and runs unchecked.
struct DescLimits {
  uint32_t nblocks;
  uint32_t ntables;
  uint64_t payload_bytes;
};

// A block descriptor the kernel can follow without leaving the payload: a
// 16-byte-aligned payload range inside the caller's arena (cp.async.bulk needs
// 16-byte alignment), 1..WS_BLOCK_BYTES weight bytes, a known kind, and a raw payload
// that holds every weight byte it XORs.
__device__ __forceinline__ bool block_in_bounds(const ws_block_desc& bd, uint64_t payload_bytes) {
  return (bd.src & 15u) == 0 && (bd.clen & 15u) == 0 && bd.src <= payload_bytes &&
         bd.clen <= payload_bytes - bd.src && bd.nbytes >= 1 && bd.nbytes <= WS_BLOCK_BYTES &&
         bd.kind <= WS_KIND_DICT_U16 && (bd.kind != WS_KIND_RAW || bd.nbytes <= bd.clen);
}

// The per-tile work shared by both apply kernels: expand the packet's tables
// into the lane replicas, set up each warp's staging barriers, then one warp
// per block of the tile. `payload` is the device address of arena byte
// `payload_offset`. With CHECKED, every descriptor is first checked against
// `lim`; one that points outside the caller's arrays is reported as
// WS_DEVERR_BOUNDS and not followed.
template <bool REVERSE, bool CHECKED, int MODE>
__device__ __forceinline__ void apply_tile(const ws_tile_desc& tile, const ws_block_desc* __restrict__ blocks,
                                           const uint32_t* __restrict__ tables, const uint8_t* __restrict__ payload,
                                           uint64_t payload_offset, ws_device_result* res, DescLimits lim) {
  extern __shared__ __align__(1024) uint8_t smem[];
  // The host picks the instantiation from the tiles' kinds; a tile of the other
  // kind is reported, not decoded.
  if (MODE != kAnyTiles && (tile.split != 0) != (MODE == kSplitTiles)) {
    if (threadIdx.x == 0) report(res, WS_DEVERR_KIND, tile.first_block);
    return;
  }
  uint32_t* tbl = reinterpret_cast<uint32_t*>(smem);
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  if (CHECKED) {
    // Uniform over the CTA: either every thread returns here or none does.
    const bool tile_ok = tile.nblocks <= kWarps && (uint64_t)tile.first_block + tile.nblocks <= lim.nblocks &&
                         (tile.table == WS_NO_TABLE || tile.table < lim.ntables) && tile.split <= 3;
    if (!tile_ok) {
      if (threadIdx.x == 0) report(res, WS_DEVERR_BOUNDS, tile.first_block);
      return;
    }
  }
  if (tile.table != WS_NO_TABLE) {
    // Thread t expands slot entry t (plane t >> 8) into its 32 replicas; the
    // rotated segment order keeps 8 consecutive threads on distinct banks.
    const uint32_t t = threadIdx.x;
    const uint32_t e = __ldg(tables + (uint64_t)tile.table * 512u + t);
    const uint4 v = make_uint4(e, e, e, e);
    uint4* row = reinterpret_cast<uint4*>(tbl + (t & 255u) * (kRowBytes / 4) + (t >> 8) * 32u);
#pragma unroll
    for (uint32_t k = 0; k < 8; ++k) row[(k + t) & 7u] = v;
  }
  if (tile.split != 0 && threadIdx.x < 256) build_split_table(ws_split_bits(tile.split << WS_FLAG_SPLIT_SHIFT), threadIdx.x);
  const uint32_t bar_base = smem_addr(smem + kBarOffset) + warp * 16u;
  if (lane == 0) {
    mbar_init(bar_base, 1);
    mbar_init(bar_base + 8, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (warp >= tile.nblocks) return;
  const uint32_t block = tile.first_block + warp;
  const ws_block_desc bd = blocks[block];
  if (CHECKED && (!block_in_bounds(bd, lim.payload_bytes) || (bd.kind != WS_KIND_RAW && tile.table == WS_NO_TABLE))) {
    if (lane == 0) report(res, WS_DEVERR_BOUNDS, block);
    return;
  }
  const uint8_t* src = payload + (bd.src - payload_offset);
  uint8_t* ring = smem + kRingOffset + warp * kRingStride;
  const uint32_t tbase = smem_addr(tbl);
  if (tbase == kFixedTableBase)
    run_block<REVERSE, true, MODE>(bd, block, src, tbase, ring, bar_base, lane, res, tile.split);
  else
    run_block<REVERSE, false, MODE>(bd, block, src, tbase, ring, bar_base, lane, res, tile.split);
}

template <bool REVERSE, int MODE>
__global__ void __launch_bounds__(kThreads, 2)
    ws_apply_kernel(const ws_tile_desc* __restrict__ tiles, uint32_t tile_begin,
                    const ws_block_desc* __restrict__ blocks, const uint32_t* __restrict__ tables,
                    const uint8_t* __restrict__ payload, uint64_t payload_offset, ws_device_result* res) {
  apply_tile<REVERSE, false, MODE>(tiles[tile_begin + blockIdx.x], blocks, tables, payload, payload_offset, res,
                                   DescLimits{});
}

}  // namespace

size_t apply_smem_bytes() { return kSmemBytes; }

using ApplyKernel = void (*)(const ws_tile_desc*, uint32_t, const ws_block_desc*, const uint32_t*, const uint8_t*,
                             uint64_t, ws_device_result*);

// The instantiation for a launch range holding the given tile kinds: whole-word
// tiles only, split-word tiles only, or both (one kernel that decodes either).
ApplyKernel apply_kernel(int reverse, uint32_t kinds) {
  if (kinds == kTilesWhole) return reverse ? ws_apply_kernel<true, kWholeTiles> : ws_apply_kernel<false, kWholeTiles>;
  if (kinds == kTilesSplit) return reverse ? ws_apply_kernel<true, kSplitTiles> : ws_apply_kernel<false, kSplitTiles>;
  return reverse ? ws_apply_kernel<true, kAnyTiles> : ws_apply_kernel<false, kAnyTiles>;
}

cudaError_t prime_kernels() {
  // Loads every kernel instantiation (lazy module loading) and sets its
  // shared-memory limit, so the first apply of each direction pays nothing.
  cudaError_t e = cudaSuccess;
  for (int reverse = 0; reverse < 2 && e == cudaSuccess; ++reverse)
    for (uint32_t kinds = 1; kinds <= 3 && e == cudaSuccess; ++kinds)
      e = cudaFuncSetAttribute(apply_kernel(reverse, kinds), cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)kSmemBytes);
  return e;
}

cudaError_t launch_apply(const ws_tile_desc* tiles, uint32_t tile_begin, uint32_t ntiles,
                         const ws_block_desc* blocks, const uint32_t* tables, const uint8_t* payload,
                         uint64_t payload_offset, ws_device_result* result, int reverse, uint32_t kinds,
                         cudaStream_t stream, uint32_t* launched) {
  if (ntiles == 0) return cudaSuccess;
  const ApplyKernel kernel = apply_kernel(reverse, kinds);
  // Set on every launch: the attribute is per device context and costs ~1 us.
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
  if (e != cudaSuccess) return e;
  kernel<<<ntiles, kThreads, kSmemBytes, stream>>>(tiles, tile_begin, blocks, tables, payload, payload_offset,
                                                     result);
  e = cudaGetLastError();
  if (e == cudaSuccess && launched) ++*launched;
  return e;
}

}  // namespace ws

// ---------------------------------------------------------------------------
// Allocation-free apply (ws_apply_device_noalloc in include/warpshift_b200.h).
//
// Some callers cannot let a library call cudaMalloc at switch time: a serving
// engine that has already handed all free HBM to its KV-cache pool, or one that
// owns every device allocation through its own allocator. This entry point
// takes descriptors, tables and payload that the caller already placed in
// device memory, writes the weights in place, and keeps its only scratch (one
// result slot per tile plus one total) in the fixed array below, which every
// GPU that loads this library holds until the process exits.
#include <mutex>
#include <string>

#include "../../include/warpshift_b200.h"

static __device__ __align__(256) ws_device_result g_noalloc_scratch[WS_NOALLOC_MAX_TILES + 1];

namespace ws {
namespace {

// Same per-tile work as ws_apply_kernel, with every caller-written descriptor
// checked against the caller's array sizes; each tile accumulates into its own
// scratch slot (slot = tile index) instead of one shared accumulator.
template <bool REVERSE>
__global__ void __launch_bounds__(kThreads, 2)
    ws_apply_noalloc_kernel(const ws_tile_desc* __restrict__ tiles, const ws_block_desc* __restrict__ blocks,
                            const uint32_t* __restrict__ tables, const uint8_t* __restrict__ payload,
                            DescLimits lim, ws_device_result* scratch) {
  apply_tile<REVERSE, true, kAnyTiles>(tiles[blockIdx.x], blocks, tables, payload, 0, scratch + blockIdx.x, lim);
}

// Sums the per-tile slots [0, n) into slot WS_NOALLOC_MAX_TILES (one CTA).
__global__ void ws_noalloc_reduce_kernel(ws_device_result* scratch, uint32_t n) {
  __shared__ unsigned long long sum[256];
  __shared__ uint32_t err[256], bad[256];
  unsigned long long s = 0;
  uint32_t e = 0, b = 0;
  for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
    s += scratch[i].checksum;
    e |= scratch[i].errors;
    if (scratch[i].bad_block_plus1) b = scratch[i].bad_block_plus1;
  }
  sum[threadIdx.x] = s;
  err[threadIdx.x] = e;
  bad[threadIdx.x] = b;
  __syncthreads();
  for (uint32_t stride = blockDim.x / 2; stride > 0; stride >>= 1) {
    if (threadIdx.x < stride) {
      sum[threadIdx.x] += sum[threadIdx.x + stride];
      err[threadIdx.x] |= err[threadIdx.x + stride];
      if (!bad[threadIdx.x]) bad[threadIdx.x] = bad[threadIdx.x + stride];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    scratch[WS_NOALLOC_MAX_TILES].checksum = sum[0];
    scratch[WS_NOALLOC_MAX_TILES].errors = err[0];
    scratch[WS_NOALLOC_MAX_TILES].bad_block_plus1 = bad[0];
  }
}

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mutex;
ws_device_result* g_noalloc_ptr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on `device` (which must be current).
// Host code cannot use the symbol itself: it names a host-side shadow. The
// first call on a device also loads every kernel a later call launches (both
// directions and the reduction) and sets their shared-memory limit: with lazy
// module loading a kernel is otherwise loaded, and memory for it allocated, at
// its first launch, which may be a later call.
int noalloc_scratch(int device, ws_device_result** out) {
  std::lock_guard<std::mutex> lk(g_noalloc_mutex);
  if (!g_noalloc_ptr[device]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    cudaFuncAttributes attr;
    for (const void* f : {(const void*)ws_apply_noalloc_kernel<true>, (const void*)ws_apply_noalloc_kernel<false>}) {
      if (e == cudaSuccess) e = cudaFuncGetAttributes(&attr, f);
      if (e == cudaSuccess) e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
    }
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&attr, (const void*)ws_noalloc_reduce_kernel);
    if (e != cudaSuccess) {
      set_last_error((std::string("no-alloc set-up: ") + cudaGetErrorString(e)).c_str());
      return WS_ERR_CUDA;
    }
    g_noalloc_ptr[device] = static_cast<ws_device_result*>(p);
  }
  *out = g_noalloc_ptr[device];
  return WS_OK;
}

}  // namespace
}  // namespace ws

static int ws_apply_device_noalloc_impl(const void* tiles, uint32_t ntiles, const void* blocks, uint32_t nblocks,
                                        const uint32_t* tables, uint32_t ntables, const void* payload,
                                        uint64_t payload_bytes, int reverse, int device, void* stream,
                                        ws_apply_result* out) {
  using namespace ws;
  auto reject = [](const std::string& why) {
    set_last_error(("ws_apply_device_noalloc: " + why).c_str());
    return WS_ERR_INVALID;
  };
  if (!out) return reject("null result pointer");
  *out = ws_apply_result{};
  if (ntiles == 0) return WS_OK;
  if (ntiles > WS_NOALLOC_MAX_TILES)
    return reject(std::to_string(ntiles) + " tiles exceed the maximum of " + std::to_string(WS_NOALLOC_MAX_TILES) +
                  " per call (its per-tile results live in a fixed device array); split the tiles over several calls");
  if (!tiles || !blocks || !payload || nblocks == 0 || payload_bytes == 0)
    return reject("null tile, block or payload array, or an empty block list or payload");
  if (ntables && !tables) return reject("null table array with ntables > 0");
  // cp.async.bulk stages payload bytes with 16-byte-aligned addresses; descriptors are read as 16-byte records.
  if (((uintptr_t)tiles & 15u) || ((uintptr_t)blocks & 15u) || ((uintptr_t)payload & 15u) || ((uintptr_t)tables & 3u))
    return reject("tiles, blocks and payload must be 16-byte aligned and tables 4-byte aligned");
  if (device < 0 || device >= kMaxDevices) return reject("bad device ordinal " + std::to_string(device));
  int prev = -1;
  cudaGetDevice(&prev);
  auto done = [&](int rc) {
    if (prev >= 0) cudaSetDevice(prev);
    return rc;
  };
  cudaError_t e = cudaSetDevice(device);
  ws_device_result* scratch = nullptr;
  if (e != cudaSuccess) {
    set_last_error((std::string("ws_apply_device_noalloc: ") + cudaGetErrorString(e)).c_str());
    return done(WS_ERR_CUDA);
  }
  int rc = noalloc_scratch(device, &scratch);
  if (rc != WS_OK) return done(rc);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto kernel = reverse ? ws_apply_noalloc_kernel<true> : ws_apply_noalloc_kernel<false>;
  // The slots used by this call start at zero; the array keeps the previous call's values otherwise.
  e = cudaMemsetAsync(scratch, 0, sizeof(ws_device_result) * ntiles, s);
  if (e == cudaSuccess) {
    kernel<<<ntiles, kThreads, kSmemBytes, s>>>(static_cast<const ws_tile_desc*>(tiles),
                                                 static_cast<const ws_block_desc*>(blocks), tables,
                                                 static_cast<const uint8_t*>(payload),
                                                 DescLimits{nblocks, ntables, payload_bytes}, scratch);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) {
    ws_noalloc_reduce_kernel<<<1, 256, 0, s>>>(scratch, ntiles);
    e = cudaGetLastError();
  }
  ws_device_result total{};
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(&total, scratch + WS_NOALLOC_MAX_TILES, sizeof(total), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) {
    set_last_error((std::string("ws_apply_device_noalloc: ") + cudaGetErrorString(e)).c_str());
    return done(WS_ERR_CUDA);
  }
  out->checksum = total.checksum;
  out->device_errors = total.errors;
  out->bad_block_plus1 = total.bad_block_plus1;
  out->launches = 2;
  if (total.errors) {
    set_last_error((total.errors & WS_DEVERR_BOUNDS)
                       ? "ws_apply_device_noalloc: a tile or block descriptor points outside the given arrays"
                       : "ws_apply_device_noalloc: device reported a corrupt block");
    return done(WS_ERR_DEVICE);
  }
  return done(WS_OK);
}

extern "C" WS_API int ws_apply_device_noalloc(const void* tiles, uint32_t ntiles, const void* blocks, uint32_t nblocks,
                                              const uint32_t* tables, uint32_t ntables, const void* payload,
                                              uint64_t payload_bytes, int reverse, int device, void* stream,
                                              ws_apply_result* out) {
  return ws::guarded([&] {
    return ws_apply_device_noalloc_impl(tiles, ntiles, blocks, nblocks, tables, ntables, payload, payload_bytes,
                                        reverse, device, stream, out);
  });
}

// ---------------------------------------------------------------------------
// Failure-path self-test (ws_selftest_wait_timeout in include/warpshift_b200.h).
// One warp waits, with the decode kernel's bounded wait, on a staging barrier
// that nothing ever arrives on: the wait gives up after `limit` polls and the
// warp reports WS_DEVERR_TIMEOUT through the usual result word, leaving no copy
// in flight, so the context stays usable. No fault, trap or endless loop.
namespace ws {
namespace {

__global__ void ws_wait_selftest_kernel(uint32_t limit, ws_device_result* res) {
  __shared__ __align__(8) uint64_t bar;
  const uint32_t b = smem_addr(&bar);
  if (threadIdx.x == 0) {
    mbar_init(b, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncwarp();
  if (!mbar_wait(b, 0, limit) && threadIdx.x == 0) report(res, WS_DEVERR_TIMEOUT, 0);
}

}  // namespace
}  // namespace ws

static int ws_selftest_wait_timeout_impl(uint32_t polls, int device, void* stream, uint32_t* device_errors) {
  using namespace ws;
  if (!device_errors || polls == 0 || polls > kWaitLimit) {
    set_last_error("ws_selftest_wait_timeout: need 1 <= polls <= 2^20 and a result pointer");
    return WS_ERR_INVALID;
  }
  int prev = -1;
  cudaGetDevice(&prev);
  cudaError_t e = cudaSetDevice(device);
  ws_device_result* d = nullptr;
  ws_device_result h{};
  cudaStream_t s = (cudaStream_t)stream;
  if (e == cudaSuccess) e = cudaMallocAsync((void**)&d, sizeof(ws_device_result), s);
  if (e == cudaSuccess) e = cudaMemsetAsync(d, 0, sizeof(ws_device_result), s);
  if (e == cudaSuccess) {
    ws_wait_selftest_kernel<<<1, 32, 0, s>>>(polls, d);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaMemcpyAsync(&h, d, sizeof(h), cudaMemcpyDeviceToHost, s);
  if (d) cudaFreeAsync(d, s);
  const cudaError_t es = cudaStreamSynchronize(s);
  if (e == cudaSuccess) e = es;
  if (prev >= 0) cudaSetDevice(prev);
  if (e != cudaSuccess) {
    set_last_error((std::string("ws_selftest_wait_timeout: ") + cudaGetErrorString(e)).c_str());
    return WS_ERR_CUDA;
  }
  *device_errors = h.errors;
  return WS_OK;
}

extern "C" WS_API int ws_selftest_wait_timeout(uint32_t polls, int device, void* stream, uint32_t* device_errors) {
  return ws::guarded([&] { return ws_selftest_wait_timeout_impl(polls, device, stream, device_errors); });
}
