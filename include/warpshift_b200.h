/*
 * warpshift_b200 C ABI: in-place BF16 model switching driven by an
 * entropy-coded delta stream, decoded and applied on B200 (sm_100a).
 *
 * The reference (DrRyanHuang/WarpShift) is pure Python. Its delta path is the
 * class warpshift/delta.py:95-327 DeltaWeights, whose prepare step encodes with
 * nvCOMP ANS and whose apply step runs nvCOMP's batched ANS decode followed by
 * the Triton kernel _restore_batch. These entry points replace that machinery;
 * warpshift_b200/delta.py binds them with ctypes behind the same Python API.
 *
 * Conventions: every function returns WS_OK (0) or a WS_ERR_* status, never
 * throws across the ABI, and records a message readable with ws_last_error()
 * on the calling thread. Streams are cudaStream_t passed as void*. No torch
 * types appear here; tensors are raw pointers plus byte counts.
 */
#ifndef WARPSHIFT_B200_H
#define WARPSHIFT_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define WS_API __attribute__((visibility("default")))
#else
#define WS_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define WS_OK 0
#define WS_ERR_INVALID 1  /* bad argument / layout (maps to ValueError, as delta.py:139-162) */
#define WS_ERR_CUDA 2     /* CUDA runtime failure */
#define WS_ERR_DEVICE 3   /* device-side decode error: corrupt frame, state or length mismatch */
#define WS_ERR_CHECKSUM 4 /* written bytes do not hash to the value recorded at prepare */
#define WS_ERR_NOMEM 5    /* host or device allocation failed */
#define WS_ERR_STATE 6    /* call out of order (e.g. apply before upload) */
#define WS_ERR_IO 7       /* file cannot be created, written or read (saved plans) */

#define WS_POLICY_AUTO 0 /* delta.py:176-194: raw XOR, else grouped/odd XOR-ANS, else U16-ANS if strictly smaller */
#define WS_POLICY_XOR 1  /* only XOR representations (modes 0/1/2) */
#define WS_POLICY_U16 2  /* BF16 packets try only U16-ANS (raw XOR if not smaller); others follow AUTO */

typedef struct ws_plan ws_plan;

/* One tensor of the A/B pair, in delta.py:147-158 order (gpu_target dict order). */
typedef struct ws_tensor_desc {
  const void* base;   /* host address of A's bytes (cpu_base tensor) */
  const void* target; /* B's bytes: device address on opts->device if target_on_device, else host */
  uint64_t nbytes;    /* tensor byte size (numel * element_size); may be 0 */
  int32_t is_bf16;    /* BF16 tensors may use the U16 mode (delta.py:190) */
  int32_t reserved;
} ws_tensor_desc;

typedef struct ws_build_options {
  int32_t policy;           /* WS_POLICY_* */
  int32_t threads;          /* host encoder threads; 0 = all online CPUs */
  int32_t target_on_device; /* 1: target pointers are device addresses (normal prepare) */
  int32_t device;           /* CUDA device ordinal of the targets */
  uint64_t batch_bytes;     /* bound on one H2D staging batch (0 = 64 MiB, delta.py:21) */
  int32_t staging_slots;    /* device staging buffers (0 = 3) */
  int32_t pin_arena;        /* 1: arena in pinned host memory (needs CUDA); 0: malloc */
  int32_t dict_slack_pct;   /* code a packet as one symbol per word (word dictionary) when its words
                               take <= 255 values and the estimated size is at most this many percent
                               above the byte-plane coding; negative: byte planes only */
  int32_t encode_on_device; /* 1 (with target_on_device): compute statistics and encode on the GPU,
                               copying only A host->device; 0: copy B device->host, encode on host threads */
  uint64_t encode_batch_bytes; /* GPU encoder: weight bytes encoded per device batch (0 = 512 MiB); the
                                  device holds up to about 4x this in temporary buffers during prepare */
  int32_t escapes;          /* word dictionaries with escapes (rare words listed after each block's
                               stream): 0 when estimated smaller, < 0 never, > 0 whenever eligible */
  int32_t host_fallback;    /* 1: when the GPU encoder cannot get its device buffers even with 32 MiB
                               batches, encode on host threads instead; 0 (default): fail with
                               WS_ERR_NOMEM */
  int32_t split;            /* split-word dictionaries (the low k = 1, 2 or 4 bits of every word
                               stored raw, the rest coded): 0 (default) the k estimated smallest,
                               a split one only when 3 % smaller than whole words (split blocks
                               decode more slowly); < 0 never; 1, 2 or 4: that k whenever eligible */
} ws_build_options;

typedef struct ws_plan_stats {
  uint64_t runtime_bytes;      /* sum of tensor bytes (delta.py:122) */
  uint64_t skipped_bytes;      /* bytes of all-zero 16 MiB packets (delta.py:211) */
  uint64_t zero_block_bytes;   /* bytes of all-zero 128 KiB blocks inside written packets */
  uint64_t touched_bytes;      /* weight bytes the kernel reads and writes per apply */
  uint64_t payload_bytes;      /* sum of packet payload sizes (delta.py:124) */
  uint64_t arena_bytes;        /* bytes staged host->device per apply (delta.py:125) */
  uint64_t table_bytes;        /* device decode tables */
  uint64_t metadata_bytes;     /* device block/tile descriptors + tables */
  uint64_t scratch_bytes;      /* device staging slots (+ resident copy when enabled) */
  uint64_t mode_counts[5];     /* packets per ws mode: XOR_RAW, XOR_GROUP2_ANS, XOR_ANS, U16_ANS, SKIP */
  uint64_t blocks, tiles, batches, packets;
  uint64_t expected_checksum[2]; /* [0] after forward (A->B), [1] after reverse (B->A) */
  double encode_seconds;
  uint32_t encoder;            /* WS_ENCODER_*: which path produced the plan */
  uint32_t reserved;
} ws_plan_stats;

#define WS_ENCODER_HOST 0   /* host threads (B copied device->host, or host targets) */
#define WS_ENCODER_GPU 1    /* GPU encoder */
#define WS_ENCODER_LOADED 2 /* ws_plan_load of a saved plan */

typedef struct ws_apply_result {
  uint64_t checksum;         /* checksum of the bytes written by this apply */
  uint64_t expected;         /* checksum recorded at prepare for this direction */
  uint32_t device_errors;    /* OR of device error bits (see ws_format.h WS_DEVERR_*) */
  uint32_t bad_block_plus1;  /* 1 + index of a failing block, 0 if none */
  uint64_t h2d_bytes;        /* bytes copied host->device by this apply */
  uint32_t launches;         /* decode kernel launches issued (a rollback's included) */
  uint32_t rollback;         /* WS_ROLLBACK_*: what ws_apply did after a failed switch */
} ws_apply_result;

#define WS_ROLLBACK_NONE 0       /* the switch succeeded, or no rollback was attempted */
#define WS_ROLLBACK_RESTORED 1   /* the inverse pass restored the source model (checksum verified) */
#define WS_ROLLBACK_UNVERIFIED 2 /* the inverse pass ran; its bytes do not hash to the source model's */
#define WS_ROLLBACK_FAILED 3     /* the inverse pass could not run or gave up: weights are undefined */

/* Host-side view of a built plan, for checkers and CPU baselines. */
typedef struct ws_plan_view {
  const void* blocks;     /* ws_block_desc[nblocks] (ws_format.h) */
  uint64_t nblocks;
  const void* tiles;      /* ws_tile_desc[ntiles] */
  uint64_t ntiles;
  const uint32_t* tables; /* 512 slot entries per packet table */
  uint64_t ntables;
  const uint8_t* arena;   /* host arena holding every block payload; when the plan keeps
                             its arena in several host chunks (GPU encoder: one per
                             encode_batch_bytes of weights), the first call makes one contiguous
                             copy that lives as long as the plan */
  uint64_t arena_bytes;
} ws_plan_view;

/* Library version (major*10000 + minor*100 + patch). */
WS_API int ws_version(void);

/* Copies the calling thread's last error message (NUL-terminated, truncated). */
WS_API int ws_last_error(char* buf, size_t len);

/* Replaces delta.py:26-34 _u16_residual: out = low-byte plane || high-byte plane of
 * zigzag((B - A) mod 2^16); nbytes must be even. Host only. */
WS_API int ws_u16_residual(const uint8_t* base, const uint8_t* target, uint64_t nbytes, uint8_t* out);

/* Replaces the prepare half of DeltaWeights.__init__ (delta.py:102-135: _bind_tensors'
 * overlap check 137-162, _encode_packets 196-216, _encode_chunk 176-194, _compress
 * 164-174, _prepare_batches/_pack_batch 218-280). With target_on_device and
 * encode_on_device, A is copied host->device in encode_batch_bytes batches (pageable A staged
 * through pinned buffers by up to `threads` host threads) and every packet is
 * encoded on the device on `stream`; the payloads come back into the host arena and
 * the temporary device buffers are freed before returning. If the device cannot
 * hold the encoder's buffers, the GPU encoder retries with batches 4x smaller (down
 * to 32 MiB); if that still fails, the build returns WS_ERR_NOMEM, or, only with
 * opts->host_fallback, hands over to the host encoder (ws_plan_stats.encoder says
 * which ran). Without encode_on_device, B is copied device->host in 16 MiB packets
 * and encoded on `threads` host threads. Both encoders produce byte-identical plans. */
WS_API int ws_plan_build(const ws_tensor_desc* tensors, uint64_t ntensors, const ws_build_options* opts,
                  void* stream, ws_plan** out);

/* Allocates device metadata and staging slots and uploads descriptors/tables
 * (the device half of delta.py:218-280). */
WS_API int ws_plan_upload(ws_plan* plan, void* stream);

/* resident=1 keeps a device copy of the whole arena so applies skip the H2D
 * staging (kernel-only timing); resident=0 frees it once the applies in flight
 * have completed. */
WS_API int ws_plan_set_resident(ws_plan* plan, int resident, void* stream);

/* Replaces DeltaWeights.apply (delta.py:294-327): A->B when reverse == 0, B->A when 1.
 * Stages the arena H2D on copy_stream in bounded batches (the first ones smaller),
 * decodes and applies the batches alternately on compute_stream and a second
 * stream of the plan that compute_stream joins at the end, reads back the device
 * result, and returns after compute_stream completes. Returns WS_ERR_DEVICE or
 * WS_ERR_CHECKSUM on failure, after rolling the switch back: the other direction
 * is applied over the same stream, which writes back exactly the bytes that were
 * resident, and the restored bytes are checked against the source model's
 * checksum; out->rollback and the error message say how that went. The
 * reference has no rollback (its server latches a failure, server.py:88-99). */
WS_API int ws_apply(ws_plan* plan, int reverse, void* compute_stream, void* copy_stream, ws_apply_result* out);

/* Asynchronous halves of ws_apply: enqueue only (no host synchronisation), then
 * wait for compute_stream and evaluate the result. ws_apply_async may be called
 * again on the same compute_stream before ws_apply_finish: the applies run in
 * stream order and ws_apply_finish reports the last one. */
WS_API int ws_apply_async(ws_plan* plan, int reverse, void* compute_stream, void* copy_stream);
WS_API int ws_apply_finish(ws_plan* plan, void* compute_stream, ws_apply_result* out);

WS_API int ws_plan_get_stats(const ws_plan* plan, ws_plan_stats* out);
WS_API int ws_plan_get_view(const ws_plan* plan, ws_plan_view* out);

/* No counterpart in the reference. Allocation-free apply for callers that cannot
 * let a library call cudaMalloc (an engine whose KV-cache pool already holds all
 * free HBM, or one that routes every device allocation through its own
 * allocator). The caller passes, in device memory on `device`, the tile and
 * block descriptors and slot tables of a plan (layouts of ws_plan_get_view) and
 * the whole payload arena (block `src` offsets are relative to `payload`), with
 * the element counts of each array and the arena's byte size. `tiles`, `blocks`
 * and `payload` must be 16-byte aligned and `tables` 4-byte aligned (else
 * WS_ERR_INVALID). On the device every tile and block descriptor is checked
 * against those sizes before it is followed (block range and table index of a
 * tile; payload range, 16-byte alignment, byte count and kind of a block): one
 * outside them is skipped and reported as device error WS_DEVERR_BOUNDS (16),
 * with the call returning WS_ERR_DEVICE. The weights named by the block
 * descriptors' `dst` are written in place; those addresses are the caller's
 * and cannot be checked. `out` receives the checksum and device errors
 * (`out->expected` stays 0: compare with ws_plan_stats.expected_checksum). Its
 * only scratch is a fixed 16-byte-per-tile device array of
 * WS_NOALLOC_MAX_TILES + 1 slots (256 KiB) inside the library, held by every
 * GPU that loads the library until exit; more than WS_NOALLOC_MAX_TILES tiles
 * per call is rejected with WS_ERR_INVALID. The first call on a device looks up
 * that array's device address and loads the entry point's kernels for both
 * directions (module set-up), so later calls allocate nothing, whatever
 * their direction. All calls on a device share the
 * array: calls that overlap on the GPU race and must be serialised by the
 * caller. The call is synchronous: it reads its result back to the host and
 * returns after `stream` completes, so it cannot be made while `stream` is
 * being captured into a CUDA graph. */
#define WS_NOALLOC_MAX_TILES 16384
WS_API int ws_apply_device_noalloc(const void* tiles, uint32_t ntiles, const void* blocks, uint32_t nblocks,
                                   const uint32_t* tables, uint32_t ntables, const void* payload,
                                   uint64_t payload_bytes, int reverse, int device, void* stream,
                                   ws_apply_result* out);

/* No counterpart in the reference, which prepares the delta again after every
 * restart (README.md:41). Writes a built plan to `path` (via `path`.tmp, then
 * rename): descriptors with destinations stored as offsets inside their tensor,
 * decode tables, tensor sizes, the expected checksums and the payload arena. */
WS_API int ws_plan_save(const ws_plan* plan, const char* path);

/* Re-creates a saved plan for `tensors`: the same count, byte sizes and BF16 flags
 * in the same order as at build (`base` pointers are ignored; A is not needed).
 * Block destinations are rebased onto the new targets; every descriptor is checked
 * against the tensors and the arena, and the metadata against its stored hash.
 * The arena is read into host memory (page-locked with opts->pin_arena) by up to
 * opts->threads readers. Follow with ws_plan_upload as after ws_plan_build; the
 * first apply's checksum confirms the resident weights were the expected source. */
WS_API int ws_plan_load(const char* path, const ws_tensor_desc* tensors, uint64_t ntensors,
                        const ws_build_options* opts, ws_plan** out);

/* No counterpart in the reference's API: replaces the acceptance check's per-tensor
 * sha256 (scripts/validate.py:50-56: D2H in 64 MiB pieces, hashed on the host)
 * with one pass over the resident bytes on `device`. out[i] = 64-bit hash of the
 * nbytes[i] bytes at ptrs[i] (device memory, any alignment): with w_j the
 * little-endian 64-bit words (last one zero-padded),
 *   hash = mix64(sum_j xmul(w_j ^ (j + 1) * 0xC2B2AE3D27D4EB4F) + (nbytes + 1) * 0x165667B19E3779F9)
 * with xmul(x) = y ^ (y >> 32), y = x * 0x9E3779B97F4A7C15 (arithmetic mod 2^64,
 * mix64 = the splitmix64 finaliser). Keeps one small
 * device buffer per device for the tensor list (allocated on the first call,
 * grown when a call lists more tensors, held until exit); calls on one device
 * are serialised; returns after `stream` completes. */
WS_API int ws_tensor_hashes(const void* const* ptrs, const uint64_t* nbytes, uint64_t n, int device, void* stream,
                            uint64_t* out);

/* No counterpart in the reference. Failure-path self-test: one warp waits on a
 * staging barrier that nothing arrives on, with the decode kernel's bounded wait
 * limited to `polls` (1 .. 2^20) polls; the wait gives up and the warp reports
 * through the device result word. *device_errors receives the reported bits
 * (WS_DEVERR_TIMEOUT = 4 expected). Nothing faults or hangs; the context stays
 * usable. Allocates one 16-byte stream-ordered buffer; returns after `stream`
 * completes. */
WS_API int ws_selftest_wait_timeout(uint32_t polls, int device, void* stream, uint32_t* device_errors);

/* Frees host and device resources (delta.py relies on GC for the same), after
 * waiting for an apply still in flight. */
WS_API void ws_plan_destroy(ws_plan* plan);

#ifdef __cplusplus
}
#endif
#endif /* WARPSHIFT_B200_H */
