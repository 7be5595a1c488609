// Host runtime behind the C ABI (include/warpshift_b200.h): prepare pipeline,
// stream layout, device upload and the staged apply.
//
// Prepare follows warpshift/delta.py:196-280 (walk tensors in dict order in
// 16 MiB packets, D2H each packet, choose a mode, pack a host arena and bounded
// batches), but packets are copied device->host through a ring of pinned staging
// buffers while a pool of host threads encodes them.
// Apply follows delta.py:294-327 (copy stream + compute stream, event-chained
// slots, blocking sync at the end), with one fused kernel per batch.
#include <cuda_runtime.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <condition_variable>
#include <deque>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "../../include/warpshift_b200.h"
#include "ws_encoder.h"
#include "ws_format.h"
#include "ws_guard.h"
#include "ws_gpu_encoder.h"
#include "ws_kernels.h"
#include "ws_plan_internal.h"

namespace {

using ws::Batch;

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
  try {
    g_last_error = msg;
  } catch (...) {
  }
  return code;
}

#define WS_CUDA_TRY(expr)                                                                             \
  do {                                                                                                \
    cudaError_t e_ = (expr);                                                                          \
    if (e_ != cudaSuccess) return fail(WS_ERR_CUDA, std::string(#expr) + ": " + cudaGetErrorString(e_)); \
  } while (0)


struct PacketRef {
  uint32_t tensor;
  uint64_t offset, nbytes;
};

int default_threads() {
  unsigned n = std::thread::hardware_concurrency();
  return n ? (int)n : 1;
}

ws::CodingOptions coding_options(const ws_build_options& o) {
  ws::CodingOptions co;
  co.dict_slack_pct = o.dict_slack_pct;
  co.escapes = o.escapes;
  co.split = o.split;
  return co;
}

// Run fn(i) for i in [0, n) on `threads` threads.
template <class F>
void parallel_for(uint64_t n, int threads, F fn) {
  if (n == 0) return;
  threads = (int)std::min<uint64_t>((uint64_t)std::max(1, threads), n);
  std::atomic<uint64_t> next{0};
  auto body = [&]() {
    for (uint64_t i = next++; i < n; i = next++) fn(i);
  };
  std::vector<std::thread> pool;
  for (int t = 1; t < threads; ++t) pool.emplace_back(body);
  body();
  for (auto& t : pool) t.join();
}

}  // namespace

namespace ws {
// Lets entry points defined in other translation units record ws_last_error().
void set_last_error(const char* msg) {
  try {
    g_last_error = msg;
  } catch (...) {  // out of memory for the message itself: keep the previous one
  }
}
}  // namespace ws


namespace {

void release_device(ws_plan* p) {
  if (p->device < 0) return;
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(p->device);
  // An apply still in flight reads these buffers and writes h_result.
  if (p->done_event) cudaEventSynchronize(p->done_event);
  cudaFree(p->d_blocks);
  cudaFree(p->d_tiles);
  cudaFree(p->d_tables);
  for (auto s : p->d_slots) cudaFree(s);
  cudaFree(p->d_resident);
  cudaFree(p->d_result);
  if (p->h_result) cudaFreeHost(p->h_result);
  for (auto e : p->copy_done) cudaEventDestroy(e);
  for (auto e : p->compute_done) cudaEventDestroy(e);
  if (p->start_event) cudaEventDestroy(p->start_event);
  if (p->aux_done) cudaEventDestroy(p->aux_done);
  if (p->done_event) cudaEventDestroy(p->done_event);
  if (p->own_copy_stream) cudaStreamDestroy(p->own_copy_stream);
  if (p->aux_stream) cudaStreamDestroy(p->aux_stream);
  p->d_blocks = nullptr;
  p->d_tiles = nullptr;
  p->d_tables = nullptr;
  p->d_slots.clear();
  p->d_resident = nullptr;
  p->d_result = nullptr;
  p->h_result = nullptr;
  p->copy_done.clear();
  p->compute_done.clear();
  p->start_event = nullptr;
  p->aux_done = nullptr;
  p->done_event = nullptr;
  p->own_copy_stream = nullptr;
  p->aux_stream = nullptr;
  p->uploaded = false;
  if (prev >= 0) cudaSetDevice(prev);
}

void free_chunks(std::vector<ws::ArenaChunk>* chunks) {
  for (const ws::ArenaChunk& c : *chunks) ws::free_host_chunk(c);
  chunks->clear();
}

void release_host(ws_plan* p) {
  free_chunks(&p->chunks);
  free(p->view_arena);
  p->view_arena = nullptr;
}

// Encode all packets. Device targets go through a ring of pinned staging
// buffers: the calling thread issues D2H copies in packet order, workers wait
// on each copy's event and encode.
int encode_all(const ws_tensor_desc* tensors, const std::vector<PacketRef>& packets, const ws_build_options& o,
               cudaStream_t stream, std::vector<ws::EncodedPacket>* out, std::vector<ws::ArenaChunk>* chunks,
               bool* external) {
  *external = false;
  const int threads = o.threads > 0 ? o.threads : default_threads();
  out->resize(packets.size());
  if (o.target_on_device && o.encode_on_device) {
    std::vector<ws::GpuPacketInput> in;
    in.reserve(packets.size());
    for (const PacketRef& pr : packets) {
      const ws_tensor_desc& t = tensors[pr.tensor];
      in.push_back(ws::GpuPacketInput{(const uint8_t*)t.base + pr.offset, (const uint8_t*)t.target + pr.offset,
                                      pr.nbytes, t.is_bf16 != 0});
    }
    // A serving process may have given most free HBM to its KV cache: on a device
    // allocation failure retry with smaller batches; the host encoder takes over
    // only when the caller allowed it.
    for (uint64_t batch = o.encode_batch_bytes ? o.encode_batch_bytes : (512ull << 20);; batch /= 4) {
      std::string err;
      bool oom = false;
      if (ws::gpu_encode_packets(in, o.policy, coding_options(o), batch, threads, o.pin_arena != 0, stream, out,
                                 chunks, &err, &oom)) {
        *external = true;
        return WS_OK;
      }
      free_chunks(chunks);
      out->assign(packets.size(), ws::EncodedPacket());
      if (!oom) return fail(WS_ERR_CUDA, err);
      cudaGetLastError();  // allocation failures are not sticky; clear the record
      if (batch / 4 < (32ull << 20)) break;
    }
    if (!o.host_fallback)
      return fail(WS_ERR_NOMEM,
                  "GPU encoder: not enough free device memory for its buffers, even with 32 MiB batches (free "
                  "device memory, or allow the host encoder with host_fallback)");
  }
  if (!o.target_on_device) {
    parallel_for(packets.size(), threads, [&](uint64_t i) {
      const PacketRef& pr = packets[i];
      const ws_tensor_desc& t = tensors[pr.tensor];
      ws::encode_packet((const uint8_t*)t.base + pr.offset, (const uint8_t*)t.target + pr.offset, pr.nbytes,
                        t.is_bf16 != 0, o.policy, coding_options(o), &(*out)[i]);
    });
    return WS_OK;
  }
  const size_t nbuf = std::min<size_t>(packets.size(), (size_t)std::max(2, 2 * threads));
  uint64_t buf_bytes = 0;
  for (auto& pr : packets) buf_bytes = std::max(buf_bytes, pr.nbytes);
  std::vector<uint8_t*> bufs(nbuf, nullptr);
  std::vector<cudaEvent_t> events(nbuf, nullptr);
  int rc = WS_OK;
  for (size_t b = 0; b < nbuf && rc == WS_OK; ++b) {
    if (cudaHostAlloc((void**)&bufs[b], buf_bytes, cudaHostAllocDefault) != cudaSuccess ||
        cudaEventCreateWithFlags(&events[b], cudaEventDisableTiming) != cudaSuccess)
      rc = fail(WS_ERR_NOMEM, "cannot allocate pinned staging for prepare");
  }
  std::mutex mu;
  std::condition_variable cv;
  std::deque<size_t> free_bufs;
  std::deque<std::pair<size_t, size_t>> jobs;  // (packet, buffer)
  bool done = false;
  std::atomic<bool> worker_error{false};
  for (size_t b = 0; b < nbuf; ++b) free_bufs.push_back(b);
  auto worker = [&]() {
    cudaSetDevice(o.device);
    for (;;) {
      std::pair<size_t, size_t> job;
      {
        std::unique_lock<std::mutex> lk(mu);
        cv.wait(lk, [&] { return !jobs.empty() || done; });
        if (jobs.empty()) return;
        job = jobs.front();
        jobs.pop_front();
      }
      const PacketRef& pr = packets[job.first];
      const ws_tensor_desc& t = tensors[pr.tensor];
      if (cudaEventSynchronize(events[job.second]) != cudaSuccess) {
        worker_error = true;
      } else {
        ws::encode_packet((const uint8_t*)t.base + pr.offset, bufs[job.second], pr.nbytes, t.is_bf16 != 0,
                          o.policy, coding_options(o), &(*out)[job.first]);
      }
      {
        std::lock_guard<std::mutex> lk(mu);
        free_bufs.push_back(job.second);
      }
      cv.notify_all();
    }
  };
  std::vector<std::thread> pool;
  if (rc == WS_OK)
    for (int t = 0; t < threads; ++t) pool.emplace_back(worker);
  for (size_t i = 0; i < packets.size() && rc == WS_OK; ++i) {
    size_t b;
    {
      std::unique_lock<std::mutex> lk(mu);
      cv.wait(lk, [&] { return !free_bufs.empty(); });
      b = free_bufs.front();
      free_bufs.pop_front();
    }
    const PacketRef& pr = packets[i];
    const uint8_t* src = (const uint8_t*)tensors[pr.tensor].target + pr.offset;
    cudaError_t e = cudaMemcpyAsync(bufs[b], src, pr.nbytes, cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess) e = cudaEventRecord(events[b], stream);
    if (e != cudaSuccess) {
      rc = fail(WS_ERR_CUDA, std::string("prepare D2H: ") + cudaGetErrorString(e));
      std::lock_guard<std::mutex> lk(mu);
      free_bufs.push_back(b);
      break;
    }
    {
      std::lock_guard<std::mutex> lk(mu);
      jobs.emplace_back(i, b);
    }
    cv.notify_all();
  }
  {
    std::lock_guard<std::mutex> lk(mu);
    done = true;
  }
  cv.notify_all();
  for (auto& t : pool) t.join();
  for (size_t b = 0; b < nbuf; ++b) {
    if (bufs[b]) cudaFreeHost(bufs[b]);
    if (events[b]) cudaEventDestroy(events[b]);
  }
  if (rc == WS_OK && worker_error) rc = fail(WS_ERR_CUDA, "prepare: waiting for a D2H copy failed");
  return rc;
}

// Descriptors, tiles, staging batches and the host arena. With `external` the
// payloads are already in p->chunks (GPU encoder); otherwise they are copied
// from the encoded blocks into one chunk.
int layout(ws_plan* p, const ws_tensor_desc* tensors, const std::vector<PacketRef>& packets,
           std::vector<ws::EncodedPacket>& enc, bool external) {
  ws_plan_stats& st = p->stats;
  std::vector<uint64_t> packet_first_block(enc.size());
  uint64_t arena = 0;
  for (size_t i = 0; i < enc.size(); ++i) {
    ws::EncodedPacket& e = enc[i];
    const PacketRef& pr = packets[i];
    st.mode_counts[e.mode]++;
    st.packets++;
    if (e.mode == WS_MODE_SKIP) {
      st.skipped_bytes += pr.nbytes;
      continue;
    }
    st.payload_bytes += e.payload_bytes;
    st.zero_block_bytes += e.zero_block_bytes;
    uint32_t table = WS_NO_TABLE;
    if (e.mode != WS_MODE_XOR_RAW) {
      table = (uint32_t)(p->tables.size() / 512);
      p->tables.insert(p->tables.end(), e.table, e.table + 512);
    }
    packet_first_block[i] = p->blocks.size();
    const uint64_t base_addr = (uint64_t)(uintptr_t)tensors[pr.tensor].target + pr.offset;
    for (size_t k = 0; k < e.blocks.size(); ++k) {
      const ws::EncodedBlock& b = e.blocks[k];
      if (k % WS_TILE_BLOCKS == 0) {
        ws_tile_desc t;
        t.first_block = (uint32_t)p->blocks.size();
        t.nblocks = (uint32_t)std::min<size_t>(WS_TILE_BLOCKS, e.blocks.size() - k);
        t.table = table;
        // Every split-word block of a packet has the packet's split code; the
        // kernel expands that code's raw-bit table once per tile.
        t.split = 0;
        for (size_t q = k; q < k + t.nblocks; ++q)
          t.split = std::max<uint32_t>(t.split, (e.blocks[q].flags & WS_FLAG_SPLIT_MASK) >> WS_FLAG_SPLIT_SHIFT);
        p->tiles.push_back(t);
      }
      ws_block_desc d;
      d.dst = base_addr + b.offset;
      d.src = arena;
      d.nbytes = b.nbytes;
      d.clen = external ? b.clen : (uint32_t)b.payload.size();
      d.nwords = b.nwords;
      d.kind = b.kind;
      d.tail = b.tail;
      d.flags = b.flags;
      const uint64_t index = p->blocks.size();
      st.expected_checksum[0] += ws_block_hash(b.lane_sum[0], index);
      st.expected_checksum[1] += ws_block_hash(b.lane_sum[1], index);
      st.touched_bytes += b.nbytes;
      p->blocks.push_back(d);
      p->block_tensor.push_back(pr.tensor);
      arena += d.clen;
    }
  }
  if (!external) {  // one chunk holding every payload
    if (arena) {
      const int threads = p->opts.threads > 0 ? p->opts.threads : default_threads();
      ws::ArenaChunk c;
      std::string err;
      if (!ws::alloc_host_chunk(arena, p->opts.pin_arena != 0, threads, &c, &err)) return fail(WS_ERR_NOMEM, err);
      p->chunks.push_back(c);
      parallel_for(enc.size(), threads, [&](uint64_t i) {
        if (enc[i].mode == WS_MODE_SKIP) return;
        uint64_t first = packet_first_block[i];
        for (size_t k = 0; k < enc[i].blocks.size(); ++k) {
          const auto& pl = enc[i].blocks[k].payload;
          memcpy(c.ptr + p->blocks[first + k].src, pl.data(), pl.size());
        }
      });
    }
  } else {
    uint64_t covered = 0;
    for (const ws::ArenaChunk& c : p->chunks) {
      if (c.off != covered) return fail(WS_ERR_STATE, "internal: arena chunks are not contiguous");
      covered += c.bytes;
    }
    if (covered != arena) return fail(WS_ERR_STATE, "internal: arena chunks do not match the block layout");
  }
  if (p->blocks.size() > 0xFFFFFFFFull) return fail(WS_ERR_INVALID, "too many blocks in one plan");
  p->arena_bytes = arena;
  st.arena_bytes = arena;
  {
    std::string err;
    const int rc = ws::form_batches(p, &err);
    if (rc != WS_OK) return fail(rc, err);
  }
  st.table_bytes = p->tables.size() * 4;
  st.metadata_bytes = p->blocks.size() * sizeof(ws_block_desc) + p->tiles.size() * sizeof(ws_tile_desc) +
                      st.table_bytes;
  st.blocks = p->blocks.size();
  st.tiles = p->tiles.size();
  return WS_OK;
}

}  // namespace

namespace ws {

int form_batches(ws_plan* p, std::string* err) {
  p->batches.clear();
  // Batches: contiguous tile ranges of one arena chunk whose payload fits one
  // staging slot. A tile never spans chunks (chunks end at packet boundaries).
  // Batches grow to `cap`: batch_bytes for large streams (fewer, longer copies),
  // down to 16 MiB for small ones (about 64 batches per stream keep the kernels
  // of consecutive batches overlapping). The first batches are smaller (cap / 16,
  // then / 4) so the first kernel starts after a short copy.
  const uint64_t cap =
      std::min<uint64_t>(p->opts.batch_bytes, std::max<uint64_t>(16ull << 20, p->arena_bytes / 64));
  uint64_t limit = std::max<uint64_t>(cap / 16, 1ull << 20);
  Batch cur{0, 0, 0, 0, 0, 0};
  bool open = false;
  uint32_t chunk = 0;
  for (uint32_t t = 0; t < p->tiles.size(); ++t) {
    const ws_tile_desc& td = p->tiles[t];
    const ws_block_desc& first = p->blocks[td.first_block];
    const ws_block_desc& last = p->blocks[td.first_block + td.nblocks - 1];
    const uint64_t bytes = last.src + last.clen - first.src;  // tiles are contiguous in the arena
    while (chunk < p->chunks.size() && first.src >= p->chunks[chunk].off + p->chunks[chunk].bytes) ++chunk;
    if (chunk >= p->chunks.size() || last.src + last.clen > p->chunks[chunk].off + p->chunks[chunk].bytes) {
      *err = "internal: a tile spans two arena chunks";
      return WS_ERR_STATE;
    }
    if (open && (cur.bytes + bytes > limit || cur.chunk != chunk)) {
      p->batches.push_back(cur);
      open = false;
      limit = std::min(limit * 4, cap);
    }
    if (!open) {
      cur = Batch{t, t, first.src, 0, chunk, 0};
      open = true;
    }
    cur.tile_end = t + 1;
    cur.bytes += bytes;
    cur.kinds |= td.split ? ws::kTilesSplit : ws::kTilesWhole;
  }
  if (open) p->batches.push_back(cur);
  p->stats.batches = p->batches.size();
  return WS_OK;
}

void free_plan_resources(ws_plan* p) {
  release_device(p);
  release_host(p);
}

int host_threads(int requested) { return requested > 0 ? requested : default_threads(); }

}  // namespace ws

extern "C" {

int ws_version(void) { return 100; }

int ws_last_error(char* buf, size_t len) {
  if (!buf || len == 0) return WS_ERR_INVALID;
  size_t n = std::min(len - 1, g_last_error.size());
  memcpy(buf, g_last_error.data(), n);
  buf[n] = 0;
  return WS_OK;
}

int ws_u16_residual(const uint8_t* base, const uint8_t* target, uint64_t nbytes, uint8_t* out) {
  if (nbytes % 2) return fail(WS_ERR_INVALID, "U16 residual needs an even byte count");
  if (nbytes && (!base || !target || !out)) return fail(WS_ERR_INVALID, "null pointer");
  ws::u16_residual_reference(base, target, nbytes, out);
  return WS_OK;
}

static int ws_plan_build_impl(const ws_tensor_desc* tensors, uint64_t ntensors, const ws_build_options* opts, void* stream,
                  ws_plan** out) {
  if (!out || !opts || (ntensors && !tensors)) return fail(WS_ERR_INVALID, "null argument");
  *out = nullptr;
  if (opts->policy < WS_POLICY_AUTO || opts->policy > WS_POLICY_U16) return fail(WS_ERR_INVALID, "unknown policy");
  const auto started = std::chrono::steady_clock::now();
  ws_plan* p = new (std::nothrow) ws_plan();
  if (!p) return fail(WS_ERR_NOMEM, "out of memory");
  p->opts = *opts;
  if (p->opts.batch_bytes == 0) p->opts.batch_bytes = 64ull << 20;
  if (p->opts.batch_bytes < (2ull << 20)) {
    delete p;
    return fail(WS_ERR_INVALID, "batch_bytes must be at least 2 MiB");
  }
  if (p->opts.staging_slots <= 0) p->opts.staging_slots = 3;
  p->device = opts->target_on_device ? opts->device : -1;
  // Destination spans must not overlap (delta.py:159-162).
  std::vector<std::pair<uint64_t, uint64_t>> spans;
  for (uint64_t i = 0; i < ntensors; ++i) {
    const ws_tensor_desc& t = tensors[i];
    if (t.nbytes && (!t.base || !t.target)) {
      delete p;
      return fail(WS_ERR_INVALID, "tensor " + std::to_string(i) + " has a null pointer");
    }
    if (t.nbytes) spans.emplace_back((uint64_t)(uintptr_t)t.target, (uint64_t)(uintptr_t)t.target + t.nbytes);
  }
  std::sort(spans.begin(), spans.end());
  for (size_t i = 1; i < spans.size(); ++i)
    if (spans[i].first < spans[i - 1].second) {
      delete p;
      return fail(WS_ERR_INVALID, "Delta cannot update overlapping tensors");
    }
  std::vector<PacketRef> packets;
  for (uint64_t i = 0; i < ntensors; ++i)
    for (uint64_t off = 0; off < tensors[i].nbytes; off += WS_PACKET_BYTES)
      packets.push_back(PacketRef{(uint32_t)i, off, std::min<uint64_t>(WS_PACKET_BYTES, tensors[i].nbytes - off)});
  for (uint64_t i = 0; i < ntensors; ++i) {
    p->stats.runtime_bytes += tensors[i].nbytes;
    p->tensor_bytes.push_back(tensors[i].nbytes);
    p->tensor_bf16.push_back(tensors[i].is_bf16 ? 1 : 0);
    p->tensor_target.push_back((uint64_t)(uintptr_t)tensors[i].target);
  }
  int prev = -1;
  if (opts->target_on_device) {
    cudaGetDevice(&prev);
    if (cudaSetDevice(opts->device) != cudaSuccess) {
      delete p;
      return fail(WS_ERR_CUDA, "cannot select device " + std::to_string(opts->device));
    }
  }
  std::vector<ws::EncodedPacket> enc;
  bool external = false;
  const auto t_enc = std::chrono::steady_clock::now();
  int rc = encode_all(tensors, packets, p->opts, (cudaStream_t)stream, &enc, &p->chunks, &external);
  const auto t_lay = std::chrono::steady_clock::now();
  if (rc == WS_OK) rc = layout(p, tensors, packets, enc, external);
  p->stats.encoder = external ? WS_ENCODER_GPU : WS_ENCODER_HOST;
  if (getenv("WS_ENCODER_TIMING"))
    fprintf(stderr, "plan build: encode %.3f s, layout %.3f s\n",
            std::chrono::duration<double>(t_lay - t_enc).count(),
            std::chrono::duration<double>(std::chrono::steady_clock::now() - t_lay).count());
  if (prev >= 0) cudaSetDevice(prev);
  if (rc != WS_OK) {
    release_host(p);
    delete p;
    return rc;
  }
  p->stats.encode_seconds =
      std::chrono::duration<double>(std::chrono::steady_clock::now() - started).count();
  *out = p;
  return WS_OK;
}

int ws_plan_build(const ws_tensor_desc* tensors, uint64_t ntensors, const ws_build_options* opts, void* stream,
                  ws_plan** out) {
  return ws::guarded([&] { return ws_plan_build_impl(tensors, ntensors, opts, stream, out); });
}

static int ws_plan_upload_impl(ws_plan* p, void* stream) {
  if (!p) return fail(WS_ERR_INVALID, "null plan");
  if (p->device < 0) return fail(WS_ERR_STATE, "plan was built for host targets; nothing to upload");
  if (p->uploaded) return WS_OK;
  int prev = -1;
  cudaGetDevice(&prev);
  WS_CUDA_TRY(cudaSetDevice(p->device));
  cudaStream_t s = (cudaStream_t)stream;
  auto alloc_copy = [&](void** dst, const void* src, size_t bytes) -> cudaError_t {
    if (!bytes) return cudaSuccess;
    cudaError_t e = cudaMalloc(dst, bytes);
    if (e != cudaSuccess) return e;
    return cudaMemcpyAsync(*dst, src, bytes, cudaMemcpyHostToDevice, s);
  };
  cudaError_t e = alloc_copy((void**)&p->d_blocks, p->blocks.data(), p->blocks.size() * sizeof(ws_block_desc));
  if (e == cudaSuccess) e = alloc_copy((void**)&p->d_tiles, p->tiles.data(), p->tiles.size() * sizeof(ws_tile_desc));
  if (e == cudaSuccess) e = alloc_copy((void**)&p->d_tables, p->tables.data(), p->tables.size() * 4);
  if (e == cudaSuccess) e = cudaMalloc((void**)&p->d_result, sizeof(ws_device_result));
  if (e == cudaSuccess) e = cudaHostAlloc((void**)&p->h_result, sizeof(ws_device_result), cudaHostAllocDefault);
  uint64_t slot = 0;
  for (auto& b : p->batches) slot = std::max(slot, b.bytes);
  p->slot_bytes = slot;
  const int nslots = p->batches.empty() ? 0 : std::min<int>(p->opts.staging_slots, (int)p->batches.size());
  for (int i = 0; i < nslots && e == cudaSuccess; ++i) {
    uint8_t* d = nullptr;
    e = cudaMalloc((void**)&d, slot);
    if (e == cudaSuccess) p->d_slots.push_back(d);
    cudaEvent_t a = nullptr, b = nullptr;
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&a, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&b, cudaEventDisableTiming);
    if (a) p->copy_done.push_back(a);
    if (b) p->compute_done.push_back(b);
  }
  if (e == cudaSuccess) e = ws::prime_kernels();
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p->start_event, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&p->own_copy_stream, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p->aux_done, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&p->aux_stream, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p->done_event, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) {
    std::string msg = std::string("upload: ") + cudaGetErrorString(e);
    release_device(p);
    if (prev >= 0) cudaSetDevice(prev);
    return fail(e == cudaErrorMemoryAllocation ? WS_ERR_NOMEM : WS_ERR_CUDA, msg);
  }
  p->stats.scratch_bytes = (uint64_t)nslots * slot + sizeof(ws_device_result);
  p->uploaded = true;
  if (prev >= 0) cudaSetDevice(prev);
  return WS_OK;
}

int ws_plan_upload(ws_plan* p, void* stream) {
  return ws::guarded([&] { return ws_plan_upload_impl(p, stream); });
}

static int ws_plan_set_resident_impl(ws_plan* p, int resident, void* stream) {
  if (!p) return fail(WS_ERR_INVALID, "null plan");
  if (!p->uploaded) return fail(WS_ERR_STATE, "upload the plan first");
  int prev = -1;
  cudaGetDevice(&prev);
  WS_CUDA_TRY(cudaSetDevice(p->device));
  if (resident && !p->d_resident && p->arena_bytes) {
    cudaError_t e = cudaMalloc((void**)&p->d_resident, p->arena_bytes);
    for (size_t c = 0; c < p->chunks.size() && e == cudaSuccess; ++c)
      e = cudaMemcpyAsync(p->d_resident + p->chunks[c].off, p->chunks[c].ptr, p->chunks[c].bytes,
                          cudaMemcpyHostToDevice, (cudaStream_t)stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize((cudaStream_t)stream);
    if (e != cudaSuccess) {
      cudaFree(p->d_resident);
      p->d_resident = nullptr;
      if (prev >= 0) cudaSetDevice(prev);
      return fail(WS_ERR_CUDA, std::string("resident copy: ") + cudaGetErrorString(e));
    }
    p->stats.scratch_bytes += p->arena_bytes;
  } else if (!resident && p->d_resident) {
    WS_CUDA_TRY(cudaEventSynchronize(p->done_event));  // applies in flight read the resident copy
    cudaFree(p->d_resident);
    p->d_resident = nullptr;
    p->stats.scratch_bytes -= p->arena_bytes;
  }
  if (prev >= 0) cudaSetDevice(prev);
  return WS_OK;
}

int ws_plan_set_resident(ws_plan* p, int resident, void* stream) {
  return ws::guarded([&] { return ws_plan_set_resident_impl(p, resident, stream); });
}

static int ws_apply_async_impl(ws_plan* p, int reverse, void* compute_stream, void* copy_stream) {
  if (!p) return fail(WS_ERR_INVALID, "null plan");
  if (!p->uploaded) return fail(WS_ERR_STATE, "upload the plan before applying");
  reverse = reverse ? 1 : 0;
  int prev = -1;
  cudaGetDevice(&prev);
  WS_CUDA_TRY(cudaSetDevice(p->device));
  cudaStream_t comp = (cudaStream_t)compute_stream;
  cudaStream_t copy = copy_stream ? (cudaStream_t)copy_stream : p->own_copy_stream;
  uint64_t h2d = 0;
  uint32_t launches = 0;
  WS_CUDA_TRY(cudaMemsetAsync(p->d_result, 0, sizeof(ws_device_result), comp));
  if (p->d_resident || p->arena_bytes == 0) {
    if (!p->tiles.empty()) {
      uint32_t kinds = 0;
      for (const Batch& bt : p->batches) kinds |= bt.kinds;
      WS_CUDA_TRY(ws::launch_apply(p->d_tiles, 0, (uint32_t)p->tiles.size(), p->d_blocks, p->d_tables,
                                   p->d_resident, 0, p->d_result, reverse, kinds, comp, &launches));
    }
  } else {
    // Staged: batch b is copied into slot b % nslots on the copy stream and
    // decoded on compute stream b % 2 (the caller's stream or the plan's second
    // one), so one batch's kernel fills the SMs the previous kernel's last wave
    // leaves idle. Slot reuse waits for the kernel that read the slot.
    const size_t nslots = p->d_slots.size();
    WS_CUDA_TRY(cudaEventRecord(p->start_event, comp));
    WS_CUDA_TRY(cudaStreamWaitEvent(copy, p->start_event, 0));
    WS_CUDA_TRY(cudaStreamWaitEvent(p->aux_stream, p->start_event, 0));
    for (size_t b = 0; b < p->batches.size(); ++b) {
      const Batch& bt = p->batches[b];
      const size_t slot = b % nslots;
      cudaStream_t run = (b & 1) ? p->aux_stream : comp;
      if (b >= nslots) WS_CUDA_TRY(cudaStreamWaitEvent(copy, p->compute_done[slot], 0));
      const ws::ArenaChunk& ch = p->chunks[bt.chunk];
      WS_CUDA_TRY(cudaMemcpyAsync(p->d_slots[slot], ch.ptr + (bt.arena_off - ch.off), bt.bytes,
                                  cudaMemcpyHostToDevice, copy));
      WS_CUDA_TRY(cudaEventRecord(p->copy_done[slot], copy));
      WS_CUDA_TRY(cudaStreamWaitEvent(run, p->copy_done[slot], 0));
      WS_CUDA_TRY(ws::launch_apply(p->d_tiles, bt.tile_begin, bt.tile_end - bt.tile_begin, p->d_blocks, p->d_tables,
                                   p->d_slots[slot], bt.arena_off, p->d_result, reverse, bt.kinds, run, &launches));
      WS_CUDA_TRY(cudaEventRecord(p->compute_done[slot], run));
      h2d += bt.bytes;
    }
    WS_CUDA_TRY(cudaEventRecord(p->aux_done, p->aux_stream));
    WS_CUDA_TRY(cudaStreamWaitEvent(comp, p->aux_done, 0));
  }
  WS_CUDA_TRY(cudaMemcpyAsync(p->h_result, p->d_result, sizeof(ws_device_result), cudaMemcpyDeviceToHost, comp));
  WS_CUDA_TRY(cudaEventRecord(p->done_event, comp));
  p->pending_reverse = reverse;
  p->pending_h2d = h2d;
  p->pending_launches = launches;
  if (prev >= 0) cudaSetDevice(prev);
  return WS_OK;
}

int ws_apply_async(ws_plan* p, int reverse, void* compute_stream, void* copy_stream) {
  return ws::guarded([&] { return ws_apply_async_impl(p, reverse, compute_stream, copy_stream); });
}

static int ws_apply_finish_impl(ws_plan* p, void* compute_stream, ws_apply_result* out) {
  if (!p) return fail(WS_ERR_INVALID, "null plan");
  if (p->pending_reverse < 0) return fail(WS_ERR_STATE, "no apply in flight");
  int prev = -1;
  cudaGetDevice(&prev);
  WS_CUDA_TRY(cudaSetDevice(p->device));
  cudaError_t e = cudaStreamSynchronize((cudaStream_t)compute_stream);
  if (prev >= 0) cudaSetDevice(prev);
  const int reverse = p->pending_reverse;
  p->pending_reverse = -1;
  if (e != cudaSuccess) return fail(WS_ERR_CUDA, std::string("apply: ") + cudaGetErrorString(e));
  ws_apply_result r{};
  r.checksum = p->h_result->checksum;
  r.expected = p->stats.expected_checksum[reverse];
  r.device_errors = p->h_result->errors;
  r.bad_block_plus1 = p->h_result->bad_block_plus1;
  r.h2d_bytes = p->pending_h2d;
  r.launches = p->pending_launches;
  if (out) *out = r;
  if (r.device_errors) {
    char msg[160];
    snprintf(msg, sizeof(msg), "delta decode failed: device errors 0x%x at block %u", r.device_errors,
             r.bad_block_plus1 ? r.bad_block_plus1 - 1 : 0);
    return fail(WS_ERR_DEVICE, msg);
  }
  if (r.checksum != r.expected) {
    char msg[200];
    snprintf(msg, sizeof(msg),
             "delta apply checksum mismatch (got %016llx, expected %016llx): resident weights were not the "
             "expected source model",
             (unsigned long long)r.checksum, (unsigned long long)r.expected);
    return fail(WS_ERR_CHECKSUM, msg);
  }
  return WS_OK;
}

int ws_apply_finish(ws_plan* p, void* compute_stream, ws_apply_result* out) {
  return ws::guarded([&] { return ws_apply_finish_impl(p, compute_stream, out); });
}

// A failed switch (corrupt stream or a checksum mismatch) has already written
// every block it decoded. Both applies are exact inverses of each other (XOR is
// its own inverse; the U16 directions add and subtract the same word), and the
// decode of a block depends only on its payload bytes, so running the other
// direction over the same stream writes back exactly the bytes that were
// resident, corrupt blocks included. The restored bytes are then hashed like
// any apply and compared with the checksum recorded at prepare for the source
// model. A decode that gave up on a staging wait is not exactly repeatable and
// its rollback is reported as unverified.
static int ws_apply_impl(ws_plan* p, int reverse, void* compute_stream, void* copy_stream, ws_apply_result* out) {
  int rc = ws_apply_async_impl(p, reverse, compute_stream, copy_stream);
  if (rc != WS_OK) return rc;
  ws_apply_result r{};
  rc = ws_apply_finish_impl(p, compute_stream, &r);
  if (rc == WS_ERR_DEVICE || rc == WS_ERR_CHECKSUM) {
    const std::string first = g_last_error;
    const int back_dir = reverse ? 0 : 1;
    ws_apply_result back{};
    int rb = ws_apply_async_impl(p, back_dir, compute_stream, copy_stream);
    if (rb == WS_OK) rb = ws_apply_finish_impl(p, compute_stream, &back);
    const char* how;
    if (rb != WS_OK && rb != WS_ERR_DEVICE && rb != WS_ERR_CHECKSUM) {
      r.rollback = WS_ROLLBACK_FAILED;
      how = "; rollback failed: weights are undefined";
    } else if ((back.device_errors & WS_DEVERR_TIMEOUT) || (r.device_errors & WS_DEVERR_TIMEOUT)) {
      r.rollback = WS_ROLLBACK_FAILED;
      how = "; rollback ran but a decode gave up on a staging wait: weights are undefined";
    } else if (back.checksum == p->stats.expected_checksum[back_dir]) {
      r.rollback = WS_ROLLBACK_RESTORED;
      how = "; rolled back: the source model's bytes are restored (checksum verified)";
    } else {
      r.rollback = WS_ROLLBACK_UNVERIFIED;
      how = "; rolled back, but the restored bytes do not hash to the source model's (the resident weights were "
            "not the package's source model)";
    }
    r.h2d_bytes += back.h2d_bytes;
    r.launches += back.launches;
    fail(rc, first + how);
  }
  if (out) *out = r;
  return rc;
}

int ws_apply(ws_plan* p, int reverse, void* compute_stream, void* copy_stream, ws_apply_result* out) {
  return ws::guarded([&] { return ws_apply_impl(p, reverse, compute_stream, copy_stream, out); });
}

int ws_plan_get_stats(const ws_plan* p, ws_plan_stats* out) {
  if (!p || !out) return fail(WS_ERR_INVALID, "null argument");
  *out = p->stats;
  return WS_OK;
}

static int ws_plan_get_view_impl(const ws_plan* p, ws_plan_view* out) {
  if (!p || !out) return fail(WS_ERR_INVALID, "null argument");
  const uint8_t* arena = p->chunks.empty() ? nullptr : p->chunks[0].ptr;
  if (p->chunks.size() > 1) {  // one contiguous host copy, made once
    ws_plan* mp = const_cast<ws_plan*>(p);
    if (!mp->view_arena) {
      if (posix_memalign((void**)&mp->view_arena, 4096, p->arena_bytes) != 0) {
        mp->view_arena = nullptr;
        return fail(WS_ERR_NOMEM, "cannot allocate the contiguous arena view");
      }
      for (const ws::ArenaChunk& c : p->chunks) memcpy(mp->view_arena + c.off, c.ptr, c.bytes);
    }
    arena = mp->view_arena;
  }
  out->blocks = p->blocks.data();
  out->nblocks = p->blocks.size();
  out->tiles = p->tiles.data();
  out->ntiles = p->tiles.size();
  out->tables = p->tables.data();
  out->ntables = p->tables.size() / 512;
  out->arena = arena;
  out->arena_bytes = p->arena_bytes;
  return WS_OK;
}

int ws_plan_get_view(const ws_plan* p, ws_plan_view* out) {
  return ws::guarded([&] { return ws_plan_get_view_impl(p, out); });
}

void ws_plan_destroy(ws_plan* p) {
  if (!p) return;
  ws::free_plan_resources(p);
  delete p;
}

}  // extern "C"
