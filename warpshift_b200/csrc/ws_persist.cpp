// Saved delta plans (ws_plan_save / ws_plan_load).
//
// The reference prepares the delta again after every restart (README.md:41:
// the package lives only in the worker process). A saved plan skips that: the
// descriptors, decode tables, expected checksums and the payload arena are
// written once and read back into a new plan for the same tensors, whose
// destinations are rebased onto the new process's target addresses.
//
// File layout (little-endian; this library's own format):
//   FileHeader
//   ws_plan_stats
//   ntensors x SavedTensor
//   nblocks  x ws_block_desc    (dst = byte offset inside the block's tensor)
//   nblocks  x uint32_t         (tensor index of each block)
//   ntiles   x ws_tile_desc
//   ntable_words x uint32_t
//   zero padding up to arena_offset (a multiple of 4096)
//   arena_bytes of payload      (blocks' payloads in block order)
// meta_hash covers every byte from the end of the header to arena_offset.
#include <errno.h>
#include <fcntl.h>
#include <stdio.h>
#include <string.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <string>
#include <thread>
#include <vector>

#include "../../include/warpshift_b200.h"
#include "ws_format.h"
#include "ws_guard.h"
#include "ws_gpu_encoder.h"
#include "ws_plan_internal.h"

namespace ws {
void set_last_error(const char* msg);
}

namespace {

constexpr char kMagic[8] = {'W', 'S', 'D', 'E', 'L', 'T', 'A', '1'};
constexpr uint32_t kVersion = 1;
constexpr uint64_t kArenaAlign = 4096;
constexpr uint64_t kReadPiece = 64ull << 20;

struct FileHeader {
  char magic[8];
  uint32_t version;
  uint32_t header_bytes;
  uint32_t stats_bytes;
  uint32_t block_desc_bytes;
  uint64_t ntensors, nblocks, ntiles, ntable_words;
  uint64_t arena_offset, arena_bytes;
  uint64_t meta_hash;
};
static_assert(sizeof(FileHeader) == 80, "FileHeader layout");

struct SavedTensor {
  uint64_t nbytes;
  uint32_t is_bf16;
  uint32_t reserved;
};

int fail(int code, const std::string& msg) {
  ws::set_last_error(msg.c_str());
  return code;
}

uint64_t meta_hash(const uint8_t* p, uint64_t n) {
  uint64_t h = 0x6A09E667F3BCC908ull ^ n;
  for (uint64_t i = 0; i < n; i += 8) {
    uint64_t w = 0;
    memcpy(&w, p + i, std::min<uint64_t>(8, n - i));
    h = ws_mix64(h ^ (w + (i / 8 + 1) * WS_CK_K1));
  }
  return h;
}

template <class T>
void append(std::vector<uint8_t>* out, const T* data, size_t count) {
  const size_t bytes = count * sizeof(T);
  const size_t at = out->size();
  out->resize(at + bytes);
  if (bytes) memcpy(out->data() + at, data, bytes);
}

template <class T>
bool take(const std::vector<uint8_t>& in, size_t* pos, T* data, size_t count) {
  const size_t bytes = count * sizeof(T);
  if (*pos + bytes > in.size()) return false;
  if (bytes) memcpy(data, in.data() + *pos, bytes);
  *pos += bytes;
  return true;
}

bool write_all(int fd, const void* data, uint64_t bytes) {
  const uint8_t* p = (const uint8_t*)data;
  while (bytes) {
    const ssize_t w = write(fd, p, std::min<uint64_t>(bytes, 1ull << 30));
    if (w < 0) {
      if (errno == EINTR) continue;
      return false;
    }
    p += w;
    bytes -= (uint64_t)w;
  }
  return true;
}

bool read_at(int fd, void* data, uint64_t bytes, uint64_t offset) {
  uint8_t* p = (uint8_t*)data;
  while (bytes) {
    const ssize_t r = pread(fd, p, std::min<uint64_t>(bytes, 1ull << 30), (off_t)offset);
    if (r < 0) {
      if (errno == EINTR) continue;
      return false;
    }
    if (r == 0) return false;  // truncated file
    p += r;
    bytes -= (uint64_t)r;
    offset += (uint64_t)r;
  }
  return true;
}

// Checks every descriptor of a loaded plan so that no kernel can address memory
// outside the new tensors or the arena.
std::string check_descriptors(const ws_plan* p) {
  const uint64_t ntables = p->tables.size() / 512;
  uint64_t next_src = 0;
  for (size_t k = 0; k < p->blocks.size(); ++k) {
    const ws_block_desc& d = p->blocks[k];
    const uint32_t t = p->block_tensor[k];
    if (t >= p->tensor_bytes.size()) return "block " + std::to_string(k) + " names a missing tensor";
    if (d.nbytes == 0 || d.nbytes > WS_BLOCK_BYTES) return "block " + std::to_string(k) + " has a bad size";
    if (d.dst > p->tensor_bytes[t] || d.nbytes > p->tensor_bytes[t] - d.dst)
      return "block " + std::to_string(k) + " writes outside its tensor";
    // Payloads are staged with bulk copies, whose sizes and addresses must be
    // multiples of 16 bytes; contiguous 16-byte lengths keep every source aligned.
    if (d.clen % 16u != 0) return "block " + std::to_string(k) + " has a payload length that is not a multiple of 16";
    if (d.src != next_src) return "block payloads are not contiguous in block order";
    next_src += d.clen;
    if (d.kind == WS_KIND_RAW) {
      if (d.clen < d.nbytes) return "raw block " + std::to_string(k) + " is shorter than its weights";
    } else if (d.kind <= WS_KIND_DICT_U16) {
      if (d.nwords < WS_HEADER_HALFWORDS || 2ull * d.nwords > d.clen)
        return "coded block " + std::to_string(k) + " has a bad stream length";
      const uint32_t split = ws_split_bits(d.flags);
      if (split && d.kind != WS_KIND_DICT_XOR && d.kind != WS_KIND_DICT_U16)
        return "block " + std::to_string(k) + " splits words but is not a word-dictionary block";
      if (split && ((2ull * d.nwords + 15u) & ~15ull) + ws_split_raw_bytes(d.nbytes / 2, split) > d.clen)
        return "coded block " + std::to_string(k) + " has a raw section outside its payload";
    } else {
      return "block " + std::to_string(k) + " has an unknown kind";
    }
  }
  if (next_src != p->arena_bytes) return "block payloads do not cover the arena";
  uint64_t covered = 0;
  for (size_t i = 0; i < p->tiles.size(); ++i) {
    const ws_tile_desc& td = p->tiles[i];
    if (td.first_block != covered || td.nblocks == 0 || td.nblocks > WS_TILE_BLOCKS ||
        td.first_block + (uint64_t)td.nblocks > p->blocks.size())
      return "tile " + std::to_string(i) + " has a bad block range";
    covered += td.nblocks;
    const bool coded = std::any_of(p->blocks.begin() + td.first_block, p->blocks.begin() + td.first_block + td.nblocks,
                                   [](const ws_block_desc& d) { return d.kind != WS_KIND_RAW; });
    if (td.table == WS_NO_TABLE ? coded : td.table >= ntables) return "tile " + std::to_string(i) + " has a bad table";
    const bool split_ok =
        td.split <= 3 && std::all_of(p->blocks.begin() + td.first_block, p->blocks.begin() + td.first_block + td.nblocks,
                                     [&](const ws_block_desc& d) {  // coded blocks share the tile's code
                                       const uint32_t c = (d.flags & WS_FLAG_SPLIT_MASK) >> WS_FLAG_SPLIT_SHIFT;
                                       return d.kind == WS_KIND_RAW ? c == 0 : c == td.split;
                                     });
    if (!split_ok) return "tile " + std::to_string(i) + " has blocks of another split code";
  }
  if (covered != p->blocks.size()) return "tiles do not cover the blocks";
  return "";
}

}  // namespace

extern "C" {

static int ws_plan_save_impl(const ws_plan* p, const char* path) {
  if (!p || !path) return fail(WS_ERR_INVALID, "null argument");
  if (p->block_tensor.size() != p->blocks.size()) return fail(WS_ERR_STATE, "plan has no tensor map");
  std::vector<uint8_t> meta;
  append(&meta, &p->stats, 1);
  for (size_t t = 0; t < p->tensor_bytes.size(); ++t) {
    const SavedTensor st{p->tensor_bytes[t], p->tensor_bf16[t], 0};
    append(&meta, &st, 1);
  }
  std::vector<ws_block_desc> rel(p->blocks);
  for (size_t k = 0; k < rel.size(); ++k) rel[k].dst -= p->tensor_target[p->block_tensor[k]];
  append(&meta, rel.data(), rel.size());
  append(&meta, p->block_tensor.data(), p->block_tensor.size());
  append(&meta, p->tiles.data(), p->tiles.size());
  append(&meta, p->tables.data(), p->tables.size());
  FileHeader h{};
  memcpy(h.magic, kMagic, 8);
  h.version = kVersion;
  h.header_bytes = sizeof(FileHeader);
  h.stats_bytes = sizeof(ws_plan_stats);
  h.block_desc_bytes = sizeof(ws_block_desc);
  h.ntensors = p->tensor_bytes.size();
  h.nblocks = p->blocks.size();
  h.ntiles = p->tiles.size();
  h.ntable_words = p->tables.size();
  h.arena_offset = (sizeof(FileHeader) + meta.size() + kArenaAlign - 1) / kArenaAlign * kArenaAlign;
  h.arena_bytes = p->arena_bytes;
  meta.resize(h.arena_offset - sizeof(FileHeader), 0);
  h.meta_hash = meta_hash(meta.data(), meta.size());
  // Written under a temporary name and renamed, so a reader never sees a partial file.
  const std::string tmp = std::string(path) + ".tmp";
  const int fd = open(tmp.c_str(), O_WRONLY | O_CREAT | O_TRUNC, 0644);
  if (fd < 0) return fail(WS_ERR_IO, "cannot create " + tmp + ": " + strerror(errno));
  bool ok = write_all(fd, &h, sizeof(h)) && write_all(fd, meta.data(), meta.size());
  for (size_t c = 0; ok && c < p->chunks.size(); ++c) ok = write_all(fd, p->chunks[c].ptr, p->chunks[c].bytes);
  const int saved_errno = errno;
  ok = ok && fsync(fd) == 0;
  if (close(fd) != 0) ok = false;
  if (!ok || rename(tmp.c_str(), path) != 0) {
    unlink(tmp.c_str());
    return fail(WS_ERR_IO, "cannot write " + std::string(path) + ": " + strerror(saved_errno ? saved_errno : errno));
  }
  return WS_OK;
}

int ws_plan_save(const ws_plan* p, const char* path) {
  return ws::guarded([&] { return ws_plan_save_impl(p, path); });
}

static int ws_plan_load_impl(const char* path, const ws_tensor_desc* tensors, uint64_t ntensors, const ws_build_options* opts,
                 ws_plan** out) {
  if (!path || !opts || !out || (ntensors && !tensors)) return fail(WS_ERR_INVALID, "null argument");
  *out = nullptr;
  const auto started = std::chrono::steady_clock::now();
  const int fd = open(path, O_RDONLY);
  if (fd < 0) return fail(WS_ERR_IO, "cannot open " + std::string(path) + ": " + strerror(errno));
  struct Closer {
    int fd;
    ~Closer() { close(fd); }
  } closer{fd};
  FileHeader h{};
  if (!read_at(fd, &h, sizeof(h), 0) || memcmp(h.magic, kMagic, 8) != 0)
    return fail(WS_ERR_INVALID, std::string(path) + " is not a saved delta plan");
  if (h.version != kVersion || h.header_bytes != sizeof(FileHeader) || h.stats_bytes != sizeof(ws_plan_stats) ||
      h.block_desc_bytes != sizeof(ws_block_desc))
    return fail(WS_ERR_INVALID, std::string(path) + " was written by an incompatible version");
  const uint64_t meta_bytes = sizeof(ws_plan_stats) + h.ntensors * sizeof(SavedTensor) +
                              h.nblocks * (sizeof(ws_block_desc) + 4) + h.ntiles * sizeof(ws_tile_desc) +
                              h.ntable_words * 4;
  if (h.ntensors > (1ull << 32) || h.nblocks > (1ull << 32) || h.ntiles > (1ull << 32) ||
      h.ntable_words > (1ull << 36) || h.ntable_words % 512 != 0 || h.arena_offset % kArenaAlign != 0 ||
      h.arena_offset < sizeof(FileHeader) + meta_bytes || h.arena_offset - sizeof(FileHeader) > (1ull << 40))
    return fail(WS_ERR_INVALID, std::string(path) + " has an inconsistent header");
  std::vector<uint8_t> meta(h.arena_offset - sizeof(FileHeader));
  if (!read_at(fd, meta.data(), meta.size(), sizeof(FileHeader)))
    return fail(WS_ERR_IO, std::string("cannot read ") + path + ": truncated or unreadable");
  if (meta_hash(meta.data(), meta.size()) != h.meta_hash)
    return fail(WS_ERR_INVALID, std::string(path) + " is corrupt (metadata hash mismatch)");
  if (h.ntensors != ntensors)
    return fail(WS_ERR_INVALID, "saved plan covers " + std::to_string(h.ntensors) + " tensors, got " +
                                    std::to_string(ntensors));

  ws_plan* p = new (std::nothrow) ws_plan();
  if (!p) return fail(WS_ERR_NOMEM, "out of memory");
  auto reject = [&](int code, const std::string& msg) {
    ws::free_plan_resources(p);
    delete p;
    return fail(code, msg);
  };
  p->opts = *opts;
  if (p->opts.batch_bytes == 0) p->opts.batch_bytes = 64ull << 20;
  if (p->opts.batch_bytes < (2ull << 20)) return reject(WS_ERR_INVALID, "batch_bytes must be at least 2 MiB");
  if (p->opts.staging_slots <= 0) p->opts.staging_slots = 3;
  p->device = opts->target_on_device ? opts->device : -1;
  size_t pos = 0;
  take(meta, &pos, &p->stats, 1);
  std::vector<SavedTensor> saved(h.ntensors);
  take(meta, &pos, saved.data(), saved.size());
  std::vector<std::pair<uint64_t, uint64_t>> spans;
  for (uint64_t i = 0; i < ntensors; ++i) {
    const ws_tensor_desc& t = tensors[i];
    if (t.nbytes != saved[i].nbytes || (t.is_bf16 != 0) != (saved[i].is_bf16 != 0))
      return reject(WS_ERR_INVALID, "tensor " + std::to_string(i) + " differs from the saved plan's (" +
                                        std::to_string(t.nbytes) + " bytes vs " + std::to_string(saved[i].nbytes) +
                                        ")");
    if (t.nbytes && !t.target) return reject(WS_ERR_INVALID, "tensor " + std::to_string(i) + " has a null target");
    if (t.nbytes) spans.emplace_back((uint64_t)(uintptr_t)t.target, (uint64_t)(uintptr_t)t.target + t.nbytes);
    p->tensor_bytes.push_back(t.nbytes);
    p->tensor_bf16.push_back(t.is_bf16 ? 1 : 0);
    p->tensor_target.push_back((uint64_t)(uintptr_t)t.target);
  }
  std::sort(spans.begin(), spans.end());
  for (size_t i = 1; i < spans.size(); ++i)
    if (spans[i].first < spans[i - 1].second) return reject(WS_ERR_INVALID, "Delta cannot update overlapping tensors");
  p->blocks.resize(h.nblocks);
  p->block_tensor.resize(h.nblocks);
  p->tiles.resize(h.ntiles);
  p->tables.resize(h.ntable_words);
  take(meta, &pos, p->blocks.data(), p->blocks.size());
  take(meta, &pos, p->block_tensor.data(), p->block_tensor.size());
  take(meta, &pos, p->tiles.data(), p->tiles.size());
  take(meta, &pos, p->tables.data(), p->tables.size());
  p->arena_bytes = h.arena_bytes;
  const std::string bad = check_descriptors(p);  // destinations still relative here
  if (!bad.empty()) return reject(WS_ERR_INVALID, std::string(path) + ": " + bad);
  for (size_t k = 0; k < p->blocks.size(); ++k) p->blocks[k].dst += p->tensor_target[p->block_tensor[k]];

  if (h.arena_bytes) {
    const int threads = ws::host_threads(opts->threads);
    ws::ArenaChunk c;
    std::string err;
    if (!ws::alloc_host_chunk(h.arena_bytes, opts->pin_arena != 0, threads, &c, &err))
      return reject(WS_ERR_NOMEM, err);
    p->chunks.push_back(c);
    const uint64_t pieces = (h.arena_bytes + kReadPiece - 1) / kReadPiece;
    std::atomic<uint64_t> next{0};
    std::atomic<bool> ok{true};
    auto body = [&] {
      for (uint64_t i = next++; i < pieces && ok; i = next++) {
        const uint64_t off = i * kReadPiece, n = std::min(kReadPiece, h.arena_bytes - off);
        if (!read_at(fd, c.ptr + off, n, h.arena_offset + off)) ok = false;
      }
    };
    std::vector<std::thread> pool;
    for (int t = 1; t < std::min<int>(threads, (int)std::min<uint64_t>(pieces, 16)); ++t) pool.emplace_back(body);
    body();
    for (auto& t : pool) t.join();
    if (!ok) return reject(WS_ERR_IO, std::string("cannot read the arena of ") + path + ": truncated or unreadable");
  }
  {
    std::string err;
    const int rc = ws::form_batches(p, &err);
    if (rc != WS_OK) return reject(rc, err);
  }
  p->stats.scratch_bytes = 0;
  p->stats.encoder = WS_ENCODER_LOADED;
  p->stats.encode_seconds = std::chrono::duration<double>(std::chrono::steady_clock::now() - started).count();
  *out = p;
  return WS_OK;
}

int ws_plan_load(const char* path, const ws_tensor_desc* tensors, uint64_t ntensors, const ws_build_options* opts,
                 ws_plan** out) {
  return ws::guarded([&] { return ws_plan_load_impl(path, tensors, ntensors, opts, out); });
}

}  // extern "C"
