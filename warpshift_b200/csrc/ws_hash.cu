// Per-tensor content hashes on the device (ws_tensor_hashes).
//
// Replaces the acceptance check's per-tensor sha256 (scripts/validate.py:50-56),
// which copies every tensor to the host in 64 MiB pieces, with one HBM-bound
// pass over the resident bytes. Definition (restated by the oracle): for a
// tensor of N bytes, let w_i be its little-endian 64-bit words (the last one
// zero-padded) and
//   sum  = sum_i xmul(w_i ^ ((i + 1) * WS_TH_KPOS))    (mod 2^64)
//   hash = mix64(sum + (N + 1) * WS_TH_KLEN)           (mod 2^64)
// where xmul(x) = y ^ (y >> 32), y = x * WS_TH_KMUL (one 64-bit multiply and a
// fold per word, ws_format.h) and mix64 is the splitmix64 finaliser applied once
// per tensor. The terms are keyed by position and summed, so any split of the
// words over warps gives the same value.
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/warpshift_b200.h"
#include "ws_format.h"
#include "ws_guard.h"

namespace ws {
void set_last_error(const char* msg);
}

namespace {

constexpr uint32_t kSegWords = 8192;  // one warp hashes 64 KiB at a time
constexpr uint32_t kHashThreads = 256;
constexpr uint32_t kHashBlocksPerSm = 8;

struct HashTensor {
  const uint8_t* ptr;
  uint64_t nbytes;
  uint64_t first_seg;  // first 64 KiB segment of this tensor in the flattened list
};

__device__ __forceinline__ uint64_t term(uint64_t w, uint64_t i) { return ws_xmul64(w ^ ((i + 1) * WS_TH_KPOS)); }

// Asks the TMA unit to pull `bytes` (a multiple of 16, from a 16-byte-aligned
// address) into L2 without waiting for them.
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Word i assembled from bytes (unaligned bases and the zero-padded tail).
__device__ __forceinline__ uint64_t word_bytes(const uint8_t* p, uint64_t nbytes, uint64_t i) {
  uint64_t w = 0;
  const uint64_t b0 = i * 8;
#pragma unroll
  for (uint32_t k = 0; k < 8; ++k)
    if (b0 + k < nbytes) w |= (uint64_t)__ldg(p + b0 + k) << (8 * k);
  return w;
}

__global__ void __launch_bounds__(kHashThreads)
    ws_tensor_hash_kernel(const HashTensor* __restrict__ tensors, uint32_t n, uint64_t nseg,
                          unsigned long long* __restrict__ acc) {
  const uint32_t lane = threadIdx.x & 31u;
  const uint64_t warps = (uint64_t)gridDim.x * (kHashThreads / 32);
  for (uint64_t seg = (uint64_t)blockIdx.x * (kHashThreads / 32) + (threadIdx.x >> 5); seg < nseg; seg += warps) {
    // Owner: the last tensor whose first segment is <= seg (tensors are non-empty).
    uint32_t lo = 0, hi = n;
    while (hi - lo > 1) {
      const uint32_t mid = (lo + hi) >> 1;
      if (tensors[mid].first_seg <= seg) lo = mid; else hi = mid;
    }
    const HashTensor t = tensors[lo];
    const uint64_t nwords = (t.nbytes + 7) / 8, full = t.nbytes / 8;
    const uint64_t w0 = (seg - t.first_seg) * kSegWords;
    const uint64_t w1 = min(w0 + kSegWords, nwords);
    uint64_t sum = 0;
    if (((uintptr_t)t.ptr & 15u) == 0) {
      // Lane l hashes words (w, w + 1) for w = w0 + 2l + 64k: 16-byte loads, 512
      // contiguous bytes per warp and step. Software-pipelined: the next four
      // steps' loads are in flight while the current four are hashed, and lane
      // 0 has the TMA unit pull the steps after those into L2, so the warp never
      // waits a full DRAM latency between batches.
      const uint4* v = reinterpret_cast<const uint4*>(t.ptr);
      const uint64_t end = min(w1, full);
      uint64_t w = w0 + 2 * lane;
      if (w0 + 4 * 64 <= end) {
        if (lane == 0 && w0 + 12 * 64 <= end) prefetch_l2(t.ptr + (w0 + 4 * 64) * 8, 8 * 64 * 8);
        uint4 cur[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) cur[k] = __ldg(v + (w + 64 * k) / 2);
        uint64_t key = (w + 1) * WS_TH_KPOS;  // key of word w; the loop below advances it
        for (; w + 3 * 64 + 2 <= end; w += 4 * 64) {
          const bool more = w + 7 * 64 + 2 <= end;
          uint4 nxt[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) nxt[k] = more ? __ldg(v + (w + 64 * (k + 4)) / 2) : make_uint4(0, 0, 0, 0);
          const uint64_t ahead = (w - 2 * lane) + 12 * 64;  // first word of the batch after next
          if (lane == 0 && ahead + 4 * 64 <= end) prefetch_l2(t.ptr + ahead * 8, 4 * 64 * 8);
          // Position keys (i + 1) * KPOS of the lane's words i = w + 64k and i + 1
          // by addition from the batch's first key: no 64-bit multiply per word.
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint64_t ka = key + (uint64_t)(64 * k) * WS_TH_KPOS;
            sum += ws_xmul64((((uint64_t)cur[k].y << 32) | cur[k].x) ^ ka) +
                   ws_xmul64((((uint64_t)cur[k].w << 32) | cur[k].z) ^ (ka + WS_TH_KPOS));
          }
          key += (uint64_t)(4 * 64) * WS_TH_KPOS;
#pragma unroll
          for (int k = 0; k < 4; ++k) cur[k] = nxt[k];
        }
      }
      for (; w < w1; w += 64) {
        if (w + 2 <= full) {
          const uint4 x = __ldg(v + w / 2);
          sum += term(((uint64_t)x.y << 32) | x.x, w) + term(((uint64_t)x.w << 32) | x.z, w + 1);
        } else {
          sum += term(word_bytes(t.ptr, t.nbytes, w), w);
          if (w + 1 < w1) sum += term(word_bytes(t.ptr, t.nbytes, w + 1), w + 1);
        }
      }
    } else {
      for (uint64_t w = w0 + lane; w < w1; w += 32) sum += term(word_bytes(t.ptr, t.nbytes, w), w);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xFFFFFFFFu, sum, o);
    if (lane == 0) atomicAdd(acc + lo, (unsigned long long)sum);
  }
}

int fail(int code, const std::string& msg) {
  ws::set_last_error(msg.c_str());
  return code;
}

// Device buffers for one device's tensor list and accumulators, allocated on
// first use, grown when a call lists more tensors, and kept until exit, so a
// call allocates nothing after the first. Calls on one device hold the mutex
// for their whole duration (they end with a stream synchronisation).
struct HashScratch {
  std::mutex lock;
  HashTensor* list = nullptr;
  unsigned long long* acc = nullptr;
  size_t capacity = 0;
};
constexpr int kHashMaxDevices = 64;
HashScratch g_hash_scratch[kHashMaxDevices];

}  // namespace

static int ws_tensor_hashes_impl(const void* const* ptrs, const uint64_t* nbytes, uint64_t n, int device, void* stream,
                                uint64_t* out) {
  if (n && (!ptrs || !nbytes || !out)) return fail(WS_ERR_INVALID, "null argument");
  std::vector<HashTensor> list;
  std::vector<uint64_t> owner;  // index into ptrs of each listed tensor
  uint64_t nseg = 0;
  for (uint64_t i = 0; i < n; ++i) {
    if (nbytes[i] == 0) continue;
    if (!ptrs[i]) return fail(WS_ERR_INVALID, "tensor " + std::to_string(i) + " has a null pointer");
    list.push_back(HashTensor{(const uint8_t*)ptrs[i], nbytes[i], nseg});
    owner.push_back(i);
    nseg += ((nbytes[i] + 7) / 8 + kSegWords - 1) / kSegWords;
  }
  if (list.size() > 0xFFFFFFFFull) return fail(WS_ERR_INVALID, "too many tensors");
  std::vector<unsigned long long> acc(list.size(), 0);
  if (!list.empty()) {
    if (device < 0 || device >= kHashMaxDevices) return fail(WS_ERR_INVALID, "bad device ordinal");
    HashScratch& scratch = g_hash_scratch[device];
    std::lock_guard<std::mutex> hold(scratch.lock);
    int prev = -1;
    cudaGetDevice(&prev);
    cudaError_t e = cudaSetDevice(device);
    cudaStream_t s = (cudaStream_t)stream;
    int sms = 0;
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    if (e == cudaSuccess && scratch.capacity < list.size()) {
      cudaFree(scratch.list);
      cudaFree(scratch.acc);
      scratch.list = nullptr;
      scratch.acc = nullptr;
      scratch.capacity = 0;
      const size_t cap = std::max<size_t>(list.size(), 1024);
      e = cudaMalloc((void**)&scratch.list, cap * sizeof(HashTensor));
      if (e == cudaSuccess) e = cudaMalloc((void**)&scratch.acc, cap * sizeof(unsigned long long));
      if (e == cudaSuccess) scratch.capacity = cap;
    }
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(scratch.list, list.data(), list.size() * sizeof(HashTensor), cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(scratch.acc, 0, acc.size() * sizeof(unsigned long long), s);
    if (e == cudaSuccess) {
      const uint64_t warps_needed = nseg;
      const uint64_t blocks = std::min<uint64_t>((uint64_t)sms * kHashBlocksPerSm,
                                                 (warps_needed + kHashThreads / 32 - 1) / (kHashThreads / 32));
      ws_tensor_hash_kernel<<<(unsigned)blocks, kHashThreads, 0, s>>>(scratch.list, (uint32_t)list.size(), nseg,
                                                                       scratch.acc);
      e = cudaGetLastError();
    }
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(acc.data(), scratch.acc, acc.size() * sizeof(unsigned long long), cudaMemcpyDeviceToHost, s);
    const cudaError_t es = cudaStreamSynchronize(s);
    if (e == cudaSuccess) e = es;
    if (prev >= 0) cudaSetDevice(prev);
    if (e != cudaSuccess) return fail(WS_ERR_CUDA, std::string("tensor hashes: ") + cudaGetErrorString(e));
  }
  for (uint64_t i = 0; i < n; ++i) out[i] = ws_mix64((uint64_t)(nbytes[i] + 1) * WS_TH_KLEN);
  for (size_t k = 0; k < list.size(); ++k)
    out[owner[k]] = ws_mix64((uint64_t)acc[k] + (uint64_t)(nbytes[owner[k]] + 1) * WS_TH_KLEN);
  return WS_OK;
}

extern "C" int ws_tensor_hashes(const void* const* ptrs, const uint64_t* nbytes, uint64_t n, int device, void* stream,
                                uint64_t* out) {
  return ws::guarded([&] { return ws_tensor_hashes_impl(ptrs, nbytes, n, device, stream, out); });
}
