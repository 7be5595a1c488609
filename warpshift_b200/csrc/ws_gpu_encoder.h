// GPU encoder for prepare (ws_gpu_encoder.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <vector>

#include "ws_encoder.h"

namespace ws {

struct GpuPacketInput {
  const uint8_t* base;    // host bytes of A (cpu_base)
  const uint8_t* target;  // device bytes of B (resident weights)
  uint64_t nbytes;
  bool is_bf16;
};

// One host piece of the delta arena: the payloads of consecutive packets' blocks,
// in packet and block order, covering arena bytes [off, off + bytes).
struct ArenaChunk {
  uint8_t* ptr;
  uint64_t off;
  uint64_t bytes;
  bool pinned;
};

// NUMA node that `device`'s PCIe link attaches to (sysfs numa_node), or -1
// when the host reports none.
int device_numa_node(int device);
// Asks the kernel to place the pages of [p, p + size) on `node` while it has
// free memory (mbind MPOL_PREFERRED, before the pages are first touched).
// Advisory: returns false, changing nothing, when the host refuses.
bool prefer_numa_node(void* p, uint64_t size, int node);

// Allocates `bytes` of host memory for an arena chunk; with `pinned` it is
// page-locked (transparent huge pages, placed on the current device's NUMA
// node, first touch on up to `threads` threads, then cudaHostRegister: about
// ten times faster than cudaHostAlloc's 4 KiB page faults). Returns false
// with *err set.
bool alloc_host_chunk(uint64_t bytes, bool pinned, int threads, ArenaChunk* out, std::string* err);
void free_host_chunk(const ArenaChunk& chunk);

// Encodes every packet on the current device; the packets, blocks, tables and
// payload bytes are identical to encode_packet() on the same bytes. Block
// payloads are not stored in EncodedBlock::payload (only their size, `clen`):
// they are copied, in arena order, into host chunks appended to *chunks
// (pinned when `pin` is set; the caller frees them, also after a failure).
// Pageable A bytes are staged through pinned buffers by up to `threads` host
// threads. Returns false with *err set on a CUDA or allocation error;
// *device_oom tells whether a device allocation was what failed (the caller may
// retry with smaller batches).
bool gpu_encode_packets(const std::vector<GpuPacketInput>& packets, int policy, const CodingOptions& co,
                        uint64_t batch_bytes, int threads, bool pin, cudaStream_t stream,
                        std::vector<EncodedPacket>* out, std::vector<ArenaChunk>* chunks, std::string* err,
                        bool* device_oom);

}  // namespace ws
