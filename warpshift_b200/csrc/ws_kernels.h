// Launch helpers for the sm_100a kernels in ws_apply.cu.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "ws_format.h"

namespace ws {

// Shared memory used by one CTA of the decode+apply kernel.
size_t apply_smem_bytes();

// Loads both kernel instantiations on the current device (call once before timing or capture).
cudaError_t prime_kernels();

// Tile kinds present in a launch range (launch_apply's `kinds`).
constexpr uint32_t kTilesWhole = 1u;  // tiles without split-word blocks
constexpr uint32_t kTilesSplit = 2u;  // tiles of packets that split words

// One launch over tiles [tile_begin, tile_begin + ntiles) of the kernel
// instantiation for the tile kinds in `kinds` (whole-word only, split-word
// only, or both), counted in *launched. `payload` is the device address of
// arena byte `payload_offset` (a staging slot or the resident copy); block
// descriptors hold arena offsets.
cudaError_t launch_apply(const ws_tile_desc* tiles, uint32_t tile_begin, uint32_t ntiles,
                         const ws_block_desc* blocks, const uint32_t* tables, const uint8_t* payload,
                         uint64_t payload_offset, ws_device_result* result, int reverse, uint32_t kinds,
                         cudaStream_t stream, uint32_t* launched);

// Records the message returned by ws_last_error() on the calling thread.
void set_last_error(const char* msg);

}  // namespace ws
