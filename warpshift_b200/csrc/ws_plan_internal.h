// Internal plan structure shared by the plan runtime (ws_plan.cpp) and plan
// persistence (ws_persist.cpp). Not part of the C ABI.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <vector>

#include "../../include/warpshift_b200.h"
#include "ws_format.h"
#include "ws_gpu_encoder.h"

namespace ws {

struct Batch {
  uint32_t tile_begin, tile_end;
  uint64_t arena_off, bytes;
  uint32_t chunk;  // arena chunk holding the whole batch
  uint32_t kinds;  // kTilesWhole | kTilesSplit: the tile kinds in the batch (one kernel launch each)
};

}  // namespace ws

struct ws_plan {
  ws_build_options opts{};
  int device = -1;
  std::vector<ws_block_desc> blocks;
  std::vector<uint32_t> block_tensor;  // tensor index of each block (rebasing saved plans)
  std::vector<uint64_t> tensor_bytes;  // per tensor, in call order
  std::vector<uint8_t> tensor_bf16;
  std::vector<uint64_t> tensor_target; // target addresses the block descriptors point into
  std::vector<ws_tile_desc> tiles;
  std::vector<uint32_t> tables;
  std::vector<ws::Batch> batches;
  std::vector<ws::ArenaChunk> chunks;  // host arena: every block payload in block order
  uint64_t arena_bytes = 0;
  uint8_t* view_arena = nullptr;       // contiguous copy made by ws_plan_get_view for a multi-chunk arena
  ws_plan_stats stats{};

  bool uploaded = false;
  ws_block_desc* d_blocks = nullptr;
  ws_tile_desc* d_tiles = nullptr;
  uint32_t* d_tables = nullptr;
  std::vector<uint8_t*> d_slots;
  uint64_t slot_bytes = 0;
  uint8_t* d_resident = nullptr;
  ws_device_result* d_result = nullptr;
  ws_device_result* h_result = nullptr;
  std::vector<cudaEvent_t> copy_done, compute_done;
  cudaEvent_t start_event = nullptr;
  cudaEvent_t aux_done = nullptr;        // end of the second compute stream's work
  cudaStream_t own_copy_stream = nullptr;
  cudaStream_t aux_stream = nullptr;     // runs every other staging batch's kernel
  cudaEvent_t done_event = nullptr;      // recorded after each apply's last operation

  int pending_reverse = -1;
  uint64_t pending_h2d = 0;
  uint32_t pending_launches = 0;
};

namespace ws {

// Splits the tiles into staging batches (contiguous tiles of one arena chunk,
// payload <= opts.batch_bytes) and fills the plan's batch count.
int form_batches(ws_plan* p, std::string* err);
// Frees everything a plan holds (device and host).
void free_plan_resources(ws_plan* p);
int host_threads(int requested);

}  // namespace ws
