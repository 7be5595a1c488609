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

// Encodes every packet on the current device; results are identical to
// encode_packet() on the same bytes. Returns false with *err set on a CUDA error.
bool gpu_encode_packets(const std::vector<GpuPacketInput>& packets, int policy, int dict_slack_pct,
                        uint64_t batch_bytes, cudaStream_t stream, std::vector<EncodedPacket>* out, std::string* err);

}  // namespace ws
