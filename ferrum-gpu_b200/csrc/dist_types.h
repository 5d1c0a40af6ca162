// Pointer tables of the peer-memory path of the distributed 2D transform,
// shared by its kernels (dist_kernels.cuh) and the host code (dist.cu).
#pragma once

#include <stdint.h>

#include <vector_types.h>

namespace ferrum {

// Ranks one node's peer path supports (one NVSwitch domain of 8 GPUs).
constexpr int kMaxPeers = 8;

// Per-rank base pointers, passed to kernels by value.
struct PeerPtrs {
  float2* p[kMaxPeers];
};

struct PeerFlags {
  uint32_t* p[kMaxPeers];
};

}  // namespace ferrum
