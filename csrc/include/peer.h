// Peer windows shared by the communication kernels (peer.cu) and the GEMMs that
// move their operands or results over NVLink themselves (comm_gemm.cu).
#pragma once

#include <cstdint>

namespace ns {

constexpr int MAX_PEERS = 8;

struct PeerTable {
  uint64_t base[MAX_PEERS];  // window base address of each rank, as seen from this rank
};

struct WindowInfo {
  PeerTable table;
  int rank, world;
  int64_t bytes;
};

// The opened window `id` (window_create + window_open); throws if it is closed.
WindowInfo window_info(int64_t id);

}  // namespace ns
