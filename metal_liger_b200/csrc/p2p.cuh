// Peer-memory exchange of the vocabulary-parallel FLCE's dX (p2p.cu): the
// exchange-buffer layout and the flag signal, shared with flce.cu, whose dX
// GEMM stores into the row owners' receive slots.
#pragma once

#include "gemm.cuh"

namespace ml {
namespace p2p {

constexpr int kMax = gemm::kMaxPeers;

// Every rank's exchange buffer as mapped on this GPU (own included).
struct Peers {
  uint8_t* ws[kMax];
};

struct XLayout {
  int64_t rows_per_owner = 0;  // multiple of 256: a GEMM tile never straddles two owners
  size_t off_recv = 0, off_gather = 0, off_stats = 0, total = 0;
};

XLayout xlayout(int world, int64_t chunk_cap, int64_t h);

// Validates the peer table (world <= kMax, 256-byte aligned buffers).
int check_peers(int world, int rank, void* const* peer_ws, Peers& pe);

// flags[which * kMax + me] = epoch on every rank (which 0: arrive, 1: done,
// 2: stats),
// release stores at system scope after a system fence.
int launch_signal(const Peers& pe, int world, int me, int which, int64_t epoch, cudaStream_t st);

}  // namespace p2p
}  // namespace ml
