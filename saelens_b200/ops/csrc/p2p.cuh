// Peer addressing for the NVLink kernels.
//
// Every rank owns one "symmetric slab": a cudaMalloc allocation of the same size whose IPC
// handle every other rank of the group has opened (saelens_b200/parallel/symm_heap.py).
// Buffers inside a slab are placed at identical byte offsets on every rank, so a peer buffer is
// addressed as `base[peer] + offset`.  Kernels store into peers' slabs directly (NVLink P2P
// stores through NVSwitch) and signal with the release/acquire flag helpers of common.cuh.
#pragma once

#include <stdint.h>

#include <vector>

namespace sb {
namespace p2p {

constexpr int kMaxRanks = 8;

struct Peers {
  uint64_t base[kMaxRanks];  // byte address of rank r's slab, as mapped in this process
  int rank;
  int world;
};

template <class T>
__device__ __forceinline__ T* at(const Peers& P, int r, int64_t byte_off) {
  return reinterpret_cast<T*>(P.base[r] + uint64_t(byte_off));
}

inline Peers make_peers(const std::vector<int64_t>& bases, int64_t rank) {
  Peers P{};
  const int n = int(bases.size());
  for (int i = 0; i < n && i < kMaxRanks; ++i) P.base[i] = uint64_t(bases[i]);
  P.rank = int(rank);
  P.world = n;
  return P;
}

}  // namespace p2p
}  // namespace sb
