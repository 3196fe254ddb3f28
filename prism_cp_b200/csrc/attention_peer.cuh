// Context-parallel tile sources for the tcgen05 attention kernels.
//
// In a zigzag team of `cp` ranks a sequence of n tokens is cut into 2*cp chunks
// of c = n / (2*cp) tokens; rank r owns chunks r and 2*cp-1-r, stored one after
// the other in its local segment for that sequence (the same local row on every
// rank). With every rank's Q/K/V/dO (and LSE, D) in a symmetric heap mapped into
// all peers, an attention kernel reads the tile at global position `pos` straight
// from its owner: tensor maps over the peers' buffers feed plain per-CTA
// TMA loads, and LSE/D rows are read with ordinary loads over NVLink. The KV
// exchange of a ring is thereby part of the attention tile loop itself.
#pragma once

#include <cuda.h>

namespace prism {

constexpr int kMaxPeers = 8;

struct PeerTiles {
  CUtensorMap a[kMaxPeers];      // K (forward, dQ kernel) or Q (dK/dV kernel), per owner
  CUtensorMap b[kMaxPeers];      // V (forward, dQ kernel) or dO (dK/dV kernel), per owner
  const float* lse[kMaxPeers];   // [hq, tq] per owner (dK/dV kernel)
  const float* dsum[kMaxPeers];  // [hq, tq] per owner (dK/dV kernel)
  const int* seq_n;              // [nseq] global sequence length (a multiple of 256 * cp)
  const int* seq_row0;           // [nseq] first local row of each sequence segment
  int cp;
};

struct NoPeers {
  int unused;
};

// Local row on the owning rank of global position `pos` (a multiple of 128) of sequence `seq`.
__device__ __forceinline__ int peer_row(const PeerTiles& pt, int seq, int pos, int& owner) {
  const int c = pt.seq_n[seq] / (2 * pt.cp);
  const int ci = pos / c;
  const bool first = ci < pt.cp;
  owner = first ? ci : 2 * pt.cp - 1 - ci;
  return pt.seq_row0[seq] + (first ? 0 : c) + (pos - ci * c);
}

}  // namespace prism
