// The fused exchange of a layer sharded over the ranks of one node (kGatherPeers / kReducePeers,
// PeerSet in kernels.h), shared by the GEMV kernels that implement it: every rank's CTAs store
// their outputs into the other ranks' exchange buffers over NVLink as 64-bit words tagged with the
// call number, and read the words they need once the tags show this call.
#pragma once

#include "common.cuh"
#include "kernels.h"

namespace i4 {

// Call number of this exchange: one more than the last completed call that used these buffers
// (counters[0] of this rank). Read by every consumer thread at the same point, after the
// dependency wait (so the previous call's update is visible), and followed by a barrier before
// any thread of the CTA can reach exchange_done.
__device__ __forceinline__ unsigned exchange_epoch(const PeerSet& peers) {
  return __ldcg(peers.counters) + 1u;
}

// The last CTA of the call to finish (counters[1] counts them) records `epoch` as the last
// completed call. One global number per call, whatever the shapes of earlier calls on the same
// buffers, so a word left by an earlier call of the same parity always carries an older tag.
__device__ __forceinline__ void exchange_done(const PeerSet& peers, unsigned epoch, int tid) {
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(peers.counters + 1, 1u) == gridDim.x - 1) {
      peers.counters[1] = 0;
      peers.counters[0] = epoch;
      __threadfence();
    }
  }
}

// The exchange words of this call: rank q's buffer, this call's half, as tagged 64-bit words.
__device__ __forceinline__ unsigned long long* exchange_words(const PeerSet& peers, int q,
                                                              unsigned epoch) {
  return reinterpret_cast<unsigned long long*>(static_cast<char*>(peers.out[q]) +
                                               (epoch & 1u) * peers.out_half);
}

// Reads the data of a tagged word of this call; after a wait has run out (*live false) it stops
// waiting and the kernel's result is undefined (status kStatusPeerTimeout).
__device__ __forceinline__ unsigned exchange_read(const unsigned long long* w, unsigned epoch,
                                                  bool* live, int* status) {
  unsigned data = static_cast<unsigned>(ld_tagged(w));
  if (*live && !wait_tagged(w, epoch, &data, kPeerWaitNs)) {
    *live = false;
    atomicExch(status, kStatusPeerTimeout);
  }
  return data;
}

}  // namespace i4
