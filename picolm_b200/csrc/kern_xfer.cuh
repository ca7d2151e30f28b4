// kern_xfer.cuh -- merge of a KV-split decode over NVLink peer memory.
//
// One long sequence's cache is split along the sequence axis over `world`
// GPUs (one process each).  Per layer every rank holds a partial (m, l, o)
// of n_heads * (head_dim + 4) floats; every rank needs the merge.  The
// exchange is the flag-in-data protocol described with XferPeers in
// kern_decode.cuh: each value crosses NVLink once, in a 16-byte store that
// carries the merge's epoch beside it, and the reader polls its own buffer
// until the epoch shows (bounded).  No fence and no separate stamp: with a
// system-scope fence and an epoch stamp per rank, one exchange took about
// 10.5 us per layer between two B200s.
//
// combine_p2p_kernel does the exchange for a partial that
// pl_attn_decode_partial_dev wrote; pl_attn_decode_p2p_dev leaves it to the
// merge grid of the partial itself (merge_kernel<HD, true>), one launch
// fewer.
#pragma once
#include <cstdint>

#include "kern_decode.cuh"

namespace pl {

constexpr int kXferThreads = 512;

// grid 1, block kXferThreads: thread t owns (head, float4 q4) pairs
// t, t + kXferThreads, ...; it pushes them all, then merges them.
template <int HD>
__global__ void __launch_bounds__(kXferThreads) combine_p2p_kernel(
    const float* __restrict__ part, XferPeers peers, int world, int rank, int n_heads,
    float* __restrict__ out, uint32_t* err) {
  __shared__ uint32_t s_epoch;
  const int tid = threadIdx.x;
  if (tid == 0) {
    uint32_t* counter = reinterpret_cast<uint32_t*>(peers.base[rank] + kXferCounterOffset);
    s_epoch = *counter + 1;
    *counter = s_epoch;
  }
  // launched behind the kernels that produce `part` (programmatic dependent
  // launch): everything above overlapped them
  asm volatile("griddepcontrol.wait;" ::: "memory");
  __syncthreads();
  const uint32_t epoch = s_epoch;
  constexpr int PS = part_stride(HD);
  const int pairs = n_heads * (HD / 4);
  for (int idx = tid; idx < pairs; idx += kXferThreads) {
    const int h = idx / (HD / 4), q4 = idx % (HD / 4);
    const float* p = part + static_cast<size_t>(h) * PS;
    const float2 ml = __ldcg(reinterpret_cast<const float2*>(p));
    const float4 o = __ldcg(reinterpret_cast<const float4*>(p + kPartO) + q4);
    ll_push<HD>(peers, world, rank, n_heads, epoch, h, q4, ml.x, ml.y, o);
  }
  for (int idx = tid; idx < pairs; idx += kXferThreads) {
    const int h = idx / (HD / 4), q4 = idx % (HD / 4);
    if (!ll_merge<HD>(peers, world, rank, n_heads, epoch, h, q4, out)) {
      atomicOr(err, ERR_TIMEOUT_FULL);
      return;
    }
  }
}

}  // namespace pl
