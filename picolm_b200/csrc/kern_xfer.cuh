// kern_xfer.cuh -- merge of a KV-split decode over NVLink peer memory.
//
// One long sequence's cache is split along the sequence axis over `world`
// GPUs (one process each).  Per layer every rank holds a partial (m, l, o)
// of n_heads * (head_dim + 4) floats; every rank needs the merge.  Each rank
// owns a receive buffer
//     [uint32 epoch stamp per rank | uint32 own epoch counter at byte 128,
//      padded to 256 B][float slots[2][world][n]]
// mapped into every other rank's address space (CUDA IPC).  One kernel per
// rank and layer:
//   1. stores this rank's partial into slot (epoch & 1, rank) of EVERY
//      rank's buffer (plain stores through the peer mappings, over NVLink);
//   2. after a system-scope fence, stamps `epoch` into stamp[rank] of every
//      buffer (release store).  The epoch is this rank's own counter, kept
//      in its buffer and advanced by the kernel, so a captured CUDA graph
//      replays correctly; all ranks call the merge equally often, so their
//      counters agree;
//   3. waits, bounded, until all stamps in its own buffer reach `epoch`
//      (acquire loads), then merges the world partials of slot parity
//      epoch & 1 in log-sum-exp form (merge_slots).
// Two slot sets alternate by epoch parity: a rank can only write epoch e+2
// after every rank has stamped e+1, i.e. after every rank finished reading
// epoch e, so no slot is overwritten while it is read.  One CTA does the
// whole exchange: one fence and one stamp per peer (measured faster than
// splitting it over a CTA per head).
#pragma once
#include <cstdint>

#include "kern_decode.cuh"

namespace pl {

constexpr int kXferMaxRanks = 8;
constexpr int kXferStampBytes = 256;
constexpr int kXferCounterOffset = 128;  // byte offset of the own epoch counter
constexpr int kXferThreads = 512;

struct XferPeers {
  uint8_t* base[kXferMaxRanks];  // each rank's receive buffer, as seen from this GPU
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// grid 1, block kXferThreads, dynamic smem (3 * kXferMaxRanks + 2) * n_heads floats
template <int HD>
__global__ void __launch_bounds__(kXferThreads) combine_p2p_kernel(
    const float* __restrict__ part, XferPeers peers, int world, int rank, int n_heads,
    float* __restrict__ out, uint32_t* err) {
  extern __shared__ float smem_w[];
  __shared__ int s_ok;
  __shared__ uint32_t s_epoch;
  const int tid = threadIdx.x;
  if (tid == 0) {
    uint32_t* counter = reinterpret_cast<uint32_t*>(peers.base[rank] + kXferCounterOffset);
    s_epoch = *counter + 1;
    *counter = s_epoch;
    s_ok = 1;
  }
  // launched behind the kernels that produce `part` (programmatic dependent
  // launch): everything above overlapped them
  asm volatile("griddepcontrol.wait;" ::: "memory");
  __syncthreads();
  const uint32_t epoch = s_epoch;
  const int n = n_heads * part_stride(HD);  // floats per partial, a multiple of 4
  const int n4 = n / 4;
  const int parity = static_cast<int>(epoch & 1u);
  // 1. this rank's partial into every rank's slot (parity, rank)
  for (int idx = tid; idx < world * n4; idx += blockDim.x) {
    const int gr = idx / n4, i4 = idx - gr * n4;
    const float4 v = __ldcg(reinterpret_cast<const float4*>(part) + i4);
    float* slots = reinterpret_cast<float*>(peers.base[gr] + kXferStampBytes);
    reinterpret_cast<float4*>(slots + (static_cast<size_t>(parity) * world + rank) * n)[i4] = v;
  }
  __threadfence_system();  // the data lands before any stamp says so
  __syncthreads();
  // 2. stamp this epoch in every rank's buffer
  if (tid < world)
    st_release_sys(reinterpret_cast<uint32_t*>(peers.base[tid]) + rank, epoch);
  // 3. wait for every rank's stamp in this rank's buffer (bounded)
  if (tid < world) {
    const uint32_t* stamp = reinterpret_cast<const uint32_t*>(peers.base[rank]) + tid;
    if (static_cast<int>(ld_acquire_sys(stamp) - epoch) < 0) {
      const uint64_t t0 = globaltimer(), lim = wait_limit_ns();
      while (static_cast<int>(ld_acquire_sys(stamp) - epoch) < 0) {
        if (globaltimer() - t0 > lim) {
          atomicOr(err, ERR_TIMEOUT_FULL);
          s_ok = 0;
          break;
        }
      }
    }
  }
  __syncthreads();
  if (!s_ok) return;
  // 4. log-sum-exp merge of the world partials of this epoch
  const float* slots = reinterpret_cast<const float*>(peers.base[rank] + kXferStampBytes) +
                       static_cast<size_t>(parity) * world * n;
  merge_slots<kXferMaxRanks, HD>(slots, static_cast<size_t>(n), world, n_heads, out, nullptr,
                                 smem_w);
}

}  // namespace pl
