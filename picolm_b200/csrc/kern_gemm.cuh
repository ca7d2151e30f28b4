// kern_gemm.cuh -- the projections of a prefill (many input rows) as
// tcgen05 GEMMs: C[M][N] = X[M][K] W[N][K]^T (+ bias, + residual), the
// batched matmuls picolm runs on the CPU for a prompt (model.c:993-1000,
// matmul_batch / matmul_dual_batch, tensor.c:323-419; output projection
// model.c:1092-1100).
//
// Accuracy.  picolm sums in FP32 over FP32 inputs and weights dequantised in
// FP32.  The tensor cores take FP16 operands, so both sides are carried as a
// high part and a residual:
//     w = w_hi + 2^-11 w_lo,   x = x_hi + 2^-11 x_lo    (all four FP16)
// with w_hi the FP16 rounding of w and w_lo the FP16 rounding of
// (w - w_hi) * 2^11, which keeps the residual in FP16's normal range.  Three
// MMAs per k-step accumulate in FP32 in tensor memory:
//     acc0 += x_hi w_hi,   acc1 += x_lo w_hi + x_hi w_lo
// and the epilogue forms acc0 + 2^-11 acc1.  The dropped x_lo w_lo term is
// 2^-22 of the product, below FP32 rounding of the sums.  Weights are
// dequantised once, when a layer is uploaded, from any GGUF type the module
// takes (dequant_split_kernel, the dequantize_row_* formulas of
// quant.c:96-222); activations are split per call (act_split_kernel, with
// the layer's RMSNorm applied on the way for the Q/K/V projections).
//
// Kernel.  One CTA computes one 128 x 128 output tile over the whole K:
//   warp 0   one lane streams the four operand tiles of each 64-wide k-step
//            (x_hi, x_lo, w_hi, w_lo; 16 KB each, 128-byte swizzle) with 2-D
//            TMA loads into a kGmStages-deep ring;
//   warp 1   one lane issues the three MMAs per 16-wide k-slice
//            (tcgen05.mma kind::f16, M128 N128) and frees each stage with a
//            tcgen05.commit;
//   warp 2   allocates the 256 TMEM columns (acc0, acc1) and frees them;
//   warps 0-3 read their 32 accumulator rows back (tcgen05.ld) and write
//            the FP32 outputs (bias, residual added).
// Every mbarrier wait is bounded; a wait that gives up sets an error bit and
// the CTA winds down (it still waits for its own copies and MMAs, then frees
// its tensor memory).
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>

#include "kern_proj.cuh"
#include "sm100.cuh"

namespace pl {

constexpr int kGmBM = 128;      // output rows per tile (TMEM lanes)
constexpr int kGmBN = 128;      // output columns per tile
constexpr int kGmBK = 64;       // k per stage: 128 bytes of FP16, one swizzle span
constexpr int kGmStages = 3;
constexpr int kGmThreads = 128;
constexpr int kGmTile = kGmBM * kGmBK * 2;  // bytes of one operand tile (16 KB)
constexpr float kGmLoScale = 2048.0f;       // 2^11
constexpr float kGmLoInv = 1.0f / 2048.0f;
// The GEMM paths from this many input rows (the skinny kernel up to
// kSkMaxRows, gemm_hilo_kernel above).  Fewer rows stream the quantised
// weights on CUDA cores / mma.sync (kern_proj.cuh): one row took 19.6 us
// there against 31.7 us on the skinny GEMM, 64 rows 64.5 against 37.8 us.
constexpr int kGmMinRows = 24;

// The weight parts are stored tiled: the 128 x 64 tile of weight rows
// [128 t, 128 t + 128) and k-step kb (64 inputs) is one contiguous 16 KB
// block, block t * kb_all + kb of a [blocks * 128][64] array, so each TMA
// box is one burst of DRAM instead of 128 pieces of 128 bytes 2 K (or
// 4 KB) apart.  First row of that block in the [blocks * 128][64] view:
__host__ __device__ __forceinline__ int wtile_row(int row0, int kb, int kb_all) {
  return ((row0 / kGmBN) * kb_all + kb) * kGmBN;
}

// Output columns [col0, col0 + cols) of the GEMM go to out[m * ld + n - col0]
// with bias[n - col0] (nullptr: none).  Q, K and V are three segments of one
// GEMM over their concatenated weight rows; each segment is a whole number
// of 128-column tiles.
struct GemmSeg {
  float* out;
  const float* bias;
  int col0, cols, ld;
};

struct GemmArgs {
  int M, N, K;
  int w_row0;          // first weight row of output column 0 (a sub-range of the rows)
  GemmSeg seg[3];
  int n_seg;
  const float* resid;  // when set: out = resid + (x W^T + b), same indexing as seg 0's out
  int ld_res;
  uint32_t* err;
};

struct GmSmem {
  uint8_t xh[kGmStages][kGmTile];
  uint8_t xl[kGmStages][kGmTile];
  uint8_t wh[kGmStages][kGmTile];
  uint8_t wl[kGmStages][kGmTile];
  uint64_t full[kGmStages], empty[kGmStages];
  uint64_t done;
  uint32_t tmem_base;
};

constexpr int gm_smem_bytes() { return static_cast<int>(sizeof(GmSmem)) + 1024; }
static_assert(gm_smem_bytes() <= 227 * 1024, "GEMM shared memory above the limit");

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* m, uint64_t* bar,
                                            int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

__global__ void __launch_bounds__(kGmThreads, 1)
    gemm_hilo_kernel(const GemmArgs a, const __grid_constant__ CUtensorMap tm_xh,
                     const __grid_constant__ CUtensorMap tm_xl,
                     const __grid_constant__ CUtensorMap tm_wh,
                     const __grid_constant__ CUtensorMap tm_wl) {
  extern __shared__ uint8_t smem_raw[];
  GmSmem& sm = *reinterpret_cast<GmSmem*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kGmBN, m0 = blockIdx.y * kGmBM;
  const int kb_n = a.K / kGmBK;

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tm_xh);
    tma_prefetch_desc(&tm_xl);
    tma_prefetch_desc(&tm_wh);
    tma_prefetch_desc(&tm_wl);
    for (int s = 0; s < kGmStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    mbar_init(&sm.done, 1);
    fence_mbar_init();
  }
  if (warp == 2) {
    tmem_alloc(&sm.tmem_base, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  bool ok = true;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer
    int issued = 0;
    for (int kb = 0; kb < kb_n; ++kb) {
      const int s = kb % kGmStages;
      if (kb >= kGmStages && !mbar_wait_bounded(&sm.empty[s], ((kb / kGmStages) - 1) & 1)) {
        atomicOr(a.err, ERR_TIMEOUT_EMPTY);
        break;
      }
      mbar_arrive_expect_tx(&sm.full[s], 4u * kGmTile);
      const int k0 = kb * kGmBK;
      tma_load_2d(sm.xh[s], &tm_xh, &sm.full[s], k0, m0);
      tma_load_2d(sm.xl[s], &tm_xl, &sm.full[s], k0, m0);
      tma_load_2d(sm.wh[s], &tm_wh, &sm.full[s], 0, wtile_row(a.w_row0 + n0, kb, kb_n));
      tma_load_2d(sm.wl[s], &tm_wl, &sm.full[s], 0, wtile_row(a.w_row0 + n0, kb, kb_n));
      ++issued;
    }
    // never leave with copies in flight: the last use of each stage must land
    for (int j = issued - kGmStages; j < issued; ++j)
      if (j >= 0) mbar_wait_bounded(&sm.full[j % kGmStages], (j / kGmStages) & 1);
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------ MMA issuer
    const uint32_t idesc = idesc_f16_f32(kGmBM, kGmBN, 0);
    const uint32_t acc0 = tmem, acc1 = tmem + kGmBN;
    for (int kb = 0; kb < kb_n; ++kb) {
      const int s = kb % kGmStages;
      if (!mbar_wait_bounded(&sm.full[s], (kb / kGmStages) & 1)) {
        atomicOr(a.err, ERR_TIMEOUT_FULL);
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t xh = smem_u32(sm.xh[s]), xl = smem_u32(sm.xl[s]);
      const uint32_t wh = smem_u32(sm.wh[s]), wl = smem_u32(sm.wl[s]);
#pragma unroll
      for (int kk = 0; kk < kGmBK / 16; ++kk) {  // 16 k per MMA, 32 bytes into the swizzle span
        const uint32_t o = kk * 32;
        const uint64_t dxh = smem_desc_sw128(xh + o, 16, 1024);
        const uint64_t dxl = smem_desc_sw128(xl + o, 16, 1024);
        const uint64_t dwh = smem_desc_sw128(wh + o, 16, 1024);
        const uint64_t dwl = smem_desc_sw128(wl + o, 16, 1024);
        const uint32_t accum = (kb > 0 || kk > 0) ? 1u : 0u;
        tc_mma_ss(acc0, dxh, dwh, idesc, accum);
        tc_mma_ss(acc1, dxl, dwh, idesc, accum);
        tc_mma_ss(acc1, dxh, dwl, idesc, 1u);
      }
      tc_commit(&sm.empty[s]);  // the stage is free once these MMAs have read it
    }
    tc_commit(&sm.done);  // after every MMA issued above (also on the error path)
  }
  __syncwarp();

  // ---------------------------------------------------------------- epilogue
  // every warp: its 32 TMEM lanes = output rows m0 + 32*warp + lane
  if (!mbar_wait_bounded(&sm.done, 0)) {
    if (lane == 0) atomicOr(a.err, ERR_TIMEOUT_MMA);
    ok = false;
  }
  tc_fence_after();
  // the tile's output segment (a tile never straddles two)
  int si = 0;
  for (int i = 1; i < a.n_seg; ++i)
    if (n0 >= a.seg[i].col0) si = i;
  const GemmSeg seg = a.seg[si];
  const int c0 = n0 - seg.col0;
  const int m = m0 + 32 * warp + lane;
  const uint32_t lane_base = tmem + (static_cast<uint32_t>(32 * warp) << 16);
  const bool any_err = __any_sync(0xffffffffu, !ok);
#pragma unroll 1
  for (int c = 0; c < kGmBN; c += 32) {
    uint32_t r0[32], r1[32];
    tc_ld_32x32b_x32(lane_base + c, r0);
    tc_ld_32x32b_x32(lane_base + kGmBN + c, r1);
    tc_wait_ld();
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      asm volatile("" : "+r"(r0[i]));
      asm volatile("" : "+r"(r1[i]));
    }
    if (any_err || m >= a.M) continue;
    float* dst = seg.out + static_cast<size_t>(m) * seg.ld + c0 + c;
    const float* res = a.resid ? a.resid + static_cast<size_t>(m) * a.ld_res + c0 + c : nullptr;
#pragma unroll
    for (int i = 0; i < 32; i += 4) {
      float4 y;
      y.x = __uint_as_float(r0[i]) + __uint_as_float(r1[i]) * kGmLoInv;
      y.y = __uint_as_float(r0[i + 1]) + __uint_as_float(r1[i + 1]) * kGmLoInv;
      y.z = __uint_as_float(r0[i + 2]) + __uint_as_float(r1[i + 2]) * kGmLoInv;
      y.w = __uint_as_float(r0[i + 3]) + __uint_as_float(r1[i + 3]) * kGmLoInv;
      if (seg.bias) {
        const float4 b = __ldg(reinterpret_cast<const float4*>(seg.bias + c0 + c + i));
        y.x += b.x;
        y.y += b.y;
        y.z += b.z;
        y.w += b.w;
      }
      if (res) {
        const float4 r = *reinterpret_cast<const float4*>(res + i);
        y.x = r.x + y.x;
        y.y = r.y + y.y;
        y.z = r.z + y.z;
        y.w = r.w + y.w;
      }
      *reinterpret_cast<float4*>(dst + i) = y;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// ---- few input rows (batched decode): the weights as the A operand -------
// With M <= kSkMaxRows input rows a 128-row tile of x would be mostly
// padding.  Here the 128 weight rows of an output tile are the A operand
// (M = 128 output columns on the TMEM lanes) and the input rows are B
// (N = M rounded up to 16), so D = [output column][input row] and no lane
// is wasted.  The producer, the ring and the three MMAs per k-slice are
// those of gemm_hilo_kernel with A and B exchanged, with x in 64-row TMA
// boxes (rows past M arrive as zeros, outside the tensor; only the first N
// feed the MMA), so a stage is 48 KB and kSkStages of them fit.  The epilogue writes D transposed: thread
// (warp w, lane l) holds output column n0 + 32w + l for every input row, so
// for each row a warp stores 32 consecutive floats (128 contiguous bytes).
//
// N / 128 tiles alone leave most SMs idle (20 for the Q/K/V rows of a
// 2048-wide layer), and one SM streams a tile's 1 MB of weight parts at
// only about 45 GB/s, so K is split over the gridDim.y CTAs of a tile,
// which form one thread-block cluster (rank = split).  Each CTA keeps its
// FP32 partial tile [kSkMaxRows][128] in its own shared memory (the idle
// operand ring); after a cluster barrier, CTA r sums rows [r M / S,
// (r + 1) M / S) of the tile over all S partials through distributed shared
// memory, in split order (the same order on every run, whichever CTA
// finishes first), adds bias and residual and stores them; a second
// cluster barrier keeps every CTA's shared memory alive until all reads are
// done.  grid = (N / 128, S), cluster (1, S, 1) with S <= 8, block =
// kGmThreads.
constexpr int kSkMaxRows = 64;
constexpr int kSkMaxSplit = 8;
constexpr int kSkStages = 4;                  // ring depth: most of a CTA's k-steps in flight
constexpr int kSkXTile = kSkMaxRows * kGmBK * 2;  // bytes of one 64-row x tile (8 KB)

struct SkSmem {
  uint8_t wh[kSkStages][kGmTile];
  uint8_t wl[kSkStages][kGmTile];
  uint8_t xh[kSkStages][kSkXTile];
  uint8_t xl[kSkStages][kSkXTile];
  uint64_t full[kSkStages], empty[kSkStages];
  uint64_t done;
  uint32_t tmem_base;
};

constexpr int sk_smem_bytes() { return static_cast<int>(sizeof(SkSmem)) + 1024; }
static_assert(sk_smem_bytes() <= 227 * 1024, "skinny GEMM shared memory above the limit");
static_assert(2 * kGmTile >= kSkMaxRows * kGmBM * 4, "partial tile must fit two weight tiles");

__global__ void __launch_bounds__(kGmThreads, 1)
    gemm_skinny_kernel(const GemmArgs a, const __grid_constant__ CUtensorMap tm_xh,
                       const __grid_constant__ CUtensorMap tm_xl,
                       const __grid_constant__ CUtensorMap tm_wh,
                       const __grid_constant__ CUtensorMap tm_wl) {
  extern __shared__ uint8_t smem_raw[];
  SkSmem& sm = *reinterpret_cast<SkSmem*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kGmBM;
  const int n_split = gridDim.y, split = blockIdx.y;
  const int kb_all = a.K / kGmBK;
  const int kb_lo = split * kb_all / n_split, kb_hi = (split + 1) * kb_all / n_split;
  const int kb_n = kb_hi - kb_lo;  // k-steps of this CTA (at least one)
  const int nx = (a.M + 15) & ~15;  // MMA N: the input rows, rounded up to 16

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tm_xh);
    tma_prefetch_desc(&tm_xl);
    tma_prefetch_desc(&tm_wh);
    tma_prefetch_desc(&tm_wl);
    for (int s = 0; s < kSkStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    mbar_init(&sm.done, 1);
    fence_mbar_init();
  }
  if (warp == 2) {
    tmem_alloc(&sm.tmem_base, 128);  // acc0 at columns [0, 64), acc1 at [64, 128)
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  bool ok = true;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer
    // Launched behind act_split_kernel with programmatic dependent launch:
    // the weight tiles of the first stages load before griddepcontrol.wait
    // (they do not depend on that kernel), the activations after it.
    const int pre = kb_n < kSkStages ? kb_n : kSkStages;
    for (int kb = 0; kb < pre; ++kb) {
      mbar_arrive_expect_tx(&sm.full[kb], 2u * kGmTile + 2u * kSkXTile);
      const int wr = wtile_row(a.w_row0 + n0, kb_lo + kb, kb_all);
      tma_load_2d(sm.wh[kb], &tm_wh, &sm.full[kb], 0, wr);
      tma_load_2d(sm.wl[kb], &tm_wl, &sm.full[kb], 0, wr);
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
    for (int kb = 0; kb < pre; ++kb) {
      const int k0 = (kb_lo + kb) * kGmBK;
      tma_load_2d(sm.xh[kb], &tm_xh, &sm.full[kb], k0, 0);
      tma_load_2d(sm.xl[kb], &tm_xl, &sm.full[kb], k0, 0);
    }
    int issued = pre;
    for (int kb = pre; kb < kb_n; ++kb) {
      const int s = kb % kSkStages;
      if (!mbar_wait_bounded(&sm.empty[s], ((kb / kSkStages) - 1) & 1)) {
        atomicOr(a.err, ERR_TIMEOUT_EMPTY);
        break;
      }
      mbar_arrive_expect_tx(&sm.full[s], 2u * kGmTile + 2u * kSkXTile);
      const int k0 = (kb_lo + kb) * kGmBK;
      const int wr = wtile_row(a.w_row0 + n0, kb_lo + kb, kb_all);
      tma_load_2d(sm.wh[s], &tm_wh, &sm.full[s], 0, wr);
      tma_load_2d(sm.wl[s], &tm_wl, &sm.full[s], 0, wr);
      tma_load_2d(sm.xh[s], &tm_xh, &sm.full[s], k0, 0);
      tma_load_2d(sm.xl[s], &tm_xl, &sm.full[s], k0, 0);
      ++issued;
    }
    for (int j = issued - kSkStages; j < issued; ++j)
      if (j >= 0) mbar_wait_bounded(&sm.full[j % kSkStages], (j / kSkStages) & 1);
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------ MMA issuer
    const uint32_t idesc = idesc_f16_f32(kGmBM, nx, 0);
    const uint32_t acc0 = tmem, acc1 = tmem + kSkMaxRows;
    for (int kb = 0; kb < kb_n; ++kb) {
      const int s = kb % kSkStages;
      if (!mbar_wait_bounded(&sm.full[s], (kb / kSkStages) & 1)) {
        atomicOr(a.err, ERR_TIMEOUT_FULL);
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t xh = smem_u32(sm.xh[s]), xl = smem_u32(sm.xl[s]);
      const uint32_t wh = smem_u32(sm.wh[s]), wl = smem_u32(sm.wl[s]);
#pragma unroll
      for (int kk = 0; kk < kGmBK / 16; ++kk) {
        const uint32_t o = kk * 32;
        const uint64_t dxh = smem_desc_sw128(xh + o, 16, 1024);
        const uint64_t dxl = smem_desc_sw128(xl + o, 16, 1024);
        const uint64_t dwh = smem_desc_sw128(wh + o, 16, 1024);
        const uint64_t dwl = smem_desc_sw128(wl + o, 16, 1024);
        const uint32_t accum = (kb > 0 || kk > 0) ? 1u : 0u;
        tc_mma_ss(acc0, dwh, dxh, idesc, accum);
        tc_mma_ss(acc1, dwh, dxl, idesc, accum);
        tc_mma_ss(acc1, dwl, dxh, idesc, 1u);
      }
      tc_commit(&sm.empty[s]);
    }
    tc_commit(&sm.done);
  }
  __syncwarp();

  // ---------------------------------------------------------------- epilogue
  if (!mbar_wait_bounded(&sm.done, 0)) {
    if (lane == 0) atomicOr(a.err, ERR_TIMEOUT_MMA);
    ok = false;
  }
  tc_fence_after();
  asm volatile("griddepcontrol.wait;" ::: "memory");  // before any global store
  int si = 0;
  for (int i = 1; i < a.n_seg; ++i)
    if (n0 >= a.seg[i].col0) si = i;
  const GemmSeg seg = a.seg[si];
  const int col = n0 - seg.col0 + 32 * warp + lane;  // this thread's output column in seg
  const float bias = seg.bias ? __ldg(seg.bias + col) : 0.f;
  const uint32_t lane_base = tmem + (static_cast<uint32_t>(32 * warp) << 16);
  const bool any_err = __any_sync(0xffffffffu, !ok);
  if (n_split == 1) {
#pragma unroll 1
    for (int c = 0; c < nx; c += 32) {
      uint32_t r0[32], r1[32];
      tc_ld_32x32b_x32(lane_base + c, r0);
      tc_ld_32x32b_x32(lane_base + kSkMaxRows + c, r1);
      tc_wait_ld();
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        asm volatile("" : "+r"(r0[i]));
        asm volatile("" : "+r"(r1[i]));
      }
      if (any_err) continue;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int m = c + i;
        if (m < a.M) {
          float y = __uint_as_float(r0[i]) + __uint_as_float(r1[i]) * kGmLoInv;
          if (seg.bias) y += bias;
          if (a.resid) y = a.resid[static_cast<size_t>(m) * a.ld_res + col] + y;
          seg.out[static_cast<size_t>(m) * seg.ld + col] = y;
        }
      }
    }
  } else {
    // every role loop has ended (the producer waited for its last copies):
    // the ring is idle, and its first two weight tiles take this CTA's
    // partial tile
    __syncthreads();
    float* P = reinterpret_cast<float*>(sm.wh[0]);  // [kSkMaxRows][kGmBM], 32 KB
    const int fr = 32 * warp + lane;
#pragma unroll 1
    for (int c = 0; c < nx; c += 32) {
      uint32_t r0[32], r1[32];
      tc_ld_32x32b_x32(lane_base + c, r0);
      tc_ld_32x32b_x32(lane_base + kSkMaxRows + c, r1);
      tc_wait_ld();
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (c + i < nx)
          P[(c + i) * kGmBM + fr] = __uint_as_float(r0[i]) + __uint_as_float(r1[i]) * kGmLoInv;
    }
    cluster_sync_all();
    const int m_lo = split * a.M / n_split, m_hi = (split + 1) * a.M / n_split;
    // thread: float4 q4 of the tile's 128 columns, rows m_lo + rg, + 4, ...
    // up to kSkRows rows at a time, all their remote loads (16 bytes each)
    // issued before any is summed
    const int q4 = threadIdx.x & 31, rg = threadIdx.x >> 5;
    const int col4 = n0 - seg.col0 + 4 * q4;
    float4 b4 = make_float4(0.f, 0.f, 0.f, 0.f);
    if (seg.bias) b4 = __ldg(reinterpret_cast<const float4*>(seg.bias + col4));
    const uint32_t p_own = smem_u32(P) + 16u * q4;
    constexpr int kSkRows = 3;
#pragma unroll 1
    for (int m0 = m_lo + rg; m0 < m_hi; m0 += 4 * kSkRows) {
      float4 v[kSkRows][kSkMaxSplit];
#pragma unroll
      for (int j = 0; j < kSkRows; ++j) {
        const int m = m0 + 4 * j;
        const uint32_t pm = p_own + static_cast<uint32_t>(m) * kGmBM * 4u;
#pragma unroll
        for (int r = 0; r < kSkMaxSplit; ++r)
          v[j][r] = (m < m_hi && r < n_split) ? ld_cluster_f32x4(cluster_map(pm, r))
                                               : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int j = 0; j < kSkRows; ++j) {
        const int m = m0 + 4 * j;
        if (m >= m_hi || any_err) continue;
        float4 y = v[j][0];
#pragma unroll
        for (int r = 1; r < kSkMaxSplit; ++r)
          if (r < n_split) {
            y.x += v[j][r].x;
            y.y += v[j][r].y;
            y.z += v[j][r].z;
            y.w += v[j][r].w;
          }
        if (seg.bias) {
          y.x += b4.x;
          y.y += b4.y;
          y.z += b4.z;
          y.w += b4.w;
        }
        if (a.resid) {
          const float4 r4 =
              *reinterpret_cast<const float4*>(a.resid + static_cast<size_t>(m) * a.ld_res + col4);
          y = make_float4(r4.x + y.x, r4.y + y.y, r4.z + y.z, r4.w + y.w);
        }
        *reinterpret_cast<float4*>(seg.out + static_cast<size_t>(m) * seg.ld + col4) = y;
      }
    }
    // the others' reads of this CTA's partial are done (a release here would
    // also wait for this CTA's output stores to be acknowledged)
    cluster_sync_relaxed();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, 128);
  }
}

// ---- operand preparation ------------------------------------------------
// FP16 high part of v and the FP16 rounding of the residual scaled by 2^11.
__device__ __forceinline__ void split_hi_lo_scaled(float v, __half& hi, __half& lo) {
  hi = __float2half_rn(v);
  lo = __float2half_rn((v - __half2float(hi)) * kGmLoScale);
}

// One row of x per block (K a multiple of 8): optional RMSNorm with weights
// norm_w (1/sqrtf(sum(x^2)/K + eps), then (x * r) * w, as the CPU-path
// kernels), then x_hi, x_lo rows.  block = 256 threads.
__global__ void __launch_bounds__(256)
    act_split_kernel(const float* __restrict__ x, int ldx, int K,
                     const float* __restrict__ norm_w, float eps, __half* __restrict__ xh,
                     __half* __restrict__ xl) {
  __shared__ float s_red[8];
  // a skinny GEMM queued behind this grid (programmatic dependent launch)
  // may start its set-up and weight loads now
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int m = blockIdx.x, t = threadIdx.x;
  const float* row = x + static_cast<size_t>(m) * ldx;
  float r = 1.0f;
  if (norm_w) {
    float ss = 0.f;
    for (int i = 4 * t; i < K; i += 4 * 256) {
      const float4 v = *reinterpret_cast<const float4*>(row + i);
      ss += (v.x * v.x + v.y * v.y) + (v.z * v.z + v.w * v.w);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((t & 31) == 0) s_red[t >> 5] = ss;
    __syncthreads();
    if (t == 0) {
      float tot = 0.f;
      for (int w = 0; w < 8; ++w) tot += s_red[w];
      s_red[0] = 1.0f / sqrtf(tot / static_cast<float>(K) + eps);
    }
    __syncthreads();
    r = s_red[0];
  }
  __half* oh = xh + static_cast<size_t>(m) * K;
  __half* ol = xl + static_cast<size_t>(m) * K;
  for (int i = 4 * t; i < K; i += 4 * 256) {
    float4 v = *reinterpret_cast<const float4*>(row + i);
    if (norm_w) {
      const float4 w = __ldg(reinterpret_cast<const float4*>(norm_w + i));
      v.x = (v.x * r) * w.x;
      v.y = (v.y * r) * w.y;
      v.z = (v.z * r) * w.z;
      v.w = (v.w * r) * w.w;
    }
    __half h[4], l[4];
    split_hi_lo_scaled(v.x, h[0], l[0]);
    split_hi_lo_scaled(v.y, h[1], l[1]);
    split_hi_lo_scaled(v.z, h[2], l[2]);
    split_hi_lo_scaled(v.w, h[3], l[3]);
    *reinterpret_cast<uint2*>(oh + i) = *reinterpret_cast<const uint2*>(h);
    *reinterpret_cast<uint2*>(ol + i) = *reinterpret_cast<const uint2*>(l);
  }
}

// Weight i of a row in the module's device layout (kern_proj.cuh), as
// picolm's dequantize_row_* computes it (quant.c:96-222; F16 and F32 as
// stored): Q4_K d*sc*q - dmin*m per 32-weight sub-block, Q6_K d*sc*(q-32)
// per 16, Q8_0 d*q.
__device__ __forceinline__ float dequant_one(const uint8_t* row, int type, int n, int i) {
  if (type == kGgufF32) return reinterpret_cast<const float*>(row)[i];
  if (type == kGgufF16) return __half2float(reinterpret_cast<const __half*>(row)[i]);
  if (type == kGgufQ8_0) {
    const int8_t q = reinterpret_cast<const int8_t*>(row)[i];
    const float d = __half2float(reinterpret_cast<const __half*>(row + n)[i / 32]);
    return d * static_cast<float>(q);
  }
  if (type == kGgufQ4K) {
    const uint8_t* blk = row + static_cast<size_t>(i / 256) * kQ4KBytes;
    const int e = i % 256, j = e / 64, hi = (e / 32) & 1, l = e % 32;
    const float d = __half2float(*reinterpret_cast<const __half*>(blk));
    const float dmin = __half2float(*reinterpret_cast<const __half*>(blk + 2));
    const uint32_t* sw = reinterpret_cast<const uint32_t*>(blk + 4);
    float sc, mn;
    scale_min_k4(2 * j + hi, sw[0], sw[1], sw[2], sc, mn);
    const uint8_t qb = blk[16 + 32 * j + l];
    const float q = static_cast<float>(hi ? (qb >> 4) : (qb & 0xF));
    return (d * sc) * q - dmin * mn;
  }
  // Q6_K (224-byte blocks {ql[128], qh[64], scales[16], d})
  const uint8_t* blk = row + static_cast<size_t>(i / 256) * kQ6KBytes;
  const int e = i % 256, half = e / 128, r = e % 128, quarter = r / 32, l = r % 32;
  const uint8_t* ql = blk + 64 * half;
  const uint8_t* qh = blk + 128 + 32 * half;
  const int8_t* sc = reinterpret_cast<const int8_t*>(blk + 192) + 8 * half;
  const float d = __half2float(*reinterpret_cast<const __half*>(blk + 208));
  const int lo4 = quarter == 0 ? (ql[l] & 0xF) : quarter == 1 ? (ql[l + 32] & 0xF)
                                : quarter == 2 ? (ql[l] >> 4) : (ql[l + 32] >> 4);
  const int hi2 = (qh[l] >> (2 * quarter)) & 3;
  const int q = (lo4 | (hi2 << 4)) - 32;
  return (d * static_cast<float>(sc[l / 16 + 2 * quarter])) * static_cast<float>(q);
}

// rows x n weights of one matrix (device layout, row stride rb) -> w_hi,
// w_lo rows [rows][n] FP16 at row offset row0 of the destination.  Sets
// *overflow if a weight does not fit FP16.
__global__ void dequant_split_kernel(const uint8_t* __restrict__ w, size_t rb, int type, int rows,
                                     int n, __half* __restrict__ wh, __half* __restrict__ wl,
                                     int row0, int* overflow) {
  const long total = static_cast<long>(rows) * n;
  for (long e = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<long>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(e / n), i = static_cast<int>(e % n);
    const float v = dequant_one(w + static_cast<size_t>(r) * rb, type, n, i);
    if (!(fabsf(v) < 65504.f)) atomicOr(overflow, 1);
    __half h, l;
    split_hi_lo_scaled(v, h, l);
    // tiled layout (wtile_row): n and the row count are multiples of 64 and 128
    const int R = row0 + r;
    const size_t o = (static_cast<size_t>(wtile_row(R, i / kGmBK, n / kGmBK)) + R % kGmBN) * kGmBK +
                     i % kGmBK;
    wh[o] = h;
    wl[o] = l;
  }
}

}  // namespace pl
