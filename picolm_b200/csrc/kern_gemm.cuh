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
// Kernel: gemm_hilo_kernel below (a persistent grid, the work split evenly
// over the SMs in 128 x 128 x 64 units), operand tiles of 16 KB (x_hi, x_lo,
// w_hi, w_lo; 128-byte swizzle) loaded by TMA, tcgen05.mma kind::f16
// M128 N128 into two double-buffered TMEM accumulator pairs.  Every mbarrier
// wait is bounded; a wait that gives up sets an error bit and the CTA winds
// down (it still waits for its own copies and MMAs, then frees its tensor
// memory).
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
constexpr int kGmMinRows = 128;             // the GEMM path from this many input rows

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

// ---- persistent, evenly split GEMM ---------------------------------------
// The work of one GEMM is n_tiles x kb_n units (a 128 x 128 tile times one
// 64-wide k-step), tiles ordered row-tile major (consecutive tiles share
// their x rows).  CTA c of the G = min(SMs, n_tiles) persistent CTAs takes
// units [c*U/G, (c+1)*U/G), so every SM does the same MMA work whatever the
// tile count (a fixed tiling of 320 tiles on 148 SMs leaves a third, mostly
// idle round).  With more tiles than SMs, G is the SM count; with fewer, G
// is a multiple of the tile count (each tile's k-steps split evenly over
// G / n_tiles CTAs), so a few input rows still stream the weights with
// every SM.  A tile whose units fall to more than one CTA is a split tile:
// each part (a CTA's first or last segment) stores its partial sum to a
// workspace, and gemm_fixup_kernel adds the parts in CTA order (earlier
// k-steps first), then bias and residual -- the split points depend only on
// the shape, so results repeat exactly, and no CTA waits on another.  Inside a CTA the two accumulators of a tile are double
// buffered in tensor memory (2 x 256 of the 512 columns): the epilogue
// warps drain one tile's while the MMA issuer fills the next one's.
//   warp 0    one lane: TMA loads of the four operand tiles of each unit,
//             a kGmStages-deep ring running on across tile boundaries;
//   warp 1    one lane: the three MMAs per 16-wide k-slice, tcgen05.commit
//             to free each stage and, at a segment's end, to hand the
//             accumulator buffer to the epilogue;
//   warps 2-5 epilogue (warp w reads TMEM lanes 32*(w%4)..), then release
//             the buffer; warp 2 also allocates and frees the tensor memory.
constexpr int kGmPThreads = 192;

struct GmSmem {
  uint8_t xh[kGmStages][kGmTile];
  uint8_t xl[kGmStages][kGmTile];
  uint8_t wh[kGmStages][kGmTile];
  uint8_t wl[kGmStages][kGmTile];
  uint64_t full[kGmStages], empty[kGmStages];
  uint64_t acc_full[2], acc_empty[2];
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

struct GemmSplit {
  int n_ntiles;        // column tiles (N / 128)
  int kb_n;            // k-steps per tile (K / 64)
  long long units;     // n_tiles * kb_n
  float* ws;           // partial tiles: [G CTAs][2: first, last segment][128][128] FP32
};

// CTA of G owning unit u (the largest c with floor(units * c / G) <= u)
__device__ __forceinline__ int gm_cta_of(const GemmSplit& sp, long long u, int G) {
  return static_cast<int>(((u + 1) * G - 1) / sp.units);
}

// units of CTA c
__device__ __forceinline__ long long gm_unit_begin(const GemmSplit& sp, int c) {
  return sp.units * c / gridDim.x;
}

__global__ void __launch_bounds__(kGmPThreads, 1)
    gemm_hilo_kernel(const GemmArgs a, const GemmSplit sp,
                     const __grid_constant__ CUtensorMap tm_xh,
                     const __grid_constant__ CUtensorMap tm_xl,
                     const __grid_constant__ CUtensorMap tm_wh,
                     const __grid_constant__ CUtensorMap tm_wl) {
  extern __shared__ uint8_t smem_raw[];
  GmSmem& sm = *reinterpret_cast<GmSmem*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x;
  const long long u0 = gm_unit_begin(sp, c), u1 = gm_unit_begin(sp, c + 1);
  const int kb_n = sp.kb_n;

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tm_xh);
    tma_prefetch_desc(&tm_xl);
    tma_prefetch_desc(&tm_wh);
    tma_prefetch_desc(&tm_wl);
    for (int s = 0; s < kGmStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.acc_full[b], 1);
      mbar_init(&sm.acc_empty[b], 4);  // one arrival per epilogue warp
    }
    fence_mbar_init();
  }
  if (warp == 2) {
    tmem_alloc(&sm.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      long long issued = 0;
      for (long long u = u0; u < u1; ++u) {
        const int it = static_cast<int>(u - u0), s = it % kGmStages;
        if (it >= kGmStages && !mbar_wait_bounded(&sm.empty[s], ((it / kGmStages) - 1) & 1)) {
          atomicOr(a.err, ERR_TIMEOUT_EMPTY);
          break;
        }
        const long long t = u / kb_n;
        const int kb = static_cast<int>(u - t * kb_n);
        const int m0 = static_cast<int>(t / sp.n_ntiles) * kGmBM;
        const int n0 = static_cast<int>(t % sp.n_ntiles) * kGmBN;
        mbar_arrive_expect_tx(&sm.full[s], 4u * kGmTile);
        const int k0 = kb * kGmBK;
        tma_load_2d(sm.xh[s], &tm_xh, &sm.full[s], k0, m0);
        tma_load_2d(sm.xl[s], &tm_xl, &sm.full[s], k0, m0);
        tma_load_2d(sm.wh[s], &tm_wh, &sm.full[s], k0, a.w_row0 + n0);
        tma_load_2d(sm.wl[s], &tm_wl, &sm.full[s], k0, a.w_row0 + n0);
        ++issued;
      }
      // never leave with copies in flight: the last use of each stage must land
      for (long long j = issued - kGmStages; j < issued; ++j)
        if (j >= 0) mbar_wait_bounded(&sm.full[j % kGmStages], static_cast<uint32_t>((j / kGmStages) & 1));
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_f16_f32(kGmBM, kGmBN, 0);
      bool ok = true;
      int seg = 0;
      for (long long u = u0; u < u1 && ok; ++seg) {
        const long long t = u / kb_n;
        const long long ue = (t + 1) * kb_n < u1 ? (t + 1) * kb_n : u1;  // this tile's units here
        const int b = seg & 1;
        // the epilogue has drained this buffer's previous tile
        if (seg >= 2 && !mbar_wait_bounded(&sm.acc_empty[b], ((seg >> 1) - 1) & 1)) {
          atomicOr(a.err, ERR_TIMEOUT_MMA);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t acc0 = tmem + b * 2 * kGmBN, acc1 = acc0 + kGmBN;
        for (long long v = u; v < ue; ++v) {
          const int it = static_cast<int>(v - u0), s = it % kGmStages;
          if (!mbar_wait_bounded(&sm.full[s], (it / kGmStages) & 1)) {
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
            const uint32_t accum = (v > u || kk > 0) ? 1u : 0u;
            tc_mma_ss(acc0, dxh, dwh, idesc, accum);
            tc_mma_ss(acc1, dxl, dwh, idesc, accum);
            tc_mma_ss(acc1, dxh, dwl, idesc, 1u);
          }
          tc_commit(&sm.empty[s]);  // the stage is free once these MMAs have read it
        }
        tc_commit(&sm.acc_full[b]);  // the tile's sums (or partial sums) are ready
        u = ue;
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int lg = warp & 3;  // TMEM lane group of this warp
    bool ok = true;
    int seg = 0;
    for (long long u = u0; u < u1; ++seg) {
      const long long t = u / kb_n;
      const long long tb = t * kb_n, te = tb + kb_n;
      const long long ue = te < u1 ? te : u1;
      const int b = seg & 1;
      if (ok && !mbar_wait_bounded(&sm.acc_full[b], (seg >> 1) & 1)) {
        if (lane == 0) atomicOr(a.err, ERR_TIMEOUT_MMA);
        ok = false;
      }
      const bool any_err = __any_sync(0xffffffffu, !ok);
      if (any_err) break;
      tc_fence_after();
      const int m0 = static_cast<int>(t / sp.n_ntiles) * kGmBM;
      const int n0 = static_cast<int>(t % sp.n_ntiles) * kGmBN;
      const int r = 32 * lg + lane;  // row of the tile
      const int m = m0 + r;
      // whole tile here: the outputs; else this CTA's part of a split tile,
      // which can only be its first or its last segment
      const bool whole = u == tb && ue == te;
      float* part = nullptr;
      if (!whole)
        part = sp.ws + (static_cast<size_t>(c) * 2 + (seg == 0 ? 0 : 1)) * kGmBM * kGmBN;
      int si = 0;
      for (int i = 1; i < a.n_seg; ++i)
        if (n0 >= a.seg[i].col0) si = i;
      const GemmSeg sg = a.seg[si];
      const int c0 = n0 - sg.col0;
      const uint32_t lane_base = tmem + (static_cast<uint32_t>(32 * lg) << 16) + b * 2 * kGmBN;
#pragma unroll 1
      for (int cc = 0; cc < kGmBN; cc += 32) {
        uint32_t r0[32], r1[32];
        tc_ld_32x32b_x32(lane_base + cc, r0);
        tc_ld_32x32b_x32(lane_base + kGmBN + cc, r1);
        tc_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          asm volatile("" : "+r"(r0[i]));
          asm volatile("" : "+r"(r1[i]));
        }
        if (!whole) {
          float* dst = part + static_cast<size_t>(r) * kGmBN + cc;
#pragma unroll
          for (int i = 0; i < 32; i += 4)
            *reinterpret_cast<float4*>(dst + i) = make_float4(
                __uint_as_float(r0[i]) + __uint_as_float(r1[i]) * kGmLoInv,
                __uint_as_float(r0[i + 1]) + __uint_as_float(r1[i + 1]) * kGmLoInv,
                __uint_as_float(r0[i + 2]) + __uint_as_float(r1[i + 2]) * kGmLoInv,
                __uint_as_float(r0[i + 3]) + __uint_as_float(r1[i + 3]) * kGmLoInv);
          continue;
        }
        if (m >= a.M) continue;
        float* dst = sg.out + static_cast<size_t>(m) * sg.ld + c0 + cc;
        const float* res = a.resid ? a.resid + static_cast<size_t>(m) * a.ld_res + c0 + cc : nullptr;
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
          float4 y;
          y.x = __uint_as_float(r0[i]) + __uint_as_float(r1[i]) * kGmLoInv;
          y.y = __uint_as_float(r0[i + 1]) + __uint_as_float(r1[i + 1]) * kGmLoInv;
          y.z = __uint_as_float(r0[i + 2]) + __uint_as_float(r1[i + 2]) * kGmLoInv;
          y.w = __uint_as_float(r0[i + 3]) + __uint_as_float(r1[i + 3]) * kGmLoInv;
          if (sg.bias) {
            const float4 bb = __ldg(reinterpret_cast<const float4*>(sg.bias + c0 + cc + i));
            y.x += bb.x;
            y.y += bb.y;
            y.z += bb.z;
            y.w += bb.w;
          }
          if (res) {
            const float4 rr = *reinterpret_cast<const float4*>(res + i);
            y.x = rr.x + y.x;
            y.y = rr.y + y.y;
            y.z = rr.z + y.z;
            y.w = rr.w + y.w;
          }
          *reinterpret_cast<float4*>(dst + i) = y;
        }
      }
      // the buffer may take the next tile's sums
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.acc_empty[b]);
      u = ue;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Split tiles: outputs = the parts of every CTA that worked on the tile,
// added in CTA order (earlier k-steps first), + bias, + residual.
// grid = n_tiles blocks (a tile one CTA did whole returns at once), block =
// 256; G = the GEMM's CTA count.
__global__ void __launch_bounds__(256) gemm_fixup_kernel(const GemmArgs a, const GemmSplit sp,
                                                         int G) {
  const long long t = blockIdx.x;
  const long long tb = t * sp.kb_n, te = tb + sp.kb_n;
  const int c_lo = gm_cta_of(sp, tb, G), c_hi = gm_cta_of(sp, te - 1, G);
  if (c_lo == c_hi) return;  // done whole by one CTA
  const int m0 = static_cast<int>(t / sp.n_ntiles) * kGmBM;
  const int n0 = static_cast<int>(t % sp.n_ntiles) * kGmBN;
  int si = 0;
  for (int i = 1; i < a.n_seg; ++i)
    if (n0 >= a.seg[i].col0) si = i;
  const GemmSeg sg = a.seg[si];
  const int c0 = n0 - sg.col0;
  for (int idx = 4 * threadIdx.x; idx < kGmBM * kGmBN; idx += 4 * 256) {
    const int r = idx / kGmBN, col = idx % kGmBN, m = m0 + r;
    if (m >= a.M) continue;
    float4 y = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int cc = c_lo; cc <= c_hi; ++cc) {
      // the tile is CTA cc's first segment if its range starts inside it
      const long long u0 = sp.units * cc / G;
      const int which = u0 >= tb ? 0 : 1;
      const float4 x = *reinterpret_cast<const float4*>(
          sp.ws + (static_cast<size_t>(cc) * 2 + which) * kGmBM * kGmBN + idx);
      y.x += x.x;
      y.y += x.y;
      y.z += x.z;
      y.w += x.w;
    }
    if (sg.bias) {
      const float4 bb = __ldg(reinterpret_cast<const float4*>(sg.bias + c0 + col));
      y.x += bb.x;
      y.y += bb.y;
      y.z += bb.z;
      y.w += bb.w;
    }
    if (a.resid) {
      const float4 rr =
          *reinterpret_cast<const float4*>(a.resid + static_cast<size_t>(m) * a.ld_res + c0 + col);
      y.x = rr.x + y.x;
      y.y = rr.y + y.y;
      y.z = rr.z + y.z;
      y.w = rr.w + y.w;
    }
    *reinterpret_cast<float4*>(sg.out + static_cast<size_t>(m) * sg.ld + c0 + col) = y;
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
    const size_t o = static_cast<size_t>(row0 + r) * n + i;
    wh[o] = h;
    wl[o] = l;
  }
}

}  // namespace pl
