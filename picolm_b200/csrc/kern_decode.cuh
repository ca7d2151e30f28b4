// kern_decode.cuh -- fused decode step: RoPE(q, k) -> FP16 KV append ->
// split-KV GQA attention (flash-decoding) -> split merge, for one or many
// sequences in one launch.
//
// Replaces picolm/model.c:820-892 (and its batched use).  One CTA handles
// one sequence and one contiguous chunk of cache rows (a "split"):
//
//   warp Hk      (producer)  one lane streams K and V tiles of TP rows x all
//                            KV heads into an NSTAGE-deep shared-memory ring
//                            with 4-D TMA loads (128-byte swizzle), one
//                            mbarrier pair per stage;
//   warps 0..Hk-1 (consumers) warp w owns KV head w and its kv_mul query
//                            heads.  Scores and P.V run on the tensor cores
//                            (mma.sync m16n8k16, FP16 in / FP32 accumulate):
//                            rows 0..7 of the A operand hold the high FP16
//                            half of q (resp. p), rows 8..15 the residual
//                            low half, so the FP16 operand costs no
//                            precision (q ~ hi + lo to 2^-22).  Online
//                            softmax in the log2 domain with quad shuffles.
//
// Why tensor cores in a memory-bound kernel: with 8 query heads per KV head
// each 256-byte K+V row feeds 2 x 8 x 64 multiply-adds, ~4.7 FP32-pipe
// instructions per byte -- at 6.5 TB/s that is ~85 % of the B200's FP32
// issue rate, so a CUDA-core dot product would cap the kernel below the HBM
// roofline.  On the tensor pipe the same work costs a few percent.
//
// The row at `pos` is appended by the CTA whose chunk contains it: the warp
// of each KV head rotates k (bit-exact picolm RoPE), encodes k and v with
// picolm's FP16 rounding, stores them to HBM and patches them into the
// shared-memory tile it reads (TMA may have fetched the row before the
// store landed).
//
// Each split leaves a partial (m, l, o) in a scratch buffer.  With few
// splits the last CTA of a sequence to finish merges them in the same
// launch (a counter per sequence); with many splits (long single-sequence
// contexts) a separate combine kernel with one CTA per head does it.
#pragma once
#include <cstdint>
#include <cuda.h>

#include "pl_fp16.cuh"
#include "sm100.cuh"

namespace pl {

constexpr int kHD = 64;               // head_dim supported by the kernels
constexpr int kPartStride = kHD + 2;  // floats per (m, l, o[64]) partial
constexpr float kLog2e = 1.4426950408889634f;
constexpr int kMaxInKernelMerge = 32; // splits merged by the last CTA

struct DecodeArgs {
  // cache geometry
  int n_layers, max_seq, n_heads, n_kv_heads, kv_mul, layer, rope_type, n_slots;
  const float* cos_tab;  // [rope_rows][32]
  const float* sin_tab;
  uint16_t* kc;          // [slots][n_layers][max_seq][kv_dim]
  uint16_t* vc;
  // per-launch inputs, gridDim.y = number of sequences
  const int* seqs;       // cache slot per sequence
  const int* pos;        // global position of the new token
  const float* q;        // [n][n_heads*64]   before RoPE
  const float* k;        // [n][kv_dim]       before RoPE
  const float* v;        // [n][kv_dim]
  float* out;            // [n][n_heads*64]   normalised output (mode 0)
  float* part;           // [n][n_split][n_heads][66] per-split partials
  float* part_out;       // mode 1: merged partial per sequence [n][n_heads][66]
  int* counters;         // [n] finished-CTA counters, self-resetting
  int n_split;
  int merge_in_kernel;   // 1: last CTA per sequence merges; 0: combine kernel
  // mode 0: attend rows [0, pos], append at row pos.
  // mode 1: shard of a KV-split sequence: attend local rows [0, n_rows),
  //         append (if append) at local row pos - row0.
  int mode, row0, n_rows, append;
  float score_scale;     // log2(e) / sqrt(head_dim)
  uint32_t* err;
};

// RoPE of the element pair (d, d+1) of one head (d even), as picolm's
// rope() computes it (tensor.c:537-601).  LLaMA rotates (d, d+1) together;
// Qwen pairs element e with e +/- 32.
__device__ __forceinline__ float2 rope_two(const float* x, int d, const float* cs,
                                           const float* sn, int rope_type) {
  float2 y;
  if (rope_type == 0) {
    const float2 xv = *reinterpret_cast<const float2*>(x + d);
    rope_pair(xv.x, xv.y, cs[d >> 1], sn[d >> 1], y.x, y.y);
  } else {
    float r[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int j = d + e;
      if (j < kHD / 2)
        r[e] = __fsub_rn(__fmul_rn(x[j], cs[j]), __fmul_rn(x[j + kHD / 2], sn[j]));
      else
        r[e] = __fadd_rn(__fmul_rn(x[j - kHD / 2], sn[j - kHD / 2]),
                         __fmul_rn(x[j], cs[j - kHD / 2]));
    }
    y.x = r[0];
    y.y = r[1];
  }
  return y;
}

// Split an FP32 pair into FP16 high parts and FP16 residuals.
__device__ __forceinline__ void split_hi_lo(float a, float b, uint32_t& hi, uint32_t& lo) {
  hi = pack_half2(a, b);
  const float2 h = unpack_half2(hi);
  lo = pack_half2(a - h.x, b - h.y);
}

// Byte offset of 16-byte chunk `chunk` of row `r` in a 128-byte-swizzled
// tile (rows of 128 bytes, 1024-byte aligned base): TMA's SWIZZLE_128B.
__device__ __forceinline__ uint32_t sw128(int r, int chunk) {
  return static_cast<uint32_t>(r * 128 + ((chunk ^ (r & 7)) << 4));
}

// Merge n_split partials of one sequence (part: [n_split][n_heads][66]).
// Writes O/L to out, or the merged (M, L, O) to part_out.
__device__ __forceinline__ void merge_partials(int n_split, int n_heads, const float* part,
                                               float* out, float* part_out, int tid,
                                               int nthreads) {
  const size_t step = static_cast<size_t>(n_heads) * kPartStride;
  for (int idx = tid; idx < n_heads * kHD; idx += nthreads) {
    const int h = idx / kHD, d = idx % kHD;
    const float* base = part + static_cast<size_t>(h) * kPartStride;
    float M = -INFINITY;
    for (int j = 0; j < n_split; ++j) M = fmaxf(M, __ldcg(base + j * step));
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
      for (int j = 0; j < n_split; ++j) {
        const float* pj = base + j * step;
        const float w = ex2(__ldcg(pj) - M);
        L += w * __ldcg(pj + 1);
        O += w * __ldcg(pj + 2 + d);
      }
    }
    if (out) {
      out[idx] = O / L;
    } else {
      float* dst = part_out + static_cast<size_t>(h) * kPartStride;
      if (d == 0) {
        dst[0] = M;
        dst[1] = L;
      }
      dst[2 + d] = O;
    }
  }
}

// One consumer warp: KV head w of sequence i over tiles [t_begin, t_begin+ntiles).
template <int TP, int NSTAGE>
__device__ __forceinline__ void decode_consumer(const DecodeArgs& a, int w, int lane, int i,
                                                int split, int pos, int att_rows, int app_row,
                                                int t_begin, int ntiles, int slab, bool appends,
                                                const uint8_t* sK, const uint8_t* sV,
                                                int tile_bytes, uint64_t* full, uint64_t* empty) {
  const int kv_dim = a.n_kv_heads * kHD;
  const int g = lane >> 2, c = lane & 3;
  const int kv_mul = a.kv_mul;
  const bool row_valid = g < kv_mul;
  const int qh = w * kv_mul + (row_valid ? g : 0);
  const float* cs = a.cos_tab + static_cast<size_t>(pos) * (kHD / 2);
  const float* sn = a.sin_tab + static_cast<size_t>(pos) * (kHD / 2);

  // q fragments: this thread needs dims 16kk+2c, +1 and 16kk+8+2c, +1
  uint32_t qa[4][4];
  {
    const float* qrow = a.q + (static_cast<size_t>(i) * a.n_heads + qh) * kHD;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int d = 16 * kk + 8 * hf + 2 * c;
        float2 y = rope_two(qrow, d, cs, sn, a.rope_type);
        if (!row_valid) y = make_float2(0.f, 0.f);
        uint32_t hi, lo;
        split_hi_lo(y.x, y.y, hi, lo);
        qa[kk][2 * hf + 0] = hi;  // rows 0..7: high halves
        qa[kk][2 * hf + 1] = lo;  // rows 8..15: residuals
      }
    }
  }

  // the appended row: rotate k, encode k and v with picolm's FP16 rounding
  uint32_t kword = 0, vword = 0;
  if (appends) {
    const float* krow = a.k + static_cast<size_t>(i) * kv_dim + w * kHD;
    const float* vrow = a.v + static_cast<size_t>(i) * kv_dim + w * kHD;
    const float2 kr = rope_two(krow, 2 * lane, cs, sn, a.rope_type);
    const float2 vv = *reinterpret_cast<const float2*>(vrow + 2 * lane);
    kword = static_cast<uint32_t>(picolm_f32_to_f16(kr.x)) |
            (static_cast<uint32_t>(picolm_f32_to_f16(kr.y)) << 16);
    vword = static_cast<uint32_t>(picolm_f32_to_f16(vv.x)) |
            (static_cast<uint32_t>(picolm_f32_to_f16(vv.y)) << 16);
    const size_t off = (static_cast<size_t>(slab) * a.max_seq + app_row) * kv_dim + w * kHD;
    reinterpret_cast<uint32_t*>(a.kc + off)[lane] = kword;
    reinterpret_cast<uint32_t*>(a.vc + off)[lane] = vword;
  }

  float m_run = -INFINITY;  // running max of row g (log2 domain)
  float l_run = 0.f;        // this thread's share of the row sum
  float o[8][4];
#pragma unroll
  for (int j = 0; j < 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;

  for (int it = 0; it < ntiles; ++it) {
    const int s = it % NSTAGE;
    if (!mbar_wait_bounded(&full[s], (it / NSTAGE) & 1)) {
      atomicOr(a.err, ERR_TIMEOUT_FULL);
      break;
    }
    const uint32_t kbase = smem_u32(sK + s * tile_bytes + w * TP * 128);
    const uint32_t vbase = smem_u32(sV + s * tile_bytes + w * TP * 128);
    const int row0 = (t_begin + it) * TP;
    const bool patch = appends && app_row >= row0 && app_row < row0 + TP;
    if (patch) {
      const int r = app_row - row0;
      const uint32_t off = sw128(r, lane >> 2) + (lane & 3) * 4;
      asm volatile("st.shared.u32 [%0], %1;" ::"r"(kbase + off), "r"(kword) : "memory");
      asm volatile("st.shared.u32 [%0], %1;" ::"r"(vbase + off), "r"(vword) : "memory");
      __syncwarp();
    }

    // S = Q K^T over TP rows
    float sacc[TP / 8][4];
#pragma unroll
    for (int nt = 0; nt < TP / 8; ++nt) {
      sacc[nt][0] = sacc[nt][1] = sacc[nt][2] = sacc[nt][3] = 0.f;
#pragma unroll
      for (int kp = 0; kp < 2; ++kp) {
        const int r = nt * 8 + (lane & 7);
        const int ch = 4 * kp + (lane >> 3);
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4(kbase + sw128(r, ch), b0, b1, b2, b3);
        mma_16816(sacc[nt], qa[2 * kp], b0, b1);
        mma_16816(sacc[nt], qa[2 * kp + 1], b2, b3);
      }
    }
    // scores of row g: column 2c+e of n-tile nt is hi-row + lo-row
    float mt = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < TP / 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int t = row0 + nt * 8 + 2 * c + e;
        float sc = (sacc[nt][e] + sacc[nt][2 + e]) * a.score_scale;
        sc = t < att_rows ? sc : -INFINITY;
        sacc[nt][e] = sc;
        mt = fmaxf(mt, sc);
      }
    }
    mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 1));
    mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 2));
    const float m_new = fmaxf(m_run, mt);
    const float alpha = ex2(m_run - m_new);
    l_run *= alpha;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      o[j][0] *= alpha;
      o[j][1] *= alpha;
      o[j][2] *= alpha;
      o[j][3] *= alpha;
    }
    // P (hi/lo) and O += P V, 16 rows per k-step
#pragma unroll
    for (int kk = 0; kk < TP / 16; ++kk) {
      const float p00 = ex2(sacc[2 * kk][0] - m_new), p01 = ex2(sacc[2 * kk][1] - m_new);
      const float p10 = ex2(sacc[2 * kk + 1][0] - m_new), p11 = ex2(sacc[2 * kk + 1][1] - m_new);
      l_run += (p00 + p01) + (p10 + p11);
      uint32_t pa[4];
      split_hi_lo(p00, p01, pa[0], pa[1]);
      split_hi_lo(p10, p11, pa[2], pa[3]);
#pragma unroll
      for (int j2 = 0; j2 < 4; ++j2) {
        const int r = 16 * kk + ((lane >> 3) & 1) * 8 + (lane & 7);
        const int ch = 2 * j2 + (lane >> 4);
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4_trans(vbase + sw128(r, ch), b0, b1, b2, b3);
        mma_16816(o[2 * j2], pa, b0, b1);
        mma_16816(o[2 * j2 + 1], pa, b2, b3);
      }
    }
    m_run = m_new;
    __syncwarp();
    if (patch) fence_proxy_async_smem();  // generic writes before the next TMA refill
    if (lane == 0) mbar_arrive(&empty[s]);
  }

  // ---------------------------------------------------------------- epilogue
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
  if (!row_valid) return;
  if (a.n_split == 1 && a.mode == 0) {
    const float inv = 1.0f / l_run;
    float* dst = a.out + (static_cast<size_t>(i) * a.n_heads + qh) * kHD;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      *reinterpret_cast<float2*>(dst + 8 * j + 2 * c) =
          make_float2((o[j][0] + o[j][2]) * inv, (o[j][1] + o[j][3]) * inv);
  } else {
    float* dst = a.part +
                 ((static_cast<size_t>(i) * a.n_split + split) * a.n_heads + qh) * kPartStride;
    if (c == 0) {
      dst[0] = m_run;
      dst[1] = l_run;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      dst[2 + 8 * j + 2 * c] = o[j][0] + o[j][2];
      dst[3 + 8 * j + 2 * c] = o[j][1] + o[j][3];
    }
  }
}

template <int TP, int NSTAGE>
__global__ void __launch_bounds__(288) decode_kernel(const DecodeArgs a,
                                                     const __grid_constant__ CUtensorMap tmk,
                                                     const __grid_constant__ CUtensorMap tmv) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ int s_last;
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int Hk = a.n_kv_heads;
  const int tile_bytes = TP * Hk * 128;  // one K (or V) tile: TP rows x all KV heads
  uint8_t* sK = smem;
  uint8_t* sV = smem + NSTAGE * tile_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + 2 * NSTAGE * tile_bytes);
  uint64_t* empty = full + NSTAGE;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int i = blockIdx.y;
  const int split = blockIdx.x;
  const int seq = a.seqs[i];
  const int pos = a.pos[i];
  const int att_rows = a.mode == 0 ? pos + 1 : a.n_rows;
  const int app_row = a.mode == 0 ? pos : (a.append ? pos - a.row0 : -1);
  const int ntiles_all = (att_rows + TP - 1) / TP;
  const int chunk = (ntiles_all + a.n_split - 1) / a.n_split;
  const int t_begin = split * chunk;
  const int t_end = min(t_begin + chunk, ntiles_all);
  const int ntiles = max(0, t_end - t_begin);
  const int slab = seq * a.n_layers + a.layer;
  const bool appends = app_row >= 0 && app_row >= t_begin * TP && app_row < t_end * TP;
  // device-side argument check (device-pointer callers): the whole sequence
  // is skipped -- every CTA of it returns here, so its merge counter stays 0
  if (seq < 0 || seq >= a.n_slots || pos < 0 || pos >= a.max_seq || att_rows > a.max_seq ||
      app_row >= a.max_seq) {
    if (threadIdx.x == 0) atomicOr(a.err, ERR_BAD_ARG);
    return;
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < NSTAGE; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], Hk);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == Hk) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && ntiles > 0) {
      tma_prefetch_desc(&tmk);
      tma_prefetch_desc(&tmv);
      int issued = 0;
      for (int it = 0; it < ntiles; ++it) {
        const int s = it % NSTAGE;
        if (it >= NSTAGE && !mbar_wait_bounded(&empty[s], ((it / NSTAGE) - 1) & 1)) {
          atomicOr(a.err, ERR_TIMEOUT_EMPTY);
          break;
        }
        mbar_arrive_expect_tx(&full[s], 2u * tile_bytes);
        const int row = (t_begin + it) * TP;
        tma_load_4d(sK + s * tile_bytes, &tmk, &full[s], 0, row, 0, slab);
        tma_load_4d(sV + s * tile_bytes, &tmv, &full[s], 0, row, 0, slab);
        ++issued;
      }
      // never leave with copies in flight: the last use of each stage must land
      for (int j = issued - NSTAGE; j < issued; ++j)
        if (j >= 0) mbar_wait_bounded(&full[j % NSTAGE], (j / NSTAGE) & 1);
    }
  } else {
    decode_consumer<TP, NSTAGE>(a, warp, lane, i, split, pos, att_rows, app_row, t_begin,
                                ntiles, slab, appends, sK, sV, tile_bytes, full, empty);
  }
  if ((a.n_split == 1 && a.mode == 0) || !a.merge_in_kernel) return;

  // -------------------------------------------------- in-kernel split merge
  __threadfence();  // this thread's partial writes, device-wide
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(&a.counters[i], 1) == a.n_split - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const size_t per_seq = static_cast<size_t>(a.n_heads) * kPartStride;
  merge_partials(a.n_split, a.n_heads, a.part + static_cast<size_t>(i) * a.n_split * per_seq,
                 a.mode == 0 ? a.out + static_cast<size_t>(i) * a.n_heads * kHD : nullptr,
                 a.mode == 0 ? nullptr : a.part_out + static_cast<size_t>(i) * per_seq,
                 threadIdx.x, blockDim.x);
  if (threadIdx.x == 0) a.counters[i] = 0;
}

// Separate log-sum-exp merge for many splits (and for partials gathered
// from several devices): grid = (n_heads, n), block = 64 (one per dim).
// part [n][n_split][n_heads][66]; writes out [n][n_heads*64] or, if out is
// null, the merged partial to part_out [n][n_heads][66].
__global__ void __launch_bounds__(64) combine_kernel(int n_split, int n_heads,
                                                     const float* __restrict__ part,
                                                     float* __restrict__ out,
                                                     float* __restrict__ part_out) {
  const int h = blockIdx.x, i = blockIdx.y, d = threadIdx.x;
  const float* base = part + (static_cast<size_t>(i) * n_split * n_heads + h) * kPartStride;
  const size_t step = static_cast<size_t>(n_heads) * kPartStride;
  float M = -INFINITY;
  for (int j = 0; j < n_split; ++j) M = fmaxf(M, __ldcg(base + j * step));
  float L = 0.f, O = 0.f;
  if (M != -INFINITY) {
    for (int j = 0; j < n_split; ++j) {
      const float* pj = base + j * step;
      const float w = ex2(__ldcg(pj) - M);
      L += w * __ldcg(pj + 1);
      O += w * __ldcg(pj + 2 + d);
    }
  }
  if (out) {
    out[(static_cast<size_t>(i) * n_heads + h) * kHD + d] = O / L;
  } else {
    float* dst = part_out + (static_cast<size_t>(i) * n_heads + h) * kPartStride;
    if (d == 0) {
      dst[0] = M;
      dst[1] = L;
    }
    dst[2 + d] = O;
  }
}

}  // namespace pl
