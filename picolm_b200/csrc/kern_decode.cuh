// kern_decode.cuh -- fused decode step: RoPE(q, k) -> FP16 KV append ->
// split-KV GQA attention (flash-decoding) -> split merge, for one or many
// sequences in ONE launch.
//
// Replaces picolm/model.c:820-892 (and its batched use).
//
// Work partition.  The cache rows to read form a flattened list of tiles
// (TP rows x all KV heads each): sequence 0's tiles, then sequence 1's, ...
// Every CTA computes the tile counts' prefix sum in shared memory and takes
// an equal contiguous slice of that list, so all CTAs stream the same number
// of bytes whatever the sequence lengths are.  A slice covers one or more
// "segments" (the part of one sequence inside the slice); the TMA pipeline
// runs on across segment boundaries.
//
// The grid is launched with programmatic dependent launch: its CTAs take the
// SMs that the kernel before it on the stream frees and run that set-up
// (from the slots and positions read as a hint) and an L2 prefetch of their
// first tiles before griddepcontrol.wait; after the wait the counts are
// checked against fresh loads and the scan redone if one differs.
//
// Inside a CTA:
//   warp Hk      (producer)  one lane streams K and V tiles into an
//                            NSTAGE-deep ring with 4-D TMA loads (128-byte
//                            swizzle), one full/empty mbarrier pair a stage;
//   warps 0..Hk-1 (consumers) warp w owns KV head w and its kv_mul query
//                            heads.  Scores and P.V run on the tensor cores
//                            (mma.sync m16n8k16, FP16 in / FP32 accumulate):
//                            rows 0..7 of the A operand hold the high FP16
//                            half of q (resp. p), rows 8..15 the residual
//                            low half, so the FP16 operand costs no precision
//                            (q ~ hi + lo to 2^-22).  Online softmax in the
//                            log2 domain with quad shuffles.
//
// Why tensor cores in a memory-bound kernel: with 8 query heads per KV head
// each 256-byte K+V row feeds 2 x 8 x 64 multiply-adds, ~4.7 FP32-pipe
// instructions per byte -- at 6.5 TB/s that is ~85 % of the B200's FP32
// issue rate, so a CUDA-core dot product would cap the kernel below the HBM
// roofline.  On the tensor pipe the same work costs a few percent.
//
// head_dim is the template parameter HD (64 or 128).  A tile row of 128
// elements is staged as two 64-element halves, each its own region under
// the 128-byte swizzle and its own TMA box; tiles stay at 16 KB (TP rows x
// all KV heads), with a 3-deep ring where the 16-row minimum makes them
// larger (128 x 8 KV heads).
//
// The row at `pos` is appended by the segment that contains it: the warp of
// each KV head rotates k (bit-exact picolm RoPE), encodes k and v with
// picolm's FP16 rounding, stores them to HBM and patches them into the
// shared-memory tile it reads (TMA may have fetched the row before the
// store landed).
//
// Merge.  A sequence covered by one segment is finished by that segment.
// Otherwise each segment leaves a partial (m, l, o) in slot (cta + seq) of
// a scratch buffer and CTA 0 records each sequence's (first slot, segment
// count).  merge_kernel, launched right behind with programmatic dependent
// launch (it is resident and waiting on griddepcontrol.wait when the decode
// grid ends), merges them: 256 threads per group of 1 to 16 heads, sized so
// the merge grid has at most one block per SM.  Merging inside the decode grid
// instead, by the CTA (or, tried later, the warp) that finishes a sequence's
// last segment, puts atomics, fences and L2 round trips at the end of the
// slowest CTA: measured on B200 it was slower than this separate grid.
#pragma once
#include <cstdint>
#include <cuda.h>

#include "pl_fp16.cuh"
#include "sm100.cuh"

namespace pl {

// Head dims supported by the kernels: 64 and 128 (template parameter HD).
// The KV tiles are staged as 64-element (128-byte) halves under the 128-byte
// swizzle, one region per half.
constexpr int kHD = 64;                 // head_dim of the tensor-core prefill
constexpr int kPartO = 4;               // offset of o in a partial (16-byte aligned)
// floats per partial of one head: m, l, 2 pad, o[HD]
__host__ __device__ constexpr int part_stride(int hd) { return hd + kPartO; }
constexpr float kLog2e = 1.4426950408889634f;
constexpr int kMaxLaunchSeqs = 1024;    // sequences per launch (prefix scan in smem)
constexpr int kMaxCombineParts = 16;    // device partials merged by combine_kernel
// A launch of at most this many sequences may carry their (slot, position)
// pairs in its arguments instead of device arrays: a host-buffer call then
// needs no copy of them (each copy costs several microseconds of the GPU's
// timeline, however small).
constexpr int kInlineSeqs = 128;

struct DecodeArgs {
  // cache geometry
  int n_layers, max_seq, n_heads, n_kv_heads, kv_mul, layer, rope_type, n_slots;
  int pos_limit;         // positions are < pos_limit (RoPE table rows); max_seq is the
                         // cache rows per slab (fewer on a device holding a KV shard)
  const float* cos_tab;  // [rope_rows][32]
  const float* sin_tab;
  uint16_t* kc;          // [slots][n_layers][max_seq][kv_dim]
  uint16_t* vc;
  // per-launch inputs
  int n;                 // sequences in this launch (<= kMaxLaunchSeqs)
  const int* seqs;       // cache slot per sequence (nullptr: seq1 for all)
  const int* pos;        // global position of the new token (nullptr: pos1)
  int seq1, pos1;        // scalar slot / position when the arrays are null
  const float* q;        // [n][n_heads*HD]   before RoPE
  const float* k;        // [n][kv_dim]       before RoPE
  const float* v;        // [n][kv_dim]
  float* out;            // [n][out_stride]   normalised output (mode 0), head h at h*HD
  int out_stride;        // floats between the output rows of consecutive sequences
  float* part;           // [gridDim.x + n][n_heads][part_stride(HD)] segment partials
  float* part_out;       // mode 1: merged partial per sequence [n][n_heads][part_stride(HD)]
  int2* seg_info;        // [n] (first slot, segment count), written by CTA 0 for
                         // inspection; the merge derives the same from the positions
  // mode 0: attend rows [0, pos], append at row pos (if append; else the row
  //         is already in the cache).
  // mode 1: shard of a KV-split sequence: attend local rows [0, n_rows),
  //         append (if append) at local row pos - row0.
  int mode, row0, n_rows, append;
  float score_scale;     // log2(e) / sqrt(head_dim)
  uint32_t* err;
  // Host-buffer calls: the last kernel of the call stores the device error
  // word here (pinned host memory mapped into the device), so the host reads
  // it without a copy.  nullptr: not wanted.
  uint32_t* err_host;
  // n_inline > 0: (slot, position) of sequence i in sp[i], and seqs / pos
  // are not read.  The kernels take the arguments as __grid_constant__, so
  // sp is read in place from the parameter space.
  int n_inline;
  int2 sp[kInlineSeqs];
};

// RoPE of the element pair (d, d+1) of one head (d even), as picolm's
// rope() computes it (tensor.c:537-601).  LLaMA rotates (d, d+1) together;
// Qwen pairs element e with e +/- HD/2.
template <int HD>
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
      if (j < HD / 2)
        r[e] = __fsub_rn(__fmul_rn(x[j], cs[j]), __fmul_rn(x[j + HD / 2], sn[j]));
      else
        r[e] = __fadd_rn(__fmul_rn(x[j - HD / 2], sn[j - HD / 2]),
                         __fmul_rn(x[j], cs[j - HD / 2]));
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

// ------------------------------------------------------------ partition
struct Partition {
  const int* prefix;  // [n+1] exclusive prefix sum of tile counts (shared memory)
  long long T;        // total tiles
  int G;              // CTAs that hold work (<= gridDim.x)
  // CTA owning flattened tile x: the largest c with floor(c*T/G) <= x
  __device__ __forceinline__ int cta_of(long long x) const {
    return static_cast<int>(((x + 1) * G - 1) / T);
  }
  __device__ __forceinline__ long long begin(int c) const { return c * T / G; }
  __device__ __forceinline__ int n_seg(int i) const {
    return cta_of(prefix[i + 1] - 1) - cta_of(prefix[i]) + 1;
  }
  // slot of sequence i's j-th segment (segments of i are CTAs cta_of(prefix[i]) + j)
  __device__ __forceinline__ int slot(int i, int j) const { return cta_of(prefix[i]) + j + i; }
};

__device__ __forceinline__ int seq_of(const DecodeArgs& a, int i) {
  return a.n_inline ? a.sp[i].x : a.seqs ? a.seqs[i] : a.seq1;
}
__device__ __forceinline__ int pos_of(const DecodeArgs& a, int i) {
  return a.n_inline ? a.sp[i].y : a.pos ? a.pos[i] : a.pos1;
}

// Rows attended and the append row of sequence i.
__device__ __forceinline__ void seq_rows(const DecodeArgs& a, int i, int& att_rows,
                                         int& app_row) {
  const int pos = pos_of(a, i);
  att_rows = a.mode == 0 ? pos + 1 : a.n_rows;
  app_row = a.mode == 0 ? (a.append ? pos : -1) : (a.append ? pos - a.row0 : -1);
}

// Tile count of sequence i of a launch; 0, with `bad` set, for a sequence
// whose slot or rows are out of range.  With `hint` the slot and position
// are read through L2 only (ld.global.cg): before griddepcontrol.wait they
// may still be changing, and no L1 line of them may outlive the wait.
template <int TP>
__device__ __forceinline__ int seq_tiles(const DecodeArgs& a, int i, bool hint, bool& bad,
                                         int& seq) {
  seq = a.n_inline ? a.sp[i].x : a.seqs ? (hint ? __ldcg(a.seqs + i) : a.seqs[i]) : a.seq1;
  const int pos =
      a.n_inline ? a.sp[i].y : a.pos ? (hint ? __ldcg(a.pos + i) : a.pos[i]) : a.pos1;
  const int att_rows = a.mode == 0 ? pos + 1 : a.n_rows;
  const int app_row = a.mode == 0 ? (a.append ? pos : -1) : (a.append ? pos - a.row0 : -1);
  bad = seq < 0 || seq >= a.n_slots || pos < 0 || pos >= a.pos_limit || att_rows < 0 ||
        att_rows > a.max_seq || app_row >= a.max_seq;
  return bad ? 0 : (att_rows + TP - 1) / TP;
}

// Exclusive prefix sum of the launch's tile counts into s_prefix[0..n]
// (s_prefix[n] = total), the same in every CTA.  Each thread counts a
// contiguous run of sequences; returns whether one of them is out of range.
// With `hint`, s_seq[i] keeps the slot read for sequence i.
template <int TP>
__device__ bool scan_tiles(const DecodeArgs& a, int* s_prefix, int* s_warp_sum, int* s_seq,
                           bool hint) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nthr = blockDim.x, n = a.n;
  const int per = (n + nthr - 1) / nthr;
  const int i0 = tid * per;
  int local = 0;
  bool any_bad = false;
  for (int i = i0; i < min(n, i0 + per); ++i) {
    bool bad;
    int seq;
    const int tiles = seq_tiles<TP>(a, i, hint, bad, seq);
    any_bad |= bad;
    if (hint) s_seq[i] = seq;
    s_prefix[i] = tiles;  // counts first, scanned below
    local += tiles;
  }
  // inclusive scan of the per-thread sums across the block
  int incl = local;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, d);
    if (lane >= d) incl += y;
  }
  if (lane == 31) s_warp_sum[warp] = incl;
  __syncthreads();
  if (tid == 0) {
    int acc = 0;
    for (int w = 0; w < nthr / 32; ++w) {
      const int t = s_warp_sum[w];
      s_warp_sum[w] = acc;
      acc += t;
    }
    s_prefix[n] = acc;
  }
  __syncthreads();
  int run = s_warp_sum[warp] + incl - local;  // exclusive prefix of this thread
  for (int i = i0; i < min(n, i0 + per); ++i) {
    const int t = s_prefix[i];
    s_prefix[i] = run;
    run += t;
  }
  __syncthreads();
  return any_bad;
}

// Smallest sequence i with prefix[i + 1] > x (x below the total).
__device__ __forceinline__ int first_seq_after(const int* prefix, int n, long long x) {
  int lo = 0, hi = n - 1;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (prefix[mid + 1] > x) hi = mid; else lo = mid + 1;
  }
  return lo;
}

// -------------------------------------------------------------- merge
// Log-sum-exp merge of `cnt` <= MAXC partials (slots src0 + j*slot_stride)
// into either a normalised output out[n_heads*HD] or a partial at dst
// (which may be the first source slot).  Whole block.  The partials were
// written by other CTAs moments ago, so the merge is bound by L2 latency,
// not bandwidth: every thread issues all of its loads before using any.
// smem_w >= 3 * MAXC * n_heads + 2 * n_heads floats.
template <int MAXC, int HD>
__device__ __forceinline__ void merge_slots(const float* src0, size_t slot_stride, int cnt,
                                            int n_heads, float* out, float* dst, float* smem_w) {
  const int tid = threadIdx.x, nthr = blockDim.x;
  float* sm_m = smem_w;                  // [MAXC][n_heads]
  float* sm_l = sm_m + MAXC * n_heads;   // [MAXC][n_heads]
  float* sm_w = sm_l + MAXC * n_heads;   // [MAXC][n_heads] weights
  float* sM = sm_w + MAXC * n_heads;     // [n_heads]
  float* sL = sM + n_heads;              // [n_heads]
  // (1) every (m, l) pair in one sweep
  for (int t = tid; t < cnt * n_heads; t += nthr) {
    const int j = t / n_heads, h = t - j * n_heads;
    const float2 ml = __ldcg(reinterpret_cast<const float2*>(src0 + j * slot_stride +
                                                             h * part_stride(HD)));
    sm_m[t] = ml.x;
    sm_l[t] = ml.y;
  }
  __syncthreads();
  // (2) per head: max, weights, sum
  for (int h = tid; h < n_heads; h += nthr) {
    float M = -INFINITY;
    for (int j = 0; j < cnt; ++j) M = fmaxf(M, sm_m[j * n_heads + h]);
    float L = 0.f;
    for (int j = 0; j < cnt; ++j) {
      const float w = M == -INFINITY ? 0.f : ex2(sm_m[j * n_heads + h] - M);
      sm_w[j * n_heads + h] = w;
      L += w * sm_l[j * n_heads + h];
    }
    sM[h] = M;
    sL[h] = L;
    if (out) {
      const float inv = 1.0f / L;
      for (int j = 0; j < cnt; ++j) sm_w[j * n_heads + h] *= inv;
    }
  }
  __syncthreads();
  // (3) the weighted sums, float4 at a time, all loads of an output issued together
  for (int idx = tid; idx < n_heads * (HD / 4); idx += nthr) {
    const int h = idx / (HD / 4), q4 = idx % (HD / 4);
    const float* base = src0 + h * part_stride(HD) + kPartO + 4 * q4;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j0 = 0; j0 < cnt; j0 += 8) {  // 8 loads in flight per thread per round
      float4 v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (j0 + j < cnt) v[j] = __ldcg(reinterpret_cast<const float4*>(base + (j0 + j) * slot_stride));
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (j0 + j < cnt) {
          const float w = sm_w[(j0 + j) * n_heads + h];
          acc.x += w * v[j].x;
          acc.y += w * v[j].y;
          acc.z += w * v[j].z;
          acc.w += w * v[j].w;
        }
    }
    if (out)
      reinterpret_cast<float4*>(out + h * HD)[q4] = acc;
    else
      reinterpret_cast<float4*>(dst + h * part_stride(HD) + kPartO)[q4] = acc;
  }
  if (!out)
    for (int h = tid; h < n_heads; h += nthr) {
      dst[h * part_stride(HD)] = sM[h];
      dst[h * part_stride(HD) + 1] = sL[h];
    }
  __syncthreads();
}

// ------------------------------------------------------------ consumer
// KV head w of sequence i over local tiles [t_lo, t_hi); pipeline index of
// tile t_lo is it0.  Writes the final result if the segment is the whole
// sequence, else its partial to slot.  A K (or V) tile is HD/64 regions of
// region_bytes (the 64-element halves of every row, all KV heads), each in
// the 128-byte swizzle; head w's rows start at w * TP * 128 in a region.
template <int TP, int NSTAGE, int HD>
__device__ __forceinline__ void consume_segment(const DecodeArgs& a, int w, int lane, int i,
                                                int t_lo, int t_hi, int it0, bool whole,
                                                int slot, const uint8_t* sK, const uint8_t* sV,
                                                int tile_bytes, int region_bytes, uint64_t* full,
                                                uint64_t* empty, bool& ok) {
  constexpr int kHalves = HD / 64;
  const int kv_dim = a.n_kv_heads * HD;
  const int g = lane >> 2, c = lane & 3;
  const int kv_mul = a.kv_mul;
  const bool row_valid = g < kv_mul;
  const int qh = w * kv_mul + (row_valid ? g : 0);
  const int pos = pos_of(a, i);
  int att_rows, app_row;
  seq_rows(a, i, att_rows, app_row);
  const int slab = seq_of(a, i) * a.n_layers + a.layer;
  const float* cs = a.cos_tab + static_cast<size_t>(pos) * (HD / 2);
  const float* sn = a.sin_tab + static_cast<size_t>(pos) * (HD / 2);
  const bool appends = app_row >= t_lo * TP && app_row < t_hi * TP;

  // q fragments: this thread needs dims 16kk+2c, +1 and 16kk+8+2c, +1
  uint32_t qa[HD / 16][4];
  {
    const float* qrow = a.q + (static_cast<size_t>(i) * a.n_heads + qh) * HD;
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int d = 16 * kk + 8 * hf + 2 * c;
        float2 y = rope_two<HD>(qrow, d, cs, sn, a.rope_type);
        if (!row_valid) y = make_float2(0.f, 0.f);
        uint32_t hi, lo;
        split_hi_lo(y.x, y.y, hi, lo);
        qa[kk][2 * hf + 0] = hi;  // rows 0..7: high halves
        qa[kk][2 * hf + 1] = lo;  // rows 8..15: residuals
      }
    }
  }

  // the appended row: rotate k, encode k and v with picolm's FP16 rounding
  // (lane l holds the element pair 2l of every 64-element half)
  uint32_t kword[kHalves] = {}, vword[kHalves] = {};
  if (appends) {
    const float* krow = a.k + static_cast<size_t>(i) * kv_dim + w * HD;
    const float* vrow = a.v + static_cast<size_t>(i) * kv_dim + w * HD;
    const size_t off = (static_cast<size_t>(slab) * a.max_seq + app_row) * kv_dim + w * HD;
#pragma unroll
    for (int hv = 0; hv < kHalves; ++hv) {
      const int d = 64 * hv + 2 * lane;
      const float2 kr = rope_two<HD>(krow, d, cs, sn, a.rope_type);
      const float2 vv = *reinterpret_cast<const float2*>(vrow + d);
      kword[hv] = static_cast<uint32_t>(picolm_f32_to_f16(kr.x)) |
                  (static_cast<uint32_t>(picolm_f32_to_f16(kr.y)) << 16);
      vword[hv] = static_cast<uint32_t>(picolm_f32_to_f16(vv.x)) |
                  (static_cast<uint32_t>(picolm_f32_to_f16(vv.y)) << 16);
    }
#pragma unroll
    for (int hv = 0; hv < kHalves; ++hv) {
      reinterpret_cast<uint32_t*>(a.kc + off)[32 * hv + lane] = kword[hv];
      reinterpret_cast<uint32_t*>(a.vc + off)[32 * hv + lane] = vword[hv];
    }
  }

  float m_run = -INFINITY;  // running max of row g (log2 domain)
  float l_run = 0.f;        // this thread's share of the row sum
  float o[HD / 8][4];
#pragma unroll
  for (int j = 0; j < HD / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;

  for (int t = t_lo; t < t_hi && ok; ++t) {
    const int it = it0 + (t - t_lo);
    const int s = it % NSTAGE;
    if (!mbar_wait_bounded(&full[s], (it / NSTAGE) & 1)) {
      atomicOr(a.err, ERR_TIMEOUT_FULL);
      ok = false;
      break;
    }
    const uint32_t kbase = smem_u32(sK + s * tile_bytes + w * TP * 128);
    const uint32_t vbase = smem_u32(sV + s * tile_bytes + w * TP * 128);
    const int row0 = t * TP;
    const bool patch = appends && app_row >= row0 && app_row < row0 + TP;
    if (patch) {
      const int r = app_row - row0;
      const uint32_t off = sw128(r, lane >> 2) + (lane & 3) * 4;
#pragma unroll
      for (int hv = 0; hv < kHalves; ++hv) {
        const uint32_t ro = off + hv * region_bytes;
        asm volatile("st.shared.u32 [%0], %1;" ::"r"(kbase + ro), "r"(kword[hv]) : "memory");
        asm volatile("st.shared.u32 [%0], %1;" ::"r"(vbase + ro), "r"(vword[hv]) : "memory");
      }
      __syncwarp();
    }

    // S = Q K^T over TP rows
    float sacc[TP / 8][4];
#pragma unroll
    for (int nt = 0; nt < TP / 8; ++nt) {
      sacc[nt][0] = sacc[nt][1] = sacc[nt][2] = sacc[nt][3] = 0.f;
#pragma unroll
      for (int kp = 0; kp < HD / 32; ++kp) {
        const int r = nt * 8 + (lane & 7);
        const int ch = 4 * kp + (lane >> 3);  // 16-byte chunk of the row, HD/8 of them
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4(kbase + (ch >> 3) * region_bytes + sw128(r, ch & 7), b0, b1, b2, b3);
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
        const int tr = row0 + nt * 8 + 2 * c + e;
        float sc = (sacc[nt][e] + sacc[nt][2 + e]) * a.score_scale;
        sc = tr < att_rows ? sc : -INFINITY;
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
    for (int j = 0; j < HD / 8; ++j) {
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
      for (int j2 = 0; j2 < HD / 16; ++j2) {
        const int r = 16 * kk + ((lane >> 3) & 1) * 8 + (lane & 7);
        const int ch = 2 * j2 + (lane >> 4);
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4_trans(vbase + (ch >> 3) * region_bytes + sw128(r, ch & 7), b0, b1, b2, b3);
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
  if (whole && a.mode == 0) {
    const float inv = 1.0f / l_run;
    float* dst = a.out + static_cast<size_t>(i) * a.out_stride + qh * HD;
#pragma unroll
    for (int j = 0; j < HD / 8; ++j)
      *reinterpret_cast<float2*>(dst + 8 * j + 2 * c) =
          make_float2((o[j][0] + o[j][2]) * inv, (o[j][1] + o[j][3]) * inv);
  } else {
    constexpr int PS = part_stride(HD);
    float* dst = (whole ? a.part_out + static_cast<size_t>(i) * a.n_heads * PS
                        : a.part + static_cast<size_t>(slot) * a.n_heads * PS) +
                 qh * PS;
    if (c == 0) {
      dst[0] = m_run;
      dst[1] = l_run;
    }
#pragma unroll
    for (int j = 0; j < HD / 8; ++j)
      *reinterpret_cast<float2*>(dst + kPartO + 8 * j + 2 * c) =
          make_float2(o[j][0] + o[j][2], o[j][1] + o[j][3]);
  }
}

template <int TP, int NSTAGE, int HD>
__global__ void __launch_bounds__(288) decode_kernel(const __grid_constant__ DecodeArgs a,
                                                     const __grid_constant__ CUtensorMap tmk,
                                                     const __grid_constant__ CUtensorMap tmv) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ int s_prefix[kMaxLaunchSeqs + 1];
  __shared__ int s_warp_sum[9];
  __shared__ int s_seq_hint[kMaxLaunchSeqs];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int Hk = a.n_kv_heads;
  // one K (or V) tile: TP rows x all KV heads, as HD/64 regions of 64 elements
  const int region_bytes = TP * Hk * 128;
  const int tile_bytes = region_bytes * (HD / 64);
  uint8_t* sK = smem;
  uint8_t* sV = smem + NSTAGE * tile_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + 2 * NSTAGE * tile_bytes);
  uint64_t* empty = full + NSTAGE;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nthr = blockDim.x, n = a.n;

  // ---- set-up, overlapped with the end of the kernel queued before this one.
  // Launched with programmatic stream serialisation, this grid may start
  // while that kernel still runs.  Until griddepcontrol.wait it writes no
  // global memory and reads only the slots and positions, through L2, as a
  // hint: it scans the tile counts, partitions the tiles and prefetches this
  // CTA's first NSTAGE tiles into L2.  After the wait every count is taken
  // again from fresh loads and the scan is redone if one differs, so a stale
  // hint costs time, never a wrong result.
  scan_tiles<TP>(a, s_prefix, s_warp_sum, s_seq_hint, true);
  if (warp == Hk && lane == 0) {
    tma_prefetch_desc(&tmk);
    tma_prefetch_desc(&tmv);
    const long long Th = s_prefix[n];
    const long long Gh = static_cast<long long>(gridDim.x) < Th ? gridDim.x : Th;
    if (blockIdx.x < Gh) {
      const Partition Ph{s_prefix, Th, static_cast<int>(Gh)};
      const long long x0 = Ph.begin(blockIdx.x), x1 = Ph.begin(blockIdx.x + 1);
      int i = first_seq_after(s_prefix, n, x0);
      for (long long x = x0; x < x1 && x < x0 + NSTAGE; ++x) {
        while (s_prefix[i + 1] <= x) ++i;
        const int seq = s_seq_hint[i];  // in range: its tile count is not 0
        const int row = static_cast<int>(x - s_prefix[i]) * TP;
        const int slab = seq * a.n_layers + a.layer;
#pragma unroll
        for (int hv = 0; hv < HD / 64; ++hv) {
          tma_prefetch_l2_4d(&tmk, 64 * hv, row, 0, slab);
          tma_prefetch_l2_4d(&tmv, 64 * hv, row, 0, slab);
        }
      }
    }
  }
  if (tid == 0) {
    for (int s = 0; s < NSTAGE; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], Hk);
    }
    fence_mbar_init();
  }
  // everything the kernel queued before this one wrote is visible from here on
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // The merge grid may launch once every CTA is here: by then the slots and
  // positions are final, so the merge reads them before its own wait.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  {
    const int per = (n + nthr - 1) / nthr, i0 = tid * per;
    bool any_bad = false;
    int differs = 0;
    for (int i = i0; i < min(n, i0 + per); ++i) {
      bool bad;
      int seq;
      const int tiles = seq_tiles<TP>(a, i, false, bad, seq);
      any_bad |= bad;
      differs |= tiles != s_prefix[i + 1] - s_prefix[i];
    }
    // (also the barrier that publishes the mbarrier initialisation)
    if (__syncthreads_or(differs))
      any_bad = scan_tiles<TP>(a, s_prefix, s_warp_sum, s_seq_hint, false);
    if (any_bad && blockIdx.x == 0) atomicOr(a.err, ERR_BAD_ARG);
  }
  const long long T = s_prefix[n];
  if (T == 0) {  // no rows anywhere: nothing to merge either
    if (blockIdx.x == 0)
      for (int i = tid; i < n; i += nthr) a.seg_info[i] = make_int2(0, 0);
    if (a.err_host && gridDim.x == 1 && tid == 0)
      *reinterpret_cast<volatile uint32_t*>(a.err_host) = atomicOr(a.err, 0u);
    return;
  }
  const long long grid_ctas = static_cast<long long>(gridDim.x);
  Partition P{s_prefix, T, static_cast<int>(grid_ctas < T ? grid_ctas : T)};
  const int cta = blockIdx.x;
  if (cta == 0)
    for (int i = tid; i < n; i += nthr)
      a.seg_info[i] = s_prefix[i + 1] > s_prefix[i]
                          ? make_int2(P.slot(i, 0), P.n_seg(i)) : make_int2(0, 0);
  if (cta >= P.G) return;
  const long long x0 = P.begin(cta), x1 = P.begin(cta + 1);
  // first sequence with tiles in [x0, x1)
  const int i_first = first_seq_after(s_prefix, n, x0);

  bool ok = true;
  if (warp == Hk) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int i = i_first;
      long long issued = 0;
      for (long long x = x0; x < x1; ++x) {
        while (s_prefix[i + 1] <= x) ++i;
        const int it = static_cast<int>(x - x0);
        const int s = it % NSTAGE;
        if (it >= NSTAGE && !mbar_wait_bounded(&empty[s], ((it / NSTAGE) - 1) & 1)) {
          atomicOr(a.err, ERR_TIMEOUT_EMPTY);
          break;
        }
        mbar_arrive_expect_tx(&full[s], 2u * tile_bytes);
        const int row = static_cast<int>(x - s_prefix[i]) * TP;
        const int slab = seq_of(a, i) * a.n_layers + a.layer;
#pragma unroll
        for (int hv = 0; hv < HD / 64; ++hv) {
          tma_load_4d(sK + s * tile_bytes + hv * region_bytes, &tmk, &full[s], 64 * hv, row, 0,
                      slab);
          tma_load_4d(sV + s * tile_bytes + hv * region_bytes, &tmv, &full[s], 64 * hv, row, 0,
                      slab);
        }
        ++issued;
      }
      // never leave with copies in flight: the last use of each stage must land
      for (long long j = issued - NSTAGE; j < issued; ++j)
        if (j >= 0) mbar_wait_bounded(&full[j % NSTAGE], static_cast<uint32_t>((j / NSTAGE) & 1));
    }
  } else {
    // ------------------------------------------------------------ consumers
    for (int i = i_first; i < n && s_prefix[i] < x1 && ok; ++i) {
      const long long p0 = s_prefix[i], p1 = s_prefix[i + 1];
      const long long a0 = x0 > p0 ? x0 : p0, a1 = x1 < p1 ? x1 : p1;
      if (a1 <= a0) continue;
      const int t_lo = static_cast<int>(a0 - s_prefix[i]), t_hi = static_cast<int>(a1 - s_prefix[i]);
      const int ns = P.n_seg(i);
      const int j = cta - P.cta_of(s_prefix[i]);
      consume_segment<TP, NSTAGE, HD>(a, warp, lane, i, t_lo, t_hi, static_cast<int>(a0 - x0),
                                      ns == 1, P.slot(i, j), sK, sV, tile_bytes, region_bytes,
                                      full, empty, ok);
    }
  }
  // a one-CTA grid is the call's last kernel (no merge follows): report the
  // error word to the host once every warp of it is done
  if (a.err_host && gridDim.x == 1) {
    __syncthreads();
    if (tid == 0) *reinterpret_cast<volatile uint32_t*>(a.err_host) = atomicOr(a.err, 0u);
  }
}

// ---- exchange of a KV split over NVLink peer memory (one process per GPU)
// Each rank owns a receive buffer, mapped into every other rank's address
// space (CUDA IPC): a 256-byte header holding the rank's merge counter at
// byte 128, then for each epoch parity, each source rank and each head the
// source's partial (m, l, o) as ll_units(HD) 16-byte units
// {a, epoch, b, epoch}: unit 0 carries (m, l), unit 1 + j carries
// (o[2j], o[2j+1]).  A source writes each unit with one 16-byte volatile
// store into every rank's buffer (over NVLink for the peers).  A reader
// that finds the merge's epoch in both flag words of a unit has both
// values, since each 8-byte half is written and read whole, so neither a
// fence nor a separate flag is needed (the "low-latency" protocol of
// collective libraries); the data crosses NVLink once, with its flag.  Two
// parities alternate: a rank writes epoch e + 2 only after it has read every
// rank's epoch e + 1 units, and a rank stores those only once its merge of
// epoch e is complete, so no unit is overwritten while it may be read.  The
// epoch is the rank's merge counter plus one, kept on the device, so CUDA
// graphs of these calls replay; every rank merges equally often, so the
// counters agree.
constexpr int kXferMaxRanks = 8;
constexpr int kXferHeaderBytes = 256;
constexpr int kXferCounterOffset = 128;  // byte offset of the own merge counter

__host__ __device__ constexpr int ll_units(int hd) { return 1 + hd / 2; }

// Bytes of one rank's receive buffer.
__host__ __device__ constexpr size_t xfer_buffer_bytes(int world, int n_heads, int hd) {
  return kXferHeaderBytes + static_cast<size_t>(2) * world * n_heads * ll_units(hd) * 16;
}

struct XferPeers {
  uint8_t* base[kXferMaxRanks];  // each rank's receive buffer, as seen from this GPU
};

// The merge grid of a KV shard's partial exchanges it itself
// (merge_kernel<HD, true>): each block pushes its head and merges it.
struct XferPush {
  XferPeers peers;
  int world, rank;
  uint32_t* arrive;  // blocks of the merge grid that have read the counter (zero at rest)
  float* out;        // [n_heads * HD] merged output
};

// Unit u of head h from source rank src, epoch parity `parity`, in the
// buffer at base.
__device__ __forceinline__ uint8_t* ll_unit(uint8_t* base, uint32_t parity, int world, int src,
                                            int n_heads, int h, int u, int hd) {
  return base + kXferHeaderBytes +
         (((static_cast<size_t>(parity) * world + src) * n_heads + h) * ll_units(hd) + u) * 16;
}

__device__ __forceinline__ void st_ll(uint8_t* p, float a, float b, uint32_t e) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p),
               "r"(__float_as_uint(a)), "r"(e), "r"(__float_as_uint(b)), "r"(e)
               : "memory");
}

__device__ __forceinline__ uint4 ld_ll(const uint8_t* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

// Thread (h, q4) of an exchange: this rank's partial of head h -- o[4q4 ..
// 4q4 + 3] as units 1 + 2q4 and 2 + 2q4 and, from q4 == 0, (m, l) as unit
// 0 -- into slot (epoch & 1, rank) of every rank's buffer.
template <int HD>
__device__ __forceinline__ void ll_push(const XferPeers& peers, int world, int rank,
                                        int n_heads, uint32_t epoch, int h, int q4, float m,
                                        float l, float4 o) {
  for (int r = 0; r < world; ++r) {
    uint8_t* u0 = ll_unit(peers.base[r], epoch & 1u, world, rank, n_heads, h, 0, HD);
    st_ll(u0 + (1 + 2 * q4) * 16, o.x, o.y, epoch);
    st_ll(u0 + (2 + 2 * q4) * 16, o.z, o.w, epoch);
    if (q4 == 0) st_ll(u0, m, l, epoch);
  }
}

// Thread (h, q4): wait, bounded, for every rank's units of head h in this
// rank's buffer and write out[h * HD + 4q4 .. + 3], merged in log-sum-exp
// form.  Two ranks at a time: their six loads are issued together, only the
// units still missing are polled, and the pair is folded into a running
// (max, sum, o) (few registers, however many ranks).  False (nothing
// written) if a wait gave up.
template <int HD>
__device__ __forceinline__ bool ll_merge(const XferPeers& peers, int world, int rank,
                                         int n_heads, uint32_t epoch, int h, int q4,
                                         float* out) {
  const uint64_t lim = wait_limit_ns();
  uint64_t t0 = 0;
  float M = -INFINITY, L = 0.f;
  float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int r0 = 0; r0 < world; r0 += 2) {
    uint4 u[2][3];
    const uint8_t* src[2];
#pragma unroll
    for (int k = 0; k < 2; ++k)
      if (r0 + k < world) {
        src[k] = ll_unit(peers.base[rank], epoch & 1u, world, r0 + k, n_heads, h, 0, HD);
        u[k][0] = ld_ll(src[k]);
        u[k][1] = ld_ll(src[k] + (1 + 2 * q4) * 16);
        u[k][2] = ld_ll(src[k] + (2 + 2 * q4) * 16);
      }
#pragma unroll
    for (int k = 0; k < 2; ++k)
      if (r0 + k < world) {
#pragma unroll
        for (int j = 0; j < 3; ++j) {
          const int off = j == 0 ? 0 : (j + 2 * q4) * 16;
          while (u[k][j].y != epoch || u[k][j].w != epoch) {
            const uint64_t now = globaltimer();
            if (!t0) t0 = now;
            else if (now - t0 > lim) return false;
            u[k][j] = ld_ll(src[k] + off);
          }
        }
        const float m = __uint_as_float(u[k][0].x);
        if (m == -INFINITY) continue;  // an empty shard: l = 0, o = 0
        if (m > M) {
          const float sc = ex2(M - m);  // 0 while M is -inf
          L *= sc;
          o.x *= sc;
          o.y *= sc;
          o.z *= sc;
          o.w *= sc;
          M = m;
        }
        const float w = ex2(m - M);
        L += w * __uint_as_float(u[k][0].z);
        o.x += w * __uint_as_float(u[k][1].x);
        o.y += w * __uint_as_float(u[k][1].z);
        o.z += w * __uint_as_float(u[k][2].x);
        o.w += w * __uint_as_float(u[k][2].z);
      }
  }
  const float inv = 1.0f / L;
  reinterpret_cast<float4*>(out + static_cast<size_t>(h) * HD)[q4] =
      make_float4(o.x * inv, o.y * inv, o.z * inv, o.w * inv);
  return true;
}

// End of a pushing merge block: thread (h, q4) of an active head pushes
// and merges; the block that took the grid's last ticket (one per block,
// taken after the block read the counter) advances the counter to `epoch`
// and rearms the ticket count for the next merge grid.
template <int HD>
__device__ __forceinline__ void xfer_finish(const DecodeArgs& a, const XferPush& x,
                                            uint32_t epoch, uint32_t ticket, bool active, int h,
                                            int q4, float M, float L, float4 o) {
  if (active) {
    ll_push<HD>(x.peers, x.world, x.rank, a.n_heads, epoch, h, q4, M, L, o);
    if (!ll_merge<HD>(x.peers, x.world, x.rank, a.n_heads, epoch, h, q4, x.out))
      atomicOr(a.err, ERR_TIMEOUT_FULL);
  }
  if (threadIdx.x == blockDim.x - 1 && ticket == gridDim.x * gridDim.y - 1) {
    *reinterpret_cast<volatile uint32_t*>(x.peers.base[x.rank] + kXferCounterOffset) = epoch;
    *x.arrive = 0;
  }
}

// Merge of the segment partials of one decode launch.
// grid = (n, ceil(n_heads / hpb)), block = kMergeThreads; a block merges
// heads [h0, h0 + hpb) of sequence i.  Thread t owns float4 column q4 of
// head hh and every lanes-th segment (lanes = kMergeThreads / (hpb * HD/4);
// hpb * HD/4 <= kMergeThreads).
// Launched with programmatic stream serialisation behind decode_kernel, the
// grid (sized to stay resident) waits on griddepcontrol.wait; after it, one
// round trip reads the segment table and one more reads everything else:
// each thread loads (m, l) and o of all its segments at once, reduces them
// locally in log-sum-exp form, and the lanes are merged through shared
// memory.
constexpr int kMergeThreads = 256;

// Tile count of sequence i as the decode grid computed it (tp rows a tile;
// 0 for a slot or position out of range).
__device__ __forceinline__ int merge_seq_tiles(const DecodeArgs& a, int i, int tp) {
  const int seq = seq_of(a, i);
  const int pos = pos_of(a, i);
  const int att_rows = a.mode == 0 ? pos + 1 : a.n_rows;
  const int app_row = a.mode == 0 ? (a.append ? pos : -1) : (a.append ? pos - a.row0 : -1);
  const bool bad = seq < 0 || seq >= a.n_slots || pos < 0 || pos >= a.pos_limit ||
                   att_rows < 0 || att_rows > a.max_seq || app_row >= a.max_seq;
  return bad ? 0 : (att_rows + tp - 1) / tp;
}

// PUSH: the grid merges one KV shard's partial (mode 1, one sequence, one
// head per block) and exchanges it (XferPush): each block pushes its head to
// every rank and merges every rank's partial of that head into x.out.
template <int HD, bool PUSH>
__global__ void __launch_bounds__(kMergeThreads) merge_kernel(const __grid_constant__ DecodeArgs a,
                                                              int hpb,
                                                              int decode_ctas, int tp,
                                                              const XferPush x) {
  __shared__ uint32_t s_epoch;
  __shared__ float4 s_acc[kMergeThreads];
  __shared__ float2 s_ml[kMergeThreads];
  __shared__ long long s_red[2][kMergeThreads / 32];
  // a merge of KV shards queued behind this grid may become resident now
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int i = blockIdx.x, h0 = blockIdx.y * hpb, tid = threadIdx.x;
  // This sequence's segments, from the same partition the decode grid used
  // (the grid launched this one after every decode CTA had passed its own
  // griddepcontrol.wait, so the slots and positions read here are final):
  // tiles before sequence i and in total, then its first slot and count.
  long long before = 0, total = 0;
  for (int j = tid; j < a.n; j += kMergeThreads) {
    const int t = merge_seq_tiles(a, j, tp);
    total += t;
    if (j < i) before += t;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    before += __shfl_xor_sync(0xffffffffu, before, o);
    total += __shfl_xor_sync(0xffffffffu, total, o);
  }
  if ((tid & 31) == 0) {
    s_red[0][tid >> 5] = before;
    s_red[1][tid >> 5] = total;
  }
  __syncthreads();
  before = total = 0;
  for (int w = 0; w < kMergeThreads / 32; ++w) {
    before += s_red[0][w];
    total += s_red[1][w];
  }
  const int mine = merge_seq_tiles(a, i, tp);
  // the decode grid's partials are visible from here on
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // every decode CTA has finished: its error bits are final
  if (a.err_host && i == 0 && blockIdx.y == 0 && tid == 0)
    *reinterpret_cast<volatile uint32_t*>(a.err_host) = atomicOr(a.err, 0u);
  constexpr int PS = part_stride(HD);
  const int pairs = hpb * (HD / 4), lanes = kMergeThreads / pairs;
  const int pair = tid % pairs, lane_j = tid / pairs;
  const int hh = pair / (HD / 4), q4 = pair % (HD / 4), h = h0 + hh;
  const bool active = lane_j == 0 && h < a.n_heads;
  // PUSH: this merge's epoch, one past the counter that the previous merge
  // grid (complete before the decode grid, and so this one, passed its
  // wait) left in this rank's buffer; then one ticket per block, taken
  // after the read
  uint32_t epoch = 0, ticket = 0;
  if constexpr (PUSH) {
    if (tid == 0)
      s_epoch = *reinterpret_cast<volatile const uint32_t*>(x.peers.base[x.rank] +
                                                            kXferCounterOffset) + 1u;
    __syncthreads();
    epoch = s_epoch;
    if (tid == kMergeThreads - 1) ticket = atomicAdd(x.arrive, 1u);
  }
  if (mine == 0 || total == 0) {
    if constexpr (PUSH)  // an empty or rejected shard contributes nothing
      xfer_finish<HD>(a, x, epoch, ticket, active, h, q4, -INFINITY, 0.f,
                      make_float4(0.f, 0.f, 0.f, 0.f));
    return;
  }
  const int G = static_cast<int>(decode_ctas < total ? decode_ctas : total);
  const int c_first = static_cast<int>(((before + 1) * G - 1) / total);
  const int c_last = static_cast<int>(((before + mine) * G - 1) / total);
  const int ns = c_last - c_first + 1;
  if (ns <= 1) {  // finished by its single segment (into part_out in mode 1)
    if constexpr (PUSH) {
      float2 ml = make_float2(-INFINITY, 0.f);
      float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
      if (active) {
        const float* src = a.part_out + static_cast<size_t>(h) * PS;
        ml = __ldcg(reinterpret_cast<const float2*>(src));
        o = __ldcg(reinterpret_cast<const float4*>(src + kPartO) + q4);
      }
      xfer_finish<HD>(a, x, epoch, ticket, active, h, q4, ml.x, ml.y, o);
    }
    return;
  }
  const int2 si = make_int2(c_first + i, ns);
  const size_t slot_stride = static_cast<size_t>(a.n_heads) * PS;
  float m_loc = -INFINITY, l_loc = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  if (lane_j < lanes && h < a.n_heads) {
    const float* base = a.part + static_cast<size_t>(si.x) * slot_stride + h * PS;
    // U segments in flight per thread: at head_dim 64 and one head per
    // block (16 lanes) one round trip covers the 148 segments of a sequence
    // split over every SM.  At head_dim 128 more would cost the registers
    // that let a merge block sit beside a decode CTA.
    constexpr int U = HD == 64 ? 10 : 8;
    for (int j0 = lane_j; j0 < ns; j0 += U * lanes) {
      float2 ml[U];
      float4 v[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int j = j0 + u * lanes;
        if (j < ns) {
          ml[u] = __ldcg(reinterpret_cast<const float2*>(base + j * slot_stride));
          v[u] = __ldcg(reinterpret_cast<const float4*>(base + j * slot_stride + kPartO) + q4);
        }
      }
      float mx = m_loc;
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (j0 + u * lanes < ns) mx = fmaxf(mx, ml[u].x);
      if (mx != -INFINITY) {
        const float sc = ex2(m_loc - mx);
        l_loc *= sc;
        acc.x *= sc;
        acc.y *= sc;
        acc.z *= sc;
        acc.w *= sc;
#pragma unroll
        for (int u = 0; u < U; ++u)
          if (j0 + u * lanes < ns) {
            const float w = ex2(ml[u].x - mx);
            l_loc += w * ml[u].y;
            acc.x += w * v[u].x;
            acc.y += w * v[u].y;
            acc.z += w * v[u].z;
            acc.w += w * v[u].w;
          }
        m_loc = mx;
      }
    }
  }
  s_acc[tid] = acc;
  s_ml[tid] = make_float2(m_loc, l_loc);
  __syncthreads();
  float M = m_loc, L = 0.f;
  float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
  if (active) {
    for (int l = 1; l < lanes; ++l) M = fmaxf(M, s_ml[tid + l * pairs].x);
    if (M != -INFINITY)
      for (int l = 0; l < lanes; ++l) {
        const float2 ml = s_ml[tid + l * pairs];
        const float4 xv = s_acc[tid + l * pairs];
        const float w = ex2(ml.x - M);
        L += w * ml.y;
        o.x += w * xv.x;
        o.y += w * xv.y;
        o.z += w * xv.z;
        o.w += w * xv.w;
      }
    if constexpr (PUSH) {
      // pushed and merged below, with the rest of the block
    } else if (a.mode == 0) {
      const float inv = 1.0f / L;
      reinterpret_cast<float4*>(a.out + static_cast<size_t>(i) * a.out_stride + h * HD)[q4] =
          make_float4(o.x * inv, o.y * inv, o.z * inv, o.w * inv);
    } else {
      float* dst = a.part_out + (static_cast<size_t>(i) * a.n_heads + h) * PS;
      reinterpret_cast<float4*>(dst + kPartO)[q4] = o;
      if (q4 == 0) {
        dst[0] = M;
        dst[1] = L;
      }
    }
  }
  if constexpr (PUSH) xfer_finish<HD>(a, x, epoch, ticket, active, h, q4, M, L, o);
}

// Log-sum-exp merge of partials gathered from several devices (one
// sequence): n_part <= kMaxCombineParts blocks of [n_heads][part_stride(HD)]
// back to back.  grid = 1, block = 256.
template <int HD>
__global__ void __launch_bounds__(256) combine_kernel(int n_part, int n_heads,
                                                      const float* __restrict__ parts,
                                                      float* __restrict__ out) {
  extern __shared__ float smem_w[];
  merge_slots<kMaxCombineParts, HD>(parts, static_cast<size_t>(n_heads) * part_stride(HD), n_part,
                                    n_heads, out, nullptr, smem_w);
}

// Log-sum-exp merge of partials that sit on several devices of one process
// (a KV split inside one module context): the n_part partial blocks are read
// straight from the other devices' memory over NVLink (plain loads; the
// device has peer access to them), after the stream has waited on each
// producer's event.  grid = ceil(n_heads * HD/4 / 256), block = 256: thread
// t owns float4 q4 of head h and loads (m, l) and o of every partial first.
constexpr int kMaxPeerParts = 16;
struct PeerParts {
  const float* p[kMaxPeerParts];
};

template <int HD>
__global__ void __launch_bounds__(256) combine_peers_kernel(PeerParts parts, int n_part,
                                                            int n_heads,
                                                            float* __restrict__ out) {
  constexpr int PS = part_stride(HD);
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n_heads * (HD / 4)) return;
  const int h = idx / (HD / 4), q4 = idx % (HD / 4);
  float2 ml[kMaxPeerParts];
  float4 o[kMaxPeerParts];
#pragma unroll
  for (int j = 0; j < kMaxPeerParts; ++j)
    if (j < n_part) {
      const float* base = parts.p[j] + h * PS;
      ml[j] = __ldcg(reinterpret_cast<const float2*>(base));
      o[j] = __ldcg(reinterpret_cast<const float4*>(base + kPartO) + q4);
    }
  float M = -INFINITY;
#pragma unroll
  for (int j = 0; j < kMaxPeerParts; ++j)
    if (j < n_part) M = fmaxf(M, ml[j].x);
  float L = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  if (M != -INFINITY) {
#pragma unroll
    for (int j = 0; j < kMaxPeerParts; ++j)
      if (j < n_part) {
        const float w = ex2(ml[j].x - M);
        L += w * ml[j].y;
        acc.x += w * o[j].x;
        acc.y += w * o[j].y;
        acc.z += w * o[j].z;
        acc.w += w * o[j].w;
      }
  }
  const float inv = 1.0f / L;
  reinterpret_cast<float4*>(out + h * HD)[q4] =
      make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
}

}  // namespace pl
