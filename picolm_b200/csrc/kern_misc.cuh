// kern_misc.cuh -- small element-wise kernels around the attention path:
// in-place RoPE (bit-exact picolm rotation) and the prefill prologue that
// rotates q/k, appends k/v to the FP16 cache and stages q as FP16 for the
// tensor-core prefill.
#pragma once
#include <cstdint>

#include "kern_decode.cuh"
#include "pl_fp16.cuh"

namespace pl {

// RoPE in place on n_tok rows of q [n_tok][n_heads*HD] and k
// [n_tok][n_kv_heads*HD]; row r uses the table row pos0 + r.
// grid = (n_tok, ceil((n_heads + n_kv_heads) / 8)), block = 256: warp w of
// block (r, y) handles head 8y + w of row r, lane l its element pairs 2l,
// 2l + 64, ...
template <int HD>
__global__ void rope_inplace_kernel(float* q, float* k, int n_heads, int n_kv_heads, int pos0,
                                    const float* cos_tab, const float* sin_tab, int rope_type) {
  const int r = blockIdx.x;
  const int head = blockIdx.y * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (head >= n_heads + n_kv_heads) return;
  const int pos = pos0 + r;
  const float* cs = cos_tab + static_cast<size_t>(pos) * (HD / 2);
  const float* sn = sin_tab + static_cast<size_t>(pos) * (HD / 2);
  float* x;
  if (head < n_heads) {
    if (!q) return;
    x = q + (static_cast<size_t>(r) * n_heads + head) * HD;
  } else {
    if (!k) return;
    x = k + (static_cast<size_t>(r) * n_kv_heads + (head - n_heads)) * HD;
  }
  // all reads of the head happen before any write (Qwen pairs cross lanes)
  float2 y[HD / 64];
#pragma unroll
  for (int hv = 0; hv < HD / 64; ++hv) y[hv] = rope_two<HD>(x, 64 * hv + 2 * lane, cs, sn, rope_type);
  __syncwarp();
#pragma unroll
  for (int hv = 0; hv < HD / 64; ++hv) *reinterpret_cast<float2*>(x + 64 * hv + 2 * lane) = y[hv];
}

// Prefill prologue for n_tok rows starting at position start_pos:
//   q16[r][h][d]  = FP16(RoPE(q[r][h][:]))[d]       (tensor-core operand,
//                                                     round-to-nearest-even)
//   q16lo[r][h][d] = FP16(y - q16[r][h][d]), y the rotated FP32 value: the
//                    residual, so that hi + lo carries y to about 2^-22
//   kc[start+r]   = picolm_FP16(RoPE(k[r]))          (bit-exact append)
//   vc[start+r]   = picolm_FP16(v[r])
// A row is cut into units of 8 elements of one head (q heads, then k heads,
// then v heads; HD/8 units per head).
// LLaMA units are 8 consecutive elements (4 rotated pairs); Qwen units are
// elements 4c..4c+3 and HD/2+4c..HD/2+4c+3, which rotate into each other.
// With q16 null the q units are skipped (the cache rows alone).  Every input and all
// RoPE factors of a unit are 16-byte loads.  q, k, v rows and the cache rows
// must be 16-byte aligned.
constexpr int kPrologueThreads = 256;

struct PrologueUnit {
  float4 xa, xb, c, s;  // inputs (xa: first 4, xb: second 4) and RoPE factors
  int kind;             // 0 q, 1 k, 2 v, -1 none
  int head, part;
};

template <int HD>
__device__ __forceinline__ PrologueUnit prologue_load(int u, int r, const float* __restrict__ q,
                                                      const float* __restrict__ k,
                                                      const float* __restrict__ v, int n_heads,
                                                      int n_kv_heads, const float* cs,
                                                      const float* sn, int rope_type) {
  PrologueUnit pu;
  constexpr int kUnits = HD / 8;  // units per head
  const int nq = n_heads * kUnits, nk = n_kv_heads * kUnits;
  const int kv_dim = n_kv_heads * HD;
  const float* x;
  if (u < nq) {
    pu.kind = 0;
    pu.head = u / kUnits;
    x = q + (static_cast<size_t>(r) * n_heads + pu.head) * HD;
  } else if (u < nq + nk) {
    pu.kind = 1;
    pu.head = (u - nq) / kUnits;
    x = k + static_cast<size_t>(r) * kv_dim + pu.head * HD;
  } else {
    pu.kind = 2;
    pu.head = (u - nq - nk) / kUnits;
    x = v + static_cast<size_t>(r) * kv_dim + pu.head * HD;
  }
  pu.part = u % kUnits;
  if (pu.kind == 2 || rope_type == 0) {
    pu.xa = *reinterpret_cast<const float4*>(x + 8 * pu.part);
    pu.xb = *reinterpret_cast<const float4*>(x + 8 * pu.part + 4);
  } else {
    pu.xa = *reinterpret_cast<const float4*>(x + 4 * pu.part);
    pu.xb = *reinterpret_cast<const float4*>(x + HD / 2 + 4 * pu.part);
  }
  if (pu.kind != 2) {
    pu.c = *reinterpret_cast<const float4*>(cs + 4 * pu.part);
    pu.s = *reinterpret_cast<const float4*>(sn + 4 * pu.part);
  }
  return pu;
}

// k and v use picolm's FP16 rounding (bit-exact cache rows); q goes to the
// tensor-core staging as an FP16 high part and FP16 residual (split_hi_lo).
__device__ __forceinline__ uint32_t prologue_pack(float a, float b, bool picolm_rounding) {
  if (!picolm_rounding) return pack_half2(a, b);
  return static_cast<uint32_t>(picolm_f32_to_f16(a)) |
         (static_cast<uint32_t>(picolm_f32_to_f16(b)) << 16);
}

// Store 2n rotated values as FP16 words: picolm's rounding for the cache
// rows (kind 1), the hi/lo split for q (kind 0, lo at dst + lo_off).
template <int N>
__device__ __forceinline__ void store_words(uint16_t* dst, long lo_off, const float* y, int kind) {
  uint32_t hi[N], lo[N];
#pragma unroll
  for (int i = 0; i < N; ++i) {
    if (kind == 0)
      split_hi_lo(y[2 * i], y[2 * i + 1], hi[i], lo[i]);
    else
      hi[i] = prologue_pack(y[2 * i], y[2 * i + 1], true);
  }
  if constexpr (N == 4) {
    *reinterpret_cast<uint4*>(dst) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    if (kind == 0) *reinterpret_cast<uint4*>(dst + lo_off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
  } else {
    *reinterpret_cast<uint2*>(dst) = make_uint2(hi[0], hi[1]);
    if (kind == 0) *reinterpret_cast<uint2*>(dst + lo_off) = make_uint2(lo[0], lo[1]);
  }
}

template <int HD>
__device__ __forceinline__ void prologue_store(const PrologueUnit& pu, int r, uint16_t* q16,
                                               long q16_lo_off, uint16_t* kc_rows,
                                               uint16_t* vc_rows, int n_heads, int n_kv_heads,
                                               int rope_type) {
  const int kv_dim = n_kv_heads * HD;
  uint16_t* dst;
  if (pu.kind == 0)
    dst = q16 + (static_cast<size_t>(r) * n_heads + pu.head) * HD;
  else
    dst = (pu.kind == 1 ? kc_rows : vc_rows) + static_cast<size_t>(r) * kv_dim + pu.head * HD;
  if (pu.kind == 2) {
    *reinterpret_cast<uint4*>(dst + 8 * pu.part) =
        make_uint4(prologue_pack(pu.xa.x, pu.xa.y, true), prologue_pack(pu.xa.z, pu.xa.w, true),
                   prologue_pack(pu.xb.x, pu.xb.y, true), prologue_pack(pu.xb.z, pu.xb.w, true));
  } else if (rope_type == 0) {
    float y[8];
    rope_pair(pu.xa.x, pu.xa.y, pu.c.x, pu.s.x, y[0], y[1]);
    rope_pair(pu.xa.z, pu.xa.w, pu.c.y, pu.s.y, y[2], y[3]);
    rope_pair(pu.xb.x, pu.xb.y, pu.c.z, pu.s.z, y[4], y[5]);
    rope_pair(pu.xb.z, pu.xb.w, pu.c.w, pu.s.w, y[6], y[7]);
    store_words<4>(dst + 8 * pu.part, q16_lo_off, y, pu.kind);
  } else {
    // Qwen: element j (< HD/2) and j + HD/2 rotate together
    const float xa[4] = {pu.xa.x, pu.xa.y, pu.xa.z, pu.xa.w};
    const float xb[4] = {pu.xb.x, pu.xb.y, pu.xb.z, pu.xb.w};
    const float c[4] = {pu.c.x, pu.c.y, pu.c.z, pu.c.w};
    const float sv[4] = {pu.s.x, pu.s.y, pu.s.z, pu.s.w};
    float lo[4], hi[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      lo[i] = __fsub_rn(__fmul_rn(xa[i], c[i]), __fmul_rn(xb[i], sv[i]));
      hi[i] = __fadd_rn(__fmul_rn(xa[i], sv[i]), __fmul_rn(xb[i], c[i]));
    }
    store_words<2>(dst + 4 * pu.part, q16_lo_off, lo, pu.kind);
    store_words<2>(dst + HD / 2 + 4 * pu.part, q16_lo_off, hi, pu.kind);
  }
}

// The (row, unit) pairs of the call are one flattened list, walked by a
// persistent grid of kPrologueBlocksPerSm blocks per SM: each thread takes
// kPrologueUnitsInFlight units per round, all their loads issued before any
// compute.  The kernel is latency-bound; resident warps hide that better
// than units per thread (same-box A/B of the 22-layer config-3 call: one
// unit at four blocks per SM 1.042-1.044 ms, two at three 1.057-1.059 ms,
// three or four at two 1.15-1.27 ms).
constexpr int kPrologueBlocksPerSm = 4;
constexpr int kPrologueUnitsInFlight = 1;

template <int HD>
__global__ void __launch_bounds__(kPrologueThreads, kPrologueBlocksPerSm)
    prefill_prologue_kernel(const float* __restrict__ q, const float* __restrict__ k,
                            const float* __restrict__ v, uint16_t* __restrict__ q16,
                            long q16_lo_off, uint16_t* __restrict__ kc_rows,
                            uint16_t* __restrict__ vc_rows,
                            int n_tok, int n_heads, int n_kv_heads, int start_pos,
                            const float* cos_tab, const float* sin_tab, int rope_type) {
  // the attention grid queued behind (programmatic dependent launch) may
  // start its set-up now; it waits for this grid before touching its output
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  constexpr int U = kPrologueUnitsInFlight;
  const int u0 = q16 ? 0 : n_heads * (HD / 8);  // without q16: the cache rows alone
  const int per_row = (n_heads + 2 * n_kv_heads) * (HD / 8) - u0;
  const long total = static_cast<long>(n_tok) * per_row;
  const long stride = static_cast<long>(gridDim.x) * kPrologueThreads * U;
  for (long f0 = static_cast<long>(blockIdx.x) * kPrologueThreads * U + threadIdx.x; f0 < total;
       f0 += stride) {
    PrologueUnit pu[U];
    int row[U];
#pragma unroll
    for (int j = 0; j < U; ++j) {
      const long f = f0 + static_cast<long>(j) * kPrologueThreads;
      pu[j].kind = -1;
      row[j] = 0;
      if (f < total) {
        const int r = static_cast<int>(f / per_row);
        const int u = u0 + static_cast<int>(f - static_cast<long>(r) * per_row);
        const size_t trow = static_cast<size_t>(start_pos + r) * (HD / 2);
        pu[j] = prologue_load<HD>(u, r, q, k, v, n_heads, n_kv_heads, cos_tab + trow,
                                  sin_tab + trow, rope_type);
        row[j] = r;
      }
    }
#pragma unroll
    for (int j = 0; j < U; ++j)
      if (pu[j].kind >= 0)
        prologue_store<HD>(pu[j], row[j], q16, q16_lo_off, kc_rows, vc_rows, n_heads,
                           n_kv_heads, rope_type);
  }
}

// Blocks of the prologue grid: enough for every unit, at most
// kPrologueBlocksPerSm per SM.
inline int prologue_grid(int n_tok, int n_heads, int n_kv_heads, int head_dim, bool with_q,
                         int num_sms) {
  const long per_row = static_cast<long>(with_q ? n_heads + 2 * n_kv_heads : 2 * n_kv_heads) *
                       (head_dim / 8);
  const long per_block = static_cast<long>(kPrologueThreads) * kPrologueUnitsInFlight;
  const long need = (static_cast<long>(n_tok) * per_row + per_block - 1) / per_block;
  const long cap = static_cast<long>(num_sms) * kPrologueBlocksPerSm;
  return static_cast<int>(need < cap ? (need < 1 ? 1 : need) : cap);
}

// Copy of n16 16-byte words from src (host memory mapped into the device:
// a registered caller buffer) to dst (HBM) by loads over the bus from every
// SM.  Used in place of a cudaMemcpyAsync for the q of a host-buffer
// decode: the decode grid is queued behind it with programmatic dependent
// launch, so it is resident and through its set-up when the copy ends.
// grid-stride, block 256.
__global__ void __launch_bounds__(256)
    bus_gather_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst, long n16) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const long stride = static_cast<long>(gridDim.x) * blockDim.x;
  long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x;
  // two words in flight per thread before either is stored
  for (; i + stride < n16; i += 2 * stride) {
    const uint4 a = src[i], b = src[i + stride];
    dst[i] = a;
    dst[i + stride] = b;
  }
  if (i < n16) dst[i] = src[i];
}

}  // namespace pl
