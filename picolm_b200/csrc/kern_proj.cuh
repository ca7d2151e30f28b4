// kern_proj.cuh -- the projections on either side of the attention path,
// on the device:
//   * RMSNorm of the residual stream and the Q, K, V projections with their
//     biases (picolm/model.c:779-799; prefill model.c:990-1012),
//   * QK-norm, a per-head RMSNorm of q and k before RoPE (model.c:807-817),
//   * the output projection, its bias and the residual add
//     (model.c:894-897; prefill model.c:1092-1100).
// The weights stay in their GGUF quantisation in HBM; every projection is a
// GEMV (decode) or a skinny GEMM over a few input rows at a time (prefill),
// bound by the weight bytes it streams.
//
// Dot products follow the factored forms of picolm's vec_dot kernels
// (quant.c:340-712): integer quants times x summed per scale group, then
// scaled -- Q4_K  d1*sum(q*x) - m1*sum(x) per 32-weight sub-block,
// Q6_K (d*sc)*sum(q*x) per 16, Q8_0 d*sum(q*x) per block.  The summation
// order differs from the CPU's (lanes, then a warp butterfly), so results
// agree with picolm to FP32 rounding, not bit for bit.
#pragma once
#include <cstdint>
#include <cuda_fp16.h>

#include "sm100.cuh"

namespace pl {

// GGUF tensor type ids (picolm/quant.h:49-63) that the projections take
constexpr int kGgufF32 = 0, kGgufF16 = 1, kGgufQ8_0 = 8, kGgufQ4K = 12, kGgufQ6K = 14;

// Device layout of one weight row of n inputs.  The caller's GGUF bytes are
// repacked at upload so that every lane load below is naturally aligned:
//   F32   n floats                          (as GGUF)
//   F16   n halves                          (as GGUF)
//   Q8_0  n int8 quants, then n/32 FP16 scales, padded to 16 bytes
//         (GGUF interleaves them as 34-byte blocks {d, qs[32]})
//   Q4_K  n/256 blocks of 144 bytes {d, dmin, scales[12], qs[128]} (as GGUF)
//   Q6_K  n/256 blocks of 224 bytes {ql[128], qh[64], scales[16], d, 14 pad}
//         (GGUF: the same fields in 210-byte blocks)
constexpr int kQ4KBytes = 144, kQ6KBytes = 224, kQ6KGgufBytes = 210;

__host__ __device__ inline bool proj_type_ok(int type) {
  return type == kGgufF32 || type == kGgufF16 || type == kGgufQ8_0 || type == kGgufQ4K ||
         type == kGgufQ6K;
}
// inputs a row length must be a multiple of
__host__ __device__ inline int proj_granule(int type) {
  return type == kGgufQ4K || type == kGgufQ6K ? 256 : type == kGgufQ8_0 ? 32 : 8;
}
__host__ __device__ inline size_t proj_row_bytes(int type, int n) {
  switch (type) {
    case kGgufF32: return static_cast<size_t>(n) * 4;
    case kGgufF16: return static_cast<size_t>(n) * 2;
    case kGgufQ8_0: return (static_cast<size_t>(n) + n / 16 + 15) & ~static_cast<size_t>(15);
    case kGgufQ4K: return static_cast<size_t>(n / 256) * kQ4KBytes;
    case kGgufQ6K: return static_cast<size_t>(n / 256) * kQ6KBytes;
    default: return 0;
  }
}

constexpr int kProjWarps = 8;                 // output rows per CTA (one per warp)
constexpr int kProjThreads = 32 * kProjWarps;
constexpr int kProjMaxM = 8;                  // input rows per CTA
constexpr int kProjSmemCap = 200 * 1024;      // staged input rows

struct ProjMat {
  const uint8_t* w;    // rows in the device layout above
  const float* bias;   // [rows] or nullptr
  float* out;          // out[m * ld_out + row]
  size_t row_bytes;
  int type, rows, ld_out;
};

// Up to three matrices over the same input rows (Q, K, V in one launch);
// row r of the launch is row r - (rows of the matrices before) of matrix i.
struct ProjArgs {
  ProjMat mat[3];
  int n_mat, total_rows;
  const float* x;      // input rows x[m * ldx + i], i < n; 16-byte aligned, ldx % 4 == 0
  int ldx, n, M;
  const float* norm_w; // RMSNorm weights [n]: the input rows are normalised first
  float eps;
  const float* resid;  // out = resid + (W x + b) when set (in place allowed: resid == out)
  int ld_res;
  int mc;              // input rows per CTA; grid.y = ceil(M / mc)
  // tensor-core path with the inputs split over grid.z slices: slice z
  // writes its raw partial sums to part[(z * M + m) * total_rows + launch
  // row], and proj_reduce_kernel adds the slices, bias and residual
  float* part;
  int ksplit;
};

__device__ __forceinline__ float f16_bits(uint32_t h) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(h)));
}
__device__ __forceinline__ uint32_t byte_of(uint32_t w0, uint32_t w1, uint32_t w2, int k) {
  const uint32_t w = k < 4 ? w0 : (k < 8 ? w1 : w2);
  return (w >> (8 * (k & 3))) & 0xFFu;
}
// picolm/quant.c:82-90 get_scale_min_k4 over the 12 scale bytes held in w0..w2
__device__ __forceinline__ void scale_min_k4(int j, uint32_t w0, uint32_t w1, uint32_t w2,
                                             float& sc, float& mn) {
  if (j < 4) {
    sc = static_cast<float>(byte_of(w0, w1, w2, j) & 63u);
    mn = static_cast<float>(byte_of(w0, w1, w2, j + 4) & 63u);
  } else {
    const uint32_t a = byte_of(w0, w1, w2, j + 4);
    sc = static_cast<float>((a & 0xFu) | ((byte_of(w0, w1, w2, j - 4) >> 6) << 4));
    mn = static_cast<float>((a >> 4) | ((byte_of(w0, w1, w2, j) >> 6) << 4));
  }
}

__device__ __forceinline__ float dot4(float4 a, float4 b, float s) {
  s = fmaf(a.x, b.x, s);
  s = fmaf(a.y, b.y, s);
  s = fmaf(a.z, b.z, s);
  return fmaf(a.w, b.w, s);
}
__device__ __forceinline__ float sum4(float4 a) { return (a.x + a.y) + (a.z + a.w); }

// Small unsigned integers (< 2^23) to float without the conversion unit:
// byte k of w becomes the low byte of 0x4B000000 (2^23 with the integer in
// its mantissa); subtracting 2^23 + bias is exact.  One byte permute and one
// add instead of an I2F, which runs at an eighth of the FMA rate.
__device__ __forceinline__ float4 bytes_to_f4(uint32_t w, float bias) {
  const float base = 8388608.0f + bias;
  return make_float4(__int_as_float(static_cast<int>(__byte_perm(w, 0x4B000000u, 0x7440))) - base,
                     __int_as_float(static_cast<int>(__byte_perm(w, 0x4B000000u, 0x7441))) - base,
                     __int_as_float(static_cast<int>(__byte_perm(w, 0x4B000000u, 0x7442))) - base,
                     __int_as_float(static_cast<int>(__byte_perm(w, 0x4B000000u, 0x7443))) - base);
}

// Each lane takes work units u = lane, lane + 32, ... of a row (4 to 16
// weights each, consecutive lanes on consecutive bytes) for R consecutive
// rows at once, U units per step with all their loads issued first, and
// adds its partial dots with every staged input row m < mc into acc[i][m].
// The R rows share the block layout, so one read of the x chunk (and of
// its sums) from shared memory serves all of them; the weights are turned
// into floats once per unit, outside the loop over input rows.

template <int R, int U>
__device__ __forceinline__ void rows_f32(const uint8_t* w0, size_t rb, const float* xs, int n,
                                         int mc, int lane, float (*acc)[kProjMaxM]) {
  const float4* x4 = reinterpret_cast<const float4*>(xs);
  const int units = n / 4, n4 = n / 4;
  for (int u0 = lane; u0 < units; u0 += 32 * U) {
    float4 w[U][R];
#pragma unroll
    for (int k = 0; k < U; ++k)
#pragma unroll
      for (int i = 0; i < R; ++i)
        w[k][i] = u0 + 32 * k < units
                      ? __ldg(reinterpret_cast<const float4*>(w0 + i * rb) + u0 + 32 * k)
                      : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int k = 0; k < U; ++k) {
      const int u = u0 + 32 * k;
      if (u >= units) break;
#pragma unroll
      for (int m = 0; m < kProjMaxM; ++m)
        if (m < mc) {
          const float4 xv = x4[m * n4 + u];
#pragma unroll
          for (int i = 0; i < R; ++i) acc[i][m] = dot4(w[k][i], xv, acc[i][m]);
        }
    }
  }
}

template <int R, int U>
__device__ __forceinline__ void rows_f16(const uint8_t* w0, size_t rb, const float* xs, int n,
                                         int mc, int lane, float (*acc)[kProjMaxM]) {
  const float4* x4 = reinterpret_cast<const float4*>(xs);
  const int units = n / 8, n4 = n / 4;
  for (int u0 = lane; u0 < units; u0 += 32 * U) {
    uint4 q[U][R];
#pragma unroll
    for (int k = 0; k < U; ++k)
#pragma unroll
      for (int i = 0; i < R; ++i)
        q[k][i] = u0 + 32 * k < units
                      ? __ldg(reinterpret_cast<const uint4*>(w0 + i * rb) + u0 + 32 * k)
                      : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
    for (int k = 0; k < U; ++k) {
      const int u = u0 + 32 * k;
      if (u >= units) break;
      float4 wa[R], wb[R];
#pragma unroll
      for (int i = 0; i < R; ++i) {
        const float2 p0 = __half22float2(*reinterpret_cast<const __half2*>(&q[k][i].x));
        const float2 p1 = __half22float2(*reinterpret_cast<const __half2*>(&q[k][i].y));
        const float2 p2 = __half22float2(*reinterpret_cast<const __half2*>(&q[k][i].z));
        const float2 p3 = __half22float2(*reinterpret_cast<const __half2*>(&q[k][i].w));
        wa[i] = make_float4(p0.x, p0.y, p1.x, p1.y);
        wb[i] = make_float4(p2.x, p2.y, p3.x, p3.y);
      }
#pragma unroll
      for (int m = 0; m < kProjMaxM; ++m)
        if (m < mc) {
          const float4 xa = x4[m * n4 + 2 * u], xb = x4[m * n4 + 2 * u + 1];
#pragma unroll
          for (int i = 0; i < R; ++i) acc[i][m] = dot4(wb[i], xb, dot4(wa[i], xa, acc[i][m]));
        }
    }
  }
}

// Q8_0: a unit is half a 32-weight block
template <int R, int U>
__device__ __forceinline__ void rows_q8_0(const uint8_t* w0, size_t rb, const float* xs, int n,
                                          int mc, int lane, float (*acc)[kProjMaxM]) {
  const float4* x4 = reinterpret_cast<const float4*>(xs);
  const int units = n / 16, n4 = n / 4;
  for (int u0 = lane; u0 < units; u0 += 32 * U) {
    uint4 q[U][R];
    unsigned short dh[U][R];
#pragma unroll
    for (int k = 0; k < U; ++k)
#pragma unroll
      for (int i = 0; i < R; ++i) {
        const int u = u0 + 32 * k < units ? u0 + 32 * k : u0;
        q[k][i] = __ldg(reinterpret_cast<const uint4*>(w0 + i * rb) + u);
        dh[k][i] = __ldg(reinterpret_cast<const unsigned short*>(w0 + i * rb + n) + (u >> 1));
      }
#pragma unroll
    for (int k = 0; k < U; ++k) {
      const int u = u0 + 32 * k;
      if (u >= units) break;
      // int8 quants: flip the sign bit to get q + 128 as an unsigned byte
      float4 qa[R], qb[R], qc[R], qd[R];
      float d[R];
#pragma unroll
      for (int i = 0; i < R; ++i) {
        qa[i] = bytes_to_f4(q[k][i].x ^ 0x80808080u, 128.f);
        qb[i] = bytes_to_f4(q[k][i].y ^ 0x80808080u, 128.f);
        qc[i] = bytes_to_f4(q[k][i].z ^ 0x80808080u, 128.f);
        qd[i] = bytes_to_f4(q[k][i].w ^ 0x80808080u, 128.f);
        d[i] = __half2float(__ushort_as_half(dh[k][i]));
      }
#pragma unroll
      for (int m = 0; m < kProjMaxM; ++m)
        if (m < mc) {
          const float4* xm = x4 + m * n4 + 4 * u;
          const float4 x0 = xm[0], x1 = xm[1], x2 = xm[2], x3 = xm[3];
#pragma unroll
          for (int i = 0; i < R; ++i) {
            const float s = dot4(qd[i], x3, dot4(qc[i], x2, dot4(qb[i], x1, dot4(qa[i], x0, 0.f))));
            acc[i][m] = fmaf(d[i], s, acc[i][m]);
          }
        }
    }
  }
}

// Q4_K: a unit is 8 quant bytes of one 32-byte pair j of a block: their low
// nibbles weigh x of sub-block 2j, their high nibbles x of sub-block 2j+1
// (quant.c:96-128, 388-512).
template <int R, int U>
__device__ __forceinline__ void rows_q4k(const uint8_t* w0, size_t rb, const float* xs, int n,
                                         int mc, int lane, float (*acc)[kProjMaxM]) {
  const float4* x4 = reinterpret_cast<const float4*>(xs);
  const int units = n / 16, n4 = n / 4;
  for (int u0 = lane; u0 < units; u0 += 32 * U) {
    uint4 hdr[U][R];
    uint2 q[U][R];
#pragma unroll
    for (int k = 0; k < U; ++k)
#pragma unroll
      for (int i = 0; i < R; ++i) {
        const int u = u0 + 32 * k < units ? u0 + 32 * k : u0;
        const int b = u >> 4, t = u & 15;
        const uint8_t* blk = w0 + i * rb + static_cast<size_t>(b) * kQ4KBytes;
        hdr[k][i] = __ldg(reinterpret_cast<const uint4*>(blk));
        q[k][i] = __ldg(reinterpret_cast<const uint2*>(blk + 16 + (t >> 2) * 32 + (t & 3) * 8));
      }
#pragma unroll
    for (int k = 0; k < U; ++k) {
      const int u = u0 + 32 * k;
      if (u >= units) break;
      const int b = u >> 4, t = u & 15, j = t >> 2, part = t & 3;
      float4 l0[R], l1[R], h0[R], h1[R];
      float d1[R], m1[R], d2[R], m2[R];
#pragma unroll
      for (int i = 0; i < R; ++i) {
        const float d = f16_bits(hdr[k][i].x & 0xFFFFu), dmin = f16_bits(hdr[k][i].x >> 16);
        float sc, mn;
        scale_min_k4(2 * j, hdr[k][i].y, hdr[k][i].z, hdr[k][i].w, sc, mn);
        d1[i] = d * sc;
        m1[i] = dmin * mn;
        scale_min_k4(2 * j + 1, hdr[k][i].y, hdr[k][i].z, hdr[k][i].w, sc, mn);
        d2[i] = d * sc;
        m2[i] = dmin * mn;
        l0[i] = bytes_to_f4(q[k][i].x & 0x0F0F0F0Fu, 0.f);
        l1[i] = bytes_to_f4(q[k][i].y & 0x0F0F0F0Fu, 0.f);
        h0[i] = bytes_to_f4((q[k][i].x >> 4) & 0x0F0F0F0Fu, 0.f);
        h1[i] = bytes_to_f4((q[k][i].y >> 4) & 0x0F0F0F0Fu, 0.f);
      }
      const int xo = (b * 256 + j * 64 + part * 8) / 4;  // float4 index of the low-nibble x
#pragma unroll
      for (int m = 0; m < kProjMaxM; ++m)
        if (m < mc) {
          const float4* xm = x4 + m * n4 + xo;
          const float4 xa = xm[0], xb = xm[1], xc = xm[8], xd = xm[9];
          const float sx1 = sum4(xa) + sum4(xb), sx2 = sum4(xc) + sum4(xd);
#pragma unroll
          for (int i = 0; i < R; ++i) {
            const float sqx1 = dot4(l1[i], xb, dot4(l0[i], xa, 0.f));
            const float sqx2 = dot4(h1[i], xd, dot4(h0[i], xc, 0.f));
            acc[i][m] += d1[i] * sqx1 - m1[i] * sx1 + d2[i] * sqx2 - m2[i] * sx2;
          }
        }
    }
  }
}

// Q6_K: a unit is 4 consecutive l of one 128-weight half c of a block; each
// l carries four weights (l, l+32, l+64, l+96 of the half), in four scale
// groups of 16 (quant.c:193-222, 517-625).  Quant bytes q + 32 = low 4 bits
// from ql, high 2 from qh, assembled four at a time.
template <int R, int U>
__device__ __forceinline__ void rows_q6k(const uint8_t* w0, size_t rb, const float* xs, int n,
                                         int mc, int lane, float (*acc)[kProjMaxM]) {
  const float4* x4 = reinterpret_cast<const float4*>(xs);
  const int units = n / 16, n4 = n / 4;
  for (int u0 = lane; u0 < units; u0 += 32 * U) {
    uint32_t qla[U][R], qlb[U][R], qh[U][R], scw[U][R];
    unsigned short dh[U][R];
#pragma unroll
    for (int k = 0; k < U; ++k)
#pragma unroll
      for (int i = 0; i < R; ++i) {
        const int u = u0 + 32 * k < units ? u0 + 32 * k : u0;
        const int b = u >> 4, t = u & 15, c = t >> 3, lg = (t & 7) * 4;
        const uint8_t* blk = w0 + i * rb + static_cast<size_t>(b) * kQ6KBytes;
        qla[k][i] = __ldg(reinterpret_cast<const uint32_t*>(blk + c * 64 + lg));
        qlb[k][i] = __ldg(reinterpret_cast<const uint32_t*>(blk + c * 64 + 32 + lg));
        qh[k][i] = __ldg(reinterpret_cast<const uint32_t*>(blk + 128 + c * 32 + lg));
        // scales is, is+2, is+4, is+6 (is = 8c + lg/16): bytes of two words
        const uint32_t* sw = reinterpret_cast<const uint32_t*>(blk + 192 + c * 8);
        scw[k][i] = (lg < 16) ? __byte_perm(__ldg(sw), __ldg(sw + 1), 0x6420)
                              : __byte_perm(__ldg(sw), __ldg(sw + 1), 0x7531);
        dh[k][i] = __ldg(reinterpret_cast<const unsigned short*>(blk + 208));
      }
#pragma unroll
    for (int k = 0; k < U; ++k) {
      const int u = u0 + 32 * k;
      if (u >= units) break;
      const int b = u >> 4, t = u & 15, c = t >> 3, lg = (t & 7) * 4;
      float4 q1[R], q2[R], q3[R], q4[R];
      float s0[R], s1[R], s2[R], s3[R];
#pragma unroll
      for (int i = 0; i < R; ++i) {
        const uint32_t la = qla[k][i], lb = qlb[k][i], h = qh[k][i];
        q1[i] = bytes_to_f4((la & 0x0F0F0F0Fu) | ((h & 0x03030303u) << 4), 32.f);
        q2[i] = bytes_to_f4((lb & 0x0F0F0F0Fu) | (((h >> 2) & 0x03030303u) << 4), 32.f);
        q3[i] = bytes_to_f4(((la >> 4) & 0x0F0F0F0Fu) | (((h >> 4) & 0x03030303u) << 4), 32.f);
        q4[i] = bytes_to_f4(((lb >> 4) & 0x0F0F0F0Fu) | (((h >> 6) & 0x03030303u) << 4), 32.f);
        const float d = __half2float(__ushort_as_half(dh[k][i]));
        const uint32_t sc = scw[k][i];
        s0[i] = d * static_cast<float>(static_cast<int8_t>(sc & 0xFFu));
        s1[i] = d * static_cast<float>(static_cast<int8_t>((sc >> 8) & 0xFFu));
        s2[i] = d * static_cast<float>(static_cast<int8_t>((sc >> 16) & 0xFFu));
        s3[i] = d * static_cast<float>(static_cast<int8_t>(sc >> 24));
      }
      const int xo = (b * 256 + c * 128 + lg) / 4;
#pragma unroll
      for (int m = 0; m < kProjMaxM; ++m)
        if (m < mc) {
          const float4* xm = x4 + m * n4 + xo;
          const float4 xa = xm[0], xb = xm[8], xc = xm[16], xd = xm[24];
#pragma unroll
          for (int i = 0; i < R; ++i) {
            float s = s0[i] * dot4(q1[i], xa, 0.f);
            s = fmaf(s1[i], dot4(q2[i], xb, 0.f), s);
            s = fmaf(s2[i], dot4(q3[i], xc, 0.f), s);
            s = fmaf(s3[i], dot4(q4[i], xd, 0.f), s);
            acc[i][m] += s;
          }
        }
    }
  }
}

// grid = (ceil(total_rows / (kProjWarps * R)), ceil(M / mc)), block =
// kProjThreads, dynamic shared memory mc * n * 4 bytes.  The CTA stages its
// mc input rows (normalised when norm_w is set) in shared memory; warp w
// then computes output rows (blockIdx.x * kProjWarps + w) * R .. + R - 1,
// which lie in one matrix (every matrix's row count is a multiple of R).
template <int R>
__global__ void __launch_bounds__(kProjThreads) proj_kernel(const __grid_constant__ ProjArgs a) {
  extern __shared__ float4 proj_xs4[];
  float* xs = reinterpret_cast<float*>(proj_xs4);
  __shared__ float ss_part[kProjWarps][kProjMaxM];
  __shared__ float inv_rms[kProjMaxM];
  const int m0 = blockIdx.y * a.mc;
  const int mc = min(a.mc, a.M - m0);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n4 = a.n / 4;
  // stage the input rows with 16-byte loads from all threads; with norm_w
  // each thread also sums the squares of what it staged, per row
  float ss[kProjMaxM];
#pragma unroll
  for (int m = 0; m < kProjMaxM; ++m) ss[m] = 0.f;
#pragma unroll
  for (int m = 0; m < kProjMaxM; ++m) {
    if (m < mc) {
      const float4* xr = reinterpret_cast<const float4*>(a.x + static_cast<size_t>(m0 + m) * a.ldx);
      for (int i4 = threadIdx.x; i4 < n4; i4 += kProjThreads) {
        const float4 v = __ldg(xr + i4);
        proj_xs4[m * n4 + i4] = v;
        ss[m] = fmaf(v.w, v.w, fmaf(v.z, v.z, fmaf(v.y, v.y, fmaf(v.x, v.x, ss[m]))));
      }
    }
  }
  if (a.norm_w) {
    // picolm/tensor.c:425-490: 1 / sqrtf(sum(x^2) / n + eps)
#pragma unroll
    for (int m = 0; m < kProjMaxM; ++m) {
      float t = ss[m];
#pragma unroll
      for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
      if (lane == 0) ss_part[warp][m] = t;
    }
    __syncthreads();
    if (threadIdx.x < mc) {
      float t = 0.f;
#pragma unroll
      for (int w = 0; w < kProjWarps; ++w) t += ss_part[w][threadIdx.x];
      inv_rms[threadIdx.x] = 1.0f / sqrtf(t / static_cast<float>(a.n) + a.eps);
    }
    __syncthreads();
    // (x * ss) * w, two rounded products as the reference, in place
    for (int idx = threadIdx.x; idx < mc * n4; idx += kProjThreads) {
      const int m = idx / n4, i4 = idx - m * n4;
      const float s = inv_rms[m];
      const float4 w = __ldg(reinterpret_cast<const float4*>(a.norm_w) + i4);
      const float4 v = proj_xs4[idx];
      proj_xs4[idx] =
          make_float4(__fmul_rn(__fmul_rn(v.x, s), w.x), __fmul_rn(__fmul_rn(v.y, s), w.y),
                      __fmul_rn(__fmul_rn(v.z, s), w.z), __fmul_rn(__fmul_rn(v.w, s), w.w));
    }
  }
  __syncthreads();
  const int row = (blockIdx.x * kProjWarps + warp) * R;
  if (row >= a.total_rows) return;
  int mi = 0, r = row;
  while (mi + 1 < a.n_mat && r >= a.mat[mi].rows) {
    r -= a.mat[mi].rows;
    ++mi;
  }
  const ProjMat& mt = a.mat[mi];
  const uint8_t* wr = mt.w + static_cast<size_t>(r) * mt.row_bytes;
  constexpr int kU = R == 1 ? 2 : 1;  // one row per warp: two units' loads in flight
  float acc[R][kProjMaxM];
#pragma unroll
  for (int i = 0; i < R; ++i)
#pragma unroll
    for (int m = 0; m < kProjMaxM; ++m) acc[i][m] = 0.f;
  switch (mt.type) {
    case kGgufF32: rows_f32<R, kU>(wr, mt.row_bytes, xs, a.n, mc, lane, acc); break;
    case kGgufF16: rows_f16<R, kU>(wr, mt.row_bytes, xs, a.n, mc, lane, acc); break;
    case kGgufQ8_0: rows_q8_0<R, kU>(wr, mt.row_bytes, xs, a.n, mc, lane, acc); break;
    case kGgufQ4K: rows_q4k<R, kU>(wr, mt.row_bytes, xs, a.n, mc, lane, acc); break;
    default: rows_q6k<R, kU>(wr, mt.row_bytes, xs, a.n, mc, lane, acc); break;
  }
  // lane i * 8 + m ends up holding the total of (row i, input row m)
  float mine = 0.f;
#pragma unroll
  for (int i = 0; i < R; ++i)
#pragma unroll
    for (int m = 0; m < kProjMaxM; ++m) {
      if (m < mc) {
        float s = acc[i][m];
#pragma unroll
        for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == i * kProjMaxM + m) mine = s;
      }
    }
  const int i = lane / kProjMaxM, m = lane % kProjMaxM;
  if (i < R && m < mc) {
    // matmul_bias (tensor.c:230-238): out = W x, then out += b; the residual
    // add of model.c:897 is x += out
    float v = mine;
    if (mt.bias) v = v + __ldg(mt.bias + r + i);
    if (a.resid) v = a.resid[static_cast<size_t>(m0 + m) * a.ld_res + r + i] + v;
    mt.out[static_cast<size_t>(m0 + m) * mt.ld_out + r + i] = v;
  }
}

// ---------------------------------------------------------------------------
// The same projections on the tensor cores, for 16 or more input rows
// (batched decode, prefill) and Q4_K, Q8_0 or F16 weights.
//
// mma.sync m16n8k16 (FP16 in, FP32 accumulate) with the quants as the A
// operand and x as B.  Quants are small integers, exact in FP16; x is split
// into an FP16 high part and the FP16 rounding of its residual (two MMAs),
// which carries it to about 2^-22.  So an MMA over one scale group gives
// sum(q * x) of that group at FP32 accuracy, and the group's scale (and, for
// Q4_K, min * sum(x)) is applied to the FP32 fragment: the factored form of
// picolm's vec_dot, with the products summed by the tensor core.  Scales
// vary every 32 inputs, so they must be applied to partial sums per group;
// register fragments allow that, a TMEM accumulator would not without a
// round trip per group.
//
// CTA: kMmaWarps warps of 16 output rows each, kMmaN input rows (two n8
// tiles).  Per chunk of kMmaKC inputs the CTA stages the input rows
// (normalised when norm_w is set) as FP16 hi and lo, row pitch padded by 16
// bytes so that ldmatrix reads are conflict-free, plus sum(x) of every
// 32-input group.  A lane loads the 32-byte quant runs of its rows g and
// g + 8 straight from global memory (the four lanes of a row share them).
constexpr int kMmaWarps = 4;
constexpr int kMmaThreads = 32 * kMmaWarps;
constexpr int kMmaRows = 16 * kMmaWarps;   // output rows per CTA
constexpr int kMmaN = 16;                  // input rows per CTA
constexpr int kMmaKC = 256;                // inputs per staged chunk
constexpr int kMmaPitch = kMmaKC + 8;      // halves per staged row

__host__ __device__ inline bool proj_mma_type(int type) {
  return type == kGgufQ4K || type == kGgufQ8_0 || type == kGgufF16;
}

struct MmaStage {
  uint16_t hi[kMmaN][kMmaPitch];
  uint16_t lo[kMmaN][kMmaPitch];
  float xsum[kMmaN][kMmaKC / 32];
  float inv_rms[kMmaN];
  float ss_part[kMmaWarps][kMmaN];
};

// two FP16 quants (as 1024 + q, exact) -> subtract 1024 + bias
__device__ __forceinline__ uint32_t h2_sub(uint32_t p, float bias) {
  const __half2 r = __hsub2(*reinterpret_cast<const __half2*>(&p),
                            __float2half2_rn(1024.f + bias));
  return *reinterpret_cast<const uint32_t*>(&r);
}
// the low (hi_nib = 0) or high nibbles of the two bytes of v as an FP16 pair
__device__ __forceinline__ uint32_t nib_pair(uint32_t v, int hi_nib) {
  const uint32_t p = hi_nib ? (((v >> 4) & 0x000Fu) | ((v & 0xF000u) << 4))
                            : ((v & 0x000Fu) | ((v & 0x0F00u) << 8));
  return h2_sub(p | 0x64006400u, 0.f);
}
// the two int8 bytes of v as an FP16 pair
__device__ __forceinline__ uint32_t s8_pair(uint32_t v) {
  const uint32_t u = v ^ 0x8080u;
  return h2_sub(((u & 0x00FFu) | ((u & 0xFF00u) << 8)) | 0x64006400u, 128.f);
}
// 16-bit half `h` of word w of a 32-byte run held as two uint4
__device__ __forceinline__ uint32_t run_u16(const uint4 (&r)[2], int w, int h) {
  const uint4 v = r[w >> 2];
  const uint32_t x = (w & 3) == 0 ? v.x : (w & 3) == 1 ? v.y : (w & 3) == 2 ? v.z : v.w;
  return (x >> (16 * h)) & 0xFFFFu;
}

// A fragment of the k-step ks (16 inputs) of a 32-input run for rows g and
// g + 8: bytes 16ks + 2t, +1 (a0a1 / a2a3) and 16ks + 2t + 8, +9 (a4a5 / a6a7)
template <typename F>
__device__ __forceinline__ void a_frag(const uint4 (&rg)[2], const uint4 (&rg8)[2], int ks, int t,
                                       F conv, uint32_t (&a)[4]) {
  const int w0 = 4 * ks + (t >> 1), w1 = w0 + 2, h = t & 1;
  a[0] = conv(run_u16(rg, w0, h));
  a[1] = conv(run_u16(rg8, w0, h));
  a[2] = conv(run_u16(rg, w1, h));
  a[3] = conv(run_u16(rg8, w1, h));
}

// B fragments (hi and lo) of both n8 tiles for inputs kk .. kk+15 of the chunk
__device__ __forceinline__ void b_frags(const MmaStage& st, int kk, int lane, uint32_t (&bh)[4],
                                        uint32_t (&bl)[4]) {
  const int mi = lane >> 3, n = (mi >> 1) * 8 + (lane & 7), ko = (mi & 1) * 8;
  ldmatrix_x4(smem_u32(&st.hi[n][kk + ko]), bh[0], bh[1], bh[2], bh[3]);
  ldmatrix_x4(smem_u32(&st.lo[n][kk + ko]), bl[0], bl[1], bl[2], bl[3]);
}

__device__ __forceinline__ void mma_hilo(float (&c)[2][4], const uint32_t (&a)[4],
                                         const uint32_t (&bh)[4], const uint32_t (&bl)[4]) {
  mma_16816(c[0], a, bh[0], bh[1]);
  mma_16816(c[0], a, bl[0], bl[1]);
  mma_16816(c[1], a, bh[2], bh[3]);
  mma_16816(c[1], a, bl[2], bl[3]);
}

// acc += scale_row * c - min_row * sum(x) for both n8 tiles (rows g, g + 8;
// input rows 8nt + 2t, +1)
__device__ __forceinline__ void apply_group(float (&acc)[2][4], const float (&c)[2][4], float dg,
                                            float dg8, float mg, float mg8, const MmaStage& st,
                                            int grp, int t) {
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    const float s0 = st.xsum[8 * nt + 2 * t][grp], s1 = st.xsum[8 * nt + 2 * t + 1][grp];
    acc[nt][0] += dg * c[nt][0] - mg * s0;
    acc[nt][1] += dg * c[nt][1] - mg * s1;
    acc[nt][2] += dg8 * c[nt][2] - mg8 * s0;
    acc[nt][3] += dg8 * c[nt][3] - mg8 * s1;
  }
}

// one staged chunk (inputs k0 .. k0 + kMmaKC) of a warp's 16 rows
__device__ __forceinline__ void mma_chunk(int type, const uint8_t* wg, const uint8_t* wg8, int n,
                                          int k0, const MmaStage& st, int lane,
                                          float (&acc)[2][4]) {
  const int t = lane & 3;
  if (type == kGgufQ4K) {
    // one super-block: four runs of 32 quant bytes, each the low nibbles of
    // sub-block 2j and the high nibbles of sub-block 2j + 1
    const uint8_t* bg = wg + static_cast<size_t>(k0 / 256) * kQ4KBytes;
    const uint8_t* bg8 = wg8 + static_cast<size_t>(k0 / 256) * kQ4KBytes;
    const uint4 hg = __ldg(reinterpret_cast<const uint4*>(bg));
    const uint4 hg8 = __ldg(reinterpret_cast<const uint4*>(bg8));
    const float d_g = f16_bits(hg.x & 0xFFFFu), dm_g = f16_bits(hg.x >> 16);
    const float d_g8 = f16_bits(hg8.x & 0xFFFFu), dm_g8 = f16_bits(hg8.x >> 16);
    // all four runs of both rows in flight before any arithmetic
    uint4 qg[4][2], qg8[4][2];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      qg[j][0] = __ldg(reinterpret_cast<const uint4*>(bg + 16 + 32 * j));
      qg[j][1] = __ldg(reinterpret_cast<const uint4*>(bg + 32 + 32 * j));
      qg8[j][0] = __ldg(reinterpret_cast<const uint4*>(bg8 + 16 + 32 * j));
      qg8[j][1] = __ldg(reinterpret_cast<const uint4*>(bg8 + 32 + 32 * j));
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4(&rg)[2] = qg[j];
      const uint4(&rg8)[2] = qg8[j];
#pragma unroll
      for (int hn = 0; hn < 2; ++hn) {
        const int sb = 2 * j + hn;
        float sc, mn, sc8, mn8;
        scale_min_k4(sb, hg.y, hg.z, hg.w, sc, mn);
        scale_min_k4(sb, hg8.y, hg8.z, hg8.w, sc8, mn8);
        float c[2][4] = {};
#pragma unroll
        for (int ks = 0; ks < 2; ++ks) {
          uint32_t a[4], bh[4], bl[4];
          a_frag(rg, rg8, ks, t, [hn](uint32_t v) { return nib_pair(v, hn); }, a);
          b_frags(st, 32 * sb + 16 * ks, lane, bh, bl);
          mma_hilo(c, a, bh, bl);
        }
        apply_group(acc, c, d_g * sc, d_g8 * sc8, dm_g * mn, dm_g8 * mn8, st, sb, t);
      }
    }
  } else if (type == kGgufQ8_0) {
    // eight blocks of 32: quants at [k], the block's scale after all quants;
    // four blocks' loads in flight at a time
#pragma unroll 1
    for (int b4 = 0; b4 < kMmaKC / 32; b4 += 4) {
    uint4 qg[4][2], qg8[4][2];
    unsigned short sg[4], sg8[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int k = k0 + 32 * (b4 + i);
      qg[i][0] = __ldg(reinterpret_cast<const uint4*>(wg + k));
      qg[i][1] = __ldg(reinterpret_cast<const uint4*>(wg + k + 16));
      qg8[i][0] = __ldg(reinterpret_cast<const uint4*>(wg8 + k));
      qg8[i][1] = __ldg(reinterpret_cast<const uint4*>(wg8 + k + 16));
      sg[i] = __ldg(reinterpret_cast<const unsigned short*>(wg + n) + k / 32);
      sg8[i] = __ldg(reinterpret_cast<const unsigned short*>(wg8 + n) + k / 32);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int blk = b4 + i;
      const uint4(&rg)[2] = qg[i];
      const uint4(&rg8)[2] = qg8[i];
      const float d_g = __half2float(__ushort_as_half(sg[i]));
      const float d_g8 = __half2float(__ushort_as_half(sg8[i]));
      float c[2][4] = {};
#pragma unroll
      for (int ks = 0; ks < 2; ++ks) {
        uint32_t a[4], bh[4], bl[4];
        a_frag(rg, rg8, ks, t, [](uint32_t v) { return s8_pair(v); }, a);
        b_frags(st, 32 * blk + 16 * ks, lane, bh, bl);
        mma_hilo(c, a, bh, bl);
      }
      apply_group(acc, c, d_g, d_g8, 0.f, 0.f, st, blk, t);
    }
    }
  } else {
    // F16 weights are the A operand as they are; no groups
    const uint32_t* rg = reinterpret_cast<const uint32_t*>(wg) + k0 / 2;
    const uint32_t* rg8 = reinterpret_cast<const uint32_t*>(wg8) + k0 / 2;
    float c[2][4] = {};
#pragma unroll 4
    for (int ks = 0; ks < kMmaKC / 16; ++ks) {
      uint32_t a[4], bh[4], bl[4];
      a[0] = __ldg(rg + 8 * ks + t);
      a[1] = __ldg(rg8 + 8 * ks + t);
      a[2] = __ldg(rg + 8 * ks + t + 4);
      a[3] = __ldg(rg8 + 8 * ks + t + 4);
      b_frags(st, 16 * ks, lane, bh, bl);
      mma_hilo(c, a, bh, bl);
    }
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[nt][e] += c[nt][e];
  }
}

// grid = (ceil(total_rows / kMmaRows), ceil(M / kMmaN)), block = kMmaThreads.
// Every matrix's row count is a multiple of 16 and n a multiple of kMmaKC
// (the host checks).
__global__ void __launch_bounds__(kMmaThreads) proj_mma_kernel(const __grid_constant__ ProjArgs a) {
  __shared__ __align__(16) MmaStage st;
  const int m0 = blockIdx.y * kMmaN;
  const int mn = min(kMmaN, a.M - m0);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n4 = a.n / 4;
  // RMSNorm scale of each input row (tensor.c:425-490)
  if (a.norm_w) {
    float ss[kMmaN];
#pragma unroll
    for (int m = 0; m < kMmaN; ++m) {
      ss[m] = 0.f;
      if (m < mn) {
        const float4* xr =
            reinterpret_cast<const float4*>(a.x + static_cast<size_t>(m0 + m) * a.ldx);
        for (int i4 = threadIdx.x; i4 < n4; i4 += kMmaThreads) {
          const float4 v = __ldg(xr + i4);
          ss[m] = fmaf(v.w, v.w, fmaf(v.z, v.z, fmaf(v.y, v.y, fmaf(v.x, v.x, ss[m]))));
        }
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) ss[m] += __shfl_xor_sync(0xffffffffu, ss[m], o);
      if (lane == 0) st.ss_part[warp][m] = ss[m];
    }
    __syncthreads();
    if (threadIdx.x < kMmaN) {
      float t = 0.f;
#pragma unroll
      for (int w = 0; w < kMmaWarps; ++w) t += st.ss_part[w][threadIdx.x];
      st.inv_rms[threadIdx.x] = 1.0f / sqrtf(t / static_cast<float>(a.n) + a.eps);
    }
  }
  // this warp's 16 rows, all in one matrix
  const int row = (blockIdx.x * kMmaWarps + warp) * 16;
  const bool active = row < a.total_rows;
  int mi = 0, r = active ? row : 0;
  while (mi + 1 < a.n_mat && r >= a.mat[mi].rows) {
    r -= a.mat[mi].rows;
    ++mi;
  }
  const ProjMat& mt = a.mat[mi];
  const int g = lane >> 2, t = lane & 3;
  const uint8_t* wg = mt.w + static_cast<size_t>(r + g) * mt.row_bytes;
  const uint8_t* wg8 = mt.w + static_cast<size_t>(r + g + 8) * mt.row_bytes;
  float acc[2][4] = {};
  // this CTA's slice of the inputs (whole chunks)
  const int n_chunks = a.n / kMmaKC;
  const int c_lo = static_cast<int>(blockIdx.z) * n_chunks / a.ksplit;
  const int c_hi = (static_cast<int>(blockIdx.z) + 1) * n_chunks / a.ksplit;
  for (int k0 = c_lo * kMmaKC; k0 < c_hi * kMmaKC; k0 += kMmaKC) {
    __syncthreads();  // the previous chunk's reads are done (and inv_rms is ready)
    // stage inputs k0 .. k0 + kMmaKC of the input rows: FP16 hi / lo and
    // the sum of every 32-input group (8 lanes = 32 consecutive inputs)
    for (int idx = threadIdx.x; idx < kMmaN * (kMmaKC / 4); idx += kMmaThreads) {
      const int m = idx / (kMmaKC / 4), c4 = idx - m * (kMmaKC / 4);
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (m < mn) {
        v = __ldg(reinterpret_cast<const float4*>(a.x + static_cast<size_t>(m0 + m) * a.ldx + k0) + c4);
        if (a.norm_w) {
          const float s = st.inv_rms[m];
          const float4 w = __ldg(reinterpret_cast<const float4*>(a.norm_w + k0) + c4);
          v = make_float4(__fmul_rn(__fmul_rn(v.x, s), w.x), __fmul_rn(__fmul_rn(v.y, s), w.y),
                          __fmul_rn(__fmul_rn(v.z, s), w.z), __fmul_rn(__fmul_rn(v.w, s), w.w));
        }
      }
      const __half2 h0 = __floats2half2_rn(v.x, v.y), h1 = __floats2half2_rn(v.z, v.w);
      const float2 f0 = __half22float2(h0), f1 = __half22float2(h1);
      const __half2 l0 = __floats2half2_rn(v.x - f0.x, v.y - f0.y);
      const __half2 l1 = __floats2half2_rn(v.z - f1.x, v.w - f1.y);
      *reinterpret_cast<uint2*>(&st.hi[m][4 * c4]) =
          make_uint2(*reinterpret_cast<const uint32_t*>(&h0), *reinterpret_cast<const uint32_t*>(&h1));
      *reinterpret_cast<uint2*>(&st.lo[m][4 * c4]) =
          make_uint2(*reinterpret_cast<const uint32_t*>(&l0), *reinterpret_cast<const uint32_t*>(&l1));
      float gs = sum4(v);
      gs += __shfl_xor_sync(0xffffffffu, gs, 1);
      gs += __shfl_xor_sync(0xffffffffu, gs, 2);
      gs += __shfl_xor_sync(0xffffffffu, gs, 4);
      if ((c4 & 7) == 0) st.xsum[m][c4 >> 3] = gs;
    }
    __syncthreads();
    if (active) mma_chunk(mt.type, wg, wg8, a.n, k0, st, lane, acc);
  }
  if (!active) return;
  // epilogue: (row r + g (+8), input row 8nt + 2t (+1)); matmul_bias then
  // the residual add, as in proj_kernel, or the raw slice sums
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int rr = r + g + (e >= 2 ? 8 : 0);
      const int m = 8 * nt + 2 * t + (e & 1);
      if (m >= mn) continue;
      float v = acc[nt][e];
      if (a.ksplit > 1) {
        a.part[(static_cast<size_t>(blockIdx.z) * a.M + m0 + m) * a.total_rows + row + g +
               (e >= 2 ? 8 : 0)] = v;
        continue;
      }
      if (mt.bias) v = v + __ldg(mt.bias + rr);
      if (a.resid) v = a.resid[static_cast<size_t>(m0 + m) * a.ld_res + rr] + v;
      mt.out[static_cast<size_t>(m0 + m) * mt.ld_out + rr] = v;
    }
}

// Sum of the ksplit slices of proj_mma_kernel in slice order (the result
// does not depend on timing), then bias and residual.  One thread per
// (input row, launch row).
__global__ void __launch_bounds__(256) proj_reduce_kernel(const __grid_constant__ ProjArgs a) {
  const size_t idx = static_cast<size_t>(blockIdx.x) * 256 + threadIdx.x;
  if (idx >= static_cast<size_t>(a.M) * a.total_rows) return;
  const int m = static_cast<int>(idx / a.total_rows);
  const int row = static_cast<int>(idx - static_cast<size_t>(m) * a.total_rows);
  float v = 0.f;
  for (int z = 0; z < a.ksplit; ++z) v += a.part[(static_cast<size_t>(z) * a.M + m) * a.total_rows + row];
  int mi = 0, r = row;
  while (mi + 1 < a.n_mat && r >= a.mat[mi].rows) {
    r -= a.mat[mi].rows;
    ++mi;
  }
  const ProjMat& mt = a.mat[mi];
  if (mt.bias) v = v + __ldg(mt.bias + r);
  if (a.resid) v = a.resid[static_cast<size_t>(m) * a.ld_res + r] + v;
  mt.out[static_cast<size_t>(m) * mt.ld_out + r] = v;
}

// QK-norm (model.c:807-817): RMSNorm of every q head with qn and every k head
// with kn, in place, for n_rows rows.  grid = (n_rows, ceil((H + Hk) / 8)),
// block = 256, one warp per head.
__global__ void __launch_bounds__(256) qk_norm_kernel(float* q, float* k, int n_heads,
                                                       int n_kv_heads, int head_dim,
                                                       const float* qn, const float* kn,
                                                       float eps) {
  const int r = blockIdx.x;
  const int head = blockIdx.y * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (head >= n_heads + n_kv_heads) return;
  float* x;
  const float* w;
  if (head < n_heads) {
    x = q + (static_cast<size_t>(r) * n_heads + head) * head_dim;
    w = qn;
  } else {
    x = k + (static_cast<size_t>(r) * n_kv_heads + (head - n_heads)) * head_dim;
    w = kn;
  }
  float ss = 0.f;
  for (int i = lane; i < head_dim; i += 32) ss = fmaf(x[i], x[i], ss);
#pragma unroll
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float s = 1.0f / sqrtf(ss / static_cast<float>(head_dim) + eps);
  for (int i = lane; i < head_dim; i += 32) x[i] = __fmul_rn(__fmul_rn(x[i], s), w[i]);
}

}  // namespace pl
