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
