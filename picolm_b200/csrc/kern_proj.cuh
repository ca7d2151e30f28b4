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

// Each lane takes work units u = lane, lane + 32, ... of the row (4 to 16
// weights each, consecutive lanes on consecutive bytes) and adds its partial
// dot with every staged input row m < mc into acc[m].

__device__ __forceinline__ void row_f32(const uint8_t* wr, const float* xs, int n, int mc,
                                        int lane, float* acc) {
  const float4* w4 = reinterpret_cast<const float4*>(wr);
  const float4* x4 = reinterpret_cast<const float4*>(xs);
  const int units = n / 4, n4 = n / 4;
  for (int u = lane; u < units; u += 32) {
    const float4 w = __ldg(w4 + u);
#pragma unroll
    for (int m = 0; m < kProjMaxM; ++m)
      if (m < mc) acc[m] = dot4(w, x4[m * n4 + u], acc[m]);
  }
}

__device__ __forceinline__ void row_f16(const uint8_t* wr, const float* xs, int n, int mc,
                                        int lane, float* acc) {
  const uint4* w8 = reinterpret_cast<const uint4*>(wr);
  const float4* x4 = reinterpret_cast<const float4*>(xs);
  const int units = n / 8, n4 = n / 4;
  for (int u = lane; u < units; u += 32) {
    const uint4 q = __ldg(w8 + u);
    const float4 wa = make_float4(f16_bits(q.x & 0xFFFFu), f16_bits(q.x >> 16),
                                  f16_bits(q.y & 0xFFFFu), f16_bits(q.y >> 16));
    const float4 wb = make_float4(f16_bits(q.z & 0xFFFFu), f16_bits(q.z >> 16),
                                  f16_bits(q.w & 0xFFFFu), f16_bits(q.w >> 16));
#pragma unroll
    for (int m = 0; m < kProjMaxM; ++m)
      if (m < mc) acc[m] = dot4(wb, x4[m * n4 + 2 * u + 1], dot4(wa, x4[m * n4 + 2 * u], acc[m]));
  }
}

__device__ __forceinline__ float4 s8x4(uint32_t w) {
  return make_float4(static_cast<float>(static_cast<int8_t>(w & 0xFFu)),
                     static_cast<float>(static_cast<int8_t>((w >> 8) & 0xFFu)),
                     static_cast<float>(static_cast<int8_t>((w >> 16) & 0xFFu)),
                     static_cast<float>(static_cast<int8_t>(w >> 24)));
}

// Q8_0: a unit is half a 32-weight block
__device__ __forceinline__ void row_q8_0(const uint8_t* wr, const float* xs, int n, int mc,
                                         int lane, float* acc) {
  const uint4* q16 = reinterpret_cast<const uint4*>(wr);
  const unsigned short* dv = reinterpret_cast<const unsigned short*>(wr + n);
  const float4* x4 = reinterpret_cast<const float4*>(xs);
  const int units = n / 16, n4 = n / 4;
  for (int u = lane; u < units; u += 32) {
    const uint4 q = __ldg(q16 + u);
    const float d = __half2float(__ushort_as_half(__ldg(dv + (u >> 1))));
    const float4 a = s8x4(q.x), b = s8x4(q.y), c = s8x4(q.z), e = s8x4(q.w);
#pragma unroll
    for (int m = 0; m < kProjMaxM; ++m)
      if (m < mc) {
        const float4* xm = x4 + m * n4 + 4 * u;
        const float s = dot4(e, xm[3], dot4(c, xm[2], dot4(b, xm[1], dot4(a, xm[0], 0.f))));
        acc[m] = fmaf(d, s, acc[m]);
      }
  }
}

__device__ __forceinline__ float4 nib4(uint32_t w, int shift) {
  return make_float4(static_cast<float>((w >> shift) & 0xFu),
                     static_cast<float>((w >> (shift + 8)) & 0xFu),
                     static_cast<float>((w >> (shift + 16)) & 0xFu),
                     static_cast<float>((w >> (shift + 24)) & 0xFu));
}

// Q4_K: a unit is 8 quant bytes of one 32-byte pair j of a block: their low
// nibbles weigh x of sub-block 2j, their high nibbles x of sub-block 2j+1
// (quant.c:96-128, 388-512).
__device__ __forceinline__ void row_q4k(const uint8_t* wr, const float* xs, int n, int mc,
                                        int lane, float* acc) {
  const float4* x4 = reinterpret_cast<const float4*>(xs);
  const int units = n / 16, n4 = n / 4;
  for (int u = lane; u < units; u += 32) {
    const int b = u >> 4, t = u & 15, j = t >> 2, part = t & 3;
    const uint8_t* blk = wr + static_cast<size_t>(b) * kQ4KBytes;
    const uint4 hdr = __ldg(reinterpret_cast<const uint4*>(blk));
    const uint2 q = __ldg(reinterpret_cast<const uint2*>(blk + 16 + j * 32 + part * 8));
    const float d = f16_bits(hdr.x & 0xFFFFu), dmin = f16_bits(hdr.x >> 16);
    float sc, mn;
    scale_min_k4(2 * j, hdr.y, hdr.z, hdr.w, sc, mn);
    const float d1 = d * sc, m1 = dmin * mn;
    scale_min_k4(2 * j + 1, hdr.y, hdr.z, hdr.w, sc, mn);
    const float d2 = d * sc, m2 = dmin * mn;
    const float4 l0 = nib4(q.x, 0), l1 = nib4(q.y, 0), h0 = nib4(q.x, 4), h1 = nib4(q.y, 4);
    const int xo = (b * 256 + j * 64 + part * 8) / 4;  // float4 index of the low-nibble x
#pragma unroll
    for (int m = 0; m < kProjMaxM; ++m)
      if (m < mc) {
        const float4* xm = x4 + m * n4 + xo;
        const float4 xa = xm[0], xb = xm[1], xc = xm[8], xd = xm[9];
        const float sqx1 = dot4(l1, xb, dot4(l0, xa, 0.f));
        const float sqx2 = dot4(h1, xd, dot4(h0, xc, 0.f));
        const float sx1 = sum4(xa) + sum4(xb), sx2 = sum4(xc) + sum4(xd);
        acc[m] += d1 * sqx1 - m1 * sx1 + d2 * sqx2 - m2 * sx2;
      }
  }
}

__device__ __forceinline__ float4 q6x4(uint32_t ql, uint32_t qh, int lshift, int hshift) {
  float v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int q = static_cast<int>(((ql >> (8 * i + lshift)) & 0xFu) |
                                   (((qh >> (8 * i + hshift)) & 3u) << 4)) - 32;
    v[i] = static_cast<float>(q);
  }
  return make_float4(v[0], v[1], v[2], v[3]);
}

// Q6_K: a unit is 4 consecutive l of one 128-weight half c of a block; each
// l carries four weights (l, l+32, l+64, l+96 of the half), in four scale
// groups of 16 (quant.c:193-222, 517-625).
__device__ __forceinline__ void row_q6k(const uint8_t* wr, const float* xs, int n, int mc,
                                        int lane, float* acc) {
  const float4* x4 = reinterpret_cast<const float4*>(xs);
  const int units = n / 16, n4 = n / 4;
  for (int u = lane; u < units; u += 32) {
    const int b = u >> 4, t = u & 15, c = t >> 3, lg = (t & 7) * 4;
    const uint8_t* blk = wr + static_cast<size_t>(b) * kQ6KBytes;
    const uint32_t qla = __ldg(reinterpret_cast<const uint32_t*>(blk + c * 64 + lg));
    const uint32_t qlb = __ldg(reinterpret_cast<const uint32_t*>(blk + c * 64 + 32 + lg));
    const uint32_t qh = __ldg(reinterpret_cast<const uint32_t*>(blk + 128 + c * 32 + lg));
    const int is = c * 8 + lg / 16;
    const int8_t* scl = reinterpret_cast<const int8_t*>(blk + 192);
    const float d = __half2float(__ushort_as_half(__ldg(reinterpret_cast<const unsigned short*>(blk + 208))));
    const float s0 = d * static_cast<float>(__ldg(scl + is)),
                s1 = d * static_cast<float>(__ldg(scl + is + 2)),
                s2 = d * static_cast<float>(__ldg(scl + is + 4)),
                s3 = d * static_cast<float>(__ldg(scl + is + 6));
    const float4 q1 = q6x4(qla, qh, 0, 0), q2 = q6x4(qlb, qh, 0, 2), q3 = q6x4(qla, qh, 4, 4),
                 q4 = q6x4(qlb, qh, 4, 6);
    const int xo = (b * 256 + c * 128 + lg) / 4;
#pragma unroll
    for (int m = 0; m < kProjMaxM; ++m)
      if (m < mc) {
        const float4* xm = x4 + m * n4 + xo;
        float s = s0 * dot4(q1, xm[0], 0.f);
        s = fmaf(s1, dot4(q2, xm[8], 0.f), s);
        s = fmaf(s2, dot4(q3, xm[16], 0.f), s);
        s = fmaf(s3, dot4(q4, xm[24], 0.f), s);
        acc[m] += s;
      }
  }
}

// grid = (ceil(total_rows / kProjWarps), ceil(M / mc)), block = kProjThreads,
// dynamic shared memory mc * n * 4 bytes.  The CTA stages its mc input rows
// (normalised when norm_w is set) in shared memory; warp w then computes
// output row blockIdx.x * kProjWarps + w for all of them.
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
  const int row = blockIdx.x * kProjWarps + warp;
  if (row >= a.total_rows) return;
  int mi = 0, r = row;
  while (mi + 1 < a.n_mat && r >= a.mat[mi].rows) {
    r -= a.mat[mi].rows;
    ++mi;
  }
  const ProjMat& mt = a.mat[mi];
  const uint8_t* wr = mt.w + static_cast<size_t>(r) * mt.row_bytes;
  float acc[kProjMaxM];
#pragma unroll
  for (int m = 0; m < kProjMaxM; ++m) acc[m] = 0.f;
  switch (mt.type) {
    case kGgufF32: row_f32(wr, xs, a.n, mc, lane, acc); break;
    case kGgufF16: row_f16(wr, xs, a.n, mc, lane, acc); break;
    case kGgufQ8_0: row_q8_0(wr, xs, a.n, mc, lane, acc); break;
    case kGgufQ4K: row_q4k(wr, xs, a.n, mc, lane, acc); break;
    default: row_q6k(wr, xs, a.n, mc, lane, acc); break;
  }
  float mine = 0.f;
#pragma unroll
  for (int m = 0; m < kProjMaxM; ++m) {
    if (m < mc) {
      float s = acc[m];
#pragma unroll
      for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (lane == m) mine = s;
    }
  }
  if (lane < mc) {
    // matmul_bias (tensor.c:230-238): out = W x, then out += b; the residual
    // add of model.c:897 is x += out
    float v = mine;
    if (mt.bias) v = v + __ldg(mt.bias + r);
    if (a.resid) v = a.resid[static_cast<size_t>(m0 + lane) * a.ld_res + r] + v;
    mt.out[static_cast<size_t>(m0 + lane) * mt.ld_out + r] = v;
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
