// kern_misc.cuh -- small element-wise kernels around the attention path:
// in-place RoPE (bit-exact picolm rotation) and the prefill prologue that
// rotates q/k, appends k/v to the FP16 cache and stages q as FP16 for the
// tensor-core prefill.
#pragma once
#include <cstdint>

#include "kern_decode.cuh"
#include "pl_fp16.cuh"

namespace pl {

// RoPE in place on n_tok rows of q [n_tok][n_heads*64] and k
// [n_tok][n_kv_heads*64]; row r uses the table row pos0 + r.
// grid = (n_tok, ceil((n_heads + n_kv_heads) / 8)), block = 256: warp w of
// block (r, y) handles head 8y + w of row r, lane l its element pair 2l.
__global__ void rope_inplace_kernel(float* q, float* k, int n_heads, int n_kv_heads, int pos0,
                                    const float* cos_tab, const float* sin_tab, int rope_type) {
  const int r = blockIdx.x;
  const int head = blockIdx.y * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (head >= n_heads + n_kv_heads) return;
  const int pos = pos0 + r;
  const float* cs = cos_tab + static_cast<size_t>(pos) * (kHD / 2);
  const float* sn = sin_tab + static_cast<size_t>(pos) * (kHD / 2);
  float* x;
  if (head < n_heads) {
    if (!q) return;
    x = q + (static_cast<size_t>(r) * n_heads + head) * kHD;
  } else {
    if (!k) return;
    x = k + (static_cast<size_t>(r) * n_kv_heads + (head - n_heads)) * kHD;
  }
  // all reads of the head happen before any write (Qwen pairs cross lanes)
  const float2 y = rope_two(x, 2 * lane, cs, sn, rope_type);
  __syncwarp();
  *reinterpret_cast<float2*>(x + 2 * lane) = y;
}

// Prefill prologue for n_tok rows starting at position start_pos:
//   q16[r][h][d]  = FP16(RoPE(q[r][h][:]))[d]       (tensor-core operand,
//                                                     round-to-nearest-even)
//   kc[start+r]   = picolm_FP16(RoPE(k[r]))          (bit-exact append)
//   vc[start+r]   = picolm_FP16(v[r])
// grid = ceil(n_tok / kPrologueRows), block = 256: each warp takes (row,
// head) tasks of its block in turn, lane l the element pair 2l.
constexpr int kPrologueRows = 4;

__global__ void __launch_bounds__(256)
    prefill_prologue_kernel(const float* __restrict__ q, const float* __restrict__ k,
                            const float* __restrict__ v, uint16_t* __restrict__ q16,
                            uint16_t* __restrict__ kc_rows, uint16_t* __restrict__ vc_rows,
                            int n_tok, int n_heads, int n_kv_heads, int start_pos,
                            const float* cos_tab, const float* sin_tab, int rope_type) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int heads = n_heads + n_kv_heads;
  const int kv_dim = n_kv_heads * kHD;
  const int r0 = blockIdx.x * kPrologueRows;
  for (int task = warp; task < kPrologueRows * heads; task += 8) {
    const int r = r0 + task / heads, head = task % heads;
    if (r >= n_tok) break;
    const int pos = start_pos + r;
    const float* cs = cos_tab + static_cast<size_t>(pos) * (kHD / 2);
    const float* sn = sin_tab + static_cast<size_t>(pos) * (kHD / 2);
    if (head < n_heads) {
      const float* x = q + (static_cast<size_t>(r) * n_heads + head) * kHD;
      const float2 y = rope_two(x, 2 * lane, cs, sn, rope_type);
      reinterpret_cast<uint32_t*>(q16 + (static_cast<size_t>(r) * n_heads + head) * kHD)[lane] =
          pack_half2(y.x, y.y);
    } else {
      const int hk = head - n_heads;
      const float* x = k + static_cast<size_t>(r) * kv_dim + hk * kHD;
      const float2 y = rope_two(x, 2 * lane, cs, sn, rope_type);
      const float2 vv = *reinterpret_cast<const float2*>(v + static_cast<size_t>(r) * kv_dim +
                                                         hk * kHD + 2 * lane);
      const size_t off = static_cast<size_t>(r) * kv_dim + hk * kHD;
      reinterpret_cast<uint32_t*>(kc_rows + off)[lane] =
          static_cast<uint32_t>(picolm_f32_to_f16(y.x)) |
          (static_cast<uint32_t>(picolm_f32_to_f16(y.y)) << 16);
      reinterpret_cast<uint32_t*>(vc_rows + off)[lane] =
          static_cast<uint32_t>(picolm_f32_to_f16(vv.x)) |
          (static_cast<uint32_t>(picolm_f32_to_f16(vv.y)) << 16);
    }
  }
}

}  // namespace pl
