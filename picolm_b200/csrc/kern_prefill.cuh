// kern_prefill.cuh -- causal prefill attention on the 5th-generation tensor
// cores (tcgen05 + tensor memory), fed by TMA.
//
// Replaces the position-by-position loop of picolm/model.c:1054-1089.  The
// prologue kernel (kern_misc.cuh) has already rotated q/k, appended k/v to
// the FP16 cache (bit-exact) and staged q as FP16 [n_tok][n_heads][64].
//
// One CTA = one (query head, 128-row query tile).  Warp roles:
//   warps 0-3  softmax + epilogue; thread r owns query row r = TMEM lane r
//   warp 4     TMA producer: the Q tile once, then K/V tiles of 128 cache
//              rows through an NS-deep ring (128-byte swizzle)
//   warp 5     TMEM allocator and the single MMA-issuing thread
// Per KV tile j:
//   S_j = Q K_j^T    tcgen05.mma M=128 N=128 K=64 -> TMEM S[j%2] (FP32)
//   softmax warps: tcgen05.ld S row, causal mask, online max (log2 domain),
//                  P = 2^(s - m) as FP16 into shared memory (SW128 K-major)
//   PV_j = P_j V_j   tcgen05.mma M=128 N=64 K=128 -> TMEM O[j%2] (fresh)
//   softmax warps: tcgen05.ld PV_j, O = O * alpha + PV_j in registers
// S and O are double-buffered in TMEM so the tensor core computes S_{j+1}
// and PV_j while the softmax warps work on tile j.  Every wait is bounded;
// a wait that gives up records an error bit and the CTA winds down (waits
// for its own MMAs and TMA copies, frees its TMEM) instead of hanging.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "sm100.cuh"

namespace pl {

constexpr int kPfBlockM = 128;  // query rows per CTA
constexpr int kPfBlockN = 128;  // cache rows per KV tile
constexpr int kPfStages = 2;    // K/V ring depth
constexpr int kPfThreads = 192;

struct PrefillArgs {
  const uint16_t* q16;   // [n_tok][n_heads][64] FP16, rotated
  float* out;            // row r at out + r*out_stride, head h at +h*64
  int out_stride;
  int n_tok, start_pos, n_heads, kv_mul, slab;
  float score_scale;     // log2(e)/sqrt(64)
  uint32_t* err;
};

struct PfSmem {
  // 1024-byte aligned tiles (128-byte swizzle atoms are 8 rows x 128 B)
  uint8_t q[kPfBlockM * 128];                 // 16 KB
  uint8_t k[kPfStages][kPfBlockN * 128];      // 16 KB each
  uint8_t v[kPfStages][kPfBlockN * 128];      // 16 KB each
  uint8_t p[2][2][kPfBlockM * 128];           // [buf][k-chunk of 64] 16 KB each
  uint64_t q_full;
  uint64_t kv_full[kPfStages], kv_empty[kPfStages];
  uint64_t s_full[2], s_free[2], p_full[2], o_full[2], o_free[2];
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort_flag;
};

constexpr int kPfSmemBytes = static_cast<int>(sizeof(PfSmem)) + 1024;

// TMEM column map (512 columns allocated)
constexpr uint32_t kColS0 = 0, kColS1 = 128, kColO0 = 256, kColO1 = 320;

__device__ __forceinline__ uint32_t pf_col_s(int b) { return b ? kColS1 : kColS0; }
__device__ __forceinline__ uint32_t pf_col_o(int b) { return b ? kColO1 : kColO0; }

__global__ void __launch_bounds__(kPfThreads, 1)
    prefill_attn_kernel(const PrefillArgs a, const __grid_constant__ CUtensorMap tm_q,
                        const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v) {
  extern __shared__ uint8_t smem_raw[];
  PfSmem& sm = *reinterpret_cast<PfSmem*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // heaviest (latest) query tiles first: b -> (tile, head)
  const int n_qt = (a.n_tok + kPfBlockM - 1) / kPfBlockM;
  const int b = blockIdx.x;
  const int qt = n_qt - 1 - b / a.n_heads;
  const int h = b % a.n_heads;
  const int kvh = h / a.kv_mul;
  const int q_row0 = qt * kPfBlockM;
  const int last_row = min(a.n_tok, q_row0 + kPfBlockM) - 1;
  const int kv_rows = a.start_pos + last_row + 1;         // cache rows this tile needs
  const int nkv = (kv_rows + kPfBlockN - 1) / kPfBlockN;   // >= 1
  const int p_min = a.start_pos + q_row0;                   // smallest query position

  if (threadIdx.x == 0) {
    mbar_init(&sm.q_full, 1);
    for (int s = 0; s < kPfStages; ++s) {
      mbar_init(&sm.kv_full[s], 1);
      mbar_init(&sm.kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.s_full[i], 1);
      mbar_init(&sm.s_free[i], 4);
      mbar_init(&sm.p_full[i], 4);
      mbar_init(&sm.o_full[i], 1);
      mbar_init(&sm.o_free[i], 4);
    }
    mbar_init(&sm.mma_done, 1);
    sm.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 5) {
    tmem_alloc(&sm.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == 4) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      mbar_arrive_expect_tx(&sm.q_full, kPfBlockM * 128);
      tma_load_3d(sm.q, &tm_q, &sm.q_full, 0, h, q_row0);
      int issued = 0;
      for (int j = 0; j < nkv; ++j) {
        const int s = j % kPfStages;
        if (j >= kPfStages &&
            !mbar_wait_bounded(&sm.kv_empty[s], ((j / kPfStages) - 1) & 1)) {
          atomicOr(a.err, ERR_TIMEOUT_EMPTY);
          sm.abort_flag = 1;
          break;
        }
        if (*reinterpret_cast<volatile int*>(&sm.abort_flag)) break;
        mbar_arrive_expect_tx(&sm.kv_full[s], 2 * kPfBlockN * 128);
        tma_load_4d(sm.k[s], &tm_k, &sm.kv_full[s], 0, j * kPfBlockN, kvh, a.slab);
        tma_load_4d(sm.v[s], &tm_v, &sm.kv_full[s], 0, j * kPfBlockN, kvh, a.slab);
        ++issued;
      }
      // never leave with copies in flight: the last use of each stage must land
      for (int j = issued - kPfStages; j < issued; ++j)
        if (j >= 0) mbar_wait_bounded(&sm.kv_full[j % kPfStages], (j / kPfStages) & 1);
      mbar_wait_bounded(&sm.q_full, 0);
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc_qk = idesc_f16_f32(128, 128, 0);
      const uint32_t idesc_pv = idesc_f16_f32(128, 64, 1);
      const uint32_t q_addr = smem_u32(sm.q);
      bool ok = mbar_wait_bounded(&sm.q_full, 0);
      auto issue_pv = [&](int i) -> bool {
        const int pb = i & 1, s = i % kPfStages;
        if (!mbar_wait_bounded(&sm.p_full[pb], (i >> 1) & 1)) return false;
        if (i >= 2 && !mbar_wait_bounded(&sm.o_free[pb], ((i >> 1) - 1) & 1)) return false;
        tc_fence_after();
        const uint32_t p_addr = smem_u32(sm.p[pb][0]);
        const uint32_t v_addr = smem_u32(sm.v[s]);
#pragma unroll
        for (int kk = 0; kk < kPfBlockN / 16; ++kk) {
          const uint64_t ad = smem_desc_sw128(p_addr + (kk >> 2) * (kPfBlockM * 128) + (kk & 3) * 32,
                                              16, 1024);
          const uint64_t bd = smem_desc_sw128(v_addr + kk * 16 * 128, 16, 1024);
          tc_mma_ss(tmem + pf_col_o(pb), ad, bd, idesc_pv, kk > 0 ? 1u : 0u);
        }
        tc_commit(&sm.o_full[pb]);
        tc_commit(&sm.kv_empty[s]);
        return true;
      };
      for (int j = 0; ok && j < nkv; ++j) {
        const int s = j % kPfStages, sb = j & 1;
        if (!mbar_wait_bounded(&sm.kv_full[s], (j / kPfStages) & 1)) { ok = false; break; }
        if (j >= 2 && !mbar_wait_bounded(&sm.s_free[sb], ((j >> 1) - 1) & 1)) { ok = false; break; }
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sm.k[s]);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint64_t ad = smem_desc_sw128(q_addr + kk * 32, 16, 1024);
          const uint64_t bd = smem_desc_sw128(k_addr + kk * 32, 16, 1024);
          tc_mma_ss(tmem + pf_col_s(sb), ad, bd, idesc_qk, kk > 0 ? 1u : 0u);
        }
        tc_commit(&sm.s_full[sb]);
        if (j >= 1 && !issue_pv(j - 1)) { ok = false; break; }
      }
      if (ok) ok = issue_pv(nkv - 1);
      if (!ok) {
        atomicOr(a.err, ERR_TIMEOUT_MMA);
        sm.abort_flag = 1;
      }
      // all issued MMAs must finish before TMEM is freed
      tc_commit(&sm.mma_done);
      mbar_wait_bounded(&sm.mma_done, 0);
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int r = threadIdx.x;                 // query row in the tile, TMEM lane
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    const int p_row = a.start_pos + q_row0 + r;  // this row's position
    float m_run = -INFINITY, l_run = 0.f, alpha_prev = 0.f;
    float o[64];
#pragma unroll
    for (int d = 0; d < 64; ++d) o[d] = 0.f;
    bool ok = true;

    auto consume_pv = [&](int i, float alpha) -> bool {
      const int ob = i & 1;
      if (!mbar_wait_bounded(&sm.o_full[ob], (i >> 1) & 1)) return false;
      tc_fence_after();
      uint32_t x[32];
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        tc_ld_32x32b_x32(lane_base + pf_col_o(ob) + 32 * half, x);
        tc_wait_ld();
#pragma unroll
        for (int d = 0; d < 32; ++d) o[32 * half + d] = fmaf(o[32 * half + d], alpha, __uint_as_float(x[d]));
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.o_free[ob]);
      return true;
    };

    for (int j = 0; j < nkv; ++j) {
      const int sb = j & 1;
      if (!mbar_wait_bounded(&sm.s_full[sb], (j >> 1) & 1)) { ok = false; break; }
      tc_fence_after();
      uint32_t sv[128];
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4) {
        tc_ld_32x32b_x32(lane_base + pf_col_s(sb) + 32 * c4,
                         *reinterpret_cast<uint32_t(*)[32]>(&sv[32 * c4]));
      }
      tc_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.s_free[sb]);

      // scale, causal mask, tile max
      const int t0 = j * kPfBlockN;
      const bool need_mask = t0 + kPfBlockN - 1 > p_min;
      float mt = -INFINITY;
#pragma unroll
      for (int cidx = 0; cidx < 128; ++cidx) {
        float s = __uint_as_float(sv[cidx]) * a.score_scale;
        if (need_mask && t0 + cidx > p_row) s = -INFINITY;
        sv[cidx] = __float_as_uint(s);
        mt = fmaxf(mt, s);
      }
      const float m_new = fmaxf(m_run, mt);
      const float alpha = ex2(m_run - m_new);
      // P = 2^(s - m_new) -> FP16 into the SW128 K-major P buffer
      float rs = 0.f;
      uint8_t* pbuf = sm.p[sb][0];
#pragma unroll
      for (int ch = 0; ch < 16; ++ch) {       // 16 chunks of 8 columns
        uint32_t w4[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float p0 = ex2(__uint_as_float(sv[8 * ch + 2 * e]) - m_new);
          const float p1 = ex2(__uint_as_float(sv[8 * ch + 2 * e + 1]) - m_new);
          rs += p0 + p1;
          w4[e] = pack_half2(p0, p1);
        }
        const int kc = ch >> 3, c16 = ch & 7;
        uint8_t* dst = pbuf + kc * (kPfBlockM * 128) + r * 128 + ((c16 ^ (r & 7)) << 4);
        *reinterpret_cast<uint4*>(dst) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
      }
      l_run = l_run * alpha + rs;
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.p_full[sb]);
      if (j >= 1 && !consume_pv(j - 1, alpha_prev)) { ok = false; break; }
      alpha_prev = alpha;
      m_run = m_new;
    }
    if (ok) ok = consume_pv(nkv - 1, alpha_prev);
    if (!ok) {
      atomicOr(a.err, ERR_TIMEOUT_MMA);
      sm.abort_flag = 1;
    } else {
      const int row = q_row0 + r;
      if (row < a.n_tok) {
        const float inv = 1.0f / l_run;
        float* dst = a.out + static_cast<size_t>(row) * a.out_stride + h * 64;
#pragma unroll
        for (int d = 0; d < 64; d += 4)
          *reinterpret_cast<float4*>(dst + d) =
              make_float4(o[d] * inv, o[d + 1] * inv, o[d + 2] * inv, o[d + 3] * inv);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Host side: encode the Q map (over the FP16 q staging buffer) and launch.
inline int launch_prefill_attention(const PrefillArgs& a, const CUtensorMap& tm_q,
                                    const CUtensorMap& tm_k, const CUtensorMap& tm_v,
                                    cudaStream_t st) {
  static bool attr_done = false;
  if (!attr_done) {
    if (cudaFuncSetAttribute(prefill_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kPfSmemBytes) != cudaSuccess)
      return -4;
    attr_done = true;
  }
  const int n_qt = (a.n_tok + kPfBlockM - 1) / kPfBlockM;
  prefill_attn_kernel<<<n_qt * a.n_heads, kPfThreads, kPfSmemBytes, st>>>(a, tm_q, tm_k, tm_v);
  return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

}  // namespace pl
