// kern_prefill.cuh -- causal prefill attention on the 5th-generation tensor
// cores (tcgen05 + tensor memory), fed by TMA.
//
// Replaces the position-by-position loop of picolm/model.c:1054-1089.  The
// prologue kernel (kern_misc.cuh) has already rotated q/k, appended k/v to
// the FP16 cache (bit-exact) and staged q as two FP16 arrays
// [n_tok][n_heads][HD]: the high part and the residual.  S = Q_hi K^T +
// Q_lo K^T (two MMAs into the same accumulator) carries q to about 2^-22,
// as the FP32 reference does; with q rounded to FP16 alone, near-tied
// scores of large q and k moved outputs by up to 2.7e-3 on projected
// inputs.  The second MMA costs tensor-pipe time, which the softmax-bound
// loop has to spare.
//
// Work item = two 128-row query tiles ("slots" A and B) sharing one KV
// head: two query heads of the same GQA group at the same rows (with one
// query head per KV head, slot B is unused).  Both slots see the same K/V
// tiles and the same causal range.  The kernel is persistent: one CTA per
// SM takes items from a global counter, heaviest (latest) query tiles
// first, and every pipeline below runs on across item boundaries (the next
// item's Q and first K/V tiles load while the current one finishes).
//
// Warp roles (384 threads = three warpgroups):
//   warps 0-3  softmax of slot A; thread r owns query row r = TMEM lane r
//   warps 4-7  softmax of slot B (same lanes, other TMEM columns)
//   warp 8     scheduler + TMA producer: fetches items, publishes them in a
//              two-entry shared-memory queue, loads Q_A/Q_B per item and
//              K/V tiles of BN cache rows through a STAGES-deep ring
//   warp 9     TMEM allocator; MMA issuer of slot A
//   warp 10    MMA issuer of slot B
//   warp 11    idle (completes the third warpgroup for the register split)
// The block launches at kPfLaunchRegs registers per thread; the two softmax
// warpgroups then raise theirs to kPfSoftmaxRegs (a BN-column S row lives
// in registers) and the third drops to kPfOtherRegs:
// 256 * 232 + 128 * 40 = 384 * 168.
// Per KV tile j the issuer of slot x issues, in order,
//   S_x(j) = Q_x K_j^T      (M=128 N=BN K=HD, twice: hi and lo parts of Q;
//                            smem x smem -> TMEM)
//   PV_x(j-1) = P_x V       (M=128 N=64 K=BN per 64 columns of O, TMEM x smem
//                            -> TMEM O_x)
// so one slot's softmax overlaps the other slot's MMAs (ping-pong).  Issue
// of tcgen05.mma is close to synchronous with its execution, and every
// mbarrier check in the issuing thread leaves the tensor pipe idle for
// about a hundred cycles; with one issuer per slot, the other slot's MMAs
// fill those gaps.  The slots touch disjoint TMEM columns, so the two
// issuers need no ordering between them; a K/V stage is released when both
// have committed their MMAs on it.  A
// softmax thread loads its BN-column S row from TMEM once, takes the row
// max (causal mask on diagonal tiles only), and writes P = 2^(s*c - m) as
// FP16 back into tensor memory (its own lane, two halves per 32-bit
// column), where the PV MMA takes it as the A operand: P never touches
// shared memory, whose bandwidth the S MMAs and the TMA ring need.  Five
// eighths of the 2^x go to the MUFU unit, three eighths to a cubic
// polynomial on the FMA pipe (see exp2_poly2); of the shares measured (1/8,
// 1/4, 3/8, 1/2 on the FMA pipe) this one is fastest.  O accumulates in TMEM; the
// running max used for P is raised only when a row's max grows by more than
// 2^8 (then the warp rescales its O rows in TMEM), so P <= 2^8 is exact in
// FP16 and the final O / l is unchanged.
//
// Every wait is bounded; a wait that gives up records an error bit and the
// CTA winds down (waits for its own MMAs and TMA copies, frees its TMEM)
// instead of hanging.
#pragma once
#include <atomic>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "sm100.cuh"

namespace pl {

constexpr int kPfBlockM = 128;  // query rows per slot
constexpr int kPfThreads = 384;
constexpr int kPfLaunchRegs = 168;   // 65536 / 384 rounded down to 8
constexpr int kPfSoftmaxRegs = 232;
constexpr int kPfOtherRegs = 40;
static_assert(256 * kPfSoftmaxRegs + 128 * kPfOtherRegs <= kPfThreads * kPfLaunchRegs,
              "register split exceeds the launch allocation");
constexpr int kPfStagePitch = 32;    // floats per row of the output staging buffer
constexpr float kPfRescaleLog2 = 8.0f;  // raise the running max only past 2^8

struct PrefillArgs {
  const uint16_t* q16;   // [n_tok][n_heads][HD] FP16, rotated (high part; TMA reads it)
  float* out;            // row r at out + r*out_stride, head h at +h*HD
  int out_stride;
  int n_tok, start_pos, n_heads, kv_mul, slab;
  float score_scale;     // log2(e)/sqrt(HD)
  int* work;             // [2] item counter, finished-CTA counter; zero at rest
  uint32_t* err;
  int o_tma;             // 1: the output leaves through tm_o (TMA stores, HD 64)
};

// The two shapes of the kernel: head_dim HD, KV tiles of BN cache rows,
// a STAGES-deep K/V ring.  <64, 128, 4>: S 128 + O 64 + P 64 TMEM columns per
// slot.  <128, 64, 3>: S 64 + O 128 + P 32 (448 of 512 columns).  Both use
// 225 KB of shared memory, most of it Q (hi and lo) and the K/V ring; at
// HD 128 the output is stored without the staging buffer.  A row of Q, K or V is HD/64 halves of 64 elements
// (128 bytes, the swizzle span); each half of a tile is its own 128-byte
// swizzled region, loaded by its own TMA box (x = 0 or 64).
template <int HD, int BN, int STAGES>
struct PfShape {
  static constexpr int kHalves = HD / 64;
  static constexpr int kQHalf = kPfBlockM * 128;       // bytes of one half of a Q tile
  static constexpr int kQBytes = kQHalf * kHalves;
  static constexpr int kKVHalf = BN * 128;             // bytes of one half of a K or V tile
  static constexpr int kKVBytes = kKVHalf * kHalves;
  // TMEM columns: S_A, S_B (BN FP32 each), O_A, O_B (HD), P_A, P_B (BN FP16)
  static __device__ __forceinline__ uint32_t col_s(int x) { return x * BN; }
  static __device__ __forceinline__ uint32_t col_o(int x) { return 2 * BN + x * HD; }
  static __device__ __forceinline__ uint32_t col_p(int x) { return 2 * BN + 2 * HD + x * (BN / 2); }
  static_assert(2 * BN + 2 * HD + BN <= 512, "TMEM columns");
  // output staged through shared memory (HD 64) or stored from registers
  static constexpr bool kStaged = HD <= 64;
  static_assert(BN % 64 == 0 && HD % 64 == 0, "tiles are whole 64-element halves");
};

template <int HD, int BN, int STAGES>
struct PfSmem {
  // 1024-byte aligned tiles (128-byte swizzle atoms are 8 rows x 128 B)
  uint8_t q[2][PfShape<HD, BN, STAGES>::kQBytes];      // Q_A, Q_B (FP16 high parts)
  uint8_t ql[2][PfShape<HD, BN, STAGES>::kQBytes];     // their FP16 residuals
  uint8_t k[STAGES][PfShape<HD, BN, STAGES>::kKVBytes];
  uint8_t v[STAGES][PfShape<HD, BN, STAGES>::kKVBytes];
  // per softmax warp, 32 rows x 32 output columns; 16-byte chunk c of row r
  // sits at chunk c ^ (r & 7), so that both the row-wise writes and the
  // transposed reads are conflict-free without padding
  float stage[PfShape<HD, BN, STAGES>::kStaged ? 8 : 1]
             [PfShape<HD, BN, STAGES>::kStaged ? 32 * kPfStagePitch : 4];
  uint64_t q_full, q_empty;
  uint64_t kv_full[STAGES], kv_empty[STAGES];
  uint64_t s_full[2], s_free[2], p_full[2][2], pv_done[2][2], o_free[2];
  uint64_t item_full[2], item_empty[2];
  uint64_t mma_done[2];
  int item[2];
  uint32_t tmem_base;
};

template <int HD, int BN, int STAGES>
constexpr int pf_smem_bytes() {
  return static_cast<int>(sizeof(PfSmem<HD, BN, STAGES>)) + 1024;
}
static_assert(pf_smem_bytes<64, 128, 4>() <= 227 * 1024, "prefill shared memory above the limit");
static_assert(pf_smem_bytes<128, 64, 3>() <= 227 * 1024, "prefill shared memory above the limit");

__device__ __forceinline__ void tc_ld_x32(uint32_t taddr, uint32_t* r) {
  tc_ld_32x32b_x32(taddr, *reinterpret_cast<uint32_t(*)[32]>(r));
}

// After tcgen05.wait::ld: make every later use of r depend on the wait (the
// load writes r asynchronously; the compiler must not read r earlier).
__device__ __forceinline__ void reg_fence32(uint32_t* r) {
#pragma unroll
  for (int i = 0; i < 32; ++i) asm volatile("" : "+r"(r[i]));
}

// 2^x for two x <= 0 on the FMA pipe: x = n + f with n = round(x) (the
// 1.5*2^23 addition leaves n in the low mantissa bits), 2^f on [-0.5, 0.5]
// by a cubic fitted for minimum relative error (max 7.5e-5, below the FP16
// rounding P gets next), and n added to the exponent field.  x is clamped at
// -126 so the exponent field cannot wrap: there (and for x = -inf) the
// result is below 2^-125, which is 0 after the FP16 rounding of P.
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
  constexpr float kC0 = 0.99992806f, kC1 = 0.69326097f, kC2 = 0.24261113f, kC3 = 0.05517166f;
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  x.x = fmaxf(x.x, -126.f);
  x.y = fmaxf(x.y, -126.f);
  const float2 t = add2(x, make_float2(kMagic, kMagic));
  const float2 n = add2(t, make_float2(-kMagic, -kMagic));
  const float2 f = fma2(n, make_float2(-1.f, -1.f), x);  // x - n, exact
  float2 p = fma2(make_float2(kC3, kC3), f, make_float2(kC2, kC2));
  p = fma2(p, f, make_float2(kC1, kC1));
  p = fma2(p, f, make_float2(kC0, kC0));
  return make_float2(__int_as_float(__float_as_int(p.x) + (__float_as_int(t.x) << 23)),
                     __int_as_float(__float_as_int(p.y) + (__float_as_int(t.y) << 23)));
}

struct PfItem {
  int q_row0, head0, head1, kvh, nkv, p_min;
};

// Item b, heaviest first: query tile n_qt-1-b/per_tile, head pair b%per_tile.
template <int BN>
__device__ __forceinline__ PfItem pf_item(const PrefillArgs& a, int b) {
  PfItem it;
  const bool dual = a.kv_mul >= 2;
  const int per_tile = dual ? a.n_heads / 2 : a.n_heads;
  const int n_qt = (a.n_tok + kPfBlockM - 1) / kPfBlockM;
  const int qt = n_qt - 1 - b / per_tile;
  const int r_item = b % per_tile;
  if (dual) {
    const int pairs = a.kv_mul / 2;
    it.head0 = (r_item / pairs) * a.kv_mul + 2 * (r_item % pairs);
    it.head1 = it.head0 + 1;
  } else {
    it.head0 = r_item;
    it.head1 = -1;
  }
  it.kvh = it.head0 / a.kv_mul;
  it.q_row0 = qt * kPfBlockM;
  const int last_row = min(a.n_tok, it.q_row0 + kPfBlockM) - 1;
  it.nkv = (a.start_pos + last_row + 1 + BN - 1) / BN;  // >= 1
  it.p_min = a.start_pos + it.q_row0;
  return it;
}

__device__ __forceinline__ int pf_n_items(const PrefillArgs& a) {
  const int per_tile = a.kv_mul >= 2 ? a.n_heads / 2 : a.n_heads;
  return ((a.n_tok + kPfBlockM - 1) / kPfBlockM) * per_tile;
}

template <int HD, int BN, int STAGES>
__global__ void __launch_bounds__(kPfThreads, 1)
    prefill_attn_kernel(const PrefillArgs a, const __grid_constant__ CUtensorMap tm_q,
                        const __grid_constant__ CUtensorMap tm_ql,
                        const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v,
                        const __grid_constant__ CUtensorMap tm_o) {
  using Sh = PfShape<HD, BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  PfSmem<HD, BN, STAGES>& sm = *reinterpret_cast<PfSmem<HD, BN, STAGES>*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_slots = a.kv_mul >= 2 ? 2 : 1;

  if (threadIdx.x == 0) {
    mbar_init(&sm.q_full, 1);
    mbar_init(&sm.q_empty, n_slots);  // one commit per active issuer
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&sm.kv_full[s], 1);
      mbar_init(&sm.kv_empty[s], n_slots);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(&sm.s_full[x], 1);
      mbar_init(&sm.s_free[x], 4);
      mbar_init(&sm.o_free[x], 4);
      for (int b2 = 0; b2 < 2; ++b2) {
        mbar_init(&sm.p_full[x][b2], 4);
        mbar_init(&sm.pv_done[x][b2], 1);
      }
      mbar_init(&sm.item_full[x], 1);
      mbar_init(&sm.item_empty[x], 10);  // 2 MMA issuers + 8 softmax warps
      mbar_init(&sm.mma_done[x], 1);
    }
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(&sm.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // launched behind the prologue with programmatic dependent launch: the
  // set-up above overlapped its tail; q16 and the cache rows it appended
  // are read only after it has finished.  The scheduler lane takes its
  // first item before its own wait: the work counter is not the
  // prologue's (the attention grid before it, complete before the prologue
  // started, left it at zero), so the fetch and the item's decoding
  // overlap the prologue's tail too.
  const bool sched_lane = warp == 8 && lane == 0;
  if (!sched_lane) asm volatile("griddepcontrol.wait;" ::: "memory");
  const uint32_t tmem = sm.tmem_base;
  if (warp >= 8) {
    regs_dec<kPfOtherRegs>();  // warp 11 only completes the warpgroup
    if (warp == 8) {
      // --------------------------------------------------- scheduler + TMA
      if (lane == 0) {
        tma_prefetch_desc(&tm_q);
        tma_prefetch_desc(&tm_ql);
        tma_prefetch_desc(&tm_k);
        tma_prefetch_desc(&tm_v);
        const int n_items = pf_n_items(a);
        int J = 0, k = 0;
        bool ok = true;
        while (true) {
          int item = ok ? atomicAdd(&a.work[0], 1) : -1;
          if (item >= n_items) item = -1;
          if (k >= 2 && !mbar_wait_bounded(&sm.item_empty[k & 1], ((k - 2) >> 1) & 1)) {
            atomicOr(a.err, ERR_TIMEOUT_EMPTY);
            break;  // consumers time out on item_full and wind down
          }
          sm.item[k & 1] = item;
          mbar_arrive(&sm.item_full[k & 1]);
          if (item < 0) break;
          const PfItem it = pf_item<BN>(a, item);
          // the first item's loads read the prologue's output
          if (k == 0) asm volatile("griddepcontrol.wait;" ::: "memory");
          // Q of the previous item is in use until its last S MMAs complete
          if (k >= 1 && !mbar_wait_bounded(&sm.q_empty, (k - 1) & 1)) {
            atomicOr(a.err, ERR_TIMEOUT_EMPTY);
            ok = false;
            ++k;
            continue;
          }
          mbar_arrive_expect_tx(&sm.q_full, 2 * n_slots * Sh::kQBytes);
#pragma unroll
          for (int hv = 0; hv < Sh::kHalves; ++hv) {
            tma_load_3d(sm.q[0] + hv * Sh::kQHalf, &tm_q, &sm.q_full, 64 * hv, it.head0,
                        it.q_row0);
            tma_load_3d(sm.ql[0] + hv * Sh::kQHalf, &tm_ql, &sm.q_full, 64 * hv, it.head0,
                        it.q_row0);
            if (n_slots == 2) {
              tma_load_3d(sm.q[1] + hv * Sh::kQHalf, &tm_q, &sm.q_full, 64 * hv, it.head1,
                          it.q_row0);
              tma_load_3d(sm.ql[1] + hv * Sh::kQHalf, &tm_ql, &sm.q_full, 64 * hv, it.head1,
                          it.q_row0);
            }
          }
          for (int j = 0; j < it.nkv; ++j, ++J) {
            const int s = J % STAGES;
            if (J >= STAGES && !mbar_wait_bounded(&sm.kv_empty[s], ((J / STAGES) - 1) & 1)) {
              atomicOr(a.err, ERR_TIMEOUT_EMPTY);
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&sm.kv_full[s], 2 * Sh::kKVBytes);
#pragma unroll
            for (int hv = 0; hv < Sh::kHalves; ++hv) {
              tma_load_4d(sm.k[s] + hv * Sh::kKVHalf, &tm_k, &sm.kv_full[s], 64 * hv, j * BN,
                          it.kvh, a.slab);
              tma_load_4d(sm.v[s] + hv * Sh::kKVHalf, &tm_v, &sm.kv_full[s], 64 * hv, j * BN,
                          it.kvh, a.slab);
            }
          }
          ++k;
        }
        // never leave with copies in flight: the last use of each stage must land
        for (int j = J - STAGES; j < J; ++j)
          if (j >= 0) mbar_wait_bounded(&sm.kv_full[j % STAGES], (j / STAGES) & 1);
        if (k >= 1) mbar_wait_bounded(&sm.q_full, (k - 1) & 1);
        // the last CTA to stop fetching resets the counters for the next launch
        __threadfence();
        if (atomicAdd(&a.work[1], 1) == static_cast<int>(gridDim.x) - 1) {
          a.work[0] = 0;
          a.work[1] = 0;
          __threadfence();
        }
      }
    } else if (warp <= 10) {
      // ------------------------------------------------- MMA issuer of slot x
      const int x = warp - 9;
      if (lane == 0) {
        const uint32_t idesc_qk = idesc_f16_f32(128, BN, 0);
        const uint32_t idesc_pv = idesc_f16_f32(128, 64, 1);  // one 64-column half of O
        const bool active = x < n_slots;
        const uint32_t q_addr = smem_u32(sm.q[x]);
        const uint32_t ql_addr = smem_u32(sm.ql[x]);
        int J = 0, k = 0;
        bool ok = true;
        // PV_x of global tile g (first tile of its item if `first`), then
        // release of its K/V stage
        auto issue_pv = [&](int g, bool first) -> bool {
          const int s = g % STAGES, pb = g & 1;
          if (!mbar_wait_bounded(&sm.p_full[x][pb], (g >> 1) & 1)) return false;
          // the previous item's O must be read out before it is overwritten
          if (first && k >= 1 && !mbar_wait_bounded(&sm.o_free[x], (k - 1) & 1)) return false;
          tc_fence_after();
          const uint32_t v_addr = smem_u32(sm.v[s]);
#pragma unroll
          for (int hv = 0; hv < Sh::kHalves; ++hv) {   // O columns 64hv .. 64hv+63
#pragma unroll
            for (int kk = 0; kk < BN / 16; ++kk) {  // 16 keys = 8 P columns per MMA
              const uint64_t bd =
                  smem_desc_sw128(v_addr + hv * Sh::kKVHalf + kk * 16 * 128, 16, 1024);
              tc_mma_ts(tmem + Sh::col_o(x) + 64 * hv, tmem + Sh::col_p(x) + kk * 8, bd,
                        idesc_pv, (first && kk == 0) ? 0u : 1u);
            }
          }
          tc_commit(&sm.pv_done[x][pb]);
          tc_commit(&sm.kv_empty[s]);
          return true;
        };
        while (ok) {
          if (!mbar_wait_bounded(&sm.item_full[k & 1], (k >> 1) & 1)) { ok = false; break; }
          const int item = *reinterpret_cast<volatile int*>(&sm.item[k & 1]);
          mbar_arrive(&sm.item_empty[k & 1]);
          if (item < 0) break;
          const PfItem it = pf_item<BN>(a, item);
          if (!active) {  // no second query head: nothing to issue
            J += it.nkv;
            ++k;
            continue;
          }
          if (!mbar_wait_bounded(&sm.q_full, k & 1)) { ok = false; break; }
          for (int j = 0; j < it.nkv && ok; ++j) {
            const int g = J + j;
            const int s = g % STAGES;
            if (!mbar_wait_bounded(&sm.kv_full[s], (g / STAGES) & 1)) { ok = false; break; }
            if (g >= 1 && !mbar_wait_bounded(&sm.s_free[x], (g - 1) & 1)) { ok = false; break; }
            tc_fence_after();
            const uint32_t k_addr = smem_u32(sm.k[s]);
#pragma unroll
            for (int kk = 0; kk < HD / 16; ++kk) {  // 16 dims per MMA, 4 per 128-byte half
              const uint32_t off_q = (kk >> 2) * Sh::kQHalf + (kk & 3) * 32;
              const uint32_t off_k = (kk >> 2) * Sh::kKVHalf + (kk & 3) * 32;
              const uint64_t bd = smem_desc_sw128(k_addr + off_k, 16, 1024);
              // Q_hi K^T, then Q_lo K^T into the same S
              tc_mma_ss(tmem + Sh::col_s(x), smem_desc_sw128(q_addr + off_q, 16, 1024), bd,
                        idesc_qk, kk > 0 ? 1u : 0u);
              tc_mma_ss(tmem + Sh::col_s(x), smem_desc_sw128(ql_addr + off_q, 16, 1024), bd,
                        idesc_qk, 1u);
            }
            tc_commit(&sm.s_full[x]);
            if (j == it.nkv - 1) tc_commit(&sm.q_empty);  // Q_x free once these S MMAs land
            if (j >= 1 && !issue_pv(g - 1, j == 1)) ok = false;
          }
          if (ok && !issue_pv(J + it.nkv - 1, it.nkv == 1)) ok = false;
          J += it.nkv;
          ++k;
        }
        if (!ok) atomicOr(a.err, ERR_TIMEOUT_MMA);
        // all issued MMAs must finish before TMEM is freed
        tc_commit(&sm.mma_done[x]);
        mbar_wait_bounded(&sm.mma_done[x], 0);
      }
    }
  } else {
    regs_inc<kPfSoftmaxRegs>();
    // ------------------------------------------------------------ softmax
    const int x = warp >> 2;                     // slot
    const int r = threadIdx.x & 127;             // query row in the tile, TMEM lane
    const uint32_t lane_base = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const float sc = a.score_scale;
    const bool active = x < n_slots;
    uint32_t sv[BN];   // this row of S (one TMEM read per tile)
    int J = 0, k = 0;
    bool ok = true;
    while (ok) {
      if (!mbar_wait_bounded(&sm.item_full[k & 1], (k >> 1) & 1)) { ok = false; break; }
      const int item = *reinterpret_cast<volatile int*>(&sm.item[k & 1]);
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.item_empty[k & 1]);
      if (item < 0) break;
      const PfItem it = pf_item<BN>(a, item);
      if (!active) {  // slot B without a second query head: nothing to do
        J += it.nkv;
        ++k;
        continue;
      }
      const int p_row = it.p_min + r;  // this row's position
      float m_used = -INFINITY, l_run = 0.f;
      for (int j = 0; j < it.nkv; ++j) {
        const int g = J + j;
        if (!mbar_wait_bounded(&sm.s_full[x], g & 1)) { ok = false; break; }
        tc_fence_after();
        const int t0 = j * BN;
        const bool need_mask = t0 + BN - 1 > it.p_min;  // diagonal tile
        const int lim = p_row - t0;  // columns c <= lim are visible
#pragma unroll
        for (int c4 = 0; c4 < BN / 32; ++c4)
          tc_ld_x32(lane_base + Sh::col_s(x) + 32 * c4, sv + 32 * c4);
        tc_wait_ld();
#pragma unroll
        for (int c4 = 0; c4 < BN / 32; ++c4) reg_fence32(sv + 32 * c4);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.s_free[x]);  // S may be overwritten now
        if (need_mask) {
#pragma unroll
          for (int c = 0; c < BN; ++c)
            if (c > lim) sv[c] = __float_as_uint(-INFINITY);
        }
        // row max as a tree: 8 independent partial maxima, then combine
        float mp[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) mp[u] = __uint_as_float(sv[u]);
#pragma unroll
        for (int c = 8; c < BN; c += 16)
#pragma unroll
          for (int u = 0; u < 8; ++u)
            mp[u] = max3(mp[u], __uint_as_float(sv[c + u]), __uint_as_float(sv[c + 8 + u]));
        const float m_tile = max3(max3(mp[0], mp[1], mp[2]), max3(mp[3], mp[4], mp[5]),
                                  fmaxf(mp[6], mp[7])) * sc;
        // lazy rescale: only when some row of the warp outgrew its max by 2^8
        // (O itself is rescaled below, once PV(g-1) has landed in it)
        const bool rescale = __any_sync(0xffffffffu, m_tile > m_used + kPfRescaleLog2);
        float alpha = 1.f;
        if (rescale) {
          const float m_new = fmaxf(m_used, m_tile);
          alpha = ex2(m_used - m_new);  // 0 on the first tile
          l_run *= alpha;
          m_used = m_new;
        }
        // P = 2^(s*c - m) packed as FP16 pairs (masked -> 0), in BN/64 parts of
        // 64 columns, each stored to TMEM as soon as it is ready
        const float2 sc2 = make_float2(sc, sc), nm2 = make_float2(-m_used, -m_used);
        float2 rs2[4];  // 4 independent partial row sums
#pragma unroll
        for (int e = 0; e < 4; ++e) rs2[e] = make_float2(0.f, 0.f);
#pragma unroll
        for (int h = 0; h < BN / 64; ++h) {
          uint32_t pw[32];
#pragma unroll
          for (int cc = 0; cc < 8; ++cc) {  // 8 chunks of 8 columns
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int c = 64 * h + 8 * cc + 2 * e;
              const float2 arg =
                  fma2(make_float2(__uint_as_float(sv[c]), __uint_as_float(sv[c + 1])), sc2, nm2);
              // five pairs in eight on MUFU, three on the FMA pipe (-inf -> 0)
              const int pe = (4 * cc + e) & 7;
              const float2 pp = (pe == 2 || pe == 5 || pe == 7)
                                    ? exp2_poly2(arg)
                                    : make_float2(ex2(arg.x), ex2(arg.y));
              rs2[e] = add2(rs2[e], pp);
              pw[4 * cc + e] = pack_half2(pp.x, pp.y);
            }
          }
          if (h == 0) {
            // P(g) overwrites P(g-1) and O is rescaled: both need PV(g-1)
            // done (PV(g) is issued only after p_full(g) below)
            if (g >= 1 && !mbar_wait_bounded(&sm.pv_done[x][(g - 1) & 1], ((g - 1) >> 1) & 1)) {
              ok = false;
              break;
            }
            tc_fence_after();
            if (rescale && j >= 1) {
#pragma unroll
              for (int q4 = 0; q4 < HD / 16; ++q4) {  // O in chunks of 16 columns
                uint32_t ov[16];
                tc_ld_32x32b_x16(lane_base + Sh::col_o(x) + 16 * q4, ov);
                tc_wait_ld();
#pragma unroll
                for (int d = 0; d < 16; ++d) asm volatile("" : "+r"(ov[d]));
#pragma unroll
                for (int d = 0; d < 16; ++d) ov[d] = __float_as_uint(__uint_as_float(ov[d]) * alpha);
                tc_st_32x32b_x16(lane_base + Sh::col_o(x) + 16 * q4, ov);
              }
            }
          }
          tc_st_32x32b_x32(lane_base + Sh::col_p(x) + 32 * h, pw);
        }
        if (!ok) break;
        tc_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.p_full[x][g & 1]);
        const float2 rsa = add2(rs2[0], rs2[1]), rsb = add2(rs2[2], rs2[3]);
        l_run += (rsa.x + rsa.y) + (rsb.x + rsb.y);
      }
      if (!ok) break;
      // O / l once the item's last PV has landed; then O is free again
      const int g_last = J + it.nkv - 1;
      if (!mbar_wait_bounded(&sm.pv_done[x][g_last & 1], (g_last >> 1) & 1)) { ok = false; break; }
      tc_fence_after();
      // O (HD columns) lands in the dead S row where it fits
      uint32_t ov_own[HD > BN ? HD : 1];
      uint32_t* ov;
      if constexpr (HD > BN)
        ov = ov_own;
      else
        ov = sv;
#pragma unroll
      for (int c4 = 0; c4 < HD / 32; ++c4) tc_ld_x32(lane_base + Sh::col_o(x) + 32 * c4, ov + 32 * c4);
      tc_wait_ld();
#pragma unroll
      for (int c4 = 0; c4 < HD / 32; ++c4) reg_fence32(ov + 32 * c4);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.o_free[x]);
      // O / l to the output through the warp's staging buffer, 32 columns
      // at a time: a thread holds one row, so direct stores would touch 32
      // rows per instruction.  With an output tensor map (o_tma) one lane
      // hands each 32 x 32 box to the TMA unit and the warp moves on to its
      // next item (stores from the threads took about 2,500 cycles of the
      // item switch); without one the warp reads the buffer back
      // transposed, each store instruction covering four rows x 128
      // contiguous bytes.  At head_dim 128 the
      // shared memory goes to a deeper K/V ring instead and the rows are
      // stored directly.
      const float inv = 1.0f / l_run;
      const int row_base = it.q_row0 + (warp & 3) * 32;
      if constexpr (!Sh::kStaged) {
        float* drow = a.out + static_cast<size_t>(row_base + lane) * a.out_stride +
                      (x ? it.head1 : it.head0) * HD;
        if (row_base + lane < a.n_tok) {
#pragma unroll
          for (int c = 0; c < HD; c += 4)
            *reinterpret_cast<float4*>(drow + c) = make_float4(
                __uint_as_float(ov[c]) * inv, __uint_as_float(ov[c + 1]) * inv,
                __uint_as_float(ov[c + 2]) * inv, __uint_as_float(ov[c + 3]) * inv);
        }
      }
      float* stg = sm.stage[Sh::kStaged ? warp : 0];
      const int o_col = (x ? it.head1 : it.head0) * HD;
      float* dst = a.out + o_col + (lane & 7) * 4;
#pragma unroll
      for (int hc = 0; hc < (Sh::kStaged ? HD / 32 : 0); ++hc) {
        if (a.o_tma) {
          // the previous TMA store from this buffer must have read it
          if (lane == 0) bulk_wait_read_all();
          __syncwarp();
        }
#pragma unroll
        for (int c = 0; c < 32; c += 4)
          *reinterpret_cast<float4*>(stg + lane * kPfStagePitch + 4 * ((c >> 2) ^ (lane & 7))) =
              make_float4(
              __uint_as_float(ov[32 * hc + c]) * inv, __uint_as_float(ov[32 * hc + c + 1]) * inv,
              __uint_as_float(ov[32 * hc + c + 2]) * inv, __uint_as_float(ov[32 * hc + c + 3]) * inv);
        if (a.o_tma) {
          // the staging layout is the 128-byte swizzle of a 32 x 32 FP32 box:
          // one bulk store per round, rows past n_tok clipped by the TMA unit;
          // the warp goes on to its next item while the store drains
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tm_o, stg, o_col + 32 * hc, row_base);
            bulk_commit();
          }
          continue;
        }
        __syncwarp();
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int rr = 4 * i + (lane >> 3);
          const float4 val = *reinterpret_cast<const float4*>(
              stg + rr * kPfStagePitch + 4 * ((lane & 7) ^ (rr & 7)));
          if (row_base + rr < a.n_tok)
            *reinterpret_cast<float4*>(dst + static_cast<size_t>(row_base + rr) * a.out_stride +
                                       32 * hc) = val;
        }
        __syncwarp();
      }
      J += it.nkv;
      ++k;
    }
    if (!ok) atomicOr(a.err, ERR_TIMEOUT_MMA);
    // no store may still read the staging buffer (or be in flight) at exit
    if (Sh::kStaged && a.o_tma && lane == 0) bulk_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Host side: one persistent CTA per SM (never more than there are items).
// With `overlap`, the launch may begin while the previous grid on the stream
// (the prologue) is still running (programmatic stream serialisation).
// HD 64 runs <64, 128, 4>, HD 128 runs <128, 64, 3>; the tensor maps carry
// boxes of 64 elements x 128 query rows (q hi and lo) and 64 x BN cache rows
// (k, v).
template <int HD, int BN, int STAGES>
inline int launch_prefill_shape(const PrefillArgs& a, const CUtensorMap& tm_q,
                                const CUtensorMap& tm_ql, const CUtensorMap& tm_k,
                                const CUtensorMap& tm_v, const CUtensorMap& tm_o, int num_sms,
                                cudaStream_t st, bool overlap) {
  auto kern = prefill_attn_kernel<HD, BN, STAGES>;
  constexpr int smem = pf_smem_bytes<HD, BN, STAGES>();
  // kernel attributes are per device: set them the first time this kernel
  // launches on each device (one bit per device)
  static std::atomic<unsigned long long> attr_done{0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -4;
  const unsigned long long bit = dev < 64 ? 1ull << dev : 0ull;
  if (!bit || !(attr_done.load(std::memory_order_acquire) & bit)) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
        cudaSuccess)
      return -4;
    // the warpgroup register split assumes exactly this launch allocation:
    // with fewer registers per thread the softmax warps' increase could
    // never be granted
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, kern) != cudaSuccess || fa.numRegs != kPfLaunchRegs) {
      fprintf(stderr, "pl_attn: prefill kernel built with %d registers per thread, needs %d\n",
              fa.numRegs, kPfLaunchRegs);
      return -4;
    }
    attr_done.fetch_or(bit, std::memory_order_release);
  }
  const int per_tile = a.kv_mul >= 2 ? a.n_heads / 2 : a.n_heads;
  const int n_items = ((a.n_tok + kPfBlockM - 1) / kPfBlockM) * per_tile;
  const int grid = n_items < num_sms ? n_items : num_sms;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kPfThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = overlap ? 1 : 0;
  if (cudaLaunchKernelEx(&cfg, kern, a, tm_q, tm_ql, tm_k, tm_v, tm_o) != cudaSuccess) return -4;
  return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

// KV tile rows of the prefill kernel at a head_dim (the tensor-map box).
constexpr int pf_block_n(int head_dim) { return head_dim == 128 ? 64 : 128; }

inline int launch_prefill_attention(int head_dim, const PrefillArgs& a, const CUtensorMap& tm_q,
                                    const CUtensorMap& tm_ql, const CUtensorMap& tm_k,
                                    const CUtensorMap& tm_v, const CUtensorMap& tm_o,
                                    int num_sms, cudaStream_t st, bool overlap) {
  if (head_dim == 128)
    return launch_prefill_shape<128, 64, 3>(a, tm_q, tm_ql, tm_k, tm_v, tm_o, num_sms, st,
                                            overlap);
  return launch_prefill_shape<64, 128, 4>(a, tm_q, tm_ql, tm_k, tm_v, tm_o, num_sms, st,
                                          overlap);
}

}  // namespace pl
