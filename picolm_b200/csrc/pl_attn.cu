// pl_attn.cu -- the module behind include/pl_attn.h: context, device KV
// cache, RoPE tables, TMA descriptors, argument checks and kernel dispatch.
//
// One global context, as picolm's gpu.c keeps one (picolm/gpu.c:34-83).
// Host-buffer calls stage their inputs through one pinned buffer and one
// H2D copy, launch, and read the output and the device error word back with
// one D2H copy.  There is no CPU fallback anywhere: every failure is a
// negative status.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <atomic>
#include <condition_variable>
#include <mutex>
#include <thread>
#include <vector>

#include "../../include/pl_attn.h"
#include "kern_decode.cuh"
#include "kern_gemm.cuh"
#include "kern_misc.cuh"
#include "kern_prefill.cuh"
#include "kern_proj.cuh"
#include "kern_xfer.cuh"

namespace {

using pl::part_stride;

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

constexpr int kDecodeStages = 4;  // K/V ring depth, 3 where a stage would exceed 32 KB

// Receive buffer of the KV-split exchange and the peers' buffers mapped here.
struct Xfer {
  int world = 0, rank = 0;
  uint8_t* local = nullptr;              // this rank's buffer (cudaMalloc)
  pl::XferPeers peers = {};              // every rank's buffer as seen from this GPU
  void* opened[pl::kXferMaxRanks] = {};  // IPC mappings to close
  // pl_attn_decode_p2p_dev: the merge grid's arrival counter (zero at rest)
  // and the shard's partial when one decode CTA covers it
  uint32_t* d_arrive = nullptr;
  float* d_part1 = nullptr;
};

// One layer's attention weights on the device (pl_attn_set_layer), all in one
// allocation: Wq, Wk, Wv, Wo rows in the kern_proj.cuh layout, then the F32
// RMSNorm weights, biases and QK-norm weights (nullptr where absent).
struct LayerW {
  uint8_t* mem = nullptr;
  const uint8_t* w[4] = {};   // q, k, v, o
  size_t row_bytes[4] = {};
  int type[4] = {};
  const float* bias[4] = {};
  const float* attn_norm = nullptr;
  const float* q_norm = nullptr;
  const float* k_norm = nullptr;
  float eps = 0.f;
  int dim = 0;
  // The same weights dequantised for the tensor-core GEMM of many input rows
  // (kern_gemm.cuh): FP16 high part and 2^11-scaled residual, Q/K/V rows
  // concatenated [q_dim + 2 kv_dim][dim], O [dim][q_dim]; one allocation.
  uint8_t* gmem = nullptr;
  bool gemm = false;
  CUtensorMap tm_qkv_h, tm_qkv_l, tm_o_h, tm_o_l;
};

struct Ctx {
  int device = -1;
  int n_layers = 0, n_heads = 0, n_kv_heads = 0, max_seq = 0, n_seqs = 0, rope_type = 0;
  int rope_rows = 0;          // positions < rope_rows (the model's max_seq_len); max_seq is the
                              // cache rows per (slot, layer), fewer on a device of a KV split
  int head_dim = 0, kv_dim = 0, q_dim = 0, kv_mul = 0;
  int part_floats = 0;        // floats of one partial block: n_heads * (head_dim + 4)
  int tp = 0;                 // decode tile rows: TP * n_kv_heads * head_dim == 8192, TP >= 16
  int nstage = 0;             // decode ring depth
  int num_sms = 0, decode_slots = 0;
  size_t layer_elems = 0;     // FP16 words per (seq, layer) slab
  uint16_t* d_k = nullptr;    // [n_seqs][n_layers][max_seq][kv_dim]
  uint16_t* d_v = nullptr;
  float* d_cos = nullptr;     // [max_seq][head_dim / 2]
  float* d_sin = nullptr;
  // staging for host-buffer calls
  uint8_t* d_stage = nullptr;
  uint8_t* h_stage = nullptr;
  uint8_t* h_stage_dev = nullptr;  // h_stage as the device addresses it (mapped)
  size_t stage_cap = 0;
  // split-KV partials
  float* d_part = nullptr;
  size_t part_cap = 0;        // floats
  int2* d_seg_info = nullptr; // [kMaxLaunchSeqs] (first slot, segments) per decode sequence
  int* d_work = nullptr;      // [2] prefill work-queue counters (self-resetting)
  // prefill FP16 q staging
  uint16_t* d_q16 = nullptr;  // high parts, then the residuals at d_q16 + q16_cap
  size_t q16_cap = 0;         // elements of each
  uint32_t* d_err = nullptr;  // device error word
  cudaStream_t stream = nullptr;
  uint32_t* h_err = nullptr;      // pinned, mapped: the error word as a host call's last kernel saw it
  uint32_t* h_err_dev = nullptr;  // its device address
  CUtensorMap tm_k_dec, tm_v_dec;  // decode: box {64, tp, Hk, 1}, head_dim/64 per tile
  CUtensorMap tm_k_pf, tm_v_pf;    // prefill: box {64, 128 rows, 1, 1}
  CUtensorMap tm_q16;              // prefill q staging: box {64, 1 head, 128 rows}, HD/64 per row
  CUtensorMap tm_q16lo;            // the same over the residuals
  EncodeTiledFn encode = nullptr;
  // profiling: event pairs around each attention kernel (see pl_attn_profile)
  int profiling = 0;
  std::vector<cudaEvent_t> ev_pool;  // even index: start, odd: end
  size_t ev_used = 0;                // events recorded since the last read
  long n_attn = 0, n_all = 0;        // attention launches / all launches
  // attention-block projections
  std::vector<LayerW> lw;            // [n_layers]
  float* d_blk = nullptr;            // q, k, v, attention output of a block call
  size_t blk_cap = 0;                // floats
  float* d_proj_part = nullptr;      // split-input partial sums of the projections
  size_t proj_part_cap = 0;          // floats
  __half* d_xh = nullptr;            // GEMM activations: FP16 high parts, then
  __half* d_xl = nullptr;            // the 2^11-scaled residuals
  size_t act_cap = 0;                // elements of each
  int sk_clusters[9] = {};           // skinny GEMM: resident clusters per cluster size (lazy)
  bool gemm_smem_set = false;
  bool proj_smem_set = false;
};

Ctx* g = nullptr;
Xfer* g_xfer = nullptr;  // KV-split exchange of the current context, if set up

// A context over several devices (pl_attn_init_devices with n_devices > 1):
// g is then its first device's context.  Defined at the end of this file.
struct Multi;
Multi* g_multi = nullptr;
void multi_free();
int multi_set_rope(const float* cos_tab, const float* sin_tab, int n_rows, int half_dim);
int multi_decode_batch(int layer, int n, const int* seqs, const int* pos, const float* q,
                       const float* k, const float* v, float* out);
int multi_prefill(int seq, int layer, int start_pos, int n_tok, const float* q, const float* k,
                  const float* v, float* out, int out_stride);
int multi_kv_copy(int seq, int layer, int pos0, int n_pos, uint16_t* k, uint16_t* v,
                  bool download);
int multi_status();
int multi_set_wait_limit(uint64_t ns);
void multi_profile(int enable);
int multi_profile_read(double* attn_ms, long* attn_launches, long* all_launches);
int multi_init(int n_layers, int n_heads, int n_kv_heads, int head_dim, int max_seq_len,
               float rope_freq_base, int rope_type, int n_seqs, int n_devices,
               const int* devices, int split);

void xfer_free() {
  if (!g_xfer) return;
  for (int r = 0; r < pl::kXferMaxRanks; ++r)
    if (g_xfer->opened[r]) cudaIpcCloseMemHandle(g_xfer->opened[r]);
  cudaFree(g_xfer->local);
  cudaFree(g_xfer->d_arrive);
  cudaFree(g_xfer->d_part1);
  delete g_xfer;
  g_xfer = nullptr;
}
std::mutex g_mu;

#define PL_CUDA(call)                                                     \
  do {                                                                    \
    cudaError_t e_ = (call);                                              \
    if (e_ != cudaSuccess) {                                              \
      std::fprintf(stderr, "pl_attn: %s failed: %s (%s:%d)\n", #call,      \
                   cudaGetErrorString(e_), __FILE__, __LINE__);           \
      return PL_ECUDA;                                                    \
    }                                                                     \
  } while (0)

// ---- device and pinned-host allocations ------------------------------
// Every allocation of the module goes through these two.  Failure injection
// for callers' tests, on the host: with PL_ATTN_FAIL_ALLOC=n in the
// environment when pl_attn_init runs, the n-th allocation the module then
// attempts (1 = the first, counting init's own) fails as if the device or
// the pinned host pool were exhausted, without calling CUDA, so PL_ENOMEM
// paths can be exercised without filling a GPU.
std::atomic<long> g_fail_alloc{0};  // countdown; 0 = off

bool inject_alloc_failure() {
  long v = g_fail_alloc.load();
  while (v > 0)
    if (g_fail_alloc.compare_exchange_weak(v, v - 1)) return v == 1;
  return false;
}

template <typename T>
cudaError_t dev_alloc(T** p, size_t bytes) {
  void* v = nullptr;
  const cudaError_t e = inject_alloc_failure() ? cudaErrorMemoryAllocation : cudaMalloc(&v, bytes);
  *p = static_cast<T*>(v);
  return e;
}

template <typename T>
cudaError_t host_alloc(T** p, size_t bytes) {
  void* v = nullptr;
  const cudaError_t e =
      inject_alloc_failure() ? cudaErrorMemoryAllocation : cudaMallocHost(&v, bytes);
  *p = static_cast<T*>(v);
  return e;
}

int make_map(EncodeTiledFn enc, CUtensorMap* m, uint16_t* base, int head_dim, int max_seq,
             int n_kv_heads, int n_slabs, int box_rows, int box_heads) {
  // dims, innermost first: head_dim, row, kv head, (seq, layer) slab; the box
  // is 64 elements (128 bytes, the swizzle span) wide
  const cuuint64_t dims[4] = {static_cast<cuuint64_t>(head_dim), static_cast<cuuint64_t>(max_seq),
                              static_cast<cuuint64_t>(n_kv_heads),
                              static_cast<cuuint64_t>(n_slabs)};
  const cuuint64_t kv_bytes = static_cast<cuuint64_t>(n_kv_heads) * head_dim * 2;
  const cuuint64_t strides[3] = {kv_bytes, static_cast<cuuint64_t>(head_dim) * 2,
                                 kv_bytes * static_cast<cuuint64_t>(max_seq)};
  const cuuint32_t box[4] = {64u, static_cast<cuuint32_t>(box_rows),
                             static_cast<cuuint32_t>(box_heads), 1u};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, base, dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    std::fprintf(stderr, "pl_attn: cuTensorMapEncodeTiled failed (%d)\n", static_cast<int>(r));
    return PL_ECUDA;
  }
  return PL_OK;
}

// The prefill output, n_tok rows of `cols` FP32 at a row stride of `stride`
// floats, as a 2-D TMA map for the attention kernel's stores: boxes of 32
// columns x 32 rows under the 128-byte swizzle.  False when TMA cannot
// address the rows (base not 16-byte aligned, stride not a multiple of four
// floats); the kernel then stores from its threads.
bool make_out_map(EncodeTiledFn enc, CUtensorMap* m, float* out, int cols, int rows,
                  int stride) {
  if ((reinterpret_cast<uintptr_t>(out) & 15) || (stride & 3) || cols > stride || rows < 1)
    return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(stride) * 4};
  const cuuint32_t box[2] = {32u, 32u};
  const cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, out, dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

void host_rope_tables(float* c, float* s, int max_seq, int head_dim, float base) {
  // picolm/model.c:545-556, same libm calls in FP32
  const int half = head_dim / 2;
  for (int p = 0; p < max_seq; ++p)
    for (int i = 0; i < half; ++i) {
      const float inv = powf(base, static_cast<float>(2 * i) / static_cast<float>(head_dim));
      const float theta = static_cast<float>(p) / inv;
      c[static_cast<size_t>(p) * half + i] = cosf(theta);
      s[static_cast<size_t>(p) * half + i] = sinf(theta);
    }
}

// A q of up to this many bytes rides in the staging area's one copy even
// when registered: a host memcpy of 16 KB costs less than a second copy.
constexpr size_t kStagedQBytes = 16384;

int ensure_stage(size_t bytes) {
  if (bytes <= g->stage_cap) return PL_OK;
  size_t cap = g->stage_cap ? g->stage_cap : (1u << 20);
  while (cap < bytes) cap *= 2;
  if (g->d_stage) cudaFree(g->d_stage);
  if (g->h_stage) cudaFreeHost(g->h_stage);
  g->d_stage = nullptr;
  g->h_stage = nullptr;
  g->stage_cap = 0;
  g->h_stage_dev = nullptr;
  if (dev_alloc(&g->d_stage, cap) != cudaSuccess) return PL_ENOMEM;
  if (host_alloc(&g->h_stage, cap) != cudaSuccess) return PL_ENOMEM;
  if (cudaHostGetDevicePointer(reinterpret_cast<void**>(&g->h_stage_dev), g->h_stage, 0) !=
      cudaSuccess)
    return PL_ECUDA;
  g->stage_cap = cap;
  return PL_OK;
}

// ---- caller buffers page-locked with pl_attn_host_register ----------------
// A host-buffer call moves an input or output that lies inside a registered
// range directly between it and the device (no copy through the staging
// area).  model.c allocates s->q, s->k, s->v and s->xb once and reuses them
// for every call, so it can register them at start-up.
// A registered range is also mapped into the device's address space:
// kernels of a host-buffer call may read an input that is used once, or
// write the output, straight over the bus.
struct HostRange {
  uintptr_t lo, hi;
  uint8_t* dev;  // device address of lo
};
std::vector<HostRange> g_pinned;

bool pinned(const void* p, size_t bytes) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  for (const HostRange& r : g_pinned)
    if (a >= r.lo && a + bytes <= r.hi) return true;
  return false;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Device address of [p, p + bytes) when it lies in a registered range and p
// is 16-byte aligned (the kernels move 8- and 16-byte vectors), else
// nullptr.
uint8_t* mapped(const void* p, size_t bytes) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  if (!aligned16(p)) return nullptr;
  for (const HostRange& r : g_pinned)
    if (a >= r.lo && a + bytes <= r.hi) return r.dev + (a - r.lo);
  return nullptr;
}

// ---- parallel copies between caller buffers and the pinned staging area ---
// The host-buffer entry points move every input and output through the
// pinned staging area; one thread copies only about 10 GB/s, which made
// those copies most of a host-buffer call.  A few sleeping helper threads
// (started on the first such call; PL_ATTN_COPY_THREADS overrides their
// number, 0 turns them off) split each copy with the calling thread.
struct CopyPiece {
  uint8_t* dst;
  const uint8_t* src;
  size_t bytes;
};

class CopyPool {
 public:
  explicit CopyPool(int n) {
    for (int i = 0; i < n; ++i) th_.emplace_back([this, i] { run(i + 1); });
  }
  ~CopyPool() {
    {
      std::lock_guard<std::mutex> lk(mu_);
      stop_ = true;
    }
    cv_.notify_all();
    for (auto& t : th_) t.join();
  }
  // all pieces copied when this returns
  void copy(const CopyPiece* pc, int n_pc) {
    size_t total = 0;
    for (int i = 0; i < n_pc; ++i) total += pc[i].bytes;
    const int parts = static_cast<int>(th_.size()) + 1;
    if (parts == 1 || total < (256u << 10)) {
      for (int i = 0; i < n_pc; ++i) std::memcpy(pc[i].dst, pc[i].src, pc[i].bytes);
      return;
    }
    {
      std::lock_guard<std::mutex> lk(mu_);
      pc_ = pc;
      n_pc_ = n_pc;
      total_ = total;
      parts_ = parts;
      left_.store(parts - 1);
      ++gen_;
    }
    cv_.notify_all();
    part(0);
    while (left_.load(std::memory_order_acquire) != 0) std::this_thread::yield();
  }

 private:
  // bytes [p*total/parts, (p+1)*total/parts) of the concatenated pieces
  void part(int p) {
    const size_t lo = total_ * p / parts_, hi = total_ * (p + 1) / parts_;
    size_t s0 = 0;
    for (int i = 0; i < n_pc_; s0 += pc_[i].bytes, ++i) {
      const size_t a = lo > s0 ? lo : s0, b = hi < s0 + pc_[i].bytes ? hi : s0 + pc_[i].bytes;
      if (a < b) std::memcpy(pc_[i].dst + (a - s0), pc_[i].src + (a - s0), b - a);
    }
  }
  void run(int p) {
    uint64_t seen = 0;
    while (true) {
      {
        std::unique_lock<std::mutex> lk(mu_);
        cv_.wait(lk, [&] { return stop_ || gen_ != seen; });
        if (stop_) return;
        seen = gen_;
      }
      part(p);
      left_.fetch_sub(1, std::memory_order_release);
    }
  }
  std::vector<std::thread> th_;
  std::mutex mu_;
  std::condition_variable cv_;
  bool stop_ = false;
  uint64_t gen_ = 0;
  const CopyPiece* pc_ = nullptr;
  int n_pc_ = 0, parts_ = 1;
  size_t total_ = 0;
  std::atomic<int> left_{0};
};

CopyPool* g_copy = nullptr;  // lives as long as the context

void host_copy(const CopyPiece* pc, int n_pc) {
  if (!g_copy) {
    int n = static_cast<int>(std::thread::hardware_concurrency()) / 2;
    if (n > 7) n = 7;
    if (const char* e = std::getenv("PL_ATTN_COPY_THREADS")) n = std::atoi(e);
    if (n < 0) n = 0;
    g_copy = new CopyPool(n);
  }
  g_copy->copy(pc, n_pc);
}

int ensure_part(size_t floats) {
  if (floats <= g->part_cap) return PL_OK;
  if (g->d_part) cudaFree(g->d_part);
  g->d_part = nullptr;
  g->part_cap = 0;
  if (dev_alloc(&g->d_part, floats * sizeof(float)) != cudaSuccess) return PL_ENOMEM;
  g->part_cap = floats;
  return PL_OK;
}

// FP16 q staging for the prefill, [rows][n_heads][head_dim] twice (the high
// parts, then the residuals), with a TMA map over each.  Rows past the
// current n_tok hold stale data; they only feed query rows whose output is
// never stored.
int ensure_q16(int n_tok) {
  const size_t rows = static_cast<size_t>(n_tok);
  if (rows * g->q_dim <= g->q16_cap) return PL_OK;
  size_t cap_rows = 256;
  while (cap_rows < rows) cap_rows *= 2;
  if (g->d_q16) cudaFree(g->d_q16);
  g->d_q16 = nullptr;
  g->q16_cap = 0;
  const size_t elems = cap_rows * g->q_dim;
  if (dev_alloc(&g->d_q16, 2 * elems * sizeof(uint16_t)) != cudaSuccess) return PL_ENOMEM;
  if (cudaMemset(g->d_q16, 0, 2 * elems * sizeof(uint16_t)) != cudaSuccess) return PL_ECUDA;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(g->head_dim),
                              static_cast<cuuint64_t>(g->n_heads),
                              static_cast<cuuint64_t>(cap_rows)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(g->head_dim) * 2,
                                 static_cast<cuuint64_t>(g->q_dim) * 2};
  const cuuint32_t box[3] = {64u, 1u, static_cast<cuuint32_t>(pl::kPfBlockM)};
  const cuuint32_t estr[3] = {1, 1, 1};
  for (int part = 0; part < 2; ++part)
    if (g->encode(part ? &g->tm_q16lo : &g->tm_q16, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                  g->d_q16 + part * elems, dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return PL_ECUDA;
  g->q16_cap = elems;
  return PL_OK;
}

// Profiling hooks: a start/end event pair around each attention kernel,
// recorded on the kernel's own stream.
cudaEvent_t prof_event() {
  if (g->ev_used == g->ev_pool.size()) {
    cudaEvent_t e;
    if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
    g->ev_pool.push_back(e);
  }
  return g->ev_pool[g->ev_used++];
}

void prof_begin(cudaStream_t st) {
  if (!g->profiling) return;
  if (cudaEvent_t e = prof_event()) cudaEventRecord(e, st);
}

void prof_end(cudaStream_t st) {
  if (!g->profiling) return;
  if (cudaEvent_t e = prof_event()) cudaEventRecord(e, st);
  ++g->n_attn;
}

void count_launch() {
  if (g->profiling) ++g->n_all;
}

// Read (and clear) the device error word.
int check_err_word(uint32_t w) {
  if (w & (pl::ERR_TIMEOUT_FULL | pl::ERR_TIMEOUT_EMPTY | pl::ERR_TIMEOUT_MMA)) return PL_ETIMEOUT;
  if (w & pl::ERR_BAD_ARG) return PL_EARG;  // a slot or position out of range on the device
  if (w) return PL_EFAIL;
  return PL_OK;
}

// Grid of the decode kernel: one CTA per resident slot, but never more CTAs
// than tiles (max_rows bounds every sequence's rows).
// A single sequence of at most this many tiles is decoded by one CTA: no
// merge grid follows (one launch fewer), and each input is read once.
constexpr int kOneCtaTiles = 8;

int decode_grid(int n, int max_rows) {
  const long long tiles = static_cast<long long>(n) * ((max_rows + g->tp - 1) / g->tp);
  if (n == 1 && tiles <= kOneCtaTiles) return 1;
  long long G = g->decode_slots;
  if (G > tiles) G = tiles;
  return G < 1 ? 1 : static_cast<int>(G);
}

// Decode arguments shared by every launch path.
pl::DecodeArgs decode_args(int layer, int n, const int* d_seqs, const int* d_pos,
                           const float* d_q, const float* d_k, const float* d_v, float* d_out,
                           int mode, int row0, int n_rows, int append, float* part_out,
                           float* part, int2* seg_info) {
  pl::DecodeArgs a;
  a.n_layers = g->n_layers;
  a.max_seq = g->max_seq;
  a.pos_limit = g->rope_rows;
  a.n_heads = g->n_heads;
  a.n_kv_heads = g->n_kv_heads;
  a.kv_mul = g->kv_mul;
  a.layer = layer;
  a.n_slots = g->n_seqs;
  a.rope_type = g->rope_type;
  a.cos_tab = g->d_cos;
  a.sin_tab = g->d_sin;
  a.kc = g->d_k;
  a.vc = g->d_v;
  a.n = n;
  a.seqs = d_seqs;
  a.pos = d_pos;
  a.seq1 = 0;
  a.pos1 = 0;
  a.q = d_q;
  a.k = d_k;
  a.v = d_v;
  a.out = d_out;
  a.out_stride = g->q_dim;
  a.part = part;
  a.part_out = part_out;
  a.seg_info = seg_info;
  a.mode = mode;
  a.row0 = row0;
  a.n_rows = n_rows;
  a.append = append;
  a.score_scale = pl::kLog2e / sqrtf(static_cast<float>(g->head_dim));
  a.err = g->d_err;
  a.err_host = nullptr;
  a.n_inline = 0;
  return a;
}

int decode_smem_bytes_for(int n_kv_heads, int tp, int nstage, int head_dim) {
  return nstage * 2 * tp * n_kv_heads * head_dim * 2 + 1024 + 2 * nstage * 8;
}

int decode_smem_bytes(int tp, int nstage, int head_dim) {
  return decode_smem_bytes_for(g->n_kv_heads, tp, nstage, head_dim);
}

// The decode kernel instantiations: (tile rows, ring depth, head_dim) for
// n_kv_heads 8, 4, 2, 1 at head_dim 64 and 128.
template <int TP, int NS, int HD>
cudaError_t decode_occupancy(int* per_sm, int threads, int smem) {
  auto kern = pl::decode_kernel<TP, NS, HD>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(per_sm, kern, threads, smem);
}

template <int TP, int NS, int HD>
int launch_decode_tp(const pl::DecodeArgs& a, int grid, cudaStream_t st, bool profile) {
  const int smem = decode_smem_bytes(TP, NS, HD);
  auto kern = pl::decode_kernel<TP, NS, HD>;
  // the shared-memory attribute is per device: set it the first time this
  // instantiation launches on each device (one bit per device)
  static std::atomic<unsigned long long> attr_done{0};
  int dev = 0;
  PL_CUDA(cudaGetDevice(&dev));
  const unsigned long long bit = dev < 64 ? 1ull << dev : 0ull;
  if (!bit || !(attr_done.load(std::memory_order_acquire) & bit)) {
    PL_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    attr_done.fetch_or(bit, std::memory_order_release);
  }
  if (profile) prof_begin(st);
  // Programmatic stream serialisation: the grid may become resident while
  // the kernel queued before it finishes and run its set-up then; the kernel
  // reads nothing that kernel writes before griddepcontrol.wait (positions
  // and slots only as a hint that it checks after the wait).
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3((g->n_kv_heads + 1) * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  PL_CUDA(cudaLaunchKernelEx(&cfg, kern, a, g->tm_k_dec, g->tm_v_dec));
  if (profile) {
    prof_end(st);
    count_launch();
  }
  return PL_OK;
}

// The split merge, queued behind the decode grid with programmatic stream
// serialisation (its CTAs become resident while the decode grid runs and
// wait on griddepcontrol.wait).  Heads per block: the fewest that keep the
// merge grid within one block per SM.  At head_dim 64 one merge block fits
// on an SM beside a decode CTA and a second does not (registers), so such a
// grid is resident from the start, and the next decode grid, which launches
// once every merge block has started, can take each SM as soon as its
// decode CTA ends (config 4: 30.2 -> 29.0 us per step).
int launch_merge(const pl::DecodeArgs& a, int decode_grid_ctas, cudaStream_t st, bool profile,
                 const pl::XferPush* push = nullptr) {
  // one CTA: every sequence is one segment (a pushing merge still exchanges)
  if (decode_grid_ctas <= 1 && !push) return PL_OK;
  int hpb = pl::kMergeThreads / (g->head_dim / 4);  // 16 at head_dim 64, 8 at 128
  while (hpb > 1 &&
         static_cast<long long>(a.n) * ((g->n_heads + hpb / 2 - 1) / (hpb / 2)) <= g->num_sms)
    hpb >>= 1;
  if (push) hpb = 1;  // a pushing merge exchanges one head per block
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.n, (g->n_heads + hpb - 1) / hpb);
  cfg.blockDim = dim3(pl::kMergeThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const pl::XferPush none = {};
  const pl::XferPush& x = push ? *push : none;
  if (g->head_dim == 128)
    PL_CUDA(cudaLaunchKernelEx(&cfg, push ? pl::merge_kernel<128, true> : pl::merge_kernel<128, false>,
                               a, hpb, decode_grid_ctas, g->tp, x));
  else
    PL_CUDA(cudaLaunchKernelEx(&cfg, push ? pl::merge_kernel<64, true> : pl::merge_kernel<64, false>,
                               a, hpb, decode_grid_ctas, g->tp, x));
  if (profile) count_launch();
  return PL_OK;
}

// Calls F.template operator()<TP, NS, HD>() for the context's decode
// configuration; PL_EUNSUPPORTED for any other.
template <typename F>
auto with_decode_config(int tp, int nstage, int head_dim, F&& f) -> decltype(f.template operator()<16, 4, 64>()) {
  if (head_dim == 64 && nstage == kDecodeStages) {
    switch (tp) {
      case 16: return f.template operator()<16, kDecodeStages, 64>();
      case 32: return f.template operator()<32, kDecodeStages, 64>();
      case 64: return f.template operator()<64, kDecodeStages, 64>();
      case 128: return f.template operator()<128, kDecodeStages, 64>();
    }
  } else if (head_dim == 128) {
    if (nstage == 3 && tp == 16) return f.template operator()<16, 3, 128>();
    if (nstage == kDecodeStages) switch (tp) {
        case 16: return f.template operator()<16, kDecodeStages, 128>();
        case 32: return f.template operator()<32, kDecodeStages, 128>();
        case 64: return f.template operator()<64, kDecodeStages, 128>();
      }
  }
  return f.unsupported();
}

struct DecodeLaunch {
  const pl::DecodeArgs& a;
  int grid;
  cudaStream_t st;
  bool profile;
  template <int TP, int NS, int HD>
  int operator()() const { return launch_decode_tp<TP, NS, HD>(a, grid, st, profile); }
  int unsupported() const { return PL_EUNSUPPORTED; }
};

struct DecodeOccupancy {
  int* per_sm;
  int threads, smem;
  template <int TP, int NS, int HD>
  cudaError_t operator()() const { return decode_occupancy<TP, NS, HD>(per_sm, threads, smem); }
  cudaError_t unsupported() const { return cudaErrorInvalidValue; }
};

int launch_decode_kernel(const pl::DecodeArgs& a, int grid, cudaStream_t st, bool profile,
                         const pl::XferPush* push = nullptr) {
  const int rc =
      with_decode_config(g->tp, g->nstage, g->head_dim, DecodeLaunch{a, grid, st, profile});
  if (rc) return rc;
  return launch_merge(a, grid, st, profile, push);
}

// Launch the fused decode for n sequences (chunks of kMaxLaunchSeqs).  All
// pointers are device pointers; mode/row0/n_rows/append as in DecodeArgs.
// In mode 1 the merged partials go to part_out instead of out.
int launch_decode(int layer, int n, const int* d_seqs, const int* d_pos, int max_rows,
                  const float* d_q, const float* d_k, const float* d_v, float* d_out,
                  int mode, int row0, int n_rows, int append, float* part_out,
                  cudaStream_t st, uint32_t* err_host = nullptr,
                  const int* h_seqs = nullptr, const int* h_pos = nullptr) {
  for (int s0 = 0; s0 < n; s0 += pl::kMaxLaunchSeqs) {
    const int m = n - s0 < pl::kMaxLaunchSeqs ? n - s0 : pl::kMaxLaunchSeqs;
    const int grid = decode_grid(m, max_rows);
    const size_t need = static_cast<size_t>(grid + m) * g->part_floats;
    int rc = ensure_part(need);
    if (rc) return rc;
    const pl::DecodeArgs a = decode_args(
        layer, m, d_seqs + s0, d_pos + s0, d_q + static_cast<size_t>(s0) * g->q_dim,
        d_k + static_cast<size_t>(s0) * g->kv_dim, d_v + static_cast<size_t>(s0) * g->kv_dim,
        d_out ? d_out + static_cast<size_t>(s0) * g->q_dim : nullptr, mode, row0, n_rows, append,
        part_out ? part_out + static_cast<size_t>(s0) * g->part_floats : nullptr,
        g->d_part, g->d_seg_info);
    pl::DecodeArgs b = a;
    b.err_host = err_host;
    if (h_seqs && h_pos && m <= pl::kInlineSeqs) {
      // (slot, position) pairs in the arguments: the device arrays are not read
      b.n_inline = m;
      for (int i = 0; i < m; ++i) b.sp[i] = make_int2(h_seqs[s0 + i], h_pos[s0 + i]);
    }
    rc = launch_decode_kernel(b, grid, st, true);
    if (rc) return rc;
  }
  return PL_OK;
}

// One KV shard's partial (mode 1) for n_rows > 0 local rows: seq and pos
// travel as kernel arguments (no copy, nothing that could make the host
// wait for the stream).
int partial_launch(int seq, int layer, int pos, int row0, int n_rows, int append,
                   const float* d_q, const float* d_k, const float* d_v, float* d_part,
                   cudaStream_t st) {
  const int grid = decode_grid(1, n_rows);
  const int rc = ensure_part(static_cast<size_t>(grid + 1) * g->part_floats);
  if (rc) return rc;
  pl::DecodeArgs a = decode_args(layer, 1, nullptr, nullptr, d_q, d_k ? d_k : d_q,
                                 d_v ? d_v : d_q, nullptr, 1, row0, n_rows, append ? 1 : 0,
                                 d_part, g->d_part, g->d_seg_info);
  a.seq1 = seq;
  a.pos1 = pos;
  return launch_decode_kernel(a, grid, st, true);
}

// Device-pointer calls run on the caller's stream; NULL is the CUDA
// default (legacy) stream, as everywhere in CUDA.
cudaStream_t pick_stream(void* s) { return static_cast<cudaStream_t>(s); }

int check_seq_layer(int seq, int layer) {
  if (!g) return PL_ESTATE;
  if (seq < 0 || seq >= g->n_seqs || layer < 0 || layer >= g->n_layers) return PL_EARG;
  return PL_OK;
}

uint16_t* slab_k(int seq, int layer) {
  return g->d_k + (static_cast<size_t>(seq) * g->n_layers + layer) * g->layer_elems;
}
uint16_t* slab_v(int seq, int layer) {
  return g->d_v + (static_cast<size_t>(seq) * g->n_layers + layer) * g->layer_elems;
}

// Synchronise the module stream, fetch the error word (already copied to
// the pinned area at `h_err`), clear it on the device if set.
int finish_host_call(const uint32_t* h_err) {
  PL_CUDA(cudaStreamSynchronize(g->stream));
  const uint32_t w = *h_err;
  if (w) {
    cudaMemsetAsync(g->d_err, 0, sizeof(uint32_t), g->stream);
    cudaStreamSynchronize(g->stream);
  }
  return check_err_word(w);
}

void free_ctx(Ctx* c) {
  if (!c) return;
  if (c->device >= 0) cudaSetDevice(c->device);
  if (c->stream) cudaStreamSynchronize(c->stream);
  cudaFree(c->d_k);
  cudaFree(c->d_v);
  cudaFree(c->d_cos);
  cudaFree(c->d_sin);
  cudaFree(c->d_stage);
  cudaFreeHost(c->h_stage);
  cudaFree(c->d_part);
  cudaFree(c->d_seg_info);
  cudaFree(c->d_work);
  cudaFree(c->d_q16);
  cudaFree(c->d_err);
  cudaFreeHost(c->h_err);
  cudaFree(c->d_blk);
  cudaFree(c->d_proj_part);
  for (LayerW& l : c->lw) {
    cudaFree(l.mem);
    cudaFree(l.gmem);
  }
  cudaFree(c->d_xh);
  cudaFree(c->d_xl);
  for (cudaEvent_t e : c->ev_pool) cudaEventDestroy(e);
  if (c->stream) cudaStreamDestroy(c->stream);
  delete c;
}

// Shape checks shared by every init path (no device needed).
int check_shape(int n_layers, int n_heads, int n_kv_heads, int head_dim, int max_seq_len,
                float rope_freq_base, int rope_type, int n_seqs) {
  if (n_layers <= 0 || n_heads <= 0 || n_kv_heads <= 0 || max_seq_len <= 0 || n_seqs <= 0 ||
      !(rope_freq_base > 0.f))
    return PL_EARG;
  if (head_dim != 64 && head_dim != 128) return PL_EUNSUPPORTED;
  if (n_heads % n_kv_heads) return PL_EUNSUPPORTED;
  const int kv_mul = n_heads / n_kv_heads;
  if (!(n_kv_heads == 1 || n_kv_heads == 2 || n_kv_heads == 4 || n_kv_heads == 8))
    return PL_EUNSUPPORTED;
  if (!(kv_mul == 1 || kv_mul == 2 || kv_mul == 4 || kv_mul == 8)) return PL_EUNSUPPORTED;
  if (rope_type != PL_ROPE_LLAMA && rope_type != PL_ROPE_QWEN) return PL_EARG;
  return PL_OK;
}

// One device's context: `n_slots` sequence slots of `cache_rows` rows per
// layer, RoPE tables for positions [0, rope_rows).  The shape is checked.
int create_ctx(int n_layers, int n_heads, int n_kv_heads, int head_dim, int rope_rows,
               float rope_freq_base, int rope_type, int n_slots, int cache_rows, int device,
               Ctx** out) {
  *out = nullptr;
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) return PL_EDEVICE;
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return PL_EDEVICE;
  if (prop.major != 10) return PL_EDEVICE;
  if (cudaSetDevice(device) != cudaSuccess) return PL_EDEVICE;

  Ctx* c = new Ctx();
  c->device = device;
  c->n_layers = n_layers;
  c->n_heads = n_heads;
  c->n_kv_heads = n_kv_heads;
  c->max_seq = cache_rows;
  c->rope_rows = rope_rows;
  c->n_seqs = n_slots;
  c->rope_type = rope_type;
  c->head_dim = head_dim;
  c->kv_dim = n_kv_heads * head_dim;
  c->q_dim = n_heads * head_dim;
  c->part_floats = n_heads * part_stride(head_dim);
  c->kv_mul = n_heads / n_kv_heads;
  // a K (or V) tile of 16 KB: all KV heads, TP rows (at least 16, the MMA
  // row block); at 128 x 8 KV heads that is 32 KB and the ring is 3 deep
  c->tp = 8192 / (n_kv_heads * head_dim);
  if (c->tp < 16) c->tp = 16;
  c->nstage = c->tp * n_kv_heads * head_dim > 8192 ? 3 : kDecodeStages;
  c->num_sms = prop.multiProcessorCount;
  c->layer_elems = static_cast<size_t>(cache_rows) * c->kv_dim;
  const size_t cache_elems = c->layer_elems * n_layers * n_slots;

  int rc = PL_OK;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult qres;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &qres) !=
          cudaSuccess ||
      qres != cudaDriverEntryPointSuccess || !fn) {
    free_ctx(c);
    return PL_ECUDA;
  }
  c->encode = reinterpret_cast<EncodeTiledFn>(fn);

  if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess ||
      dev_alloc(&c->d_k, cache_elems * 2) != cudaSuccess ||
      dev_alloc(&c->d_v, cache_elems * 2) != cudaSuccess ||
      dev_alloc(&c->d_cos, sizeof(float) * rope_rows * (head_dim / 2)) != cudaSuccess ||
      dev_alloc(&c->d_sin, sizeof(float) * rope_rows * (head_dim / 2)) != cudaSuccess ||
      dev_alloc(&c->d_err, 256) != cudaSuccess ||
      dev_alloc(&c->d_seg_info, sizeof(int2) * pl::kMaxLaunchSeqs) != cudaSuccess ||
      dev_alloc(&c->d_work, 2 * sizeof(int)) != cudaSuccess ||
      host_alloc(&c->h_err, sizeof(uint32_t)) != cudaSuccess) {
    free_ctx(c);
    return PL_ENOMEM;
  }
  if (cudaHostGetDevicePointer(reinterpret_cast<void**>(&c->h_err_dev), c->h_err, 0) !=
      cudaSuccess) {
    free_ctx(c);
    return PL_ECUDA;
  }
  *c->h_err = 0;
  cudaMemsetAsync(c->d_k, 0, cache_elems * 2, c->stream);
  cudaMemsetAsync(c->d_v, 0, cache_elems * 2, c->stream);
  cudaMemsetAsync(c->d_err, 0, 256, c->stream);
  cudaMemsetAsync(c->d_seg_info, 0, sizeof(int2) * pl::kMaxLaunchSeqs, c->stream);
  cudaMemsetAsync(c->d_work, 0, 2 * sizeof(int), c->stream);
  {
    const uint64_t ns = pl::kDefaultWaitLimitNs;
    cudaMemcpyToSymbolAsync(pl::g_wait_limit_ns, &ns, sizeof(ns), 0, cudaMemcpyHostToDevice,
                            c->stream);
  }
  {
    const size_t n = static_cast<size_t>(rope_rows) * (head_dim / 2);
    float* hc = static_cast<float*>(std::malloc(n * sizeof(float)));
    float* hs = static_cast<float*>(std::malloc(n * sizeof(float)));
    if (!hc || !hs) {
      std::free(hc);
      std::free(hs);
      free_ctx(c);
      return PL_ENOMEM;
    }
    host_rope_tables(hc, hs, rope_rows, head_dim, rope_freq_base);
    cudaMemcpy(c->d_cos, hc, n * sizeof(float), cudaMemcpyHostToDevice);
    cudaMemcpy(c->d_sin, hs, n * sizeof(float), cudaMemcpyHostToDevice);
    std::free(hc);
    std::free(hs);
  }
  const int n_slabs = n_slots * n_layers;
  if ((rc = make_map(c->encode, &c->tm_k_dec, c->d_k, head_dim, cache_rows, n_kv_heads, n_slabs,
                     c->tp, n_kv_heads)) ||
      (rc = make_map(c->encode, &c->tm_v_dec, c->d_v, head_dim, cache_rows, n_kv_heads, n_slabs,
                     c->tp, n_kv_heads)) ||
      (rc = make_map(c->encode, &c->tm_k_pf, c->d_k, head_dim, cache_rows, n_kv_heads, n_slabs,
                     pl::pf_block_n(head_dim), 1)) ||
      (rc = make_map(c->encode, &c->tm_v_pf, c->d_v, head_dim, cache_rows, n_kv_heads, n_slabs,
                     pl::pf_block_n(head_dim), 1))) {
    free_ctx(c);
    return rc;
  }
  // decode grid: as many CTAs as can be resident at once (registers, shared
  // memory), so the balanced partition runs in a single wave
  {
    int per_sm = 0;
    const int smem = decode_smem_bytes_for(c->n_kv_heads, c->tp, c->nstage, head_dim);
    const int threads = (n_kv_heads + 1) * 32;
    const cudaError_t e =
        with_decode_config(c->tp, c->nstage, head_dim, DecodeOccupancy{&per_sm, threads, smem});
    if (e != cudaSuccess || per_sm < 1) {
      free_ctx(c);
      return PL_ECUDA;
    }
    c->decode_slots = c->num_sms * per_sm;
  }
  c->lw.resize(static_cast<size_t>(n_layers));
  if (cudaStreamSynchronize(c->stream) != cudaSuccess) {
    free_ctx(c);
    return PL_ECUDA;
  }
  *out = c;
  return PL_OK;
}

}  // namespace

extern "C" {

const char* pl_attn_strerror(int rc) {
  switch (rc) {
    case PL_OK: return "success";
    case PL_EFAIL: return "failure";
    case PL_EARG: return "argument out of range";
    case PL_ENOMEM: return "out of device or pinned host memory";
    case PL_ECUDA: return "CUDA error";
    case PL_ETIMEOUT: return "a bounded device-side wait expired";
    case PL_ESTATE: return "attention module not initialised (or initialised twice)";
    case PL_EDEVICE: return "no usable sm_100 CUDA device";
    case PL_EUNSUPPORTED: return "shape not supported by the B200 attention kernels";
    default: return "unknown status";
  }
}

int pl_attn_available(void) { return g != nullptr; }

int pl_attn_init(int n_layers, int n_heads, int n_kv_heads, int head_dim, int max_seq_len,
                 float rope_freq_base, int rope_type, int n_seqs, int device) {
  return pl_attn_init_devices(n_layers, n_heads, n_kv_heads, head_dim, max_seq_len,
                              rope_freq_base, rope_type, n_seqs, 1, &device, PL_SPLIT_SEQS);
}

int pl_attn_init_devices(int n_layers, int n_heads, int n_kv_heads, int head_dim,
                         int max_seq_len, float rope_freq_base, int rope_type, int n_seqs,
                         int n_devices, const int* devices, int split) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (g) return PL_ESTATE;
  if (n_devices < 1 || n_devices > 16 || !devices) return PL_EARG;
  if (split != PL_SPLIT_SEQS && split != PL_SPLIT_KV) return PL_EARG;
  for (int d = 0; d < n_devices; ++d)
    if (devices[d] < 0) return PL_EARG;
  int rc = check_shape(n_layers, n_heads, n_kv_heads, head_dim, max_seq_len, rope_freq_base,
                       rope_type, n_seqs);
  if (rc) return rc;
  {
    const char* fa = std::getenv("PL_ATTN_FAIL_ALLOC");
    g_fail_alloc.store(fa ? std::atol(fa) : 0);
  }
  if (n_devices == 1) {
    Ctx* c = nullptr;
    rc = create_ctx(n_layers, n_heads, n_kv_heads, head_dim, max_seq_len, rope_freq_base,
                    rope_type, n_seqs, max_seq_len, devices[0], &c);
    if (rc) return rc;
    g = c;
    return PL_OK;
  }
  return multi_init(n_layers, n_heads, n_kv_heads, head_dim, max_seq_len, rope_freq_base,
                    rope_type, n_seqs, n_devices, devices, split);
}

void pl_attn_shutdown(void) {
  std::lock_guard<std::mutex> lk(g_mu);
  for (const HostRange& r : g_pinned) cudaHostUnregister(reinterpret_cast<void*>(r.lo));
  g_pinned.clear();
  delete g_copy;
  g_copy = nullptr;
  if (g && g->device >= 0) cudaSetDevice(g->device);
  xfer_free();
  if (g_multi) {
    multi_free();  // every device's context, g included
  } else {
    free_ctx(g);
  }
  g = nullptr;
}

int pl_attn_set_rope(const float* cos_tab, const float* sin_tab, int n_rows, int half_dim) {
  if (!g) return PL_ESTATE;
  if (!cos_tab || !sin_tab || half_dim != g->head_dim / 2 || n_rows <= 0) return PL_EARG;
  if (g_multi) return multi_set_rope(cos_tab, sin_tab, n_rows, half_dim);
  if (cudaSetDevice(g->device) != cudaSuccess) return PL_ECUDA;
  const int rows = n_rows < g->rope_rows ? n_rows : g->rope_rows;
  const size_t bytes = static_cast<size_t>(rows) * half_dim * sizeof(float);
  PL_CUDA(cudaMemcpyAsync(g->d_cos, cos_tab, bytes, cudaMemcpyHostToDevice, g->stream));
  PL_CUDA(cudaMemcpyAsync(g->d_sin, sin_tab, bytes, cudaMemcpyHostToDevice, g->stream));
  PL_CUDA(cudaStreamSynchronize(g->stream));
  return PL_OK;
}

// Output (qb bytes at d_out on the device) and the error word to the caller:
// straight into a registered `out`, else through the staging area at h (qb
// + 4 bytes) with one read-back.  Waits for the stream.
static int read_back(const float* d_out, float* out, size_t qb, uint8_t* h) {
  uint8_t* d = reinterpret_cast<uint8_t*>(const_cast<float*>(d_out));
  PL_CUDA(cudaMemcpyAsync(d + qb, g->d_err, sizeof(uint32_t), cudaMemcpyDeviceToDevice,
                          g->stream));
  const bool direct = pinned(out, qb);
  if (direct) {
    PL_CUDA(cudaMemcpyAsync(out, d, qb, cudaMemcpyDeviceToHost, g->stream));
    PL_CUDA(cudaMemcpyAsync(h + qb, d + qb, sizeof(uint32_t), cudaMemcpyDeviceToHost, g->stream));
  } else {
    PL_CUDA(cudaMemcpyAsync(h, d, qb + sizeof(uint32_t), cudaMemcpyDeviceToHost, g->stream));
  }
  const int rc = finish_host_call(reinterpret_cast<uint32_t*>(h + qb));
  if (rc || direct) return rc;
  const CopyPiece o = {reinterpret_cast<uint8_t*>(out), h, qb};
  host_copy(&o, 1);
  return PL_OK;
}

// Host-buffer decode of one sequence.  The slot and position travel as
// kernel arguments.  When one CTA covers the sequence every input is read
// once, so the kernel reads q, k and v over the bus (from registered
// buffers, else from the mapped staging area after a host memcpy) and the
// call queues no copy at all; otherwise q, k and v go to the device in one
// copy.  The output is written over the bus either way.
static int decode_one_host(int layer, int seq, int pos, const float* q, const float* k,
                           const float* v, float* out) {
  const size_t qb = static_cast<size_t>(g->q_dim) * sizeof(float);
  const size_t kb = static_cast<size_t>(g->kv_dim) * sizeof(float);
  const size_t in_bytes = qb + 2 * kb;
  const size_t out_off = (in_bytes + 255) & ~static_cast<size_t>(255);
  int rc = ensure_stage(out_off + qb + 256);
  if (rc) return rc;
  uint8_t* h = g->h_stage;
  uint8_t* hd = g->h_stage_dev;
  uint8_t* d = g->d_stage;
  const int grid = decode_grid(1, pos + 1);
  const float* src[3] = {q, k, v};
  const size_t off[3] = {0, qb, qb + kb};
  const size_t bytes[3] = {qb, kb, kb};
  const float* dptr[3];
  CopyPiece pc[3];
  int n_pc = 0;
  for (int j = 0; j < 3; ++j) {
    const uint8_t* m = grid == 1 ? mapped(src[j], bytes[j]) : nullptr;
    if (m) {
      dptr[j] = reinterpret_cast<const float*>(m);
    } else {
      pc[n_pc++] = {h + off[j], reinterpret_cast<const uint8_t*>(src[j]), bytes[j]};
      dptr[j] = reinterpret_cast<const float*>((grid == 1 ? hd : d) + off[j]);
    }
  }
  if (n_pc) host_copy(pc, n_pc);
  if (grid != 1) PL_CUDA(cudaMemcpyAsync(d, h, in_bytes, cudaMemcpyHostToDevice, g->stream));
  *reinterpret_cast<volatile uint32_t*>(g->h_err) = 0;
  uint8_t* mo = mapped(out, qb);
  float* d_out = reinterpret_cast<float*>(mo ? mo : hd + out_off);
  pl::DecodeArgs a = decode_args(layer, 1, nullptr, nullptr, dptr[0], dptr[1], dptr[2], d_out, 0,
                                 0, 0, 1, nullptr, g->d_part, g->d_seg_info);
  a.seq1 = seq;
  a.pos1 = pos;
  a.err_host = g->h_err_dev;
  if (grid > 1) {
    rc = ensure_part(static_cast<size_t>(grid + 1) * g->part_floats);
    if (rc) return rc;
    a.part = g->d_part;
  }
  rc = launch_decode_kernel(a, grid, g->stream, true);
  if (rc) return rc;
  PL_CUDA(cudaStreamSynchronize(g->stream));
  const uint32_t w = *reinterpret_cast<volatile uint32_t*>(g->h_err);
  if (w) {
    cudaMemsetAsync(g->d_err, 0, sizeof(uint32_t), g->stream);
    cudaStreamSynchronize(g->stream);
    return check_err_word(w);
  }
  if (!mo) {
    const CopyPiece o = {reinterpret_cast<uint8_t*>(out), h + out_off, qb};
    host_copy(&o, 1);
  }
  return PL_OK;
}

int pl_attn_decode_batch(int layer, int n, const int* seqs, const int* pos, const float* q,
                         const float* k, const float* v, float* out) {
  if (!g) return PL_ESTATE;
  if (g_multi) return multi_decode_batch(layer, n, seqs, pos, q, k, v, out);
  if (n <= 0 || n > g->n_seqs || !seqs || !pos || !q || !k || !v || !out) return PL_EARG;
  if (layer < 0 || layer >= g->n_layers) return PL_EARG;
  int max_pos = 0;
  for (int i = 0; i < n; ++i) {
    if (seqs[i] < 0 || seqs[i] >= g->n_seqs || pos[i] < 0 || pos[i] >= g->max_seq)
      return PL_EARG;
    for (int j = 0; j < i; ++j)
      if (seqs[j] == seqs[i]) return PL_EARG;
    if (pos[i] > max_pos) max_pos = pos[i];
  }
  if (cudaSetDevice(g->device) != cudaSuccess) return PL_ECUDA;
  if (n == 1) return decode_one_host(layer, seqs[0], pos[0], q, k, v, out);
  const size_t qb = static_cast<size_t>(n) * g->q_dim * sizeof(float);
  const size_t kb = static_cast<size_t>(n) * g->kv_dim * sizeof(float);
  const size_t ib = static_cast<size_t>(n) * sizeof(int);
  const size_t in_bytes = qb + 2 * kb + 2 * ib;
  const size_t out_off = (in_bytes + 255) & ~static_cast<size_t>(255);
  const size_t total = out_off + qb + 256;
  int rc = ensure_stage(total);
  if (rc) return rc;
  uint8_t* h = g->h_stage;
  uint8_t* d = g->d_stage;
  // k and v are read once, by the segment that appends: from registered
  // buffers the kernel reads them over the bus.  q is read by every segment
  // of its sequence, so it goes to the device once: straight from a
  // registered q when it is large, else through the staging area with the
  // slots and positions (one copy).
  const uint8_t* mk = mapped(k, kb);
  const uint8_t* mv = mapped(v, kb);
  const bool kv_mapped = mk && mv;
  const bool q_direct = qb > kStagedQBytes && pinned(q, qb);
  CopyPiece in[3];
  int n_in = 0;
  if (!q_direct) in[n_in++] = {h, reinterpret_cast<const uint8_t*>(q), qb};
  if (!kv_mapped) {
    in[n_in++] = {h + qb, reinterpret_cast<const uint8_t*>(k), kb};
    in[n_in++] = {h + qb + kb, reinterpret_cast<const uint8_t*>(v), kb};
  }
  if (n_in) host_copy(in, n_in);
  // up to kInlineSeqs sequences carry their slots and positions in the
  // kernel arguments; more are staged and copied with the rest
  const bool sp_inline = n <= pl::kInlineSeqs;
  if (!sp_inline) {
    std::memcpy(h + qb + 2 * kb, seqs, ib);
    std::memcpy(h + qb + 2 * kb + ib, pos, ib);
  }
  if (q_direct) {
    // q from the caller; then the staged rest, if any: k and v (unless
    // mapped), slots and positions (unless inline).  Every copy costs
    // several microseconds of the GPU's timeline, so none is queued for
    // nothing.
    const size_t rest = kv_mapped ? qb + 2 * kb : qb;
    const size_t rest_end = sp_inline ? qb + 2 * kb : in_bytes;
    // q read over the bus by every SM into HBM (a kernel: the decode grid
    // queues behind it with programmatic dependent launch), else copied
    const uint8_t* mq = mapped(q, qb);
    if (mq) {
      pl::bus_gather_kernel<<<g->num_sms, 256, 0, g->stream>>>(
          reinterpret_cast<const uint4*>(mq), reinterpret_cast<uint4*>(d),
          static_cast<long>(qb / 16));
      PL_CUDA(cudaGetLastError());
      count_launch();
    } else {
      PL_CUDA(cudaMemcpyAsync(d, q, qb, cudaMemcpyHostToDevice, g->stream));
    }
    if (rest_end > rest)
      PL_CUDA(cudaMemcpyAsync(d + rest, h + rest, rest_end - rest, cudaMemcpyHostToDevice,
                              g->stream));
  } else {
    PL_CUDA(cudaMemcpyAsync(d, h, in_bytes, cudaMemcpyHostToDevice, g->stream));
  }
  // the kernels write the output straight into host memory (mapped): the
  // caller's registered out, else the staging area; and the call's last
  // kernel stores the device error word in mapped pinned memory.  No copy
  // comes back.
  *reinterpret_cast<volatile uint32_t*>(g->h_err) = 0;
  uint8_t* mo = mapped(out, qb);
  float* d_out = reinterpret_cast<float*>(mo ? mo : g->h_stage_dev + out_off);
  rc = launch_decode(layer, n, reinterpret_cast<int*>(d + qb + 2 * kb),
                     reinterpret_cast<int*>(d + qb + 2 * kb + ib), max_pos + 1,
                     reinterpret_cast<float*>(d),
                     kv_mapped ? reinterpret_cast<const float*>(mk)
                               : reinterpret_cast<const float*>(d + qb),
                     kv_mapped ? reinterpret_cast<const float*>(mv)
                               : reinterpret_cast<const float*>(d + qb + kb),
                     d_out, 0, 0, 0, 1, nullptr, g->stream, g->h_err_dev,
                     sp_inline ? seqs : nullptr, sp_inline ? pos : nullptr);
  if (rc) return rc;
  PL_CUDA(cudaStreamSynchronize(g->stream));
  const uint32_t w = *reinterpret_cast<volatile uint32_t*>(g->h_err);
  if (w) {
    cudaMemsetAsync(g->d_err, 0, sizeof(uint32_t), g->stream);
    cudaStreamSynchronize(g->stream);
    return check_err_word(w);
  }
  if (!mo) {
    const CopyPiece o = {reinterpret_cast<uint8_t*>(out), h + out_off, qb};
    host_copy(&o, 1);
  }
  return PL_OK;
}

int pl_attn_decode(int seq, int layer, int pos, const float* q, const float* k, const float* v,
                   float* out) {
  return pl_attn_decode_batch(layer, 1, &seq, &pos, q, k, v, out);
}

int pl_attn_host_register(void* ptr, size_t bytes) {
  if (!g) return PL_ESTATE;
  if (!ptr || bytes == 0) return PL_EARG;
  const uintptr_t a = reinterpret_cast<uintptr_t>(ptr);
  for (const HostRange& r : g_pinned)
    if (a < r.hi && a + bytes > r.lo) return PL_EARG;  // overlaps a registered range
  if (cudaSetDevice(g->device) != cudaSuccess) return PL_ECUDA;
  // portable: pinned for every device of a multi-device context; mapped:
  // addressable by the kernels of a host-buffer call
  cudaError_t e = cudaHostRegister(ptr, bytes, cudaHostRegisterPortable | cudaHostRegisterMapped);
  void* dev = nullptr;
  if (e == cudaSuccess) {
    e = cudaHostGetDevicePointer(&dev, ptr, 0);
    if (e != cudaSuccess) cudaHostUnregister(ptr);
  }
  if (e != cudaSuccess) {
    cudaGetLastError();  // the call stays usable through the staging area
    std::fprintf(stderr, "pl_attn_host_register: %s\n", cudaGetErrorString(e));
    return PL_ECUDA;
  }
  g_pinned.push_back({a, a + bytes, static_cast<uint8_t*>(dev)});
  return PL_OK;
}

int pl_attn_host_unregister(void* ptr) {
  if (!g) return PL_ESTATE;
  const uintptr_t a = reinterpret_cast<uintptr_t>(ptr);
  for (size_t i = 0; i < g_pinned.size(); ++i)
    if (g_pinned[i].lo == a) {
      PL_CUDA(cudaStreamSynchronize(g->stream));
      const cudaError_t e = cudaHostUnregister(ptr);
      g_pinned.erase(g_pinned.begin() + static_cast<long>(i));
      if (e != cudaSuccess) {
        cudaGetLastError();
        return PL_ECUDA;
      }
      return PL_OK;
    }
  return PL_EARG;
}

int pl_attn_decode_batch_dev(int layer, int n, const int* d_seqs, const int* d_pos, int max_pos,
                             const float* d_q, const float* d_k, const float* d_v, float* d_out,
                             void* stream) {
  if (!g) return PL_ESTATE;
  if (g_multi) return PL_EUNSUPPORTED;
  if (n <= 0 || n > g->n_seqs || layer < 0 || layer >= g->n_layers || max_pos < 0 ||
      max_pos >= g->max_seq)
    return PL_EARG;
  if (!d_seqs || !d_pos || !d_q || !d_k || !d_v || !d_out) return PL_EARG;
  return launch_decode(layer, n, d_seqs, d_pos, max_pos + 1, d_q, d_k, d_v, d_out, 0, 0, 0, 1,
                       nullptr, pick_stream(stream));
}

int pl_attn_decode_partial_dev(int seq, int layer, int pos, int row0, int n_rows, int append,
                               const float* d_q, const float* d_k, const float* d_v,
                               float* d_part, void* stream) {
  int rc = check_seq_layer(seq, layer);
  if (rc) return rc;
  if (g_multi) return PL_EUNSUPPORTED;
  if (pos < 0 || row0 < 0 || n_rows < 0 || n_rows > g->max_seq || !d_q || !d_part) return PL_EARG;
  if (append && (pos - row0 < 0 || pos - row0 >= n_rows || !d_k || !d_v)) return PL_EARG;
  // the RoPE table must cover the global position
  if (pos >= g->rope_rows) return PL_EARG;
  cudaStream_t st = pick_stream(stream);
  if (n_rows == 0) {
    // an empty shard contributes nothing: m = -inf, l = 0, o = 0
    const int ps = part_stride(g->head_dim);
    std::vector<float> empty(static_cast<size_t>(g->part_floats), 0.f);
    for (int h = 0; h < g->n_heads; ++h) empty[static_cast<size_t>(h) * ps] = -INFINITY;
    PL_CUDA(cudaMemcpyAsync(d_part, empty.data(), empty.size() * sizeof(float),
                            cudaMemcpyHostToDevice, st));
    return PL_OK;
  }
  return partial_launch(seq, layer, pos, row0, n_rows, append, d_q, d_k, d_v, d_part, st);
}

int pl_attn_combine_dev(int n_part, const float* d_parts, float* d_out, void* stream) {
  if (!g) return PL_ESTATE;
  if (g_multi) return PL_EUNSUPPORTED;
  if (n_part <= 0 || !d_parts || !d_out) return PL_EARG;
  if (n_part > pl::kMaxCombineParts) return PL_EARG;
  cudaStream_t st = pick_stream(stream);
  const size_t smem = static_cast<size_t>(3 * pl::kMaxCombineParts + 2) * g->n_heads * sizeof(float);
  if (g->head_dim == 128)
    pl::combine_kernel<128><<<1, 256, smem, st>>>(n_part, g->n_heads, d_parts, d_out);
  else
    pl::combine_kernel<64><<<1, 256, smem, st>>>(n_part, g->n_heads, d_parts, d_out);
  PL_CUDA(cudaGetLastError());
  count_launch();
  return PL_OK;
}

// ------------------------------------------------ KV-split exchange (P2P)
int pl_attn_xfer_handle_bytes(void) { return static_cast<int>(sizeof(cudaIpcMemHandle_t)); }

int pl_attn_xfer_setup(int world, int rank, void* handle_out) {
  if (!g) return PL_ESTATE;
  if (g_multi) return PL_EUNSUPPORTED;
  if (g_xfer) return PL_ESTATE;
  if (world < 1 || world > pl::kXferMaxRanks || rank < 0 || rank >= world || !handle_out)
    return PL_EARG;
  if (cudaSetDevice(g->device) != cudaSuccess) return PL_ECUDA;
  const size_t bytes = pl::xfer_buffer_bytes(world, g->n_heads, g->head_dim);
  Xfer* x = new Xfer;
  x->world = world;
  x->rank = rank;
  if (dev_alloc(&x->local, bytes) != cudaSuccess ||
      dev_alloc(&x->d_arrive, sizeof(uint32_t)) != cudaSuccess ||
      dev_alloc(&x->d_part1, g->part_floats * sizeof(float)) != cudaSuccess) {
    cudaFree(x->local);
    cudaFree(x->d_arrive);
    cudaFree(x->d_part1);
    delete x;
    return PL_ENOMEM;
  }
  if (cudaMemset(x->d_arrive, 0, sizeof(uint32_t)) != cudaSuccess ||
      cudaMemset(x->local, 0, bytes) != cudaSuccess ||
      cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle_out), x->local) != cudaSuccess) {
    cudaFree(x->local);
    cudaFree(x->d_arrive);
    cudaFree(x->d_part1);
    delete x;
    return PL_ECUDA;
  }
  x->peers.base[rank] = x->local;
  g_xfer = x;
  return PL_OK;
}

int pl_attn_xfer_connect(const void* handles) {
  if (!g || !g_xfer) return PL_ESTATE;
  if (g_multi) return PL_EUNSUPPORTED;
  if (!handles) return PL_EARG;
  if (cudaSetDevice(g->device) != cudaSuccess) return PL_ECUDA;
  const auto* h = static_cast<const cudaIpcMemHandle_t*>(handles);
  for (int r = 0; r < g_xfer->world; ++r) {
    if (r == g_xfer->rank || g_xfer->opened[r]) continue;
    void* p = nullptr;
    if (cudaIpcOpenMemHandle(&p, h[r], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
      return PL_ECUDA;
    g_xfer->opened[r] = p;
    g_xfer->peers.base[r] = static_cast<uint8_t*>(p);
  }
  return PL_OK;
}

int pl_attn_combine_p2p_dev(const float* d_part, float* d_out, void* stream) {
  if (!g || !g_xfer) return PL_ESTATE;
  if (g_multi) return PL_EUNSUPPORTED;
  if (!d_part || !d_out) return PL_EARG;
  for (int r = 0; r < g_xfer->world; ++r)
    if (!g_xfer->peers.base[r]) return PL_ESTATE;  // not connected yet
  cudaStream_t st = pick_stream(stream);
  // queued behind the partial's kernels (programmatic dependent launch)
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(pl::kXferThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (g->head_dim == 128)
    PL_CUDA(cudaLaunchKernelEx(&cfg, pl::combine_p2p_kernel<128>, d_part, g_xfer->peers,
                               g_xfer->world, g_xfer->rank, g->n_heads, d_out, g->d_err));
  else
    PL_CUDA(cudaLaunchKernelEx(&cfg, pl::combine_p2p_kernel<64>, d_part, g_xfer->peers,
                               g_xfer->world, g_xfer->rank, g->n_heads, d_out, g->d_err));
  count_launch();
  return PL_OK;
}

int pl_attn_decode_p2p_dev(int seq, int layer, int pos, int row0, int n_rows, int append,
                           const float* d_q, const float* d_k, const float* d_v, float* d_out,
                           void* stream) {
  int rc = check_seq_layer(seq, layer);
  if (rc) return rc;
  if (g_multi) return PL_EUNSUPPORTED;
  if (!g_xfer) return PL_ESTATE;
  for (int r = 0; r < g_xfer->world; ++r)
    if (!g_xfer->peers.base[r]) return PL_ESTATE;  // not connected yet
  if (pos < 0 || row0 < 0 || n_rows < 0 || n_rows > g->max_seq || !d_q || !d_out) return PL_EARG;
  if (append && (pos - row0 < 0 || pos - row0 >= n_rows || !d_k || !d_v)) return PL_EARG;
  if (pos >= g->rope_rows) return PL_EARG;
  cudaStream_t st = pick_stream(stream);
  const pl::XferPush push = {g_xfer->peers, g_xfer->world, g_xfer->rank, g_xfer->d_arrive, d_out};
  const int grid = n_rows ? decode_grid(1, n_rows) : 0;
  if (grid) {
    rc = ensure_part(static_cast<size_t>(grid + 1) * g->part_floats);
    if (rc) return rc;
  }
  pl::DecodeArgs a = decode_args(layer, 1, nullptr, nullptr, d_q, d_k ? d_k : d_q,
                                 d_v ? d_v : d_q, nullptr, 1, row0, n_rows, append ? 1 : 0,
                                 g_xfer->d_part1, g->d_part, g->d_seg_info);
  a.seq1 = seq;
  a.pos1 = pos;
  // an empty shard runs only the merge grid, which pushes an empty partial
  if (!grid) return launch_merge(a, 0, st, true, &push);
  return launch_decode_kernel(a, grid, st, true, &push);
}

int pl_attn_rope(int pos0, int n_tok, float* q, float* k) {
  if (!g) return PL_ESTATE;
  if (n_tok <= 0 || pos0 < 0 || pos0 + n_tok > g->rope_rows || (!q && !k)) return PL_EARG;
  if (cudaSetDevice(g->device) != cudaSuccess) return PL_ECUDA;
  const size_t qb = q ? static_cast<size_t>(n_tok) * g->q_dim * sizeof(float) : 0;
  const size_t kb = k ? static_cast<size_t>(n_tok) * g->kv_dim * sizeof(float) : 0;
  int rc = ensure_stage(qb + kb + 256);
  if (rc) return rc;
  if (q) std::memcpy(g->h_stage, q, qb);
  if (k) std::memcpy(g->h_stage + qb, k, kb);
  PL_CUDA(cudaMemcpyAsync(g->d_stage, g->h_stage, qb + kb, cudaMemcpyHostToDevice, g->stream));
  float* dq = q ? reinterpret_cast<float*>(g->d_stage) : nullptr;
  float* dk = k ? reinterpret_cast<float*>(g->d_stage + qb) : nullptr;
  const dim3 rgrid(n_tok, (g->n_heads + g->n_kv_heads + 7) / 8);
  if (g->head_dim == 128)
    pl::rope_inplace_kernel<128><<<rgrid, 256, 0, g->stream>>>(
        dq, dk, g->n_heads, g->n_kv_heads, pos0, g->d_cos, g->d_sin, g->rope_type);
  else
    pl::rope_inplace_kernel<64><<<rgrid, 256, 0, g->stream>>>(
        dq, dk, g->n_heads, g->n_kv_heads, pos0, g->d_cos, g->d_sin, g->rope_type);
  PL_CUDA(cudaGetLastError());
  PL_CUDA(cudaMemcpyAsync(g->h_stage, g->d_stage, qb + kb, cudaMemcpyDeviceToHost, g->stream));
  PL_CUDA(cudaStreamSynchronize(g->stream));
  if (q) std::memcpy(q, g->h_stage, qb);
  if (k) std::memcpy(k, g->h_stage + qb, kb);
  return PL_OK;
}

int pl_kv_download(int seq, int layer, int pos0, int n_pos, uint16_t* k, uint16_t* v) {
  if (g_multi) return multi_kv_copy(seq, layer, pos0, n_pos, k, v, true);
  int rc = check_seq_layer(seq, layer);
  if (rc) return rc;
  if (pos0 < 0 || n_pos < 0 || pos0 + n_pos > g->max_seq) return PL_EARG;
  if (n_pos == 0) return PL_OK;
  const size_t off = static_cast<size_t>(pos0) * g->kv_dim;
  const size_t bytes = static_cast<size_t>(n_pos) * g->kv_dim * 2;
  if (k) PL_CUDA(cudaMemcpyAsync(k, slab_k(seq, layer) + off, bytes, cudaMemcpyDeviceToHost,
                                 g->stream));
  if (v) PL_CUDA(cudaMemcpyAsync(v, slab_v(seq, layer) + off, bytes, cudaMemcpyDeviceToHost,
                                 g->stream));
  PL_CUDA(cudaStreamSynchronize(g->stream));
  return PL_OK;
}

int pl_kv_upload(int seq, int layer, int pos0, int n_pos, const uint16_t* k, const uint16_t* v) {
  if (g_multi)
    return multi_kv_copy(seq, layer, pos0, n_pos, const_cast<uint16_t*>(k),
                         const_cast<uint16_t*>(v), false);
  int rc = check_seq_layer(seq, layer);
  if (rc) return rc;
  if (pos0 < 0 || n_pos < 0 || pos0 + n_pos > g->max_seq) return PL_EARG;
  if (n_pos == 0) return PL_OK;
  const size_t off = static_cast<size_t>(pos0) * g->kv_dim;
  const size_t bytes = static_cast<size_t>(n_pos) * g->kv_dim * 2;
  if (k) PL_CUDA(cudaMemcpyAsync(slab_k(seq, layer) + off, k, bytes, cudaMemcpyHostToDevice,
                                 g->stream));
  if (v) PL_CUDA(cudaMemcpyAsync(slab_v(seq, layer) + off, v, bytes, cudaMemcpyHostToDevice,
                                 g->stream));
  PL_CUDA(cudaStreamSynchronize(g->stream));
  return PL_OK;
}

int pl_attn_kv_ptr(int seq, int layer, uint16_t** d_k, uint16_t** d_v) {
  int rc = check_seq_layer(seq, layer);
  if (rc) return rc;
  if (g_multi) return PL_EUNSUPPORTED;
  if (d_k) *d_k = slab_k(seq, layer);
  if (d_v) *d_v = slab_v(seq, layer);
  return PL_OK;
}

// ---------------------------------------------------------------- prefill

// Prologue + tensor-core attention over the rows of one cache slab: kc_slab /
// vc_slab are its row 0 (the prologue appends at row start_pos), tmk / tmv
// and `slab` address it for the attention kernel's TMA loads.
static int launch_prefill_rows(uint16_t* kc_slab, uint16_t* vc_slab, const CUtensorMap& tmk,
                               const CUtensorMap& tmv, int slab, int start_pos, int n_tok,
                               const float* d_q, const float* d_k, const float* d_v,
                               float* d_out, int out_stride, cudaStream_t st) {
  int rc = ensure_q16(n_tok);
  if (rc) return rc;
  const size_t off = static_cast<size_t>(start_pos) * g->kv_dim;
  const int pgrid =
      pl::prologue_grid(n_tok, g->n_heads, g->n_kv_heads, g->head_dim, true, g->num_sms);
  if (g->head_dim == 128)
    pl::prefill_prologue_kernel<128><<<pgrid, pl::kPrologueThreads, 0, st>>>(
        d_q, d_k, d_v, g->d_q16, static_cast<long>(g->q16_cap), kc_slab + off, vc_slab + off,
        n_tok, g->n_heads, g->n_kv_heads, start_pos, g->d_cos, g->d_sin, g->rope_type);
  else
    pl::prefill_prologue_kernel<64><<<pgrid, pl::kPrologueThreads, 0, st>>>(
        d_q, d_k, d_v, g->d_q16, static_cast<long>(g->q16_cap), kc_slab + off, vc_slab + off,
        n_tok, g->n_heads, g->n_kv_heads, start_pos, g->d_cos, g->d_sin, g->rope_type);
  PL_CUDA(cudaGetLastError());
  count_launch();
  pl::PrefillArgs a;
  a.q16 = g->d_q16;
  a.out = d_out;
  a.out_stride = out_stride;
  a.n_tok = n_tok;
  a.start_pos = start_pos;
  a.n_heads = g->n_heads;
  a.kv_mul = g->kv_mul;
  a.slab = slab;
  a.score_scale = pl::kLog2e / sqrtf(static_cast<float>(g->head_dim));
  a.work = g->d_work;
  a.err = g->d_err;
  CUtensorMap tm_o;
  std::memset(&tm_o, 0, sizeof(tm_o));
  a.o_tma = g->head_dim == 64 &&
            make_out_map(g->encode, &tm_o, d_out, g->q_dim, n_tok, out_stride) ? 1 : 0;
  prof_begin(st);
  // overlap with the prologue except when events separate the two for timing
  if (pl::launch_prefill_attention(g->head_dim, a, g->tm_q16, g->tm_q16lo, tmk, tmv, tm_o,
                                   g->num_sms, st, !g->profiling) != 0)
    return PL_ECUDA;
  prof_end(st);
  count_launch();
  return PL_OK;
}

static int launch_prefill(int seq, int layer, int start_pos, int n_tok, const float* d_q,
                          const float* d_k, const float* d_v, float* d_out, int out_stride,
                          cudaStream_t st) {
  return launch_prefill_rows(slab_k(seq, layer), slab_v(seq, layer), g->tm_k_pf, g->tm_v_pf,
                             seq * g->n_layers + layer, start_pos, n_tok, d_q, d_k, d_v, d_out,
                             out_stride, st);
}

int pl_attn_prefill(int seq, int layer, int start_pos, int n_tok, const float* q, const float* k,
                    const float* v, float* out, int out_stride) {
  if (g_multi) return multi_prefill(seq, layer, start_pos, n_tok, q, k, v, out, out_stride);
  int rc = check_seq_layer(seq, layer);
  if (rc) return rc;
  if (n_tok <= 0 || start_pos < 0 || start_pos + n_tok > g->max_seq || !q || !k || !v || !out ||
      out_stride < g->q_dim)
    return PL_EARG;
  if (cudaSetDevice(g->device) != cudaSuccess) return PL_ECUDA;
  const size_t qb = static_cast<size_t>(n_tok) * g->q_dim * sizeof(float);
  const size_t kb = static_cast<size_t>(n_tok) * g->kv_dim * sizeof(float);
  const size_t in_bytes = qb + 2 * kb;
  const size_t out_off = (in_bytes + 255) & ~static_cast<size_t>(255);
  const size_t total = out_off + qb + 256;
  rc = ensure_stage(total);
  if (rc) return rc;
  uint8_t* h = g->h_stage;
  uint8_t* d = g->d_stage;
  if (pinned(q, qb) && pinned(k, kb) && pinned(v, kb)) {
    PL_CUDA(cudaMemcpyAsync(d, q, qb, cudaMemcpyHostToDevice, g->stream));
    PL_CUDA(cudaMemcpyAsync(d + qb, k, kb, cudaMemcpyHostToDevice, g->stream));
    PL_CUDA(cudaMemcpyAsync(d + qb + kb, v, kb, cudaMemcpyHostToDevice, g->stream));
  } else {
    const CopyPiece in[3] = {{h, reinterpret_cast<const uint8_t*>(q), qb},
                             {h + qb, reinterpret_cast<const uint8_t*>(k), kb},
                             {h + qb + kb, reinterpret_cast<const uint8_t*>(v), kb}};
    host_copy(in, 3);
    PL_CUDA(cudaMemcpyAsync(d, h, in_bytes, cudaMemcpyHostToDevice, g->stream));
  }
  float* d_out = reinterpret_cast<float*>(d + out_off);
  rc = launch_prefill(seq, layer, start_pos, n_tok, reinterpret_cast<float*>(d),
                      reinterpret_cast<float*>(d + qb), reinterpret_cast<float*>(d + qb + kb),
                      d_out, g->q_dim, g->stream);
  if (rc) return rc;
  if (out_stride == g->q_dim) return read_back(d_out, out, qb, h + out_off);
  PL_CUDA(cudaMemcpyAsync(d + out_off + qb, g->d_err, sizeof(uint32_t), cudaMemcpyDeviceToDevice,
                          g->stream));
  PL_CUDA(cudaMemcpyAsync(h + out_off, d + out_off, qb + sizeof(uint32_t), cudaMemcpyDeviceToHost,
                          g->stream));
  rc = finish_host_call(reinterpret_cast<uint32_t*>(h + out_off + qb));
  if (rc) return rc;
  for (int r = 0; r < n_tok; ++r)
    std::memcpy(out + static_cast<size_t>(r) * out_stride,
                h + out_off + static_cast<size_t>(r) * g->q_dim * sizeof(float),
                g->q_dim * sizeof(float));
  return PL_OK;
}

int pl_attn_prefill_dev(int seq, int layer, int start_pos, int n_tok, const float* d_q,
                        const float* d_k, const float* d_v, float* d_out, int out_stride,
                        void* stream) {
  int rc = check_seq_layer(seq, layer);
  if (rc) return rc;
  if (g_multi) return PL_EUNSUPPORTED;
  if (n_tok <= 0 || start_pos < 0 || start_pos + n_tok > g->max_seq || !d_q || !d_k || !d_v ||
      !d_out || out_stride < g->q_dim)
    return PL_EARG;
  // the prologue reads q, k, v and the attention kernel writes out rows in
  // 16-byte vectors
  if (!aligned16(d_q) || !aligned16(d_k) || !aligned16(d_v) || !aligned16(d_out) ||
      out_stride % 4 != 0) {
    std::fprintf(stderr,
                 "pl_attn_prefill_dev: q, k, v and out must be 16-byte aligned and out_stride a "
                 "multiple of 4\n");
    return PL_EARG;
  }
  return launch_prefill(seq, layer, start_pos, n_tok, d_q, d_k, d_v, d_out, out_stride,
                        pick_stream(stream));
}

int pl_attn_set_wait_limit(double seconds) {
  if (!g) return PL_ESTATE;
  if (!(seconds >= 1e-4 && seconds <= 60.0)) return PL_EARG;
  const uint64_t ns = static_cast<uint64_t>(seconds * 1e9);
  if (g_multi) return multi_set_wait_limit(ns);
  if (cudaSetDevice(g->device) != cudaSuccess) return PL_ECUDA;
  PL_CUDA(cudaMemcpyToSymbol(pl::g_wait_limit_ns, &ns, sizeof(ns)));
  return PL_OK;
}

int pl_attn_status(void* stream) {
  if (!g) return PL_ESTATE;
  if (g_multi) return multi_status();
  if (cudaSetDevice(g->device) != cudaSuccess) return PL_ECUDA;
  PL_CUDA(cudaStreamSynchronize(pick_stream(stream)));
  uint32_t w = 0;
  PL_CUDA(cudaMemcpy(&w, g->d_err, sizeof(w), cudaMemcpyDeviceToHost));
  if (w) PL_CUDA(cudaMemset(g->d_err, 0, sizeof(uint32_t)));
  return check_err_word(w);
}

int pl_attn_profile(int enable) {
  if (!g) return PL_ESTATE;
  if (g_multi) {
    multi_profile(enable);
    return PL_OK;
  }
  g->profiling = enable ? 1 : 0;
  g->ev_used = 0;
  g->n_attn = 0;
  g->n_all = 0;
  return PL_OK;
}

int pl_attn_profile_read(double* attn_ms, long* attn_launches, long* all_launches) {
  if (!g) return PL_ESTATE;
  if (g_multi) return multi_profile_read(attn_ms, attn_launches, all_launches);
  double ms = 0.0;
  for (size_t i = 0; i + 1 < g->ev_used; i += 2) {
    PL_CUDA(cudaEventSynchronize(g->ev_pool[i + 1]));
    float t = 0.f;
    PL_CUDA(cudaEventElapsedTime(&t, g->ev_pool[i], g->ev_pool[i + 1]));
    ms += t;
  }
  if (attn_ms) *attn_ms = ms;
  if (attn_launches) *attn_launches = g->n_attn;
  if (all_launches) *all_launches = g->n_all;
  g->ev_used = 0;
  g->n_attn = 0;
  g->n_all = 0;
  return PL_OK;
}

}  // extern "C"

// =====================================================================
// Decode that allocates nothing.
//
// pl_attn_decode_batch_dev may allocate device memory for its split-KV
// partials the first time a launch needs more than it holds.  Some callers
// cannot let a library allocate: serving engines that reserve the whole
// device up front in their own pool (a late cudaMalloc can then fail, or
// fragment that pool), and latency-critical decode loops, where cudaMalloc
// and cudaFree may synchronise the device and stall every other stream.
// pl_attn_decode_batch_dev_noalloc runs the same decode kernel with its
// scratch in one file-scope __device__ array of fixed size instead.
// =====================================================================
namespace {

constexpr int kNoAllocMaxSeqs = pl::kMaxLaunchSeqs;                 // per call
constexpr size_t kNoAllocInfoBytes = static_cast<size_t>(kNoAllocMaxSeqs) * sizeof(int2);  // 8 KiB
constexpr size_t kNoAllocPartBytes = static_cast<size_t>(4) << 20;  // 4 MiB of partials
constexpr size_t kNoAllocScratchBytes = kNoAllocInfoBytes + kNoAllocPartBytes;
constexpr int kNoAllocMaxDevices = 64;

// 4 MiB + 8 KiB, held by every GPU that loads this library until exit.  In
// host code the name is only a host-side stand-in for the symbol: its
// device address comes from cudaGetSymbolAddress, once per device.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

void* g_noalloc_addr[kNoAllocMaxDevices];
std::mutex g_noalloc_mu;

// Device address of g_noalloc_scratch on `device`, which the caller has
// checked is the current device; looked up on the first call for it.
int noalloc_scratch(int device, uint8_t** addr) {
  if (device < 0 || device >= kNoAllocMaxDevices) return PL_EDEVICE;
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_addr[device]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      std::fprintf(stderr, "pl_attn: cudaGetSymbolAddress(scratch) failed: %s\n",
                   cudaGetErrorString(e));
      return PL_ECUDA;
    }
    g_noalloc_addr[device] = p;
  }
  *addr = static_cast<uint8_t*>(g_noalloc_addr[device]);
  return PL_OK;
}

}  // namespace

extern "C" int pl_attn_decode_batch_dev_noalloc(int layer, int n, const int* d_seqs,
                                                const int* d_pos, int max_pos, const float* d_q,
                                                const float* d_k, const float* d_v,
                                                float* d_out, void* stream) {
  if (!g) return PL_ESTATE;
  if (g_multi) return PL_EUNSUPPORTED;
  if (n <= 0 || n > g->n_seqs || layer < 0 || layer >= g->n_layers || max_pos < 0 ||
      max_pos >= g->max_seq)
    return PL_EARG;
  if (!d_seqs || !d_pos || !d_q || !d_k || !d_v || !d_out) return PL_EARG;
  // partial slots needed: one per CTA plus one per sequence
  const size_t slot_bytes = static_cast<size_t>(g->part_floats) * sizeof(float);
  const long long fit = static_cast<long long>(kNoAllocPartBytes / slot_bytes) - n;
  if (n > kNoAllocMaxSeqs || fit < 1) {
    std::fprintf(stderr,
                 "pl_attn_decode_batch_dev_noalloc: %d sequences exceed its fixed scratch "
                 "(at most %d sequences and %zu partial slots of %zu bytes in a static "
                 "%zu-byte device array)\n",
                 n, kNoAllocMaxSeqs, kNoAllocPartBytes / slot_bytes, slot_bytes,
                 kNoAllocScratchBytes);
    return PL_EARG;
  }
  // the kernels run on the caller's current device, with this context's
  // cache pointers: it must be the context's device
  int cur = -1;
  PL_CUDA(cudaGetDevice(&cur));
  if (cur != g->device) {
    std::fprintf(stderr,
                 "pl_attn_decode_batch_dev_noalloc: current device %d is not the module's "
                 "device %d\n", cur, g->device);
    return PL_EDEVICE;
  }
  uint8_t* scratch = nullptr;
  int rc = noalloc_scratch(g->device, &scratch);
  if (rc) return rc;
  int2* seg_info = reinterpret_cast<int2*>(scratch);
  float* part = reinterpret_cast<float*>(scratch + kNoAllocInfoBytes);
  int grid = decode_grid(n, max_pos + 1);
  if (grid > fit) grid = static_cast<int>(fit);  // fewer, longer CTAs when slots run short
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // the array keeps the previous call's contents; every word the kernels
  // read (the segment table, the partial slots of this launch) is written
  // by this launch first, so nothing needs clearing
  const pl::DecodeArgs a = decode_args(layer, n, d_seqs, d_pos, d_q, d_k, d_v, d_out, 0, 0, 0,
                                       1, nullptr, part, seg_info);
  return launch_decode_kernel(a, grid, st, false);
}

// ---- the projections around the attention path ---------------------------
// pl_attn_set_layer keeps one layer's attention weights on the device in
// their GGUF quantisation; the block calls then run model.c's whole
// attention sub-block (model.c:779-897 for decode, 990-1100 for prefill) on
// the device: RMSNorm, Q/K/V projections and biases, QK-norm, RoPE, the FP16
// KV append, attention, the output projection, its bias and the residual
// add, with only the residual stream x crossing PCIe.

namespace {

size_t gguf_row_bytes(int type, int n) {
  // picolm/quant.c:290-320 (block size and bytes per block)
  switch (type) {
    case pl::kGgufF32: return static_cast<size_t>(n) * 4;
    case pl::kGgufF16: return static_cast<size_t>(n) * 2;
    case pl::kGgufQ8_0: return static_cast<size_t>(n / 32) * 34;
    case pl::kGgufQ4K: return static_cast<size_t>(n / 256) * pl::kQ4KBytes;
    case pl::kGgufQ6K: return static_cast<size_t>(n / 256) * pl::kQ6KGgufBytes;
    default: return 0;
  }
}

// `rows` GGUF rows of n inputs -> the device layout of kern_proj.cuh
void repack_rows(int type, const uint8_t* src, int rows, int n, uint8_t* dst) {
  const size_t drb = pl::proj_row_bytes(type, n);
  const size_t srb = gguf_row_bytes(type, n);
  if (type == pl::kGgufF32 || type == pl::kGgufF16 || type == pl::kGgufQ4K) {
    std::memcpy(dst, src, drb * static_cast<size_t>(rows));
    return;
  }
  for (int r = 0; r < rows; ++r) {
    const uint8_t* s = src + static_cast<size_t>(r) * srb;
    uint8_t* d = dst + static_cast<size_t>(r) * drb;
    std::memset(d, 0, drb);
    if (type == pl::kGgufQ8_0) {
      // {d, qs[32]} blocks -> all quants, then all scales
      for (int b = 0; b < n / 32; ++b) {
        std::memcpy(d + static_cast<size_t>(b) * 32, s + static_cast<size_t>(b) * 34 + 2, 32);
        std::memcpy(d + n + static_cast<size_t>(b) * 2, s + static_cast<size_t>(b) * 34, 2);
      }
    } else {  // Q6_K: 210-byte blocks -> 224-byte blocks, same field order
      for (int b = 0; b < n / 256; ++b)
        std::memcpy(d + static_cast<size_t>(b) * pl::kQ6KBytes,
                    s + static_cast<size_t>(b) * pl::kQ6KGgufBytes, pl::kQ6KGgufBytes);
    }
  }
}

int ensure_blk(size_t floats) {
  if (floats <= g->blk_cap) return PL_OK;
  if (g->d_blk) {
    cudaStreamSynchronize(g->stream);
    cudaFree(g->d_blk);
  }
  g->d_blk = nullptr;
  g->blk_cap = 0;
  if (dev_alloc(&g->d_blk, floats * sizeof(float)) != cudaSuccess) return PL_ENOMEM;
  g->blk_cap = floats;
  return PL_OK;
}

// One projection launch.  With 16 or more input rows, Q4_K / Q8_0 / F16
// weights and tile-aligned shapes, proj_mma_kernel (tensor cores; x passes
// as FP16 high part and residual, so |x| must stay below 65504: true of
// RMSNorm outputs and attention outputs, which is why only the block calls
// allow it).  Otherwise proj_kernel: mc (input rows per CTA) as large as the
// staged rows fit in shared memory, at most kProjMaxM; with a few input
// rows a warp takes one output row (most CTAs for a latency-bound GEMV),
// with more, four rows that share its reads of the staged x.
int launch_proj(pl::ProjArgs a, cudaStream_t st, bool allow_mma) {
  bool mma = allow_mma && a.M >= pl::kMmaN && a.n % pl::kMmaKC == 0;
  for (int i = 0; i < a.n_mat; ++i)
    mma = mma && pl::proj_mma_type(a.mat[i].type) && a.mat[i].rows % 16 == 0;
  if (mma) {
    const long long gy = (a.M + pl::kMmaN - 1) / pl::kMmaN;
    if (gy > 65535) return PL_EUNSUPPORTED;
    const int gx = (a.total_rows + pl::kMmaRows - 1) / pl::kMmaRows;
    // a few tiles (batched decode): split the inputs so that about four
    // CTAs per SM run, the slices summed by a second, deterministic kernel
    const long long tiles = gx * gy;
    int ks = static_cast<int>((4LL * g->num_sms + tiles - 1) / tiles);
    if (ks > a.n / pl::kMmaKC) ks = a.n / pl::kMmaKC;
    if (ks < 1) ks = 1;
    a.ksplit = ks;
    a.part = nullptr;
    if (ks > 1) {
      const size_t need = static_cast<size_t>(ks) * a.M * a.total_rows;
      if (need > g->proj_part_cap) {
        if (g->d_proj_part) {
          cudaStreamSynchronize(g->stream);
          cudaFree(g->d_proj_part);
        }
        g->d_proj_part = nullptr;
        g->proj_part_cap = 0;
        if (dev_alloc(&g->d_proj_part, need * sizeof(float)) != cudaSuccess) return PL_ENOMEM;
        g->proj_part_cap = need;
      }
      a.part = g->d_proj_part;
    }
    const dim3 grid(gx, static_cast<unsigned>(gy), ks);
    pl::proj_mma_kernel<<<grid, pl::kMmaThreads, 0, st>>>(a);
    PL_CUDA(cudaGetLastError());
    count_launch();
    if (ks > 1) {
      const size_t n_out = static_cast<size_t>(a.M) * a.total_rows;
      pl::proj_reduce_kernel<<<static_cast<unsigned>((n_out + 255) / 256), 256, 0, st>>>(a);
      PL_CUDA(cudaGetLastError());
      count_launch();
    }
    return PL_OK;
  }
  const size_t row_b = static_cast<size_t>(a.n) * sizeof(float);
  long long mc = pl::kProjSmemCap / static_cast<long long>(row_b);
  if (mc > pl::kProjMaxM) mc = pl::kProjMaxM;
  if (mc > a.M) mc = a.M;
  if (mc < 1) return PL_EUNSUPPORTED;
  a.mc = static_cast<int>(mc);
  const long long gy = (a.M + mc - 1) / mc;
  if (gy > 65535) return PL_EUNSUPPORTED;
  bool by4 = a.M >= 4;
  for (int i = 0; i < a.n_mat; ++i) by4 = by4 && a.mat[i].rows % 4 == 0;
  const int rows_per_cta = pl::kProjWarps * (by4 ? 4 : 1);
  const int gx = (a.total_rows + rows_per_cta - 1) / rows_per_cta;
  if (!g->proj_smem_set) {
    PL_CUDA(cudaFuncSetAttribute(pl::proj_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 pl::kProjSmemCap));
    PL_CUDA(cudaFuncSetAttribute(pl::proj_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 pl::kProjSmemCap));
    g->proj_smem_set = true;
  }
  const dim3 grid(gx, static_cast<unsigned>(gy));
  if (by4)
    pl::proj_kernel<4><<<grid, pl::kProjThreads, mc * row_b, st>>>(a);
  else
    pl::proj_kernel<1><<<grid, pl::kProjThreads, mc * row_b, st>>>(a);
  PL_CUDA(cudaGetLastError());
  count_launch();
  return PL_OK;
}

// the activations of one block call in d_blk: q [rows][q_dim], k and v
// [rows][kv_dim], attention output [rows][q_dim] (all 16-byte aligned)
struct BlkBufs {
  float *q, *k, *v, *att;
};
int blk_bufs(int rows, BlkBufs* b) {
  const size_t r = static_cast<size_t>(rows);
  const int rc = ensure_blk(r * (2 * static_cast<size_t>(g->q_dim) + 2 * g->kv_dim));
  if (rc) return rc;
  b->q = g->d_blk;
  b->k = b->q + r * g->q_dim;
  b->v = b->k + r * g->kv_dim;
  b->att = b->v + r * g->kv_dim;
  return PL_OK;
}

pl::ProjMat proj_mat(const LayerW& L, int which, float* out, int ld_out) {
  pl::ProjMat m;
  m.w = L.w[which];
  m.bias = L.bias[which];
  m.out = out;
  m.row_bytes = L.row_bytes[which];
  m.type = L.type[which];
  m.rows = which == 0 ? g->q_dim : (which == 3 ? L.dim : g->kv_dim);
  m.ld_out = ld_out;
  return m;
}

// ---- tensor-core GEMM of many input rows (kern_gemm.cuh) -------------------
// A row-major FP16 matrix [rows][k] as a 2-D TMA map, box 64 x 128 under the
// 128-byte swizzle.
int make_map_2d(CUtensorMap* m, const __half* base, int k, int rows, int box_rows = pl::kGmBM) {
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(k) * 2};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(pl::kGmBK), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  if (g->encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(base), dims, strides,
                box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return PL_ECUDA;
  return PL_OK;
}

// The layer's weights as the GEMM's FP16 high parts and scaled residuals,
// dequantised on the device from the uploaded rows.  Layers whose shapes do
// not tile (q_dim, kv_dim, dim multiples of 128), or with a weight beyond
// FP16's range, keep the CUDA-core / mma.sync paths for every row count.
int gemm_prepare_layer(LayerW& L) {
  L.gemm = false;
  const int dim = L.dim, qd = g->q_dim, kvd = g->kv_dim;
  if (dim % pl::kGmBN || qd % pl::kGmBN || kvd % pl::kGmBN) return PL_OK;
  const size_t n_qkv = static_cast<size_t>(qd + 2 * kvd) * dim, n_o = static_cast<size_t>(dim) * qd;
  const size_t bytes = 2 * (n_qkv + n_o) * sizeof(__half);
  if (dev_alloc(&L.gmem, bytes) != cudaSuccess) return PL_ENOMEM;
  __half* qkv_h = reinterpret_cast<__half*>(L.gmem);
  __half* qkv_l = qkv_h + n_qkv;
  __half* o_h = qkv_l + n_qkv;
  __half* o_l = o_h + n_o;
  int* d_over = nullptr;
  if (dev_alloc(&d_over, sizeof(int)) != cudaSuccess) return PL_ENOMEM;
  PL_CUDA(cudaMemsetAsync(d_over, 0, sizeof(int), g->stream));
  const int rows[4] = {qd, kvd, kvd, dim};
  const int row0[4] = {0, qd, qd + kvd, 0};
  for (int i = 0; i < 4; ++i) {
    const int n_in = i == 3 ? qd : dim;
    const long total = static_cast<long>(rows[i]) * n_in;
    const int blocks = static_cast<int>((total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096);
    pl::dequant_split_kernel<<<blocks, 256, 0, g->stream>>>(
        L.w[i], L.row_bytes[i], L.type[i], rows[i], n_in, i == 3 ? o_h : qkv_h,
        i == 3 ? o_l : qkv_l, row0[i], d_over);
  }
  PL_CUDA(cudaGetLastError());
  int over = 0;
  PL_CUDA(cudaMemcpyAsync(&over, d_over, sizeof(int), cudaMemcpyDeviceToHost, g->stream));
  PL_CUDA(cudaStreamSynchronize(g->stream));
  cudaFree(d_over);
  if (over) {
    cudaFree(L.gmem);
    L.gmem = nullptr;
    return PL_OK;
  }
  // the parts are tiled (pl::wtile_row): a [blocks * 128][64] view, one
  // 128 x 64 tile per box
  const int qkv_rows = static_cast<int>(n_qkv / pl::kGmBK), o_rows = static_cast<int>(n_o / pl::kGmBK);
  int rc = make_map_2d(&L.tm_qkv_h, qkv_h, pl::kGmBK, qkv_rows);
  if (!rc) rc = make_map_2d(&L.tm_qkv_l, qkv_l, pl::kGmBK, qkv_rows);
  if (!rc) rc = make_map_2d(&L.tm_o_h, o_h, pl::kGmBK, o_rows);
  if (!rc) rc = make_map_2d(&L.tm_o_l, o_l, pl::kGmBK, o_rows);
  if (rc) return rc;
  L.gemm = true;
  return PL_OK;
}

int ensure_act(size_t elems) {
  if (elems <= g->act_cap) return PL_OK;
  size_t cap = g->act_cap ? g->act_cap : (static_cast<size_t>(1) << 20);
  while (cap < elems) cap *= 2;
  if (g->d_xh) {
    cudaStreamSynchronize(g->stream);
    cudaFree(g->d_xh);
    cudaFree(g->d_xl);
  }
  g->d_xh = g->d_xl = nullptr;
  g->act_cap = 0;
  if (dev_alloc(&g->d_xh, cap * sizeof(__half)) != cudaSuccess ||
      dev_alloc(&g->d_xl, cap * sizeof(__half)) != cudaSuccess)
    return PL_ENOMEM;
  g->act_cap = cap;
  return PL_OK;
}

// x [M][ldx] (RMSNorm with norm_w first, if set) -> y = x W^T over weight
// rows [w_row0, w_row0 + N) of the layer's Q/K/V (qkv) or O matrices, routed
// to the output segments; resid (may equal seg 0's out) added when set.
int launch_gemm(const LayerW& L, bool qkv, const float* d_x, int ldx, int M, int K,
                const float* norm_w, float eps, int w_row0, int N, const pl::GemmSeg* segs,
                int n_seg, const float* resid, int ld_res, cudaStream_t st) {
  int rc = ensure_act(static_cast<size_t>(M) * K);
  if (rc) return rc;
  pl::act_split_kernel<<<M, 256, 0, st>>>(d_x, ldx, K, norm_w, eps, g->d_xh, g->d_xl);
  PL_CUDA(cudaGetLastError());
  count_launch();
  CUtensorMap tm_xh, tm_xl;
  const int box_rows = M <= pl::kSkMaxRows ? pl::kSkMaxRows : pl::kGmBM;
  if ((rc = make_map_2d(&tm_xh, g->d_xh, K, M, box_rows)) ||
      (rc = make_map_2d(&tm_xl, g->d_xl, K, M, box_rows)))
    return rc;
  if (!g->gemm_smem_set) {
    PL_CUDA(cudaFuncSetAttribute(pl::gemm_hilo_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 pl::gm_smem_bytes()));
    PL_CUDA(cudaFuncSetAttribute(pl::gemm_skinny_kernel,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, pl::sk_smem_bytes()));
    g->gemm_smem_set = true;
  }
  pl::GemmArgs a = {};
  a.M = M;
  a.N = N;
  a.K = K;
  a.w_row0 = w_row0;
  for (int i = 0; i < n_seg; ++i) a.seg[i] = segs[i];
  a.n_seg = n_seg;
  a.resid = resid;
  a.ld_res = ld_res;
  a.err = g->d_err;
  if (M <= pl::kSkMaxRows) {
    // few rows: the weights are the A operand, 128 output columns per tile,
    // K split over a cluster of S CTAs per tile: the largest S (at most 8,
    // at least two k-steps per CTA) whose clusters all fit on the GPU at
    // once, from the occupancy the driver reports for each cluster size
    const int tiles = N / pl::kGmBM, kb_all = K / pl::kGmBK;
    if (!g->sk_clusters[1]) {
      g->sk_clusters[1] = g->num_sms;
      for (int sz = 2; sz <= pl::kSkMaxSplit; ++sz) {
        cudaLaunchConfig_t q = {};
        q.gridDim = dim3(1, sz);
        q.blockDim = dim3(pl::kGmThreads);
        q.dynamicSmemBytes = pl::sk_smem_bytes();
        cudaLaunchAttribute ca[1];
        ca[0].id = cudaLaunchAttributeClusterDimension;
        ca[0].val.clusterDim.x = 1;
        ca[0].val.clusterDim.y = sz;
        ca[0].val.clusterDim.z = 1;
        q.attrs = ca;
        q.numAttrs = 1;
        int n_cl = 0;
        if (cudaOccupancyMaxActiveClusters(&n_cl, pl::gemm_skinny_kernel, &q) != cudaSuccess) {
          cudaGetLastError();
          n_cl = 0;
        }
        g->sk_clusters[sz] = n_cl;
      }
    }
    int split = 1;
    for (int sz = 2; sz <= pl::kSkMaxSplit && sz <= kb_all / 2; ++sz)
      if (tiles <= g->sk_clusters[sz]) split = sz;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(tiles, split);
    cfg.blockDim = dim3(pl::kGmThreads);
    cfg.dynamicSmemBytes = pl::sk_smem_bytes();
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;  // behind act_split_kernel
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 1;
    attr[1].val.clusterDim.y = split;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = split > 1 ? 2 : 1;
    PL_CUDA(cudaLaunchKernelEx(&cfg, pl::gemm_skinny_kernel, a, tm_xh, tm_xl,
                               qkv ? L.tm_qkv_h : L.tm_o_h, qkv ? L.tm_qkv_l : L.tm_o_l));
    count_launch();
    return PL_OK;
  }
  const dim3 grid(N / pl::kGmBN, (M + pl::kGmBM - 1) / pl::kGmBM);
  pl::gemm_hilo_kernel<<<grid, pl::kGmThreads, pl::gm_smem_bytes(), st>>>(
      a, tm_xh, tm_xl, qkv ? L.tm_qkv_h : L.tm_o_h, qkv ? L.tm_qkv_l : L.tm_o_l);
  PL_CUDA(cudaGetLastError());
  count_launch();
  return PL_OK;
}

// rmsnorm + Q, K, V projections + biases of M rows of x [M][dim]
int run_qkv(const LayerW& L, const float* d_x, int M, const BlkBufs& b, cudaStream_t st) {
  pl::ProjArgs a = {};
  a.mat[0] = proj_mat(L, 0, b.q, g->q_dim);
  a.mat[1] = proj_mat(L, 1, b.k, g->kv_dim);
  a.mat[2] = proj_mat(L, 2, b.v, g->kv_dim);
  a.n_mat = 3;
  a.total_rows = g->q_dim + 2 * g->kv_dim;
  a.x = d_x;
  a.ldx = L.dim;
  a.n = L.dim;
  a.M = M;
  a.norm_w = L.attn_norm;
  a.eps = L.eps;
  int rc;
  if (L.gemm && M >= pl::kGmMinRows) {
    // many rows: the tensor-core GEMM over the concatenated Q, K, V rows
    const pl::GemmSeg segs[3] = {{b.q, L.bias[0], 0, g->q_dim, g->q_dim},
                                 {b.k, L.bias[1], g->q_dim, g->kv_dim, g->kv_dim},
                                 {b.v, L.bias[2], g->q_dim + g->kv_dim, g->kv_dim, g->kv_dim}};
    rc = launch_gemm(L, true, d_x, L.dim, M, L.dim, L.attn_norm, L.eps, 0,
                     g->q_dim + 2 * g->kv_dim, segs, 3, nullptr, 0, st);
  } else {
    rc = launch_proj(a, st, true);
  }
  if (rc || !L.q_norm) return rc;
  const dim3 grid(static_cast<unsigned>(M), (g->n_heads + g->n_kv_heads + 7) / 8);
  pl::qk_norm_kernel<<<grid, 256, 0, st>>>(b.q, b.k, g->n_heads, g->n_kv_heads, g->head_dim,
                                           L.q_norm, L.k_norm, L.eps);
  PL_CUDA(cudaGetLastError());
  count_launch();
  return PL_OK;
}

// x [M][dim] += Wo att + bo
int run_out(const LayerW& L, const float* d_att, int M, float* d_x, cudaStream_t st) {
  pl::ProjArgs a = {};
  a.mat[0] = proj_mat(L, 3, d_x, L.dim);
  a.n_mat = 1;
  a.total_rows = L.dim;
  a.x = d_att;
  a.ldx = g->q_dim;
  a.n = g->q_dim;
  a.M = M;
  a.resid = d_x;
  a.ld_res = L.dim;
  if (L.gemm && M >= pl::kGmMinRows) {
    const pl::GemmSeg seg = {d_x, L.bias[3], 0, L.dim, L.dim};
    return launch_gemm(L, false, d_att, g->q_dim, M, g->q_dim, nullptr, 0.f, 0, L.dim, &seg, 1,
                       d_x, L.dim, st);
  }
  return launch_proj(a, st, true);
}

int block_decode(int layer, int n, const int* d_seqs, const int* d_pos, int max_rows, float* d_x,
                 cudaStream_t st) {
  const LayerW& L = g->lw[static_cast<size_t>(layer)];
  BlkBufs b;
  int rc = blk_bufs(n, &b);
  if (!rc) rc = run_qkv(L, d_x, n, b, st);
  if (!rc)
    rc = launch_decode(layer, n, d_seqs, d_pos, max_rows, b.q, b.k, b.v, b.att, 0, 0, 0, 1,
                       nullptr, st);
  if (!rc) rc = run_out(L, b.att, n, d_x, st);
  return rc;
}

int block_prefill(int seq, int layer, int start_pos, int n_tok, float* d_x, cudaStream_t st) {
  const LayerW& L = g->lw[static_cast<size_t>(layer)];
  BlkBufs b;
  int rc = blk_bufs(n_tok, &b);
  if (!rc) rc = run_qkv(L, d_x, n_tok, b, st);
  if (!rc) rc = launch_prefill(seq, layer, start_pos, n_tok, b.q, b.k, b.v, b.att, g->q_dim, st);
  if (!rc) rc = run_out(L, b.att, n_tok, d_x, st);
  return rc;
}

int check_layer_set(int layer) {
  if (!g) return PL_ESTATE;
  if (g_multi) return PL_EUNSUPPORTED;
  if (layer < 0 || layer >= g->n_layers) return PL_EARG;
  return g->lw[static_cast<size_t>(layer)].mem ? PL_OK : PL_ESTATE;
}

}  // namespace

extern "C" {

int pl_attn_set_layer(int layer, int dim, const float* attn_norm, float rms_eps, const void* wq,
                      int type_q, const void* wk, int type_k, const void* wv, int type_v,
                      const void* wo, int type_o, const float* bq, const float* bk,
                      const float* bv, const float* bo, const float* q_norm,
                      const float* k_norm) {
  if (!g) return PL_ESTATE;
  if (g_multi) return PL_EUNSUPPORTED;
  if (layer < 0 || layer >= g->n_layers || dim <= 0 || !wq || !wk || !wv || !wo ||
      (q_norm == nullptr) != (k_norm == nullptr) || !(rms_eps >= 0.f))
    return PL_EARG;
  const int types[4] = {type_q, type_k, type_v, type_o};
  const int in[4] = {dim, dim, dim, g->q_dim};
  const int rows[4] = {g->q_dim, g->kv_dim, g->kv_dim, dim};
  const void* src[4] = {wq, wk, wv, wo};
  for (int i = 0; i < 4; ++i)
    if (!pl::proj_type_ok(types[i]) || in[i] % pl::proj_granule(types[i]) != 0) {
      std::fprintf(stderr,
                   "pl_attn_set_layer: weight %d: GGUF type %d over %d inputs is not supported "
                   "(F32, F16, Q8_0, Q4_K, Q6_K; inputs a multiple of the block size)\n",
                   i, types[i], in[i]);
      return PL_EUNSUPPORTED;
    }
  // section offsets in the layer's allocation, 256-byte aligned
  auto up = [](size_t v) { return (v + 255) & ~static_cast<size_t>(255); };
  size_t off[4], total = 0;
  for (int i = 0; i < 4; ++i) {
    off[i] = total;
    total = up(total + pl::proj_row_bytes(types[i], in[i]) * static_cast<size_t>(rows[i]));
  }
  const float* fsrc[7] = {attn_norm, bq, bk, bv, bo, q_norm, k_norm};
  const int flen[7] = {dim, g->q_dim, g->kv_dim, g->kv_dim, dim, g->head_dim, g->head_dim};
  size_t foff[7];
  for (int i = 0; i < 7; ++i) {
    foff[i] = total;
    if (fsrc[i]) total = up(total + static_cast<size_t>(flen[i]) * sizeof(float));
  }
  std::vector<uint8_t> h(total);
  for (int i = 0; i < 4; ++i)
    repack_rows(types[i], static_cast<const uint8_t*>(src[i]), rows[i], in[i], h.data() + off[i]);
  for (int i = 0; i < 7; ++i)
    if (fsrc[i]) std::memcpy(h.data() + foff[i], fsrc[i], static_cast<size_t>(flen[i]) * 4);
  if (cudaSetDevice(g->device) != cudaSuccess) return PL_ECUDA;
  uint8_t* mem = nullptr;
  if (dev_alloc(&mem, total) != cudaSuccess) return PL_ENOMEM;
  if (cudaMemcpy(mem, h.data(), total, cudaMemcpyHostToDevice) != cudaSuccess) {
    cudaFree(mem);
    return PL_ECUDA;
  }
  LayerW& L = g->lw[static_cast<size_t>(layer)];
  if (L.mem) {
    cudaStreamSynchronize(g->stream);
    cudaFree(L.mem);
    cudaFree(L.gmem);
  }
  L = LayerW();
  L.mem = mem;
  L.dim = dim;
  L.eps = rms_eps;
  for (int i = 0; i < 4; ++i) {
    L.w[i] = mem + off[i];
    L.row_bytes[i] = pl::proj_row_bytes(types[i], in[i]);
    L.type[i] = types[i];
  }
  auto fp = [&](int i) { return fsrc[i] ? reinterpret_cast<const float*>(mem + foff[i]) : nullptr; };
  L.attn_norm = fp(0);
  for (int i = 0; i < 4; ++i) L.bias[i] = fp(1 + i);
  L.q_norm = fp(5);
  L.k_norm = fp(6);
  return gemm_prepare_layer(L);
}

int pl_attn_block_decode(int layer, int n, const int* seqs, const int* pos, float* x) {
  int rc = check_layer_set(layer);
  if (rc) return rc;
  if (n <= 0 || n > g->n_seqs || !seqs || !pos || !x) return PL_EARG;
  int max_pos = 0;
  for (int i = 0; i < n; ++i) {
    if (seqs[i] < 0 || seqs[i] >= g->n_seqs || pos[i] < 0 || pos[i] >= g->max_seq)
      return PL_EARG;
    for (int j = 0; j < i; ++j)
      if (seqs[j] == seqs[i]) return PL_EARG;
    if (pos[i] > max_pos) max_pos = pos[i];
  }
  if (cudaSetDevice(g->device) != cudaSuccess) return PL_ECUDA;
  const size_t xb = static_cast<size_t>(n) * g->lw[static_cast<size_t>(layer)].dim * sizeof(float);
  const size_t ib = static_cast<size_t>(n) * sizeof(int);
  const size_t x_off = (2 * ib + 255) & ~static_cast<size_t>(255);
  rc = ensure_stage(x_off + xb + 256);
  if (rc) return rc;
  uint8_t* h = g->h_stage;
  uint8_t* d = g->d_stage;
  std::memcpy(h, seqs, ib);
  std::memcpy(h + ib, pos, ib);
  if (pinned(x, xb)) {
    PL_CUDA(cudaMemcpyAsync(d, h, 2 * ib, cudaMemcpyHostToDevice, g->stream));
    PL_CUDA(cudaMemcpyAsync(d + x_off, x, xb, cudaMemcpyHostToDevice, g->stream));
  } else {
    const CopyPiece in = {h + x_off, reinterpret_cast<const uint8_t*>(x), xb};
    host_copy(&in, 1);
    PL_CUDA(cudaMemcpyAsync(d, h, x_off + xb, cudaMemcpyHostToDevice, g->stream));
  }
  float* d_x = reinterpret_cast<float*>(d + x_off);
  rc = block_decode(layer, n, reinterpret_cast<int*>(d), reinterpret_cast<int*>(d + ib),
                    max_pos + 1, d_x, g->stream);
  if (rc) return rc;
  return read_back(d_x, x, xb, h + x_off);
}

int pl_attn_block_decode_dev(int layer, int n, const int* d_seqs, const int* d_pos, int max_pos,
                             float* d_x, void* stream) {
  int rc = check_layer_set(layer);
  if (rc) return rc;
  if (n <= 0 || n > g->n_seqs || max_pos < 0 || max_pos >= g->max_seq || !d_seqs || !d_pos ||
      !d_x || !aligned16(d_x))
    return PL_EARG;
  return block_decode(layer, n, d_seqs, d_pos, max_pos + 1, d_x, pick_stream(stream));
}

int pl_attn_block_prefill(int seq, int layer, int start_pos, int n_tok, float* x) {
  int rc = check_layer_set(layer);
  if (rc) return rc;
  if (seq < 0 || seq >= g->n_seqs || n_tok <= 0 || start_pos < 0 ||
      start_pos + n_tok > g->max_seq || !x)
    return PL_EARG;
  if (cudaSetDevice(g->device) != cudaSuccess) return PL_ECUDA;
  const size_t xb =
      static_cast<size_t>(n_tok) * g->lw[static_cast<size_t>(layer)].dim * sizeof(float);
  rc = ensure_stage(xb + 256);
  if (rc) return rc;
  uint8_t* h = g->h_stage;
  uint8_t* d = g->d_stage;
  if (pinned(x, xb)) {
    PL_CUDA(cudaMemcpyAsync(d, x, xb, cudaMemcpyHostToDevice, g->stream));
  } else {
    const CopyPiece in = {h, reinterpret_cast<const uint8_t*>(x), xb};
    host_copy(&in, 1);
    PL_CUDA(cudaMemcpyAsync(d, h, xb, cudaMemcpyHostToDevice, g->stream));
  }
  float* d_x = reinterpret_cast<float*>(d);
  rc = block_prefill(seq, layer, start_pos, n_tok, d_x, g->stream);
  if (rc) return rc;
  return read_back(d_x, x, xb, h);
}

int pl_attn_block_prefill_dev(int seq, int layer, int start_pos, int n_tok, float* d_x,
                              void* stream) {
  int rc = check_layer_set(layer);
  if (rc) return rc;
  if (seq < 0 || seq >= g->n_seqs || n_tok <= 0 || start_pos < 0 ||
      start_pos + n_tok > g->max_seq || !d_x || !aligned16(d_x))
    return PL_EARG;
  return block_prefill(seq, layer, start_pos, n_tok, d_x, pick_stream(stream));
}

int pl_attn_proj(int layer, int which, int n, const float* x, float* y) {
  int rc = check_layer_set(layer);
  if (rc) return rc;
  if (which < 0 || which > 3 || n <= 0 || !x || !y) return PL_EARG;
  if (cudaSetDevice(g->device) != cudaSuccess) return PL_ECUDA;
  const LayerW& L = g->lw[static_cast<size_t>(layer)];
  const int in = which == 3 ? g->q_dim : L.dim;
  const int rows = which == 0 ? g->q_dim : (which == 3 ? L.dim : g->kv_dim);
  const size_t xb = static_cast<size_t>(n) * in * sizeof(float);
  const size_t yb = static_cast<size_t>(n) * rows * sizeof(float);
  const size_t y_off = (xb + 255) & ~static_cast<size_t>(255);
  rc = ensure_stage(y_off + yb + 256);
  if (rc) return rc;
  uint8_t* h = g->h_stage;
  uint8_t* d = g->d_stage;
  const CopyPiece cp = {h, reinterpret_cast<const uint8_t*>(x), xb};
  host_copy(&cp, 1);
  PL_CUDA(cudaMemcpyAsync(d, h, xb, cudaMemcpyHostToDevice, g->stream));
  float* d_y = reinterpret_cast<float*>(d + y_off);
  pl::ProjArgs a = {};
  a.mat[0] = proj_mat(L, which, d_y, rows);
  a.n_mat = 1;
  a.total_rows = rows;
  a.x = reinterpret_cast<const float*>(d);
  a.ldx = in;
  a.n = in;
  a.M = n;
  // the tensor-core paths carry x as FP16 parts: only for inputs in range
  bool in_range = true;
  for (size_t i = 0; i < static_cast<size_t>(n) * in && in_range; ++i)
    in_range = std::fabs(x[i]) < 60000.f;
  if (in_range && L.gemm && n >= pl::kGmMinRows) {
    const int w_row0 = which == 0 ? 0 : which == 1 ? g->q_dim : which == 2 ? g->q_dim + g->kv_dim : 0;
    const pl::GemmSeg seg = {d_y, L.bias[which], 0, rows, rows};
    rc = launch_gemm(L, which != 3, reinterpret_cast<const float*>(d), in, n, in, nullptr, 0.f,
                     w_row0, rows, &seg, 1, nullptr, 0, g->stream);
  } else {
    rc = launch_proj(a, g->stream, in_range);
  }
  if (rc) return rc;
  return read_back(d_y, y, yb, h + y_off);
}

}  // extern "C"

// =====================================================================
// One context over several devices of this process (pl_attn_init_devices).
//
// Every device has an ordinary context (Ctx); g is the first one.  Host
// calls fan out from the one host thread that drives the module: inputs
// are staged per device, every device's kernels are queued on its own
// stream before any host wait, and the calls return once every stream is
// done.  Two layouts:
//   PL_SPLIT_SEQS  device d holds global slots [slot0[d], slot0[d+1]) as its
//                  local slots 0..; a batch is split by slot owner.
//   PL_SPLIT_KV    every device holds every slot, but only the rows of the
//                  position blocks b (kKvBlockRows each) with b % D == d,
//                  packed in position order: global row r is local row
//                  (r / B / D) * B + r % B of device (r / B) % D.  A
//                  device's rows at or below a position are therefore its
//                  local rows [0, n), so each device attends them with the
//                  KV-shard partial of the decode kernel (mode 1), and
//                  devices[0] merges the partials, read over NVLink after
//                  waiting on each device's event.  A prefill gathers the
//                  earlier rows of the (slot, layer) onto devices[0], runs
//                  there, and returns each new row to its owner.
// =====================================================================
namespace {

constexpr int kKvBlockRows = 512;

struct Multi {
  int split = PL_SPLIT_SEQS;
  int n_seqs = 0, max_seq = 0;        // global slots and positions
  std::vector<Ctx*> devs;
  std::vector<int> slot0;             // PL_SPLIT_SEQS: first global slot per device, + n_seqs
  std::vector<cudaEvent_t> ev;        // per device: its partial is written
  std::vector<float*> d_mpart;        // PL_SPLIT_KV, per device: partial blocks of one call
  std::vector<size_t> mpart_cap;      // floats
  uint16_t* gk = nullptr;             // PL_SPLIT_KV prefill: one (slot, layer) at full length
  uint16_t* gv = nullptr;             // on devs[0], [max_seq][kv_dim]
  CUtensorMap tm_gk, tm_gv;
};

// Makes devs[d] the module context (and its device current) for the helpers
// above, which all work on g; restores the first device's context.
struct UseCtx {
  explicit UseCtx(Ctx* c) {
    g = c;
    cudaSetDevice(c->device);
  }
  ~UseCtx() {
    g = g_multi->devs[0];
    cudaSetDevice(g->device);
  }
};

int n_dev() { return static_cast<int>(g_multi->devs.size()); }

// ---- PL_SPLIT_KV row map
int kv_owner(int r) { return (r / kKvBlockRows) % n_dev(); }
int kv_local(int r) { return (r / kKvBlockRows / n_dev()) * kKvBlockRows + r % kKvBlockRows; }
// rows of [0, P) that device d holds
int kv_rows_below(int d, int P) {
  const int D = n_dev(), fb = P / kKvBlockRows, rem = P % kKvBlockRows;
  int n = (fb / D + (d < fb % D ? 1 : 0)) * kKvBlockRows;
  if (rem && fb % D == d) n += rem;
  return n;
}
// local cache rows of device d for positions [0, max_seq)
int kv_cache_rows(int d, int D, int max_seq) {
  const int nb = (max_seq + kKvBlockRows - 1) / kKvBlockRows;
  const int blocks = nb > d ? (nb - 1 - d) / D + 1 : 0;
  return (blocks > 0 ? blocks : 1) * kKvBlockRows;
}

int seq_owner(int seq) {
  int d = 0;
  while (seq >= g_multi->slot0[d + 1]) ++d;
  return d;
}

void multi_free() {
  Multi* m = g_multi;
  if (!m) return;
  for (size_t d = 0; d < m->devs.size(); ++d) {
    cudaSetDevice(m->devs[d]->device);
    cudaStreamSynchronize(m->devs[d]->stream);
    if (d < m->ev.size() && m->ev[d]) cudaEventDestroy(m->ev[d]);
    if (d < m->d_mpart.size()) cudaFree(m->d_mpart[d]);
  }
  if (!m->devs.empty()) {
    cudaSetDevice(m->devs[0]->device);
    cudaFree(m->gk);
    cudaFree(m->gv);
  }
  for (Ctx* c : m->devs) free_ctx(c);
  delete m;
  g_multi = nullptr;
}

int multi_init(int n_layers, int n_heads, int n_kv_heads, int head_dim, int max_seq_len,
               float rope_freq_base, int rope_type, int n_seqs, int n_devices,
               const int* devices, int split) {
  if (split == PL_SPLIT_SEQS && n_seqs < n_devices) return PL_EARG;
  g_multi = new Multi;
  Multi* m = g_multi;
  m->split = split;
  m->n_seqs = n_seqs;
  m->max_seq = max_seq_len;
  const int D = n_devices;
  for (int d = 0; d <= D; ++d)
    m->slot0.push_back(static_cast<int>(static_cast<long long>(n_seqs) * d / D));
  int rc = PL_OK;
  for (int d = 0; d < D && !rc; ++d) {
    const int slots = split == PL_SPLIT_SEQS ? m->slot0[d + 1] - m->slot0[d] : n_seqs;
    const int rows = split == PL_SPLIT_SEQS ? max_seq_len : kv_cache_rows(d, D, max_seq_len);
    Ctx* c = nullptr;
    rc = create_ctx(n_layers, n_heads, n_kv_heads, head_dim, max_seq_len, rope_freq_base,
                    rope_type, slots, rows, devices[d], &c);
    if (!rc) m->devs.push_back(c);
  }
  // the KV split reads other devices' partials and rows: peer access between
  // every pair of distinct devices (a repeated id needs none)
  for (int a = 0; a < D && !rc && split == PL_SPLIT_KV; ++a)
    for (int b = 0; b < D && !rc; ++b) {
      if (devices[a] == devices[b]) continue;
      int ok = 0;
      if (cudaDeviceCanAccessPeer(&ok, devices[a], devices[b]) != cudaSuccess || !ok) {
        std::fprintf(stderr, "pl_attn_init_devices: device %d cannot access device %d\n",
                     devices[a], devices[b]);
        rc = PL_EDEVICE;
        break;
      }
      cudaSetDevice(devices[a]);
      const cudaError_t e = cudaDeviceEnablePeerAccess(devices[b], 0);
      if (e == cudaErrorPeerAccessAlreadyEnabled)
        cudaGetLastError();
      else if (e != cudaSuccess)
        rc = PL_ECUDA;
    }
  for (int d = 0; d < D && !rc; ++d) {
    cudaSetDevice(devices[d]);
    cudaEvent_t e = nullptr;
    if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) rc = PL_ECUDA;
    m->ev.push_back(e);
    m->d_mpart.push_back(nullptr);
    m->mpart_cap.push_back(0);
  }
  if (!rc && split == PL_SPLIT_KV) {
    Ctx* c0 = m->devs[0];
    cudaSetDevice(c0->device);
    const size_t bytes = static_cast<size_t>(max_seq_len) * c0->kv_dim * 2;
    if (dev_alloc(&m->gk, bytes) != cudaSuccess || dev_alloc(&m->gv, bytes) != cudaSuccess)
      rc = PL_ENOMEM;
    if (!rc)
      rc = make_map(c0->encode, &m->tm_gk, m->gk, head_dim, max_seq_len, n_kv_heads, 1,
                    pl::pf_block_n(head_dim), 1);
    if (!rc)
      rc = make_map(c0->encode, &m->tm_gv, m->gv, head_dim, max_seq_len, n_kv_heads, 1,
                    pl::pf_block_n(head_dim), 1);
  }
  if (rc) {
    multi_free();
    return rc;
  }
  g = m->devs[0];
  cudaSetDevice(g->device);
  return PL_OK;
}

// Wait for every device's stream; read and clear every error word.  The
// word's read-back is queued on each stream (into the device's pinned word)
// before the first host wait, so the waits overlap.
int multi_finish() {
  int rc = PL_OK;
  std::vector<char> queued(g_multi->devs.size(), 0);
  for (size_t d = 0; d < g_multi->devs.size(); ++d) {
    Ctx* c = g_multi->devs[d];
    UseCtx u(c);
    queued[d] = cudaMemcpyAsync(c->h_err, c->d_err, sizeof(uint32_t), cudaMemcpyDeviceToHost,
                                c->stream) == cudaSuccess;
  }
  for (size_t d = 0; d < g_multi->devs.size(); ++d) {
    Ctx* c = g_multi->devs[d];
    UseCtx u(c);
    if (!queued[d] || cudaStreamSynchronize(c->stream) != cudaSuccess) {
      rc = PL_ECUDA;
      continue;
    }
    const uint32_t w = *reinterpret_cast<volatile uint32_t*>(c->h_err);
    if (w) cudaMemset(c->d_err, 0, sizeof(uint32_t));
    const int r = check_err_word(w);
    if (r && !rc) rc = r;
  }
  return rc;
}

int multi_status() { return multi_finish(); }

int multi_set_wait_limit(uint64_t ns) {
  for (Ctx* c : g_multi->devs) {
    UseCtx u(c);
    PL_CUDA(cudaMemcpyToSymbol(pl::g_wait_limit_ns, &ns, sizeof(ns)));
  }
  return PL_OK;
}

int multi_set_rope(const float* cos_tab, const float* sin_tab, int n_rows, int half_dim) {
  for (Ctx* c : g_multi->devs) {
    UseCtx u(c);
    const int rows = n_rows < c->rope_rows ? n_rows : c->rope_rows;
    const size_t bytes = static_cast<size_t>(rows) * half_dim * sizeof(float);
    PL_CUDA(cudaMemcpyAsync(c->d_cos, cos_tab, bytes, cudaMemcpyHostToDevice, c->stream));
    PL_CUDA(cudaMemcpyAsync(c->d_sin, sin_tab, bytes, cudaMemcpyHostToDevice, c->stream));
  }
  return multi_finish();
}

void multi_profile(int enable) {
  for (Ctx* c : g_multi->devs) {
    c->profiling = enable ? 1 : 0;
    c->ev_used = 0;
    c->n_attn = 0;
    c->n_all = 0;
  }
}

int multi_profile_read(double* attn_ms, long* attn_launches, long* all_launches) {
  double ms = 0.0;
  long na = 0, nall = 0;
  for (Ctx* c : g_multi->devs) {
    UseCtx u(c);
    for (size_t i = 0; i + 1 < c->ev_used; i += 2) {
      PL_CUDA(cudaEventSynchronize(c->ev_pool[i + 1]));
      float t = 0.f;
      PL_CUDA(cudaEventElapsedTime(&t, c->ev_pool[i], c->ev_pool[i + 1]));
      ms += t;
    }
    na += c->n_attn;
    nall += c->n_all;
    c->ev_used = 0;
    c->n_attn = 0;
    c->n_all = 0;
  }
  if (attn_ms) *attn_ms = ms;
  if (attn_launches) *attn_launches = na;
  if (all_launches) *all_launches = nall;
  return PL_OK;
}

int check_batch(int layer, int n, const int* seqs, const int* pos, int* max_pos) {
  if (n <= 0 || n > g_multi->n_seqs || !seqs || !pos) return PL_EARG;
  if (layer < 0 || layer >= g->n_layers) return PL_EARG;
  *max_pos = 0;
  for (int i = 0; i < n; ++i) {
    if (seqs[i] < 0 || seqs[i] >= g_multi->n_seqs || pos[i] < 0 || pos[i] >= g_multi->max_seq)
      return PL_EARG;
    for (int j = 0; j < i; ++j)
      if (seqs[j] == seqs[i]) return PL_EARG;
    if (pos[i] > *max_pos) *max_pos = pos[i];
  }
  return PL_OK;
}

// PL_SPLIT_SEQS decode: each device gets the batch entries of its slots,
// gathered into its staging area; every device is queued before any wait.
int multi_decode_seqs(int layer, int n, const int* seqs, const int* pos, const float* q,
                      const float* k, const float* v, float* out) {
  Multi* m = g_multi;
  const int D = n_dev();
  const size_t qf = g->q_dim, kf = g->kv_dim;
  std::vector<std::vector<int>> idx(D);
  for (int i = 0; i < n; ++i) idx[seq_owner(seqs[i])].push_back(i);
  std::vector<size_t> out_off(D, 0);
  int rc = PL_OK;
  for (int d = 0; d < D && !rc; ++d) {
    const int nd = static_cast<int>(idx[d].size());
    if (!nd) continue;
    Ctx* c = m->devs[d];
    UseCtx u(c);
    const size_t qb = nd * qf * sizeof(float), kb = nd * kf * sizeof(float);
    const size_t ib = nd * sizeof(int), in_bytes = qb + 2 * kb + 2 * ib;
    out_off[d] = (in_bytes + 255) & ~static_cast<size_t>(255);
    rc = ensure_stage(out_off[d] + qb + 256);
    if (rc) break;
    uint8_t* h = c->h_stage;
    std::vector<CopyPiece> pc;
    int* hs = reinterpret_cast<int*>(h + qb + 2 * kb);
    int* hp = hs + nd;
    int max_pos = 0;
    for (int j = 0; j < nd; ++j) {
      const int i = idx[d][j];
      pc.push_back({h + j * qf * 4, reinterpret_cast<const uint8_t*>(q + i * qf), qf * 4});
      pc.push_back({h + qb + j * kf * 4, reinterpret_cast<const uint8_t*>(k + i * kf), kf * 4});
      pc.push_back(
          {h + qb + kb + j * kf * 4, reinterpret_cast<const uint8_t*>(v + i * kf), kf * 4});
      hs[j] = seqs[i] - m->slot0[d];
      hp[j] = pos[i];
      if (pos[i] > max_pos) max_pos = pos[i];
    }
    host_copy(pc.data(), static_cast<int>(pc.size()));
    uint8_t* dst = c->d_stage;
    if (cudaMemcpyAsync(dst, h, in_bytes, cudaMemcpyHostToDevice, c->stream) != cudaSuccess) {
      rc = PL_ECUDA;
      break;
    }
    float* d_out = reinterpret_cast<float*>(dst + out_off[d]);
    rc = launch_decode(layer, nd, reinterpret_cast<int*>(dst + qb + 2 * kb),
                       reinterpret_cast<int*>(dst + qb + 2 * kb + ib), max_pos + 1,
                       reinterpret_cast<float*>(dst), reinterpret_cast<float*>(dst + qb),
                       reinterpret_cast<float*>(dst + qb + kb), d_out, 0, 0, 0, 1, nullptr,
                       c->stream);
    if (!rc && cudaMemcpyAsync(h + out_off[d], d_out, qb, cudaMemcpyDeviceToHost, c->stream) !=
                   cudaSuccess)
      rc = PL_ECUDA;
  }
  const int rc2 = multi_finish();
  if (rc) return rc;
  if (rc2) return rc2;
  for (int d = 0; d < D; ++d) {
    const int nd = static_cast<int>(idx[d].size());
    if (!nd) continue;
    std::vector<CopyPiece> pc;
    const uint8_t* h = m->devs[d]->h_stage + out_off[d];
    for (int j = 0; j < nd; ++j)
      pc.push_back({reinterpret_cast<uint8_t*>(out + idx[d][j] * qf), h + j * qf * 4, qf * 4});
    host_copy(pc.data(), static_cast<int>(pc.size()));
  }
  return PL_OK;
}

// PL_SPLIT_KV decode: per sequence, a partial on every device holding rows
// at or below its position (the owner of the position appends), merged on
// devices[0] after waiting on each device's event.
int multi_decode_kv(int layer, int n, const int* seqs, const int* pos, const float* q,
                    const float* k, const float* v, float* out) {
  Multi* m = g_multi;
  const int D = n_dev();
  const size_t qf = g->q_dim, kf = g->kv_dim;
  const size_t qb = n * qf * sizeof(float), kb = n * kf * sizeof(float);
  const size_t in_bytes = qb + 2 * kb;
  const size_t out_off = (in_bytes + 255) & ~static_cast<size_t>(255);
  int rc = PL_OK;
  // stage q, k, v of the whole batch on every device holding rows
  for (int d = 0; d < D && !rc; ++d) {
    Ctx* c = m->devs[d];
    UseCtx u(c);
    rc = ensure_stage(out_off + qb + 256);
    const size_t need = static_cast<size_t>(n) * c->part_floats;
    if (!rc && need > m->mpart_cap[d]) {
      cudaFree(m->d_mpart[d]);
      m->d_mpart[d] = nullptr;
      m->mpart_cap[d] = 0;
      if (dev_alloc(&m->d_mpart[d], need * sizeof(float)) != cudaSuccess)
        rc = PL_ENOMEM;
      else
        m->mpart_cap[d] = need;
    }
    if (rc) break;
    const CopyPiece in[3] = {{c->h_stage, reinterpret_cast<const uint8_t*>(q), qb},
                             {c->h_stage + qb, reinterpret_cast<const uint8_t*>(k), kb},
                             {c->h_stage + qb + kb, reinterpret_cast<const uint8_t*>(v), kb}};
    host_copy(in, 3);
    if (cudaMemcpyAsync(c->d_stage, c->h_stage, in_bytes, cudaMemcpyHostToDevice, c->stream) !=
        cudaSuccess)
      rc = PL_ECUDA;
  }
  Ctx* c0 = m->devs[0];
  for (int i = 0; i < n && !rc; ++i) {
    const int p = pos[i], owner = kv_owner(p);
    pl::PeerParts parts = {};
    int n_part = 0;
    for (int d = 0; d < D && !rc; ++d) {
      const int rows = kv_rows_below(d, p + 1);
      if (!rows) continue;
      Ctx* c = m->devs[d];
      UseCtx u(c);
      const float* dq = reinterpret_cast<const float*>(c->d_stage) + i * qf;
      const float* dk = reinterpret_cast<const float*>(c->d_stage + qb) + i * kf;
      const float* dv = reinterpret_cast<const float*>(c->d_stage + qb + kb) + i * kf;
      float* part = m->d_mpart[d] + static_cast<size_t>(i) * c->part_floats;
      const bool app = d == owner;
      rc = partial_launch(seqs[i], layer, p, app ? p - kv_local(p) : 0, rows, app ? 1 : 0, dq,
                          dk, dv, part, c->stream);
      if (!rc && cudaEventRecord(m->ev[d], c->stream) != cudaSuccess) rc = PL_ECUDA;
      if (!rc && d && cudaStreamWaitEvent(c0->stream, m->ev[d], 0) != cudaSuccess) rc = PL_ECUDA;
      parts.p[n_part++] = part;
    }
    if (rc) break;
    const int blocks = (g->n_heads * (g->head_dim / 4) + 255) / 256;
    float* o = reinterpret_cast<float*>(c0->d_stage + out_off) + i * qf;
    if (g->head_dim == 128)
      pl::combine_peers_kernel<128><<<blocks, 256, 0, c0->stream>>>(parts, n_part, g->n_heads, o);
    else
      pl::combine_peers_kernel<64><<<blocks, 256, 0, c0->stream>>>(parts, n_part, g->n_heads, o);
    if (cudaGetLastError() != cudaSuccess) rc = PL_ECUDA;
    count_launch();
  }
  if (!rc && cudaMemcpyAsync(c0->h_stage + out_off, c0->d_stage + out_off, qb,
                             cudaMemcpyDeviceToHost, c0->stream) != cudaSuccess)
    rc = PL_ECUDA;
  const int rc2 = multi_finish();
  if (rc) return rc;
  if (rc2) return rc2;
  const CopyPiece o = {reinterpret_cast<uint8_t*>(out), c0->h_stage + out_off, qb};
  host_copy(&o, 1);
  return PL_OK;
}

int multi_decode_batch(int layer, int n, const int* seqs, const int* pos, const float* q,
                       const float* k, const float* v, float* out) {
  int max_pos = 0;
  int rc = check_batch(layer, n, seqs, pos, &max_pos);
  if (rc) return rc;
  if (!q || !k || !v || !out) return PL_EARG;
  if (g_multi->split == PL_SPLIT_SEQS) return multi_decode_seqs(layer, n, seqs, pos, q, k, v, out);
  return multi_decode_kv(layer, n, seqs, pos, q, k, v, out);
}

// Copy rows [r0, r1) of (seq, layer) between device d's cache and host or
// device memory at `other` (a pointer to row r0's K words; V likewise),
// on stream st.  K and V words of a row are kv_dim apart in the caller's
// arrays only through the two separate pointers.
int kv_rows_copy(Ctx* c, int seq_local, int layer, int local_row, int rows, void* k_other,
                 void* v_other, cudaMemcpyKind kind, cudaStream_t st) {
  const size_t off = (static_cast<size_t>(seq_local) * c->n_layers + layer) * c->layer_elems +
                     static_cast<size_t>(local_row) * c->kv_dim;
  const size_t bytes = static_cast<size_t>(rows) * c->kv_dim * 2;
  const bool to_dev = kind == cudaMemcpyHostToDevice;
  if (k_other)
    PL_CUDA(cudaMemcpyAsync(to_dev ? static_cast<void*>(c->d_k + off) : k_other,
                            to_dev ? k_other : static_cast<void*>(c->d_k + off), bytes, kind, st));
  if (v_other)
    PL_CUDA(cudaMemcpyAsync(to_dev ? static_cast<void*>(c->d_v + off) : v_other,
                            to_dev ? v_other : static_cast<void*>(c->d_v + off), bytes, kind, st));
  return PL_OK;
}

int multi_kv_copy(int seq, int layer, int pos0, int n_pos, uint16_t* k, uint16_t* v,
                  bool download) {
  Multi* m = g_multi;
  if (seq < 0 || seq >= m->n_seqs || layer < 0 || layer >= g->n_layers) return PL_EARG;
  if (pos0 < 0 || n_pos < 0 || pos0 + n_pos > m->max_seq) return PL_EARG;
  if (n_pos == 0) return PL_OK;
  const cudaMemcpyKind kind = download ? cudaMemcpyDeviceToHost : cudaMemcpyHostToDevice;
  const size_t kv = g->kv_dim;
  int rc = PL_OK;
  if (m->split == PL_SPLIT_SEQS) {
    const int d = seq_owner(seq);
    Ctx* c = m->devs[d];
    UseCtx u(c);
    rc = kv_rows_copy(c, seq - m->slot0[d], layer, pos0, n_pos, k, v, kind, c->stream);
  } else {
    for (int r = pos0; r < pos0 + n_pos && !rc;) {
      const int end_blk = (r / kKvBlockRows + 1) * kKvBlockRows;
      const int r1 = end_blk < pos0 + n_pos ? end_blk : pos0 + n_pos;
      Ctx* c = m->devs[kv_owner(r)];
      UseCtx u(c);
      const size_t o = static_cast<size_t>(r - pos0) * kv;
      rc = kv_rows_copy(c, seq, layer, kv_local(r), r1 - r, k ? k + o : nullptr,
                        v ? v + o : nullptr, kind, c->stream);
      r = r1;
    }
  }
  const int rc2 = multi_finish();
  return rc ? rc : rc2;
}

// Rows [r0, r1) of (seq, layer) between the owners' caches and the
// gathering slab on devices[0] (to_slab: owners -> slab), on devices[0]'s
// stream; peer copies where the owner is another GPU.
int kv_slab_move(int seq, int layer, int r0, int r1, bool to_slab) {
  Multi* m = g_multi;
  Ctx* c0 = m->devs[0];
  const size_t kv = c0->kv_dim;
  for (int r = r0; r < r1;) {
    const int end_blk = (r / kKvBlockRows + 1) * kKvBlockRows;
    const int re = end_blk < r1 ? end_blk : r1;
    Ctx* c = m->devs[kv_owner(r)];
    const size_t off = (static_cast<size_t>(seq) * c->n_layers + layer) * c->layer_elems +
                       static_cast<size_t>(kv_local(r)) * kv;
    const size_t bytes = static_cast<size_t>(re - r) * kv * 2;
    for (int x = 0; x < 2; ++x) {
      uint16_t* own = (x ? c->d_v : c->d_k) + off;
      uint16_t* slab = (x ? m->gv : m->gk) + static_cast<size_t>(r) * kv;
      uint16_t* dst = to_slab ? slab : own;
      uint16_t* src = to_slab ? own : slab;
      const int ddev = to_slab ? c0->device : c->device, sdev = to_slab ? c->device : c0->device;
      if (ddev == sdev)
        PL_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, c0->stream));
      else
        PL_CUDA(cudaMemcpyPeerAsync(dst, ddev, src, sdev, bytes, c0->stream));
    }
    r = re;
  }
  return PL_OK;
}

int multi_prefill(int seq, int layer, int start_pos, int n_tok, const float* q, const float* k,
                  const float* v, float* out, int out_stride) {
  Multi* m = g_multi;
  if (seq < 0 || seq >= m->n_seqs || layer < 0 || layer >= g->n_layers) return PL_EARG;
  if (n_tok <= 0 || start_pos < 0 || start_pos + n_tok > m->max_seq || !q || !k || !v || !out ||
      out_stride < g->q_dim)
    return PL_EARG;
  if (m->split == PL_SPLIT_SEQS) {
    // the slot's owner runs it as a single device would
    const int d = seq_owner(seq);
    Ctx* c = m->devs[d];
    Multi* saved = g_multi;
    int rc;
    {
      UseCtx u(c);
      g_multi = nullptr;  // the single-device path, on this device's context
      rc = pl_attn_prefill(seq - saved->slot0[d], layer, start_pos, n_tok, q, k, v, out,
                           out_stride);
      g_multi = saved;
    }
    return rc;
  }
  Ctx* c0 = m->devs[0];
  const size_t qb = static_cast<size_t>(n_tok) * g->q_dim * sizeof(float);
  const size_t kb = static_cast<size_t>(n_tok) * g->kv_dim * sizeof(float);
  const size_t in_bytes = qb + 2 * kb;
  const size_t out_off = (in_bytes + 255) & ~static_cast<size_t>(255);
  int rc = ensure_stage(out_off + qb + 256);
  if (rc) return rc;
  cudaSetDevice(c0->device);
  // the earlier rows of this (slot, layer) onto devices[0]
  rc = kv_slab_move(seq, layer, 0, start_pos, true);
  if (rc) return rc;
  const CopyPiece in[3] = {{c0->h_stage, reinterpret_cast<const uint8_t*>(q), qb},
                           {c0->h_stage + qb, reinterpret_cast<const uint8_t*>(k), kb},
                           {c0->h_stage + qb + kb, reinterpret_cast<const uint8_t*>(v), kb}};
  host_copy(in, 3);
  PL_CUDA(cudaMemcpyAsync(c0->d_stage, c0->h_stage, in_bytes, cudaMemcpyHostToDevice,
                          c0->stream));
  float* d_out = reinterpret_cast<float*>(c0->d_stage + out_off);
  rc = launch_prefill_rows(m->gk, m->gv, m->tm_gk, m->tm_gv, 0, start_pos, n_tok,
                           reinterpret_cast<float*>(c0->d_stage),
                           reinterpret_cast<float*>(c0->d_stage + qb),
                           reinterpret_cast<float*>(c0->d_stage + qb + kb), d_out, g->q_dim,
                           c0->stream);
  // the new rows back to their owners
  if (!rc) rc = kv_slab_move(seq, layer, start_pos, start_pos + n_tok, false);
  if (!rc && cudaMemcpyAsync(c0->h_stage + out_off, d_out, qb, cudaMemcpyDeviceToHost,
                             c0->stream) != cudaSuccess)
    rc = PL_ECUDA;
  const int rc2 = multi_finish();
  if (rc) return rc;
  if (rc2) return rc2;
  for (int r = 0; r < n_tok; ++r)
    std::memcpy(out + static_cast<size_t>(r) * out_stride,
                c0->h_stage + out_off + static_cast<size_t>(r) * g->q_dim * sizeof(float),
                g->q_dim * sizeof(float));
  return PL_OK;
}

}  // namespace
