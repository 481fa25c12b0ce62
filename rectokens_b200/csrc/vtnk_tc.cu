// Tensor-core beam step for sm_100a: tcgen05.mma with TMEM accumulators fed
// by TMA, fused with the trie child mask, per-row top-n, log-sum-exp and the
// next-node lookup.  Full logits never leave the SM.
//
// Per level the contraction is a dense GEMM  D[R, 256] = A[R, H] . Wwin[256, H]^T
// where Wwin = the LM-head rows of the level's token window (every child of
// every node at this depth lies in [window_lo, window_lo + 256)).  Columns
// that are not children of a row's node are dropped in the epilogue, using
// the depth's child-bitmask index (32 bytes per node, built once per trie).
//
// CTA layout (persistent; a cluster of two CTAs on two SMs; 320 threads each):
//   warp 0      TMA producer      per stage: this CTA's A tile [128 x 64] and half
//                                 of the W window [128 x 64] (SWIZZLE_128B, K-major)
//   warp 1      MMA issuer        pair variant: the leader issues
//                                 tcgen05.mma.cta_group::2.kind::f16, M=256 N=256 K=16
//                                 over both CTAs' operands; split variant: each CTA
//                                 issues cta_group::1 M=128 N=128 on its own half of
//                                 the window.  Also allocates / frees TMEM (two
//                                 accumulators, so the epilogue of tile i overlaps
//                                 the MMAs of tile i + 1)
//   warps 2..9  epilogue          thread = row: tcgen05.ld 32x32b, mask, log-sum-exp
//                                 and top-n (or Gumbel-max); two warps per TMEM lane
//                                 group split the columns, the upper half hands its
//                                 partial result to the lower half (split variant:
//                                 then CTA 1 to CTA 0 through distributed shared
//                                 memory)
// Shared memory: a 5-stage x 32 KB operand ring (4 in the split variant; one
// stage more where the epilogue's buffers leave room), the
// epilogue's chunk staging and hand-off buffers, the window's bias, mbarriers.
//
// Every mbarrier wait is bounded in time; on expiry the CTA records a status
// code in a device word (read by vtnk_device_status), drains its in-flight
// copies and MMAs with bounded waits, frees its TMEM and exits.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <climits>
#include <cstdlib>
#include <mutex>

#include "vtnk_internal.h"

namespace vtnk {

__device__ int g_tc_status = 0;  // 0 ok; else the first failing wait's code

// Phase timers for tuning builds (-DVTNK_TC_PROFILE): cycles summed over CTAs.
#ifdef VTNK_TC_PROFILE
__device__ unsigned long long g_prof[8];
#define PROF_T0(name) const long long name = clock64()
#define PROF_ACC(acc, t0) acc += clock64() - (t0)
#define PROF_FLUSH(i, acc) atomicAdd(&g_prof[i], static_cast<unsigned long long>(acc))
// Per-CTA %globaltimer stamps of one launch's first tile (tuning builds).
__device__ unsigned long long g_trace[512][32];
#define TRACE(i)                                                                  \
  do {                                                                            \
    if (blockIdx.x < 512) {                                                       \
      unsigned long long t_;                                                      \
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                     \
      g_trace[blockIdx.x][i] = t_;                                                \
    }                                                                             \
  } while (0)
#define TRACE_VAL(i, v)                                                           \
  do {                                                                            \
    if (blockIdx.x < 512) g_trace[blockIdx.x][i] = static_cast<unsigned long long>(v); \
  } while (0)
#else
#define TRACE(i)
#define TRACE_VAL(i, v)
#define PROF_T0(name)
#define PROF_ACC(acc, t0)
#define PROF_FLUSH(i, acc)
#endif

namespace tc {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;
constexpr int PAIR_M = 2 * BM;  // rows per CTA pair (one cta_group::2 MMA tile)
#ifndef VTNK_TC_STAGES
#define VTNK_TC_STAGES 5
#endif
constexpr int STAGES = VTNK_TC_STAGES;
// Column groups of the epilogue's lower bound for NC up to this many (a power of two).
#ifndef VTNK_TC_GROUPS
#define VTNK_TC_GROUPS 16
#endif
constexpr int A_BYTES = BM * BK * 2;        // this CTA's 128 rows
constexpr int B_BYTES = (BN / 2) * BK * 2;  // this CTA's half of the 256 window rows
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int EPI_WARPS = 8;  // two per TMEM lane group, splitting the 256 columns
constexpr int MAX_NC = 32;
constexpr int THREADS = (2 + EPI_WARPS) * 32;
constexpr uint64_t WAIT_LIMIT_NS = 2000000000ull;  // default bound of every wait: 2 s

// A partial result (top-n, max, sum) travels between warps as rows of a
// [*][32] table (lane = row): NC values, the NC window columns packed four to
// a word, max, sum.
template <int NC>
struct ListRows {
  static constexpr int COLS = NC;                 // first row of the packed columns
  static constexpr int MX = NC + (NC + 3) / 4;    // the running max
  static constexpr int SUM = MX + 1;              // the running sum
  static constexpr int N = SUM + 1;
};

// The split variant's cross-CTA hand-off buffers (none in the pair variant).
template <bool SPLIT, int NC>
struct XMerge {
  float x[4][ListRows<NC>::N][32];
};
template <int NC>
struct XMerge<false, NC> {};

// Candidate-list slots per lane of the top-n epilogue: 16, and at least NC
// (the hand-off merge stages a warp's NC-entry list in the same slots);
// sampling stages one whole 32-column chunk in the same buffer.
template <bool SAMPLE, int NC>
constexpr int cand_slots() { return SAMPLE ? 32 : (NC > 16 ? NC : 16); }

// Shared memory of one CTA with ST operand stages.  SPLIT: the split-window
// variant's cross-CTA hand-off buffers.
template <bool SPLIT, int NC, bool SAMPLE, int ST_>
struct SharedBody {
  static constexpr int ST = ST_;
  static constexpr int CS = cand_slots<SAMPLE, NC>();
  uint8_t ring[ST][STAGE_BYTES];  // 1024-aligned stages
  float chunk_x[EPI_WARPS][CS][32];    // epilogue, per warp, [slot][lane]: top-n candidate
                                       // values (sampling: one 32-column chunk)
  uint8_t chunk_c[EPI_WARPS][CS][32];  // their window columns
  float merge[4][ListRows<NC>::N][32];  // upper-half -> lower-half partial results
  XMerge<SPLIT, NC> xm;  // split: window half 1 -> half 0 (empty in the pair variant)
  float bias[BN];
  uint64_t full[ST];
  uint64_t empty[ST];
  uint64_t xmerge_full[4];
  uint64_t xmerge_empty[4];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t merge_full[4];
  uint64_t merge_empty[4];
  uint64_t mma_done;
  uint64_t epi_sync;  // the epilogue warps of this CTA (split-tile hand-over)
  uint32_t tmem_base;
  int abort;
  int sk_last;  // epilogue: this CTA finishes the current split tile
};
constexpr size_t SMEM_LIMIT = 232448;  // 227 KB of opt-in shared memory per CTA
// One operand stage more than STAGES when it fits beside the epilogue's
// buffers (the operand pipeline is latency-bound: more bytes in flight help).
template <bool SPLIT, int NC, bool SAMPLE>
constexpr int stages_for() {
  constexpr int base = SPLIT ? STAGES - 1 : STAGES;
  return sizeof(SharedBody<SPLIT, NC, SAMPLE, base + 1>) + 1024 <= SMEM_LIMIT ? base + 1 : base;
}
template <bool SPLIT, int NC, bool SAMPLE>
using SharedT = SharedBody<SPLIT, NC, SAMPLE, stages_for<SPLIT, NC, SAMPLE>()>;
template <bool SPLIT, int NC, bool SAMPLE>
constexpr size_t smem_bytes() {
  return sizeof(SharedT<SPLIT, NC, SAMPLE>) + 1024;
}
static_assert(smem_bytes<false, 32, false>() <= SMEM_LIMIT &&
                  smem_bytes<true, 32, false>() <= SMEM_LIMIT &&
                  smem_bytes<true, 1, true>() <= SMEM_LIMIT,
              "shared memory above the 227 KB per-CTA limit");

struct Params {
  int64_t rows, H;
  const int64_t* cur_node;
  Csr csr;
  int64_t mb;
  int64_t window_lo;
  int window_n;
  int n_cand;
  const uint32_t* masks;
  const uint32_t* flags;  // index flag word or nullptr (bit 0: child node id = edge index + 1)
  int64_t idx_lo, idx_hi;
  const __nv_bfloat16* a;
  int64_t a_stride;
  const __nv_bfloat16* w;
  int64_t w_stride;
  const __nv_bfloat16* bias;
  int64_t n_vocab;
  int64_t* cand_tok;
  float* cand_logit;
  int64_t* cand_node;
  float* row_lse;
  uint64_t seed;             // sampling: Philox key
  const float* temperature;  // sampling: device scalar (nullptr: 1)
  float* sample_f;           // sampling: token id as float, -1 when none (optional)
  int64_t* l0_ids;           // level 0 of a beam search: beams written directly (optional)
  float* l0_logp;
  int64_t* l0_node;
  int l0_k;
  int vec_out;  // outputs aligned for paired stores, n_cand and l0_k even (set by the host)
  // Schedule: tiles [0, dp_tiles) go to pairs round-robin (whole tiles); the
  // k-block iterations of tiles [dp_tiles, n_tiles) are split evenly over the
  // first sk_pairs pairs (stream-K).  A tile split between pairs is summed
  // from fp32 partials by its last contributor.
  int64_t dp_tiles;
  int64_t sk_iters;                  // (n_tiles - dp_tiles) * k-blocks
  int sk_pairs;                      // 0: no stream-K part
  float* sk_part;                    // [sk_pairs][2 slots][2 ranks][BM][BN] fp32
  unsigned long long* sk_count;      // [stream-K tiles][2 ranks]: epoch << 32 | k-blocks done
  uint32_t sk_epoch;                 // distinct per launch on the same workspace
  uint64_t wait_ns;  // bound of every mbarrier wait (ns); on expiry the CTA aborts
  int stall;         // test hook: the producers issue no copies, so the first wait expires
};

// ------------------------------------------------------------------ PTX wrappers
constexpr float kLog2e = 1.4426950408889634f;
// 2^x by the SFU's base-2 exponential (PTX ex2.approx.ftz.f32).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ uint32_t su32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ int64_t ld_relaxed_s64(const int64_t* q) {
  int64_t v;
  asm volatile("ld.relaxed.gpu.global.s64 %0, [%1];" : "=l"(v) : "l"(q) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(b)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(su32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Wait for phase `parity` of barrier b; false when the CTA is aborting or the
// time limit ran out (then the abort flag and the device status are set).
__device__ __forceinline__ bool wait_phase(uint64_t* b, uint32_t parity, volatile int* abort,
                                           int code, uint64_t lim) {
  if (mbar_try_wait(b, parity)) return true;
  const uint64_t t0 = gtimer();
  uint32_t ns = 0;
  for (uint32_t i = 1;; ++i) {
#ifndef VTNK_TC_SPIN
    if (ns) __nanosleep(ns);  // back off so a waiting role does not steal issue slots
#endif
    if (mbar_try_wait(b, parity)) return true;
    if (i >= 4) ns = ns ? (ns < 128 ? ns * 2 : ns) : 16;
    if ((i & 15) == 0) {
      if (*abort) return false;
      if (gtimer() - t0 > lim || i > (1u << 30)) {
        *abort = 1;
        atomicCAS(&g_tc_status, 0, code);
        return false;
      }
    }
  }
}
// --- CTA-pair helpers (cluster of two CTAs sharing one cta_group::2 MMA)
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address of the same shared-memory object in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_to_rank(const void* p, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(su32(p)), "r"(rank));
  return out;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(su32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait with cluster-scope acquire (for arrivals from the peer CTA).
__device__ __forceinline__ bool wait_phase_cluster(uint64_t* b, uint32_t parity,
                                                   volatile int* abort, int code, uint64_t lim) {
  if (mbar_try_wait_cluster(b, parity)) return true;
  const uint64_t t0 = gtimer();
  uint32_t ns = 0;
  for (uint32_t i = 1;; ++i) {
#ifndef VTNK_TC_SPIN
    if (ns) __nanosleep(ns);
#endif
    if (mbar_try_wait_cluster(b, parity)) return true;
    if (i >= 4) ns = ns ? (ns < 128 ? ns * 2 : ns) : 16;
    if ((i & 15) == 0) {
      if (*abort) return false;
      if (gtimer() - t0 > lim || i > (1u << 30)) {
        *abort = 1;
        atomicCAS(&g_tc_status, 0, code);
        return false;
      }
    }
  }
}
// TMA load into this CTA's shared memory whose completion is counted on the
// pair leader's barrier (cluster address); no multicast.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map,
                                                 uint32_t leader_bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(su32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(leader_bar), "r"(x), "r"(y)
      : "memory");
}
// Warp-level wait for the epilogue: one lane polls, with a growing sleep
// between polls, so 128 waiting threads do not compete with the tensor
// core's operand reads for shared memory.  Result in every lane.
__device__ __forceinline__ bool warp_wait_phase(uint64_t* b, uint32_t parity, volatile int* abort,
                                                int code, uint64_t lim) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) {
    if (!mbar_try_wait(b, parity)) {
      const uint64_t t0 = gtimer();
      uint32_t ns = 32;
      for (;;) {
        __nanosleep(ns);
        if (mbar_try_wait(b, parity)) break;
        if (ns < 512) ns <<= 1;
        if (*abort) {
          ok = 0;
          break;
        }
        if (gtimer() - t0 > lim) {
          *abort = 1;
          atomicCAS(&g_tc_status, 0, code);
          ok = 0;
          break;
        }
      }
    }
  }
  ok = __shfl_sync(0xffffffffu, ok, 0);
  return ok != 0;
}

// One arrival for the whole warp on a CTA-local barrier, ordered after every
// lane's earlier shared-memory accesses (__syncwarp orders them before lane
// 0's release).  One arrival instead of 32: arrivals on one barrier are
// serialised.
__device__ __forceinline__ void warp_arrive(uint64_t* b) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(b);
}
// The same on a barrier of another CTA of the cluster; every lane first
// fences its own (remote) stores at cluster scope.
__device__ __forceinline__ void warp_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("fence.acq_rel.cluster;" ::: "memory");
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive_cluster(cluster_addr);
}

// warp_wait_phase for a barrier that the other CTA of the cluster arrives on
// (cluster-scope acquire).
__device__ __forceinline__ bool warp_wait_phase_cluster(uint64_t* b, uint32_t parity,
                                                        volatile int* abort, int code,
                                                        uint64_t lim) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) {
    if (!mbar_try_wait_cluster(b, parity)) {
      const uint64_t t0 = gtimer();
      uint32_t ns = 32;
      for (;;) {
        __nanosleep(ns);
        if (mbar_try_wait_cluster(b, parity)) break;
        if (ns < 512) ns <<= 1;
        if (*abort) {
          ok = 0;
          break;
        }
        if (gtimer() - t0 > lim) {
          *abort = 1;
          atomicCAS(&g_tc_status, 0, code);
          ok = 0;
          break;
        }
      }
    }
  }
  ok = __shfl_sync(0xffffffffu, ok, 0);
  if (ok) mbar_try_wait_cluster(b, parity);  // every lane acquires
  return ok != 0;
}

// Drain wait at teardown: bounded, never sets abort.
__device__ __forceinline__ void drain_phase(uint64_t* b, uint32_t parity, uint64_t lim) {
  const uint64_t t0 = gtimer();
  while (!mbar_try_wait(b, parity))
    if (gtimer() - t0 > lim / 4) return;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(su32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(su32(bar)), "r"(x), "r"(y)
      : "memory");
}

// UMMA shared-memory descriptor: K-major operand in the 128-byte swizzle
// layout TMA writes (8-row x 128-byte atoms, 1024 B between atoms).
__device__ __forceinline__ uint64_t umma_desc_sw128(const void* smem) {
  const uint64_t addr = su32(smem);
  return ((addr & 0x3FFFF) >> 4)                      // start address (16 B units)
         | (1ull << 16)                               // leading byte offset (unused here)
         | (static_cast<uint64_t>(1024 >> 4) << 32)   // stride byte offset: 8 rows x 128 B
         | (1ull << 46)                               // descriptor version (sm_100)
         | (2ull << 61);                              // layout: SWIZZLE_128B
}
// Instruction descriptor: kind::f16, A = B = bf16, D = fp32, both K-major,
// N = 256, M = 256 (a cta_group::2 pair, 128 rows per CTA).
constexpr uint32_t idesc(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}
constexpr uint32_t IDESC = idesc(PAIR_M, BN);
// Split-window variant: one CTA, M = 128 rows, N = 128 columns (half the window).
constexpr uint32_t IDESC_SPLIT = idesc(BM, BN / 2);

__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t da, uint64_t db,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(da), "l"(db), "r"(IDESC), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_bf16_cta(uint32_t d_tmem, uint64_t da, uint64_t db,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(da), "l"(db), "r"(IDESC_SPLIT), "r"(accumulate)
      : "memory");
}
// Arrive on this CTA's barrier `bar` once all previously issued MMAs of this
// thread are complete.
__device__ __forceinline__ void umma_commit_cta(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          su32(bar))
      : "memory");
}
// Store to the same shared-memory offset in another CTA of the cluster.
__device__ __forceinline__ void st_cluster_f32(uint32_t cluster_addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(cluster_addr), "f"(v) : "memory");
}
// Arrive on barrier `bar` (same offset) in both CTAs of the pair once all
// previously issued MMAs of this thread are complete.
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b16 m;\n\tmov.b16 m, 3;\n\t"
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], m;\n\t}" ::"r"(su32(bar))
      : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]),
        "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]),
        "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ------------------------------------------------------------------ schedule
// One unit of a pair's work: k-blocks [kb0, kb1) of a 256-row tile.
struct Seg {
  int64_t tile;
  int kb0, kb1;
  int64_t sk_tile;  // index among the stream-K tiles, -1 for a round-robin tile
  int slot;         // 0: the pair's first stream-K segment, 1: a later one
};

__device__ __forceinline__ int64_t sk_begin(const Params& p, int64_t q) {
  return (q * p.sk_iters) / p.sk_pairs;
}
// The pair whose stream-K range holds iteration g.
__device__ __forceinline__ int64_t sk_owner(const Params& p, int64_t g) {
  return ((g + 1) * p.sk_pairs + p.sk_iters - 1) / p.sk_iters - 1;
}

// Enumerates a pair's segments in order; producer, MMA issuer and epilogue
// walk the same sequence.  Small state: it lives through the whole kernel.
struct SegIter {
  int64_t g, gend;  // stream-K iteration cursor and end
  int i;            // round-robin tiles taken
  int pair;
  bool first;       // the next stream-K segment is the pair's first
  __device__ __forceinline__ void init(const Params& p, int pr) {
    i = 0;
    pair = pr;
    first = true;
    g = gend = 0;
    if (pr < p.sk_pairs) {
      g = sk_begin(p, pr);
      gend = sk_begin(p, pr + 1);
    }
  }
  __device__ __forceinline__ bool next(const Params& p, int kblocks, int64_t n_pairs, Seg& s) {
    const int64_t t = pair + static_cast<int64_t>(i) * n_pairs;
    if (t < p.dp_tiles) {
      ++i;
      s.tile = t;
      s.kb0 = 0;
      s.kb1 = kblocks;
      s.sk_tile = -1;
      s.slot = 0;
      return true;
    }
    if (g < gend) {
      s.sk_tile = g / kblocks;
      s.tile = p.dp_tiles + s.sk_tile;
      s.kb0 = static_cast<int>(g - s.sk_tile * kblocks);
      const int64_t left = gend - g;
      s.kb1 = left < kblocks - s.kb0 ? s.kb0 + static_cast<int>(left) : kblocks;
      s.slot = first ? 0 : 1;
      first = false;
      g += s.kb1 - s.kb0;
      return true;
    }
    return false;
  }
};

// Adds `add` k-blocks to a split tile's counter; true for the contributor
// that completes the tile (which then resets the counter).  Values tagged
// with another launch's epoch count as zero.
__device__ __forceinline__ bool sk_arrive(unsigned long long* w, uint32_t epoch, int add,
                                          int kblocks) {
  unsigned long long old = atomicAdd(w, 0ull), seen;
  uint32_t done = 0;
  for (int tries = 0; tries < (1 << 20); ++tries) {
    const uint32_t have = (static_cast<uint32_t>(old >> 32) == epoch) ? static_cast<uint32_t>(old)
                                                                       : 0u;
    done = have + static_cast<uint32_t>(add);
    const unsigned long long nv = (static_cast<unsigned long long>(epoch) << 32) | done;
    seen = atomicCAS(w, old, nv);
    if (seen == old) break;
    old = seen;
  }
  if (done != static_cast<uint32_t>(kblocks)) return false;
  atomicExch(w, 0ull);
  return true;
}

// ------------------------------------------------------------------ per-row selection
template <int NC>
struct TopN {
  float v[NC];
  int c[NC];
  __device__ __forceinline__ void init() {
#pragma unroll
    for (int i = 0; i < NC; ++i) {
      v[i] = -INFINITY;
      c[i] = -1;
    }
  }
  // Larger value first; an equal value never displaces an earlier entry, so
  // feeding columns in increasing order breaks ties toward the lower column.
  __device__ __forceinline__ void push(float x, int col) {
    if (!(x > v[NC - 1])) return;
    insert(x, col);
  }
  // Branch-free insert.  ge[i] = (v[i] >= x) holds exactly for the slots
  // before x's position (the list is sorted, and never holds a NaN: push
  // rejects one and the candidate pass never lists one), so every slot is
  // one select between keeping its entry, taking x, or taking its
  // predecessor -- two dependent selects after one compare, no position
  // count.  A value not above the n-th largest leaves the list unchanged.
  __device__ __forceinline__ void insert(float x, int col) {
    bool ge[NC];
#pragma unroll
    for (int i = 0; i < NC; ++i) ge[i] = v[i] >= x;
#pragma unroll
    for (int i = NC - 1; i > 0; --i) {
      v[i] = ge[i] ? v[i] : (ge[i - 1] ? x : v[i - 1]);
      c[i] = ge[i] ? c[i] : (ge[i - 1] ? col : c[i - 1]);
    }
    v[0] = ge[0] ? v[0] : x;
    c[0] = ge[0] ? c[0] : col;
  }
};

template <int N>
__device__ __forceinline__ float tree_max(const float (&x)[N]) {
  float t[N / 2];
#pragma unroll
  for (int i = 0; i < N / 2; ++i) t[i] = fmaxf(x[2 * i], x[2 * i + 1]);
#pragma unroll
  for (int w = N / 4; w >= 1; w >>= 1)
#pragma unroll
    for (int i = 0; i < w; ++i) t[i] = fmaxf(t[2 * i], t[2 * i + 1]);
  return t[0];
}

// The K-th largest of N values (N a power of two): bitonic sort, descending.
template <int N, int K>
__device__ __forceinline__ float nth_largest(float (&a)[N]) {
  if constexpr (K == N) {
    float t = a[0];
#pragma unroll
    for (int i = 1; i < N; ++i) t = fminf(t, a[i]);
    return t;
  } else if constexpr (K == 1) {
    return tree_max<N>(a);
  } else {
#pragma unroll
    for (int k = 2; k <= N; k <<= 1)
#pragma unroll
      for (int j = k >> 1; j > 0; j >>= 1)
#pragma unroll
        for (int i = 0; i < N; ++i) {
          const int l = i ^ j;
          if (l > i) {
            const float hi = fmaxf(a[i], a[l]), lo = fminf(a[i], a[l]);
            const bool desc = (i & k) == 0;
            a[i] = desc ? hi : lo;
            a[l] = desc ? lo : hi;
          }
        }
    return a[K - 1];
  }
}

// One 32-column chunk of this warp's 32 rows from TMEM (warp-collective):
// the child mask applied (non-children are -inf) and the bias added.
__device__ __forceinline__ void load_chunk(uint32_t taddr, int chunk, const uint32_t (&m)[BN / 32],
                                           bool has_bias, const float* sbias, float (&x)[32]) {
  uint32_t v[32];
  __syncwarp();
  tmem_ld32(taddr + chunk * 32, v);
  uint32_t mw = 0;
#pragma unroll
  for (int i = 0; i < BN / 32; ++i) mw = (i == chunk) ? m[i] : mw;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    float y = __uint_as_float(v[i]);
    if (has_bias) y += sbias[chunk * 32 + i];
    x[i] = ((mw >> i) & 1u) ? y : -INFINITY;
  }
}

// Partial accumulators of split tiles: per (pair, slot, rank) a [BM, BN]
// fp32 block stored as [chunk][vec][row][4] so that a warp's 16-byte
// accesses to one (chunk, vec) are 512 contiguous bytes.
__device__ __forceinline__ float4* part_at(const Params& p, int64_t q, int slot, uint32_t rank,
                                           int chunk, int vec, int r_local) {
  return reinterpret_cast<float4*>(p.sk_part) +
         ((q * 2 + slot) * 2 + rank) * (BM * BN / 4) + (chunk * 8 + vec) * BM + r_local;
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
      "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]),
      "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]),
      "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}

// The finisher of a split tile: the sum of every contributor's partial
// (contributors in pair order, so the result does not depend on which pair
// finishes) replaces this warp's 32 rows x 128 columns of the TMEM buffer.
__device__ __forceinline__ void sum_partials_to_tmem(const Params& p, int64_t sk_tile, int kblocks,
                                                  uint32_t rank, int r_local, int c0,
                                                  uint32_t taddr) {
  const int64_t q0 = sk_owner(p, sk_tile * kblocks);
  const int64_t q1 = sk_owner(p, (sk_tile + 1) * kblocks - 1);
#pragma unroll 1
  for (int ci = 0; ci < BN / 64; ++ci) {
    const int chunk = c0 + ci;
    float acc[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) acc[i] = 0.f;
#pragma unroll 1
    for (int64_t q = q0; q <= q1; ++q) {
      const int slot = (sk_begin(p, q) / kblocks == sk_tile) ? 0 : 1;
      float4 f[8];
#pragma unroll
      for (int v = 0; v < 8; ++v) f[v] = __ldcg(part_at(p, q, slot, rank, chunk, v, r_local));
#pragma unroll
      for (int v = 0; v < 8; ++v) {
        acc[4 * v] += f[v].x;
        acc[4 * v + 1] += f[v].y;
        acc[4 * v + 2] += f[v].z;
        acc[4 * v + 3] += f[v].w;
      }
    }
    uint32_t u[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) u[i] = __float_as_uint(acc[i]);
    __syncwarp();
    tmem_st32(taddr + chunk * 32, u);
  }
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Exact per-row path for a row whose node is outside the index or whose
// children are not a clean sorted in-window set (slow, never taken for a
// sorted catalog trie queried at the right depth).
// With `sample`, the value pushed for slot j is the Gumbel score
// logit / temp + g(row * mb + j) and no log-sum-exp is formed.
template <int NC>
__device__ void row_scalar(const Params& p, int64_t row, int64_t start, int count, TopN<NC>& t,
                           float& lse, bool sample, float temp) {
  const __nv_bfloat16* ar = p.a + row * p.a_stride;
  float m = -INFINITY, s = 0.f;
  for (int j = 0; j < count; ++j) {
    const int64_t col = __ldg(p.csr.cols + start + j);
    if (col < 0 || col >= p.n_vocab) continue;
    const __nv_bfloat16* wr = p.w + col * p.w_stride;
    float acc = 0.f;
    for (int64_t h = 0; h < p.H; ++h)
      acc = fmaf(__bfloat162float(ar[h]), __bfloat162float(wr[h]), acc);
    if (p.bias) acc += __bfloat162float(p.bias[col]);
    if (acc > m) {
      s = s * __expf(m - acc) + 1.f;
      m = acc;
    } else {
      s += __expf(acc - m);
    }
    if (sample)
      t.push(acc / temp + gumbel_at(p.seed, static_cast<uint32_t>(row * p.mb + j)), j);
    else
      t.push(acc, j);  // slot index; mapped to token / node by the caller
  }
  lse = (m > -INFINITY) ? m + __logf(s) : -INFINITY;
}

// SAMPLE: Gumbel-max sampling (NC == 1) instead of top-n + log-sum-exp.
// SPLIT: the split-window variant for launches with fewer 256-row tiles than
// SM pairs.  Both CTAs of a cluster take the same 128 rows; CTA r multiplies
// them by window columns [128 r, 128 r + 128) with its own cta_group::1 MMAs
// (M = 128, N = 128), so a tile's MMA chain and each epilogue warp's columns
// are half as long.  CTA 1 hands its partial result to CTA 0 through
// distributed shared memory; CTA 0 writes the outputs.
template <int NC, bool SAMPLE, bool SPLIT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
beam_step_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                 const Params p) {
  using Shared = SharedT<SPLIT, NC, SAMPLE>;
  using LR = ListRows<NC>;
  constexpr int ST = Shared::ST;
  constexpr int64_t TILE_ROWS = SPLIT ? BM : PAIR_M;
  constexpr int BUF_COLS = SPLIT ? BN / 2 : BN;  // TMEM columns of one accumulator
  constexpr uint32_t ALLOC_COLS = 2 * BUF_COLS;
  constexpr int NCW = SPLIT ? BN / 128 : BN / 64;  // 32-column chunks per epilogue warp
  extern __shared__ uint8_t smem_raw[];
  Shared& S = *reinterpret_cast<Shared*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                         ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();            // 0 = pair leader (issues the MMAs)
  const int64_t pair = blockIdx.x >> 1;
  const int64_t n_pairs = gridDim.x >> 1;
  const int kblocks = static_cast<int>((p.H + BK - 1) / BK);
  volatile int* abort = &S.abort;
  if (threadIdx.x == 0) TRACE(0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) {
      mbar_init(&S.full[s], 1);   // leader: its expect_tx arrival + both CTAs' bytes
      mbar_init(&S.empty[s], 1);  // both: the leader's MMA commit
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&S.tfull[b], 1);  // both: the leader's MMA commit
      // pair: every epilogue warp of both CTAs arrives on the leader's; split: own warps
      mbar_init(&S.tempty[b], SPLIT ? EPI_WARPS : 2 * EPI_WARPS);
    }
    for (int g = 0; g < 4; ++g) {
      // one arrival per warp (lane 0 after the warp's writes; see warp_arrive)
      mbar_init(&S.merge_full[g], 1);
      mbar_init(&S.merge_empty[g], 1);
      mbar_init(&S.xmerge_full[g], 1);
      mbar_init(&S.xmerge_empty[g], 1);
    }
    mbar_init(&S.mma_done, 1);
    mbar_init(&S.epi_sync, EPI_WARPS);
    S.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {  // same warp and same smem offset in both CTAs
    if constexpr (SPLIT) {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                       su32(&S.tmem_base)),
                   "r"(ALLOC_COLS)
                   : "memory");
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    } else {
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                       su32(&S.tmem_base)),
                   "r"(ALLOC_COLS)
                   : "memory");
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
  }
  for (int i = threadIdx.x; i < BN; i += THREADS) {
    const int64_t col = p.window_lo + i;
    S.bias[i] =
        (p.bias && i < p.window_n && col < p.n_vocab) ? __bfloat162float(p.bias[col]) : 0.f;
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers exist before any cross-CTA signal
  tc_fence_after();
  const uint32_t tmem = S.tmem_base;
  if (threadIdx.x == 0) TRACE(1);
  // Programmatic dependent launch (inside a search): the next kernel (the
  // merge) may be scheduled now; it waits for this grid's results itself.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer (both CTAs)
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmW)) : "memory");
      uint32_t armed[ST] = {};
      [[maybe_unused]] long long prof_wait = 0;
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      const int wrow = static_cast<int>(p.window_lo) + static_cast<int>(rank) * (BN / 2);
      SegIter seg;
      seg.init(p, static_cast<int>(pair));
      Seg sg;
      while (ok && seg.next(p, kblocks, n_pairs, sg)) {
        const int arow = static_cast<int>(sg.tile * TILE_ROWS) + (SPLIT ? 0 : static_cast<int>(rank) * BM);
        for (int kb = sg.kb0; kb < sg.kb1; ++kb) {
          PROF_T0(t_w);
          if (!wait_phase(&S.empty[stage], phase ^ 1, abort, 1, p.wait_ns)) {
            ok = false;
            break;
          }
          PROF_ACC(prof_wait, t_w);
          uint8_t* st = S.ring[stage];
          if (p.stall) {  // test hook: no copies, so the consumers' waits run out
            if (++stage == ST) {
              stage = 0;
              phase ^= 1;
            }
            continue;
          }
          if constexpr (SPLIT) {  // this CTA's own barrier and bytes
            mbar_expect_tx(&S.full[stage], STAGE_BYTES);
            tma_load_2d(st, &tmA, &S.full[stage], kb * BK, arow);
            tma_load_2d(st + A_BYTES, &tmW, &S.full[stage], kb * BK, wrow);
          } else {
#ifdef VTNK_TC_EXPERIMENT_NOW
            // tuning experiment only (outputs meaningless): A copies alone
            if (rank == 0) mbar_expect_tx(&S.full[stage], 2 * A_BYTES);
#else
            if (rank == 0) mbar_expect_tx(&S.full[stage], 2 * STAGE_BYTES);
#endif
            const uint32_t lbar = map_to_rank(&S.full[stage], 0);
            tma_load_2d_pair(st, &tmA, lbar, kb * BK, arow);
#ifndef VTNK_TC_EXPERIMENT_NOW
            tma_load_2d_pair(st + A_BYTES, &tmW, lbar, kb * BK, wrow);
#endif
          }
#ifdef VTNK_TC_PREFETCH
          // tuning option: pull this tile's A k-block VTNK_TC_PREFETCH stages
          // ahead into L2, so its copy later hits L2
          if (kb + VTNK_TC_PREFETCH < sg.kb1)
            asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                             reinterpret_cast<uint64_t>(&tmA)),
                         "r"((kb + VTNK_TC_PREFETCH) * BK), "r"(arow)
                         : "memory");
#endif
          if (armed[stage] == 0 && stage == 0) TRACE(2);
          ++armed[stage];
          if (++stage == ST) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // the leader's barriers count both CTAs' copies: it waits for any still in
      // flight; the peer stays resident until the teardown cluster barrier
      if (SPLIT || rank == 0)
        for (int s = 0; s < ST; ++s)
          if (armed[s]) drain_phase(&S.full[s], (armed[s] - 1) & 1, p.wait_ns);
      PROF_FLUSH(0, prof_wait);
    }
  } else if (warp == 1) {
    // ------------------------------------------- MMA issuer (pair: leader; split: each CTA)
    if (lane == 0 && (SPLIT || rank == 0)) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t it = 0;
      bool ok = true;
      [[maybe_unused]] long long prof_full = 0, prof_tempty = 0;
      SegIter seg;
      seg.init(p, static_cast<int>(pair));
      Seg sg;
      for (; ok && seg.next(p, kblocks, n_pairs, sg); ++it) {
        const uint32_t buf = it & 1;
        PROF_T0(t_e);
        if (SPLIT ? !wait_phase(&S.tempty[buf], ((it >> 1) & 1) ^ 1, abort, 2, p.wait_ns)
                  : !wait_phase_cluster(&S.tempty[buf], ((it >> 1) & 1) ^ 1, abort, 2, p.wait_ns))
          break;
        PROF_ACC(prof_tempty, t_e);
        tc_fence_after();
        const uint32_t d = tmem + buf * BUF_COLS;
        for (int kb = sg.kb0; kb < sg.kb1; ++kb) {
          PROF_T0(t_f);
          if (!wait_phase(&S.full[stage], phase, abort, 3, p.wait_ns)) {
            ok = false;
            break;
          }
          PROF_ACC(prof_full, t_f);
          if (it == 0 && kb == sg.kb0) TRACE(3);
          tc_fence_after();
          const uint64_t da = umma_desc_sw128(S.ring[stage]);
          const uint64_t db = umma_desc_sw128(S.ring[stage] + A_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {  // +32 B per K=16 step inside the swizzle atom
            const uint32_t acc = (kb != sg.kb0 || k != 0) ? 1u : 0u;
            if constexpr (SPLIT)
              umma_bf16_cta(d, da + 2 * k, db + 2 * k, acc);
            else
              umma_bf16(d, da + 2 * k, db + 2 * k, acc);
          }
          if constexpr (SPLIT)
            umma_commit_cta(&S.empty[stage]);
          else
            umma_commit_pair(&S.empty[stage]);
          if (++stage == ST) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (ok) {
          if constexpr (SPLIT)
            umma_commit_cta(&S.tfull[buf]);
          else
            umma_commit_pair(&S.tfull[buf]);
        }
      }
      TRACE(4);
      if constexpr (SPLIT)
        umma_commit_cta(&S.mma_done);
      else
        umma_commit_pair(&S.mma_done);
      drain_phase(&S.mma_done, 0, p.wait_ns);
      PROF_FLUSH(1, prof_full);
      PROF_FLUSH(2, prof_tempty);
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    // The rows' nodes (and the candidate buffers) belong to the previous
    // kernel of a search: wait for it to finish.  The producer and the MMA
    // issuer only read the hidden states and the head, which no kernel of
    // the search writes, so they start streaming at once.  A no-op in a
    // plain launch.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int lg = warp & 3;             // TMEM lane group this warp may access
    // pair: half 0 = columns 0..127 (+ merge, outputs), half 1 = 128..255;
    // split: the same two halves of this CTA's 128 columns
    const int half = (warp - 2) >> 2;
    const int r_local = lg * 32 + lane;  // row within the tile == TMEM lane
    uint32_t it = 0;
    [[maybe_unused]] long long pe_pro = 0, pe_wait = 0, pe_tmem = 0, pe_out = 0, pe_ld = 0;
    const uint32_t tempty_leader[2] = {map_to_rank(&S.tempty[0], 0), map_to_rank(&S.tempty[1], 0)};
    // Give the accumulator back to the MMA issuer (every lane is done reading it).
    auto release_acc = [&](uint32_t b) {
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (SPLIT)
          mbar_arrive(&S.tempty[b]);
        else
          mbar_arrive_cluster(tempty_leader[b]);  // the leader's MMA may reuse it
      }
    };
    uint32_t mit = 0;  // hand-offs between the two column halves so far
    uint32_t xit = 0;  // split: hand-offs from CTA 1 to CTA 0 so far
    const bool edge_ids = p.flags != nullptr && (__ldg(p.flags) & 1u) != 0u;
    uint32_t eb = 0;   // epi_sync phases so far
    // All epilogue warps of the CTA meet (bounded wait; false on abort).
    auto epi_sync = [&]() {
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.epi_sync);
      const bool ok = warp_wait_phase(&S.epi_sync, eb & 1, abort, 7, p.wait_ns);
      if (ok) mbar_try_wait(&S.epi_sync, eb & 1);  // every lane acquires
      ++eb;
      return ok;
    };
    SegIter seg;
    seg.init(p, static_cast<int>(pair));
    Seg sg;
    for (; seg.next(p, kblocks, n_pairs, sg); ++it) {
      const int64_t tile = sg.tile;
      PROF_T0(t_pro);
      const int64_t row = tile * TILE_ROWS + (SPLIT ? 0 : static_cast<int64_t>(rank) * BM) + r_local;
      const bool live = row < p.rows;
      // The row's children as a 256-bit mask over the window, read from the
      // depth's child index (two 16-byte loads).  A row whose node is outside
      // the index, or whose mask does not hold exactly its `count` children
      // (unsorted / out-of-window children, or more than max_branches), takes
      // the exact per-row path.
      int64_t start = 0;
      int count = 0;
      uint32_t m[BN / 32];
#pragma unroll
      for (int i = 0; i < BN / 32; ++i) m[i] = 0u;
      int spill = 0;
      if (live) {
        // written by the previous kernel of a search (a PDL predecessor): a
        // coherent load, never the non-coherent read-only path
        const int64_t cur = p.cur_node ? ld_relaxed_s64(p.cur_node + row) : 0;
        node_children(p.csr, cur, p.mb, start, count);
        if (cur >= p.idx_lo && cur < p.idx_hi) {
          const uint4* q = reinterpret_cast<const uint4*>(p.masks + (cur - p.idx_lo) * (BN / 32));
          const uint4 x = __ldg(q), y = __ldg(q + 1);
          m[0] = x.x; m[1] = x.y; m[2] = x.z; m[3] = x.w;
          m[4] = y.x; m[5] = y.y; m[6] = y.z; m[7] = y.w;
        }
        int pc = 0;
#pragma unroll
        for (int i = 0; i < BN / 32; ++i) pc += __popc(m[i]);
        spill = pc != count;
      }

      PROF_ACC(pe_pro, t_pro);
      PROF_T0(t_wt);
      const uint32_t buf = it & 1;
      const bool ok = warp_wait_phase(&S.tfull[buf], (it >> 1) & 1, abort, 4, p.wait_ns);
      if (!ok) break;
      // every lane observes the completed phase before touching TMEM
      mbar_try_wait(&S.tfull[buf], (it >> 1) & 1);
      tc_fence_after();
      if (warp == 2 && lane == 0 && it == 0) TRACE(5);
      PROF_ACC(pe_wait, t_wt);
      PROF_T0(t_tm);
#ifdef VTNK_TC_EXPERIMENT_NOEPI
      // tuning experiment only (no outputs written): release the accumulator at once
      release_acc(buf);
      continue;
#endif

      // TMEM address of window chunk c is taddr + 32 c (split: this CTA's
      // chunks 4 r .. 4 r + 3 map to its buffer's columns 0..127).
      const uint32_t taddr = tmem + (static_cast<uint32_t>(lg * 32) << 16) + buf * BUF_COLS -
                             (SPLIT ? rank * (BN / 2) : 0u);
      const bool has_bias = p.bias != nullptr;
      // this warp's first 32-column chunk of the window
      const int c0 = SPLIT ? static_cast<int>(rank) * (BN / 64) + half * NCW : half * NCW;
      // A segment that covers part of a tile stores its raw accumulator
      // (this warp's 32 rows x 128 columns) as an fp32 partial and counts
      // its k-blocks.  The contributor that completes the tile replaces its
      // TMEM buffer by the sum of all partials and runs the epilogue; the
      // others free the buffer.
      if constexpr (!SPLIT) {  // stream-K (whole tiles only in the split variant)
        if (sg.kb0 != 0 || sg.kb1 != kblocks) {
          // This CTA's raw accumulator of the segment (coalesced fp32 partial).
#pragma unroll 1
          for (int ci = 0; ci < BN / 64; ++ci) {
            uint32_t v[32];
            __syncwarp();
            tmem_ld32(taddr + (c0 + ci) * 32, v);
#pragma unroll
            for (int q = 0; q < 8; ++q)
              __stcg(part_at(p, pair, sg.slot, rank, c0 + ci, q, r_local),
                     make_float4(__uint_as_float(v[4 * q]), __uint_as_float(v[4 * q + 1]),
                                 __uint_as_float(v[4 * q + 2]), __uint_as_float(v[4 * q + 3])));
          }
          __threadfence();
          if (!epi_sync()) break;
          if (warp == 2 && lane == 0)
            S.sk_last = sk_arrive(p.sk_count + sg.sk_tile * 2 + rank, p.sk_epoch,
                                  sg.kb1 - sg.kb0, kblocks) ? 1 : 0;
          if (!epi_sync()) break;
          const int finisher = *reinterpret_cast<volatile int*>(&S.sk_last);
          if (!finisher) {
            release_acc(buf);
            continue;
          }
          __threadfence();
          sum_partials_to_tmem(p, sg.sk_tile, kblocks, rank, r_local, c0, taddr);
        }
      }

      TopN<NC> top;  // initialised where it first comes into use (fewer live registers in pass 1)
      float mx = -INFINITY, sum = 0.f;
      const float temp = (SAMPLE && p.temperature) ? __ldg(p.temperature) : 1.f;
      if constexpr (SAMPLE) {
        // Gumbel-max over this half's children: score = logit / T + g, with
        // g drawn at the reference's flat offset row * mb + slot (int32 wrap).
        // Each lane visits its children in slot order and keeps the first
        // maximum; the lower half wins ties in the hand-off below.
        top.init();
        int pre_h = 0;  // children in the chunks before this warp's first
#pragma unroll
        for (int i = 0; i < BN / 32; ++i) pre_h += (i < c0) ? __popc(m[i]) : 0;
        float* sx = &S.chunk_x[warp - 2][0][0];
        const uint32_t off0 = static_cast<uint32_t>(row * p.mb);
#pragma unroll 1
        for (int ci = 0; ci < NCW; ++ci) {
          const int chunk = c0 + ci;
          uint32_t mw = 0;
#pragma unroll
          for (int i = 0; i < BN / 32; ++i) mw = (i == chunk) ? m[i] : mw;
          if (spill) mw = 0u;  // recomputed exactly below
          if (__any_sync(0xffffffffu, mw != 0u)) {
            float x[32];
            load_chunk(taddr, chunk, m, has_bias, S.bias, x);
            __syncwarp();
#pragma unroll
            for (int i = 0; i < 32; ++i) sx[i * 32 + lane] = x[i];
            __syncwarp();
            // Two children per iteration, in slot order: their Philox draws
            // are independent chains, so they overlap (a lane with one child
            // left draws a discarded value for the second).
            uint32_t pend = mw;
            while (__any_sync(0xffffffffu, pend != 0u)) {
              const int i1 = pend ? __ffs(pend) - 1 : -1;
              pend &= pend - 1;
              const int i2 = pend ? __ffs(pend) - 1 : -1;
              pend &= pend - 1;
              const int j1 = i1 < 0 ? 0 : i1, j2 = i2 < 0 ? j1 : i2;
              const int s1 = pre_h + __popc(mw & ((1u << j1) - 1u));
              const int s2 = pre_h + __popc(mw & ((1u << j2) - 1u));
              const float g1 = gumbel_at(p.seed, off0 + static_cast<uint32_t>(s1));
              const float g2 = gumbel_at(p.seed, off0 + static_cast<uint32_t>(s2));
              if (i1 >= 0) top.push(sx[j1 * 32 + lane] / temp + g1, chunk * 32 + j1);
              if (i2 >= 0) top.push(sx[j2 * 32 + lane] / temp + g2, chunk * 32 + j2);
            }
          }
          pre_h += __popc(mw);
        }
      } else {
        // Pass 1 over the accumulator: online log-sum-exp, and the maxima of G
        // column groups (column j of the half in group j % G).  The NC-th largest
        // group maximum is a lower bound of the NC-th largest value (the NC
        // largest group maxima are NC distinct entries), so pass 2 only inserts
        // values at or above it.
        // G >= NC groups: 16 up to NC = 16, else 32 (the NC-th largest maximum
        // by a sorting network).  With 32 groups of 4 columns a top-20 row
        // lists ~27 candidates per lane; with 20 groups of ~6, ~54.
        constexpr int G = NC <= VTNK_TC_GROUPS ? VTNK_TC_GROUPS : 32;
        float gm[G];
#pragma unroll
        for (int g = 0; g < G; ++g) gm[g] = -INFINITY;
        float cmax[NCW];
#pragma unroll
        for (int ci = 0; ci < NCW; ++ci) {
          const int chunk = c0 + ci;
          float x[32];
          load_chunk(taddr, chunk, m, has_bias, S.bias, x);
          const float cm = tree_max<32>(x);
          cmax[ci] = cm;
#pragma unroll
          for (int i = 0; i < 32; ++i) gm[i % G] = fmaxf(gm[i % G], x[i]);
          const float nm = fmaxf(mx, cm);
          sum *= (nm == mx) ? 1.f : __expf(mx - nm);
          mx = nm;
          float e[32];
#pragma unroll
          // exp(x - mx) = 2^(x log2e - mx log2e): one FFMA and one ex2 per value
          // (a -inf value gives 2^-inf = 0)
          const float nmx = mx > -INFINITY ? -mx * kLog2e : 0.f;
#pragma unroll
          for (int i = 0; i < 32; ++i) e[i] = ex2_approx(fmaf(x[i], kLog2e, nmx));
#pragma unroll
          for (int w = 16; w >= 1; w >>= 1)
#pragma unroll
            for (int i = 0; i < w; ++i) e[i] += e[i + w];
          sum += e[0];
        }
        if (warp == 2 && lane == 0 && it == 0) TRACE(8);
      const float lb = nth_largest<G, NC>(gm);
        top.init();
        // Pass 2: the values >= lb of each lane, in column order, are appended
        // to the lane's candidate list in shared memory ([slot][lane], value
        // and window column); the list is then inserted into the top-n.  The
        // warp's insert loop runs max-over-lanes(list length) times once per
        // tile instead of once per chunk; a list that could overflow its 32
        // slots is inserted early.
        float* sv = &S.chunk_x[warp - 2][0][0];
        uint8_t* sc = &S.chunk_c[warp - 2][0][0];
        int cnt = 0;
        [[maybe_unused]] long long fl_cyc = 0, fl_cnt = 0, fl_sum = 0;
        auto flush = [&]() {
          PROF_T0(t_fl);
          const int n = static_cast<int>(__reduce_max_sync(0xffffffffu, static_cast<unsigned>(cnt)));
          __syncwarp();
          float ynext = cnt > 0 ? sv[lane] : -INFINITY;
          int cnext = sc[lane];
#pragma unroll 1
          for (int j = 0; j < n; ++j) {  // software-pipelined: next read overlaps the insert
            const float y = ynext;
            const int col = cnext;
            ynext = j + 1 < cnt ? sv[(j + 1) * 32 + lane] : -INFINITY;
            cnext = sc[((j + 1) % Shared::CS) * 32 + lane];
            top.insert(y, col);  // no-op for -inf / values not above the n-th best
          }
          cnt = 0;
          __syncwarp();
          if (warp == 2 && lane == 0 && it == 0) TRACE_VAL(14, n);
          PROF_ACC(fl_cyc, t_fl);
#ifdef VTNK_TC_PROFILE
          ++fl_cnt;
          fl_sum += n;
#endif
        };
#pragma unroll 1
        for (int ci = 0; ci < NCW; ++ci) {
#ifdef VTNK_TC_EXPERIMENT_NOPASS2
          break;  // tuning experiment only: pass 1 alone
#endif
          if (!__any_sync(0xffffffffu, cmax[ci] >= lb && cmax[ci] > -INFINITY)) continue;
          const int chunk = c0 + ci;
          float x[32];
          load_chunk(taddr, chunk, m, has_bias, S.bias, x);
#ifdef VTNK_TC_PROFILE
          if (warp == 2 && lane == 0 && it == 0) {
            float z = 0.f;
#pragma unroll
            for (int i = 0; i < 32; ++i) z += x[i];
            if (z != 1234.5f) TRACE(16 + 2 * ci);
          }
#endif
          // the candidate bits, ORed in four independent chains
          uint32_t pq[4] = {0u, 0u, 0u, 0u};
#pragma unroll
          for (int i = 0; i < 32; ++i)
            pq[i & 3] |= (x[i] >= lb && x[i] > -INFINITY) ? (1u << i) : 0u;
          uint32_t pend = (pq[0] | pq[1]) | (pq[2] | pq[3]);
#ifdef VTNK_TC_EXPERIMENT_NOSELECT
          pend = 0u;  // tuning experiment only: measures the pipeline without top-n work
#endif
#pragma unroll
          for (int h = 0; h < 2; ++h) {  // 16 columns at a time: at most 16 new entries
            if (__any_sync(0xffffffffu, cnt + __popc((pend >> (16 * h)) & 0xFFFFu) > Shared::CS))
              flush();
#pragma unroll
            for (int i = 16 * h; i < 16 * h + 16; ++i) {
              // Branch-free: every column is written to slot cnt and counted
              // only when listed; an unlisted column's write is overwritten
              // by the next listed one or lies past the list's end (slots
              // >= cnt are never read).  cnt < CS always holds while listed
              // columns remain in this half (checked above).
              if (cnt < Shared::CS) {
                sv[cnt * 32 + lane] = x[i];
                sc[cnt * 32 + lane] = static_cast<uint8_t>(chunk * 32 + i);
              }
              cnt += static_cast<int>((pend >> i) & 1u);
            }
          }
          if (warp == 2 && lane == 0 && it == 0) TRACE(17 + 2 * ci);
        }
        if (warp == 2 && lane == 0 && it == 0) TRACE(13);
        flush();
        if (warp == 2 && lane == 0 && it == 0) {
          TRACE_VAL(26, fl_cyc);
          TRACE_VAL(27, fl_cnt);
          TRACE_VAL(28, fl_sum);
        }
      }
      __syncwarp();
      release_acc(buf);

      if (warp == 2 && lane == 0 && it == 0) TRACE(9);
      // A partial result (top-n, max, sum) travels as rows of a [*][32] table
      // (lane = row): NC values, NC byte-packed columns (window columns are
      // < 256; 0xFF = none), max, sum.
      auto put_list = [&](auto store) {
#pragma unroll
        for (int j = 0; j < NC; ++j) store(j, top.v[j]);
#pragma unroll
        for (int j = 0; j < NC; j += 4) {
          uint32_t w = 0;
#pragma unroll
          for (int q = 0; q < 4; ++q)
            if (j + q < NC) w |= static_cast<uint32_t>(top.c[j + q] & 0xFF) << (8 * q);
            else w |= 0xFFu << (8 * q);
          store(LR::COLS + j / 4, __uint_as_float(w));
        }
        store(LR::MX, mx);
        store(LR::SUM, sum);
      };
      // Merges a table written by put_list whose columns are all higher than
      // this warp's: inserting its sorted list after ours keeps ties on the
      // lower column.
      auto absorb = [&](float (*src)[32]) {
        const float omx = src[LR::MX][lane];
        const float osum = src[LR::SUM][lane];
        const float nm = fmaxf(mx, omx);
        sum = (mx > -INFINITY ? sum * __expf(mx - nm) : 0.f) +
              (omx > -INFINITY ? osum * __expf(omx - nm) : 0.f);
        mx = nm;
        // Two sorted lists, ours with the lower columns: a two-pointer merge
        // through shared memory (our list goes to this warp's candidate
        // slots), ties to ours, i.e. to the lower column.
        float* ov = &S.chunk_x[warp - 2][0][0];
        uint8_t* oc = &S.chunk_c[warp - 2][0][0];
        __syncwarp();
#pragma unroll
        for (int j = 0; j < NC; ++j) {
          ov[j * 32 + lane] = top.v[j];
          oc[j * 32 + lane] = static_cast<uint8_t>(top.c[j] & 0xFF);
        }
        __syncwarp();
        int ia = 0, ib = 0;
#pragma unroll
        for (int j = 0; j < NC; ++j) {
          const float va = ia < NC ? ov[ia * 32 + lane] : -INFINITY;
          const int ca = oc[(ia < NC ? ia : 0) * 32 + lane];
          const int ibc = ib < NC ? ib : 0;
          const float vb = ib < NC ? src[ibc][lane] : -INFINITY;
          const int cb = static_cast<int>(
              (__float_as_uint(src[LR::COLS + ibc / 4][lane]) >> (8 * (ibc & 3))) & 0xFFu);
          const bool take_a = !(vb > va);
          const float v = take_a ? va : vb;
          top.v[j] = v;
          top.c[j] = v > -INFINITY ? (take_a ? ca : cb) : -1;
          ia += take_a ? 1 : 0;
          ib += take_a ? 0 : 1;
        }
        __syncwarp();
      };

      // The upper-half warp hands its partial result to the lower-half warp
      // of the same rows through shared memory; bounded waits on both sides.
      float (*mg)[32] = S.merge[lg];
      if (half == 1) {
        if (!warp_wait_phase(&S.merge_empty[lg], (mit & 1) ^ 1, abort, 5, p.wait_ns)) break;
        mbar_try_wait(&S.merge_empty[lg], (mit & 1) ^ 1);
        put_list([&](int r, float v) { mg[r][lane] = v; });
        warp_arrive(&S.merge_full[lg]);
        ++mit;
        PROF_ACC(pe_tmem, t_tm);
        continue;
      }
      if (!warp_wait_phase(&S.merge_full[lg], mit & 1, abort, 6, p.wait_ns)) break;
      mbar_try_wait(&S.merge_full[lg], mit & 1);
      absorb(mg);
      warp_arrive(&S.merge_empty[lg]);
      ++mit;
      if (warp == 2 && lane == 0 && it == 0) TRACE(10);

      if constexpr (SPLIT) {
        // CTA 1 (window columns 128..255) hands its rows' result to CTA 0
        // through distributed shared memory (remote stores, release/acquire
        // at cluster scope on the barriers); CTA 0 writes the outputs.
        if (rank == 1) {
          if (!warp_wait_phase_cluster(&S.xmerge_empty[lg], (xit & 1) ^ 1, abort, 8, p.wait_ns)) break;
          put_list([&](int r, float v) { st_cluster_f32(map_to_rank(&S.xm.x[lg][r][lane], 0), v); });
          warp_arrive_cluster(map_to_rank(&S.xmerge_full[lg], 0));
          ++xit;
          PROF_ACC(pe_tmem, t_tm);
          continue;
        }
        if (!warp_wait_phase_cluster(&S.xmerge_full[lg], xit & 1, abort, 9, p.wait_ns)) break;
        absorb(S.xm.x[lg]);
        warp_arrive_cluster(map_to_rank(&S.xmerge_empty[lg], 1));
        ++xit;
      }

      PROF_ACC(pe_tmem, t_tm);
      PROF_T0(t_out);
      if (warp == 2 && lane == 0 && it == 0) TRACE(11);
      float lse = (mx > -INFINITY) ? mx + __logf(sum) : -INFINITY;
      bool by_slot = false;
      if (spill && live) {  // exact scalar recompute of this row
        top.init();
        row_scalar<NC>(p, row, start, count, top, lse, SAMPLE, temp);
        by_slot = true;
      }
      if (warp == 2 && lane == 0 && it == 0) TRACE(12);
      if (live) {
        int pre[BN / 32];
        int acc = 0;
#pragma unroll
        for (int i = 0; i < BN / 32; ++i) {
          pre[i] = acc;
          acc += __popc(m[i]);
        }
        const int64_t o = row * p.n_cand;
        // candidate j of this row: token, node id and value (-1 / -inf when none)
        auto cand_at = [&](int j, int64_t& tok, int64_t& node, float& lv) {
          const int c = top.c[j];
          tok = -1;
          node = -1;
          lv = -INFINITY;
          if (c >= 0) {
            int slot;
            if (by_slot) {
              slot = c;
              tok = __ldg(p.csr.cols + start + slot);
            } else {
              const int wi = c >> 5;
              int base = 0;
              uint32_t word = 0;
#pragma unroll
              for (int i = 0; i < BN / 32; ++i) {
                base = (i == wi) ? pre[i] : base;
                word = (i == wi) ? m[i] : word;
              }
              slot = base + __popc(word & ((1u << (c & 31)) - 1u));
              tok = p.window_lo + c;
            }
            // BFS-numbered depth (checked when the index was built): the child's
            // node id is its edge index + 1, no random read of vals
            node = (edge_ids && !by_slot) ? start + slot + 1 : __ldg(p.csr.vals + start + slot);
            lv = top.v[j];
          }
        };
        bool stored = false;
        if constexpr (NC % 2 == 0) {
          // Two candidates per store (16-byte token / node pairs, 8-byte value
          // pairs) when the host found every output aligned and n_cand (and
          // the level-0 beam count) even: half the store instructions and
          // the L2 sectors of the lane-per-row layout.
          if (p.vec_out) {
#pragma unroll
            for (int j = 0; j < NC; j += 2) {
              if (j >= p.n_cand) break;
              int64_t t0, t1, n0, n1;
              float v0, v1;
              cand_at(j, t0, n0, v0);
              cand_at(j + 1, t1, n1, v1);
              if (p.cand_tok) *reinterpret_cast<longlong2*>(p.cand_tok + o + j) = make_longlong2(t0, t1);
              if (p.cand_logit) *reinterpret_cast<float2*>(p.cand_logit + o + j) = make_float2(v0, v1);
              if (p.cand_node) *reinterpret_cast<longlong2*>(p.cand_node + o + j) = make_longlong2(n0, n1);
              if (p.l0_ids && j < p.l0_k) {  // level 0: the row's j-th best child is its beam j
                const int64_t ob = row * p.l0_k + j;
                *reinterpret_cast<longlong2*>(p.l0_ids + ob) = make_longlong2(t0, t1);
                *reinterpret_cast<float2*>(p.l0_logp + ob) =
                    make_float2(v0 > -INFINITY ? v0 - lse : -INFINITY, v1 > -INFINITY ? v1 - lse : -INFINITY);
                *reinterpret_cast<longlong2*>(p.l0_node + ob) = make_longlong2(n0, n1);
              }
            }
            stored = true;
          }
        }
        if (!stored) {
#pragma unroll
          for (int j = 0; j < NC; ++j) {
            if (j >= p.n_cand) break;
            int64_t tok, node;
            float lv;
            cand_at(j, tok, node, lv);
#ifdef VTNK_TC_EXPERIMENT_NOOUT
            if (lv != 12345.f) continue;  // tuning experiment only: outputs (almost) never stored
#endif
            if (p.cand_tok) p.cand_tok[o + j] = tok;
            if (p.cand_logit) p.cand_logit[o + j] = lv;  // sampling: the winning score
            if (p.cand_node) p.cand_node[o + j] = node;
            if (p.l0_ids && j < p.l0_k) {  // level 0: the row's j-th best child is its beam j
              const int64_t ob = row * p.l0_k + j;
              p.l0_ids[ob] = tok;
              p.l0_logp[ob] = lv > -INFINITY ? lv - lse : -INFINITY;
              p.l0_node[ob] = node;
            }
            if (SAMPLE && p.sample_f) p.sample_f[row] = tok >= 0 ? static_cast<float>(tok) : -1.f;
          }
        }
        if (p.row_lse) p.row_lse[row] = lse;
      }
      if (warp == 2 && lane == 0 && it == 0) TRACE(6);
      PROF_ACC(pe_out, t_out);
    }
    if (lane == 0) {
      PROF_FLUSH(3, pe_pro);
      PROF_FLUSH(4, pe_wait);
      PROF_FLUSH(5, pe_tmem);
      PROF_FLUSH(6, pe_out);
      PROF_FLUSH(7, pe_ld);
    }
  }

  // ------------------------------------------------------------------ teardown
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the pair's MMAs and copies are done before either CTA frees or exits
  if (threadIdx.x == 0) TRACE(7);
  if (warp == 1) {
    tc_fence_after();
    if constexpr (SPLIT)
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                   "r"(ALLOC_COLS)
                   : "memory");
    else
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                   "r"(ALLOC_COLS)
                   : "memory");
  }
}

// Child-bitmask index: one warp per node.  Bits for children inside the
// window; an all-zero mask when a child is outside it or out of order.
// `flags` (optional, preset to bit 0 = 1 by the host): bit 0 is cleared when
// a child's node id is not its edge index + 1.
__global__ void build_index_kernel(const Csr csr, uint32_t* __restrict__ masks,
                                   uint32_t* __restrict__ flags, int64_t node_lo,
                                   int64_t node_hi, int64_t window_lo, int window_n) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t node = node_lo + static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) +
                      (threadIdx.x >> 5);
       node < node_hi; node += warps) {
    int64_t start;
    int count;
    node_children(csr, node, INT32_MAX, start, count);
    uint32_t word[BN / 32];
#pragma unroll
    for (int i = 0; i < BN / 32; ++i) word[i] = 0u;
    int bad = 0;
    int not_bfs = 0;
    int64_t carry = INT64_MIN;
    for (int j0 = 0; j0 < count; j0 += 32) {
      const int j = j0 + lane;
      const bool has = j < count;
      const int64_t t = has ? __ldg(csr.cols + start + j) - window_lo : INT64_MAX;
      int64_t tp = __shfl_up_sync(0xffffffffu, t, 1);
      if (lane == 0) tp = carry;
      carry = __shfl_sync(0xffffffffu, t, 31);
      const bool inwin = has && t >= 0 && t < window_n;
      if (has && __ldg(csr.vals + start + j) != start + j + 1) not_bfs = 1;
      if (has && (!inwin || t <= tp)) bad = 1;
#pragma unroll
      for (int i = 0; i < BN / 32; ++i) {
        const uint32_t bit = (inwin && (t >> 5) == i) ? (1u << (t & 31)) : 0u;
        word[i] |= __reduce_or_sync(0xffffffffu, bit);
      }
    }
    bad = __any_sync(0xffffffffu, bad);
    if (flags && __any_sync(0xffffffffu, not_bfs) && lane == 0) atomicAnd(flags, ~1u);
    if (lane < BN / 32) {
      uint32_t w = 0;
#pragma unroll
      for (int i = 0; i < BN / 32; ++i) w = (i == lane) ? word[i] : w;
      masks[(node - node_lo) * (BN / 32) + lane] = bad ? 0u : w;
    }
  }
}

// ------------------------------------------------------------------ host side
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* f = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

bool make_map(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer,
              uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t es[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
            es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int sm_count() {
  constexpr int kMaxDev = 64;
  static std::atomic<int> cached[kMaxDev] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < kMaxDev && cached[dev] > 0) return cached[dev];
  int n = 148;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (dev >= 0 && dev < kMaxDev) cached[dev] = n;
  return n;
}

template <int NC, bool SAMPLE, bool SPLIT>
int launch_variant(const CUtensorMap& a, const CUtensorMap& w, const Params& p, int pairs,
                   bool pdl, cudaStream_t s) {
  auto k = beam_step_kernel<NC, SAMPLE, SPLIT>;
  constexpr size_t smem = smem_bytes<SPLIT, NC, SAMPLE>();
  // The shared-memory opt-in is per kernel and device; set it once each.
  static std::atomic<uint64_t> set_on{0};  // bit d: done on device d
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64 || !((set_on.load(std::memory_order_relaxed) >> dev) & 1)) {
    const cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(smem));
    if (e != cudaSuccess) return cuda_status(e, "beam_step_tc smem attribute");
    if (dev < 64) set_on.fetch_or(1ull << dev, std::memory_order_relaxed);
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs));
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cuda_status(cudaLaunchKernelEx(&cfg, k, a, w, p), "beam_step_tc launch");
}

template <int NC, bool SAMPLE = false>
int launch_nc(const CUtensorMap& a, const CUtensorMap& w, const Params& p, int pairs, bool split,
              bool pdl, cudaStream_t s) {
  return split ? launch_variant<NC, SAMPLE, true>(a, w, p, pairs, pdl, s)
               : launch_variant<NC, SAMPLE, false>(a, w, p, pairs, pdl, s);
}

}  // namespace tc

bool tc_enabled() {
  static int enabled = -1;
  if (enabled < 0) {
    const char* e = getenv("VTNK_DISABLE_TC");
    enabled = (e && e[0] == '1') ? 0 : 1;
  }
  return enabled == 1;
}

// Bound of the tile kernel's waits (ns) and the test hook's pending stalled
// launches; process-wide, read at each launch.
static std::atomic<uint64_t> g_wait_limit_ns{tc::WAIT_LIMIT_NS};
static std::atomic<int> g_stall_launches{0};

int launch_beam_step_tc(const TcArgs& t, cudaStream_t s) {
  using namespace tc;
  auto aligned = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  if (!t.masks || !aligned(t.masks) || t.idx_hi < t.idx_lo || t.window_n < 1 ||
      t.window_lo + BN > (int64_t(1) << 31) ||
      t.window_n > BN || t.n_cand < 1 || t.n_cand > 32 || t.rows < 1 || t.H % 8 != 0 ||
      t.a_stride % 8 != 0 || t.w_stride % 8 != 0 || !aligned(t.a) || !aligned(t.w) || t.mb < 1 ||
      t.window_lo < 0 || t.rows > (int64_t(1) << 31) - BM)
    return VTNK_ERR_UNSUPPORTED;
  Params p{};
  p.rows = t.rows;
  p.H = t.H;
  p.cur_node = t.cur_node;
  p.csr = t.csr;
  p.mb = t.mb;
  p.window_lo = t.window_lo;
  p.window_n = t.window_n;
  p.n_cand = t.n_cand;
  p.masks = t.masks;
  p.flags = t.flags;
  p.idx_lo = t.idx_lo;
  p.idx_hi = t.idx_hi;
  p.a = static_cast<const __nv_bfloat16*>(t.a);
  p.a_stride = t.a_stride;
  p.w = static_cast<const __nv_bfloat16*>(t.w);
  p.w_stride = t.w_stride;
  p.bias = static_cast<const __nv_bfloat16*>(t.bias);
  p.n_vocab = t.n_vocab;
  p.cand_tok = t.cand_tok;
  p.cand_logit = t.cand_logit;
  p.cand_node = t.cand_node;
  p.row_lse = t.row_lse;
  p.seed = t.seed;
  p.temperature = t.temperature;
  p.sample_f = t.sample_f;
  p.l0_ids = t.l0_ids;
  p.l0_logp = t.l0_logp;
  p.l0_node = t.l0_node;
  p.l0_k = t.l0_k;
  {
    auto aligned = [](const void* q, uintptr_t a) {
      return q == nullptr || reinterpret_cast<uintptr_t>(q) % a == 0;
    };
    const bool l0_ok = t.l0_ids == nullptr ||
                       (t.l0_k % 2 == 0 && aligned(t.l0_ids, 16) && aligned(t.l0_node, 16) &&
                        aligned(t.l0_logp, 8));
    p.vec_out = (t.n_cand % 2 == 0 && aligned(t.cand_tok, 16) && aligned(t.cand_node, 16) &&
                 aligned(t.cand_logit, 8) && l0_ok)
                    ? 1
                    : 0;
  }
  p.wait_ns = g_wait_limit_ns.load(std::memory_order_relaxed);
  for (int n = g_stall_launches.load(); n > 0;)
    if (g_stall_launches.compare_exchange_weak(n, n - 1)) {
      p.stall = 1;
      break;
    }
  // Schedule.  Whole tiles round-robin over the pairs; when the last round
  // would leave pairs idle, the last two rounds' tiles are split into equal
  // k-block ranges instead (at least MIN_SEG k-blocks per pair).
  constexpr int64_t MIN_SEG = 4;
  const int64_t n_tiles = (t.rows + PAIR_M - 1) / PAIR_M;
  const int64_t kblocks = (t.H + BK - 1) / BK;
  const int64_t max_pairs = sm_count() / 2;
  int64_t pairs = n_tiles < max_pairs ? n_tiles : max_pairs;
  p.dp_tiles = n_tiles;
  p.sk_iters = 0;
  p.sk_pairs = 0;
  // Fewer 256-row tiles than pairs: the split-window variant (128-row tiles,
  // two CTAs per tile with half the window each) puts up to twice as many
  // SMs to work.  Measured on B200 it shortens sampling launches (cfg4
  // 0.19 -> 0.15 ms per search) and leaves top-n launches unchanged, whose
  // one-tile time is bound by operand delivery (~100 GB/s per SM) and the
  // cross-CTA hand-off; so by default it serves sampling only.
  // VTNK_SPLIT=1: top-n too; VTNK_SPLIT=0: never.
  static const int split_mode = [] {
    const char* e = getenv("VTNK_SPLIT");
    return (e && e[0] == '0') ? 0 : (e && e[0] == '1') ? 2 : 1;
  }();
  const bool split = n_tiles < max_pairs && (split_mode == 2 || (split_mode == 1 && t.sample));
  if (split) {
    const int64_t tiles128 = (t.rows + BM - 1) / BM;
    p.dp_tiles = tiles128;
    pairs = tiles128 < max_pairs ? tiles128 : max_pairs;
  } else if (t.sk_part && t.sk_count && n_tiles % max_pairs != 0) {
    const int64_t rounds = n_tiles / max_pairs;
    const int64_t dp = rounds > 0 ? (rounds - 1) * max_pairs : 0;
    const int64_t iters = (n_tiles - dp) * kblocks;
    int64_t skp = iters / MIN_SEG;
    if (skp > max_pairs) skp = max_pairs;
    if (skp > t.sk_cap_pairs) skp = t.sk_cap_pairs;
    if (skp >= 2 && 2 * (n_tiles - dp) <= t.sk_count_cap) {
      p.dp_tiles = dp;
      p.sk_iters = iters;
      p.sk_pairs = static_cast<int>(skp);
      p.sk_part = t.sk_part;
      p.sk_count = t.sk_count;
      p.sk_epoch = t.sk_epoch;
      pairs = dp > 0 ? max_pairs : skp;
    }
  }
  const int np = static_cast<int>(pairs);
  CUtensorMap ma, mw;
  if (!make_map(&ma, t.a, t.H, t.rows, t.a_stride * 2, BK, BM) ||
      !make_map(&mw, t.w, t.H, t.n_vocab, t.w_stride * 2, BK, BN / 2)) {
    set_error("cuTensorMapEncodeTiled failed");
    return VTNK_ERR_CUDA;
  }
  if (t.sample) return t.n_cand == 1 ? launch_nc<1, true>(ma, mw, p, np, split, t.pdl, s) : VTNK_ERR_UNSUPPORTED;
  switch (t.n_cand) {  // exact widths for the common beam sizes
    case 1: return launch_nc<1>(ma, mw, p, np, split, t.pdl, s);
    case 5: return launch_nc<5>(ma, mw, p, np, split, t.pdl, s);
    case 10: return launch_nc<10>(ma, mw, p, np, split, t.pdl, s);
    case 20: return launch_nc<20>(ma, mw, p, np, split, t.pdl, s);
    default: break;
  }
  if (t.n_cand <= 4) return launch_nc<4>(ma, mw, p, np, split, t.pdl, s);
  if (t.n_cand <= 8) return launch_nc<8>(ma, mw, p, np, split, t.pdl, s);
  if (t.n_cand <= 16) return launch_nc<16>(ma, mw, p, np, split, t.pdl, s);
  return launch_nc<32>(ma, mw, p, np, split, t.pdl, s);
}

int launch_build_child_index(const Csr& csr, uint32_t* masks, uint32_t* flags, int64_t node_lo,
                             int64_t node_hi, int64_t window_lo, int window_n, cudaStream_t s) {
  if (flags) {  // bit 0 set (bytes 0x01), cleared by the kernel on the first violation
    const cudaError_t e = cudaMemsetAsync(flags, 1, sizeof(uint32_t), s);
    if (e != cudaSuccess) return cuda_status(e, "child index flags");
  }
  if (node_hi <= node_lo) return VTNK_OK;
  const int64_t warps = node_hi - node_lo;
  int64_t blocks = (warps + 7) / 8;
  if (blocks > 148 * 32) blocks = 148 * 32;
  tc::build_index_kernel<<<static_cast<int>(blocks), 256, 0, s>>>(csr, masks, flags, node_lo,
                                                                  node_hi, window_lo, window_n);
  return cuda_status(cudaGetLastError(), "build_index_kernel launch");
}

int read_tc_status(int* out, bool reset) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_tc_status, sizeof(int));
  if (e != cudaSuccess) return cuda_status(e, "read device status");
  if (reset && v != 0) {
    const int z = 0;
    e = cudaMemcpyToSymbol(g_tc_status, &z, sizeof(int));
    if (e != cudaSuccess) return cuda_status(e, "reset device status");
  }
  *out = v;
  return VTNK_OK;
}

}  // namespace vtnk

extern "C" int vtnk_set_wait_limit_ns(uint64_t ns) {
  vtnk::g_wait_limit_ns.store(ns ? ns : vtnk::tc::WAIT_LIMIT_NS);
  return VTNK_OK;
}

extern "C" int vtnk_debug_stall_launches(int n) {
  if (n < 0) {
    vtnk::set_error("vtnk_debug_stall_launches: n < 0");
    return VTNK_ERR_ARG;
  }
  vtnk::g_stall_launches.store(n);
  return VTNK_OK;
}

#ifdef VTNK_TC_PROFILE
// Tuning builds only: copy (and optionally clear) the phase timers.
extern "C" int vtnk_tc_trace(unsigned long long* out) {
  cudaDeviceSynchronize();
  cudaMemcpyFromSymbol(out, vtnk::g_trace, sizeof(unsigned long long) * 512 * 32);
  return 0;
}

extern "C" int vtnk_tc_profile(unsigned long long* out, int reset) {
  cudaDeviceSynchronize();
  cudaMemcpyFromSymbol(out, vtnk::g_prof, sizeof(unsigned long long) * 8);
  if (reset) {
    unsigned long long z[8] = {};
    cudaMemcpyToSymbol(vtnk::g_prof, z, sizeof(z));
  }
  return 0;
}
#endif
