// Warp-per-row kernels of the constrained decoding step (CUDA cores).
//
// One warp owns one row (beam) end to end: it reads the row's CSR slice,
// computes the logit of every child (a[row] . W[col]) with 16-byte vector
// loads, and finishes the row in registers / shared memory -- dense masked
// logits, top-k, Gumbel-max or beam candidates -- so no cross-warp or
// cross-CTA reduction is needed (the reference's sampling kernel merges CTAs
// under a global spin lock, rectokens/kernels/constrained_node_transition.py:761-783).
//
// This path serves every shape: rows < 128, windows wider than one tensor-core
// tile, fp32 / fp16 operands and arbitrary b strides.  bf16 rows >= 128 with a
// <= 256-column window go to the tcgen05 tile kernel (vtnk_tc.cu).
#include <climits>

#include "vtnk_common.cuh"
#include "vtnk_internal.h"

namespace vtnk {

namespace {

constexpr int kWarps = 8;   // rows per CTA
constexpr int kGroup = 4;   // children whose dot products share one pass over a[row]

template <typename T, int MODE, bool VEC>
__global__ void __launch_bounds__(kWarps * 32)
rows_kernel(const RowsArgs p) {
  extern __shared__ float smem[];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  float* buf = smem + warp * p.buf_cap;
  const T* A = static_cast<const T*>(p.a);
  const T* Bm = static_cast<const T*>(p.b);
  const T* bias = static_cast<const T*>(p.bias);
  const int64_t* cols = p.csr.cols;
  const int64_t* vals = p.csr.vals;

  for (int64_t row = static_cast<int64_t>(blockIdx.x) * kWarps + warp; row < p.rows;
       row += static_cast<int64_t>(gridDim.x) * kWarps) {
    const int64_t cur = p.cur_node ? __ldg(p.cur_node + row) : 0;
    int64_t start;
    int count;
    node_children(p.csr, cur, p.mb, start, count);

    if (MODE != MODE_BEAM && p.next_node) {  // branch tables [rows, mb], -1 padded
      int64_t* vi = p.valid_idxs + row * p.mb;
      int64_t* nn = p.next_node + row * p.mb;
      for (int j = lane; j < p.mb; j += 32) {
        const bool ok = j < count;
        vi[j] = ok ? __ldg(cols + start + j) : -1;
        nn[j] = ok ? __ldg(vals + start + j) : -1;
      }
    }
    float* crow = nullptr;
    if (MODE == MODE_FUSED) {
      crow = p.corrected + row * p.N;
      if ((p.N & 3) == 0) {
        float4* c4 = reinterpret_cast<float4*>(crow);
        const float4 ninf = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
        for (int64_t n = lane; n < p.N / 4; n += 32) c4[n] = ninf;
      } else {
        for (int64_t n = lane; n < p.N; n += 32) crow[n] = -INFINITY;
      }
      __syncwarp();  // orders the fill before lane 0's child stores below
    }

    const T* arow = A + row * p.a_stride;
    for (int base = 0; base < count; base += kGroup) {
      int64_t col[kGroup];
#pragma unroll
      for (int g = 0; g < kGroup; ++g) {
        const int j = base + g;
        int64_t c = (j < count) ? __ldg(cols + start + j) : -1;
        col[g] = (c >= 0 && c < p.N) ? c : -1;
      }
      float acc[kGroup];
#pragma unroll
      for (int g = 0; g < kGroup; ++g) acc[g] = 0.f;
      if (VEC) {
        constexpr int V = Vec16<T>::N;
        for (int64_t h = static_cast<int64_t>(lane) * V; h < p.H; h += 32 * V) {
          Vec16<T> av;
          av.load(arow + h);
#pragma unroll
          for (int g = 0; g < kGroup; ++g) {
            if (col[g] < 0) continue;
            Vec16<T> bv;
            bv.load(Bm + col[g] * p.b_sn + h);
#pragma unroll
            for (int i = 0; i < V; ++i) acc[g] = fmaf(av.v[i], bv.v[i], acc[g]);
          }
        }
      } else {
        for (int64_t h = lane; h < p.H; h += 32) {
          const float av = to_f32<T>(arow[h]);
#pragma unroll
          for (int g = 0; g < kGroup; ++g) {
            if (col[g] < 0) continue;
            acc[g] = fmaf(av, to_f32<T>(Bm[h * p.b_sk + col[g] * p.b_sn]), acc[g]);
          }
        }
      }
#pragma unroll
      for (int g = 0; g < kGroup; ++g) {
        const int j = base + g;
        const float s = warp_sum(acc[g]);
        if (j >= count || lane != 0) continue;
        float v = -INFINITY;
        if (col[g] >= 0) {
          v = s;
          if (bias) v += to_f32<T>(bias[col[g]]);
        }
        if (MODE == MODE_FUSED) {
          if (col[g] >= 0) crow[col[g]] = v;
        } else {
          buf[j] = v;
        }
      }
    }
    __syncwarp();

    if (MODE == MODE_BEAM) {  // row log-sum-exp over every child
      float m = -INFINITY;
      for (int j = lane; j < count; j += 32) m = fmaxf(m, buf[j]);
      m = warp_max(m);
      float s = 0.f;
      if (m > -INFINITY)
        for (int j = lane; j < count; j += 32) s += expf(buf[j] - m);
      s = warp_sum(s);
      if (lane == 0) p.out_lse[row] = (m > -INFINITY) ? m + logf(s) : -INFINITY;
    }

    if (MODE == MODE_TOPK || MODE == MODE_BEAM) {
      for (int r = 0; r < p.k; ++r) {
        float bv = -INFINITY;
        int bj = INT_MAX;
        for (int j = lane; j < count; j += 32) {
          const float v = buf[j];
          if (v > bv || (v == bv && j < bj)) {
            bv = v;
            bj = j;
          }
        }
        warp_argmax(bv, bj);
        if (lane == 0) {
          const int64_t o = row * p.k + r;
          const bool ok = bj != INT_MAX && bv > -INFINITY;
          p.out_logit[o] = ok ? bv : -INFINITY;
          p.out_tok[o] = ok ? __ldg(cols + start + bj) : -1;
          if (MODE == MODE_BEAM) p.out_node[o] = ok ? __ldg(vals + start + bj) : -1;
          if (bj != INT_MAX) buf[bj] = __int_as_float(0x7fc00000);  // taken
        }
        __syncwarp();
      }
    }

    if (MODE == MODE_SAMPLE) {
      const float t = p.temperature ? __ldg(p.temperature) : 1.f;
      float bv = -INFINITY;
      int bj = INT_MAX;
      for (int j = lane; j < count; j += 32) {
        const float g = gumbel_at(p.seed, static_cast<uint32_t>(row * p.mb + j));
        const float s = buf[j] / t + g;
        if (s > bv) {  // slots visited in increasing order: first maximum kept
          bv = s;
          bj = j;
        }
      }
      warp_argmax(bv, bj);
      if (lane == 0) {
        const bool ok = bj != INT_MAX && bv > -INFINITY;
        p.sample[row] = ok ? static_cast<float>(__ldg(cols + start + bj)) : -1.f;
        if (p.out_node) p.out_node[row] = ok ? __ldg(vals + start + bj) : -1;
      }
    }
    __syncwarp();
  }
}

// Beam candidates from precomputed logits (a language model that returns the
// full vocabulary): per row, the children's logits are gathered from the
// logits row (the other columns are the -inf of the reference's mask), then
// the row's log-sum-exp over the children and its n_cand best children
// (ties to the lower slot) with their tokens and node ids -- the work of
// decode_one_step's mask op, log_softmax, topk(beam_size) and next-node
// lookup in one pass (rectokens/decoding/constrained_decoding.py:271-303,
// 372-383).  Warp per row.
template <typename T>
__global__ void __launch_bounds__(kWarps * 32)
logits_beam_kernel(const T* __restrict__ logits, int64_t B, int64_t N, int64_t ls,
                   const int64_t* __restrict__ cur_node, const Csr csr, int64_t mb, int k,
                   int buf_cap, int64_t* __restrict__ out_tok, float* __restrict__ out_logit,
                   int64_t* __restrict__ out_node, float* __restrict__ out_lse) {
  extern __shared__ float smem[];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  float* buf = smem + warp * buf_cap;
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * kWarps + warp; row < B;
       row += static_cast<int64_t>(gridDim.x) * kWarps) {
    int64_t start;
    int count;
    node_children(csr, cur_node ? cur_node[row] : 0, mb, start, count);
    for (int j = lane; j < count; j += 32) {
      const int64_t c = __ldg(csr.cols + start + j);
      buf[j] = (c >= 0 && c < N) ? to_f32<T>(logits[row * ls + c]) : -INFINITY;
    }
    __syncwarp();
    float m = -INFINITY;
    for (int j = lane; j < count; j += 32) m = fmaxf(m, buf[j]);
    m = warp_max(m);
    float sum = 0.f;
    if (m > -INFINITY)
      for (int j = lane; j < count; j += 32) sum += expf(buf[j] - m);
    sum = warp_sum(sum);
    if (lane == 0) out_lse[row] = (m > -INFINITY) ? m + logf(sum) : -INFINITY;
    for (int r = 0; r < k; ++r) {
      float bv = -INFINITY;
      int bj = INT_MAX;
      for (int j = lane; j < count; j += 32) {
        const float v = buf[j];
        if (v > bv || (v == bv && j < bj)) {
          bv = v;
          bj = j;
        }
      }
      warp_argmax(bv, bj);
      if (lane == 0) {
        const int64_t o = row * k + r;
        const bool ok = bj != INT_MAX && bv > -INFINITY;
        out_logit[o] = ok ? bv : -INFINITY;
        out_tok[o] = ok ? __ldg(csr.cols + start + bj) : -1;
        out_node[o] = ok ? __ldg(csr.vals + start + bj) : -1;
        if (bj != INT_MAX) buf[bj] = __int_as_float(0x7fc00000);  // taken
      }
      __syncwarp();
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kWarps * 32)
mask_kernel(const T* __restrict__ logits, int64_t B, int64_t N, int64_t ls,
            const int64_t* __restrict__ cur_node, const Csr csr, int64_t mb, T* __restrict__ out,
            int64_t* __restrict__ next_node, int64_t* __restrict__ valid_idxs) {
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const T ninf = from_f32<T>(-INFINITY);
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * kWarps + warp; row < B;
       row += static_cast<int64_t>(gridDim.x) * kWarps) {
    int64_t start;
    int count;
    node_children(csr, cur_node[row], mb, start, count);
    for (int j = lane; j < mb; j += 32) {
      const bool ok = j < count;
      valid_idxs[row * mb + j] = ok ? __ldg(csr.cols + start + j) : -1;
      next_node[row * mb + j] = ok ? __ldg(csr.vals + start + j) : -1;
    }
    T* orow = out + row * N;
    for (int64_t n = lane; n < N; n += 32) orow[n] = ninf;
    __syncwarp();
    for (int j = lane; j < count; j += 32) {
      const int64_t c = __ldg(csr.cols + start + j);
      if (c >= 0 && c < N) orow[c] = logits[row * ls + c];
    }
    __syncwarp();
  }
}

// Beam merge: one warp per query.  Candidate scores and tokens are staged in
// shared memory; the k selection rounds touch only shared memory and
// registers, then k lanes fetch the chosen candidates' nodes in parallel.
constexpr int kMergeWarps = 8;

__global__ void __launch_bounds__(kMergeWarps * 32)
merge_kernel(const MergeArgs p) {
  extern __shared__ float msm[];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t b = static_cast<int64_t>(blockIdx.x) * kMergeWarps + warp;
  if (b >= p.B) return;
  const int ncand = p.level == 0 ? p.n_cand : p.k * p.n_cand;
  // per warp: cap floats (scores) + cap ints (tokens) + k ints (choice) + k floats (score)
  float* tot = msm + static_cast<size_t>(warp) * (2 * p.cap + 2 * p.k);
  int* tok = reinterpret_cast<int*>(tot + p.cap);
  int* sel = tok + p.cap;
  float* selv = reinterpret_cast<float*>(sel + p.k);
  const int64_t base = p.level == 0 ? b * p.n_cand : b * p.k * p.n_cand;

  for (int c = lane; c < ncand; c += 32) {
    const int64_t row = p.level == 0 ? b : b * p.k + c / p.n_cand;
    const int64_t t = p.cand_tok[base + c];
    const float lv = p.cand_logit[base + c];  // -inf: a missing candidate
    const float lp = (lv > -INFINITY) ? lv - p.row_lse[row] : -INFINITY;
    const float v = p.level == 0 ? lp : p.prev_logp[row] + lp;
    tot[c] = (v == v) ? v : -INFINITY;  // a NaN score (never produced by the step kernels) ranks last
    tok[c] = static_cast<int>(t);
  }
  __syncwarp();
  for (int r = 0; r < p.k; ++r) {
    float bv = -INFINITY;
    int bc = INT_MAX;
    for (int c = lane; c < ncand; c += 32) {
      const float v = tot[c];
      if (v > bv || (v == bv && c < bc)) {
        bv = v;
        bc = c;
      }
    }
    warp_argmax(bv, bc);
    if (lane == 0) {
      sel[r] = bc;
      selv[r] = bv;
      tot[bc] = __int_as_float(0x7fc00000);  // taken
    }
    __syncwarp();
  }
  for (int r = lane; r < p.k; r += 32) {
    const int bc = sel[r];
    const int64_t o = b * p.k + r;
    const int64_t parent = p.level == 0 ? b : b * p.k + bc / p.n_cand;
    p.out_logp[o] = selv[r];
    p.out_node[o] = p.cand_node[base + bc];
    p.out_parent[o] = parent;
    p.out_ids[o * (p.level + 1) + p.level] = tok[bc];
  }
  if (p.level > 0) {  // copy each new beam's history from its parent
    const int w = static_cast<int>(p.level);
    for (int t = lane; t < p.k * w; t += 32) {
      const int r = t / w, i = t % w;
      const int64_t parent = b * p.k + sel[r] / p.n_cand;
      p.out_ids[(b * p.k + r) * (w + 1) + i] = p.prev_ids[parent * w + i];
    }
  }
}

// Beam merge, one thread per query (levels with at most 32 parent rows).
// Every parent's candidate list is sorted (the beam step emits them by
// descending logit, ties to the lower token) and a candidate's total
// prev_logp + (logit - lse) is monotone within its list, so a query's k best
// come from a k-way merge of its lists: each round takes the best list head
// (ties to the lower flat candidate index) and advances that list.
//   * A warp first stages its 32 queries' candidate logits (-inf where padded)
//     in shared memory with coalesced loads, stride k*n+1 per query
//     (conflict-free per-thread reads).
//   * The selection rounds touch only shared memory and registers; every
//     global read / write of the outputs is issued after them, together.
//   * A query whose lists are not sorted (possible only for an arbitrary
//     caller of vtnk_beam_merge) is merged by an exact successor scan instead.
template <int KM>
__global__ void __launch_bounds__(128)
merge_sorted_kernel(const MergeArgs p) {
  extern __shared__ float ssm[];
  const int lane = threadIdx.x & 31;
  const int n = p.n_cand;
  const int L = p.level == 0 ? 1 : p.k;
  const int per_q = L * n;
  const int stride = per_q + 1;
  float* st = ssm + static_cast<size_t>(threadIdx.x >> 5) * 32 * stride;
  const int64_t qbase = static_cast<int64_t>(blockIdx.x) * blockDim.x + (threadIdx.x & ~31);
  if (qbase >= p.B) return;  // warp-uniform
  {
    const int nq = static_cast<int>((p.B - qbase) < 32 ? (p.B - qbase) : 32);
    const int total = nq * per_q;
    const int64_t e0 = qbase * per_q;  // consecutive queries' candidates are contiguous
    // flat index t -> (query, candidate) without division: walk t in steps
    // of 32 and carry (q, c); 8 loads in flight per lane
    int q = lane / per_q, c = lane - (lane / per_q) * per_q;
    const int dq = 32 / per_q, dc = 32 - dq * per_q;
#pragma unroll 8
    for (int t = lane; t < total; t += 32) {
      st[q * stride + c] = p.cand_logit[e0 + t];  // -inf: a missing candidate
      q += dq;
      c += dc;
      if (c >= per_q) {
        c -= per_q;
        ++q;
      }
    }
  }
  __syncwarp();
  const int64_t b = qbase + lane;
  if (b >= p.B) return;
  const float* my = st + lane * stride;
  const int64_t row0 = p.level == 0 ? b : b * p.k;
  bool sorted = true;
  for (int i = 0; i < L; ++i)
    for (int j = 1; j < n; ++j) sorted = sorted && !(my[i * n + j] > my[i * n + j - 1]);
  float pv[KM], ls[KM], head[KM];
  int pos[KM];
#pragma unroll
  for (int i = 0; i < KM; ++i) {
    const bool in = i < L;
    pv[i] = (in && p.level > 0) ? p.prev_logp[row0 + i] : 0.f;
    ls[i] = in ? p.row_lse[row0 + i] : 0.f;
    head[i] = in ? my[i * n] : -INFINITY;
    pos[i] = 0;
  }
  // Chosen flat candidate and score per round (small per-thread arrays; the
  // rounds are not unrolled, so these live in L1-cached local memory).
  int sel_c[KM];
  float sel_v[KM];
  if (sorted) {
#pragma unroll 1
    for (int r = 0; r < p.k; ++r) {
      float bv = -INFINITY;
      int bc = INT_MAX, bi = 0;
#pragma unroll
      for (int i = 0; i < KM; ++i) {
        if (i >= L || pos[i] >= n) continue;
        const float lp = head[i] > -INFINITY ? head[i] - ls[i] : -INFINITY;
        float v = p.level == 0 ? lp : pv[i] + lp;
        if (!(v == v)) v = -INFINITY;
        const int c = i * n + pos[i];
        if (v > bv || (v == bv && c < bc)) {
          bv = v;
          bc = c;
          bi = i;
        }
      }
#pragma unroll
      for (int i = 0; i < KM; ++i)
        if (i == bi) {
          ++pos[i];
          if (pos[i] < n) head[i] = my[i * n + pos[i]];
        }
      sel_c[r] = bc;
      sel_v[r] = bv;
    }
  } else {
    // successor scan: each round, the best candidate ordered after the previous pick
    float prev_v = INFINITY;
    int prev_c = -1;
#pragma unroll 1
    for (int r = 0; r < p.k; ++r) {
      float bv = -INFINITY;
      int bc = INT_MAX;
#pragma unroll 1
      for (int c = 0; c < per_q; ++c) {
        const int i = c / n;
        const float lv = my[c];
        const float lp = lv > -INFINITY ? lv - p.row_lse[row0 + i] : -INFINITY;
        float v = p.level == 0 ? lp : p.prev_logp[row0 + i] + lp;
        if (!(v == v)) v = -INFINITY;  // NaN ranks last: every round finds a candidate
        const bool after = v < prev_v || (v == prev_v && c > prev_c);
        if (after && (v > bv || (v == bv && c < bc) || bc == INT_MAX)) {
          bv = v;
          bc = c;
        }
      }
      prev_v = bv;
      prev_c = bc;
      sel_c[r] = bc;
      sel_v[r] = bv;
    }
  }
#pragma unroll
  for (int r = 0; r < KM; ++r) {  // unrolled: the output loads of all rounds overlap
    if (r >= p.k) break;
    const int bi = sel_c[r] / n;
    const int64_t parent = row0 + bi;
    const int64_t e = parent * n + (sel_c[r] - bi * n);
    const int64_t o = b * p.k + r;
    p.out_logp[o] = sel_v[r];
    p.out_node[o] = p.cand_node[e];
    p.out_parent[o] = parent;
    p.out_ids[o * (p.level + 1) + p.level] = p.cand_tok[e];
    for (int t = 0; t < p.level; ++t)
      p.out_ids[o * (p.level + 1) + t] = p.prev_ids[parent * p.level + t];
  }
}

// Beam merge, one group of G lanes per query (G = 16 or 32, k <= G lists):
// lane i owns parent list i.  Lists are sorted (descending logit), so each
// round is a G-lane argmax over the list heads (ties to the lower flat
// candidate index) and the winning lane advances its head; lane r keeps
// round r's choice and writes output beam r.  Candidates are staged in shared
// memory by coalesced loads of the block's queries.  A query with an
// unsorted list is merged by its lane 0 with the exact successor scan.
template <int G>
__device__ __forceinline__ void merge_group_block(const MergeArgs& p, float* gsm, int64_t q0,
                                                  int n, int L, int per_q) {
  constexpr int QPB = 128 / G;
  const int g = threadIdx.x / G;        // query slot in the block
  const int li = threadIdx.x % G;       // list (parent) index
  const int64_t b = q0 + g;
  const int64_t row0 = p.level == 0 ? b : b * p.k;
  const bool has = li < L && b < p.B;
  // the list's previous log-prob and log-sum-exp, loaded before (and in
  // flight with) the staging loads
  const float pv = (has && p.level > 0) ? p.prev_logp[row0 + li] : 0.f;
  const float ls = has ? p.row_lse[row0 + li] : 0.f;
  __syncthreads();  // the previous block's readers are done with gsm
  {
    const int64_t nq64 = p.B - q0 < QPB ? p.B - q0 : QPB;
    const int total = static_cast<int>(nq64) * per_q;
    const int64_t e0 = q0 * per_q;
    // all of a thread's loads issued before its stores: one memory latency
    constexpr int U = 8;
    for (int t0 = threadIdx.x; t0 < total; t0 += 128 * U) {
      float v[U];
#pragma unroll
      for (int j = 0; j < U; ++j) {
        const int t = t0 + j * 128;
        v[j] = t < total ? p.cand_logit[e0 + t] : 0.f;  // -inf: a missing candidate
      }
#pragma unroll
      for (int j = 0; j < U; ++j)
        if (t0 + j * 128 < total) gsm[t0 + j * 128] = v[j];
    }
  }
  __syncthreads();
  if (b >= p.B) return;                 // whole groups retire together (the last block)
  const unsigned gmask = (G == 32) ? 0xffffffffu : (0xffffu << ((threadIdx.x & 31) & 16));
  const float* my = gsm + g * per_q;
  bool ok = true;
  if (has)
    for (int j = 1; j < n; ++j) ok = ok && !(my[li * n + j] > my[li * n + j - 1]);
  const bool sorted = __all_sync(gmask, ok);
  int pos = 0;
  int my_c = 0;
  float my_v = -INFINITY;
  if (sorted) {
    for (int r = 0; r < p.k; ++r) {
      float v = -INFINITY;
      int c = INT_MAX;
      if (has && pos < n) {
        const float lv = my[li * n + pos];
        const float lp = lv > -INFINITY ? lv - ls : -INFINITY;
        v = p.level == 0 ? lp : pv + lp;
        c = li * n + pos;
      }
      // best value over the group: one max-reduction of an order-preserving
      // key, then the lowest lane holding it (lower parent, and within a
      // list the head is its lowest remaining slot: the reference's tie order)
      const unsigned key = order_key(v);
      const unsigned best = __reduce_max_sync(gmask, key);
      const unsigned holders = __ballot_sync(gmask, key == best && c != INT_MAX) & gmask;
      const int wl = __ffs(holders) - 1;
      const bool mine = (threadIdx.x & 31) == wl;
      v = __shfl_sync(gmask, v, wl);
      c = __shfl_sync(gmask, c, wl);
      if (mine) ++pos;  // the winning list advances
      if (li == r) {
        my_c = c;
        my_v = v;
      }
    }
  } else if (li == 0) {
    // exact successor scan for this query; lane 0 writes all k outputs below
    float prev_v = INFINITY;
    int prev_c = -1;
    for (int r = 0; r < p.k; ++r) {
      float bv = -INFINITY;
      int bc = INT_MAX;
      for (int c = 0; c < per_q; ++c) {
        const int i = c / n;
        const float lv = my[c];
        const float lp = lv > -INFINITY ? lv - p.row_lse[row0 + i] : -INFINITY;
        float v = p.level == 0 ? lp : p.prev_logp[row0 + i] + lp;
        if (!(v == v)) v = -INFINITY;  // NaN ranks last: every round finds a candidate
        const bool after = v < prev_v || (v == prev_v && c > prev_c);
        if (after && (v > bv || (v == bv && c < bc) || bc == INT_MAX)) {
          bv = v;
          bc = c;
        }
      }
      prev_v = bv;
      prev_c = bc;
      const int bi = bc / n;
      const int64_t parent = row0 + bi;
      const int64_t e = parent * n + (bc - bi * n);
      const int64_t o = b * p.k + r;
      p.out_logp[o] = bv;
      p.out_node[o] = p.cand_node[e];
      p.out_parent[o] = parent;
      p.out_ids[o * (p.level + 1) + p.level] = p.cand_tok[e];
      for (int t = 0; t < p.level; ++t)
        p.out_ids[o * (p.level + 1) + t] = p.prev_ids[parent * p.level + t];
    }
    return;
  }
  if (!sorted || li >= p.k) return;
  const int r = li;
  const int bi = my_c / n;
  const int64_t parent = row0 + bi;
  const int64_t e = parent * n + (my_c - bi * n);
  const int64_t o = b * p.k + r;
  // every load of the outputs issued before the first store
  const int64_t node = p.cand_node[e];
  const int64_t tok = p.cand_tok[e];
  constexpr int HB = 8;
  int64_t hist[HB];
#pragma unroll
  for (int t = 0; t < HB; ++t) hist[t] = t < p.level ? p.prev_ids[parent * p.level + t] : 0;
  p.out_logp[o] = my_v;
  p.out_node[o] = node;
  p.out_parent[o] = parent;
  p.out_ids[o * (p.level + 1) + p.level] = tok;
#pragma unroll
  for (int t = 0; t < HB; ++t)
    if (t < p.level) p.out_ids[o * (p.level + 1) + t] = hist[t];
  for (int t = HB; t < p.level; ++t)
    p.out_ids[o * (p.level + 1) + t] = p.prev_ids[parent * p.level + t];
}

template <int G>
__global__ void __launch_bounds__(128)
merge_group_kernel(const MergeArgs p) {
  extern __shared__ float gsm[];
  // Launched as a programmatic dependent of the step kernel (inside a
  // search).  The next level's step kernel may be scheduled at once: its
  // CTAs take the SMs the step kernel's last tile round leaves idle and start
  // streaming their operands (their epilogues wait for this merge).  Then
  // wait for the step kernel's results.  Both are no-ops in a plain launch.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  constexpr int QPB = 128 / G;  // queries per block
  const int n = p.n_cand;
  const int L = p.level == 0 ? 1 : p.k;
  const int per_q = L * n;
  // grid-stride over blocks of QPB queries
  for (int64_t q0 = static_cast<int64_t>(blockIdx.x) * QPB; q0 < p.B;
       q0 += static_cast<int64_t>(gridDim.x) * QPB) {
    merge_group_block<G>(p, gsm, q0, n, L, per_q);
  }
}

template <typename T>
__global__ void synth_kernel(uint64_t key, int64_t e0, int64_t count, const T* __restrict__ table,
                             T* __restrict__ out) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint64_t z = mix64(static_cast<uint64_t>(e0 + i) ^ key);
    out[i] = table[z >> 48];
  }
}

// Branch tables alone: valid_idxs / next_node [rows, mb], -1 padded (warp per row).
__global__ void __launch_bounds__(kWarps * 32)
tables_kernel(int64_t rows, const int64_t* __restrict__ cur_node, const Csr csr, int64_t mb,
              int64_t* __restrict__ next_node, int64_t* __restrict__ valid_idxs) {
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * kWarps + warp; row < rows;
       row += static_cast<int64_t>(gridDim.x) * kWarps) {
    int64_t start;
    int count;
    node_children(csr, cur_node ? __ldg(cur_node + row) : 0, mb, start, count);
    for (int j = lane; j < mb; j += 32) {
      const bool ok = j < count;
      valid_idxs[row * mb + j] = ok ? __ldg(csr.cols + start + j) : -1;
      next_node[row * mb + j] = ok ? __ldg(csr.vals + start + j) : -1;
    }
  }
}

__global__ void gumbel_kernel(uint64_t seed, int64_t rows, int64_t mb, float* out) {
  const int64_t n = rows * mb;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    out[i] = gumbel_at(seed, static_cast<uint32_t>(i));
}

int grid_for(int64_t items, int per_block) {
  int64_t g = (items + per_block - 1) / per_block;
  const int64_t cap = 148LL * 64;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return static_cast<int>(g);
}

template <typename T, int MODE>
int launch_rows_t(const RowsArgs& p, cudaStream_t s) {
  const size_t sm = static_cast<size_t>(kWarps) * p.buf_cap * sizeof(float);
  const int grid = grid_for(p.rows, kWarps);
  if (p.vec) {
    auto k = rows_kernel<T, MODE, true>;
    if (sm > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    k<<<grid, kWarps * 32, sm, s>>>(p);
  } else {
    auto k = rows_kernel<T, MODE, false>;
    if (sm > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    k<<<grid, kWarps * 32, sm, s>>>(p);
  }
  return cuda_status(cudaGetLastError(), "rows_kernel launch");
}

template <int MODE>
int launch_rows_mode(const RowsArgs& p, int dtype, cudaStream_t s) {
  switch (dtype) {
    case VTNK_F32: return launch_rows_t<float, MODE>(p, s);
    case VTNK_BF16: return launch_rows_t<__nv_bfloat16, MODE>(p, s);
    case VTNK_F16: return launch_rows_t<__half, MODE>(p, s);
  }
  set_error("unsupported dtype %d", dtype);
  return VTNK_ERR_ARG;
}

}  // namespace

int launch_rows(const RowsArgs& p, int mode, int dtype, cudaStream_t s) {
  if (p.rows == 0) return VTNK_OK;
  const size_t sm = static_cast<size_t>(kWarps) * p.buf_cap * sizeof(float);
  if (sm > 200 * 1024) {
    set_error("max_branches %lld too large for the row kernel", (long long)p.mb);
    return VTNK_ERR_UNSUPPORTED;
  }
  switch (mode) {
    case MODE_FUSED: return launch_rows_mode<MODE_FUSED>(p, dtype, s);
    case MODE_TOPK: return launch_rows_mode<MODE_TOPK>(p, dtype, s);
    case MODE_SAMPLE: return launch_rows_mode<MODE_SAMPLE>(p, dtype, s);
    case MODE_BEAM: return launch_rows_mode<MODE_BEAM>(p, dtype, s);
  }
  set_error("bad mode");
  return VTNK_ERR_ARG;
}

int launch_mask(const void* logits, int dtype, int64_t B, int64_t N, int64_t ls,
                const int64_t* cur_node, const Csr& csr, int64_t mb, void* out, int64_t* nn,
                int64_t* vi, cudaStream_t s) {
  if (B == 0) return VTNK_OK;
  const int grid = grid_for(B, kWarps);
  switch (dtype) {
    case VTNK_F32:
      mask_kernel<float><<<grid, kWarps * 32, 0, s>>>(static_cast<const float*>(logits), B, N, ls,
                                                      cur_node, csr, mb, static_cast<float*>(out), nn, vi);
      break;
    case VTNK_BF16:
      mask_kernel<__nv_bfloat16><<<grid, kWarps * 32, 0, s>>>(
          static_cast<const __nv_bfloat16*>(logits), B, N, ls, cur_node, csr, mb,
          static_cast<__nv_bfloat16*>(out), nn, vi);
      break;
    case VTNK_F16:
      mask_kernel<__half><<<grid, kWarps * 32, 0, s>>>(static_cast<const __half*>(logits), B, N, ls,
                                                       cur_node, csr, mb, static_cast<__half*>(out), nn, vi);
      break;
    default:
      set_error("unsupported dtype %d", dtype);
      return VTNK_ERR_ARG;
  }
  return cuda_status(cudaGetLastError(), "mask_kernel launch");
}

int launch_logits_beam(const void* logits, int dtype, int64_t B, int64_t N, int64_t ls,
                       const int64_t* cur_node, const Csr& csr, int64_t mb, int k,
                       int64_t* tok, float* logit, int64_t* node, float* lse, cudaStream_t s) {
  if (B == 0) return VTNK_OK;
  const int cap = static_cast<int>(mb > 0 ? mb : 1);
  const size_t sm = static_cast<size_t>(kWarps) * cap * sizeof(float);
  if (sm > 200 * 1024) {
    set_error("max_branches too large for the candidates kernel");
    return VTNK_ERR_UNSUPPORTED;
  }
  const int grid = grid_for(B, kWarps);
#define VTNK_LB_LAUNCH(T)                                                                       \
  do {                                                                                          \
    if (sm > 48 * 1024)                                                                         \
      cudaFuncSetAttribute(logits_beam_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,  \
                           static_cast<int>(sm));                                               \
    logits_beam_kernel<T><<<grid, kWarps * 32, sm, s>>>(static_cast<const T*>(logits), B, N,   \
                                                        ls, cur_node, csr, mb, k, cap, tok,     \
                                                        logit, node, lse);                      \
  } while (0)
  switch (dtype) {
    case VTNK_F32: VTNK_LB_LAUNCH(float); break;
    case VTNK_BF16: VTNK_LB_LAUNCH(__nv_bfloat16); break;
    case VTNK_F16: VTNK_LB_LAUNCH(__half); break;
    default:
      set_error("unsupported dtype %d", dtype);
      return VTNK_ERR_ARG;
  }
#undef VTNK_LB_LAUNCH
  return cuda_status(cudaGetLastError(), "logits_beam_kernel launch");
}

int launch_merge(const MergeArgs& p, cudaStream_t s) {
  if (p.B == 0) return VTNK_OK;
  const int lists = p.level == 0 ? 1 : p.k;
  if (p.k <= 32 && p.level > 0) {  // one list per query at level 0: thread-per-query below
    const int G = p.k <= 16 ? 16 : 32;
    const size_t sm = static_cast<size_t>(128 / G) * lists * p.n_cand * sizeof(float);
    if (sm <= 96 * 1024) {
      const int64_t grid = (p.B + 128 / G - 1) / (128 / G);
      auto k = G == 16 ? merge_group_kernel<16> : merge_group_kernel<32>;
      if (sm > 48 * 1024)
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(sm));
      cudaLaunchConfig_t cfg{};
      cfg.gridDim = dim3(static_cast<unsigned>(grid));
      cfg.blockDim = dim3(128);
      cfg.dynamicSmemBytes = sm;
      cfg.stream = s;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[0].val.programmaticStreamSerializationAllowed = 1;
      cfg.attrs = attr;
      cfg.numAttrs = p.pdl ? 1 : 0;
      return cuda_status(cudaLaunchKernelEx(&cfg, k, p), "merge_group_kernel launch");
    }
  }
  const size_t per_warp = 32 * static_cast<size_t>(lists * p.n_cand + 1) * sizeof(float);
  if (lists <= 32 && p.k <= 32 && 4 * per_warp <= 96 * 1024) {
    const int grid = static_cast<int>((p.B + 127) / 128);
    const size_t sm = 4 * per_warp;
#define VTNK_MERGE_LAUNCH(KM)                                                                   \
  do {                                                                                          \
    if (sm > 48 * 1024)                                                                         \
      cudaFuncSetAttribute(merge_sorted_kernel<KM>,                                             \
                           cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(sm));  \
    merge_sorted_kernel<KM><<<grid, 128, sm, s>>>(p);                                           \
  } while (0)
    const int km = lists > p.k ? lists : p.k;
    if (km <= 1) VTNK_MERGE_LAUNCH(1);
    else if (km <= 4) VTNK_MERGE_LAUNCH(4);
    else if (km <= 10) VTNK_MERGE_LAUNCH(10);
    else if (km <= 16) VTNK_MERGE_LAUNCH(16);
    else VTNK_MERGE_LAUNCH(32);
#undef VTNK_MERGE_LAUNCH
    return cuda_status(cudaGetLastError(), "merge_sorted_kernel launch");
  }
  const size_t sm = static_cast<size_t>(kMergeWarps) * (2 * p.cap + 2 * p.k) * sizeof(float);
  if (sm > 200 * 1024) {
    set_error("beams * candidates too large for the merge kernel");
    return VTNK_ERR_UNSUPPORTED;
  }
  if (sm > 48 * 1024)
    cudaFuncSetAttribute(merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
  const int grid = static_cast<int>((p.B + kMergeWarps - 1) / kMergeWarps);
  merge_kernel<<<grid, kMergeWarps * 32, sm, s>>>(p);
  return cuda_status(cudaGetLastError(), "merge_kernel launch");
}

int launch_synth(uint64_t key, int64_t e0, int64_t count, const void* table, int dtype, void* out,
                 cudaStream_t s) {
  if (count == 0) return VTNK_OK;
  const int grid = grid_for(count, 256 * 8);
  if (dtype == VTNK_BF16 || dtype == VTNK_F16)
    synth_kernel<uint16_t><<<grid, 256, 0, s>>>(key, e0, count, static_cast<const uint16_t*>(table),
                                                static_cast<uint16_t*>(out));
  else
    synth_kernel<float><<<grid, 256, 0, s>>>(key, e0, count, static_cast<const float*>(table),
                                             static_cast<float*>(out));
  return cuda_status(cudaGetLastError(), "synth_kernel launch");
}

int launch_tables(int64_t rows, const int64_t* cur_node, const Csr& csr, int64_t mb,
                  int64_t* next_node, int64_t* valid_idxs, cudaStream_t s) {
  if (rows == 0 || mb == 0) return VTNK_OK;
  tables_kernel<<<grid_for(rows, kWarps), kWarps * 32, 0, s>>>(rows, cur_node, csr, mb, next_node,
                                                               valid_idxs);
  return cuda_status(cudaGetLastError(), "tables_kernel launch");
}

int launch_gumbel(uint64_t seed, int64_t rows, int64_t mb, float* out, cudaStream_t s) {
  if (rows * mb == 0) return VTNK_OK;
  gumbel_kernel<<<grid_for(rows * mb, 256 * 4), 256, 0, s>>>(seed, rows, mb, out);
  return cuda_status(cudaGetLastError(), "gumbel_kernel launch");
}

}  // namespace vtnk
