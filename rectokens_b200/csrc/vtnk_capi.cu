// extern "C" entry points of libvtnk_b200: argument checks, dispatch, and the
// device-resident beam-search driver.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <cstdlib>
#include <mutex>

#include "vtnk_common.cuh"
#include "vtnk_internal.h"

namespace vtnk {

namespace {
thread_local char g_err[512] = "";
}

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return VTNK_OK;
  set_error("%s: %s", what, cudaGetErrorString(e));
  return VTNK_ERR_CUDA;
}

SkWorkspace sk_workspace(cudaStream_t s) {
  struct Entry {
    int dev;
    cudaStream_t stream;
    SkWorkspace w;
  };
  constexpr int kMaxEntries = 16;  // streams with a workspace; others run whole tiles only
  static std::mutex mu;
  static Entry entries[kMaxEntries];
  static int n_entries = 0;
  // Opt-in (VTNK_STREAMK=1): on B200 the split-tile hand-over measured
  // slower than whole-tile rounds for every configuration tried.
  static const bool enabled = [] {
    const char* e = getenv("VTNK_STREAMK");
    return e && e[0] == '1';
  }();
  SkWorkspace none{};
  int dev = 0;
  if (!enabled || cudaGetDevice(&dev) != cudaSuccess) return none;
  std::lock_guard<std::mutex> lock(mu);
  Entry* e = nullptr;
  for (int i = 0; i < n_entries; ++i)
    if (entries[i].dev == dev && entries[i].stream == s) e = &entries[i];
  if (!e) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (n_entries == kMaxEntries || cudaStreamIsCapturing(s, &cs) != cudaSuccess ||
        cs != cudaStreamCaptureStatusNone)
      return none;  // no allocation inside a graph capture
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    SkWorkspace w{};
    w.cap_pairs = sms / 2;
    w.count_cap = 4 * w.cap_pairs;  // fewer than 2 * pairs split tiles, 2 ranks each
    const size_t part_bytes = static_cast<size_t>(w.cap_pairs) * 2 * 2 * 128 * 256 * 4;
    if (cudaMalloc(&w.part, part_bytes) != cudaSuccess) {
      cudaGetLastError();
      return none;
    }
    if (cudaMalloc(&w.count, w.count_cap * sizeof(unsigned long long)) != cudaSuccess ||
        cudaMemset(w.count, 0, w.count_cap * sizeof(unsigned long long)) != cudaSuccess) {
      cudaGetLastError();
      cudaFree(w.part);
      return none;
    }
    entries[n_entries] = Entry{dev, s, w};
    e = &entries[n_entries++];
  }
  if (++e->w.epoch == 0) e->w.epoch = 1;
  return e->w;
}

namespace {

int elem_size(int dtype) { return dtype == VTNK_F32 ? 4 : 2; }

int check_csr(const vtnk_csr_t* c) {
  VTNK_REQUIRE(c != nullptr, "csr is NULL");
  VTNK_REQUIRE(c->n_nodes >= 1 && c->nnz >= 0, "csr sizes invalid");
  VTNK_REQUIRE(c->row_ptrs && c->cols && c->vals, "csr pointer is NULL");
  return VTNK_OK;
}

int check_linear(const vtnk_linear_t* l) {
  VTNK_REQUIRE(l != nullptr, "linear operand is NULL");
  VTNK_REQUIRE(l->dtype == VTNK_F32 || l->dtype == VTNK_BF16 || l->dtype == VTNK_F16,
               "unsupported dtype %d", l->dtype);
  VTNK_REQUIRE(l->rows >= 0 && l->hidden >= 1 && l->n_vocab >= 1, "bad linear shape");
  VTNK_REQUIRE(l->rows == 0 || (l->a && l->b), "linear pointer is NULL");
  VTNK_REQUIRE(l->a_stride >= l->hidden, "a row stride < hidden");
  return VTNK_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

RowsArgs rows_from(const vtnk_linear_t* l, const int64_t* cur_node, const vtnk_csr_t* c,
                   int64_t mb) {
  RowsArgs p{};
  p.a = l->a;
  p.rows = l->rows;
  p.H = l->hidden;
  p.a_stride = l->a_stride;
  p.b = l->b;
  p.N = l->n_vocab;
  p.b_sk = l->b_stride_k;
  p.b_sn = l->b_stride_n;
  p.bias = l->bias;
  p.cur_node = cur_node;
  p.csr = make_csr(*c);
  p.mb = mb;
  const int v = 16 / elem_size(l->dtype);
  p.vec = l->b_stride_k == 1 && (l->hidden % v) == 0 && (l->a_stride % v) == 0 &&
          (l->b_stride_n % v) == 0 && aligned16(l->a) && aligned16(l->b);
  return p;
}

int check_step(const vtnk_linear_t* l, const vtnk_csr_t* c, int64_t mb) {
  int rc = check_linear(l);
  if (rc) return rc;
  rc = check_csr(c);
  if (rc) return rc;
  VTNK_REQUIRE(mb >= 0 && mb <= (1 << 20), "max_branches out of range");
  return VTNK_OK;
}

size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

struct SearchLayout {
  size_t cand_tok, cand_node, cand_logit, lse, ids[2], logp[2], node[2], parent, total;
};

SearchLayout search_layout(const vtnk_search_t* s) {
  const size_t bk = static_cast<size_t>(s->batch) * s->beams;
  const size_t rmax = bk > static_cast<size_t>(s->batch) ? bk : s->batch;
  const size_t nc = rmax * s->n_cand;
  SearchLayout L{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off += align256(bytes);
    return o;
  };
  L.cand_tok = take(nc * 8);
  L.cand_node = take(nc * 8);
  L.cand_logit = take(nc * 4);
  L.lse = take(rmax * 4);
  for (int i = 0; i < 2; ++i) {
    L.ids[i] = take(bk * s->levels * 8);
    L.logp[i] = take(bk * 4);
    L.node[i] = take(bk * 8);
  }
  L.parent = take(bk * 8);
  L.total = off;
  return L;
}

// The tcgen05 tile kernel for one level when the shape allows it;
// VTNK_ERR_UNSUPPORTED (nothing launched) otherwise.  `sample` selects
// Gumbel-max sampling (n_cand 1) instead of top-n + log-sum-exp.
int tc_step(const vtnk_linear_t* lin, const int64_t* cur_node, const vtnk_csr_t* csr, int64_t mb,
            int64_t n_cand, const vtnk_child_index_t* index, int64_t* cand_tok,
            float* cand_logit, int64_t* cand_node, float* row_lse, int sample, uint64_t seed,
            const float* temperature, float* sample_f, bool stream_k, cudaStream_t s,
            const TcArgs* l0 = nullptr, bool pdl = false) {
  if (tc_enabled() && index && index->masks && lin->dtype == VTNK_BF16 && lin->b_stride_k == 1 &&
      lin->rows >= 128) {
    TcArgs t{};
    t.a = lin->a;
    t.rows = lin->rows;
    t.H = lin->hidden;
    t.a_stride = lin->a_stride;
    t.w = lin->b;
    t.w_stride = lin->b_stride_n;
    t.n_vocab = lin->n_vocab;
    t.window_lo = index->window_lo;
    t.window_n = static_cast<int>(index->window_n);
    t.masks = index->masks;
    t.flags = index->flags;
    t.idx_lo = index->node_lo;
    t.idx_hi = index->node_hi;
    t.bias = lin->bias;
    t.cur_node = cur_node;
    t.csr = make_csr(*csr);
    t.mb = mb;
    t.n_cand = static_cast<int>(n_cand);
    t.cand_tok = cand_tok;
    t.cand_logit = cand_logit;
    t.cand_node = cand_node;
    t.row_lse = row_lse;
    t.sample = sample;
    t.seed = seed;
    t.temperature = temperature;
    t.sample_f = sample_f;
    t.pdl = pdl;
    if (l0) {
      t.l0_ids = l0->l0_ids;
      t.l0_logp = l0->l0_logp;
      t.l0_node = l0->l0_node;
      t.l0_k = l0->l0_k;
    }
    if (stream_k) {
      const SkWorkspace w = sk_workspace(s);
      t.sk_part = w.part;
      t.sk_count = w.count;
      t.sk_cap_pairs = w.cap_pairs;
      t.sk_count_cap = w.count_cap;
      t.sk_epoch = w.epoch;
    }
    return launch_beam_step_tc(t, s);
  }
  return VTNK_ERR_UNSUPPORTED;
}

// One fused level: tcgen05 tile kernel when the shape allows, else rows kernel.
int beam_step_impl(const vtnk_linear_t* lin, const int64_t* cur_node, const vtnk_csr_t* csr,
                   int64_t mb, int64_t n_cand, const vtnk_child_index_t* index,
                   int64_t* cand_tok, float* cand_logit, int64_t* cand_node, float* row_lse,
                   bool stream_k, cudaStream_t s, bool pdl = false) {
  if (lin->rows == 0) return VTNK_OK;
  const int rc = tc_step(lin, cur_node, csr, mb, n_cand, index, cand_tok, cand_logit, cand_node,
                         row_lse, 0, 0, nullptr, nullptr, stream_k, s, nullptr, pdl);
  if (rc != VTNK_ERR_UNSUPPORTED) return rc;
  RowsArgs p = rows_from(lin, cur_node, csr, mb);
  p.k = static_cast<int>(n_cand);
  p.buf_cap = static_cast<int>(mb > 0 ? mb : 1);
  p.out_logit = cand_logit;
  p.out_tok = cand_tok;
  p.out_node = cand_node;
  p.out_lse = row_lse;
  return launch_rows(p, MODE_BEAM, lin->dtype, s);
}

}  // namespace

int merge_impl(int64_t level, int64_t B, int64_t k, int64_t n_cand, const int64_t* cand_tok,
               const float* cand_logit, const int64_t* cand_node, const float* row_lse,
               const float* prev_logp, const int64_t* prev_ids, int64_t* out_ids, float* out_logp,
               int64_t* out_node, int64_t* out_parent, bool pdl, cudaStream_t stream) {
  VTNK_REQUIRE(level >= 0 && B >= 0 && k >= 1 && n_cand >= 1, "bad merge sizes");
  VTNK_REQUIRE(level > 0 || k <= n_cand, "first level needs k <= n_cand");
  VTNK_REQUIRE(B == 0 || (cand_tok && cand_logit && cand_node && row_lse && out_ids && out_logp &&
                          out_node && out_parent),
               "NULL pointer");
  VTNK_REQUIRE(level == 0 || B == 0 || (prev_logp && prev_ids), "NULL previous beams");
  MergeArgs p{};
  p.level = level;
  p.B = B;
  p.k = static_cast<int>(k);
  p.n_cand = static_cast<int>(n_cand);
  p.cap = static_cast<int>(level == 0 ? n_cand : k * n_cand);
  p.cand_tok = cand_tok;
  p.cand_logit = cand_logit;
  p.cand_node = cand_node;
  p.row_lse = row_lse;
  p.prev_logp = prev_logp;
  p.prev_ids = prev_ids;
  p.out_ids = out_ids;
  p.out_logp = out_logp;
  p.out_node = out_node;
  p.out_parent = out_parent;
  p.pdl = pdl;
  return launch_merge(p, stream);
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("VTNK_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

}  // namespace vtnk

using namespace vtnk;

extern "C" {

const char* vtnk_last_error(void) { return g_err; }

int vtnk_version(void) { return 100; }

int vtnk_constrained_node_transition(const void* logits, int32_t dtype, int64_t B, int64_t N,
                                     int64_t logits_stride, const int64_t* cur_node,
                                     const vtnk_csr_t* csr, int64_t max_branches,
                                     void* corrected_logits, int64_t* next_node,
                                     int64_t* valid_idxs, void* stream) {
  int rc = check_csr(csr);
  if (rc) return rc;
  VTNK_REQUIRE(B >= 0 && N >= 1 && logits_stride >= N, "bad logits shape");
  VTNK_REQUIRE(max_branches >= 0, "max_branches < 0");
  VTNK_REQUIRE(B == 0 || (logits && cur_node && corrected_logits), "NULL pointer");
  VTNK_REQUIRE(B == 0 || max_branches == 0 || (next_node && valid_idxs), "NULL pointer");
  return launch_mask(logits, dtype, B, N, logits_stride, cur_node, make_csr(*csr), max_branches,
                     corrected_logits, next_node, valid_idxs, as_stream(stream));
}

int vtnk_fused_linear_constrained_node_transition(const vtnk_linear_t* lin,
                                                  const int64_t* cur_node,
                                                  const vtnk_csr_t* csr, int64_t max_branches,
                                                  float* corrected_logits, int64_t* next_node,
                                                  int64_t* valid_idxs, void* stream) {
  int rc = check_step(lin, csr, max_branches);
  if (rc) return rc;
  VTNK_REQUIRE(lin->rows == 0 || (cur_node && corrected_logits), "NULL pointer");
  VTNK_REQUIRE(lin->rows == 0 || max_branches == 0 || (next_node && valid_idxs), "NULL pointer");
  RowsArgs p = rows_from(lin, cur_node, csr, max_branches);
  p.corrected = corrected_logits;
  p.next_node = next_node;
  p.valid_idxs = valid_idxs;
  return launch_rows(p, MODE_FUSED, lin->dtype, as_stream(stream));
}

int vtnk_fused_linear_constrained_node_transition_topk(const vtnk_linear_t* lin,
                                                       const int64_t* cur_node,
                                                       const vtnk_csr_t* csr, int64_t max_branches,
                                                       int64_t k, int64_t* next_node,
                                                       int64_t* valid_idxs, float* topk_logits,
                                                       int64_t* topk_idxs, void* stream) {
  int rc = check_step(lin, csr, max_branches);
  if (rc) return rc;
  VTNK_REQUIRE(k >= 1 && k <= max_branches, "k (%lld) must be in [1, max_branches=%lld]",
               (long long)k, (long long)max_branches);
  VTNK_REQUIRE(lin->rows == 0 || (cur_node && next_node && valid_idxs && topk_logits && topk_idxs),
               "NULL pointer");
  RowsArgs p = rows_from(lin, cur_node, csr, max_branches);
  p.k = static_cast<int>(k);
  p.buf_cap = static_cast<int>(max_branches);
  p.next_node = next_node;
  p.valid_idxs = valid_idxs;
  p.out_logit = topk_logits;
  p.out_tok = topk_idxs;
  return launch_rows(p, MODE_TOPK, lin->dtype, as_stream(stream));
}

int vtnk_fused_linear_constrained_node_transition_sampling(
    const vtnk_linear_t* lin, const int64_t* cur_node, const vtnk_csr_t* csr,
    int64_t max_branches, uint64_t seed, const float* temperature, int64_t* next_node,
    int64_t* valid_idxs, float* sample, void* stream) {
  int rc = check_step(lin, csr, max_branches);
  if (rc) return rc;
  VTNK_REQUIRE(lin->rows == 0 || (cur_node && sample), "NULL pointer");
  VTNK_REQUIRE(lin->rows == 0 || max_branches == 0 || (next_node && valid_idxs), "NULL pointer");
  RowsArgs p = rows_from(lin, cur_node, csr, max_branches);
  p.seed = seed;
  p.temperature = temperature;
  p.buf_cap = static_cast<int>(max_branches > 0 ? max_branches : 1);
  p.next_node = next_node;
  p.valid_idxs = valid_idxs;
  p.sample = sample;
  return launch_rows(p, MODE_SAMPLE, lin->dtype, as_stream(stream));
}

int vtnk_fused_linear_constrained_node_transition_topk_ix(
    const vtnk_linear_t* lin, const int64_t* cur_node, const vtnk_csr_t* csr,
    int64_t max_branches, int64_t k, const vtnk_child_index_t* index, int64_t* next_node,
    int64_t* valid_idxs, float* topk_logits, int64_t* topk_idxs, void* stream) {
  int rc = check_step(lin, csr, max_branches);
  if (rc) return rc;
  VTNK_REQUIRE(k >= 1 && k <= max_branches, "k (%lld) must be in [1, max_branches=%lld]",
               (long long)k, (long long)max_branches);
  VTNK_REQUIRE(lin->rows == 0 || (topk_logits && topk_idxs), "NULL pointer");
  VTNK_REQUIRE((next_node == nullptr) == (valid_idxs == nullptr),
               "next_node and valid_idxs are both given or both NULL");
  if (lin->rows == 0) return VTNK_OK;
  cudaStream_t s = as_stream(stream);
  rc = tc_step(lin, cur_node, csr, max_branches, k, index, topk_idxs, topk_logits, nullptr,
               nullptr, 0, 0, nullptr, nullptr, true, s);
  if (rc == VTNK_ERR_UNSUPPORTED) {
    RowsArgs p = rows_from(lin, cur_node, csr, max_branches);
    p.k = static_cast<int>(k);
    p.buf_cap = static_cast<int>(max_branches);
    p.next_node = next_node;
    p.valid_idxs = valid_idxs;
    p.out_logit = topk_logits;
    p.out_tok = topk_idxs;
    return launch_rows(p, MODE_TOPK, lin->dtype, s);
  }
  if (rc || !next_node) return rc;
  return launch_tables(lin->rows, cur_node, make_csr(*csr), max_branches, next_node, valid_idxs,
                       s);
}

int vtnk_fused_linear_constrained_node_transition_sampling_ix(
    const vtnk_linear_t* lin, const int64_t* cur_node, const vtnk_csr_t* csr,
    int64_t max_branches, uint64_t seed, const float* temperature,
    const vtnk_child_index_t* index, int64_t* next_node, int64_t* valid_idxs, float* sample,
    int64_t* sample_node, void* stream) {
  int rc = check_step(lin, csr, max_branches);
  if (rc) return rc;
  VTNK_REQUIRE(lin->rows == 0 || sample, "NULL pointer");
  VTNK_REQUIRE((next_node == nullptr) == (valid_idxs == nullptr),
               "next_node and valid_idxs are both given or both NULL");
  if (lin->rows == 0) return VTNK_OK;
  cudaStream_t s = as_stream(stream);
  rc = tc_step(lin, cur_node, csr, max_branches, 1, index, nullptr, nullptr, sample_node, nullptr,
               1, seed, temperature, sample, true, s);
  if (rc == VTNK_ERR_UNSUPPORTED) {
    RowsArgs p = rows_from(lin, cur_node, csr, max_branches);
    p.seed = seed;
    p.temperature = temperature;
    p.buf_cap = static_cast<int>(max_branches > 0 ? max_branches : 1);
    p.next_node = next_node;
    p.valid_idxs = valid_idxs;
    p.sample = sample;
    p.out_node = sample_node;
    return launch_rows(p, MODE_SAMPLE, lin->dtype, s);
  }
  if (rc || !next_node) return rc;
  return launch_tables(lin->rows, cur_node, make_csr(*csr), max_branches, next_node, valid_idxs,
                       s);
}

int vtnk_gumbel_noise(uint64_t seed, int64_t rows, int64_t max_branches, float* out,
                      void* stream) {
  VTNK_REQUIRE(rows >= 0 && max_branches >= 0, "bad shape");
  VTNK_REQUIRE(rows * max_branches == 0 || out, "NULL pointer");
  return launch_gumbel(seed, rows, max_branches, out, as_stream(stream));
}

int vtnk_build_child_index(const vtnk_csr_t* csr, const vtnk_child_index_t* index,
                           void* stream) {
  int rc = check_csr(csr);
  if (rc) return rc;
  VTNK_REQUIRE(index != nullptr, "index is NULL");
  VTNK_REQUIRE(index->node_lo >= 0 && index->node_hi >= index->node_lo, "bad node range");
  VTNK_REQUIRE(index->window_n >= 1 && index->window_n <= 256 && index->window_lo >= 0,
               "window must hold 1..256 tokens");
  VTNK_REQUIRE(index->node_hi == index->node_lo || index->masks, "masks is NULL");
  VTNK_REQUIRE((reinterpret_cast<uintptr_t>(index->masks) & 15) == 0,
               "masks must be 16-byte aligned");
  return launch_build_child_index(make_csr(*csr), const_cast<uint32_t*>(index->masks),
                                  index->flags, index->node_lo, index->node_hi, index->window_lo,
                                  static_cast<int>(index->window_n), as_stream(stream));
}

int vtnk_beam_step(const vtnk_linear_t* lin, const int64_t* cur_node, const vtnk_csr_t* csr,
                   int64_t max_branches, int64_t n_cand, const vtnk_child_index_t* index,
                   int64_t* cand_tok, float* cand_logit, int64_t* cand_node, float* row_lse,
                   void* stream) {
  int rc = check_step(lin, csr, max_branches);
  if (rc) return rc;
  VTNK_REQUIRE(n_cand >= 1 && n_cand <= 1024, "n_cand out of range");
  VTNK_REQUIRE(lin->rows == 0 || (cand_tok && cand_logit && cand_node && row_lse),
               "NULL pointer");
  return beam_step_impl(lin, cur_node, csr, max_branches, n_cand, index, cand_tok, cand_logit,
                        cand_node, row_lse, true, as_stream(stream));
}

int vtnk_beam_candidates_from_logits(const void* logits, int32_t dtype, int64_t B, int64_t N,
                                     int64_t logits_stride, const int64_t* cur_node,
                                     const vtnk_csr_t* csr, int64_t max_branches, int64_t n_cand,
                                     int64_t* cand_tok, float* cand_logit, int64_t* cand_node,
                                     float* row_lse, void* stream) {
  int rc = check_csr(csr);
  if (rc) return rc;
  VTNK_REQUIRE(B >= 0 && N >= 1 && logits_stride >= N, "bad logits shape");
  VTNK_REQUIRE(max_branches >= 0 && max_branches <= (1 << 20), "max_branches out of range");
  VTNK_REQUIRE(n_cand >= 1 && n_cand <= 1024, "n_cand out of range");
  VTNK_REQUIRE(B == 0 || (logits && cand_tok && cand_logit && cand_node && row_lse),
               "NULL pointer");
  return launch_logits_beam(logits, dtype, B, N, logits_stride, cur_node, make_csr(*csr),
                            max_branches, static_cast<int>(n_cand), cand_tok, cand_logit,
                            cand_node, row_lse, as_stream(stream));
}

int vtnk_beam_merge(int64_t level, int64_t B, int64_t k, int64_t n_cand,
                    const int64_t* cand_tok, const float* cand_logit, const int64_t* cand_node,
                    const float* row_lse, const float* prev_logp, const int64_t* prev_ids,
                    int64_t* out_ids, float* out_logp, int64_t* out_node, int64_t* out_parent,
                    void* stream) {
  return merge_impl(level, B, k, n_cand, cand_tok, cand_logit, cand_node, row_lse, prev_logp,
                    prev_ids, out_ids, out_logp, out_node, out_parent, false, as_stream(stream));
}

size_t vtnk_beam_search_workspace_bytes(const vtnk_search_t* s) {
  if (!s) return 0;
  return search_layout(s).total;
}

int vtnk_beam_search(const vtnk_search_t* s, void* workspace, size_t workspace_bytes,
                     int64_t* out_ids, float* out_logp, int64_t* out_node, void* stream) {
  return beam_search_run(s, workspace, workspace_bytes, out_ids, out_logp, out_node, stream, true);
}

}  // extern "C"

namespace vtnk {
int beam_search_run(const vtnk_search_t* s, void* workspace, size_t workspace_bytes,
                    int64_t* out_ids, float* out_logp, int64_t* out_node, void* stream,
                    bool stream_k) {
  VTNK_REQUIRE(s != nullptr, "search is NULL");
  VTNK_REQUIRE(s->levels >= 1 && s->batch >= 0 && s->beams >= 1 && s->n_cand >= 1,
               "bad search sizes");
  VTNK_REQUIRE(s->beams <= s->n_cand, "beams must not exceed candidates per beam");
  VTNK_REQUIRE(s->hidden && s->weight && s->layer_max_branches, "NULL search pointer");
  int rc = check_csr(&s->csr);
  if (rc) return rc;
  if (s->batch == 0) return VTNK_OK;
  const SearchLayout L = search_layout(s);
  VTNK_REQUIRE(workspace && workspace_bytes >= L.total, "workspace too small (%zu < %zu)",
               workspace_bytes, L.total);
  VTNK_REQUIRE(out_ids && out_logp && out_node, "NULL output");
  char* ws = static_cast<char*>(workspace);
  auto at = [&](size_t off) { return static_cast<void*>(ws + off); };
  int64_t* cand_tok = static_cast<int64_t*>(at(L.cand_tok));
  int64_t* cand_node = static_cast<int64_t*>(at(L.cand_node));
  float* cand_logit = static_cast<float*>(at(L.cand_logit));
  float* lse = static_cast<float*>(at(L.lse));
  int64_t* parent = static_cast<int64_t*>(at(L.parent));
  cudaStream_t st = as_stream(stream);

  const int64_t* prev_node = nullptr;
  const float* prev_logp = nullptr;
  const int64_t* prev_ids = nullptr;
  for (int64_t level = 0; level < s->levels; ++level) {
    vtnk_linear_t lin{};
    lin.a = s->hidden[level];
    lin.rows = level == 0 ? s->batch : s->batch * s->beams;
    lin.hidden = s->hidden_dim;
    lin.a_stride = s->hidden_stride;
    lin.b = s->weight;
    lin.n_vocab = s->n_vocab;
    lin.b_stride_k = 1;
    lin.b_stride_n = s->hidden_dim;
    lin.bias = s->bias;
    lin.dtype = s->dtype;
    rc = check_linear(&lin);
    if (rc) return rc;
    const vtnk_child_index_t* idx = s->index ? &s->index[level] : nullptr;
    const bool last = level + 1 == s->levels;
    const int slot = static_cast<int>(level & 1);
    int64_t* ids = last ? out_ids : static_cast<int64_t*>(at(L.ids[slot]));
    float* logp = last ? out_logp : static_cast<float*>(at(L.logp[slot]));
    int64_t* node = last ? out_node : static_cast<int64_t*>(at(L.node[slot]));
    // Level 0 has one candidate list per query, so its merge is the list
    // itself: the tile kernel writes the beams directly when it takes the
    // level (k <= n_cand); otherwise the step and the merge run as below.
    rc = VTNK_ERR_UNSUPPORTED;
    if (level == 0 && s->beams <= s->n_cand && lin.rows > 0) {
      TcArgs l0{};
      l0.l0_ids = ids;
      l0.l0_logp = logp;
      l0.l0_node = node;
      l0.l0_k = static_cast<int>(s->beams);
      rc = tc_step(&lin, prev_node, &s->csr, s->layer_max_branches[level], s->n_cand, idx,
                   nullptr, nullptr, nullptr, nullptr, 0, 0, nullptr, nullptr, stream_k, st, &l0);
      if (rc != VTNK_OK && rc != VTNK_ERR_UNSUPPORTED) return rc;
    }
    if (rc == VTNK_ERR_UNSUPPORTED) {
      // After the first kernel of the search, step and merge are chained
      // with programmatic dependent launch: each waits for its predecessor's
      // results inside the kernel, so launch gaps and the next level's
      // operand stream overlap the previous kernel's tail.
      const bool pdl = level > 0 && pdl_enabled();
      rc = beam_step_impl(&lin, prev_node, &s->csr, s->layer_max_branches[level], s->n_cand,
                          idx, cand_tok, cand_logit, cand_node, lse, stream_k, st, pdl);
      if (rc) return rc;
      rc = merge_impl(level, s->batch, s->beams, s->n_cand, cand_tok, cand_logit, cand_node, lse,
                      prev_logp, prev_ids, ids, logp, node, parent, pdl, st);
      if (rc) return rc;
    }
    prev_node = node;
    prev_logp = logp;
    prev_ids = ids;
  }
  return VTNK_OK;
}
}  // namespace vtnk

extern "C" {

int vtnk_device_status(int reset) {
  const cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_status(e, "device synchronize");
  int v = 0;
  const int rc = read_tc_status(&v, reset != 0);
  if (rc) return rc;
  if (v != 0) {
    set_error("a tile kernel's bounded wait expired (code %d)", v);
    return VTNK_ERR_DEVICE;
  }
  return VTNK_OK;
}

int vtnk_synth_normal(uint64_t seed, uint64_t stream_id, int64_t row0, int64_t rows, int64_t H,
                      const void* table, int32_t dtype, void* out, void* stream) {
  VTNK_REQUIRE(rows >= 0 && H >= 1 && row0 >= 0, "bad synth shape");
  VTNK_REQUIRE(rows == 0 || (table && out), "NULL pointer");
  VTNK_REQUIRE(dtype == VTNK_F32 || dtype == VTNK_BF16, "synth dtype must be F32 or BF16");
  const uint64_t key = mix64((seed << 20) ^ stream_id);
  return launch_synth(key, row0 * H, rows * H, table, dtype, out, as_stream(stream));
}

}  // extern "C"
