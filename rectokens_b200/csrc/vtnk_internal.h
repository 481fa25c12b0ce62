// Internal launch interfaces shared by the vtnk_b200 translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "vtnk_common.cuh"

namespace vtnk {

enum { MODE_FUSED = 0, MODE_TOPK = 1, MODE_SAMPLE = 2, MODE_BEAM = 3 };

struct RowsArgs {
  const void* a;
  int64_t rows, H, a_stride;
  const void* b;
  int64_t N, b_sk, b_sn;
  const void* bias;
  const int64_t* cur_node;  // nullptr: every row at the root
  Csr csr;
  int64_t mb;
  int k;                    // top-k (MODE_TOPK) or candidates per row (MODE_BEAM)
  uint64_t seed;
  const float* temperature;
  bool vec;                 // 16-byte vector loads of a and W rows are legal
  int buf_cap;              // shared-memory floats per warp
  float* corrected;         // MODE_FUSED  [rows, N]
  int64_t* next_node;       // MODE_FUSED/TOPK/SAMPLE [rows, mb]
  int64_t* valid_idxs;
  float* out_logit;         // MODE_TOPK topk_logits / MODE_BEAM cand_logit [rows, k]
  int64_t* out_tok;         // MODE_TOPK topk_idxs / MODE_BEAM cand_tok
  int64_t* out_node;        // MODE_BEAM cand_node / MODE_SAMPLE sampled child (optional)
  float* out_lse;           // MODE_BEAM [rows]
  float* sample;            // MODE_SAMPLE [rows]
};

struct MergeArgs {
  int64_t level, B;
  int k, n_cand, cap;
  const int64_t* cand_tok;
  const float* cand_logit;
  const int64_t* cand_node;
  const float* row_lse;
  const float* prev_logp;
  const int64_t* prev_ids;
  int64_t* out_ids;
  float* out_logp;
  int64_t* out_node;
  int64_t* out_parent;
  // Programmatic dependent launch inside a search: the merge may be scheduled
  // before the step kernel ends (it waits for the step's results itself).
  bool pdl;
};

// Whether searches chain their launches with programmatic dependent launch
// (VTNK_PDL=0 turns it off).
bool pdl_enabled();
// vtnk_beam_merge with the launch mode (pdl: inside a search, see MergeArgs).
int merge_impl(int64_t level, int64_t B, int64_t k, int64_t n_cand, const int64_t* cand_tok,
               const float* cand_logit, const int64_t* cand_node, const float* row_lse,
               const float* prev_logp, const int64_t* prev_ids, int64_t* out_ids, float* out_logp,
               int64_t* out_node, int64_t* out_parent, bool pdl, cudaStream_t stream);

// Tensor-core beam step (vtnk_tc.cu).
struct TcArgs {
  const void* a;            // bf16 [rows, H], row stride a_stride
  int64_t rows, H, a_stride;
  const void* w;            // bf16 W rows [N, H] (row stride w_stride), window rows used
  int64_t w_stride;
  int64_t n_vocab;          // rows of W
  int64_t window_lo;        // first token of the column window
  int window_n;             // <= 256
  const uint32_t* masks;    // child-bitmask index [idx_hi - idx_lo, 8]
  const uint32_t* flags;    // index flag word or nullptr (bit 0: node id = edge index + 1)
  int64_t idx_lo, idx_hi;
  const void* bias;         // bf16 [N] or nullptr
  const int64_t* cur_node;  // nullptr: root
  Csr csr;
  int64_t mb;
  int n_cand;
  int64_t* cand_tok;
  float* cand_logit;
  int64_t* cand_node;        // optional
  float* row_lse;            // optional
  int sample;                // 1: Gumbel-max sampling (n_cand == 1)
  uint64_t seed;
  const float* temperature;  // device scalar or nullptr (1)
  float* sample_f;           // optional: sampled token id as float, -1 when none
  // Level 0 of a beam search (every row its own query): the k <= n_cand best
  // candidates of each row become its beams directly -- ids [rows*k],
  // logp = logit - lse, node -- in place of the beam merge (optional).
  int64_t* l0_ids;
  float* l0_logp;
  int64_t* l0_node;
  int l0_k;
  bool pdl;  // launch as a programmatic dependent of the previous kernel (inside a search)
  // Stream-K workspace (all nullptr: whole tiles round-robin only).
  float* sk_part;                // sk_cap_pairs * 512 KB
  unsigned long long* sk_count;  // sk_count_cap words, zero before first use
  int64_t sk_cap_pairs, sk_count_cap;
  uint32_t sk_epoch;             // distinct per launch on this workspace, never 0
};

// Stream-K workspace of the library for (current device, stream): allocated
// on first use and kept; nullptr members when it cannot be had.
struct SkWorkspace {
  float* part;
  unsigned long long* count;
  int64_t cap_pairs, count_cap;
  uint32_t epoch;  // of this launch
};
SkWorkspace sk_workspace(cudaStream_t s);

// vtnk_beam_search with stream-K scheduling optional (off: no library
// workspace is allocated, for the allocation-free entry point).
int beam_search_run(const vtnk_search_t* s, void* workspace, size_t workspace_bytes,
                    int64_t* out_ids, float* out_logp, int64_t* out_node, void* stream,
                    bool stream_k);

int launch_rows(const RowsArgs& p, int mode, int dtype, cudaStream_t s);
int launch_mask(const void* logits, int dtype, int64_t B, int64_t N, int64_t ls,
                const int64_t* cur_node, const Csr& csr, int64_t mb, void* out, int64_t* nn,
                int64_t* vi, cudaStream_t s);
int launch_merge(const MergeArgs& p, cudaStream_t s);
int launch_logits_beam(const void* logits, int dtype, int64_t B, int64_t N, int64_t ls,
                       const int64_t* cur_node, const Csr& csr, int64_t mb, int k,
                       int64_t* tok, float* logit, int64_t* node, float* lse, cudaStream_t s);
int launch_synth(uint64_t key, int64_t e0, int64_t count, const void* table, int dtype, void* out,
                 cudaStream_t s);
int launch_gumbel(uint64_t seed, int64_t rows, int64_t mb, float* out, cudaStream_t s);
int launch_tables(int64_t rows, const int64_t* cur_node, const Csr& csr, int64_t mb,
                  int64_t* next_node, int64_t* valid_idxs, cudaStream_t s);

// Returns VTNK_ERR_UNSUPPORTED (without launching) when the shape does not
// fit the tile kernel; the caller then uses the row kernel.
int launch_beam_step_tc(const TcArgs& p, cudaStream_t s);
bool tc_enabled();
int launch_build_child_index(const Csr& csr, uint32_t* masks, uint32_t* flags, int64_t node_lo,
                             int64_t node_hi, int64_t window_lo, int window_n, cudaStream_t s);
// Reads (and optionally clears) the tile kernel's device status word.
int read_tc_status(int* out, bool reset);

}  // namespace vtnk
