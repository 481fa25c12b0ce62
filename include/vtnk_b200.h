/*
 * vtnk_b200 -- C ABI of the B200 (sm_100a) trie-constrained decoding step.
 *
 * Every entry point takes plain device pointers and sizes, launches on the
 * given CUDA stream (NULL = legacy default stream), never synchronises the
 * host, never allocates device memory and returns VTNK_OK or an error code
 * (message via vtnk_last_error()).  Outputs are written in full, including
 * the -1 / -inf padding the reference's ops pre-fill.
 *
 * Reference: EdoardoBotta/RecTokens, Python/Triton.  Each declaration cites the
 * reference interface it replaces.
 */
#ifndef VTNK_B200_H
#define VTNK_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* element types of the dense operands */
enum { VTNK_F32 = 0, VTNK_BF16 = 1, VTNK_F16 = 2 };

/* status codes */
enum {
  VTNK_OK = 0,
  VTNK_ERR_ARG = 1,         /* bad argument (shape, stride, null pointer) */
  VTNK_ERR_CUDA = 2,        /* a CUDA runtime call failed */
  VTNK_ERR_UNSUPPORTED = 3, /* valid input this build does not handle */
  VTNK_ERR_DEVICE = 4       /* a kernel reported a failure (bounded wait ran out) */
};

/* CSR trie: the reference's CompactCSRTrie (rectokens/schemas/compact_csr_trie.py:14-35).
 * row_ptrs [n_nodes] int64 (no trailing nnz entry), cols = stacked_cols_vals[0],
 * vals = stacked_cols_vals[1], both [nnz + 1] int64 with a -1 sentinel last. */
typedef struct {
  const int64_t* row_ptrs;
  const int64_t* cols;
  const int64_t* vals;
  int64_t n_nodes;
  int64_t nnz;
} vtnk_csr_t;

/* The fused linear operand: a [rows, hidden] (row stride a_stride elements,
 * unit column stride), b = W.T viewed as [hidden, n_vocab] with element strides
 * (b_stride_k, b_stride_n) -- the reference's (b_stride_K, b_stride_N),
 * rectokens/kernels/constrained_node_transition.py:426-430.  bias [n_vocab] or
 * NULL.  a, b and bias share `dtype`. */
typedef struct {
  const void* a;
  int64_t rows;
  int64_t hidden;
  int64_t a_stride;
  const void* b;
  int64_t n_vocab;
  int64_t b_stride_k;
  int64_t b_stride_n;
  const void* bias;
  int32_t dtype;
} vtnk_linear_t;

/* Replaces vtnk::_constrained_node_transition_op
 * (rectokens/kernels/constrained_node_transition.py:14-61): copy `logits`
 * [B, N] (row stride logits_stride) to corrected_logits [B, N] (contiguous,
 * same dtype) with every column that is not a child of cur_node[b] set to
 * -inf; next_node / valid_idxs [B, max_branches] get the child node ids /
 * tokens, -1 padded. */
int vtnk_constrained_node_transition(const void* logits, int32_t dtype, int64_t B, int64_t N,
                                     int64_t logits_stride, const int64_t* cur_node,
                                     const vtnk_csr_t* csr, int64_t max_branches,
                                     void* corrected_logits, int64_t* next_node,
                                     int64_t* valid_idxs, void* stream);

/* Replaces vtnk::_fused_linear_constrained_node_transition_op (kernels:388-447):
 * corrected_logits [rows, n_vocab] fp32 = a @ b (+ bias) on child columns,
 * -inf elsewhere; next_node / valid_idxs [rows, max_branches]. */
int vtnk_fused_linear_constrained_node_transition(const vtnk_linear_t* lin,
                                                  const int64_t* cur_node,
                                                  const vtnk_csr_t* csr, int64_t max_branches,
                                                  float* corrected_logits, int64_t* next_node,
                                                  int64_t* valid_idxs, void* stream);

/* Replaces vtnk::_fused_linear_constrained_node_transition_topk_op (kernels:791-853):
 * topk_logits [rows, k] fp32 descending and topk_idxs [rows, k] token ids
 * (-1 / -inf when a row has fewer than k children; ties go to the lower
 * branch slot); next_node / valid_idxs [rows, max_branches].
 * Requires 1 <= k <= max_branches (torch.topk raises otherwise). */
int vtnk_fused_linear_constrained_node_transition_topk(const vtnk_linear_t* lin,
                                                       const int64_t* cur_node,
                                                       const vtnk_csr_t* csr, int64_t max_branches,
                                                       int64_t k, int64_t* next_node,
                                                       int64_t* valid_idxs, float* topk_logits,
                                                       int64_t* topk_idxs, void* stream);

/* Replaces vtnk::_fused_linear_constrained_node_transition_sampling_op
 * (kernels:562-635): Gumbel-max sample per row, argmax over children of
 * logit / T + g with g from Philox(seed, row * max_branches + slot) exactly as
 * the reference's kernel draws it (kernels:359-380); sample [rows] fp32 token
 * id, -1.0 when none.  temperature: device pointer to one fp32 (NULL = 1). */
int vtnk_fused_linear_constrained_node_transition_sampling(
    const vtnk_linear_t* lin, const int64_t* cur_node, const vtnk_csr_t* csr,
    int64_t max_branches, uint64_t seed, const float* temperature, int64_t* next_node,
    int64_t* valid_idxs, float* sample, void* stream);

/* The Gumbel noise the sampling kernel adds at (row, slot), written to
 * out [rows, max_branches] fp32 so a checker can replay a sampling call
 * (kernels:372-374 formula; no reference counterpart as an entry point). */
int vtnk_gumbel_noise(uint64_t seed, int64_t rows, int64_t max_branches, float* out,
                      void* stream);

/* Child-bitmask index of one trie depth, for the tensor-core beam step: for
 * every node id in [node_lo, node_hi) a 256-bit mask (8 uint32 words, bit i =
 * token window_lo + i is a child).  A node whose children are not in
 * ascending token order or not all inside the window has an all-zero mask
 * (its rows are then computed by an exact per-row path).  Derived data: the
 * CSR arrays stay the reference layout; no reference counterpart. */
typedef struct {
  const uint32_t* masks;  /* [node_hi - node_lo, 8], 16-byte aligned */
  int64_t node_lo;
  int64_t node_hi;
  int64_t window_lo;
  int64_t window_n;       /* 1..256 */
  uint32_t* flags;        /* optional, one word written by vtnk_build_child_index: bit 0 set
                             when every child of every node in range has node id = its
                             edge index + 1 (BFS numbering, as the reference's builders
                             produce); the beam step then computes child node ids
                             instead of reading vals.  NULL: always read vals. */
} vtnk_child_index_t;

/* The _topk entry point with the depth's child index: the tcgen05 tile
 * kernel computes the logits of the 256-token window on the tensor cores and
 * selects the top k in its epilogue (same outputs and tie rule as
 * vtnk_fused_linear_constrained_node_transition_topk, which it falls back to
 * when index is NULL or the shape is not tile-able: bf16, W row-contiguous,
 * rows >= 128, k <= 32).  cur_node NULL: every row at the root.
 * next_node / valid_idxs may both be NULL to skip the
 * [rows, max_branches] tables.  Called by the ops layer's
 * fused_linear_constrained_node_transition_topk (ops/...:73-92 in the
 * reference) when the trie depth has an index. */
int vtnk_fused_linear_constrained_node_transition_topk_ix(
    const vtnk_linear_t* lin, const int64_t* cur_node, const vtnk_csr_t* csr,
    int64_t max_branches, int64_t k, const vtnk_child_index_t* index, int64_t* next_node,
    int64_t* valid_idxs, float* topk_logits, int64_t* topk_idxs, void* stream);

/* The _sampling entry point with the depth's child index: Gumbel-max in the
 * tile kernel's epilogue (same noise, temperature division and first-maximum
 * rule as vtnk_fused_linear_constrained_node_transition_sampling, its
 * fallback).  sample_node (optional, [rows] int64) receives the sampled
 * child's node id (-1 when none), the next level's cur_node.  next_node /
 * valid_idxs may both be NULL. */
int vtnk_fused_linear_constrained_node_transition_sampling_ix(
    const vtnk_linear_t* lin, const int64_t* cur_node, const vtnk_csr_t* csr,
    int64_t max_branches, uint64_t seed, const float* temperature,
    const vtnk_child_index_t* index, int64_t* next_node, int64_t* valid_idxs, float* sample,
    int64_t* sample_node, void* stream);

/* Builds index->masks (caller memory, (node_hi - node_lo) * 32 bytes) and,
 * when index->flags is given, its flag word, for the nodes and window
 * described by `index` (no reference counterpart). */
int vtnk_build_child_index(const vtnk_csr_t* csr, const vtnk_child_index_t* index,
                           void* stream);

/* One beam-search level, fused: for every row, the n_cand best children by
 * logit (ties to the lower slot), their logits, tokens and child node ids, and
 * the row's log-sum-exp over all children.  Replaces the per-level work of
 * decode_one_step (rectokens/decoding/constrained_decoding.py:245-297: LM-head
 * logits, constrained_node_transition, topk(beam_size), log_softmax) for the
 * item-token rows of the head.  cur_node NULL = every row at the root.
 * index: the child-bitmask index of this depth (enables the tcgen05 tile
 * kernel for bf16, rows >= 128, n_cand <= 32), or NULL (CUDA-core row kernel).
 * Outputs: cand_tok / cand_node int64 [rows, n_cand], cand_logit fp32
 * [rows, n_cand] (-1 / -inf padded), row_lse fp32 [rows]. */
int vtnk_beam_step(const vtnk_linear_t* lin, const int64_t* cur_node, const vtnk_csr_t* csr,
                   int64_t max_branches, int64_t n_cand, const vtnk_child_index_t* index,
                   int64_t* cand_tok, float* cand_logit, int64_t* cand_node, float* row_lse,
                   void* stream);

/* The per-level candidate work of decode_one_step on a CSR level for a
 * language model that returns full-vocabulary logits
 * (rectokens/decoding/constrained_decoding.py:271-303 and 372-383: the mask
 * op, log_softmax, topk(beam_size) and the next-node lookup), in one pass:
 * for each row of logits [B, N] (row stride logits_stride, dtype F32 / BF16 /
 * F16) at trie node cur_node[b] (NULL = root), the n_cand best children by
 * logit (ties to the lower slot) with token ids and child node ids, and the
 * row's log-sum-exp over its children -- the outputs of vtnk_beam_step, ready
 * for vtnk_beam_merge.  Only the children's columns are read. */
int vtnk_beam_candidates_from_logits(const void* logits, int32_t dtype, int64_t B, int64_t N,
                                     int64_t logits_stride, const int64_t* cur_node,
                                     const vtnk_csr_t* csr, int64_t max_branches, int64_t n_cand,
                                     int64_t* cand_tok, float* cand_logit, int64_t* cand_node,
                                     float* row_lse, void* stream);

/* Beam merge (rectokens/decoding/constrained_decoding.py:305-349, next node
 * :368-383).  Inputs are vtnk_beam_step's outputs: a candidate whose logit is
 * -inf is missing (its token and node are -1).  level 0: each of the B
 * queries keeps its k best of n_cand candidates (rows = B).  level > 0: total = prev_logp[parent] + cand logp over
 * the k * n_cand candidates of a query (rows = B * k), the k best kept, ties to
 * the lower candidate index.  prev_ids [B*k, level] int64; out_ids
 * [B*k, level+1]; out_logp, out_node, out_parent [B*k]. */
int vtnk_beam_merge(int64_t level, int64_t B, int64_t k, int64_t n_cand,
                    const int64_t* cand_tok, const float* cand_logit, const int64_t* cand_node,
                    const float* row_lse, const float* prev_logp, const int64_t* prev_ids,
                    int64_t* out_ids, float* out_logp, int64_t* out_node, int64_t* out_parent,
                    void* stream);

/* A full L-level constrained beam search (autoregressive_generate with
 * GenerationConfig(steps=L, k=beams, beam_size=n_cand, temperature=0),
 * rectokens/decoding/constrained_decoding.py:140-179) for an LM whose item-token
 * hidden state at level l is hidden[l] (rows = batch at level 0, batch * beams
 * after, row stride hidden_stride).  weight = W [n_vocab, hidden] row-major. */
typedef struct {
  const void* const* hidden;          /* host array [levels] of device pointers */
  int64_t hidden_stride;
  const void* weight;
  int64_t n_vocab;
  int64_t hidden_dim;
  const void* bias;
  int32_t dtype;
  vtnk_csr_t csr;
  const int64_t* layer_max_branches;  /* host array [levels] */
  const vtnk_child_index_t* index;    /* host array [levels] (entries with masks
                                         NULL use the row kernel), or NULL */
  int64_t levels;
  int64_t batch;
  int64_t beams;
  int64_t n_cand;
} vtnk_search_t;

/* Bytes of device scratch vtnk_beam_search needs for `s`. */
size_t vtnk_beam_search_workspace_bytes(const vtnk_search_t* s);

/* Runs the search; out_ids [batch*beams, levels] int64, out_logp
 * [batch*beams] fp32, out_node [batch*beams] int64 (final trie node). */
int vtnk_beam_search(const vtnk_search_t* s, void* workspace, size_t workspace_bytes,
                     int64_t* out_ids, float* out_logp, int64_t* out_node, void* stream);

/* Size of the scratch array built into the library for
 * vtnk_beam_search_noalloc (held on every GPU that loads the library). */
#define VTNK_NOALLOC_SCRATCH_BYTES (32u << 20)

/* vtnk_beam_search without a caller workspace, for callers that may not
 * allocate device memory on the decode path (a plugin whose host process owns
 * all device memory through its own pool, or code that must avoid the device
 * synchronisation an allocation can trigger).  Inputs and outputs are as for
 * vtnk_beam_search; the scratch is a fixed array of VTNK_NOALLOC_SCRATCH_BYTES
 * inside the library, so searches whose vtnk_beam_search_workspace_bytes
 * exceed it are rejected (VTNK_ERR_UNSUPPORTED, message names both sizes).
 * The first call on each device looks up that array's device address (make
 * it with the device current, before any stream capture).  Every call on a
 * device shares the one array: calls that overlap on the GPU (different
 * streams, or host threads) race and corrupt each other's results.  No
 * counterpart in the reference. */
int vtnk_beam_search_noalloc(const vtnk_search_t* s, int64_t* out_ids, float* out_logp,
                             int64_t* out_node, void* stream);

/* Device CSR trie builder (replaces CompactCSRTrie.from_sorted_batch,
 * rectokens/schemas/compact_csr_trie.py:97-177, and the catalog sort of
 * ItemAwareTokenizer.build_item_trie, rectokens/integrations/hf/tokenizer.py:
 * 198-230): the same row_ptrs / stacked_cols_vals / layer_max_branches /
 * dense tables, built by sort, scan and segment kernels.  Two phases, because
 * the output sizes depend on the catalog:
 *   1. vtnk_trie_count: packs each item's `levels` token ids (each in
 *      [0, vocab)) into a 64-bit key, radix-sorts the keys unless
 *      assume_sorted (the reference requires sorted input; duplicates are
 *      allowed), numbers the nodes in BFS order and writes counts[0] =
 *      n_nodes (-1 when a token is out of range), counts[1] = nnz and
 *      counts[2 + d] = nodes at depth d (device int64[levels + 2]).
 *   2. vtnk_trie_fill (after the caller read the counts and sized the
 *      outputs): row_ptrs [n_nodes], cols_vals [2, nnz + 1] (with the -1
 *      sentinel column), layer_max_branches [levels] (device int64), and for
 *      dense_layers > 0 the prefix masks dense_masks[d] (vocab^(d+1) bytes
 *      of 0/1) and dense_states (vocab^dense_layers int64).
 * Both read and write the caller's workspace (vtnk_trie_workspace_bytes);
 * nothing is allocated.  Requires levels * bits(vocab - 1) <= 64 and
 * n_items * levels < 2^31. */
size_t vtnk_trie_workspace_bytes(int64_t n_items, int64_t levels);
int vtnk_trie_count(const int64_t* sem_ids, int64_t n_items, int64_t levels, int64_t vocab,
                    int assume_sorted, void* workspace, size_t workspace_bytes, int64_t* counts,
                    void* stream);
int vtnk_trie_fill(int64_t n_items, int64_t levels, int64_t vocab, int64_t dense_layers,
                   void* workspace, size_t workspace_bytes, int64_t n_nodes, int64_t nnz,
                   int64_t* row_ptrs, int64_t* cols_vals, int64_t* layer_max_branches,
                   uint8_t* const* dense_masks, int64_t* dense_states, void* stream);

/* Result all-gather over peer memory for the batch-sharded search (replaces
 * the NCCL all-gather of the ranks' results; the reference has no
 * multi-GPU path).  Every rank owns a gather buffer of 2 * world *
 * record_bytes bytes and a flag array of 8 uint32 words (both zeroed before
 * the first call, opened on the other ranks through the IPC helpers below),
 * plus two local uint32 epoch words and one int status word (zeroed).
 * vtnk_peer_gather packs this rank's search result (ids int64 [n, levels],
 * logp fp32 [n], node int64 [n]) into the record layout
 *   ids int32 [n, levels] | node int32 [n] | logp fp32 [n]   (16-byte aligned regions)
 * stores it into slot `rank` of half (e & 1) of every rank's buffer, where e
 * counts this rank's calls from 1, then waits -- bounded by wait_ns (0: 2 s)
 * -- until every rank has pushed its record e.  On return (stream order)
 * half (e & 1) of this rank's buffer holds every rank's record, valid until
 * this rank's call after next.  status: 1 = a wait ran out, 2 = an id did not
 * fit int32.  world <= 8; plain stores over NVLink, no multicast. */
typedef struct {
  int32_t world;
  int32_t rank;
  int64_t record_bytes;    /* >= vtnk_peer_record_bytes(n, levels) */
  void* records[8];        /* every rank's gather buffer, as mapped in this process */
  uint32_t* flags[8];      /* every rank's flag array, as mapped in this process */
  uint32_t* epoch;         /* this rank's 2 epoch words (device) */
  int* status;             /* this rank's status word (device) */
  uint64_t wait_ns;
} vtnk_peer_group_t;

int64_t vtnk_peer_record_bytes(int64_t n, int64_t levels);
int vtnk_peer_gather(const vtnk_peer_group_t* g, const int64_t* ids, const float* logp,
                     const int64_t* node, int64_t n, int64_t levels, void* stream);
/* CUDA IPC helpers for setting up a peer group (one process per GPU).  The
 * handle names the allocation that holds dev_ptr; offset_out is dev_ptr's
 * offset inside it, to be added to the pointer the peer opens. */
int vtnk_ipc_handle_bytes(void);
int vtnk_ipc_get_handle(const void* dev_ptr, void* handle_out, int64_t* offset_out);
int vtnk_ipc_open_handle(const void* handle, void** dev_ptr_out);
int vtnk_ipc_close_handle(void* dev_ptr);

/* Synthetic hidden states (benchmark / test input generator, no reference
 * counterpart): out[r, h] = table[mix64(key(seed, stream_id) ^ ((row0 + r) * H + h)) >> 48]
 * with the 65,536-entry quantile table given as bf16 bits (dtype BF16) or fp32
 * (dtype F32).  Same function as rectokens_b200/synthetic.py. */
int vtnk_synth_normal(uint64_t seed, uint64_t stream_id, int64_t row0, int64_t rows,
                      int64_t H, const void* table, int32_t dtype, void* out, void* stream);

/* Synchronises the current device and reports whether any tile kernel on it
 * gave up a bounded wait since the last reset (VTNK_ERR_DEVICE, with the wait's
 * code in vtnk_last_error()); reset != 0 clears the record.  Diagnostic, not on
 * the hot path (no reference counterpart: the reference's kernels have no
 * bounded waits). */
int vtnk_device_status(int reset);

/* Bound, in nanoseconds, of every wait inside the tile kernel (process-wide,
 * read at each launch; 0 restores the default of 2 s).  A wait that runs out
 * makes its CTA drain its copies and MMAs with bounded waits, free its tensor
 * memory and exit; vtnk_device_status then reports VTNK_ERR_DEVICE.  No
 * reference counterpart (the reference's kernels do not wait on barriers). */
int vtnk_set_wait_limit_ns(uint64_t ns);

/* Test hook for the failure path above: the next n tile-kernel launches
 * issue no operand copies, so their first wait runs out after the wait
 * limit and the launch ends with the device status set (its outputs are
 * then undefined).  n = 0 cancels.  No reference counterpart. */
int vtnk_debug_stall_launches(int n);

/* Human-readable description of the last error on this host thread. */
const char* vtnk_last_error(void);

/* Library ABI version (major * 100 + minor). */
int vtnk_version(void);

#ifdef __cplusplus
}
#endif

#endif /* VTNK_B200_H */
