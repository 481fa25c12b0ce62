// Device CSR trie builder: the reference's CompactCSRTrie.from_sorted_batch
// (rectokens/schemas/compact_csr_trie.py:97-177) and the catalog sort of
// ItemAwareTokenizer.build_item_trie (rectokens/integrations/hf/tokenizer.py:
// 198-230), as sort / scan / segment kernels.
//
//   pack     each item's L tokens into one 64-bit key (b bits per level,
//            b = bits of vocab - 1): key order == lexicographic row order
//   sort     LSD radix sort of the keys, 8-bit digits, stable block-local
//            ranking (warp match + per-warp digit counters), one histogram,
//            one exclusive scan and one scatter launch per digit
//   opens    item i opens a node at depth d when its prefix [0, d] differs
//            from item i-1's: d >= first differing level (from the keys' XOR)
//   number   inclusive scan of the opens, depth-major: the node id of
//            (depth d, item i) -- BFS order, root 0 -- exactly the reference's
//            cumsum numbering
//   fill     every opening writes its edge (token, node id); a node whose
//            parent opened at the same item is that parent's first child and
//            writes the parent's row pointer; last-level nodes (leaves) point
//            at nnz
//   branches each internal node's child count from consecutive row pointers,
//            max per depth
//   dense    prefix-membership masks and the depth-(dl-1) node table of the
//            first dense_lookup_layers levels
//
// Everything runs on the given stream; the two entry points never allocate
// (the caller passes a workspace of vtnk_trie_workspace_bytes).
#include <cstdint>

#include "vtnk_common.cuh"
#include "vtnk_internal.h"

namespace vtnk {
namespace trie {

constexpr int SCAN_THREADS = 1024;
constexpr int SCAN_ITEMS = 4;
constexpr int SCAN_TILE = SCAN_THREADS * SCAN_ITEMS;
constexpr int RS_THREADS = 256;
constexpr int RS_WARPS = RS_THREADS / 32;
constexpr int RS_PER_WARP = 256;
constexpr int RS_TILE = RS_WARPS * RS_PER_WARP;  // 2048 keys per block
constexpr int RADIX = 256;

// ------------------------------------------------------------------ scan (int32)
// Block-wide inclusive scan of one value per thread; returns the block total.
__device__ __forceinline__ int32_t block_scan_incl(int32_t v, int32_t* warp_tot, int32_t& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int32_t u = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += u;
  }
  if (lane == 31) warp_tot[warp] = v;
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    int32_t t = lane < nw ? warp_tot[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t u = __shfl_up_sync(0xffffffffu, t, o);
      if (lane >= o) t += u;
    }
    if (lane < nw) warp_tot[lane] = t;  // inclusive warp prefix
  }
  __syncthreads();
  const int32_t before = warp > 0 ? warp_tot[warp - 1] : 0;
  total = warp_tot[(blockDim.x >> 5) - 1];
  __syncthreads();
  return v + before;
}

__global__ void __launch_bounds__(SCAN_THREADS) scan_reduce(const int32_t* __restrict__ in,
                                                            int64_t n, int32_t* __restrict__ sums) {
  __shared__ int32_t wt[32];
  const int64_t base = static_cast<int64_t>(blockIdx.x) * SCAN_TILE + threadIdx.x * SCAN_ITEMS;
  int32_t s = 0;
#pragma unroll
  for (int j = 0; j < SCAN_ITEMS; ++j)
    if (base + j < n) s += in[base + j];
  int32_t total;
  block_scan_incl(s, wt, total);
  if (threadIdx.x == 0) sums[blockIdx.x] = total;
}

// Exclusive scan of the block sums in place (one block, chunks of 1024).
__global__ void __launch_bounds__(SCAN_THREADS) scan_sums(int32_t* sums, int64_t nb) {
  __shared__ int32_t wt[32];
  int32_t carry = 0;
  for (int64_t c0 = 0; c0 < nb; c0 += SCAN_THREADS) {
    const int64_t i = c0 + threadIdx.x;
    const int32_t v = i < nb ? sums[i] : 0;
    int32_t total;
    const int32_t incl = block_scan_incl(v, wt, total);
    if (i < nb) sums[i] = carry + incl - v;
    carry += total;
  }
}

__global__ void __launch_bounds__(SCAN_THREADS) scan_apply(const int32_t* in, int32_t* out,
                                                           int64_t n, const int32_t* sums,
                                                           int inclusive) {
  __shared__ int32_t wt[32];
  const int64_t base = static_cast<int64_t>(blockIdx.x) * SCAN_TILE + threadIdx.x * SCAN_ITEMS;
  int32_t x[SCAN_ITEMS];
  int32_t s = 0;
#pragma unroll
  for (int j = 0; j < SCAN_ITEMS; ++j) {
    x[j] = base + j < n ? in[base + j] : 0;
    s += x[j];
  }
  int32_t total;
  int32_t run = block_scan_incl(s, wt, total) - s + sums[blockIdx.x];
#pragma unroll
  for (int j = 0; j < SCAN_ITEMS; ++j) {
    if (inclusive) run += x[j];
    if (base + j < n) out[base + j] = run;
    if (!inclusive) run += x[j];
  }
}

int scan(const int32_t* in, int32_t* out, int64_t n, int32_t* sums, bool inclusive,
         cudaStream_t s) {
  if (n <= 0) return VTNK_OK;
  const int64_t nb = (n + SCAN_TILE - 1) / SCAN_TILE;
  scan_reduce<<<static_cast<unsigned>(nb), SCAN_THREADS, 0, s>>>(in, n, sums);
  scan_sums<<<1, SCAN_THREADS, 0, s>>>(sums, nb);
  scan_apply<<<static_cast<unsigned>(nb), SCAN_THREADS, 0, s>>>(in, out, n, sums,
                                                                 inclusive ? 1 : 0);
  return cuda_status(cudaGetLastError(), "trie scan");
}

// ------------------------------------------------------------------ pack
// keys[i] = tokens of item i, level 0 in the most significant field.  A token
// outside [0, vocab) sets err[0].
__global__ void pack_kernel(const int64_t* __restrict__ sem, int64_t n, int L, int b, int64_t vocab,
                            uint64_t* __restrict__ keys, unsigned long long* err) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    uint64_t k = 0;
    bool bad = false;
    for (int d = 0; d < L; ++d) {
      const int64_t t = sem[i * L + d];
      bad |= t < 0 || t >= vocab;
      k = (k << b) | (static_cast<uint64_t>(t) & ((1ull << b) - 1));
    }
    keys[i] = k;
    if (bad) atomicOr(err, 1ull);
  }
}

// ------------------------------------------------------------------ radix sort
__global__ void __launch_bounds__(RS_THREADS) rs_hist(const uint64_t* __restrict__ keys, int64_t n,
                                                      int shift, int32_t* __restrict__ counts,
                                                      int64_t nblk) {
  __shared__ int32_t h[RADIX];
  h[threadIdx.x] = 0;
  __syncthreads();
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * RS_TILE;
  for (int j = threadIdx.x; j < RS_TILE; j += RS_THREADS) {
    const int64_t i = t0 + j;
    if (i < n) atomicAdd(&h[(keys[i] >> shift) & 0xFF], 1);
  }
  __syncthreads();
  counts[static_cast<int64_t>(threadIdx.x) * nblk + blockIdx.x] = h[threadIdx.x];
}

// Stable scatter of one 2048-key tile: warp w owns keys [w*256, w*256+256) of
// the tile, 32 at a time in order; a key's place is the digit's global offset
// for this block + the keys of that digit in earlier warps + the earlier keys
// of that digit in its own warp.
__global__ void __launch_bounds__(RS_THREADS) rs_scatter(const uint64_t* __restrict__ in,
                                                         uint64_t* __restrict__ out, int64_t n,
                                                         int shift,
                                                         const int32_t* __restrict__ offs,
                                                         int64_t nblk) {
  __shared__ int32_t cnt[RS_WARPS][RADIX];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int w = 0; w < RS_WARPS; ++w) cnt[w][threadIdx.x] = 0;
  __syncthreads();
  const int64_t base = static_cast<int64_t>(blockIdx.x) * RS_TILE + warp * RS_PER_WARP;
  const uint32_t lt = (1u << lane) - 1u;
  uint64_t kv[RS_PER_WARP / 32];
  int dg[RS_PER_WARP / 32];
#pragma unroll
  for (int c = 0; c < RS_PER_WARP / 32; ++c) {
    const int64_t i = base + c * 32 + lane;
    kv[c] = i < n ? in[i] : 0;
    dg[c] = i < n ? static_cast<int>((kv[c] >> shift) & 0xFF) : RADIX;  // RADIX: no key
    const uint32_t peers = __match_any_sync(0xffffffffu, dg[c]);
    if (dg[c] < RADIX && (peers & lt) == 0) cnt[warp][dg[c]] += __popc(peers);
    __syncwarp();
  }
  __syncthreads();
  {  // per digit: exclusive prefix over the warps
    int32_t acc = 0;
    for (int w = 0; w < RS_WARPS; ++w) {
      const int32_t c = cnt[w][threadIdx.x];
      cnt[w][threadIdx.x] = acc;
      acc += c;
    }
  }
  __syncthreads();
#pragma unroll
  for (int c = 0; c < RS_PER_WARP / 32; ++c) {
    const uint32_t peers = __match_any_sync(0xffffffffu, dg[c]);
    int32_t start = 0;
    if (dg[c] < RADIX) start = cnt[warp][dg[c]];
    __syncwarp();
    if (dg[c] < RADIX) {
      const int64_t pos = static_cast<int64_t>(offs[static_cast<int64_t>(dg[c]) * nblk + blockIdx.x]) +
                          start + __popc(peers & lt);
      out[pos] = kv[c];
      if ((peers & lt) == 0) cnt[warp][dg[c]] = start + __popc(peers);
    }
    __syncwarp();
  }
}

// ------------------------------------------------------------------ structure
__device__ __forceinline__ int first_diff_level(uint64_t x, uint64_t p, int L, int b) {
  const uint64_t d = x ^ p;
  if (d == 0) return L;
  return (__clzll(static_cast<long long>(d)) - (64 - L * b)) / b;
}

__global__ void opens_kernel(const uint64_t* __restrict__ keys, int64_t n, int L, int b,
                             int32_t* __restrict__ opens) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int fd = i == 0 ? 0 : first_diff_level(keys[i], keys[i - 1], L, b);
    for (int d = 0; d < L; ++d) opens[d * n + i] = d >= fd ? 1 : 0;
  }
}

// counts[0] = n_nodes, counts[1] = nnz, counts[2 + d] = nodes opened at depth d
// (meta keeps the same values for the fill phase), counts[0] = -1 when a
// token was out of range.
__global__ void counts_kernel(const int32_t* __restrict__ node_of, int64_t n, int L,
                              const unsigned long long* err, int64_t* counts, int64_t* meta) {
  if (threadIdx.x != 0) return;
  int64_t prev = 0;
  for (int d = 0; d < L; ++d) {
    const int64_t last = n > 0 ? node_of[d * n + n - 1] : 0;
    counts[2 + d] = last - prev;
    meta[2 + d] = last - prev;
    prev = last;
  }
  counts[0] = *err ? -1 : prev + 1;
  counts[1] = prev;
  meta[0] = prev + 1;
  meta[1] = prev;
}

__global__ void fill_kernel(const uint64_t* __restrict__ keys, const int32_t* __restrict__ node_of,
                            int64_t n, int L, int b, int64_t nnz, int64_t* __restrict__ row_ptrs,
                            int64_t* __restrict__ cols, int64_t* __restrict__ vals) {
  const int64_t total = n * L;
  const uint64_t mask = (1ull << b) - 1;
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    row_ptrs[0] = 0;  // the root's first child is edge 0 (also for an empty catalog)
    cols[nnz] = -1;   // sentinel column
    vals[nnz] = -1;
  }
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int d = static_cast<int>(t / n);
    const int64_t i = t - static_cast<int64_t>(d) * n;
    const int32_t v = node_of[t];
    if (i > 0 && node_of[t - 1] == v) continue;  // no node opens here
    const int64_t e = v - 1;
    cols[e] = static_cast<int64_t>((keys[i] >> (b * (L - 1 - d))) & mask);
    vals[e] = v;
    if (d > 0) {
      const int64_t pt = t - n;  // (depth d-1, item i)
      if (i == 0 || node_of[pt - 1] != node_of[pt]) row_ptrs[node_of[pt]] = e;
    }
    if (d == L - 1) row_ptrs[v] = nnz;  // leaf
  }
}

// Child count of every internal node (root and depths 0..L-2), max per depth.
__global__ void branches_kernel(const int64_t* __restrict__ row_ptrs, const int64_t* __restrict__ meta,
                                int L, unsigned long long* __restrict__ lmb) {
  int64_t hi[16];  // last node id of each depth
  int64_t acc = 0;
  for (int d = 0; d < L; ++d) {
    acc += meta[2 + d];
    hi[d] = acc;
  }
  const int64_t n_internal = L >= 2 ? hi[L - 2] + 1 : 1;
  for (int64_t v = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; v < n_internal;
       v += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t c = row_ptrs[v + 1 < meta[0] ? v + 1 : v] - row_ptrs[v];
    int depth = 0;  // depth of v's children
    while (depth < L - 1 && v > (depth == 0 ? 0 : hi[depth - 1])) ++depth;
    if (v == 0) depth = 0;
    atomicMax(&lmb[depth], static_cast<unsigned long long>(c > 0 ? c : 0));
  }
}

struct DenseOut {
  uint8_t* mask[4];
  int64_t* states;
};

__global__ void dense_kernel(const uint64_t* __restrict__ keys, const int32_t* __restrict__ node_of,
                             int64_t n, int L, int b, int dl, int64_t vocab, DenseOut o) {
  const uint64_t m = (1ull << b) - 1;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int64_t flat = 0;
    for (int d = 0; d < dl; ++d) {
      flat = flat * vocab + static_cast<int64_t>((keys[i] >> (b * (L - 1 - d))) & m);
      o.mask[d][flat] = 1;
    }
    o.states[flat] = node_of[static_cast<int64_t>(dl - 1) * n + i];
  }
}

struct Layout {
  size_t keys_a, keys_b, counts, opens, sums, meta, err, total;
  int64_t nblk;
};

size_t a256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

Layout layout(int64_t n, int64_t L) {
  Layout ly{};
  ly.nblk = (n + RS_TILE - 1) / RS_TILE;
  const int64_t ncount = RADIX * (ly.nblk > 0 ? ly.nblk : 1);
  const int64_t scan_max = ncount > n * L ? ncount : n * L;
  size_t off = 0;
  auto take = [&](size_t b) {
    const size_t o = off;
    off += a256(b > 0 ? b : 1);
    return o;
  };
  ly.keys_a = take(n * 8);
  ly.keys_b = take(n * 8);
  ly.counts = take(ncount * 4);
  ly.opens = take(n * L * 4);
  ly.sums = take(((scan_max + SCAN_TILE - 1) / SCAN_TILE + 1) * 4);
  ly.meta = take(32 * 8);
  ly.err = take(8);
  ly.total = off;
  return ly;
}

int bits_for(int64_t vocab) {
  int b = 1;
  while ((int64_t(1) << b) < vocab) ++b;
  return b;
}

int grid_for(int64_t n, int threads) {
  int64_t g = (n + threads - 1) / threads;
  if (g > 148 * 16) g = 148 * 16;
  return static_cast<int>(g < 1 ? 1 : g);
}

}  // namespace trie
}  // namespace vtnk

using namespace vtnk;
using namespace vtnk::trie;

extern "C" {

size_t vtnk_trie_workspace_bytes(int64_t n_items, int64_t levels) {
  if (n_items < 0 || levels < 1) return 0;
  return layout(n_items, levels).total;
}

int vtnk_trie_count(const int64_t* sem_ids, int64_t n_items, int64_t levels, int64_t vocab,
                    int assume_sorted, void* workspace, size_t workspace_bytes, int64_t* counts,
                    void* stream) {
  VTNK_REQUIRE(n_items >= 0 && levels >= 1 && levels <= 16 && vocab >= 1, "bad trie sizes");
  const int b = bits_for(vocab);
  VTNK_REQUIRE(b * levels <= 64 && b <= 62,
               "levels x token bits (%lld x %d) exceed a 64-bit key", (long long)levels, b);
  VTNK_REQUIRE(n_items * levels < (int64_t(1) << 31) - 2, "catalog too large for 32-bit node ids");
  const Layout ly = layout(n_items, levels);
  VTNK_REQUIRE(workspace && workspace_bytes >= ly.total, "trie workspace too small (%zu < %zu)",
               workspace_bytes, ly.total);
  VTNK_REQUIRE(counts && (n_items == 0 || sem_ids), "NULL pointer");
  cudaStream_t s = as_stream(stream);
  char* ws = static_cast<char*>(workspace);
  uint64_t* ka = reinterpret_cast<uint64_t*>(ws + ly.keys_a);
  uint64_t* kb = reinterpret_cast<uint64_t*>(ws + ly.keys_b);
  int32_t* cnt = reinterpret_cast<int32_t*>(ws + ly.counts);
  int32_t* opens = reinterpret_cast<int32_t*>(ws + ly.opens);
  int32_t* sums = reinterpret_cast<int32_t*>(ws + ly.sums);
  int64_t* meta = reinterpret_cast<int64_t*>(ws + ly.meta);
  unsigned long long* err = reinterpret_cast<unsigned long long*>(ws + ly.err);
  cudaError_t e = cudaMemsetAsync(err, 0, 8, s);
  if (e != cudaSuccess) return cuda_status(e, "trie error word");
  const int L = static_cast<int>(levels);
  if (n_items > 0) {
    pack_kernel<<<grid_for(n_items, 256), 256, 0, s>>>(sem_ids, n_items, L, b, vocab, ka, err);
    if (!assume_sorted) {
      const int key_bits = b * L;
      for (int shift = 0; shift < key_bits; shift += 8) {
        rs_hist<<<static_cast<unsigned>(ly.nblk), RS_THREADS, 0, s>>>(ka, n_items, shift, cnt,
                                                                      ly.nblk);
        int rc = scan(cnt, cnt, RADIX * ly.nblk, sums, false, s);
        if (rc) return rc;
        rs_scatter<<<static_cast<unsigned>(ly.nblk), RS_THREADS, 0, s>>>(ka, kb, n_items, shift,
                                                                         cnt, ly.nblk);
        uint64_t* t = ka;
        ka = kb;
        kb = t;
      }
      if (ka != reinterpret_cast<uint64_t*>(ws + ly.keys_a)) {  // odd pass count
        e = cudaMemcpyAsync(ws + ly.keys_a, ka, n_items * 8, cudaMemcpyDeviceToDevice, s);
        if (e != cudaSuccess) return cuda_status(e, "trie key copy");
      }
    }
    opens_kernel<<<grid_for(n_items, 256), 256, 0, s>>>(
        reinterpret_cast<uint64_t*>(ws + ly.keys_a), n_items, L, b, opens);
    int rc = scan(opens, opens, n_items * L, sums, true, s);
    if (rc) return rc;
  }
  counts_kernel<<<1, 32, 0, s>>>(opens, n_items, L, err, counts, meta);
  return cuda_status(cudaGetLastError(), "trie count");
}

int vtnk_trie_fill(int64_t n_items, int64_t levels, int64_t vocab, int64_t dense_layers,
                   void* workspace, size_t workspace_bytes, int64_t n_nodes, int64_t nnz,
                   int64_t* row_ptrs, int64_t* cols_vals, int64_t* layer_max_branches,
                   uint8_t* const* dense_masks, int64_t* dense_states, void* stream) {
  VTNK_REQUIRE(n_items >= 0 && levels >= 1 && levels <= 16 && vocab >= 1, "bad trie sizes");
  VTNK_REQUIRE(dense_layers >= 0 && dense_layers <= 4 && dense_layers <= levels,
               "dense_lookup_layers must be in [0, min(4, levels)]");
  VTNK_REQUIRE(n_nodes == nnz + 1 && nnz >= 0, "n_nodes must be nnz + 1");
  const Layout ly = layout(n_items, levels);
  VTNK_REQUIRE(workspace && workspace_bytes >= ly.total, "trie workspace too small");
  VTNK_REQUIRE(row_ptrs && cols_vals && layer_max_branches, "NULL output");
  VTNK_REQUIRE(dense_layers == 0 || (dense_masks && dense_states), "NULL dense output");
  cudaStream_t s = as_stream(stream);
  char* ws = static_cast<char*>(workspace);
  const uint64_t* keys = reinterpret_cast<const uint64_t*>(ws + ly.keys_a);
  const int32_t* node_of = reinterpret_cast<const int32_t*>(ws + ly.opens);
  const int64_t* meta = reinterpret_cast<const int64_t*>(ws + ly.meta);
  const int L = static_cast<int>(levels);
  const int b = bits_for(vocab);
  int64_t* cols = cols_vals;
  int64_t* vals = cols_vals + nnz + 1;
  fill_kernel<<<grid_for(n_items * L, 256), 256, 0, s>>>(keys, node_of, n_items, L, b, nnz,
                                                          row_ptrs, cols, vals);
  cudaError_t e = cudaMemsetAsync(layer_max_branches, 0, L * sizeof(int64_t), s);
  if (e != cudaSuccess) return cuda_status(e, "trie branch maxima");
  branches_kernel<<<grid_for(n_nodes, 256), 256, 0, s>>>(
      row_ptrs, meta, L, reinterpret_cast<unsigned long long*>(layer_max_branches));
  if (dense_layers > 0) {
    DenseOut o{};
    int64_t sz = 1;
    for (int d = 0; d < dense_layers; ++d) {
      sz *= vocab;
      o.mask[d] = dense_masks[d];
      e = cudaMemsetAsync(o.mask[d], 0, sz, s);
      if (e != cudaSuccess) return cuda_status(e, "trie dense mask");
    }
    o.states = dense_states;
    e = cudaMemsetAsync(dense_states, 0, sz * sizeof(int64_t), s);
    if (e != cudaSuccess) return cuda_status(e, "trie dense states");
    if (n_items > 0)
      dense_kernel<<<grid_for(n_items, 256), 256, 0, s>>>(keys, node_of, n_items, L, b,
                                                          static_cast<int>(dense_layers), vocab, o);
  }
  return cuda_status(cudaGetLastError(), "trie fill");
}

}  // extern "C"
