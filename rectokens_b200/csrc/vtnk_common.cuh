// Shared device helpers for the vtnk_b200 kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cmath>
#include <string>

#include "vtnk_b200.h"

namespace vtnk {

// ----------------------------------------------------------------- host errors
void set_error(const char* fmt, ...);
int cuda_status(cudaError_t e, const char* what);
inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

#define VTNK_REQUIRE(cond, ...)            \
  do {                                     \
    if (!(cond)) {                         \
      ::vtnk::set_error(__VA_ARGS__);      \
      return VTNK_ERR_ARG;                 \
    }                                      \
  } while (0)

// ----------------------------------------------------------------- element I/O
template <typename T> __device__ __forceinline__ float to_f32(T x);
template <> __device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) {
  return __bfloat162float(x);
}
template <> __device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }

template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}
template <> __device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }

// 16-byte vector of T unpacked to fp32.
template <typename T> struct Vec16 {
  static constexpr int N = 16 / sizeof(T);
  float v[N];
  __device__ __forceinline__ void load(const T* p) {
    const uint4 raw = __ldg(reinterpret_cast<const uint4*>(p));
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < N; ++i) v[i] = to_f32<T>(e[i]);
  }
};

// ----------------------------------------------------------------- CSR access
struct Csr {
  const int64_t* row_ptrs;
  const int64_t* cols;
  const int64_t* vals;
  int64_t n_nodes;
  int64_t nnz;
};

inline Csr make_csr(const vtnk_csr_t& c) {
  return Csr{c.row_ptrs, c.cols, c.vals, c.n_nodes, c.nnz};
}

// Child list of `cur`: first edge and the number of slots in use (capped at
// max_branches).  Out-of-range nodes have no children; the last node's end is
// nnz (the reference layout has no trailing row pointer).
__device__ __forceinline__ void node_children(const Csr& c, int64_t cur, int64_t max_branches,
                                              int64_t& start, int& count) {
  start = 0;
  count = 0;
  if (cur < 0 || cur >= c.n_nodes) return;
  int64_t s = __ldg(c.row_ptrs + cur);
  int64_t e = (cur + 1 < c.n_nodes) ? __ldg(c.row_ptrs + cur + 1) : c.nnz;
  if (s < 0) s = 0;
  if (e > c.nnz) e = c.nnz;
  int64_t n = e - s;
  if (n < 0) n = 0;
  if (n > max_branches) n = max_branches;
  start = s;
  count = static_cast<int>(n);
}

// ----------------------------------------------------------------- warp helpers
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
// (value, index) argmax over the warp: larger value wins, ties to the smaller
// index.  NaN never wins against a number.  Result in every lane.
__device__ __forceinline__ void warp_argmax(float& v, int& i) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, i, o);
    if (ov > v || (ov == v && oi < i) || (v != v && ov == ov)) {
      v = ov;
      i = oi;
    }
  }
}

// Order-preserving 32-bit key of a float (a > b  <=>  key(a) > key(b); -0
// and +0 share a key).  No NaN reaches the merges.
__device__ __forceinline__ unsigned order_key(float f) {
  const unsigned u = __float_as_uint(f + 0.0f);  // -0 -> +0
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// ----------------------------------------------------------------- Philox noise
// Philox4x32-10 (Salmon, Moraes, Dror & Shaw, SC'11), first output word, with
// the lane order and constants Triton's tl.rand uses; counter (c0, 0, 0, 0),
// key (seed_lo, seed_hi).
__device__ __forceinline__ uint32_t philox_word0(uint32_t c0, uint32_t k0, uint32_t k1) {
  uint32_t c1 = 0, c2 = 0, c3 = 0;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t a0 = c0, a2 = c2;
    c0 = __umulhi(0xCD9E8D57u, a2) ^ c1 ^ k0;
    c2 = __umulhi(0xD2511F53u, a0) ^ c3 ^ k1;
    c1 = 0xCD9E8D57u * a2;
    c3 = 0xD2511F53u * a0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return c0;
}

// The reference sampling kernel's noise at flat offset `off` (int32 wrap):
// u = uniform(philox), g = -log(-log(u + 1e-10) + 1e-10).
__device__ __forceinline__ float gumbel_at(uint64_t seed, uint32_t off) {
  const uint32_t w = philox_word0(off, static_cast<uint32_t>(seed),
                                  static_cast<uint32_t>(seed >> 32));
  int32_t x = static_cast<int32_t>(w);
  x = x < 0 ? ~x : x;
  const float u = __int2float_rn(x) * 4.6566127342e-10f;
  return -logf(-logf(u + 1e-10f) + 1e-10f);
}

// ----------------------------------------------------------------- synthetic values
__host__ __device__ __forceinline__ uint64_t mix64(uint64_t x) {
  uint64_t z = x + 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

}  // namespace vtnk
