// Result all-gather over peer memory (NVLink / NVSwitch), for the batch-
// sharded search: every rank pushes its packed result record into the
// gather buffer of every rank, then the ranks meet at a flag barrier.
// Each gather buffer holds two halves of `world` records; push number e
// (counted from 1) fills half (e & 1), so the result of a push stays intact
// until the same rank's push after next.
//
// Record layout of one rank (n beams, L levels), 16-byte aligned regions:
//   ids  int32 [n, L] | node int32 [n] | logp f32 [n]
// The push kernel reads the search's int64 / fp32 outputs, narrows token and
// node ids to int32 (checked: a value outside int32 sets the status word) and
// stores each 16-byte group to the rank's slot in all `world` buffers (peer
// pointers opened through CUDA IPC).  The last block to finish releases a
// flag in every rank's flag array and waits -- bounded in time -- until all
// ranks' flags for this epoch have arrived.  The epoch lives in device
// memory, so a captured graph replays correctly.
//
// No multicast and no TMA: plain 16-byte stores and flag loads/stores with
// system-scope release / acquire.
#include <cstdint>
#include <cstring>

#include <cuda.h>
#include <cudaTypedefs.h>

#include "vtnk_common.cuh"
#include "vtnk_internal.h"

namespace vtnk {
namespace peer {

constexpr int MAX_WORLD = 8;

struct Args {
  int world, rank;
  int64_t n, L;
  int64_t record_bytes;
  int64_t off_node, off_logp;  // byte offsets of the regions inside a record
  char* records[MAX_WORLD];     // every rank's gather buffer (this rank's own is local)
  uint32_t* flags[MAX_WORLD];   // every rank's flag array [MAX_WORLD]
  uint32_t* epoch;              // this rank's epoch and block ticket (2 words, local)
  int* status;                  // this rank's status word (local)
  const int64_t* ids;
  const int64_t* node;
  const float* logp;
  uint64_t wait_ns;
};

__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ int32_t narrow(int64_t v, int* bad) {
  if (v < INT32_MIN || v > INT32_MAX) *bad = 1;
  return static_cast<int32_t>(v);
}

// Copies groups of 4 elements of one region to every rank's slot.
__global__ void __launch_bounds__(256) push_kernel(Args a) {
  const uint32_t e = a.epoch[0] + 1;  // this push's epoch (incremented by the last block)
  int bad = 0;
  const int64_t n_ids = a.n * a.L;
  const int64_t g_ids = (n_ids + 3) / 4, g_n = (a.n + 3) / 4;
  const int64_t total = g_ids + 2 * g_n;
  for (int64_t g = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; g < total;
       g += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int4 v;
    int64_t off;
    if (g < g_ids) {
      const int64_t i = 4 * g;
      int32_t x[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) x[j] = i + j < n_ids ? narrow(a.ids[i + j], &bad) : 0;
      v = make_int4(x[0], x[1], x[2], x[3]);
      off = i * 4;
    } else if (g < g_ids + g_n) {
      const int64_t i = 4 * (g - g_ids);
      int32_t x[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) x[j] = i + j < a.n ? narrow(a.node[i + j], &bad) : 0;
      v = make_int4(x[0], x[1], x[2], x[3]);
      off = a.off_node + i * 4;
    } else {
      const int64_t i = 4 * (g - g_ids - g_n);
      float x[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) x[j] = i + j < a.n ? a.logp[i + j] : 0.f;
      v = make_int4(__float_as_int(x[0]), __float_as_int(x[1]), __float_as_int(x[2]),
                    __float_as_int(x[3]));
      off = a.off_logp + i * 4;
    }
    // two halves by epoch parity: a peer's next push never overwrites the
    // gather a slower rank may still be reading
    const int64_t slot = (static_cast<int64_t>(e & 1u) * a.world + a.rank) * a.record_bytes + off;
    for (int r = 0; r < a.world; ++r) {
      const int rr = (a.rank + r) % a.world;  // spread the peers' links
      *reinterpret_cast<int4*>(a.records[rr] + slot) = v;
    }
  }
  if (bad) atomicCAS(a.status, 0, 2);
  // the last block releases this rank's flag everywhere and waits for all
  __threadfence_system();
  __syncthreads();
  __shared__ bool last;
  if (threadIdx.x == 0) last = atomicAdd(&a.epoch[1], 1u) == gridDim.x - 1;
  __syncthreads();
  if (!last) return;
  __threadfence_system();  // every block's stores (fenced before its ticket) precede the flags
  if (threadIdx.x < a.world) st_release_sys(a.flags[threadIdx.x] + a.rank, e);
  if (threadIdx.x < a.world) {
    const uint32_t* f = a.flags[a.rank] + threadIdx.x;
    const uint64_t t0 = now_ns();
    while (static_cast<int32_t>(ld_acquire_sys(f) - e) < 0) {
      if (now_ns() - t0 > a.wait_ns) {
        atomicCAS(a.status, 0, 1);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    a.epoch[1] = 0;
    a.epoch[0] = e;
  }
}

}  // namespace peer
}  // namespace vtnk

using namespace vtnk;

extern "C" {

int vtnk_ipc_handle_bytes(void) { return static_cast<int>(sizeof(cudaIpcMemHandle_t)); }

int vtnk_ipc_get_handle(const void* dev_ptr, void* handle_out, int64_t* offset_out) {
  VTNK_REQUIRE(dev_ptr && handle_out && offset_out, "NULL pointer");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(dev_ptr));
  if (e != cudaSuccess) return cuda_status(e, "cudaIpcGetMemHandle");
  // the handle names the whole allocation; the opener adds the offset
  static PFN_cuMemGetAddressRange_v3020 range_fn = nullptr;
  if (!range_fn) {
    cudaDriverEntryPointQueryResult q;
    void* f = nullptr;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      set_error("cuMemGetAddressRange unavailable");
      return VTNK_ERR_CUDA;
    }
    range_fn = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(f);
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range_fn(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS) {
    set_error("cuMemGetAddressRange failed");
    return VTNK_ERR_CUDA;
  }
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = static_cast<int64_t>(reinterpret_cast<CUdeviceptr>(dev_ptr) - base);
  return VTNK_OK;
}

int vtnk_ipc_open_handle(const void* handle, void** dev_ptr_out) {
  VTNK_REQUIRE(handle && dev_ptr_out, "NULL pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(dev_ptr_out, h, cudaIpcMemLazyEnablePeerAccess);
  return cuda_status(e, "cudaIpcOpenMemHandle");
}

int vtnk_ipc_close_handle(void* dev_ptr) {
  return cuda_status(cudaIpcCloseMemHandle(dev_ptr), "cudaIpcCloseMemHandle");
}

int vtnk_peer_gather(const vtnk_peer_group_t* g, const int64_t* ids, const float* logp,
                     const int64_t* node, int64_t n, int64_t levels, void* stream) {
  VTNK_REQUIRE(g != nullptr, "peer group is NULL");
  VTNK_REQUIRE(g->world >= 1 && g->world <= peer::MAX_WORLD && g->rank >= 0 &&
                   g->rank < g->world,
               "bad world / rank (world <= %d)", peer::MAX_WORLD);
  VTNK_REQUIRE(n >= 0 && levels >= 1, "bad record shape");
  const int64_t need = vtnk_peer_record_bytes(n, levels);
  VTNK_REQUIRE(g->record_bytes >= need, "record_bytes %lld < %lld", (long long)g->record_bytes,
               (long long)need);
  VTNK_REQUIRE(g->epoch && g->status, "NULL epoch / status");
  VTNK_REQUIRE(g->record_bytes % 16 == 0, "record_bytes must be a multiple of 16");
  for (int r = 0; r < g->world; ++r)
    VTNK_REQUIRE(g->records[r] && g->flags[r], "NULL peer pointer %d", r);
  VTNK_REQUIRE(n == 0 || (ids && logp && node), "NULL input");
  peer::Args a{};
  a.world = g->world;
  a.rank = g->rank;
  a.n = n;
  a.L = levels;
  a.record_bytes = g->record_bytes;
  a.off_node = ((n * levels * 4 + 15) / 16) * 16;
  a.off_logp = a.off_node + ((n * 4 + 15) / 16) * 16;
  for (int r = 0; r < g->world; ++r) {
    a.records[r] = static_cast<char*>(g->records[r]);
    a.flags[r] = g->flags[r];
  }
  a.epoch = g->epoch;
  a.status = g->status;
  a.ids = ids;
  a.node = node;
  a.logp = logp;
  a.wait_ns = g->wait_ns ? g->wait_ns : 2000000000ull;
  const int64_t groups = (n * levels + 3) / 4 + 2 * ((n + 3) / 4);
  int64_t blocks = (groups + 255) / 256;
  if (blocks > 148 * 4) blocks = 148 * 4;
  if (blocks < 1) blocks = 1;
  peer::push_kernel<<<static_cast<unsigned>(blocks), 256, 0, as_stream(stream)>>>(a);
  return cuda_status(cudaGetLastError(), "peer gather launch");
}

int64_t vtnk_peer_record_bytes(int64_t n, int64_t levels) {
  if (n < 0 || levels < 1) return 0;
  return ((n * levels * 4 + 15) / 16) * 16 + 2 * (((n * 4) + 15) / 16) * 16;
}

}  // extern "C"
