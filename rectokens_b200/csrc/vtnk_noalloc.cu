// Allocation-free variant of vtnk_beam_search.
//
// Some callers cannot call cudaMalloc or any allocating routine on the decode
// path: a plugin inside an inference server whose device memory is owned by
// the host process's own pool, code that must not trigger the implicit device
// synchronisation an allocation can cause, or an embedder with a fixed memory
// budget.  They still pass every input and output buffer, but the search's
// scratch (per-level candidate tables and the beam histories) comes from one
// fixed array compiled into this library instead of a caller workspace.
//
// The array is a file-scope __device__ variable: every GPU that loads the
// library holds VTNK_NOALLOC_SCRATCH_BYTES of it until the process exits.
// Host code only sees a stand-in for its name, so the device address is
// looked up with cudaGetSymbolAddress once per device (with that device
// current) on the first call made on it.
#include <mutex>

#include "vtnk_common.cuh"
#include "vtnk_internal.h"

namespace vtnk {
namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[VTNK_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_addr[kMaxDevices] = {};

// Device address of the scratch array on the current device (looked up once).
int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) {
    set_error("device ordinal %d out of range for the scratch table", dev);
    return VTNK_ERR_UNSUPPORTED;
  }
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_status(e, "cudaGetSymbolAddress(scratch)");
    g_addr[dev] = p;
  }
  *out = g_addr[dev];
  return VTNK_OK;
}

}  // namespace
}  // namespace vtnk

extern "C" int vtnk_beam_search_noalloc(const vtnk_search_t* s, int64_t* out_ids,
                                        float* out_logp, int64_t* out_node, void* stream) {
  using namespace vtnk;
  VTNK_REQUIRE(s != nullptr, "search is NULL");
  const size_t need = vtnk_beam_search_workspace_bytes(s);
  if (need > static_cast<size_t>(VTNK_NOALLOC_SCRATCH_BYTES)) {
    set_error(
        "vtnk_beam_search_noalloc: this search needs %zu bytes of scratch, more than the "
        "built-in %zu-byte array; use vtnk_beam_search with a caller workspace",
        need, static_cast<size_t>(VTNK_NOALLOC_SCRATCH_BYTES));
    return VTNK_ERR_UNSUPPORTED;
  }
  void* scratch = nullptr;
  const int rc = scratch_address(&scratch);
  if (rc) return rc;
  // Every scratch byte the search reads is written earlier in the same call,
  // so nothing needs clearing between calls.
  // Whole-tile scheduling only: stream-K would allocate the library's
  // workspace on first use.
  return beam_search_run(s, scratch, VTNK_NOALLOC_SCRATCH_BYTES, out_ids, out_logp, out_node,
                         stream, false);
}
