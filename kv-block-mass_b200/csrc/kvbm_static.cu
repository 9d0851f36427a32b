// kvbm_block_mass_static: the block-mass computation for callers that cannot
// allocate device memory.
//
// The two passes need scratch space: the per-row lse2 values and the per-key
// partial sums.  kvbm_block_mass takes that workspace from the caller.  Some
// callers have no way to provide it.  A serving engine may reserve all free
// device memory for its own KV-cache pool at start-up, so a cudaMalloc would
// fail.  Its step loop also cannot afford cudaMalloc/cudaFree, which
// synchronise the device and stall its other streams.  A C or FFI host may
// only hold the input and output pointers that another framework handed it.
// This entry point needs no allocation: its scratch lives in a fixed
// file-scope device array that every GPU using this library holds until the
// process exits.
#include <cuda_runtime.h>

#include <atomic>

#include "kvbm_internal.cuh"

namespace kvbm {
namespace {

// 64 MiB covers the whole Llama-3-8B N=32768 problem (20 MiB) and one
// (batch, kv-head) unit of the Llama-3-70B N=131072 shape (36 MiB).
constexpr size_t kStaticScratchBytes = size_t(64) << 20;

static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 64;
// Device address of g_static_scratch, looked up once per device.  In host
// code the array's name is only a host-side stand-in, not a device address.
std::atomic<void*> g_scratch_addr[kMaxDevices] = {};

}  // namespace
}  // namespace kvbm

extern "C" size_t kvbm_static_scratch_bytes(void) { return kvbm::kStaticScratchBytes; }

extern "C" int kvbm_block_mass_static(const kvbm_problem* p, void* mass_out, void* stream) {
  using namespace kvbm;
  const int st = validate(p);
  if (st != KVBM_OK) return st;
  if (mass_out == nullptr) return KVBM_ERR_NULL;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return KVBM_ERR_CUDA;
  }
  if (dev < 0 || dev >= kMaxDevices) return KVBM_ERR_DEVICE;
  // The scratch a call needs covers only the batches x kv-heads of its unit
  // range: a range inside one batch entry needs its own units' rows.
  size_t need = 0;
  int pst = planned_workspace_bytes(p, &need);
  if (pst != KVBM_OK) return pst;
  // The one-pass method's segment slots and per-tile partials take more
  // scratch than the two-pass method; the array may fit only the latter.
  kvbm_options o{};
  if (need > kStaticScratchBytes) {
    o.method = KVBM_METHOD_TWO_PASS;
    pst = planned_workspace_bytes(p, &need, &o);
    if (pst != KVBM_OK) return pst;
  }
  if (need > kStaticScratchBytes) return KVBM_ERR_SCRATCH;
  void* ptr = g_scratch_addr[dev].load(std::memory_order_acquire);
  if (ptr == nullptr) {
    // First call on this device: resolve the array's device address with
    // this device current (threads racing here store the same address).
    if (cudaGetSymbolAddress(&ptr, g_static_scratch) != cudaSuccess || ptr == nullptr) {
      cudaGetLastError();
      return KVBM_ERR_CUDA;
    }
    g_scratch_addr[dev].store(ptr, std::memory_order_release);
  }
  return kvbm_block_mass_ex(p, &o, mass_out, ptr, kStaticScratchBytes, stream);
}
