// memt_gdn2_update_noalloc: the update with its scratch in a static device array, for callers
// that cannot allocate device memory when they call (see include/memt_gdn2.h).
#include <cuda_runtime.h>

#include <mutex>

#include "launch.h"
#include "memt_gdn2.h"

namespace {

// One copy per device on which this module is loaded (at the latest by the first call of the
// entry point there); it lives until the process exits.
static __device__ __align__(256) unsigned char g_noalloc_scratch[MEMT_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device, looked up once per device.
// The array's host-side name is only a stand-in; kernels must be given this address.
int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return memt::cuda_status(e);
  if (dev < 0 || dev >= kMaxDevices) return MEMT_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return memt::cuda_status(e);
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return MEMT_OK;
}

}  // namespace

extern "C" int memt_gdn2_update_noalloc(const memt_gdn2_update_args* args, memt_stream_t stream) {
  if (args == nullptr || args->struct_size != sizeof(memt_gdn2_update_args)) return MEMT_ERR_INVALID_ARGUMENT;
  const size_t need = memt_gdn2_update_workspace_size(args->num_samples, args->total_tokens, args->num_heads,
                                                      args->key_dim, args->value_dim, args->chunk_tokens,
                                                      args->dtype);
  if (need > MEMT_NOALLOC_SCRATCH_BYTES) return MEMT_ERR_WORKSPACE;  // too large for the static scratch
  void* scratch = nullptr;
  const int st = scratch_address(&scratch);
  if (st != MEMT_OK) return st;
  // Same kernels and argument checks as the allocating entry point.
  return memt_gdn2_update(args, scratch, MEMT_NOALLOC_SCRATCH_BYTES, stream);
}

// The status word the last memt_gdn2_update_noalloc on this device left at the start of the
// static scratch; the same word memt_gdn2_workspace_status reads from a caller's workspace.
extern "C" int memt_gdn2_noalloc_status(memt_stream_t stream, int32_t* status_out) {
  if (status_out == nullptr) return MEMT_ERR_INVALID_ARGUMENT;
  void* scratch = nullptr;
  const int st = scratch_address(&scratch);
  if (st != MEMT_OK) return st;
  return memt_gdn2_workspace_status(scratch, stream, status_out);
}
