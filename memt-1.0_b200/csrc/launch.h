// Internal launchers, one translation unit per kernel family (built in parallel).
#pragma once

#include <cuda_runtime.h>

#include <map>
#include <mutex>
#include <set>
#include <utility>

#include "common.cuh"
#include "memt_gdn2.h"

namespace memt {

// Maps a CUDA error to MEMT_ERR_CUDA and records it for memt_last_cuda_error().
int cuda_status(cudaError_t e);

// Opt a kernel into large dynamic shared memory once per (kernel, device).
template <typename Kernel>
cudaError_t ensure_smem(Kernel kernel, size_t bytes) {
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  auto key = std::make_pair(reinterpret_cast<const void*>(kernel), dev);
  if (done.count(key)) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
  // the whole unified L1 as shared memory, so that two large-tile CTAs fit on one SM
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
  if (e == cudaSuccess) done.insert(key);
  return e;
}

// Optional per-launch CUDA-event timing (memt_profiler_*). Usage around a launch:
//   ProfScope prof(kProfIntra, stream);  kernel<<<...>>>(...);
enum ProfFamily { kProfPlan = 0, kProfIntra, kProfScan, kProfReadGemv, kProfReadTile, kProfRecurrent, kProfPrologue };
void prof_begin(int family, cudaStream_t s, void** token);
void prof_end(void* token, cudaStream_t s);
struct ProfScope {
  void* token = nullptr;
  cudaStream_t s;
  ProfScope(int family, cudaStream_t stream) : s(stream) { prof_begin(family, stream, &token); }
  ~ProfScope() { prof_end(token, s); }
};

// CTAs of this kernel that fit on the device at once (SM count x occupancy), cached per
// (kernel, device).
template <typename Kernel>
cudaError_t resident_slots(Kernel kernel, int threads, size_t smem, int* slots) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, int> cache;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  auto key = std::make_pair(reinterpret_cast<const void*>(kernel), dev);
  auto it = cache.find(key);
  if (it != cache.end()) {
    *slots = it->second;
    return cudaSuccess;
  }
  int sms = 0, per_sm = 0;
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem);
  if (e != cudaSuccess) return e;
  *slots = sms * (per_sm > 0 ? per_sm : 1);
  cache[key] = *slots;
  return cudaSuccess;
}

// Launch with programmatic stream serialization (the kernel calls griddep_wait() before it
// reads anything earlier work produces).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

int launch_plan(const int32_t* cu, int32_t N, int64_t L, int32_t chunk_tokens, int32_t max_chunks,
                WsHeader* hdr, ChunkDesc* table, int32_t* sample_off, cudaStream_t s);
int launch_intra(int D, bool erase, const IntraParams& p, int64_t max_chunks, cudaStream_t s);
int launch_scan(int D, const ScanParams& p, cudaStream_t s);
int launch_recurrent(int D, const RecurrentParams& p, cudaStream_t s);
// exact: fp32 query and state (no bf16 rounding); maxlen: bound on tokens per block
// Where a read runs. kReadAlone: on its own. kReadBeside: on the caller's stream beside the
// commit's scan (short CTAs, which the scan's SMs are not held by). kReadAfterScan: on the
// scan's stream right after it, by programmatic dependent launch, so that its CTAs are placed
// only once every scan CTA is resident; it never waits for the scan (it reads nothing the scan
// writes). Only the tcgen05 tile read takes kReadAfterScan (read_uses_tc).
enum ReadPlacement { kReadAlone = 0, kReadBeside = 1, kReadAfterScan = 2 };
bool read_uses_tc(const ReadParams& p, int D, bool exact, int64_t maxlen);
int launch_read(const ReadParams& p, int D, bool exact, int64_t maxlen, cudaStream_t s, int placement = kReadAlone);

}  // namespace memt
