// Launcher for the device-side varlen plan (plan.cuh).
#include "launch.h"
#include "plan.cuh"

namespace memt {

int launch_plan(const int32_t* cu, int32_t N, int64_t L, int32_t chunk_tokens, int32_t max_chunks,
                WsHeader* hdr, ChunkDesc* table, int32_t* sample_off, cudaStream_t s) {
  ProfScope prof(kProfPlan, s);
  plan_kernel<<<1, 1024, 0, s>>>(cu, N, L, chunk_tokens, max_chunks, hdr, table, sample_off);
  return cuda_status(cudaGetLastError());
}

}  // namespace memt
