// Tensor-memory-accelerator (TMA) descriptors: host-side encoding through the driver entry
// point (no link-time dependency on libcuda) and the 2-D tiled load used by the kernels.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace memt {

// 2-D bf16 tensor map over rows of `inner` elements, `row_stride` bytes apart, boxes of
// box_inner x box_rows elements with the 128-byte swizzle (box_inner * 2 must be 128) and
// zero fill outside the tensor. Returns cudaSuccess or the failing error.
cudaError_t make_tmap_bf16_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows,
                              uint64_t row_stride, uint32_t box_inner, uint32_t box_rows);

#ifdef __CUDACC__
// Load the box at (x elements, y rows) into shared memory (1024-byte aligned for the
// 128-byte swizzle); completion is signalled on the mbarrier as transaction bytes.
// x * 2 bytes must be a multiple of 16; y may lie outside the tensor (zero fill).
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t mbar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(mbar)
      : "memory");
}
// Store the shared-memory box at smem address src to (x, y) of the tensor (bulk group of this
// thread; rows outside the tensor are not written). x * 2 bytes must be a multiple of 16.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, int x, int y, uint32_t src) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];\n" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(x), "r"(y), "r"(src)
      : "memory");
}
#endif

}  // namespace memt
