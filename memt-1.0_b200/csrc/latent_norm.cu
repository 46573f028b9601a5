// memt_latent_rms_norm: the grouped latent RMS norm of the DeepSeek memory block's low-rank
// q/k/v expansion (_latent_norm as expand_grouped_qkv applies it, models/deepseek/ops/
// compiled_tensor_ops.py:12-41 of inference/memt_sglang):
//     y[t, g, :] = bf16( (x * rsqrt(mean(x^2) + eps[g])) * weight[g, :] ),  x = fp32(x[t, g, :])
// One warp per (token, group) row: a first pass sums the squares in fp32 (16-byte loads, 8 bf16
// per lane), a second pass (the row is in L1 by then) scales and stores. HBM-bound.
#include "launch.h"

namespace {

using namespace memt;

struct LatentNormParams {
  int64_t L;
  int32_t G, R;
  const __nv_bfloat16* x;
  int64_t sx;
  const __nv_bfloat16* w;
  const float* eps;  // [G] or null
  float eps_scalar;
  __nv_bfloat16* out;
};

__global__ void __launch_bounds__(256) latent_norm_kernel(LatentNormParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t rows = p.L * p.G;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < rows; row += warps) {
    const int64_t t = row / p.G;
    const int g = (int)(row - t * p.G);
    const __nv_bfloat16* xr = p.x + t * p.sx + (int64_t)g * p.R;
    float ss = 0.f;
    for (int c = 8 * lane; c < p.R; c += 256) {
      const uint4 u = *reinterpret_cast<const uint4*>(xr + c);
      const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = unpack_bf16x2(w4[i]);
        ss = fmaf(f.x, f.x, ss);
        ss = fmaf(f.y, f.y, ss);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float eps = p.eps != nullptr ? p.eps[g] : p.eps_scalar;
    const float r = rsqrtf(ss / (float)p.R + eps);
    const __nv_bfloat16* wr = p.w + (int64_t)g * p.R;
    __nv_bfloat16* yr = p.out + row * p.R;
    for (int c = 8 * lane; c < p.R; c += 256) {
      const uint4 u = *reinterpret_cast<const uint4*>(xr + c);
      const uint4 wv = *reinterpret_cast<const uint4*>(wr + c);
      const uint32_t x4[4] = {u.x, u.y, u.z, u.w}, g4[4] = {wv.x, wv.y, wv.z, wv.w};
      uint32_t o4[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = unpack_bf16x2(x4[i]), wg = unpack_bf16x2(g4[i]);
        o4[i] = pack_bf16x2((f.x * r) * wg.x, (f.y * r) * wg.y);
      }
      *reinterpret_cast<uint4*>(yr + c) = make_uint4(o4[0], o4[1], o4[2], o4[3]);
    }
  }
}

bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

}  // namespace

extern "C" int memt_latent_rms_norm(const memt_latent_norm_args* a, memt_stream_t stream) {
  if (a == nullptr || a->struct_size != sizeof(memt_latent_norm_args)) return MEMT_ERR_INVALID_ARGUMENT;
  if (a->total_tokens < 0 || a->groups < 1 || a->rank < 8 || a->x == nullptr || a->weight == nullptr ||
      a->out == nullptr || a->x_stride < int64_t(a->groups) * a->rank)
    return MEMT_ERR_INVALID_ARGUMENT;
  if (a->rank % 8 != 0 || a->x_stride % 8 != 0 || !aligned16(a->x) || !aligned16(a->weight) || !aligned16(a->out))
    return MEMT_ERR_MISALIGNED;  // 16-byte rows
  if (a->total_tokens == 0) return MEMT_OK;
  LatentNormParams p{};
  p.L = a->total_tokens;
  p.G = a->groups;
  p.R = a->rank;
  p.x = static_cast<const __nv_bfloat16*>(a->x);
  p.sx = a->x_stride;
  p.w = static_cast<const __nv_bfloat16*>(a->weight);
  p.eps = a->eps;
  p.eps_scalar = a->eps_scalar;
  p.out = static_cast<__nv_bfloat16*>(a->out);
  int slots = 0;
  cudaError_t e = resident_slots(latent_norm_kernel, 256, 0, &slots);
  if (e != cudaSuccess) return cuda_status(e);
  const int64_t rows = p.L * p.G;
  int64_t grid = (rows + 7) / 8;
  if (grid > slots) grid = slots;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  ProfScope prof(kProfPrologue, s);
  latent_norm_kernel<<<static_cast<unsigned>(grid), 256, 0, s>>>(p);
  return cuda_status(cudaGetLastError());
}
