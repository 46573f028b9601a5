// Exact fp32 GDN-2 update (the fp32 mode of memt_gdn2_update).
//
// Token-by-token gated delta rule on CUDA cores, no tensor-core rounding:
//     S~ = diag(exp g_t) S ;  d = w_t*v_t - S~^T (b_t*k'_t) ;  S = S~ + k'_t d^T
// with k'_t = sqrt(beta_t) k_t. This is the mathematical definition the chunked WY
// algorithm reorganises (the reference's kernels compute it in 64-token chunks; in
// fp32 they agree with this recurrence to rounding). One CTA per (sample, head,
// 32-wide value slice); the slice of S lives in registers, 4 row groups x 32 columns.
#pragma once

#include "common.cuh"

namespace memt {

template <int D>
__global__ void __launch_bounds__(128) recurrent_kernel(RecurrentParams p) {
  constexpr int RG = 4;          // row groups
  constexpr int RPG = D / RG;    // rows per group
  __shared__ float s_k[D], s_kb[D], s_a[D];
  __shared__ float s_red[RG][32];
  const int tid = threadIdx.x, col = tid & 31, grp = tid >> 5;
  constexpr int NV = D / 32;
  const int vp = blockIdx.x % NV, nh = blockIdx.x / NV;
  const int h = nh % p.H, n = nh / p.H;
  const int v = vp * 32 + col;
  int64_t bos = p.cu[n], eos = p.cu[n + 1];
  bos = bos < 0 ? 0 : (bos > p.L ? p.L : bos);
  eos = eos < bos ? bos : (eos > p.L ? p.L : eos);
  const int64_t in_slot = pool_slot(p.slots_in, p.num_in, n), out_slot = pool_slot(p.slots_out, p.num_out, n);
  const int64_t in_off = (in_slot * p.H + h) * D * D, out_off = (out_slot * p.H + h) * D * D;
  float S[RPG];
#pragma unroll
  for (int i = 0; i < RPG; ++i) S[i] = in_slot >= 0 ? p.h0[in_off + (int64_t)(grp * RPG + i) * D + v] : 0.f;
  const int64_t rs = (int64_t)p.H * D;
  for (int64_t t = bos; t < eos; ++t) {
    const int64_t base = t * rs + (int64_t)h * D;
    for (int c = tid; c < D; c += 128) {
      float kk = p.k[base + c];
      if (p.beta_layout == 1) kk *= sqrtf(p.beta[t * p.H + h]);
      if (p.beta_layout == 2) kk *= sqrtf(p.beta[base + c]);
      const float gg = (p.g_layout == 2) ? p.g[base + c] : p.g[t * p.H + h];
      s_k[c] = kk;
      s_kb[c] = p.erase ? kk * p.erase[base + c] : kk;
      s_a[c] = expf(gg);
    }
    __syncthreads();
    float part = 0.f;
#pragma unroll
    for (int i = 0; i < RPG; ++i) {
      const int r = grp * RPG + i;
      S[i] *= s_a[r];
      part = fmaf(S[i], s_kb[r], part);
    }
    s_red[grp][col] = part;
    __syncthreads();
    float wv = p.v[base + v];
    if (p.write) wv *= p.write[base + v];
    float dl = wv;
#pragma unroll
    for (int r = 0; r < RG; ++r) dl -= s_red[r][col];
#pragma unroll
    for (int i = 0; i < RPG; ++i) S[i] = fmaf(s_k[grp * RPG + i], dl, S[i]);
    __syncthreads();
  }
  if (out_slot < 0) return;
#pragma unroll
  for (int i = 0; i < RPG; ++i) p.ht[out_off + (int64_t)(grp * RPG + i) * D + v] = S[i];
}

}  // namespace memt
