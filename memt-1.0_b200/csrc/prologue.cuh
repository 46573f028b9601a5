// Qwen memory-block prologue: everything QwenMemoryBlock.packed computes between its input
// projection GEMMs and the GDN-2 update, in one pass over the token rows
// (models/qwen/layer.py:71-97 and the FLA l2norm, _vendor/fla/modules/l2norm.py:84-109):
//
//   q_hat      = bf16(q * 1/sqrt(sum q^2 + eps))                 l2norm(q)
//   k_hat      = bf16(k * 1/sqrt(sum k^2 + eps))                 l2norm(k)
//                (or x * rsqrt(sum x^2 + eps): the DeepSeek block's l2norm,
//                 models/deepseek/ops/normalization.py:6-8)
//   erase_sqrt = bf16(exp(0.5 * logsigmoid(e)))                  _write_gates, erase
//   k'         = bf16(erase_sqrt * k_hat)                        _symmetric_inputs
//   write      = bf16(sigmoid(w))                                _write_gates, write
//   log_decay  = -exp(decay_scale_log[h]) * softplus(d + decay_bias)   _log_decay (fp32)
//
// All arithmetic is fp32 with the reference's rounding points; e, w and d are the bf16
// pre-activations the reference splits out of its gate projection (d after f_down). The
// erase factor the update then sees is 1 (the reference passes torch.ones_like), so the
// update runs without one.
//
// Layout: one (token, head) row of D elements per D/8 lanes, 16-byte loads and stores
// (8 bf16 per lane), 32/(D/8) rows per warp, grid-stride over the L*H rows. HBM-bound:
// 5 bf16 inputs and 3 bf16 + 1 fp32 outputs per element.
#pragma once

#include "common.cuh"

namespace memt {

struct PrologueParams {
  int32_t H;
  int64_t L;
  const __nv_bfloat16 *q, *k, *erase, *write, *decay;  // token rows with the strides below
  int64_t sq, sk, se, sw, sd;                           // elements per token row
  const __nv_bfloat16* bias;                            // [H*D]
  const __nv_bfloat16* scale_log;                       // [H]
  float eps;
  int32_t rsqrt_norm;                                   // l2norm as x * rsqrt(.) instead of x / sqrt(.)
  __nv_bfloat16 *q_out, *k_out, *w_out;                 // [L, H, D]
  float* g_out;                                         // [L, H, D]
};

__device__ __forceinline__ void load_bf16x8(const __nv_bfloat16* p, float* x) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = unpack_bf16x2(w[i]);
    x[2 * i] = f.x;
    x[2 * i + 1] = f.y;
  }
}

__device__ __forceinline__ void store_bf16x8(__nv_bfloat16* p, const float* x) {
  *reinterpret_cast<uint4*>(p) = make_uint4(pack_bf16x2(x[0], x[1]), pack_bf16x2(x[2], x[3]),
                                            pack_bf16x2(x[4], x[5]), pack_bf16x2(x[6], x[7]));
}

// sum over the LPR lanes that share a row (aligned groups, so xor stays inside the group)
template <int LPR>
__device__ __forceinline__ float row_sum(float v) {
#pragma unroll
  for (int o = LPR / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <int D>
__global__ void __launch_bounds__(256) qwen_prologue_kernel(PrologueParams p) {
  constexpr int LPR = D / 8;     // lanes per row
  constexpr int RPW = 32 / LPR;  // rows per warp
  const int lane = threadIdx.x & 31;
  const int sub = lane / LPR, c0 = (lane % LPR) * 8;
  const int64_t rows = p.L * p.H;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t base = ((int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * RPW; base < rows;
       base += warps * RPW) {
    const int64_t row = base + sub;
    const bool ok = row < rows;
    const int64_t t = ok ? row / p.H : 0;
    const int h = ok ? (int)(row - t * p.H) : 0;
    const int64_t col = (int64_t)h * D + c0;
    float q[8], k[8], e[8], w[8], d[8], b[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) q[i] = k[i] = e[i] = w[i] = d[i] = b[i] = 0.f;
    float sl = 0.f;
    if (ok) {
      load_bf16x8(p.q + t * p.sq + col, q);
      load_bf16x8(p.k + t * p.sk + col, k);
      load_bf16x8(p.erase + t * p.se + col, e);
      load_bf16x8(p.write + t * p.sw + col, w);
      load_bf16x8(p.decay + t * p.sd + col, d);
      load_bf16x8(p.bias + col, b);
      sl = __bfloat162float(p.scale_log[h]);
    }
    float qq = 0.f, kk = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      qq = fmaf(q[i], q[i], qq);
      kk = fmaf(k[i], k[i], kk);
    }
    qq = row_sum<LPR>(qq);
    kk = row_sum<LPR>(kk);
    if (!ok) continue;
    const float rq = p.rsqrt_norm ? rsqrtf(qq + p.eps) : 1.f / sqrtf(qq + p.eps);
    const float rk = p.rsqrt_norm ? rsqrtf(kk + p.eps) : 1.f / sqrtf(kk + p.eps);
    const float dscale = -expf(sl);
    float qo[8], ko[8], wo[8], go[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      qo[i] = q[i] * rq;
      const float kn = bf16_round(k[i] * rk);
      // logsigmoid(x) = min(0, x) - log1p(exp(-|x|)); erase_sqrt = bf16(exp(0.5 logsigmoid(x))).
      // erase_sqrt and the write gate are stored in bf16 (8-bit significand): CUDA's fast exp and
      // log intrinsics (relative error ~1e-7 here) leave them unchanged except at rounding ties.
      // log(1 + t) for t = exp(-|x|) in (0, 1]: where 1 + t rounds to 1 the true value (< 6e-8)
      // moves erase_sqrt by less than half a bf16 unit.
      const float t = __expf(-fabsf(e[i]));
      const float ls = fminf(0.f, e[i]) - __logf(1.f + t);
      const float es = bf16_round(__expf(0.5f * ls));
      ko[i] = es * kn;
      wo[i] = __frcp_rn(1.f + __expf(-w[i]));
      // the fp32 log-decay keeps the accurate functions (the reference's own fp32 arithmetic)
      const float x = d[i] + b[i];
      const float sp = x > 20.f ? x : log1pf(expf(x));  // softplus, threshold 20
      go[i] = dscale * sp;
    }
    const int64_t o = row * D + c0;
    store_bf16x8(p.q_out + o, qo);
    store_bf16x8(p.k_out + o, ko);
    store_bf16x8(p.w_out + o, wo);
    float4* g4 = reinterpret_cast<float4*>(p.g_out + o);
    g4[0] = make_float4(go[0], go[1], go[2], go[3]);
    g4[1] = make_float4(go[4], go[5], go[6], go[7]);
  }
}

}  // namespace memt
