// Snapshot readout kernels.
//
// Every token t of block n reads that block's incoming fp32 snapshot:
//     o[t,h,:] = scale * q[t,h,:] . cast(S[n,h])
// (models/qwen/ops/_triton/read.py:22-71 — state cast to the query dtype, fp32
// accumulation, scale, cast to the output dtype; models/deepseek/ops/read.py:6-31 is
// the same product through bf16 baddbmm). Two kernels:
//   read_gemv_kernel  few tokens per block (decode): HBM-bound stream over the fp32
//                     state with 128-bit loads; one CTA per (block, head, 4 tokens).
//   read_tile_kernel  many tokens per block (commit / prefill queries): bf16 state panel
//                     in shared memory, 64-token tiles on mma.sync tensor cores.
// Both can apply the fused epilogue of the query path: l2norm(q) before the product and
//   y = bf16(w * bf16(o * rsqrt(mean o^2 + eps))) * L tanh(SiLU(gate)/L)
//   out = bf16(residual + y)
// (models/qwen/layer.py:15-31,116; models/qwen/integration.py:61-64).
#pragma once

#include "common.cuh"

namespace memt {

__device__ __forceinline__ void block_range(const ReadParams& p, int n, int64_t& bos, int64_t& eos) {
  int64_t a = p.cu[n], b = p.cu[n + 1];
  bos = a < 0 ? 0 : (a > p.L ? p.L : a);
  eos = b < bos ? bos : (b > p.L ? p.L : b);
}

// Tiles of a block owned by the CTA with blockIdx.y = y: runs of `per` consecutive tiles,
// run y, y + gridDim.y, ...; strided_tile_index(i) is the block-relative index of the CTA's
// i-th tile and strided_tiles the number of them for a block of `len` tokens.
__device__ __forceinline__ int64_t strided_tile_index(int i, int per) {
  return ((int64_t)blockIdx.y + (int64_t)(i / per) * gridDim.y) * per + i % per;
}
__device__ __forceinline__ int strided_tiles(int64_t len, int tok, int per) {
  const int64_t total = (len + tok - 1) / tok;
  int64_t count = 0;
  for (int64_t run = blockIdx.y; run * per < total; run += gridDim.y) {
    const int64_t left = total - run * per;
    count += left < per ? left : per;
  }
  return (int)count;
}

// snapshot of block n: n itself, or slots[n] when the caller passes slot indices into a state
// pool; -1 for an index outside the pool (the block is skipped and its outputs left unwritten)
__device__ __forceinline__ int64_t state_slot(const ReadParams& p, int n) {
  if (p.slots == nullptr) return n;
  const int s = p.slots[n];
  return (s >= 0 && s < p.num_slots) ? s : -1;
}

// softcapped SiLU gate and the gated RMSNorm output for one element (fp32 math, bf16
// rounding points of MemTRMSNormGated.forward)
__device__ __forceinline__ float gated_norm_value(float o, float rstd, float w, float gate, float softcap) {
  const float xn = bf16_round(o * rstd);
  const float hs = bf16_round(w * xn);
  const float sg = gate / (1.f + expf(-gate));
  const float gv = softcap > 0.f ? softcap * tanhf(sg / softcap) : sg;
  return hs * gv;
}

// ---------------------------------------------------------------------------
// GEMV: CTA = (block, head, group of TQ tokens), 256 threads.
// The fp32 state is the only large operand, so every thread issues its state loads
// (16 x 128-bit for D = 128, double-buffered batches for D = 256) before the query,
// gate and residual loads and the query normalisation: the state stream and the
// prologue latencies overlap and each SM keeps >= 64 KB in flight.
// ---------------------------------------------------------------------------
template <int D>
struct GemvCfg {
  static constexpr int kTPR = D / 4;                     // threads per state row (one float4 each)
  static constexpr int kRPP = 256 / kTPR;                // rows per pass
  static constexpr int kPer = D / kRPP;                  // float4 loads per thread
  static constexpr int kBatch = kPer < 16 ? kPer : (D >= 256 ? 8 : 16);
  static constexpr int kBatches = kPer / kBatch;
};

// one-token (decode) CTAs at three per SM, so that one CTA's reduction and epilogue overlap
// two others' state streams
// one group of up to TQ tokens [t0, t0 + nt) of head h reading snapshot `slot`; every thread
// of the CTA calls it (it synchronises the CTA)
template <int D, int TQ, bool EXACT>
__device__ __forceinline__ void gemv_group(const ReadParams& p, int h, int64_t slot, int64_t t0, int nt) {
  using Cfg = GemvCfg<D>;
  constexpr int RPP = Cfg::kRPP, TPR = Cfg::kTPR, BATCH = Cfg::kBatch;
  // declared here rather than passed in, so that every access compiles to a shared-memory one
  __shared__ float s_q[TQ][D];
  __shared__ float s_red[RPP][TQ][D];
  __shared__ float s_ss[TQ][8];
  const int tid = threadIdx.x;
  const int64_t qrow = (int64_t)p.H * D;

  // 1. state stream: first batch in flight before anything else
  const int cg = tid % TPR, ro = tid / TPR;
  const float4* S4 = reinterpret_cast<const float4*>(p.states + (slot * p.H + h) * D * D) + ro * TPR + cg;
  float4 cur[BATCH];
#pragma unroll
  for (int i = 0; i < BATCH; ++i) cur[i] = __ldg(S4 + (int64_t)i * RPP * TPR);

  // 2. prologue loads: queries, and for the fused epilogue this thread's gate and residual
  const int v = tid;
  float gt[TQ], res[TQ];
#pragma unroll
  for (int j = 0; j < TQ; ++j) gt[j] = res[j] = 0.f;
  if (p.fused && v < D) {
#pragma unroll
    for (int j = 0; j < TQ; ++j) {
      if (j < nt) {
        const int64_t tok = t0 + j;
        gt[j] = __bfloat162float(p.gate[tok * qrow + (int64_t)h * D + v]);
        if (p.residual != nullptr)
          res[j] = __bfloat162float(p.residual[tok * p.row_stride + (int64_t)(p.head_offset + h) * D + v]);
      }
    }
  }
  for (int idx = tid; idx < TQ * D; idx += 256) {
    const int j = idx / D, c = idx % D;
    float x = 0.f;
    if (j < nt) {
      const int64_t off = (t0 + j) * qrow + (int64_t)h * D + c;
      x = EXACT ? static_cast<const float*>(p.q)[off]
                : __bfloat162float(static_cast<const __nv_bfloat16*>(p.q)[off]);
    }
    s_q[j][c] = x;
  }
  __syncthreads();
  // queries optionally l2-normalised (fp32 sum of squares, bf16 output as in FLA l2norm)
  if (p.normalize_q) {
    const int warp = tid >> 5, lane = tid & 31;
    if (warp < TQ) {
      float ss = 0.f;
      for (int c = lane; c < D; c += 32) ss += s_q[warp][c] * s_q[warp][c];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      const float rstd = 1.f / sqrtf(ss + p.q_eps);
      for (int c = lane; c < D; c += 32) {
        const float y = s_q[warp][c] * rstd;
        s_q[warp][c] = EXACT ? y : bf16_round(y);
      }
    }
    __syncthreads();
  }

  // 3. products, batch by batch (the next batch is in flight while one is consumed)
  float acc[TQ][4];
#pragma unroll
  for (int j = 0; j < TQ; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
#pragma unroll
  for (int b = 0; b < Cfg::kBatches; ++b) {
    float4 nxt[BATCH];
    if (b + 1 < Cfg::kBatches) {
#pragma unroll
      for (int i = 0; i < BATCH; ++i) nxt[i] = __ldg(S4 + (int64_t)((b + 1) * BATCH + i) * RPP * TPR);
    }
#pragma unroll
    for (int i = 0; i < BATCH; ++i) {
      float4 s = cur[i];
      if (!EXACT) {
        s.x = bf16_round(s.x);
        s.y = bf16_round(s.y);
        s.z = bf16_round(s.z);
        s.w = bf16_round(s.w);
      }
      const int row = ro + (b * BATCH + i) * RPP;
#pragma unroll
      for (int j = 0; j < TQ; ++j) {
        const float qv = s_q[j][row];
        acc[j][0] = fmaf(qv, s.x, acc[j][0]);
        acc[j][1] = fmaf(qv, s.y, acc[j][1]);
        acc[j][2] = fmaf(qv, s.z, acc[j][2]);
        acc[j][3] = fmaf(qv, s.w, acc[j][3]);
      }
    }
    if (b + 1 < Cfg::kBatches) {
#pragma unroll
      for (int i = 0; i < BATCH; ++i) cur[i] = nxt[i];
    }
  }
#pragma unroll
  for (int j = 0; j < TQ; ++j)
    *reinterpret_cast<float4*>(&s_red[ro][j][4 * cg]) = make_float4(acc[j][0], acc[j][1], acc[j][2], acc[j][3]);
  __syncthreads();

  if (!p.fused) {
    for (int idx = tid; idx < nt * D; idx += 256) {
      const int j = idx / D, c = idx % D;
      float o = 0.f;
#pragma unroll
      for (int r = 0; r < RPP; ++r) o += s_red[r][j][c];
      o *= p.scale;
      const int64_t off = (t0 + j) * qrow + (int64_t)h * D + c;
      if (p.out_bf16)
        static_cast<__nv_bfloat16*>(p.out)[off] = __float2bfloat16_rn(o);
      else
        static_cast<float*>(p.out)[off] = o;
    }
    return;
  }

  // 4. fused epilogue: one value per thread and token (D <= 256)
  float o[TQ];
#pragma unroll
  for (int j = 0; j < TQ; ++j) {
    float x = 0.f;
    if (v < D) {
#pragma unroll
      for (int r = 0; r < RPP; ++r) x += s_red[r][j][v];
      x = bf16_round(x * p.scale);  // the read output is bf16 in the reference
    }
    o[j] = x;
    float ss = x * x;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if ((tid & 31) == 0) s_ss[j][tid >> 5] = ss;
  }
  __syncthreads();
  if (v < D) {
    const float w = __bfloat162float(p.norm_w[v]);
#pragma unroll
    for (int j = 0; j < TQ; ++j) {
      if (j >= nt) break;
      float ss = 0.f;
#pragma unroll
      for (int wi = 0; wi < 8; ++wi) ss += s_ss[j][wi];
      const float rstd = rsqrtf(ss / D + p.norm_eps);
      const int64_t tok = t0 + j;
      float y = bf16_round(gated_norm_value(o[j], rstd, w, gt[j], p.softcap));
      const int64_t oo = tok * p.row_stride + (int64_t)(p.head_offset + h) * D + v;
      if (p.residual != nullptr) y = res[j] + y;
      static_cast<__nv_bfloat16*>(p.out)[oo] = __float2bfloat16_rn(y);
    }
  }
}

// Status of the one-token decode kernel on this device: bit 0 = a block held more tokens than
// the grid's bound covered (its tokens past the first were not read). Read and cleared by
// memt_read_status.
static __device__ int g_read_status;

// CTA (block, head, y). Multi-token CTAs (TQ > 1) take token groups y, y + gridDim.y, ... of
// the block, so every token is read whatever bound the host sized the grid with. The one-token
// decode CTA runs its group alone: a loop costs it registers it does not have (18 % of its
// time), so a block longer than the bound is only detected, in g_read_status (the host rejects
// bounds that are provably short before launch).
template <int D, int TQ, bool EXACT>
__global__ void __launch_bounds__(256, (TQ == 1 && D <= 128) ? 3 : 2) read_gemv_kernel(ReadParams p) {
  const int n = blockIdx.x / p.H, h = blockIdx.x % p.H;
  int64_t bos, eos;
  block_range(p, n, bos, eos);
  int64_t t0 = bos + (int64_t)blockIdx.y * TQ;
  if (t0 >= eos) return;
  const int64_t slot = state_slot(p, n);
  if (slot < 0) return;
  const int64_t stride = (int64_t)gridDim.y * TQ;
  if constexpr (TQ == 1) {
    if (t0 + stride < eos && threadIdx.x == 0) atomicOr(&g_read_status, 1);
    gemv_group<D, TQ, EXACT>(p, h, slot, t0, 1);
  } else {
    for (;;) {
      gemv_group<D, TQ, EXACT>(p, h, slot, t0, (int)((eos - t0) < TQ ? (eos - t0) : TQ));
      t0 += stride;
      if (t0 >= eos) break;
      __syncthreads();  // the shared buffers are reused by the next group
    }
  }
}

// ---------------------------------------------------------------------------
// Tile kernel: CTA = (block, head, run of up to kTilesPerCta 64-token tiles).
// bf16 state panel [D][D] (swizzled) resident in shared memory; warps split rows
// (4 row blocks of 16 tokens) and, for D = 256, column halves.
// ---------------------------------------------------------------------------
// 64-token tiles per CTA run: each CTA stages its block's bf16 snapshot (D^2 * 2 bytes) once, so
// a wider state takes longer runs (d = 256: 128 KB of staging per 2,048 tokens)
template <int D>
constexpr int read_tiles_per_cta() { return D >= 256 ? 32 : 8; }

template <int D>
struct ReadTileCfg {
  static constexpr int kNW = D <= 128 ? 4 : 8;
  static constexpr int kColSplit = kNW / 4;
  static constexpr int kNT = D / 8 / kColSplit;  // n-tiles per warp
  static constexpr size_t kBytesS = size_t(D) * D * 2;
  static constexpr size_t kBytesQ = size_t(kTile) * D * 2;
  // + slack: the kernel rounds the dynamic base up to 128 bytes itself
  static constexpr size_t kSmem = kBytesS + 2 * kBytesQ + 4 * 16 * 2 * 4 + 128;
};

template <int RL>
__device__ __forceinline__ int rswz(int row, int col) {
  return row * RL + ((((col >> 3) ^ row) & 7) | ((col >> 3) & ~7)) * 8 + (col & 7);
}

template <int D>
__global__ void __launch_bounds__(ReadTileCfg<D>::kNW * 32) read_tile_kernel(ReadParams p) {
  using Cfg = ReadTileCfg<D>;
  extern __shared__ __align__(128) unsigned char smem_read[];
  unsigned char* smem = smem_read + ((128u - (smem_u32(smem_read) & 127u)) & 127u);
  __nv_bfloat16* sS = reinterpret_cast<__nv_bfloat16*>(smem);
  __nv_bfloat16* sQ[2] = {reinterpret_cast<__nv_bfloat16*>(smem + Cfg::kBytesS),
                          reinterpret_cast<__nv_bfloat16*>(smem + Cfg::kBytesS + Cfg::kBytesQ)};
  float* sRow = reinterpret_cast<float*>(smem + Cfg::kBytesS + 2 * Cfg::kBytesQ);  // [4][16][2]
  constexpr int NT = Cfg::kNW * 32;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int n = blockIdx.x / p.H, h = blockIdx.x % p.H;
  int64_t bos, eos;
  block_range(p, n, bos, eos);
  // this CTA's tiles: runs y, y + gridDim.y, ... of kReadTilesPerCta tiles, so that every token
  // is read whatever bound on the block length the host sized the grid with
  constexpr int kReadTilesPerCta = read_tiles_per_cta<D>();
  const int ntiles = strided_tiles(eos - bos, kTile, kReadTilesPerCta);
  if (ntiles == 0) return;
  const int64_t slot = state_slot(p, n);
  if (slot < 0) return;
  auto tile_start = [&](int i) { return bos + strided_tile_index(i, kReadTilesPerCta) * kTile; };
  const int64_t qrow = (int64_t)p.H * D;
  const __nv_bfloat16* q = static_cast<const __nv_bfloat16*>(p.q);

  auto load_q = [&](int tile, int buf) {
    const int64_t tb = tile_start(tile);
    for (int i = tid; i < kTile * D / 8; i += NT) {
      const int row = i / (D / 8), col = (i % (D / 8)) * 8;
      const bool valid = tb + row < eos;
      const __nv_bfloat16* src = q + (valid ? (tb + row) * qrow + (int64_t)h * D + col : 0);
      cp_async16_zfill(sQ[buf] + rswz<D>(row, col), src, valid);
    }
    cp_async_commit();
  };
  load_q(0, 0);

  // bf16(S) -> shared (read.py:64)
  const float4* S4 = reinterpret_cast<const float4*>(p.states + (slot * p.H + h) * D * D);
  for (int i = tid; i < D * D / 4; i += NT) {
    const int row = i / (D / 4), col = (i % (D / 4)) * 4;
    const float4 s = __ldg(S4 + i);
    uint2 pk = make_uint2(pack_bf16x2(s.x, s.y), pack_bf16x2(s.z, s.w));
    *reinterpret_cast<uint2*>(sS + rswz<D>(row, col)) = pk;
  }

  const int rb = warp % 4, cs = warp / 4;
  const int n0 = cs * Cfg::kNT * 8;
  for (int tile = 0; tile < ntiles; ++tile) {
    const int buf = tile & 1;
    cp_async_wait<0>();
    __syncthreads();
    if (tile + 1 < ntiles) load_q(tile + 1, buf ^ 1);
    __nv_bfloat16* sq = sQ[buf];
    if (p.fused && p.normalize_q) {
      // l2norm of the 64 query rows in place (fp32 math, bf16 result): warp w rows w, w+NW, ...
      for (int row = warp; row < kTile; row += Cfg::kNW) {
        float ss = 0.f;
        for (int c = lane; c < D; c += 32) {
          const float x = __bfloat162float(sq[rswz<D>(row, c)]);
          ss += x * x;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float rstd = 1.f / sqrtf(ss + p.q_eps);
        for (int c = lane; c < D; c += 32) {
          const float x = __bfloat162float(sq[rswz<D>(row, c)]);
          sq[rswz<D>(row, c)] = __float2bfloat16_rn(x * rstd);
        }
      }
      __syncthreads();
    }
    float acc[Cfg::kNT][4];
#pragma unroll
    for (int i = 0; i < Cfg::kNT; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      uint32_t a[4];
      ldsm_x4(a, smem_u32(sq + rswz<D>(16 * rb + (lane & 15), 16 * ks + 8 * (lane >> 4))));
#pragma unroll
      for (int np = 0; np < Cfg::kNT; np += 2) {
        uint32_t b[4];
        ldsm_x4_t(b, smem_u32(sS + rswz<D>(16 * ks + (lane & 15), n0 + 8 * np + 8 * (lane >> 4))));
        uint32_t b0[2] = {b[0], b[1]}, b1[2] = {b[2], b[3]};
        mma_bf16_16816(acc[np], a, b0);
        mma_bf16_16816(acc[np + 1], a, b1);
      }
    }
    const int64_t tb = tile_start(tile);
    const int64_t r0 = tb + 16 * rb + g, r1 = r0 + 8;
    const bool ok0 = r0 < eos, ok1 = r1 < eos;
    if (!p.fused) {
#pragma unroll
      for (int i = 0; i < Cfg::kNT; ++i) {
        const int col = n0 + 8 * i + 2 * t;
        const float o00 = acc[i][0] * p.scale, o01 = acc[i][1] * p.scale;
        const float o10 = acc[i][2] * p.scale, o11 = acc[i][3] * p.scale;
        if (p.out_bf16) {
          __nv_bfloat16* out = static_cast<__nv_bfloat16*>(p.out);
          if (ok0) *reinterpret_cast<uint32_t*>(out + r0 * qrow + (int64_t)h * D + col) = pack_bf16x2(o00, o01);
          if (ok1) *reinterpret_cast<uint32_t*>(out + r1 * qrow + (int64_t)h * D + col) = pack_bf16x2(o10, o11);
        } else {
          float* out = static_cast<float*>(p.out);
          if (ok0) *reinterpret_cast<float2*>(out + r0 * qrow + (int64_t)h * D + col) = make_float2(o00, o01);
          if (ok1) *reinterpret_cast<float2*>(out + r1 * qrow + (int64_t)h * D + col) = make_float2(o10, o11);
        }
      }
      continue;
    }
    // fused epilogue: row sums of squares of the bf16 read output
    float ss0 = 0.f, ss1 = 0.f;
#pragma unroll
    for (int i = 0; i < Cfg::kNT; ++i) {
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[i][e] = bf16_round(acc[i][e] * p.scale);
      ss0 += acc[i][0] * acc[i][0] + acc[i][1] * acc[i][1];
      ss1 += acc[i][2] * acc[i][2] + acc[i][3] * acc[i][3];
    }
    ss0 += __shfl_xor_sync(0xffffffffu, ss0, 1);
    ss0 += __shfl_xor_sync(0xffffffffu, ss0, 2);
    ss1 += __shfl_xor_sync(0xffffffffu, ss1, 1);
    ss1 += __shfl_xor_sync(0xffffffffu, ss1, 2);
    if (Cfg::kColSplit > 1) {
      if (t == 0) {
        sRow[(rb * 16 + g) * 2 + cs] = ss0;
        sRow[(rb * 16 + g + 8) * 2 + cs] = ss1;
      }
      __syncthreads();
      ss0 = sRow[(rb * 16 + g) * 2] + sRow[(rb * 16 + g) * 2 + 1];
      ss1 = sRow[(rb * 16 + g + 8) * 2] + sRow[(rb * 16 + g + 8) * 2 + 1];
    }
    const float rstd0 = rsqrtf(ss0 / D + p.norm_eps), rstd1 = rsqrtf(ss1 / D + p.norm_eps);
    __nv_bfloat16* out = static_cast<__nv_bfloat16*>(p.out);
#pragma unroll
    for (int i = 0; i < Cfg::kNT; ++i) {
      const int col = n0 + 8 * i + 2 * t;
      const float2 w = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(p.norm_w + col));
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int64_t r = half ? r1 : r0;
        if (!(half ? ok1 : ok0)) continue;
        const float rstd = half ? rstd1 : rstd0;
        const float2 gt = unpack_bf16x2(
            *reinterpret_cast<const uint32_t*>(p.gate + r * qrow + (int64_t)h * D + col));
        float y0 = bf16_round(gated_norm_value(acc[i][2 * half], rstd, w.x, gt.x, p.softcap));
        float y1 = bf16_round(gated_norm_value(acc[i][2 * half + 1], rstd, w.y, gt.y, p.softcap));
        const int64_t oo = r * p.row_stride + (int64_t)(p.head_offset + h) * D + col;
        if (p.residual != nullptr) {
          const float2 res = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(p.residual + oo));
          y0 += res.x;
          y1 += res.y;
        }
        *reinterpret_cast<uint32_t*>(out + oo) = pack_bf16x2(y0, y1);
      }
    }
  }
}

}  // namespace memt
