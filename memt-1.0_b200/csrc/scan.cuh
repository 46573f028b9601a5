// GDN-2 inter-chunk state scan: one CTA per (sample, head, 64-wide value panel).
//
// Replaces _fwd_h_kernel (models/qwen/ops/_triton/state.py:31-115; the DeepSeek copy
// models/deepseek/ops/_triton/state.py:11-93). For every chunk of the sample, in order:
//     v_new = u - w . bf16(S)                         (state.py:95-98)
//     S     = diag(2^G_last) S + kg^T . bf16(v_new)   (state.py:101-112)
// The fp32 state panel [D x 64] stays in registers for the whole sample (C fragments
// of the second product); w, kg and the u panel of the next chunk stream in with
// cp.async while the current chunk computes. Rows of padded tokens are zero in w, u and
// kg, so the loop needs no masking.
#pragma once

#include "common.cuh"

namespace memt {

// XOR-swizzled bf16 tile with RL elements per row (RL % 64 == 0): the 16-byte chunk
// index is XORed with (row & 7), so ldmatrix over 8 consecutive rows is conflict-free.
template <int RL>
__device__ __forceinline__ int swz(int row, int col) {
  return row * RL + ((((col >> 3) ^ row) & 7) | ((col >> 3) & ~7)) * 8 + (col & 7);
}

template <int D, int BV, int NW>
struct ScanCfg {
  static constexpr int kThreads = NW * 32;
  static constexpr int kRowsPerWarp = D / NW;       // state rows (key channels) per warp
  static constexpr int kMT = kRowsPerWarp / 16;     // m-tiles per warp in the update product
  static constexpr int kNT = BV / 8;                // n-tiles of the value panel
  static constexpr int kXWarpsPerRow = NW / 4;      // warps sharing a 16-token row block
  static constexpr int kXNT = kNT / kXWarpsPerRow;  // n-tiles per warp in the first product
  static constexpr size_t kBytesWK = size_t(kTile) * D * 2;
  static constexpr size_t kBytesU = size_t(kTile) * BV * 2;
  static constexpr size_t kBytesStage = 2 * kBytesWK + kBytesU + size_t(D) * 4;
  static constexpr size_t kBytesSb = size_t(D) * BV * 2;
  static constexpr size_t kBytesVn = size_t(kTile) * BV * 2;
  static constexpr size_t kSmem = 2 * kBytesStage + kBytesSb + kBytesVn;
  static_assert(kRowsPerWarp % 16 == 0, "state rows per warp");
  static_assert(NW % 4 == 0, "warps");
};

template <int D, int BV, int NW>
__global__ void __launch_bounds__(NW * 32) scan_kernel(ScanParams p) {
  using Cfg = ScanCfg<D, BV, NW>;
  extern __shared__ __align__(128) unsigned char smem_scan[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  constexpr int NV = D / BV;
  const int vp = blockIdx.x % NV;
  const int nh = blockIdx.x / NV;
  const int h = nh % p.H, n = nh / p.H;
  const int v0 = vp * BV;

  unsigned char* smem = smem_scan;
  unsigned char* stage_base[2] = {smem, smem + Cfg::kBytesStage};
  __nv_bfloat16* sSb = reinterpret_cast<__nv_bfloat16*>(smem + 2 * Cfg::kBytesStage);
  __nv_bfloat16* sVn = reinterpret_cast<__nv_bfloat16*>(smem + 2 * Cfg::kBytesStage + Cfg::kBytesSb);

  auto sW = [&](int st) { return reinterpret_cast<__nv_bfloat16*>(stage_base[st]); };
  auto sKG = [&](int st) { return reinterpret_cast<__nv_bfloat16*>(stage_base[st] + Cfg::kBytesWK); };
  auto sU = [&](int st) {
    return reinterpret_cast<__nv_bfloat16*>(stage_base[st] + 2 * Cfg::kBytesWK);
  };
  auto sEl = [&](int st) {
    return reinterpret_cast<float*>(stage_base[st] + 2 * Cfg::kBytesWK + Cfg::kBytesU);
  };

  auto prefetch = [&](int c, int st) {
    const int64_t ch = (int64_t)c * p.H + h;
    const __nv_bfloat16* gw = p.W + ch * kTile * D;
    const __nv_bfloat16* gk = p.KG + ch * kTile * D;
    const __nv_bfloat16* gu = p.U + ch * kTile * D + v0;
    constexpr int kChunksWK = kTile * D / 8;
    for (int i = tid; i < kChunksWK; i += Cfg::kThreads) {
      const int row = i / (D / 8), col = (i % (D / 8)) * 8;
      cp_async16(sW(st) + swz<D>(row, col), gw + row * D + col);
      cp_async16(sKG(st) + swz<D>(row, col), gk + row * D + col);
    }
    constexpr int kChunksU = kTile * BV / 8;
    for (int i = tid; i < kChunksU; i += Cfg::kThreads) {
      const int row = i / (BV / 8), col = (i % (BV / 8)) * 8;
      cp_async16(sU(st) + swz<BV>(row, col), gu + row * D + col);
    }
    for (int i = tid; i < D / 4; i += Cfg::kThreads)
      cp_async16(sEl(st) + 4 * i, p.Elast + ch * D + 4 * i);
    cp_async_commit();
  };

  // ---- load the initial state panel into C fragments ----
  float S[Cfg::kMT][Cfg::kNT][4];
  const int64_t state_off = ((int64_t)n * p.H + h) * D * D;
  const int row_base = warp * Cfg::kRowsPerWarp;
#pragma unroll
  for (int mt = 0; mt < Cfg::kMT; ++mt)
#pragma unroll
    for (int nt = 0; nt < Cfg::kNT; ++nt) {
      const int r0 = row_base + 16 * mt + g;
      const int col = v0 + 8 * nt + 2 * t;
      float2 a = *reinterpret_cast<const float2*>(p.h0 + state_off + (int64_t)r0 * D + col);
      float2 b = *reinterpret_cast<const float2*>(p.h0 + state_off + (int64_t)(r0 + 8) * D + col);
      S[mt][nt][0] = a.x;
      S[mt][nt][1] = a.y;
      S[mt][nt][2] = b.x;
      S[mt][nt][3] = b.y;
    }

  const int c0 = p.sample_off[n], c1 = p.sample_off[n + 1];
  if (c0 < c1) prefetch(c0, 0);

  const int xrb = warp % 4;                     // 16-token row block of the first product
  const int xn0 = (warp / 4) * Cfg::kXNT * 8;   // its first value column
  for (int c = c0; c < c1; ++c) {
    const int st = (c - c0) & 1;
    cp_async_wait<0>();
    __syncthreads();  // chunk c landed everywhere; all warps are done with chunk c-1
    if (c + 1 < c1) prefetch(c + 1, st ^ 1);

    // bf16(S) -> sSb [D][BV]  (state.py:98: the state is cast to bf16 for the product)
#pragma unroll
    for (int mt = 0; mt < Cfg::kMT; ++mt)
#pragma unroll
      for (int nt = 0; nt < Cfg::kNT; ++nt) {
        const int r0 = row_base + 16 * mt + g;
        const int col = 8 * nt + 2 * t;
        *reinterpret_cast<uint32_t*>(sSb + swz<BV>(r0, col)) = pack_bf16x2(S[mt][nt][0], S[mt][nt][1]);
        *reinterpret_cast<uint32_t*>(sSb + swz<BV>(r0 + 8, col)) =
            pack_bf16x2(S[mt][nt][2], S[mt][nt][3]);
      }
    __syncthreads();

    // X = w . bf16(S) for tokens 16*xrb.., columns xn0..; v_new = u - X -> bf16 -> sVn
    {
      float X[Cfg::kXNT][4];
#pragma unroll
      for (int i = 0; i < Cfg::kXNT; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) X[i][j] = 0.f;
      const __nv_bfloat16* w = sW(st);
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        uint32_t a[4];
        ldsm_x4(a, smem_u32(w + swz<D>(16 * xrb + (lane & 15), 16 * ks + 8 * (lane >> 4))));
#pragma unroll
        for (int np = 0; np < Cfg::kXNT; np += 2) {
          uint32_t b[4];
          ldsm_x4_t(b, smem_u32(sSb + swz<BV>(16 * ks + (lane & 15), xn0 + 8 * np + 8 * (lane >> 4))));
          uint32_t b0[2] = {b[0], b[1]}, b1[2] = {b[2], b[3]};
          mma_bf16_16816(X[np], a, b0);
          mma_bf16_16816(X[np + 1], a, b1);
        }
      }
      const __nv_bfloat16* u = sU(st);
#pragma unroll
      for (int nt = 0; nt < Cfg::kXNT; ++nt) {
        const int row = 16 * xrb + g;
        const int col = xn0 + 8 * nt + 2 * t;
        float2 u0 = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(u + swz<BV>(row, col)));
        float2 u1 = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(u + swz<BV>(row + 8, col)));
        *reinterpret_cast<uint32_t*>(sVn + swz<BV>(row, col)) = pack_bf16x2(u0.x - X[nt][0], u0.y - X[nt][1]);
        *reinterpret_cast<uint32_t*>(sVn + swz<BV>(row + 8, col)) =
            pack_bf16x2(u1.x - X[nt][2], u1.y - X[nt][3]);
      }
    }
    __syncthreads();

    // S = diag(2^G_last) S + kg^T . bf16(v_new)
    {
      const float* el = sEl(st);
      const __nv_bfloat16* kg = sKG(st);
#pragma unroll
      for (int mt = 0; mt < Cfg::kMT; ++mt) {
        const float e0 = el[row_base + 16 * mt + g], e1 = el[row_base + 16 * mt + g + 8];
#pragma unroll
        for (int nt = 0; nt < Cfg::kNT; ++nt) {
          S[mt][nt][0] *= e0;
          S[mt][nt][1] *= e0;
          S[mt][nt][2] *= e1;
          S[mt][nt][3] *= e1;
        }
      }
#pragma unroll
      for (int ks = 0; ks < kTile / 16; ++ks) {
        uint32_t bfr[Cfg::kNT][2];
#pragma unroll
        for (int np = 0; np < Cfg::kNT; np += 2) {
          uint32_t b[4];
          ldsm_x4_t(b, smem_u32(sVn + swz<BV>(16 * ks + (lane & 15), 8 * np + 8 * (lane >> 4))));
          bfr[np][0] = b[0];
          bfr[np][1] = b[1];
          bfr[np + 1][0] = b[2];
          bfr[np + 1][1] = b[3];
        }
#pragma unroll
        for (int mt = 0; mt < Cfg::kMT; ++mt) {
          // A = kg^T: rows = key channels, k = tokens; kg is stored [token][channel]
          const int tok = 16 * ks + (lane & 7) + 8 * (lane >> 4);
          const int chn = row_base + 16 * mt + 8 * ((lane >> 3) & 1);
          uint32_t a[4];
          ldsm_x4_t(a, smem_u32(kg + swz<D>(tok, chn)));
#pragma unroll
          for (int nt = 0; nt < Cfg::kNT; ++nt) mma_bf16_16816(S[mt][nt], a, bfr[nt]);
        }
      }
    }
  }

  // ---- final state ----
#pragma unroll
  for (int mt = 0; mt < Cfg::kMT; ++mt)
#pragma unroll
    for (int nt = 0; nt < Cfg::kNT; ++nt) {
      const int r0 = row_base + 16 * mt + g;
      const int col = v0 + 8 * nt + 2 * t;
      *reinterpret_cast<float2*>(p.ht + state_off + (int64_t)r0 * D + col) =
          make_float2(S[mt][nt][0], S[mt][nt][1]);
      *reinterpret_cast<float2*>(p.ht + state_off + (int64_t)(r0 + 8) * D + col) =
          make_float2(S[mt][nt][2], S[mt][nt][3]);
    }
}

}  // namespace memt
