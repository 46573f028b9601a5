// GDN-2 inter-chunk state scan: one CTA per (sample, head, 64-wide value panel).
//
// Replaces _fwd_h_kernel (models/qwen/ops/_triton/state.py:31-115; the DeepSeek copy
// models/deepseek/ops/_triton/state.py:11-93). For every chunk of the sample, in order:
//     v_new = u - w . bf16(S)                         (state.py:95-98)
//     S     = diag(2^G_last) S + kg^T . bf16(v_new)   (state.py:101-112)
// The fp32 state panel [D x 64] stays in registers for the whole sample (C fragments of the
// second product, one 16-row m-tile per warp). The next chunk's w, kg, u panel and 2^G_last
// arrive with four bulk (TMA) copies issued by one thread into the other stage while the
// current chunk computes; the intra kernel stored them in exactly the shared-memory layout
// used here (64-column panels, each swz<64>). Rows of padded tokens are zero in w, u and kg, so no masking is needed.
#pragma once

#include "common.cuh"

namespace memt {

template <int D>
struct ScanCfg {
  static constexpr int BV = 64;                 // value panel per CTA
  static constexpr int NW = D / 16;             // one 16-row state m-tile per warp
  static constexpr int kThreads = NW * 32;
  static constexpr int kNT = BV / 8;            // n-tiles of the value panel
  static constexpr int kXWarpsPerRow = NW / 4;  // warps sharing a 16-token row block of X
  static constexpr int kXNT = kNT / kXWarpsPerRow;
  static constexpr uint32_t kBytesWK = uint32_t(kTile) * D * 2;
  static constexpr uint32_t kBytesU = uint32_t(kTile) * BV * 2;
  static constexpr uint32_t kBytesEl = uint32_t(D) * 4;
  static constexpr uint32_t kBytesStage = 2 * kBytesWK + kBytesU + kBytesEl;
  static constexpr uint32_t kBytesSb = uint32_t(D) * BV * 2;
  static constexpr uint32_t kBytesVn = uint32_t(kTile) * BV * 2;
  // + slack: the kernel rounds the dynamic base up to 128 bytes itself
  static constexpr size_t kSmem = 2 * size_t(kBytesStage) + kBytesSb + kBytesVn + 64 + 128;
  static_assert(kXNT % 2 == 0 && kXNT >= 2, "value tiles per warp");
};

template <int D>
__global__ void __launch_bounds__(ScanCfg<D>::kThreads) scan_kernel(ScanParams p) {
  using Cfg = ScanCfg<D>;
  constexpr int BV = Cfg::BV;
  extern __shared__ __align__(128) unsigned char smem_scan_raw[];
  unsigned char* smem_scan = smem_scan_raw + ((128u - (smem_u32(smem_scan_raw) & 127u)) & 127u);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  constexpr int NV = D / BV;
  const int vp = blockIdx.x % NV;
  const int nh = blockIdx.x / NV;
  const int h = nh % p.H, n = nh / p.H;
  const int v0 = vp * BV;

  __nv_bfloat16* sSb = reinterpret_cast<__nv_bfloat16*>(smem_scan + 2 * Cfg::kBytesStage);
  __nv_bfloat16* sVn = reinterpret_cast<__nv_bfloat16*>(smem_scan + 2 * Cfg::kBytesStage + Cfg::kBytesSb);
  uint64_t* mbar = reinterpret_cast<uint64_t*>(smem_scan + 2 * Cfg::kBytesStage + Cfg::kBytesSb + Cfg::kBytesVn);
  auto stage = [&](int st) { return smem_scan + st * Cfg::kBytesStage; };
  auto sW = [&](int st) { return reinterpret_cast<__nv_bfloat16*>(stage(st)); };
  auto sKG = [&](int st) { return reinterpret_cast<__nv_bfloat16*>(stage(st) + Cfg::kBytesWK); };
  auto sU = [&](int st) { return reinterpret_cast<__nv_bfloat16*>(stage(st) + 2 * Cfg::kBytesWK); };
  auto sEl = [&](int st) { return reinterpret_cast<const float*>(stage(st) + 2 * Cfg::kBytesWK + Cfg::kBytesU); };

  // one thread arms the stage barrier and issues the four bulk copies of chunk c
  auto prefetch = [&](int c, int st) {
    const int64_t ch = (int64_t)c * p.H + h;
    const uint32_t mb = smem_u32(&mbar[st]);
    mbar_expect_tx(mb, Cfg::kBytesStage);
    bulk_g2s(smem_u32(sW(st)), p.W + ch * kTile * D, Cfg::kBytesWK, mb);
    bulk_g2s(smem_u32(sKG(st)), p.KG + ch * kTile * D, Cfg::kBytesWK, mb);
    bulk_g2s(smem_u32(sU(st)), p.U + (ch * (D / BV) + vp) * kTile * BV, Cfg::kBytesU, mb);
    bulk_g2s(smem_u32(sEl(st)), p.Elast + ch * D, Cfg::kBytesEl, mb);
  };

  griddep_wait();
  griddep_launch_dependents();
  const int c0 = p.sample_off[n], c1 = p.sample_off[n + 1];
  if (tid == 0) {
    mbar_init(smem_u32(&mbar[0]), 1);
    mbar_init(smem_u32(&mbar[1]), 1);
    mbar_fence_init();
  }
  __syncthreads();
  if (tid == 0 && c0 < c1) prefetch(c0, 0);

  // ---- initial state panel: warp w owns rows 16w..16w+15 (C fragments) ----
  float S[Cfg::kNT][4];
  const int64_t in_slot = pool_slot(p.slots_in, p.num_in, n), out_slot = pool_slot(p.slots_out, p.num_out, n);
  if (tid == 0 && (in_slot < 0 || out_slot < 0)) atomicOr(&p.hdr->status, 8);  // slot outside its pool
  const int64_t in_off = (in_slot * p.H + h) * D * D, out_off = (out_slot * p.H + h) * D * D;
  const int r0 = warp * 16 + g;
#pragma unroll
  for (int nt = 0; nt < Cfg::kNT; ++nt) {
    const int col = v0 + 8 * nt + 2 * t;
    float2 a = make_float2(0.f, 0.f), b = a;  // zero state for an input slot outside the pool
    if (in_slot >= 0) {
      a = *reinterpret_cast<const float2*>(p.h0 + in_off + (int64_t)r0 * D + col);
      b = *reinterpret_cast<const float2*>(p.h0 + in_off + (int64_t)(r0 + 8) * D + col);
    }
    S[nt][0] = a.x;
    S[nt][1] = a.y;
    S[nt][2] = b.x;
    S[nt][3] = b.y;
  }

  const int xrb = warp % 4;                    // 16-token row block of the first product
  const int xn0 = (warp / 4) * Cfg::kXNT * 8;  // its first value column
  bool ok = true;
  for (int c = c0; c < c1; ++c) {
    const int it = c - c0, st = it & 1;
    // bf16(S) -> sSb [D][BV]  (state.py:98: the state is cast to bf16 for the product)
#pragma unroll
    for (int nt = 0; nt < Cfg::kNT; ++nt) {
      const int col = 8 * nt + 2 * t;
      *reinterpret_cast<uint32_t*>(sSb + swz<BV>(r0, col)) = pack_bf16x2(S[nt][0], S[nt][1]);
      *reinterpret_cast<uint32_t*>(sSb + swz<BV>(r0 + 8, col)) = pack_bf16x2(S[nt][2], S[nt][3]);
    }
    // sSb complete; every warp finished chunk c-1 (stage st^1 is free); chunk c landed
    ok = __syncthreads_and(mbar_wait(smem_u32(&mbar[st]), (it >> 1) & 1)) != 0;
    if (!ok) break;
    if (tid == 0 && c + 1 < c1) prefetch(c + 1, st ^ 1);

    // X = w . bf16(S) for tokens 16*xrb.., value columns xn0..; v_new = u - X -> bf16 -> sVn
    {
      float X[Cfg::kXNT][4];
#pragma unroll
      for (int i = 0; i < Cfg::kXNT; ++i) X[i][0] = X[i][1] = X[i][2] = X[i][3] = 0.f;
      const __nv_bfloat16* w = sW(st);
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        uint32_t a[4];
        ldsm_x4(a, smem_u32(w + pswz(16 * xrb + (lane & 15), 16 * ks + 8 * (lane >> 4))));
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
      const int row = 16 * xrb + g;
#pragma unroll
      for (int nt = 0; nt < Cfg::kXNT; ++nt) {
        const int col = xn0 + 8 * nt + 2 * t;
        const float2 u0 = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(u + swz<BV>(row, col)));
        const float2 u1 = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(u + swz<BV>(row + 8, col)));
        *reinterpret_cast<uint32_t*>(sVn + swz<BV>(row, col)) = pack_bf16x2(u0.x - X[nt][0], u0.y - X[nt][1]);
        *reinterpret_cast<uint32_t*>(sVn + swz<BV>(row + 8, col)) = pack_bf16x2(u1.x - X[nt][2], u1.y - X[nt][3]);
      }
    }
    __syncthreads();  // sVn complete

    // S = diag(2^G_last) S + kg^T . bf16(v_new)
    {
      const float* el = sEl(st);
      const float e0 = el[r0], e1 = el[r0 + 8];
#pragma unroll
      for (int nt = 0; nt < Cfg::kNT; ++nt) {
        S[nt][0] *= e0;
        S[nt][1] *= e0;
        S[nt][2] *= e1;
        S[nt][3] *= e1;
      }
      const __nv_bfloat16* kg = sKG(st);
#pragma unroll
      for (int ks = 0; ks < kTile / 16; ++ks) {
        // A = kg^T: rows = key channels, k = tokens; kg is stored [token][channel]
        const int tok = 16 * ks + (lane & 7) + 8 * (lane >> 4);
        const int chn = warp * 16 + 8 * ((lane >> 3) & 1);
        uint32_t a[4];
        ldsm_x4_t(a, smem_u32(kg + pswz(tok, chn)));
#pragma unroll
        for (int np = 0; np < Cfg::kNT; np += 2) {
          uint32_t b[4];
          ldsm_x4_t(b, smem_u32(sVn + swz<BV>(16 * ks + (lane & 15), 8 * np + 8 * (lane >> 4))));
          uint32_t b0[2] = {b[0], b[1]}, b1[2] = {b[2], b[3]};
          mma_bf16_16816(S[np], a, b0);
          mma_bf16_16816(S[np + 1], a, b1);
        }
      }
    }
  }
  if (!ok) {
    // a bulk copy never completed: flag it and leave the state untouched
    if (tid == 0) atomicOr(&p.hdr->status, 4);
    return;
  }

  // ---- final state ----
  if (out_slot < 0) return;
#pragma unroll
  for (int nt = 0; nt < Cfg::kNT; ++nt) {
    const int col = v0 + 8 * nt + 2 * t;
    *reinterpret_cast<float2*>(p.ht + out_off + (int64_t)r0 * D + col) = make_float2(S[nt][0], S[nt][1]);
    *reinterpret_cast<float2*>(p.ht + out_off + (int64_t)(r0 + 8) * D + col) = make_float2(S[nt][2], S[nt][3]);
  }
}

}  // namespace memt
