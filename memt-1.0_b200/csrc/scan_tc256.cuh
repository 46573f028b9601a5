// GDN-2 inter-chunk state scan on tcgen05 tensor cores, d = 256: one CTA per (sample, head,
// 128-value half), so N x H x 2 CTAs of one per SM run in a single wave.
//
// The recurrence of scan_tc.cuh (_fwd_h_kernel, models/qwen/ops/_triton/state.py:31-115 and
// models/deepseek/ops/_triton/state.py:11-93), for every chunk of the sample in order:
//     v_new = u - w . bf16(S)                         (state.py:95-98)
//     S     = diag(2^G_last) S + kg^T . bf16(v_new)   (state.py:101-112)
// restricted to this CTA's 128 value columns (the recurrence never mixes value columns), and
// computed transposed so that the value index is the tensor-memory lane throughout:
//     X^T = bf16(S)^T . w^T    M = 128 values, N = 64 tokens, K = 256 keys   (16 MMAs)
//     P^T = bf16(v_new)^T . kg M = 128 values, N = 256 keys, K = 64 tokens   (4 MMAs)
// Both A operands, bf16(S)^T and bf16(v_new)^T, are written by the threads straight into tensor
// memory (tcgen05.st), so the state never passes through shared memory; w (K-major) and kg
// (MN-major) come from shared memory as the intra kernel wrote them.
// Tensor memory (512 columns): P^T 0..255, X^T 256..319, bf16(S)^T 320..447 (two keys per
// column), bf16(v_new)^T 448..479.
// Sixteen warps hold the fp32 state transposed: warp w, lane l owns value row 32 (w % 4) + l of
// the half and keys 64 (w / 4) .. + 63 (64 registers); it folds its slice of P^T in, writes its
// slice of bf16(S)^T, and later the 16 tokens 16 (w / 4) .. of its value row of bf16(v_new)^T,
// handing each over with one mbarrier arrival per warp. Warp 0 also issues the MMAs and the bulk
// copies (one elected lane) at points of its own chunk step where it waits anyway.
// Shared memory (163 KB): w of two chunks (w(c + 2) is issued once the X^T MMAs of chunk c have
// completed), kg + this half's u + 2^G_last of two chunks (kg(c + 1) is issued with the X^T MMAs of
// chunk c, once every thread has folded chunk c - 1 into its state).
// Every wait is bounded: a thread whose wait runs out flags the workspace header and stops
// waiting, warp 0 issues nothing more, and the CTA frees its tensor memory and leaves the final
// state untouched.
#pragma once

#include "common.cuh"
#include "tc.cuh"

namespace memt {

struct ScanTc256Cfg {
  static constexpr int D = 256, VH = 128;  // keys, values per CTA
  static constexpr int kWarps = 16;
  static constexpr int kThreads = kWarps * 32;
  static constexpr uint32_t kBytesWK = uint32_t(kTile) * D * 2;  // 32 KB: w or kg of a chunk (4 key panels)
  static constexpr uint32_t kBytesU = uint32_t(kTile) * VH * 2;  // 16 KB: u of this half (2 value panels)
  static constexpr uint32_t kBytesEl = D * 4;                    // 2^G_last per key
  static constexpr uint32_t kOffW = 0;                           // w: 2 x 32 KB
  static constexpr uint32_t kOffStage = 2 * kBytesWK;            // 2 stages of kg, u, 2^G_last
  static constexpr uint32_t kStageKG = 0, kStageU = kBytesWK, kStageEl = kBytesWK + kBytesU;
  static constexpr uint32_t kStageStride = kBytesWK + kBytesU + 1024;  // 49 KB, 1 KB aligned
  static constexpr uint32_t kOffBar = kOffStage + 2 * kStageStride;
  static constexpr size_t kSmem = kOffBar + 256 + 1024;  // + alignment slack for the 1 KB base
  static constexpr uint32_t kTmemCols = 512;
  static constexpr uint32_t kColP = 0, kColX = 256, kColSb = 320, kColVn = 448;
  static_assert(kColVn + kTile / 2 <= kTmemCols, "tensor-memory plan");
  static_assert(kSmem <= 227 * 1024, "one CTA per SM");
};

__global__ void __launch_bounds__(ScanTc256Cfg::kThreads, 1) scan_tc256_kernel(ScanParams p) {
  using Cfg = ScanTc256Cfg;
  constexpr int D = Cfg::D, VH = Cfg::VH;
  extern __shared__ __align__(1024) unsigned char smem_scan256[];
  unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_scan256) + 1023) &
                                                       ~static_cast<uintptr_t>(1023));
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int vhalf = blockIdx.x & 1;
  const int nh = blockIdx.x >> 1;
  const int h = nh % p.H, n = nh / p.H;

  // barriers: 0-1 w stages, 2-3 kg + u + 2^G_last stages landed; 4 X^T ready, 5 P^T ready
  // (tcgen05.commit); 6 bf16(S)^T written, 7 bf16(v_new)^T written (one arrival per warp)
  constexpr int BW = 0, BKU = 2, BX = 4, BP = 5, BSB = 6, BVN = 7;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + Cfg::kOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + Cfg::kOffBar + 128);
  auto B = [&](int i) { return smem_u32(&bar[i]); };
  const uint32_t s_base = smem_u32(sm);
  auto st_w = [&](int st) { return s_base + Cfg::kOffW + st * Cfg::kBytesWK; };
  auto stage = [&](int st) { return sm + Cfg::kOffStage + st * Cfg::kStageStride; };

  if (tid == 0) {
    for (int i = 0; i < 6; ++i) mbar_init(B(i), 1);
    mbar_init(B(BSB), Cfg::kWarps);
    mbar_init(B(BVN), Cfg::kWarps);
    mbar_fence_init();
  }
  if (warp == 0) tc::alloc(smem_u32(tmem_slot), Cfg::kTmemCols);
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tP = tmem + Cfg::kColP, tX = tmem + Cfg::kColX, tSb = tmem + Cfg::kColSb, tVn = tmem + Cfg::kColVn;
  griddep_wait();  // the intra kernel's tiles and the chunk offsets are complete
  griddep_launch_dependents();
  const int c0 = p.sample_off[n], c1 = p.sample_off[n + 1];
  const int nchunks = c1 - c0;

  bool alive = true;
  auto wait = [&](int b, uint32_t parity) {
    if (alive && !mbar_wait(B(b), parity)) {
      alive = false;
      atomicOr(&p.hdr->status, 4);
    }
  };

  const int64_t in_slot = pool_slot(p.slots_in, p.num_in, n), out_slot = pool_slot(p.slots_out, p.num_out, n);
  if (tid == 0 && vhalf == 0 && (in_slot < 0 || out_slot < 0)) atomicOr(&p.hdr->status, 8);
  const int quad = warp & 3, kq = warp >> 2;  // lane quadrant; key quarter (and token block of v_new)
  const int vr = 32 * quad + lane;            // value row of this half
  const int key0 = 64 * kq;
  // element (key0 + j, value) of the state lies j * D floats after this offset
  const int64_t col_off = (int64_t)key0 * D + VH * vhalf + vr;
  const int64_t in_off = (in_slot * p.H + h) * D * D + col_off, out_off = (out_slot * p.H + h) * D * D + col_off;

  // ---- issue side (warp 0, one elected lane) ----
  const bool issuer = warp == 0;
  auto load_w = [&](int c, int st) {
    const int64_t ch = (int64_t)c * p.H + h;
    mbar_expect_tx(B(BW + st), Cfg::kBytesWK);
    bulk_g2s(st_w(st), p.W + ch * kTile * D, Cfg::kBytesWK, B(BW + st));
  };
  auto load_kgu = [&](int c, int st) {
    const int64_t ch = (int64_t)c * p.H + h;
    const uint32_t sg = smem_u32(stage(st));
    mbar_expect_tx(B(BKU + st), Cfg::kBytesWK + Cfg::kBytesEl + Cfg::kBytesU);
    bulk_g2s(sg + Cfg::kStageKG, p.KG + ch * kTile * D, Cfg::kBytesWK, B(BKU + st));
    bulk_g2s(sg + Cfg::kStageEl, p.Elast + ch * D, Cfg::kBytesEl, B(BKU + st));
    bulk_g2s(sg + Cfg::kStageU, p.U + ch * kTile * D + (int64_t)vhalf * 2 * kTile * 64, Cfg::kBytesU, B(BKU + st));
  };
  constexpr uint32_t kIdX = tc::idesc(tc::kBF16, 128, 64, false, false);  // Sb^T in TMEM, w K-major
  constexpr uint32_t kIdP = tc::idesc(tc::kBF16, 128, 256, false, true);  // v_new^T in TMEM, kg MN-major
  if (issuer) {
    if (tc::elect_one()) {
      if (nchunks > 0) {
        load_w(c0, 0);
        load_kgu(c0, 0);
      }
      if (nchunks > 1) load_w(c0 + 1, 1);
    }
    __syncwarp();
  }

  float S[64];  // S[key0 + j][value vr]; zero state for an input slot outside the pool
#pragma unroll
  for (int j = 0; j < 64; ++j) S[j] = in_slot >= 0 ? p.h0[in_off + (int64_t)j * D] : 0.f;

  // S = 2^G_last S + P^T (16 keys at a time: register pressure); 2^G_last of the chunk in stage st
  auto update_state = [&](int st) {
    tc::fence_after();
    const float* el = reinterpret_cast<const float*>(stage(st) + Cfg::kStageEl) + key0;
#pragma unroll
    for (int q4 = 0; q4 < 4; ++q4) {
      float P0[16];
      tc::ld16(tc::lane_addr(tP, 32 * quad, key0 + 16 * q4), P0);
#pragma unroll
      for (int j = 0; j < 16; j += 4) {
        const float4 e = *reinterpret_cast<const float4*>(el + 16 * q4 + j);  // same address across the warp
        const int i = 16 * q4 + j;
        const uint64_t a = fma_f32x2(f32x2_pack(e.x, e.y), f32x2_pack(S[i], S[i + 1]), f32x2_pack(P0[j], P0[j + 1]));
        const uint64_t b =
            fma_f32x2(f32x2_pack(e.z, e.w), f32x2_pack(S[i + 2], S[i + 3]), f32x2_pack(P0[j + 2], P0[j + 3]));
        S[i] = f32x2_lo(a);
        S[i + 1] = f32x2_hi(a);
        S[i + 2] = f32x2_lo(b);
        S[i + 3] = f32x2_hi(b);
      }
    }
  };
  auto hand_over = [&](int b) {  // tensor-memory operand written: make it visible to the MMA issue
    tc::wait_st();
    tc::fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(B(b));
  };
  const int t0 = 16 * kq;  // first token of this thread's v_new columns
  for (int it = 0; it < nchunks; ++it) {
    const int st = it & 1;
    const uint32_t ph = it & 1;
    // ---- previous chunk's P^T into the state; bf16(S)^T -> tensor memory ----
    if (it > 0) {
      wait(BP, ph ^ 1);
      update_state(st ^ 1);
    }
#pragma unroll
    for (int q4 = 0; q4 < 4; ++q4) {
      uint32_t r[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) r[c] = pack_bf16x2(S[16 * q4 + 2 * c], S[16 * q4 + 2 * c + 1]);
      tc::st8(tc::lane_addr(tSb, 32 * quad, key0 / 2 + 8 * q4), r);
    }
    hand_over(BSB);
    if (issuer) {  // X^T once every warp's bf16(S)^T and this chunk's w are in place
      wait(BW + st, (it >> 1) & 1);
      wait(BSB, ph);
      tc::fence_after();
      if (__all_sync(~0u, alive) && tc::elect_one()) {  // nothing more is issued after a wait ran out
        const uint32_t w = st_w(st);
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks)
          tc::mma_bf16_ts(tX, tSb + 8 * ks, tc::desc_kmajor(w + (ks >> 2) * (kTile * 128), (ks & 3) * 32), kIdX,
                          ks > 0);
        tc::commit(B(BX));
        // every thread has folded chunk it - 1 (BSB) and its P^T completed: the stage that held
        // chunk it - 1 takes chunk it + 1
        if (it + 1 < nchunks) load_kgu(c0 + it + 1, st ^ 1);
      }
      __syncwarp();
    }
    // ---- bf16(v_new)^T = bf16(u - X)^T -> tensor memory ----
    const unsigned char* sg = stage(st);
    wait(BKU + st, (it >> 1) & 1);
    float uv[16];
    {
      const unsigned char* u = sg + Cfg::kStageU + (vr >> 6) * (kTile * 128);  // value panel of u
      const int vc = (vr & 63) >> 3, vb = (vr & 7) * 2;
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const int t = t0 + e;
        uv[e] = __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(u + t * 128 + ((vc ^ (t & 7)) << 4) + vb));
      }
    }
    wait(BX, ph);
    tc::fence_after();
    if (issuer) {  // X^T of this chunk complete: its w stage takes chunk it + 2
      if (it + 2 < nchunks && __all_sync(~0u, alive) && tc::elect_one()) load_w(c0 + it + 2, st);
      __syncwarp();
    }
    {
      float X[16];
      tc::ld16(tc::lane_addr(tX, 32 * quad, t0), X);  // value vr, tokens t0 ..
      uint32_t r[8];
#pragma unroll
      for (int e = 0; e < 16; e += 2)
        r[e / 2] = f32x2_to_bf16x2(sub_f32x2(f32x2_pack(uv[e], uv[e + 1]), f32x2_pack(X[e], X[e + 1])));
      tc::st8(tc::lane_addr(tVn, 32 * quad, t0 / 2), r);
    }
    hand_over(BVN);
    if (issuer) {  // P^T once every warp's v_new is in place (kg of this chunk landed: waited above)
      wait(BVN, ph);
      tc::fence_after();
      if (__all_sync(~0u, alive) && tc::elect_one()) {
        const uint32_t kg = smem_u32(sg) + Cfg::kStageKG;
#pragma unroll
        for (int ks = 0; ks < kTile / 16; ++ks)
          tc::mma_bf16_ts(tP, tVn + 8 * ks, tc::desc_mnmajor(kg, kTile * 128, ks), kIdP, ks > 0);
        tc::commit(B(BP));
      }
      __syncwarp();
    }
  }
  if (nchunks > 0) {
    wait(BP, (nchunks - 1) & 1);
    update_state((nchunks - 1) & 1);
  }
  // a wait that ran out anywhere in the CTA: leave the final state untouched
  const bool ok = __syncthreads_and(alive) != 0;
  if (ok && out_slot >= 0) {
#pragma unroll
    for (int j = 0; j < 64; ++j) p.ht[out_off + (int64_t)j * D] = S[j];
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 0) tc::dealloc(tmem, Cfg::kTmemCols);
}

}  // namespace memt
