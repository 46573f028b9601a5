// GDN-2 inter-chunk state scan on tcgen05 tensor cores, d = 256: one CTA per (sample, head,
// 128-value block), so N x H x 2 CTAs of one per SM.
//
// The recurrence of scan_tc.cuh (_fwd_h_kernel, models/qwen/ops/_triton/state.py:31-115 and
// models/deepseek/ops/_triton/state.py:11-93), for every chunk of the sample in order:
//     v_new = u - w . bf16(S)                         (state.py:95-98)
//     S     = diag(2^G_last) S + kg^T . bf16(v_new)   (state.py:101-112)
// restricted to this CTA's 128 value columns (the recurrence never mixes value columns). The
// chunks of a sample form a dependent chain, so the kernel minimises the latency of one chunk
// step. Everything is computed transposed, so that the value index is the tensor-memory lane:
//     X^T = bf16(S)^T . w^T     M = 128 values, N = 64 tokens, K = 256 keys  (16 MMAs)
//     P^T = bf16(v_new)^T . kg  M = 128 values, N = 256 keys, K = 64 tokens  (4 MMAs)
// Both A operands are written by the threads straight into tensor memory (tcgen05.st), so no
// operand passes through shared memory; w (K-major) and kg (MN-major) come from shared memory in
// the layout the intra kernel stored them (pswz). At d = 256 this is what the chain step is made
// of: the key-major form of scan_tc.cuh would write a 64 KB bf16(S)^T tile to shared memory and
// read it back into 16 MMAs every chunk (the d = 128 chain, with half of that, is faster in the
// key-major form: 0.186 against 0.218 ms for the config-1 scan on a B200).
// The fp32 state is held transposed in registers: warp w, lane l owns value row 32 (w % 4) + l and
// keys 64 (w / 4) .. + 63 (64 registers), 16 warps. A thread folds its 64 columns of P^T into the
// state (S = 2^G_last S + P) and writes bf16(S)^T of its keys into the first 32 of those same
// columns (already read: the K step of 16 keys 16 ks .. lies at column 64 (ks / 4) + 8 (ks % 4)).
// Likewise it reads its 16-token block of X^T and writes bf16(u - X)^T over the first half of
// that block. So tensor memory needs 320 columns: P^T 0..255, X^T 256..319.
// Warp 0 also issues the MMAs and the bulk copies (one elected lane), at points of its own chunk
// step where it waits anyway; handovers are one mbarrier arrival per warp.
// w, kg, this block's u and 2^G_last of chunk c + 2 stream into a two-deep ring by bulk copies
// (163 KB of shared memory), issued once every thread has folded chunk c into its state.
// Every wait is bounded: a thread whose wait runs out flags the workspace header and stops
// waiting, warp 0 issues nothing more, and the CTA frees its tensor memory and leaves the final
// state untouched.
#pragma once

#include "common.cuh"
#include "tc.cuh"

namespace memt {

struct ScanTc256Cfg {
  static constexpr int D = 256, VH = 128;  // keys, values per CTA
  static constexpr int kBlocks = D / VH;  // CTAs per (sample, head)
  static constexpr int kKeyQ = D / 64;    // key blocks of 64 per value row
  static constexpr int kWarps = 4 * kKeyQ;
  static constexpr int kThreads = kWarps * 32;
  static constexpr int kTokBlock = kTile / kKeyQ;                 // v_new tokens per thread
  static constexpr int kStages = 2;  // operand ring depth
  static constexpr uint32_t kBytesWK = uint32_t(kTile) * D * 2;  // w or kg of a chunk (D/64 key panels)
  static constexpr uint32_t kBytesU = uint32_t(kTile) * VH * 2;  // 16 KB: u of this value block (2 panels)
  static constexpr uint32_t kBytesEl = D * 4;                    // 2^G_last per key
  static constexpr uint32_t kStageW = 0, kStageKG = kBytesWK, kStageU = 2 * kBytesWK, kStageEl = 2 * kBytesWK + kBytesU;
  static constexpr uint32_t kStageStride = 2 * kBytesWK + kBytesU + 1024;  // 1 KB aligned
  static constexpr uint32_t kOffBar = kStages * kStageStride;
  static constexpr size_t kSmem = kOffBar + 256 + 1024;  // + alignment slack for the 1 KB base
  static constexpr uint32_t kColP = 0, kColX = D;
  static constexpr uint32_t kTmemCols = 512;
  static_assert(kBytesEl <= 1024, "2^G_last slot");
  static_assert(kSmem <= 227 * 1024, "one CTA per SM");
};

__global__ void __launch_bounds__(ScanTc256Cfg::kThreads, 1) scan_tc256_kernel(ScanParams p) {
  using Cfg = ScanTc256Cfg;
  constexpr int D = Cfg::D, VH = Cfg::VH, TB = Cfg::kTokBlock;
  extern __shared__ __align__(1024) unsigned char smem_scan256[];
  unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_scan256) + 1023) &
                                                       ~static_cast<uintptr_t>(1023));
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int vblk = blockIdx.x % Cfg::kBlocks;
  const int nh = blockIdx.x / Cfg::kBlocks;
  const int h = nh % p.H, n = nh / p.H;

  // barriers: 0-1 stages landed; 2 X^T ready, 3 P^T ready (tcgen05.commit);
  // 4 bf16(S)^T written, 5 bf16(v_new)^T written (one arrival per warp)
  constexpr int BS = 0, BX = Cfg::kStages, BP = BX + 1, BSB = BX + 2, BVN = BX + 3;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + Cfg::kOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + Cfg::kOffBar + 128);
  auto B = [&](int i) { return smem_u32(&bar[i]); };
  auto stage = [&](int st) { return sm + st * Cfg::kStageStride; };

  if (tid == 0) {
    for (int i = 0; i < BSB; ++i) mbar_init(B(i), 1);
    mbar_init(B(BSB), Cfg::kWarps);
    mbar_init(B(BVN), Cfg::kWarps);
    mbar_fence_init();
  }
  if (warp == 0) tc::alloc(smem_u32(tmem_slot), Cfg::kTmemCols);
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tP = tmem + Cfg::kColP, tX = tmem + Cfg::kColX;
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
  if (tid == 0 && vblk == 0 && (in_slot < 0 || out_slot < 0)) atomicOr(&p.hdr->status, 8);
  const int quad = warp & 3, kq = warp >> 2;  // lane quadrant; key block (and token block of v_new)
  const int vr = 32 * quad + lane;            // value row of this block
  const int key0 = 64 * kq;
  // element (key0 + j, value) of the state lies j * D floats after this offset
  const int64_t col_off = (int64_t)key0 * D + VH * vblk + vr;
  const int64_t in_off = (in_slot * p.H + h) * D * D + col_off, out_off = (out_slot * p.H + h) * D * D + col_off;

  // ---- issue side (warp 0, one elected lane) ----
  const bool issuer = warp == 0;
  auto load = [&](int c, int st) {
    const int64_t ch = (int64_t)c * p.H + h;
    const uint32_t sg = smem_u32(stage(st));
    mbar_expect_tx(B(BS + st), 2 * Cfg::kBytesWK + Cfg::kBytesEl + Cfg::kBytesU);
    bulk_g2s(sg + Cfg::kStageW, p.W + ch * kTile * D, Cfg::kBytesWK, B(BS + st));
    bulk_g2s(sg + Cfg::kStageKG, p.KG + ch * kTile * D, Cfg::kBytesWK, B(BS + st));
    bulk_g2s(sg + Cfg::kStageEl, p.Elast + ch * D, Cfg::kBytesEl, B(BS + st));
    bulk_g2s(sg + Cfg::kStageU, p.U + ch * kTile * D + (int64_t)vblk * 2 * kTile * 64, Cfg::kBytesU, B(BS + st));
  };
  constexpr uint32_t kIdX = tc::idesc(tc::kBF16, 128, 64, false, false);  // Sb^T in TMEM, w K-major
  constexpr uint32_t kIdP = tc::idesc(tc::kBF16, 128, D, false, true);    // v_new^T in TMEM, kg MN-major
  if (issuer) {
    if (tc::elect_one())
      for (int i = 0; i < Cfg::kStages && i < nchunks; ++i) load(c0 + i, i);
    __syncwarp();
  }

  float S[64];  // S[key0 + j][value vr]; zero state for an input slot outside the pool
#pragma unroll
  for (int j = 0; j < 64; ++j) S[j] = in_slot >= 0 ? p.h0[in_off + (int64_t)j * D] : 0.f;

  // S = 2^G_last S + P^T, 16 keys at a time (register pressure), 2^G_last of the chunk in stage st;
  // with SB, bf16(S)^T of those keys goes over P^T columns this thread has already read
  auto fold = [&](int i, const float4& e, const float* P4, uint32_t* r2) {  // keys i .. i + 3
    const uint64_t a = fma_f32x2(f32x2_pack(e.x, e.y), f32x2_pack(S[i], S[i + 1]), f32x2_pack(P4[0], P4[1]));
    const uint64_t b = fma_f32x2(f32x2_pack(e.z, e.w), f32x2_pack(S[i + 2], S[i + 3]), f32x2_pack(P4[2], P4[3]));
    S[i] = f32x2_lo(a);
    S[i + 1] = f32x2_hi(a);
    S[i + 2] = f32x2_lo(b);
    S[i + 3] = f32x2_hi(b);
    r2[0] = f32x2_to_bf16x2(a);
    r2[1] = f32x2_to_bf16x2(b);
  };
  auto update_state = [&](int st, bool sb) {
    tc::fence_after();
    const float4* el = reinterpret_cast<const float4*>(stage(st) + Cfg::kStageEl) + key0 / 4;
#pragma unroll
    for (int q4 = 0; q4 < 4; ++q4) {
      float P0[16];
      tc::ld16(tc::lane_addr(tP, 32 * quad, key0 + 16 * q4), P0);
      uint32_t r[8];
#pragma unroll
      for (int j = 0; j < 16; j += 4) fold(16 * q4 + j, el[(16 * q4 + j) / 4], P0 + j, r + j / 2);
      if (sb) tc::st8(tc::lane_addr(tP, 32 * quad, key0 + 8 * q4), r);
    }
  };
  auto hand_over = [&](int b) {  // tensor-memory operand written: make it visible to the MMA issue
    tc::wait_st();
    tc::fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(B(b));
  };
  const int t0 = TB * kq;  // first token of this thread's v_new block
  for (int it = 0; it < nchunks; ++it) {
    const int st = it % Cfg::kStages, prev = (it + Cfg::kStages - 1) % Cfg::kStages;
    const uint32_t ph = it & 1, sph = (it / Cfg::kStages) & 1;
    // ---- previous chunk's P^T into the state; bf16(S)^T -> tensor memory ----
    if (it > 0) {
      wait(BP, ph ^ 1);
      update_state(prev, true);
    } else {
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        uint32_t r[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) r[c] = pack_bf16x2(S[16 * q4 + 2 * c], S[16 * q4 + 2 * c + 1]);
        tc::st8(tc::lane_addr(tP, 32 * quad, key0 + 8 * q4), r);
      }
    }
    hand_over(BSB);
    const unsigned char* sg = stage(st);
    if (issuer) {  // X^T once every warp's bf16(S)^T and this chunk's operands are in place
      wait(BS + st, sph);
      wait(BSB, ph);
      tc::fence_after();
      if (__all_sync(~0u, alive) && tc::elect_one()) {  // nothing more is issued after a wait ran out
        const uint32_t w = smem_u32(sg) + Cfg::kStageW;
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks)
          tc::mma_bf16_ts(tX, tP + 64 * (ks >> 2) + 8 * (ks & 3),
                          tc::desc_kmajor(w + (ks >> 2) * (kTile * 128), (ks & 3) * 32), kIdX, ks > 0);
        tc::commit(B(BX));
        // every thread has folded chunk it - 1 (BSB) and its P^T completed: the stage that held
        // it takes chunk it + 1
        if (it >= 1 && it - 1 + Cfg::kStages < nchunks) load(c0 + it - 1 + Cfg::kStages, prev);
      }
      __syncwarp();
    }
    // ---- bf16(v_new)^T = bf16(u - X)^T -> tensor memory (over X^T columns already read) ----
    wait(BS + st, sph);
    const unsigned char* u = sg + Cfg::kStageU + (vr >> 6) * (kTile * 128);  // value panel of u
    const int vc = (vr & 63) >> 3, vb = (vr & 7) * 2;
    auto u_at = [&](int t) {
      return __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(u + t * 128 + ((vc ^ (t & 7)) << 4) + vb));
    };
    float uv[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) uv[e] = u_at(t0 + e);
    wait(BX, ph);
    tc::fence_after();
    float X[16];
    tc::ld16(tc::lane_addr(tX, 32 * quad, t0), X);  // value vr, tokens t0 ..
    uint32_t r[8];
#pragma unroll
    for (int e = 0; e < 16; e += 2)
      r[e / 2] = f32x2_to_bf16x2(sub_f32x2(f32x2_pack(uv[e], uv[e + 1]), f32x2_pack(X[e], X[e + 1])));
    tc::st8(tc::lane_addr(tX, 32 * quad, t0), r);
    hand_over(BVN);
    if (issuer) {  // P^T once every warp's v_new is in place
      wait(BVN, ph);
      tc::fence_after();
      if (__all_sync(~0u, alive) && tc::elect_one()) {
        const uint32_t kg = smem_u32(sg) + Cfg::kStageKG;
#pragma unroll
        for (int ks = 0; ks < kTile / 16; ++ks)  // tokens 16 ks .. : block 16 ks / TB, half-columns
          tc::mma_bf16_ts(tP, tX + 8 * ks + (TB / 2) * ((16 * ks) / TB), tc::desc_mnmajor(kg, kTile * 128, ks), kIdP,
                          ks > 0);
        tc::commit(B(BP));
      }
      __syncwarp();
    }
  }
  if (nchunks > 0) {
    wait(BP, (nchunks - 1) & 1);
    update_state((nchunks - 1) % Cfg::kStages, false);
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
