// GDN-2 inter-chunk state scan on tcgen05 tensor cores, d = 256: one CTA per (sample, head,
// 128-value half), so N x H x 2 CTAs of one per SM run in a single wave.
//
// The recurrence of scan_tc.cuh (_fwd_h_kernel, models/qwen/ops/_triton/state.py:31-115 and
// models/deepseek/ops/_triton/state.py:11-93), for every chunk of the sample in order:
//     v_new = u - w . bf16(S)                         (state.py:95-98)
//     S     = diag(2^G_last) S + kg^T . bf16(v_new)   (state.py:101-112)
// restricted to this CTA's 128 value columns (the recurrence never mixes value columns):
//     X^T = bf16(S)^T . w^T   M = 128 values, N = 64 tokens, K = 256 keys   (16 MMAs, TMEM 256..319)
//     P   = kg^T . v_new      two M = 128 key halves, N = 128 values, K = 64 tokens
//                                                                         (2 x 4 MMAs, TMEM 0..255)
// Sixteen warps hold the fp32 state (thread = key row 32 (w % 8) + lane, values 64 (w / 8) .. + 63
// of the half: 64 registers), fold P into it, and write bf16(S)^T and bf16(u - X) into the operand
// tiles of the next MMA, handing each over with one mbarrier arrival per warp. Warp 0 also issues
// the MMAs and the bulk copies (one elected lane), at the points of its own chunk step where it
// waits anyway: a seventeenth, control-only warp would cost every thread its registers (the CTA's
// register share is taken per four warps).
// Shared memory (193 KB): w of two chunks (a two-deep ring: w(c + 1) streams in while chunk c
// runs), kg + 2^G_last + this half's u of one chunk (refilled as soon as the P MMAs of the
// previous chunk have completed, which is also after every worker has read that chunk's u and
// 2^G_last), bf16(S)^T (two 64-value panels of 256 key rows) and v_new.
// Every wait is bounded: a thread whose wait runs out flags the workspace header and stops
// waiting; the CTA then frees its tensor memory and leaves the final state untouched.
#pragma once

#include "common.cuh"
#include "tc.cuh"

namespace memt {

struct ScanTc256Cfg {
  static constexpr int D = 256, VH = 128;  // keys, values per CTA
  static constexpr int kWorkerWarps = 16;
  static constexpr int kThreads = kWorkerWarps * 32;  // warp 0 also issues the MMAs and copies
  static constexpr uint32_t kBytesWK = uint32_t(kTile) * D * 2;   // 32 KB: w or kg of a chunk (4 key panels)
  static constexpr uint32_t kBytesU = uint32_t(kTile) * VH * 2;   // 16 KB: u of this half (2 value panels)
  static constexpr uint32_t kBytesEl = D * 4;                     // 2^G_last per key
  static constexpr uint32_t kOffW = 0;                            // w ring: 2 x 32 KB
  static constexpr uint32_t kOffKG = 2 * kBytesWK;
  static constexpr uint32_t kOffEl = kOffKG + kBytesWK;           // 1 KB
  static constexpr uint32_t kOffU = kOffEl + 1024;
  static constexpr uint32_t kOffSb = kOffU + kBytesU;             // bf16(S)^T: 2 panels x [256 keys][64 values]
  static constexpr uint32_t kBytesSbPanel = uint32_t(D) * 128;    // 32 KB
  static constexpr uint32_t kOffVn = kOffSb + 2 * kBytesSbPanel;  // v_new: [128 values][64 tokens]
  static constexpr uint32_t kOffBar = kOffVn + uint32_t(VH) * 128;
  static constexpr size_t kSmem = kOffBar + 256 + 1024;  // + alignment slack for the 1 KB base
  static constexpr uint32_t kTmemCols = 512;             // P0 0..127, P1 128..255, X^T 256..319
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

  // barriers: 0-1 w ring; 2 kg + 2^G_last + u landed; 3 X^T ready, 4 P ready (tcgen05.commit);
  // 5 bf16(S)^T written, 6 v_new written (one arrival per worker warp)
  constexpr int BW = 0, BKU = 2, BX = 3, BP = 4, BSB = 5, BVN = 6;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + Cfg::kOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + Cfg::kOffBar + 128);
  auto B = [&](int i) { return smem_u32(&bar[i]); };
  const uint32_t s_base = smem_u32(sm);
  auto st_w = [&](int st) { return s_base + Cfg::kOffW + st * Cfg::kBytesWK; };
  const uint32_t s_kg = s_base + Cfg::kOffKG;
  const float* s_el = reinterpret_cast<const float*>(sm + Cfg::kOffEl);
  const unsigned char* s_u = sm + Cfg::kOffU;
  unsigned char* sSb = sm + Cfg::kOffSb;
  unsigned char* sVn = sm + Cfg::kOffVn;

  if (tid == 0) {
    for (int i = 0; i < 5; ++i) mbar_init(B(i), 1);
    mbar_init(B(BSB), Cfg::kWorkerWarps);
    mbar_init(B(BVN), Cfg::kWorkerWarps);
    mbar_fence_init();
  }
  if (warp == 0) tc::alloc(smem_u32(tmem_slot), Cfg::kTmemCols);
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tP = tmem, tX = tmem + 256;
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
  // key row and 64-value slice of the half
  const int kq = warp & 7, vq = (warp >> 3) & 1;
  const int key = 32 * kq + lane;
  const int64_t row_off = (int64_t)key * D + VH * vhalf + 64 * vq;
  const int64_t in_off = (in_slot * p.H + h) * D * D + row_off, out_off = (out_slot * p.H + h) * D * D + row_off;

  // ---- issue side (warp 0, one elected lane) ----
  const bool issuer = warp == 0;
  auto load_w = [&](int c, int st) {
    const int64_t ch = (int64_t)c * p.H + h;
    mbar_expect_tx(B(BW + st), Cfg::kBytesWK);
    bulk_g2s(st_w(st), p.W + ch * kTile * D, Cfg::kBytesWK, B(BW + st));
  };
  auto load_kgu = [&](int c) {
    const int64_t ch = (int64_t)c * p.H + h;
    mbar_expect_tx(B(BKU), Cfg::kBytesWK + Cfg::kBytesEl + Cfg::kBytesU);
    bulk_g2s(s_kg, p.KG + ch * kTile * D, Cfg::kBytesWK, B(BKU));
    bulk_g2s(smem_u32(s_el), p.Elast + ch * D, Cfg::kBytesEl, B(BKU));
    bulk_g2s(smem_u32(s_u), p.U + ch * kTile * D + (int64_t)vhalf * 2 * kTile * 64, Cfg::kBytesU, B(BKU));
  };
  constexpr uint32_t kIdX = tc::idesc(tc::kBF16, 128, 64, true, false);   // Sb^T MN-major, w K-major
  constexpr uint32_t kIdP = tc::idesc(tc::kBF16, 128, 128, true, false);  // kg^T MN-major, v_new K-major
  const uint32_t sb = smem_u32(sSb), vn = smem_u32(sVn);
  if (issuer) {
    if (tc::elect_one()) {
      if (nchunks > 0) {
        load_w(c0, 0);
        load_kgu(c0);
      }
      if (nchunks > 1) load_w(c0 + 1, 1);
    }
    __syncwarp();
  }

  float S[64];
#pragma unroll
  for (int j = 0; j < 64; j += 4) {  // zero state for an input slot outside the pool
    const float4 v = in_slot >= 0 ? *reinterpret_cast<const float4*>(p.h0 + in_off + j) : make_float4(0.f, 0.f, 0.f, 0.f);
    S[j] = v.x;
    S[j + 1] = v.y;
    S[j + 2] = v.z;
    S[j + 3] = v.w;
  }
  float el = 1.f;  // 2^G_last of the previous chunk for this key row
  const int kh = kq >> 2;  // key half: P accumulator, lanes 32 (warp % 4) ..
  auto update_state = [&]() {  // S = 2^G_last S + P, 16 columns at a time (register pressure)
    tc::fence_after();
    const uint64_t e2 = f32x2_splat(el);
#pragma unroll
    for (int q4 = 0; q4 < 4; ++q4) {
      float P0[16];
      tc::ld16(tc::lane_addr(tP + 128 * kh, 32 * (warp & 3), 64 * vq + 16 * q4), P0);
#pragma unroll
      for (int j = 0; j < 16; j += 2) {
        const uint64_t a = fma_f32x2(e2, f32x2_pack(S[16 * q4 + j], S[16 * q4 + j + 1]), f32x2_pack(P0[j], P0[j + 1]));
        S[16 * q4 + j] = f32x2_lo(a);
        S[16 * q4 + j + 1] = f32x2_hi(a);
      }
    }
  };
  auto hand_over = [&](int b) {  // operand tile written: make it visible to the tensor cores
    tc::fence_smem_async();
    tc::fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(B(b));
  };
  const int vr = 32 * (warp & 3) + lane;  // value row of X^T and v_new (of this half)
  const int t0 = 16 * (warp >> 2);        // first token of this thread's v_new columns
  for (int it = 0; it < nchunks; ++it) {
    const int st = it & 1;
    const uint32_t ph = it & 1;
    // ---- previous chunk's P into the state; bf16(S) -> Sb^T (MN-major, panel = value quarter vq) ----
    if (it > 0) {
      wait(BP, ph ^ 1);
      update_state();
      // P of the previous chunk done: its kg, 2^G_last and u were read (before v_new was handed
      // over), so they are refilled with this chunk's
      if (issuer) {
        if (__all_sync(~0u, alive) && tc::elect_one()) load_kgu(c0 + it);
        __syncwarp();
      }
    }
    {
      unsigned char* row = sSb + vq * Cfg::kBytesSbPanel + (key >> 3) * 1024 + (key & 7) * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint4 pk;
        pk.x = pack_bf16x2(S[8 * c], S[8 * c + 1]);
        pk.y = pack_bf16x2(S[8 * c + 2], S[8 * c + 3]);
        pk.z = pack_bf16x2(S[8 * c + 4], S[8 * c + 5]);
        pk.w = pack_bf16x2(S[8 * c + 6], S[8 * c + 7]);
        *reinterpret_cast<uint4*>(row + ((c ^ (key & 7)) << 4)) = pk;
      }
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
          tc::mma_bf16(tX, tc::desc_mnmajor(sb, Cfg::kBytesSbPanel, ks),
                       tc::desc_kmajor(w + (ks >> 2) * (kTile * 128), (ks & 3) * 32), kIdX, ks > 0);
        tc::commit(B(BX));
        // the other w stage held chunk it - 1, whose X^T completed before its P (waited above)
        if (it >= 1 && it + 1 < nchunks) load_w(c0 + it + 1, st ^ 1);
      }
      __syncwarp();
    }
    // ---- v_new = bf16(u - X) -> K-major operand [value row][64 tokens] ----
    wait(BKU, ph);
    el = s_el[key];
    float uv[16];
    {
      const unsigned char* u = s_u + (vr >> 6) * (kTile * 128);  // value panel of u
      const int vc = (vr & 63) >> 3, vb = (vr & 7) * 2;
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const int t = t0 + e;
        uv[e] = __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(u + t * 128 + ((vc ^ (t & 7)) << 4) + vb));
      }
    }
    wait(BX, ph);
    tc::fence_after();
    {
      float X[16];
      tc::ld16(tc::lane_addr(tX, 32 * (warp & 3), t0), X);  // value vr, tokens t0 ..
      unsigned char* vrow = sVn + (vr >> 3) * 1024 + (vr & 7) * 128;
      auto vnew = [&](int e) {  // bf16(u - X) of columns e, e + 1
        return f32x2_to_bf16x2(sub_f32x2(f32x2_pack(uv[e], uv[e + 1]), f32x2_pack(X[e], X[e + 1])));
      };
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint4 pk;
        pk.x = vnew(8 * c);
        pk.y = vnew(8 * c + 2);
        pk.z = vnew(8 * c + 4);
        pk.w = vnew(8 * c + 6);
        *reinterpret_cast<uint4*>(vrow + ((((t0 >> 3) + c) ^ (vr & 7)) << 4)) = pk;
      }
    }
    hand_over(BVN);
    if (issuer) {  // P once every warp's v_new is in place (kg of this chunk landed: waited above)
      wait(BVN, ph);
      tc::fence_after();
      if (__all_sync(~0u, alive) && tc::elect_one()) {
#pragma unroll
        for (int kh2 = 0; kh2 < 2; ++kh2)
#pragma unroll
          for (int ks = 0; ks < kTile / 16; ++ks)
            tc::mma_bf16(tP + 128 * kh2, tc::desc_mnmajor(s_kg + kh2 * 2 * (kTile * 128), kTile * 128, ks),
                         tc::desc_kmajor(vn, ks * 32), kIdP, ks > 0);
        tc::commit(B(BP));
      }
      __syncwarp();
    }
  }
  if (nchunks > 0) {
    wait(BP, (nchunks - 1) & 1);
    update_state();
  }
  // a wait that ran out anywhere in the CTA: leave the final state untouched
  const bool ok = __syncthreads_and(alive) != 0;
  if (ok && out_slot >= 0) {
#pragma unroll
    for (int j = 0; j < 64; j += 4)
      *reinterpret_cast<float4*>(p.ht + out_off + j) = make_float4(S[j], S[j + 1], S[j + 2], S[j + 3]);
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 0) tc::dealloc(tmem, Cfg::kTmemCols);
}

}  // namespace memt
