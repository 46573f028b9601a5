// GDN-2 inter-chunk state scan on tcgen05 tensor cores, d = 128: one CTA per (sample, head), or
// per (sample, head, 64-value half) when twice as many CTAs still fit on the SMs (VB = 2).
//
// Same recurrence as scan.cuh (_fwd_h_kernel, models/qwen/ops/_triton/state.py:31-115), for
// every chunk of the sample in order:
//     v_new = u - w . bf16(S)                         (state.py:95-98)
//     S     = diag(2^G_last) S + kg^T . bf16(v_new)   (state.py:101-112)
// The chunks of a sample form a dependent chain, so the kernel minimises the latency of one
// chunk step. A tcgen05 MMA costs about the same per K = 16 slice for any N up to 128, so both
// products use the full M = 128 shape (12 MMAs per chunk):
//     X^T = bf16(S)^T . w^T   M = 128 values, N = 64 tokens, K = 128 keys  (tensor memory 128..191)
//     P   = kg^T . v_new      M = 128 keys,   N = 128 values, K = 64 tokens (tensor memory 0..127)
// A control warp issues the MMAs and the bulk copies; eight worker warps hold the fp32 state
// in registers (thread = key row 32 (w % 4) + lane, values 64 (w / 4) .. + 63), fold P into it
// (S = 2^G_last S + P), and write bf16(S) and bf16(u - X) straight into the swizzled operand
// tiles of the next MMA, handing them over with one mbarrier arrival per warp.
// Value split (VB = 2, for few chains: the recurrence never mixes value columns): a CTA takes 64
// of the values, so X^T is an M = 64 product (value r of the block in tensor-memory lane
// 32 (r / 16) + r % 16: lanes 0-15 of each warp form v_new) and P an N = 64 one; a worker thread
// holds 32 values of its key row. The chain step has the same MMA count but half the state
// traffic per thread.
// w, kg, u of chunk c + 2 and 2^G_last stream into a three-deep ring by bulk copies (the intra
// kernel stores them in the operand layout, pswz).
// Every wait is bounded: a thread whose wait runs out flags the workspace header and stops
// waiting; the CTA then frees its tensor memory and leaves the final state untouched.
#pragma once

#include "common.cuh"
#include "tc.cuh"

namespace memt {

template <int VB>
struct ScanTcCfg {
  static constexpr int D = 128;
  static constexpr int VH = D / VB;   // values per CTA
  static constexpr int SV = VH / 2;   // values per worker thread
  static constexpr int kWorkerWarps = 8;
  static constexpr int kThreads = (kWorkerWarps + 1) * 32;  // + control warp
  static constexpr int kStages = 3;
  static constexpr uint32_t kBytesTile = uint32_t(kTile) * D * 2;  // 16 KB: w or kg of one chunk
  static constexpr uint32_t kBytesU = uint32_t(kTile) * VH * 2;    // u of this CTA's values
  static constexpr uint32_t kBytesEl = D * 4;
  static constexpr uint32_t kStageStride = 2 * kBytesTile + kBytesU + 1024;  // + 2^G_last, 1 KB aligned
  static constexpr uint32_t kBytesPanelSb = uint32_t(D) * 128;     // 64 values of the 128 key rows
  static constexpr uint32_t kOffSb = kStages * kStageStride;       // bf16(S)^T operand: VH/64 panels
  static constexpr uint32_t kOffVn = kOffSb + (VH / 64) * kBytesPanelSb;  // bf16(v_new): [VH rows][64 tokens]
  static constexpr uint32_t kOffBar = kOffVn + uint32_t(VH) * 128;
  static constexpr size_t kSmem = kOffBar + 256 + 1024;  // + alignment slack for the 1 KB base
  static constexpr uint32_t kTmemCols = VB == 1 ? 256 : 128;       // P: VH columns, X^T: 64
  static_assert(VB == 1 || VB == 2, "one or two value blocks");
};

template <int VB>
__global__ void __launch_bounds__(ScanTcCfg<VB>::kThreads, 1) scan_tc_kernel(ScanParams p) {
  using Cfg = ScanTcCfg<VB>;
  constexpr int D = Cfg::D, VH = Cfg::VH, SV = Cfg::SV;
  extern __shared__ __align__(1024) unsigned char smem_scan_tc[];
  unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_scan_tc) + 1023) &
                                                       ~static_cast<uintptr_t>(1023));
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int vblk = blockIdx.x % VB, nh = blockIdx.x / VB;
  const int h = nh % p.H, n = nh / p.H;

  // barriers: 0-2 stage ring; 3 X^T ready, 4 P ready (tcgen05.commit);
  // 5 bf16(S)^T written, 6 v_new written (one arrival per worker warp)
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + Cfg::kOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + Cfg::kOffBar + 128);
  auto B = [&](int i) { return smem_u32(&bar[i]); };
  const uint32_t s_base = smem_u32(sm);
  auto st_w = [&](int st) { return s_base + st * Cfg::kStageStride; };
  auto st_kg = [&](int st) { return s_base + st * Cfg::kStageStride + Cfg::kBytesTile; };
  auto st_u = [&](int st) { return sm + st * Cfg::kStageStride + 2 * Cfg::kBytesTile; };
  auto st_el = [&](int st) {
    return reinterpret_cast<const float*>(sm + st * Cfg::kStageStride + 2 * Cfg::kBytesTile + Cfg::kBytesU);
  };
  unsigned char* sSb = sm + Cfg::kOffSb;  // Sb^T: VH/64 value panels of [128 key rows][64 values]
  unsigned char* sVn = sm + Cfg::kOffVn;  // v_new: [VH value rows][64 tokens]

  if (tid == 0) {
    for (int i = 0; i < 5; ++i) mbar_init(B(i), 1);
    mbar_init(B(5), Cfg::kWorkerWarps);
    mbar_init(B(6), Cfg::kWorkerWarps);
    mbar_fence_init();
  }
  if (warp == Cfg::kWorkerWarps) tc::alloc(smem_u32(tmem_slot), Cfg::kTmemCols);
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tP = tmem, tX = tmem + VH;
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

  const int quarter = warp & 3, half = (warp >> 2) & 1;
  const int key = 32 * quarter + lane;  // state row; also the value row of X^T and v_new
  const int64_t in_slot = pool_slot(p.slots_in, p.num_in, n), out_slot = pool_slot(p.slots_out, p.num_out, n);
  if (tid == 0 && vblk == 0 && (in_slot < 0 || out_slot < 0)) atomicOr(&p.hdr->status, 8);  // slot outside its pool
  const int64_t row_off = (int64_t)key * D + VH * vblk + SV * half;
  const int64_t in_off = (in_slot * p.H + h) * D * D + row_off, out_off = (out_slot * p.H + h) * D * D + row_off;
  float S[SV];

  if (warp == Cfg::kWorkerWarps) {
    // ---------------- control warp (converged; one elected lane issues) ----------------
    auto prefetch = [&](int c, int st) {
      const int64_t ch = (int64_t)c * p.H + h;
      const uint32_t mb = B(st);
      mbar_expect_tx(mb, 2 * Cfg::kBytesTile + Cfg::kBytesU + Cfg::kBytesEl);
      bulk_g2s(st_w(st), p.W + ch * kTile * D, Cfg::kBytesTile, mb);
      bulk_g2s(st_kg(st), p.KG + ch * kTile * D, Cfg::kBytesTile, mb);
      // u is stored as 64-value panels [64 tokens][64 values]: this CTA's VH/64 of them
      bulk_g2s(smem_u32(st_u(st)), p.U + ch * kTile * D + (int64_t)vblk * kTile * VH, Cfg::kBytesU, mb);
      bulk_g2s(smem_u32(st_el(st)), p.Elast + ch * D, Cfg::kBytesEl, mb);
    };
    if (tc::elect_one())
      for (int i = 0; i < Cfg::kStages - 1 && i < nchunks; ++i) prefetch(c0 + i, i);
    __syncwarp();
    constexpr uint32_t kIdX = tc::idesc(tc::kBF16, VH, 64, true, false);  // Sb^T MN-major, w K-major
    constexpr uint32_t kIdP = tc::idesc(tc::kBF16, 128, VH, true, false);  // kg^T MN-major, v_new K-major
    const uint32_t sb = smem_u32(sSb), vn = smem_u32(sVn);
    for (int it = 0; it < nchunks; ++it) {
      const int st = it % Cfg::kStages;
      const uint32_t ph = it & 1;
      const uint32_t w = st_w(st), kg = st_kg(st);
      wait(st, (it / Cfg::kStages) & 1);
      wait(5, ph);
      tc::fence_after();
      if (tc::elect_one()) {
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks)
          tc::mma_bf16(tX, tc::desc_mnmajor(sb, Cfg::kBytesPanelSb, ks),
                       tc::desc_kmajor(w + (ks >> 2) * (kTile * 128), (ks & 3) * 32), kIdX, ks > 0);
        tc::commit(B(3));
        // every reader of the stage that chunk it - 1 used has arrived on barrier 5 above
        if (it + Cfg::kStages - 1 < nchunks)
          prefetch(c0 + it + Cfg::kStages - 1, (it + Cfg::kStages - 1) % Cfg::kStages);
      }
      __syncwarp();
      wait(6, ph);
      tc::fence_after();
      if (tc::elect_one()) {
#pragma unroll
        for (int ks = 0; ks < kTile / 16; ++ks)
          tc::mma_bf16(tP, tc::desc_mnmajor(kg, kTile * 128, ks), tc::desc_kmajor(vn, ks * 32), kIdP, ks > 0);
        tc::commit(B(4));
      }
      __syncwarp();
    }
  } else {
    // ---------------- worker warps ----------------
#pragma unroll
    for (int j = 0; j < SV; j += 4) {  // zero state for an input slot outside the pool
      const float4 v = in_slot >= 0 ? *reinterpret_cast<const float4*>(p.h0 + in_off + j) : make_float4(0.f, 0.f, 0.f, 0.f);
      S[j] = v.x;
      S[j + 1] = v.y;
      S[j + 2] = v.z;
      S[j + 3] = v.w;
    }
    float el = 1.f;  // 2^G_last of the previous chunk for this key row
    auto update_state = [&]() {  // S = 2^G_last S + P
      tc::fence_after();
      const uint64_t e2 = f32x2_splat(el);  // packed fp32 pairs: the same rounding per lane
      auto fold32 = [&](int j0, const float (&P)[32]) {
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          const uint64_t a = fma_f32x2(e2, f32x2_pack(S[j0 + j], S[j0 + j + 1]), f32x2_pack(P[j], P[j + 1]));
          S[j0 + j] = f32x2_lo(a);
          S[j0 + j + 1] = f32x2_hi(a);
        }
      };
      if constexpr (SV == 64) {
        float P0[32], P1[32];
        tc::ld32x2(tc::lane_addr(tP, 32 * quarter, 64 * half), tc::lane_addr(tP, 32 * quarter, 64 * half + 32), P0,
                   P1);
        fold32(0, P0);
        fold32(32, P1);
      } else {
        float P0[32];
        tc::ld32(tc::lane_addr(tP, 32 * quarter, 32 * half), P0);
        fold32(0, P0);
      }
    };
    auto hand_over = [&](int b) {  // operand tile written: make it visible to the tensor cores
      tc::fence_smem_async();
      tc::fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(B(b));
    };
    for (int it = 0; it < nchunks; ++it) {
      const int st = it % Cfg::kStages;
      const uint32_t ph = it & 1;
      // ---- previous chunk's P into the state; bf16(S) -> Sb^T (MN-major, 64-value panels) ----
      if (it > 0) {
        wait(4, ph ^ 1);
        update_state();
      }
      {
        // this thread's values SV half .. + SV - 1: panel (SV half) / 64, 16-byte chunks from
        // ((SV half) % 64) / 8 on
        constexpr int kChunks = SV / 8;
        const int c_base = ((SV * half) % 64) / 8;
        unsigned char* row = sSb + ((SV * half) / 64) * Cfg::kBytesPanelSb + (key >> 3) * 1024 + (key & 7) * 128;
#pragma unroll
        for (int c = 0; c < kChunks; ++c) {
          uint4 pk;
          pk.x = pack_bf16x2(S[8 * c], S[8 * c + 1]);
          pk.y = pack_bf16x2(S[8 * c + 2], S[8 * c + 3]);
          pk.z = pack_bf16x2(S[8 * c + 4], S[8 * c + 5]);
          pk.w = pack_bf16x2(S[8 * c + 6], S[8 * c + 7]);
          *reinterpret_cast<uint4*>(row + (((c_base + c) ^ (key & 7)) << 4)) = pk;
        }
      }
      hand_over(5);
      // ---- v_new = bf16(u - X) -> K-major operand [value row][64 tokens] ----
      // u of this thread's value column is read while X^T is still being computed
      wait(st, (it / Cfg::kStages) & 1);
      el = st_el(st)[key];
      float uv[32];
      // value row of X^T and v_new: lane of the M = 128 (all lanes) or M = 64 (lanes 0-15) product
      const int vr = VB == 1 ? key : 16 * quarter + (lane & 15);
      const bool vrow_here = VB == 1 || lane < 16;
      {
        const unsigned char* u = st_u(st) + (vr >> 6) * (kTile * 128);  // value panel of u
        const int vc = (vr & 63) >> 3, vb = (vr & 7) * 2;
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int t = 32 * half + e;
          uv[e] = __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(u + t * 128 + ((vc ^ (t & 7)) << 4) + vb));
        }
      }
      wait(3, ph);
      tc::fence_after();
      {
        float X[32];
        tc::ld32(tc::lane_addr(tX, 32 * quarter, 32 * half), X);  // value vr, tokens 32 half ..
        unsigned char* vrow = sVn + (vr >> 3) * 1024 + (vr & 7) * 128;
        auto vnew = [&](int e) {  // bf16(u - X) of columns e, e + 1
          return f32x2_to_bf16x2(sub_f32x2(f32x2_pack(uv[e], uv[e + 1]), f32x2_pack(X[e], X[e + 1])));
        };
        if (vrow_here) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint4 pk;
            pk.x = vnew(8 * c);
            pk.y = vnew(8 * c + 2);
            pk.z = vnew(8 * c + 4);
            pk.w = vnew(8 * c + 6);
            *reinterpret_cast<uint4*>(vrow + (((4 * half + c) ^ (vr & 7)) << 4)) = pk;
          }
        }
      }
      hand_over(6);
    }
    if (nchunks > 0) {
      wait(4, (nchunks - 1) & 1);
      update_state();
    }
  }
  // a wait that ran out anywhere in the CTA: leave the final state untouched
  const bool ok = __syncthreads_and(alive) != 0;
  if (ok && warp < Cfg::kWorkerWarps && out_slot >= 0) {
#pragma unroll
    for (int j = 0; j < SV; j += 4)
      *reinterpret_cast<float4*>(p.ht + out_off + j) = make_float4(S[j], S[j + 1], S[j + 2], S[j + 3]);
  }
  tc::fence_before();
  __syncthreads();
  if (warp == Cfg::kWorkerWarps) tc::dealloc(tmem, Cfg::kTmemCols);
}

}  // namespace memt
