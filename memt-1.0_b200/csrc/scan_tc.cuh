// GDN-2 inter-chunk state scan on tcgen05 tensor cores, d = 128: one CTA per (sample, head).
//
// Same recurrence as scan.cuh (_fwd_h_kernel, models/qwen/ops/_triton/state.py:31-115), for
// every chunk of the sample in order:
//     v_new = u - w . bf16(S)                         (state.py:95-98)
//     S     = diag(2^G_last) S + kg^T . bf16(v_new)   (state.py:101-112)
// Value columns never mix, so the 128 state columns form two independent half-chains a and b
// (columns 0-63 and 64-127) that share the chunk's w and kg tiles. They run in ping-pong so
// that one half-chain's tensor-core latency hides behind the other's elementwise work:
//     update S_a -> [X_a = w . bf16(S_a)] ; update S_b -> [X_b]
//     v_new_a    -> [P_a = kg^T . v_new_a] ; v_new_b -> [P_b]
// where [..] is an MMA issued by a dedicated control warp (tcgen05, shared-memory operands,
// tensor-memory accumulators) and the rest runs on eight worker warps:
//   * the fp32 state lives in registers for the whole sample: worker (warp w, lane l) owns key
//     row 32 (w % 4) + l, columns 32 (w / 4) .. + 31 of each half-chain;
//   * X_h (M = 64 tokens, N = 64) and P_h (M = 128 keys, N = 64) come back through tensor
//     memory; workers write bf16(S_h) and bf16(v_new_h) straight into the swizzled operand
//     tiles of the next MMA and hand them over with mbarrier arrivals;
//   * w, kg, u of chunk c + 2 and 2^G_last arrive by bulk copies into a three-deep ring (the
//     intra kernel stores them in the operand layout, pswz).
// Every wait is bounded: a thread whose wait runs out flags the workspace header and stops
// waiting; the CTA then frees its tensor memory and leaves the final state untouched.
#pragma once

#include "common.cuh"
#include "tc.cuh"

namespace memt {

struct ScanTcCfg {
  static constexpr int D = 128;
  static constexpr int kWorkers = 256;
  static constexpr int kThreads = kWorkers + 32;  // + control warp
  static constexpr int kStages = 3;
  static constexpr uint32_t kBytesTile = uint32_t(kTile) * D * 2;  // 16 KB: w, kg or u of one chunk
  static constexpr uint32_t kBytesEl = D * 4;
  static constexpr uint32_t kStageStride = 3 * kBytesTile + 1024;  // tiles + 2^G_last, 1 KB aligned
  static constexpr uint32_t kOffSb = kStages * kStageStride;       // bf16(S) operands: 2 x [128][64]
  static constexpr uint32_t kOffVn = kOffSb + 2 * kBytesTile;       // bf16(v_new) operands: 2 x [64][64]
  static constexpr uint32_t kOffBar = kOffVn + kBytesTile;
  static constexpr size_t kSmem = kOffBar + 256 + 1024;  // + alignment slack for the 1 KB base
  static constexpr uint32_t kTmemCols = 256;             // P_a, P_b, X_a, X_b: 64 columns each
};

__global__ void __launch_bounds__(ScanTcCfg::kThreads, 1) scan_tc_kernel(ScanParams p) {
  using Cfg = ScanTcCfg;
  constexpr int D = Cfg::D;
  extern __shared__ __align__(1024) unsigned char smem_scan_tc[];
  unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_scan_tc) + 1023) &
                                                       ~static_cast<uintptr_t>(1023));
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int h = blockIdx.x % p.H, n = blockIdx.x / p.H;

  // barriers: 0-2 stage ring; 3/4 X_a/X_b and 5/6 P_a/P_b (tcgen05.commit);
  // 7/8 bf16(S_a)/(S_b) and 9/10 v_new_a/v_new_b written (one arrival per worker)
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + Cfg::kOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + Cfg::kOffBar + 128);
  auto B = [&](int i) { return smem_u32(&bar[i]); };
  const uint32_t s_base = smem_u32(sm);
  auto st_w = [&](int st) { return s_base + st * Cfg::kStageStride; };
  auto st_kg = [&](int st) { return s_base + st * Cfg::kStageStride + Cfg::kBytesTile; };
  auto st_u = [&](int st) { return sm + st * Cfg::kStageStride + 2 * Cfg::kBytesTile; };
  auto st_el = [&](int st) { return reinterpret_cast<const float*>(sm + st * Cfg::kStageStride + 3 * Cfg::kBytesTile); };
  unsigned char* sSb = sm + Cfg::kOffSb;  // half-chain hc at + hc * 16 KB: [128 key rows][64 values]
  unsigned char* sVn = sm + Cfg::kOffVn;  // half-chain hc at + hc * 8 KB:  [64 token rows][64 values]

  const int c0 = p.sample_off[n], c1 = p.sample_off[n + 1];
  const int nchunks = c1 - c0;

  if (tid == 0) {
    for (int i = 0; i < 7; ++i) mbar_init(B(i), 1);
    for (int i = 7; i < 11; ++i) mbar_init(B(i), Cfg::kWorkers);
    mbar_fence_init();
  }
  if (warp == 8) tc::alloc(smem_u32(tmem_slot), Cfg::kTmemCols);
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = *tmem_slot;
  auto tP = [&](int hc) { return tmem + 64 * hc; };
  auto tX = [&](int hc) { return tmem + 128 + 64 * hc; };

  bool alive = true;
  auto wait = [&](int b, uint32_t parity) {
    if (alive && !mbar_wait(B(b), parity)) {
      alive = false;
      atomicOr(&p.hdr->status, 4);
    }
  };

  // worker geometry (unused by the control warp)
  const int quarter = warp & 3, half = (warp >> 2) & 1;
  const int key = 32 * quarter + lane;  // state row
  const int tok = 16 * quarter + lane;  // token row of X / v_new (lanes 0-15)
  const int64_t state_off = ((int64_t)n * p.H + h) * D * D + (int64_t)key * D + 32 * half;
  float S[2][32];

  if (warp == 8) {
    // ---------------- control warp: bulk copies and MMA issue (lane 0) ----------------
    if (lane == 0) {
      auto prefetch = [&](int c, int st) {
        const int64_t ch = (int64_t)c * p.H + h;
        const uint32_t mb = B(st);
        mbar_expect_tx(mb, 3 * Cfg::kBytesTile + Cfg::kBytesEl);
        bulk_g2s(st_w(st), p.W + ch * kTile * D, Cfg::kBytesTile, mb);
        bulk_g2s(st_kg(st), p.KG + ch * kTile * D, Cfg::kBytesTile, mb);
        bulk_g2s(smem_u32(st_u(st)), p.U + ch * kTile * D, Cfg::kBytesTile, mb);
        bulk_g2s(smem_u32(st_el(st)), p.Elast + ch * D, Cfg::kBytesEl, mb);
      };
      for (int i = 0; i < Cfg::kStages - 1 && i < nchunks; ++i) prefetch(c0 + i, i);
      constexpr uint32_t kIdX = tc::idesc(tc::kBF16, 64, 64, false, true);  // w K-major, S MN-major
      constexpr uint32_t kIdP = tc::idesc(tc::kBF16, 128, 64, true, true);  // kg^T MN-major, v_new MN-major
      const uint32_t sb = smem_u32(sSb), vn = smem_u32(sVn);
      for (int it = 0; it < nchunks; ++it) {
        const int st = it % Cfg::kStages;
        const uint32_t ph = it & 1;
        wait(st, (it / Cfg::kStages) & 1);
        const uint32_t w = st_w(st), kg = st_kg(st);
        for (int hc = 0; hc < 2; ++hc) {  // X_h = w . bf16(S_h)
          wait(7 + hc, ph);
          tc::fence_after();
#pragma unroll
          for (int ks = 0; ks < D / 16; ++ks)
            tc::mma_bf16(tX(hc), tc::desc_kmajor(w + (ks >> 2) * (kTile * 128), (ks & 3) * 32),
                         tc::desc_mnmajor(sb + hc * Cfg::kBytesTile, Cfg::kBytesTile, ks), kIdX, ks > 0);
          tc::commit(B(3 + hc));
        }
        // every reader of the stage that chunk it - 1 used has arrived on barrier 8 above
        if (it + Cfg::kStages - 1 < nchunks)
          prefetch(c0 + it + Cfg::kStages - 1, (it + Cfg::kStages - 1) % Cfg::kStages);
        for (int hc = 0; hc < 2; ++hc) {  // P_h = kg^T . v_new_h
          wait(9 + hc, ph);
          tc::fence_after();
#pragma unroll
          for (int ks = 0; ks < kTile / 16; ++ks)
            tc::mma_bf16(tP(hc), tc::desc_mnmajor(kg, kTile * 128, ks),
                         tc::desc_mnmajor(vn + hc * (Cfg::kBytesTile / 2), Cfg::kBytesTile / 2, ks), kIdP,
                         ks > 0);
          tc::commit(B(5 + hc));
        }
      }
    }
  } else {
    // ---------------- workers ----------------
#pragma unroll
    for (int hc = 0; hc < 2; ++hc)
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        const float4 v = *reinterpret_cast<const float4*>(p.h0 + state_off + 64 * hc + j);
        S[hc][j] = v.x;
        S[hc][j + 1] = v.y;
        S[hc][j + 2] = v.z;
        S[hc][j + 3] = v.w;
      }
    float el = 1.f;  // 2^G_last of the previous chunk for this key row
    auto update_state = [&](int hc) {  // S_h = 2^G_last S_h + P_h
      __syncwarp();
      tc::fence_after();
      float P[32];
      tc::ld32(tc::lane_addr(tP(hc), 32 * quarter, 32 * half), P);
#pragma unroll
      for (int j = 0; j < 32; ++j) S[hc][j] = fmaf(el, S[hc][j], P[j]);
    };
    for (int it = 0; it < nchunks; ++it) {
      const int st = it % Cfg::kStages;
      const uint32_t ph = it & 1;
#pragma unroll
      for (int hc = 0; hc < 2; ++hc) {
        // ---- previous chunk's P_h into the state; bf16(S_h) -> MN-major [key][64] operand ----
        if (it > 0) {
          wait(5 + hc, ph ^ 1);
          update_state(hc);
        }
        unsigned char* row = sSb + hc * Cfg::kBytesTile + (key >> 3) * 1024 + (key & 7) * 128;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint4 pk;
          pk.x = pack_bf16x2(S[hc][8 * c], S[hc][8 * c + 1]);
          pk.y = pack_bf16x2(S[hc][8 * c + 2], S[hc][8 * c + 3]);
          pk.z = pack_bf16x2(S[hc][8 * c + 4], S[hc][8 * c + 5]);
          pk.w = pack_bf16x2(S[hc][8 * c + 6], S[hc][8 * c + 7]);
          *reinterpret_cast<uint4*>(row + (((4 * half + c) ^ (key & 7)) << 4)) = pk;
        }
        tc::fence_smem_async();
        tc::fence_before();
        mbar_arrive(B(7 + hc));
      }
      wait(st, (it / Cfg::kStages) & 1);
      el = st_el(st)[key];
#pragma unroll
      for (int hc = 0; hc < 2; ++hc) {
        // ---- v_new_h = bf16(u - X_h) -> MN-major [token][64] operand (lanes 0-15) ----
        wait(3 + hc, ph);
        __syncwarp();
        tc::fence_after();
        float X[32];
        tc::ld32(tc::lane_addr(tX(hc), 32 * quarter, 32 * half), X);
        if (lane < 16) {
          const unsigned char* urow = st_u(st) + hc * (kTile * 128) + tok * 128;
          unsigned char* vrow = sVn + hc * (Cfg::kBytesTile / 2) + (tok >> 3) * 1024 + (tok & 7) * 128;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const int pc = ((4 * half + c) ^ (tok & 7)) << 4;
            const uint4 uv = *reinterpret_cast<const uint4*>(urow + pc);
            const uint32_t* uw = reinterpret_cast<const uint32_t*>(&uv);
            uint4 pk;
            uint32_t* pw = reinterpret_cast<uint32_t*>(&pk);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 u2 = unpack_bf16x2(uw[e]);
              pw[e] = pack_bf16x2(u2.x - X[8 * c + 2 * e], u2.y - X[8 * c + 2 * e + 1]);
            }
            *reinterpret_cast<uint4*>(vrow + pc) = pk;
          }
        }
        tc::fence_smem_async();
        tc::fence_before();
        mbar_arrive(B(9 + hc));
      }
    }
    if (nchunks > 0) {
#pragma unroll
      for (int hc = 0; hc < 2; ++hc) {
        wait(5 + hc, (nchunks - 1) & 1);
        update_state(hc);
      }
    }
  }
  // a wait that ran out anywhere in the CTA: leave the final state untouched
  const bool ok = __syncthreads_and(alive) != 0;
  if (ok && warp < 8) {
#pragma unroll
    for (int hc = 0; hc < 2; ++hc)
#pragma unroll
      for (int j = 0; j < 32; j += 4)
        *reinterpret_cast<float4*>(p.ht + state_off + 64 * hc + j) =
            make_float4(S[hc][j], S[hc][j + 1], S[hc][j + 2], S[hc][j + 3]);
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 8) tc::dealloc(tmem, Cfg::kTmemCols);
}

}  // namespace memt
