// Snapshot read o = scale * q . bf16(S) on tcgen05 tensor cores for d = 128 and 256 and blocks of
// many tokens (the commit read of token_memory_packed, models/qwen/ops/read.py:42-89 and
// models/deepseek/ops/read.py:6-31): one CTA per (block, head, run of up to RUN 64-token
// tiles).
//
//   * the block's fp32 snapshot is read once, rounded to bf16 (read.py:64) and written as the
//     MN-major B operand [D key rows][D/64 panels of 64 values] in shared memory (32 KB for
//     d = 128, 128 KB for d = 256);
//   * 64-token query tiles arrive by TMA (2-D tensor map over the [L, H*D] query rows, D/64
//     64-key boxes with the 128-byte swizzle = the K-major A operand) into a ring of four
//     (d = 128, two CTAs per SM) or three (d = 256, one CTA per SM) stages;
//   * a control warp issues the M = 64, N = D, K = D MMA of each tile into one of two
//     tensor-memory accumulators (2 x D columns);
//   * eight worker warps drain the other accumulator (token r in lane 32 (r / 16) + r % 16),
//     64 columns at a time, scale and round. At d = 128 a bf16 output tile goes back into the
//     ring stage it came from (the MMA has consumed it) in the TMA box layout and leaves with
//     D/64 TMA stores, after which the stage takes a later query tile. At d = 256 the rows go
//     straight to global memory and a stage takes a later query tile as soon as its MMA has
//     completed: with three stages of 32 KB, every stage but the one being multiplied is then
//     a load in flight (config-4 read 0.290 -> 0.249 ms; the same at d = 128 measured no
//     faster alone and slower beside the scan).
// The last tile of a block may straddle into the next block (or past L): its rows are
// computed from whatever the TMA brought (zeros past L) and stored row by row up to the block
// end instead. Every wait is bounded.
#pragma once

#include "common.cuh"
#include "read.cuh"
#include "tc.cuh"
#include "tma.h"

namespace memt {

// 64-token tiles per run: 16 where the read shares the GPU with the commit's scan (short CTAs
// take the SMs as the scan frees them), 32 for a d = 128 read on its own (half the snapshot
// conversions: config-1 read 0.145 -> 0.131 ms)
constexpr int kReadTcTiles = 16;
constexpr int kReadTcTilesAlone = 32;

struct ReadTcParams {
  CUtensorMap q_map;  // bf16 [L, H*D], boxes of 64 keys x 64 tokens
  CUtensorMap o_map;  // bf16 output, same geometry (d = 128 with out_bf16)
  ReadParams p;
};

template <int D_>
struct ReadTcCfg {
  static constexpr int D = D_, kTok = 64;
  static constexpr int kPanels = D / 64;                  // 64-value panels (TMA boxes, B operand panels)
  static constexpr int kWorkerWarps = 8;
  static constexpr int kThreads = (kWorkerWarps + 1) * 32;
  static constexpr int kStages = D <= 128 ? 4 : 3;        // query (d = 128: and output) tile ring
  static constexpr bool kTmaOut = D <= 128;               // bf16 output tiles leave by TMA stores
  // a stage is refilled kRefill iterations after its output store was issued: the control thread
  // then waits only for stores older than kRefill - 1 groups, and the refill runs
  // kStages - kRefill tiles ahead of its MMA
  static constexpr int kRefill = kStages >= 4 ? 2 : 1;
  static constexpr int kAcc = 2;                          // tensor-memory accumulators
  static constexpr uint32_t kBytesS = D * D * 2;          // bf16 snapshot: 32 KB (d = 128) / 128 KB (d = 256)
  static constexpr uint32_t kBytesQ = kTok * D * 2;       // per stage (query tile, then output tile)
  static constexpr uint32_t kBytesBox = kTok * 64 * 2;    // one 64-wide panel of a tile (8 KB)
  static constexpr uint32_t kBytesPanelS = kBytesS / kPanels;  // one 64-value panel of the snapshot
  static constexpr uint32_t kOffQ = kBytesS;
  static constexpr uint32_t kOffBar = kOffQ + kStages * kBytesQ;
  static constexpr size_t kSmem = kOffBar + 256 + 1024;
  static constexpr uint32_t kTmemCols = kAcc * D;         // kAcc M = 64 accumulators of D columns
  static constexpr int kMinBlocks = D <= 128 ? 2 : 1;
  static_assert(kSmem <= 227 * 1024 && kTmemCols <= 512, "one CTA's resources");
};

// RUN: 64-token tiles per run, a compile-time constant (the tile index arithmetic divides by it)
template <int D, int RUN>
__global__ void __launch_bounds__(ReadTcCfg<D>::kThreads, ReadTcCfg<D>::kMinBlocks)
    read_tc_kernel(const __grid_constant__ ReadTcParams P) {
  using Cfg = ReadTcCfg<D>;
  constexpr int NS = Cfg::kStages, NA = Cfg::kAcc, NP = Cfg::kPanels;
  const ReadParams& p = P.p;
  extern __shared__ __align__(1024) unsigned char smem_read_tc[];
  unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_read_tc) + 1023) &
                                                       ~static_cast<uintptr_t>(1023));
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n = blockIdx.x / p.H, h = blockIdx.x % p.H;
  int64_t bos, eos;
  block_range(p, n, bos, eos);
  // this CTA's tiles: runs y, y + gridDim.y, ... of RUN tiles, so that every token is
  // read whatever bound on the block length the host sized the grid with
  const int ntiles = strided_tiles(eos - bos, Cfg::kTok, RUN);
  if (ntiles == 0) return;
  const int64_t slot = state_slot(p, n);
  if (slot < 0) return;
  const bool tma_out = Cfg::kTmaOut && p.out_bf16 != 0;
  auto tile_start = [&](int i) { return bos + strided_tile_index(i, RUN) * Cfg::kTok; };
  auto full_tile = [&](int i) { return tile_start(i) + Cfg::kTok <= eos; };

  // barriers: [0, NS) stage holds the query tile (TMA); [AF, AF + NA) accumulator full
  // (commit); [AE, AE + NA) accumulator drained; SR snapshot operand written; [OR, OR + NS)
  // output tile written to the stage (AE.. and SR.. : one arrival per worker warp) or, without
  // TMA stores, the stage's MMA has completed (commit)
  constexpr int AF = NS, AE = NS + NA, SR = NS + 2 * NA, OR = SR + 1, NBAR = OR + NS;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + Cfg::kOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + Cfg::kOffBar + 8 * NBAR);
  auto B = [&](int i) { return smem_u32(&bar[i]); };
  unsigned char* sS = sm;
  const uint32_t sQ = smem_u32(sm + Cfg::kOffQ);

  if (tid == 0) {
    for (int i = 0; i < AE; ++i) mbar_init(B(i), 1);
    for (int i = AE; i < NBAR; ++i) mbar_init(B(i), Cfg::kTmaOut || i <= SR ? Cfg::kWorkerWarps : 1);
    mbar_fence_init();
  }
  if (warp == Cfg::kWorkerWarps) tc::alloc(smem_u32(tmem_slot), Cfg::kTmemCols);
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = *tmem_slot;

  bool alive = true;
  auto wait = [&](int b, uint32_t parity) {
    if (alive && !mbar_wait(B(b), parity)) alive = false;
  };

  if (warp == Cfg::kWorkerWarps) {
    if (lane == 0) {
      // Stage s cycles: query tile i (TMA load) -> MMA(i) -> output tile i (workers) ->
      // TMA store -> query tile i + NS, loaded R iterations after the store was issued so that
      // the control thread never waits for a store's read of shared memory.
      auto load_q = [&](int i) {
        const int s = i % NS;
        const int y = static_cast<int>(tile_start(i));
        mbar_expect_tx(B(s), Cfg::kBytesQ);
#pragma unroll
        for (int b = 0; b < NP; ++b)
          tma_load_2d(sQ + s * Cfg::kBytesQ + b * Cfg::kBytesBox, &P.q_map, h * D + 64 * b, y, B(s));
      };
      // one bulk group per tile (empty when the tile is stored row by row), so that the read
      // of tile j's output is complete once at most R - 1 younger groups are pending
      constexpr int R = Cfg::kRefill;
      auto store_out = [&](int i) {  // output tile i has been written to its stage
        const int s = i % NS;
        wait(OR + s, (i / NS) & 1);
        if (tma_out && full_tile(i)) {
          fence_proxy_async_smem();
          const int y = static_cast<int>(tile_start(i));
#pragma unroll
          for (int b = 0; b < NP; ++b)
            tma_store_2d(&P.o_map, h * D + 64 * b, y, sQ + s * Cfg::kBytesQ + b * Cfg::kBytesBox);
        }
        bulk_commit();
      };
      for (int i = 0; i < NS && i < ntiles; ++i) load_q(i);
      wait(SR, 0);
      constexpr uint32_t kId = tc::idesc(tc::kBF16, 64, D, false, true);  // q K-major, S MN-major
      const uint32_t ss = smem_u32(sS);
      for (int i = 0; i < ntiles; ++i) {
        const int s = i % NS, a = i % NA;
        wait(s, (i / NS) & 1);
        if (i >= NA) wait(AE + a, ((i / NA) - 1) & 1);
        tc::fence_after();
        const uint32_t q = sQ + s * Cfg::kBytesQ;
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks)
          tc::mma_bf16(tmem + D * a, tc::desc_kmajor(q + (ks >> 2) * Cfg::kBytesBox, (ks & 3) * 32),
                       tc::desc_mnmajor(ss, Cfg::kBytesPanelS, ks), kId, ks > 0);
        tc::commit(B(AF + a));
        if constexpr (Cfg::kTmaOut) {
          if (i >= 1) store_out(i - 1);
          // refill the stage of tile i - R, whose output store was committed R - 1 groups ago
          if (i >= R && i - R + NS < ntiles) {
            asm volatile("cp.async.bulk.wait_group.read %0;\n" ::"n"(R - 1) : "memory");
            load_q(i - R + NS);
          }
        } else {
          tc::commit(B(OR + s));
          // the stage of tile i - 1 takes tile i - 1 + NS once MMA(i - 1) has read it
          if (i >= 1 && i - 1 + NS < ntiles) {
            wait(OR + (i - 1) % NS, ((i - 1) / NS) & 1);
            load_q(i - 1 + NS);
          }
        }
      }
      if constexpr (Cfg::kTmaOut) {
        store_out(ntiles - 1);
        bulk_wait_all();
      }
    }
  } else {
    // snapshot -> bf16 MN-major operand [D key rows][NP panels of 64 values]: the worker threads
    // take the (row, panel) pieces in turn, 128 bytes of the bf16 row each
    {
      const float* base = p.states + (slot * p.H + h) * D * D;
      for (int u = tid; u < D * NP; u += Cfg::kWorkerWarps * 32) {
        const int row = u / NP, pan = u % NP;
        const float4* src = reinterpret_cast<const float4*>(base + (int64_t)row * D + 64 * pan);
        unsigned char* dst = sS + pan * Cfg::kBytesPanelS + (row >> 3) * 1024 + (row & 7) * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const float4 a = __ldg(src + 2 * c), b = __ldg(src + 2 * c + 1);
          uint4 pk;
          pk.x = pack_bf16x2(a.x, a.y);
          pk.y = pack_bf16x2(a.z, a.w);
          pk.z = pack_bf16x2(b.x, b.y);
          pk.w = pack_bf16x2(b.z, b.w);
          *reinterpret_cast<uint4*>(dst + ((c ^ (row & 7)) << 4)) = pk;
        }
      }
      tc::fence_smem_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(B(SR));
    }
    // M = 64 accumulator: token r of the tile sits in lane 32 (r / 16) + r % 16, so warp w uses
    // lanes 0-15 for tokens 16 (w % 4) .. and the columns of half w / 4, 64 at a time (one box)
    constexpr int CH = D / 128;  // 64-column boxes per warp
    const int quarter = warp & 3, half = warp >> 2;
    const int64_t qrow = (int64_t)p.H * D;
    const int r = 16 * quarter + lane;  // token row of the tile (lanes 0-15)
    for (int i = 0; i < ntiles; ++i) {
      const int s = i % NS, a = i % NA;
      wait(AF + a, (i / NA) & 1);  // MMA(i) done: its query stage is free for the output
      __syncwarp();
      tc::fence_after();
      const int64_t tok = tile_start(i) + r;
      const bool staged = tma_out && full_tile(i);
#pragma unroll
      for (int j = 0; j < CH; ++j) {
        const int box = half * CH + j;
        float o[2][32];
        tc::ld32x2(tc::lane_addr(tmem + D * a, 32 * quarter, 64 * box),
                   tc::lane_addr(tmem + D * a, 32 * quarter, 64 * box + 32), o[0], o[1]);
        if (j == CH - 1) {
          tc::fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(B(AE + a));  // the accumulator may be overwritten
        }
        if (lane < 16) {
          if (staged) {
            // output tile in the box layout of the TMA store: value panel `box`, row r
            unsigned char* row = sm + Cfg::kOffQ + s * Cfg::kBytesQ + box * Cfg::kBytesBox + (r >> 3) * 1024 +
                                 (r & 7) * 128;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              const float* v = &o[c >> 2][(c & 3) * 8];
              *reinterpret_cast<uint4*>(row + ((c ^ (r & 7)) << 4)) =
                  make_uint4(pack_bf16x2(v[0] * p.scale, v[1] * p.scale), pack_bf16x2(v[2] * p.scale, v[3] * p.scale),
                             pack_bf16x2(v[4] * p.scale, v[5] * p.scale), pack_bf16x2(v[6] * p.scale, v[7] * p.scale));
            }
          } else if (tok < eos) {
            const int64_t off = tok * qrow + (int64_t)h * D + 64 * box;
            if (p.out_bf16) {
              uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.out) + off);
#pragma unroll
              for (int c = 0; c < 8; ++c) {
                const float* v = &o[c >> 2][(c & 3) * 8];
                dst[c] = make_uint4(pack_bf16x2(v[0] * p.scale, v[1] * p.scale), pack_bf16x2(v[2] * p.scale, v[3] * p.scale),
                                    pack_bf16x2(v[4] * p.scale, v[5] * p.scale), pack_bf16x2(v[6] * p.scale, v[7] * p.scale));
              }
            } else {
              float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.out) + off);
#pragma unroll
              for (int c = 0; c < 16; ++c) {
                const float* v = &o[c >> 3][(c & 7) * 4];
                dst[c] = make_float4(v[0] * p.scale, v[1] * p.scale, v[2] * p.scale, v[3] * p.scale);
              }
            }
          }
        }
      }
      if constexpr (Cfg::kTmaOut) {
        if (staged) fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(B(OR + s));  // output tile i is in the stage (or stored)
      }
    }
  }
  tc::fence_before();
  __syncthreads();
  if (warp == Cfg::kWorkerWarps) tc::dealloc(tmem, Cfg::kTmemCols);
}

}  // namespace memt
