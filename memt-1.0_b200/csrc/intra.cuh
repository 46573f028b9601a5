// GDN-2 intra-chunk kernel: one CTA (8 warps) per (64-token chunk, head).
//
// Fuses what the reference runs as four launches with HBM round trips between them
// (paths relative to inference/memt_sglang):
//   chunk_local_cumsum                   _vendor/fla/ops/utils/cumsum.py:76-133
//   diagonal key-key blocks              _vendor/fla/ops/gdn2/chunk_intra_token_parallel.py:25-132
//   off-diagonal blocks + blocked solve  _vendor/fla/ops/gdn2/chunk_intra.py:153-417
//   WY operands u, w, kg                 _vendor/fla/ops/gdn2/wy_fast.py:36-142
// and writes only what the state scan consumes: w and kg ([chunk][head][64][D]), u
// ([chunk][head][D/64][64][64]), all bf16 in the scan's swizzled tile layout, and the chunk's
// total decay 2^G_last (fp32, [chunk][head][D]).
//
// Numerics follow the reference's GPU rounding points: fp32 cumulative log2 decay; fp32
// diagonal 16x16 key-key blocks; off-diagonal blocks from tf32 operands scaled to the first
// token of the row sub-chunk (per-channel decay); fp32 forward substitution on the diagonal
// blocks and tf32 products for the off-diagonal inverse blocks; A^-1 stored as bf16;
// u = A^-1 bf16(v*w), w = A^-1 bf16(bf16(k*b) 2^G), kg = bf16(k 2^(G_last-G)), all with fp32
// accumulation. With a per-head decay every key-key block, diagonal or not, is the exact
// bf16 product k'_i . k'_j (fp32 accumulation) times 2^(G_i - G_j) <= 1: more accurate than
// the reference's tf32 operands for the off-diagonal blocks, and free of their conversions.
//
// Operand staging: k, erase, v, write (bf16) and the decay arrive by cp.async into
// XOR-swizzled shared tiles. The tf32 score products take their fragments straight from
// ldmatrix: the k dimension is permuted so that the bf16 pair (2t, 2t+1) a lane receives
// feeds k-slots t and t+4 of an m16n8k8 fragment (a permutation of the summation index
// leaves the product unchanged). Fragment loads of a k-step are issued before its MMAs.
//
// Work split: the 20 (16-row block, 8-column tile) pieces of the lower-triangular score
// matrix are spread over the 8 warps (at most 3 each, one row block per warp). For D <= 128
// warps 0-3 run the serial blocked solve while warps 4-7 stage the u and w operands and
// write kg (named barriers keep the two groups independent).
//
// Gate layouts:
//   per head (one decay per token): every factor is a row or column scalar, so all key-key
//     blocks are exact bf16 products (fp32 accumulation) times the per-pair 2^(G_i-G_j),
//     applied after the sum (exponents <= 0: no overflow).
//   per channel: 2^G and 2^-G are tabulated once when every exponent of the panel lies in
//     [-60, 60] and factors are products of table entries (diagonal blocks in 3xTF32);
//     otherwise factors are exp2 of differences and the diagonal blocks are evaluated pair
//     by pair, exactly as the reference's token-parallel kernel does.
#pragma once

#include <type_traits>

#include "common.cuh"
#include "tma.h"

namespace memt {

template <int D, bool HEAD, bool ERASE>
struct IntraCfg {
  static constexpr int kPanel = D < 128 ? D : 128;
  static constexpr int kPanels = D / kPanel;
  static constexpr int kThreads = 256;
  static constexpr int kLdE = kPanel;       // fp32 cumulative log2 decay (per channel), eidx layout
  static constexpr int kLdA = kTile + 4;    // fp32 64x64 scores / inverse blocks
  static constexpr int kLdAi = kTile + 8;   // bf16 64x64 inverse
  static constexpr size_t kTileB = size_t(kTile) * kPanel * 2;  // one bf16 [64][panel] tile
  static constexpr size_t kBytesE = HEAD ? 0 : size_t(kTile) * kLdE * 4;
  static constexpr size_t kBytesA = size_t(kTile) * kLdA * 4;
  static constexpr size_t kBytesAi = size_t(kTile) * kLdAi * 2;
  // per-head decay without erase, D <= 128: k, v and write tiles arrive by TMA (the tiles need
  // the 1024-byte aligned base of the 128-byte swizzle)
  static constexpr bool kTma = HEAD && !ERASE && kPanels == 1;
  // the fifth tile: the TMA loop's second k buffer (the panel loop of D = 256 writes its products
  // into the write-gate tile, which is free at those points)
  static constexpr bool kNeedO = kTma;
  // sK | sB? | sV | sW (later the w operand) | sO? | sE? | sA | sAi
  static constexpr size_t offK = 0;
  static constexpr size_t offB = offK + kTileB;
  static constexpr size_t offV = offB + (ERASE ? kTileB : 0);
  static constexpr size_t offW = offV + kTileB;
  static constexpr size_t offO = offW + kTileB;
  static constexpr size_t offE = offO + (kNeedO ? kTileB : 0);
  static constexpr size_t offA = offE + kBytesE;
  static constexpr size_t offAi = offA + kBytesA;
  // Every configuration rounds the dynamic base up itself (the slack below; 1024 bytes for the
  // swizzled TMA tiles, 128 otherwise): the kernel also declares static shared arrays, and where
  // the dynamic region starts after them is the toolchain's choice (a build with relocatable
  // device code started it at an address that broke 16-byte accesses).
  static constexpr uint32_t kAlign = kTma ? 1024u : 128u;
  static constexpr size_t kSmem = offAi + kBytesAi + kAlign;
  static constexpr int kSmall = 9 * kTile + kThreads;  // static per-head factors + scan totals
  // static factor buffer: two units' per-head factors, or the per-channel scan totals
  static constexpr int kFacFloats = HEAD ? 2 * kSmall : 2 * 128;
};

__device__ __forceinline__ void named_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(nthreads) : "memory");
}

// 16x16x16 tf32 product on one warp: acc[nt] += A (16x16 fp32, row-major, lda) . B (16x16,
// [k][n], ldb); acc[nt] is the C fragment of columns 8*nt..8*nt+7.
__device__ __forceinline__ void warp_tf32_16x16x16(float (&acc)[2][4], const float* A, int lda,
                                                   const float* B, int ldb, int lane) {
  const int g = lane >> 2, t = lane & 3;
  uint32_t a[2][4], b[2][2][2];
#pragma unroll
  for (int kq = 0; kq < 2; ++kq) {
    const int kk = 8 * kq;
    a[kq][0] = to_tf32(A[g * lda + kk + t]);
    a[kq][1] = to_tf32(A[(g + 8) * lda + kk + t]);
    a[kq][2] = to_tf32(A[g * lda + kk + t + 4]);
    a[kq][3] = to_tf32(A[(g + 8) * lda + kk + t + 4]);
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      b[kq][nt][0] = to_tf32(B[(kk + t) * ldb + nt * 8 + g]);
      b[kq][nt][1] = to_tf32(B[(kk + t + 4) * ldb + nt * 8 + g]);
    }
  }
#pragma unroll
  for (int kq = 0; kq < 2; ++kq)
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) mma_tf32_1688(acc[nt], a[kq], b[kq][nt]);
}

// acc[nt] += A . (B0 + B1 [+ B2]): the B operand is the fp32 sum of two or three 16x16
// blocks (added left to right, then rounded to tf32), as the reference sums separate dots
// before the outer product (chunk_intra.py:377-395).
__device__ __forceinline__ void warp_tf32_A_sumB(float (&acc)[2][4], const float* A, int lda, const float* B0,
                                                 const float* B1, const float* B2, int ldb, int lane) {
  const int g = lane >> 2, t = lane & 3;
  uint32_t a[2][4], b[2][2][2];
#pragma unroll
  for (int kq = 0; kq < 2; ++kq) {
    const int kk = 8 * kq;
    a[kq][0] = to_tf32(A[g * lda + kk + t]);
    a[kq][1] = to_tf32(A[(g + 8) * lda + kk + t]);
    a[kq][2] = to_tf32(A[g * lda + kk + t + 4]);
    a[kq][3] = to_tf32(A[(g + 8) * lda + kk + t + 4]);
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int o = (kk + t + 4 * e) * ldb + nt * 8 + g;
        float s = B0[o] + B1[o];
        if (B2 != nullptr) s += B2[o];
        b[kq][nt][e] = to_tf32(s);
      }
    }
  }
#pragma unroll
  for (int kq = 0; kq < 2; ++kq)
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) mma_tf32_1688(acc[nt], a[kq], b[kq][nt]);
}

__device__ __forceinline__ void zero_acc(float (&acc)[2][4]) {
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
}

__device__ __forceinline__ void warp_store_f32(float* C, int ldc, const float (&acc)[2][4], int lane) {
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    *reinterpret_cast<float2*>(C + g * ldc + nt * 8 + 2 * t) = make_float2(acc[nt][0], acc[nt][1]);
    *reinterpret_cast<float2*>(C + (g + 8) * ldc + nt * 8 + 2 * t) = make_float2(acc[nt][2], acc[nt][3]);
  }
}

// Store a 16x16 C fragment pair as fp32 (sign applied) into A and, rows masked by `len`,
// as bf16 into Ai.
__device__ __forceinline__ void warp_store_block(float* A, int lda, __nv_bfloat16* Ai, int ldai,
                                                 const float (&acc)[2][4], int lane, float sign,
                                                 int row0, int len) {
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    const float x0 = sign * acc[nt][0], x1 = sign * acc[nt][1];
    const float x2 = sign * acc[nt][2], x3 = sign * acc[nt][3];
    const int c = nt * 8 + 2 * t;
    if (A != nullptr) {
      *reinterpret_cast<float2*>(A + g * lda + c) = make_float2(x0, x1);
      *reinterpret_cast<float2*>(A + (g + 8) * lda + c) = make_float2(x2, x3);
    }
    const bool ok0 = row0 + g < len, ok1 = row0 + g + 8 < len;
    *reinterpret_cast<uint32_t*>(Ai + g * ldai + c) = ok0 ? pack_bf16x2(x0, x1) : 0u;
    *reinterpret_cast<uint32_t*>(Ai + (g + 8) * ldai + c) = ok1 ? pack_bf16x2(x2, x3) : 0u;
  }
}

__device__ __forceinline__ float bf_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf_hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }

// Score pieces of each warp: one row block r, up to three 8-column tiles (-1 = none).
// Row block r has 2(r+1) tiles; 20 tiles over 8 warps, at most 3 per warp.
__device__ __forceinline__ void score_pieces(int warp, int& r, int (&nt)[3]) {
  switch (warp) {
    case 0: r = 0; nt[0] = 0; nt[1] = 1; nt[2] = -1; break;
    case 1: r = 1; nt[0] = 0; nt[1] = 2; nt[2] = -1; break;
    case 2: r = 1; nt[0] = 1; nt[1] = 3; nt[2] = -1; break;
    case 3: r = 2; nt[0] = 0; nt[1] = 2; nt[2] = 4; break;
    case 4: r = 2; nt[0] = 1; nt[1] = 3; nt[2] = 5; break;
    case 5: r = 3; nt[0] = 0; nt[1] = 3; nt[2] = 6; break;
    case 6: r = 3; nt[0] = 1; nt[1] = 4; nt[2] = 7; break;
    default: r = 3; nt[0] = 2; nt[1] = 5; nt[2] = -1; break;
  }
}

template <int D, bool HEAD, bool ERASE>
struct IntraKernel {
  using Cfg = IntraCfg<D, HEAD, ERASE>;
  static constexpr int P = Cfg::kPanel;
  static constexpr int NT = Cfg::kThreads;
  static constexpr bool kOverlap = Cfg::kPanels == 1;  // solve || staging (D <= 128)
  static constexpr bool kTma = Cfg::kTma;
  static constexpr uint32_t kTileBytes = static_cast<uint32_t>(Cfg::kTileB);

  __nv_bfloat16 *sK, *sB, *sV, *sW, *sO, *sAi;
  float *sE, *sA;  // sE (per channel): G, the cumulative log2 decay of the panel, [64][P] (eidx)
  // per-head factors: G, left (row) factor, right factors per row block, 2^G, 2^(G_last-G),
  // bf16(sqrt(beta)) per token
  float *sG, *sLf, *sRf, *sEh, *sKgf;
  float* sPre;  // [2][128]: per-token scalars of the current / next unit (fetch_scalars)
  int pre;      // which half of sPre belongs to the current unit
  float* sSeg;
  float* sFac;  // [2][kSmall]: factors of the current / next unit (per-head decay)
  float* sScr;  // 4 fp32 16x16 scratch blocks of the blocked solve
  uint32_t sMb;  // TMA path: mbarriers [k buffer 0, k buffer 1, v + write] (8 bytes each)

  int tid, lane, warp, len, tok0, h;
  int64_t row_stride;
  bool fast;

  // async copy of one [64][P] bf16 panel (rows >= len zero-filled) into a swizzled tile
  __device__ __forceinline__ void load_tile(__nv_bfloat16* dst, const __nv_bfloat16* src, int c0, int64_t stride) {
    load_tile_for<0, NT>(dst, src, c0, tok0, len, h, stride);
  }
  // the same for an explicit (token range, head) and the threads [T0, T0 + NTH)
  template <int T0, int NTH>
  __device__ __forceinline__ void load_tile_for(__nv_bfloat16* dst, const __nv_bfloat16* src, int c0, int tk0,
                                                int ln, int hd, int64_t stride) {
    const __nv_bfloat16* base = src + (int64_t)tk0 * stride + (int64_t)hd * D + c0;
    constexpr int kChunks = kTile * P / 8;
    static_assert(kChunks % NTH == 0, "chunks per thread");
#pragma unroll
    for (int i = tid - T0; i < kChunks; i += NTH) {
      const int row = i / (P / 8), col = (i % (P / 8)) * 8;
      const bool valid = row < ln;
      cp_async16_zfill(dst + pswz(row, col), valid ? base + (int64_t)row * stride + col : src, valid);
    }
  }

  // Chunk walk of a [64][P] pswz tile by threads [T0, T0 + NTH): thread t = tid - T0 visits the
  // 16-byte chunks t, t + NTH, ..., i.e. chunk column t % (P/8) in rows t / (P/8) + j * kRows.
  // kRows is a multiple of 8, so the swizzle key (row & 7), and with it the chunk's position in
  // its row, is the same on every visit: visit j lies j * kStride bytes after the first.
  template <int NTH>
  struct Walk {
    static constexpr int kRows = NTH / (P / 8);
    static constexpr int kSteps = kTile / kRows;
    static constexpr uint32_t kStride = kRows * 128u;
    static_assert(kRows % 8 == 0 && kTile % kRows == 0, "swizzle key fixed along the walk");
  };
  // first visit of thread tid: its row and column, and the chunk's byte offset in the tile
  template <int T0>
  __device__ __forceinline__ uint32_t walk_start(int& row0, int& col) const {
    const int t = tid - T0;
    row0 = t / (P / 8);
    col = (t % (P / 8)) * 8;
    return 2u * static_cast<uint32_t>(pswz(row0, col));
  }

  // Per-token scalars of a unit into buf: [0, 64) the per-head log-decay, [64, 128)
  // bf16(sqrt(beta)) of a per-head beta. Threads [t0, t0 + 64); issued one unit ahead so the
  // global-load latency hides behind the previous unit's solve.
  __device__ void fetch_scalars(const IntraParams& p, int tk0, int ln, int hd, float* buf, int t0) {
    float gv;
    uint32_t bv;
    load_scalars(p, tk0, ln, hd, t0, gv, bv);
    store_scalars(buf, t0, gv, bv);
  }
  // the two halves of fetch_scalars: issue the loads early, store once other work is done
  // (beta stays as raw bf16 bits until the store: nothing waits on the loads before then)
  __device__ __forceinline__ void load_scalars(const IntraParams& p, int tk0, int ln, int hd, int t0, float& gv,
                                               uint32_t& bv) const {
    const int i = tid - t0;
    gv = 0.f;
    bv = 0u;
    if (i >= 0 && i < ln && i < kTile) {
      if constexpr (HEAD) gv = p.g[(int64_t)(tk0 + i) * p.H + hd];
      if (p.beta_layout == 1)
        bv = *reinterpret_cast<const unsigned short*>(p.beta + (int64_t)(tk0 + i) * p.H + hd);
    }
  }
  __device__ __forceinline__ void store_scalars(float* buf, int t0, float gv, uint32_t bits) const {
    const int i = tid - t0;
    if (i < 0 || i >= kTile) return;
    const float bv = __uint_as_float(bits << 16);
    buf[i] = gv;
    buf[kTile + i] = bv > 0.f ? bf16_round(sqrtf(bv)) : 0.f;
  }

  // Fold sqrt(beta) into k in place: k' = bf16( bf16(sqrt(beta)) * k ) (models/qwen/layer.py:81-96)
  // for the unit (tk0, ln, hd) whose per-head scalars are in sPre half `ph`; threads [T0, T0 + NTH)
  template <int T0, int NTH>
  __device__ void fold_beta_for(const IntraParams& p, __nv_bfloat16* kbuf, int c0, int tk0, int ln, int hd, int ph) {
    using Wk = Walk<NTH>;
    int row0, col;
    unsigned char* kb = reinterpret_cast<unsigned char*>(kbuf) + walk_start<T0>(row0, col);
    const __nv_bfloat16* bsrc = p.beta + (int64_t)(tk0 + row0) * row_stride + (int64_t)hd * D + c0 + col;
#pragma unroll
    for (int j = 0; j < Wk::kSteps; ++j) {
      const int row = row0 + j * Wk::kRows;
      const bool in = row < ln;  // rows past the chunk become zero
      uint4* ptr = reinterpret_cast<uint4*>(kb + j * Wk::kStride);
      uint4 kv = *ptr;
      // both factors are bf16, so bf16(k * s) is one packed bf16 multiply
      uint32_t sw[4];
      if (p.beta_layout == 1) {
        const uint32_t s = __float_as_uint(sPre[ph * 2 * kTile + kTile + row]);  // bf16-exact
        sw[0] = sw[1] = sw[2] = sw[3] = (s >> 16) | (s & 0xffff0000u);
      } else {
        uint4 be = make_uint4(0, 0, 0, 0);
        if (in) be = *reinterpret_cast<const uint4*>(bsrc + (int64_t)j * Wk::kRows * row_stride);
        const uint32_t* bw = reinterpret_cast<const uint32_t*>(&be);
#pragma unroll
        for (int e = 0; e < 4; ++e) sw[e] = pack_bf16x2(sqrtf(bf_lo(bw[e])), sqrtf(bf_hi(bw[e])));
      }
      kv.x = in ? mul_bf16x2(kv.x, sw[0]) : 0u;
      kv.y = in ? mul_bf16x2(kv.y, sw[1]) : 0u;
      kv.z = in ? mul_bf16x2(kv.z, sw[2]) : 0u;
      kv.w = in ? mul_bf16x2(kv.w, sw[3]) : 0u;
      *ptr = kv;
    }
  }
  __device__ void fold_beta(const IntraParams& p, __nv_bfloat16* kbuf, int c0) {
    fold_beta_for<0, NT>(p, kbuf, c0, tok0, len, h, pre);
  }

  // ---- decay, per-head layout: one warp computes every factor a chunk needs ----
  // From the unit's per-token log-decays gbuf[0, 64) (zero past ln) into the factor buffer
  // fac (layout of use_factors). Executed by one whole warp.
  __device__ void head_factors(const float* gbuf, float* fac, int ln) {
    float* fG = fac;
    float* fLf = fac + kTile;
    float* fEh = fac + 2 * kTile;
    float* fKgf = fac + 3 * kTile;
    float* fRf = fac + 4 * kTile;
    float* fSeg = fac + 9 * kTile;
    // G_t = (sum_{s<=t} g_s) / ln2 over the 64 tokens; lane owns tokens 2*lane, 2*lane+1
    const int t0 = 2 * lane, t1 = 2 * lane + 1;
    const float g0 = gbuf[t0];
    const float g1 = gbuf[t1];
    float s = g0 + g1;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    const float excl = s - (g0 + g1);
    const float G0 = (excl + g0) * kRcpLn2, G1 = (excl + g0 + g1) * kRcpLn2;
    fG[t0] = G0;
    fG[t1] = G1;
    // G at the last token and at the sub-chunk starts 16r, by shuffles
    const int last = ln - 1;
    const float Gl = __shfl_sync(0xffffffffu, (last & 1) ? G1 : G0, last >> 1);
    float Gn[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) Gn[r] = __shfl_sync(0xffffffffu, G0, 8 * r);
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int i = 2 * lane + q;
      const float Gi = q ? G1 : G0;
      const float Gs = Gn[i >> 4];
      fLf[i] = fast_exp2(Gi - Gs);                  // left factor 2^(G_i - G_n(i))
      fEh[i] = fast_exp2(Gi);                       // 2^G_i
      fKgf[i] = i < ln ? fast_exp2(Gl - Gi) : 0.f;  // 2^(G_last - G_i)
#pragma unroll
      for (int r = 1; r < 4; ++r)                   // right factors 2^(G_n(r) - G_j), j < 16r
        fRf[r * kTile + i] = i < 16 * r ? fast_exp2(Gn[r] - Gi) : 0.f;
    }
    if (lane == 0) fSeg[0] = fast_exp2(Gl);         // 2^G_last
  }
  // point the factor arrays at buffer b of sFac
  __device__ __forceinline__ void use_factors(int b) {
    if constexpr (!HEAD) {  // per channel: only the scan totals of channel_tables
      sSeg = sFac;
      return;
    }
    float* f = sFac + b * Cfg::kSmall;
    sG = f;
    sLf = f + kTile;
    sEh = f + 2 * kTile;
    sKgf = f + 3 * kTile;
    sRf = f + 4 * kTile;  // [4][64], rows 1..3 used
    sSeg = f + 9 * kTile;
  }

  // Element (row, col) of the per-channel decay table: rows of P floats whose 16-byte chunks q
  // are XOR-permuted within groups of eight by (2 row ^ q / 8) & 7, so that a half-warp's score
  // fragment reads (4 rows x two adjacent chunks) and a quarter-warp's 16-byte staging reads
  // (every other chunk of one row) fall in distinct banks without padding; chunk-granular, so
  // cp.async fills it directly and a chunk stays 16 contiguous bytes.
  __device__ __forceinline__ static int eidx(int row, int col) {
    const int q = col >> 2;  // 16-byte chunk
    return row * Cfg::kLdE + (((q ^ (row << 1) ^ (q >> 3)) & 7) | (q & ~7)) * 4 + (col & 3);
  }

  // ---- decay, per-channel layout: cumulative sum and factor tables of one panel ----
  __device__ void channel_tables() {
    // sE holds the raw decay (cp.async); segmented scan over the 64 tokens per channel. A thread's
    // segment is read into registers first and written once at the end: a running sum stored and
    // reloaded through sE would serialise every step on a store-to-load dependence
    constexpr int kSeg = NT / P, kSegLen = kTile / kSeg;
    const int c = tid % P, sg = tid / P;
    float x[kSegLen];
#pragma unroll
    for (int i = 0; i < kSegLen; ++i) x[i] = sE[eidx(sg * kSegLen + i, c)];
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < kSegLen; ++i) {
      acc += x[i];
      x[i] = acc;
    }
    sSeg[sg * P + c] = acc;
    __syncthreads();
    float off = 0.f;
    for (int s2 = 0; s2 < sg; ++s2) off += sSeg[s2 * P + c];
    bool ok = true;
#pragma unroll
    for (int i = 0; i < kSegLen; ++i) {
      const float G = (x[i] + off) * kRcpLn2;
      ok = ok && (G >= -60.f) && (G <= 60.f);
      sE[eidx(sg * kSegLen + i, c)] = G;
    }
    // fast: every exponent of the panel in [-60, 60], so that the factorised diagonal blocks
    // (left factor <= 1, right factor >= 1) cannot overflow; otherwise the diagonal blocks are
    // evaluated pair by pair
    fast = __syncthreads_and(ok) != 0;
  }
  __device__ __forceinline__ float2 ld2(const float* a, int row, int col) const {
    return *reinterpret_cast<const float2*>(a + eidx(row, col));  // col even
  }
  // 2^(G_i - G_n) for the channel pair (c, c+1): one exp2 of the difference, which stays
  // finite whatever the decay (the shared memory of a second, 2^-G table goes to a second CTA)
  __device__ __forceinline__ float2 p2d2(int i, int n, int c) const {
    const float2 gi = ld2(sE, i, c), gn = ld2(sE, n, c);
    return make_float2(fast_exp2(gi.x - gn.x), fast_exp2(gi.y - gn.y));
  }

  // ---- key-key scores of this panel, accumulated into acc[piece] ----
  // Per-head decay: every piece is the exact product k'_i . k'_j (bf16 operands, fp32
  // accumulation; with an erase factor the fp32 product k'*b is split into bf16 hi + lo parts,
  // so the two bf16 products sum to the exact value); store_scores applies the per-pair decay
  // 2^(G_i - G_j) <= 1 in fp32.
  __device__ void scores_panel_head(float (&acc)[3][4], const __nv_bfloat16* sK) {
    int r, nts[3];
    score_pieces(warp, r, nts);
    if (16 * r >= len) return;  // whole row block beyond the chunk (chunk_intra.py:242-278)
    if constexpr (ERASE) {
      scores_head_erase(acc, sK, r, nts);
    } else {
      if (nts[2] >= 0)
        scores_head_np<3>(acc, sK, r, nts);
      else
        scores_head_np<2>(acc, sK, r, nts);
    }
  }
  // Exact bf16 products of NP pieces. Every ldmatrix row of a k-step starts at a multiple of 8
  // rows, so its swizzle key is lane & 7 for the whole loop: a fragment address is a per-thread
  // base plus (k-step chunk XOR a per-thread key), the k-step parts being constants.
  template <int NP>
  __device__ __forceinline__ void scores_head_np(float (&acc)[3][4], const __nv_bfloat16* sK, int r,
                                                 const int (&nts)[3]) {
    const uint32_t key = lane & 7;
    const uint32_t base = smem_u32(sK);
    const uint32_t a_row = base + (16 * r + (lane & 15)) * 128;      // A: rows 16r + (lane & 15)
    const uint32_t a_x = ((uint32_t(lane >> 4)) ^ key) << 4;         //    k chunk 2kk + (lane >> 4)
    const uint32_t b_x = ((uint32_t(lane >> 3) & 1u) ^ key) << 4;    // B: k chunk 2kk + ((lane >> 3) & 1)
    uint32_t b_row[NP];
#pragma unroll
    for (int s = 0; s < NP; ++s) b_row[s] = base + (8 * nts[s] + (lane & 7)) * 128;
#pragma unroll
    for (int kk = 0; kk < P / 16; ++kk) {
      const uint32_t pan = (kk >> 2) * 8192u;           // 64-column panel of the k-step
      const uint32_t cx = uint32_t((2 * kk) & 7) << 4;  // its first 16-byte chunk in the panel
      uint32_t a[4], bq[NP][2];
      ldsm_x4(a, a_row + pan + (cx ^ a_x));
#pragma unroll
      for (int s = 0; s < NP; ++s) ldsm_x2(bq[s], b_row[s] + pan + (cx ^ b_x));
#pragma unroll
      for (int s = 0; s < NP; ++s) mma_bf16_16816(acc[s], a, bq[s]);
    }
  }
  // with an erase factor: the fp32 product k'*b split into bf16 hi + lo parts
  __device__ __forceinline__ void scores_head_erase(float (&acc)[3][4], const __nv_bfloat16* sK, int r,
                                                    const int (&nts)[3]) {
    const int n_ref = 16 * r;
#pragma unroll 4
    for (int kk = 0; kk < P / 16; ++kk) {
      uint32_t a[4], bq[3][2];
      ldsm_x4(a, smem_u32(sK + pswz(n_ref + (lane & 15), 16 * kk + 8 * (lane >> 4))));
#pragma unroll
      for (int s = 0; s < 3; ++s)
        if (nts[s] >= 0)
          ldsm_x2(bq[s], smem_u32(sK + pswz(8 * nts[s] + (lane & 7), 16 * kk + 8 * ((lane >> 3) & 1))));
      uint32_t eb[4], hi[4], lo[4];
      ldsm_x4(eb, smem_u32(sB + pswz(n_ref + (lane & 15), 16 * kk + 8 * (lane >> 4))));
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float p0 = bf_lo(a[q]) * bf_lo(eb[q]), p1 = bf_hi(a[q]) * bf_hi(eb[q]);
        hi[q] = pack_bf16x2(p0, p1);
        lo[q] = pack_bf16x2(p0 - bf_lo(hi[q]), p1 - bf_hi(hi[q]));
      }
#pragma unroll
      for (int s = 0; s < 3; ++s)
        if (nts[s] >= 0) {
          mma_bf16_16816(acc[s], hi, bq[s]);
          mma_bf16_16816(acc[s], lo, bq[s]);
        }
    }
  }

  __device__ void scores_panel(float (&acc)[3][4], const __nv_bfloat16* sK) {
    if constexpr (HEAD) {
      scores_panel_head(acc, sK);
      return;
    }
    int r, nts[3];
    score_pieces(warp, r, nts);
    if (16 * r >= len) return;  // whole row block beyond the chunk (chunk_intra.py:242-278)
    const int g = lane >> 2, t = lane & 3;
    const int n_ref = 16 * r;
    const int i0 = n_ref + g, i1 = n_ref + g + 8;
    bool offdiag = false;
#pragma unroll
    for (int s = 0; s < 3; ++s) offdiag = offdiag || (nts[s] >= 0 && (nts[s] >> 1) < r);
    float lf0 = 0.f, lf1 = 0.f, rf[3] = {0.f, 0.f, 0.f};
    if constexpr (HEAD) {
      lf0 = i0 < len ? sLf[i0] : 0.f;
      lf1 = i1 < len ? sLf[i1] : 0.f;
#pragma unroll
      for (int s = 0; s < 3; ++s)
        if (nts[s] >= 0 && (nts[s] >> 1) < r) rf[s] = sRf[r * kTile + 8 * nts[s] + g];
    }
#pragma unroll 2
    for (int kk = 0; kk < P / 16; ++kk) {
      // all fragment loads of the k-step first
      uint32_t a[4], eb[4] = {0u, 0u, 0u, 0u}, bq[3][2];
      ldsm_x4(a, smem_u32(sK + pswz(n_ref + (lane & 15), 16 * kk + 8 * (lane >> 4))));
      if constexpr (ERASE)
        ldsm_x4(eb, smem_u32(sB + pswz(n_ref + (lane & 15), 16 * kk + 8 * (lane >> 4))));
#pragma unroll
      for (int s = 0; s < 3; ++s)
        if (nts[s] >= 0)
          ldsm_x2(bq[s], smem_u32(sK + pswz(8 * nts[s] + (lane & 7), 16 * kk + 8 * ((lane >> 3) & 1))));
      // left operand (tf32, two k8 slices) when the warp owns an off-diagonal piece, or per
      // channel (the diagonal pieces then use 3xTF32 as well)
      const int cA = 16 * kk + 2 * t;  // channel of the lo element of a[0]/a[1]
      float lv[2][4];
      uint32_t ah[2][4], al[2][4];
      if (!HEAD || offdiag) {
#pragma unroll
        for (int sl = 0; sl < 2; ++sl) {
          const uint32_t r0 = a[2 * sl], r1 = a[2 * sl + 1];  // rows g / g+8
          float x0 = bf_lo(r0), x1 = bf_hi(r0), x2 = bf_lo(r1), x3 = bf_hi(r1);
          if constexpr (ERASE) {
            x0 *= bf_lo(eb[2 * sl]);
            x1 *= bf_hi(eb[2 * sl]);
            x2 *= bf_lo(eb[2 * sl + 1]);
            x3 *= bf_hi(eb[2 * sl + 1]);
          }
          // (row g, k-slot t), (row g+8, k-slot t), (row g, k-slot t+4), (row g+8, k-slot t+4)
          if constexpr (HEAD) {
            lv[sl][0] = x0 * lf0;
            lv[sl][1] = x2 * lf1;
            lv[sl][2] = x1 * lf0;
            lv[sl][3] = x3 * lf1;
          } else {
            const int c = cA + 8 * sl;
            const float2 f0 = p2d2(i0, n_ref, c), f1 = p2d2(i1, n_ref, c);
            lv[sl][0] = i0 < len ? x0 * f0.x : 0.f;
            lv[sl][1] = i1 < len ? x2 * f1.x : 0.f;
            lv[sl][2] = i0 < len ? x1 * f0.y : 0.f;
            lv[sl][3] = i1 < len ? x3 * f1.y : 0.f;
          }
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            ah[sl][q] = to_tf32(lv[sl][q]);
            if constexpr (!HEAD) al[sl][q] = to_tf32(lv[sl][q] - __uint_as_float(ah[sl][q]));
          }
        }
      }
#pragma unroll
      for (int s = 0; s < 3; ++s) {
        if (nts[s] < 0) continue;
        const int nt = nts[s];
        const bool diag = (nt >> 1) == r;
        if constexpr (HEAD) {
          if (diag) {
            // exact bf16 products; the per-pair exponent is applied after the sum. With an
            // erase factor the fp32 product kb = k*b (16 significant bits) is split into bf16
            // hi + lo parts, so the two bf16 products sum to the exact fp32 value.
            if constexpr (ERASE) {
              uint32_t hi[4], lo[4];
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const float p0 = bf_lo(a[q]) * bf_lo(eb[q]), p1 = bf_hi(a[q]) * bf_hi(eb[q]);
                hi[q] = pack_bf16x2(p0, p1);
                lo[q] = pack_bf16x2(p0 - bf_lo(hi[q]), p1 - bf_hi(hi[q]));
              }
              mma_bf16_16816(acc[s], hi, bq[s]);
              mma_bf16_16816(acc[s], lo, bq[s]);
            } else {
              mma_bf16_16816(acc[s], a, bq[s]);
            }
          } else {
            uint32_t bb[2][2];
#pragma unroll
            for (int sl = 0; sl < 2; ++sl) {
              bb[sl][0] = to_tf32(bf_lo(bq[s][sl]) * rf[s]);
              bb[sl][1] = to_tf32(bf_hi(bq[s][sl]) * rf[s]);
            }
            mma_tf32_1688(acc[s], ah[0], bb[0]);
            mma_tf32_1688(acc[s], ah[1], bb[1]);
          }
        } else {
          const int j = 8 * nt + g;
#pragma unroll
          for (int sl = 0; sl < 2; ++sl) {
            const int c = cA + 8 * sl;
            const float2 f = p2d2(n_ref, j, c);
            const float y0 = bf_lo(bq[s][sl]) * f.x, y1 = bf_hi(bq[s][sl]) * f.y;
            uint32_t bh[2] = {to_tf32(y0), to_tf32(y1)};
            if (diag) {
              if (!fast) continue;  // exact pairwise evaluation below
              uint32_t bl[2] = {to_tf32(y0 - __uint_as_float(bh[0])), to_tf32(y1 - __uint_as_float(bh[1]))};
              mma_tf32_1688(acc[s], al[sl], bh);
              mma_tf32_1688(acc[s], ah[sl], bl);
            }
            mma_tf32_1688(acc[s], ah[sl], bh);
          }
        }
      }
    }
    if constexpr (!HEAD) {
      if (!fast) {
        // diagonal pieces with exact per-pair exponents (chunk_intra_token_parallel.py:114-123)
#pragma unroll
        for (int s = 0; s < 3; ++s) {
          if (nts[s] < 0 || (nts[s] >> 1) != r) continue;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int i = n_ref + g + ((q & 2) ? 8 : 0);
            const int j = 8 * nts[s] + 2 * t + (q & 1);
            float sum = 0.f;
            if (i < len && j < i) {
              for (int c = 0; c < P; ++c) {
                float kb = __bfloat162float(sK[pswz(i, c)]);
                if constexpr (ERASE) kb *= __bfloat162float(sB[pswz(i, c)]);
                sum += kb * __bfloat162float(sK[pswz(j, c)]) *
                       fast_exp2(sE[eidx(i, c)] - sE[eidx(j, c)]);
              }
            }
            acc[s][q] += sum;
          }
        }
      }
    }
  }

  // scores -> sA (strictly lower on the diagonal blocks; per-head diagonal scaled by 2^(G_i-G_j))
  __device__ void store_scores(const float (&acc)[3][4]) {
    if constexpr (HEAD) {
      store_scores_head(acc);
      return;
    }
    int r, nts[3];
    score_pieces(warp, r, nts);
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int s = 0; s < 3; ++s) {
      if (nts[s] < 0) continue;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int i = 16 * r + g + ((q & 2) ? 8 : 0);
        const int j = 8 * nts[s] + 2 * t + (q & 1);
        float x = acc[s][q];
        if constexpr (HEAD) x = (j < i && i < len) ? x * fast_exp2(sG[i] - sG[j]) : 0.f;
        if (j >= i || i >= len) x = 0.f;
        sA[i * Cfg::kLdA + j] = x;
      }
    }
  }

  // Per-head decay: a piece left of the diagonal block (columns j < 16r <= rows i) is scaled by
  // 2^(G_i - G_16r) * 2^(G_16r - G_j), the row and column factors of the unit's factor table
  // (both <= 1, as G does not increase along the chunk); a piece of the diagonal block by
  // 2^(G_i - G_j) per pair. Rows past the chunk and entries on or above the diagonal are zero.
  __device__ void store_scores_head(const float (&acc)[3][4]) {
    int r, nts[3];
    score_pieces(warp, r, nts);
    const int g = lane >> 2, t = lane & 3;
    const int i0 = 16 * r + g, i1 = i0 + 8;
    const bool v0 = i0 < len, v1 = i1 < len;
    const float G0 = sG[i0], G1 = sG[i1], L0 = sLf[i0], L1 = sLf[i1];
    float* row0 = sA + i0 * Cfg::kLdA;
    float* row1 = sA + i1 * Cfg::kLdA;
#pragma unroll
    for (int s = 0; s < 3; ++s) {
      if (nts[s] < 0) continue;
      const int j = 8 * nts[s] + 2 * t;
      float f00, f01, f10, f11;  // rows i0, i1 x columns j, j + 1
      if (nts[s] < 2 * r) {
        const float2 R = *reinterpret_cast<const float2*>(sRf + r * kTile + j);
        f00 = L0 * R.x;
        f01 = L0 * R.y;
        f10 = L1 * R.x;
        f11 = L1 * R.y;
      } else {
        const float2 Gj = *reinterpret_cast<const float2*>(sG + j);
        f00 = j < i0 ? fast_exp2(G0 - Gj.x) : 0.f;
        f01 = j + 1 < i0 ? fast_exp2(G0 - Gj.y) : 0.f;
        f10 = j < i1 ? fast_exp2(G1 - Gj.x) : 0.f;
        f11 = j + 1 < i1 ? fast_exp2(G1 - Gj.y) : 0.f;
      }
      *reinterpret_cast<float2*>(row0 + j) = v0 ? make_float2(acc[s][0] * f00, acc[s][1] * f01) : make_float2(0.f, 0.f);
      *reinterpret_cast<float2*>(row1 + j) = v1 ? make_float2(acc[s][2] * f10, acc[s][3] * f11) : make_float2(0.f, 0.f);
    }
  }

  // Blocked inverse of (I + A) (chunk_intra.py:326-395), run by warps 0-3 only (named
  // barrier 1). fp32 blocks stay in sA (diagonal in place, off-diagonal (r, s) in the unused
  // upper slot (s, r)); every finished block is also written as bf16 into sAi (rows >= len zero).
  __device__ void solve() {
    constexpr int LD = Cfg::kLdA, LDI = Cfg::kLdAi;
    if (warp < 2) {
      // Diagonal blocks by forward substitution in fp32: warp w inverts blocks 2w (lanes 0-15)
      // and 2w + 1 (lanes 16-31); lane c holds column c of X = (I + L)^-1 - I:
      //   X[j][c] = -(L[j][c] + sum_{c < i < j} L[j][i] X[i][c])   (X[i][c] = 0 for i <= c)
      // Right-looking: acc[j] collects the sum as soon as each X[i][c] is known, so the
      // dependent chain per row is one select and one fma. Columns are taken four at a time:
      // the group's own 4x4 triangle first, then every row below it with one 128-bit broadcast
      // load of its four entries.
      const int r = 2 * warp + (lane >> 4);
      const int c = lane & 15;
      float* blk = sA + (16 * r) * LD + 16 * r;
      float acc[16], x[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) acc[j] = blk[j * LD + c];  // L[j][c]; zero on and above the diagonal
#pragma unroll
      for (int j0 = 0; j0 < 16; j0 += 4) {
        float4 l[3];
#pragma unroll
        for (int q = 0; q < 3; ++q) l[q] = *reinterpret_cast<const float4*>(blk + (j0 + 1 + q) * LD + j0);
        x[j0] = (c < j0) ? -acc[j0] : 0.f;
        acc[j0 + 1] = fmaf(l[0].x, x[j0], acc[j0 + 1]);
        x[j0 + 1] = (c < j0 + 1) ? -acc[j0 + 1] : 0.f;
        acc[j0 + 2] = fmaf(l[1].y, x[j0 + 1], fmaf(l[1].x, x[j0], acc[j0 + 2]));
        x[j0 + 2] = (c < j0 + 2) ? -acc[j0 + 2] : 0.f;
        acc[j0 + 3] = fmaf(l[2].z, x[j0 + 2], fmaf(l[2].y, x[j0 + 1], fmaf(l[2].x, x[j0], acc[j0 + 3])));
        x[j0 + 3] = (c < j0 + 3) ? -acc[j0 + 3] : 0.f;
#pragma unroll
        for (int j = j0 + 4; j < 16; ++j) {
          const float4 m = *reinterpret_cast<const float4*>(blk + j * LD + j0);
          acc[j] = fmaf(m.w, x[j0 + 3], fmaf(m.z, x[j0 + 2], fmaf(m.y, x[j0 + 1], fmaf(m.x, x[j0], acc[j]))));
        }
      }
      __syncwarp();
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float v = x[j] + (j == c ? 1.f : 0.f);
        blk[j * LD + c] = v;
        sAi[(16 * r + j) * LDI + 16 * r + c] = __float2bfloat16_rn((16 * r + j < len) ? v : 0.f);
      }
    }
    named_sync(1, 128);
    auto Dg = [&](int r) { return sA + (16 * r) * LD + 16 * r; };         // Ai_rr
    auto Ak = [&](int r, int s) { return sA + (16 * r) * LD + 16 * s; };  // Akk_rs, r > s
    auto Ao = [&](int r, int s) { return sA + (16 * s) * LD + 16 * r; };  // Ai_rs kept at (s, r)
    auto Ab = [&](int r, int s) { return sAi + (16 * r) * LDI + 16 * s; };
    float acc[2][4];
    if (warp < 3) {  // Ai_{s+1,s} = -(Ai_{s+1,s+1} Akk_{s+1,s}) Ai_{s,s}
      const int s = warp;
      float* tmp = (s == 0) ? Ao(2, 0) : (s == 1) ? Ao(3, 1) : Ao(3, 0);
      zero_acc(acc);
      warp_tf32_16x16x16(acc, Dg(s + 1), LD, Ak(s + 1, s), LD, lane);
      warp_store_f32(tmp, LD, acc, lane);
      __syncwarp();
      zero_acc(acc);
      warp_tf32_16x16x16(acc, tmp, LD, Dg(s), LD, lane);
      warp_store_block(Ao(s + 1, s), LD, Ab(s + 1, s), LDI, acc, lane, -1.f, 16 * (s + 1), len);
    }
    named_sync(1, 128);
    // Ai20 = -Ai22 (Akk20 Ai00 + Akk21 Ai10), Ai31 = -Ai33 (Akk31 Ai11 + Akk32 Ai21):
    // one dot per warp into the scratch blocks, then the two outer products
    {
      constexpr int LS = 16;
      // warp 0: Akk20 Ai00, 1: Akk21 Ai10, 2: Akk31 Ai11, 3: Akk32 Ai21
      const int lr = 2 + (warp >> 1), ls = (warp >> 1) + (warp & 1);
      const float* rhs = (warp & 1) ? Ao(ls, ls - 1) : Dg(ls);
      zero_acc(acc);
      warp_tf32_16x16x16(acc, Ak(lr, ls), LD, rhs, LD, lane);
      warp_store_f32(sScr + warp * 256, LS, acc, lane);
      named_sync(1, 128);
      if (warp < 2) {
        const int r = warp + 2;
        zero_acc(acc);
        warp_tf32_A_sumB(acc, Dg(r), LD, sScr + (2 * warp) * 256, sScr + (2 * warp + 1) * 256, nullptr, LS, lane);
        warp_store_block(Ao(r, r - 2), LD, Ab(r, r - 2), LDI, acc, lane, -1.f, 16 * r, len);
      }
      named_sync(1, 128);
      // Ai30 = -Ai33 (Akk30 Ai00 + Akk31 Ai10 + Akk32 Ai20)
      if (warp < 3) {
        // warp s: Akk3s Ai_s0
        const float* rhs = (warp == 0) ? Dg(0) : Ao(warp, 0);
        zero_acc(acc);
        warp_tf32_16x16x16(acc, Ak(3, warp), LD, rhs, LD, lane);
        warp_store_f32(sScr + warp * 256, LS, acc, lane);
      }
      named_sync(1, 128);
      if (warp == 0) {
        zero_acc(acc);
        warp_tf32_A_sumB(acc, Dg(3), LD, sScr, sScr + 256, sScr + 512, LS, lane);
        warp_store_block(nullptr, LD, Ab(3, 0), LDI, acc, lane, -1.f, 48, len);
      }
    }
  }

  // zero rows [len, 64) of a [64][P] tile; threads [T0, T0 + NTH)
  template <int T0, int NTH>
  __device__ void zero_rows(__nv_bfloat16* t) {
    constexpr int kChunks = kTile * P / 8;
    for (int i = tid - T0 + len * (P / 8); i < kChunks; i += NTH)
      *reinterpret_cast<uint4*>(t + pswz(i / (P / 8), (i % (P / 8)) * 8)) = make_uint4(0, 0, 0, 0);
  }

  // u operand in place: vt = bf16(v * w) (wy_fast.py:98-100), by default of the value tiles sV and
  // sW; threads [T0, T0 + NTH); in the TMA path rows past the chunk become zero
  template <int T0, int NTH>
  __device__ void stage_u(const IntraParams& p, __nv_bfloat16* vt = nullptr, const __nv_bfloat16* wt = nullptr) {
    if (vt == nullptr) vt = sV;
    if (wt == nullptr) wt = sW;
    constexpr int kChunks = kTile * P / 8;
    static_assert(kChunks % NTH == 0, "chunks per thread");
    if (p.write == nullptr) {
      if constexpr (kTma) {  // rows past the chunk hold the next sample's tokens: zero them
        if (len < kTile) zero_rows<T0, NTH>(vt);
      }
      return;
    }
    using Wk = Walk<NTH>;
    int row0, col;
    const uint32_t off = walk_start<T0>(row0, col);
    unsigned char* vb = reinterpret_cast<unsigned char*>(vt) + off;
    const unsigned char* wb = reinterpret_cast<const unsigned char*>(wt) + off;
#pragma unroll
    for (int j = 0; j < Wk::kSteps; ++j) {
      uint4 vv = make_uint4(0, 0, 0, 0);
      if (!kTma || row0 + j * Wk::kRows < len) {
        vv = *reinterpret_cast<const uint4*>(vb + j * Wk::kStride);
        const uint4 ww = *reinterpret_cast<const uint4*>(wb + j * Wk::kStride);
        vv.x = mul_bf16x2(vv.x, ww.x);
        vv.y = mul_bf16x2(vv.y, ww.y);
        vv.z = mul_bf16x2(vv.z, ww.z);
        vv.w = mul_bf16x2(vv.w, ww.w);
      }
      *reinterpret_cast<uint4*>(vb + j * Wk::kStride) = vv;
    }
  }

  // w operand bf16( bf16(k*b) * 2^G ) in place of k, or into wdst (wy_fast.py:110-116),
  // kg = bf16(k 2^(G_last-G)) to global (wy_fast.py:125-139) and 2^G_last; threads [T0, T0 + NTH)
  template <int T0, int NTH>
  __device__ void stage_w_kg(__nv_bfloat16* kt, __nv_bfloat16* gKG, float* gEl, int c0,
                             __nv_bfloat16* wdst = nullptr) {
    const int last = len - 1;
    using Wk = Walk<NTH>;
    int row0, col;
    const uint32_t off = walk_start<T0>(row0, col);
    unsigned char* kb = reinterpret_cast<unsigned char*>(kt) + off;
    unsigned char* wb = reinterpret_cast<unsigned char*>(wdst != nullptr ? wdst : kt) + off;
    unsigned char* gb = reinterpret_cast<unsigned char*>(gKG) + (c0 >> 6) * 8192 + off;  // same layout
    const unsigned char* bb = reinterpret_cast<const unsigned char*>(sB) + off;
#pragma unroll
    for (int j = 0; j < Wk::kSteps; ++j) {
      const int row = row0 + j * Wk::kRows;
      uint4 kv = *reinterpret_cast<const uint4*>(kb + j * Wk::kStride);
      uint32_t* kw = reinterpret_cast<uint32_t*>(&kv);
      uint4 kgv;
      uint32_t* kgw = reinterpret_cast<uint32_t*>(&kgv);
      uint4 bv = make_uint4(0, 0, 0, 0);
      if constexpr (ERASE) bv = *reinterpret_cast<const uint4*>(bb + j * Wk::kStride);
      const uint32_t* bw = reinterpret_cast<const uint32_t*>(&bv);
      uint64_t eh = 0, qh = 0;
      float gr[8], gl[8];  // per channel: G of this row and of the last token, channels col..col+7
      if constexpr (HEAD) {
        eh = f32x2_splat(sEh[row]);
        qh = f32x2_splat(sKgf[row]);
      } else {
#pragma unroll
        for (int h4 = 0; h4 < 2; ++h4) {
          const float4 a = *reinterpret_cast<const float4*>(sE + eidx(row, col + 4 * h4));
          const float4 b = *reinterpret_cast<const float4*>(sE + eidx(last, col + 4 * h4));
          gr[4 * h4] = a.x, gr[4 * h4 + 1] = a.y, gr[4 * h4 + 2] = a.z, gr[4 * h4 + 3] = a.w;
          gl[4 * h4] = b.x, gl[4 * h4 + 1] = b.y, gl[4 * h4 + 2] = b.z, gl[4 * h4 + 3] = b.w;
        }
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const uint64_t k2 = bf16x2_to_f32x2(kw[e]);
        uint64_t e2, q2;
        if constexpr (HEAD) {
          e2 = eh;
          q2 = qh;
        } else {
          // 2^G (w operand) and 2^(G_last - G) (kg), wy_fast.py:110-116,125-139
          e2 = f32x2_pack(fast_exp2(gr[2 * e]), fast_exp2(gr[2 * e + 1]));
          q2 = row < len ? f32x2_pack(fast_exp2(gl[2 * e] - gr[2 * e]), fast_exp2(gl[2 * e + 1] - gr[2 * e + 1]))
                         : f32x2_pack(0.f, 0.f);
        }
        kgw[e] = f32x2_to_bf16x2(mul_f32x2(k2, q2));
        if constexpr (ERASE) {
          const float k0 = bf_lo(kw[e]), k1 = bf_hi(kw[e]);
          kw[e] = f32x2_to_bf16x2(mul_f32x2(f32x2_pack(bf16_round(k0 * bf_lo(bw[e])), bf16_round(k1 * bf_hi(bw[e]))), e2));
        } else {
          kw[e] = f32x2_to_bf16x2(mul_f32x2(k2, e2));
        }
      }
      *reinterpret_cast<uint4*>(wb + j * Wk::kStride) = kv;  // w operand (in place of k by default)
      *reinterpret_cast<uint4*>(gb + j * Wk::kStride) = kgv;
    }
    const int j = tid - T0;
    if (j >= 0 && j < P) {
      if constexpr (HEAD)
        gEl[c0 + j] = sSeg[0];
      else
        gEl[c0 + j] = fast_exp2(sE[eidx(last, j)]);
    }
  }

  // Both WY products in one pass: w = A^-1 . (w operand in kt) -> dw and
  // u = A^-1 . (u operand in sV) -> du, all [64][P] pswz tiles; the A^-1 fragment of a k-step
  // feeds both. Row block r needs k-steps 0..r: warps 0-3 take row blocks 3 and 0, warps 4-7
  // blocks 2 and 1, each in column quarter warp % 4 -- the same work on every warp. The sources
  // are only read and the destinations are other tiles: no barrier between reads and writes.
  template <int R>
  __device__ __forceinline__ void wy_block(const __nv_bfloat16* kt, __nv_bfloat16* dw, __nv_bfloat16* du) {
    constexpr int CW = P / 4;    // columns of a quarter
    constexpr int NTW = CW / 8;  // 8-column tiles of a quarter
    // The quarter starts at 16-byte chunk cq of a row; the swizzle key of every fragment row is
    // lane & 7 (fragment rows start at multiples of 8), and the chunk offsets within a 64-column
    // panel (cq & 7, the tile np, the lane's half) occupy disjoint bits, so each fragment
    // address is a per-thread base plus (constant XOR a per-thread key).
    const int cq = (warp & 3) * (CW / 8);
    const uint32_t key = lane & 7;
    const uint32_t b_off = (cq >> 3) * 8192u + (lane & 15) * 128u;
    const uint32_t b_x = ((uint32_t(cq & 7) + uint32_t(lane >> 4)) ^ key) << 4;
    const uint32_t kt_b = smem_u32(kt) + b_off, v_b = smem_u32(sV) + b_off;
    const uint32_t a_b = smem_u32(sAi + (16 * R + (lane & 15)) * Cfg::kLdAi + 8 * (lane >> 4));
    float aw[NTW][4], au[NTW][4];
#pragma unroll
    for (int i = 0; i < NTW; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) aw[i][j] = au[i][j] = 0.f;
#pragma unroll
    for (int ks = 0; ks <= R; ++ks) {
      uint32_t a[4], bw[NTW / 2][4], bu[NTW / 2][4];
      ldsm_x4(a, a_b + ks * 32u);
#pragma unroll
      for (int np = 0; np < NTW; np += 2) {
        const uint32_t o = ks * 2048u + ((uint32_t(np) << 4) ^ b_x);
        ldsm_x4_t(bw[np / 2], kt_b + o);
        ldsm_x4_t(bu[np / 2], v_b + o);
      }
#pragma unroll
      for (int np = 0; np < NTW; np += 2) {
        const uint32_t w0[2] = {bw[np / 2][0], bw[np / 2][1]}, w1[2] = {bw[np / 2][2], bw[np / 2][3]};
        const uint32_t u0[2] = {bu[np / 2][0], bu[np / 2][1]}, u1[2] = {bu[np / 2][2], bu[np / 2][3]};
        mma_bf16_16816(aw[np], a, w0);
        mma_bf16_16816(aw[np + 1], a, w1);
        mma_bf16_16816(au[np], a, u0);
        mma_bf16_16816(au[np + 1], a, u1);
      }
    }
    // bf16 accumulators as 8x8 matrices (tile nt, rows 16R + 8 half ..): stmatrix x4 takes tiles
    // nt, nt + 1 with both halves; lane l addresses row l % 8 of matrix l / 8 = (tile, half)
    const int mj = lane & 7, mh = (lane >> 3) & 1, mt = lane >> 4;
    const uint32_t m_off = (cq >> 3) * 8192u + (16 * R + 8 * mh + mj) * 128u +
                           ((uint32_t((cq & 7) | mt) ^ uint32_t(mj)) << 4);
    const uint32_t dwa = smem_u32(dw) + m_off, dua = smem_u32(du) + m_off;
#pragma unroll
    for (int nt = 0; nt < NTW; nt += 2) {
      const uint32_t o = uint32_t(nt) << 4;  // tiles nt, nt + 1: chunk bit 1 flips
      stsm_x4(dwa ^ o, pack_bf16x2(aw[nt][0], aw[nt][1]), pack_bf16x2(aw[nt][2], aw[nt][3]),
              pack_bf16x2(aw[nt + 1][0], aw[nt + 1][1]), pack_bf16x2(aw[nt + 1][2], aw[nt + 1][3]));
      stsm_x4(dua ^ o, pack_bf16x2(au[nt][0], au[nt][1]), pack_bf16x2(au[nt][2], au[nt][3]),
              pack_bf16x2(au[nt + 1][0], au[nt + 1][1]), pack_bf16x2(au[nt + 1][2], au[nt + 1][3]));
    }
  }
  __device__ void wy_products(const __nv_bfloat16* kt, __nv_bfloat16* dw, __nv_bfloat16* du) {
    if (warp < 4) {
      wy_block<3>(kt, dw, du);
      wy_block<0>(kt, dw, du);
    } else {
      wy_block<2>(kt, dw, du);
      wy_block<1>(kt, dw, du);
    }
  }

  // shared [64][P] tile (pswz) -> global [64][D] tile at column c0: shared tiles use the panel
  // layout of the global tiles (64-column panels of 128-byte swizzled rows), so the tile is the
  // same bytes at panel c0 / 64 and moves with one bulk copy, issued by thread 0 after the
  // writers fenced their stores to the async proxy and a barrier. Thread 0 waits for the read
  // (bulk_wait_read) before the shared tile is overwritten.
  __device__ __forceinline__ void store_tile_async(__nv_bfloat16* out, int c0, const __nv_bfloat16* src) {
    if (tid == 0) {
      bulk_s2g(out + (c0 >> 6) * (kTile * 64), smem_u32(src), static_cast<uint32_t>(Cfg::kTileB));
      bulk_commit();
    }
  }

  // ---- persistent loop over (chunk, head) units: unit = chunk * H + head ----
  __device__ void set_unit(const IntraParams& p, int64_t unit) {
    const int c = static_cast<int>(unit / p.H);
    h = static_cast<int>(unit % p.H);
    const ChunkDesc d = p.table[c];
    tok0 = d.tok0;
    len = d.len;
  }

  __device__ void run(const IntraParams& p) {
    griddep_wait();               // the chunk table and every input are complete
    griddep_launch_dependents();  // the scan may set up while the last units run
    const int64_t units = (int64_t)p.hdr->num_chunks * p.H;
    int64_t unit = blockIdx.x;
    if (unit >= units) return;
    row_stride = (int64_t)p.H * D;
    __nv_bfloat16* kcur = sK;

    // the decay panel of unit (tk0, ln, hd) by threads [T0, T0 + NTH)
    auto load_decay_for = [&](auto t0_tag, auto nth_tag, int c0, int tk0, int ln, int hd) {
      constexpr int T0 = decltype(t0_tag)::value, NTH = decltype(nth_tag)::value;
      const float* base = p.g + (int64_t)tk0 * row_stride + (int64_t)hd * D + c0;
      constexpr int kChunks = kTile * P / 4;
#pragma unroll
      for (int i = tid - T0; i < kChunks; i += NTH) {
        const int row = i / (P / 4), col = (i % (P / 4)) * 4;
        const bool valid = row < ln;
        cp_async16_zfill(sE + eidx(row, col), valid ? base + (int64_t)row * row_stride + col : p.g, valid);
      }
    };
    auto load_decay = [&](int c0) {
      load_decay_for(std::integral_constant<int, 0>{}, std::integral_constant<int, NT>{}, c0, tok0, len, h);
    };
    // per channel with the solve / staging split, the staging warps load the next unit's decay
    // table as soon as their staging is done (the table is free then), a whole WY phase before
    // the unit starts; the key tile follows at the unit's end as before
    constexpr bool kEarlyDecay = kOverlap && !HEAD;
    auto load_key_panel = [&](int c0, bool decay) {
      load_tile(kcur, p.k, c0, p.sk);
      if constexpr (ERASE) load_tile(sB, p.erase, c0, row_stride);
      if constexpr (!HEAD)
        if (decay) load_decay(c0);
    };
    auto load_value_panel = [&](int c0) {
      load_tile(sV, p.v, c0, p.sv);
      if (p.write != nullptr) load_tile(sW, p.write, c0, p.sw);
    };
    // with the solve / staging split only the staging warps use v and w: they load them alone
    auto load_value_panel_staging = [&]() {
      if (warp >= 4) {
        load_tile_for<128, 128>(sV, p.v, 0, tok0, len, h, p.sv);
        if (p.write != nullptr) load_tile_for<128, 128>(sW, p.write, 0, tok0, len, h, p.sw);
      }
    };
    auto prepare_key_panel = [&](int c0) {  // after the key panel landed
      __syncthreads();
      if (p.beta_layout != 0) {
        fold_beta(p, kcur, c0);
        __syncthreads();
      }
      if constexpr (!HEAD) channel_tables();
    };

    // per-head decay with overlap: the staging warps compute the next unit's factors
    constexpr bool kNextFactors = kOverlap && HEAD;
    bool first = true;
    set_unit(p, unit);
    load_key_panel(0, true);
    cp_async_commit();
    pre = 0;
    fetch_scalars(p, tok0, len, h, sPre, 0);
    for (;;) {
      const int64_t next = unit + gridDim.x;
      const bool has_next = next < units;
      const int64_t chunk_head = unit;  // == chunk * H + head
      __nv_bfloat16* gW = p.W + chunk_head * kTile * D;
      __nv_bfloat16* gU = p.U + chunk_head * kTile * D;
      __nv_bfloat16* gKG = p.KG + chunk_head * kTile * D;
      float* gEl = p.Elast + chunk_head * D;

      if constexpr (kOverlap) load_value_panel_staging();
      cp_async_commit();
      if constexpr (HEAD) {
        use_factors(pre);
        if (!kNextFactors || first) {
          __syncthreads();  // the unit's scalars are visible
          if (warp == 0) head_factors(sPre + pre * 2 * kTile, sFac + pre * Cfg::kSmall, len);
        }
        first = false;
      }

      float acc[3][4];
#pragma unroll
      for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;

      // ---- key-key scores over the channel panels ----
      for (int pn = 0; pn < Cfg::kPanels; ++pn) {
        if (pn > 0) {
          __syncthreads();
          load_key_panel(pn * P, true);
          cp_async_commit();
          cp_async_wait<0>();
        } else {
          // the key group landed (warps 4-7 also have the younger value group in flight)
          if (kOverlap && warp < 4)
            cp_async_wait<0>();
          else
            cp_async_wait<1>();
        }
        prepare_key_panel(pn * P);
        scores_panel(acc, kcur);
        // D = 256: panel 0's w operand (and kg, 2^G_last) now, while its keys and decay table are
        // resident (it needs neither the scores nor the inverse), into the value tile, which is
        // free until the u operands; the next panel's load waits for every thread (barrier above)
        if constexpr (Cfg::kPanels == 2)
          if (pn == 0) stage_w_kg<0, NT>(kcur, gKG, gEl, 0, sV);
      }
      store_scores(acc);  // nothing reads the score buffer while the scores are formed
      if constexpr (!kOverlap) cp_async_wait<0>();  // every thread's copies of v and w are complete
      __syncthreads();

      if constexpr (kOverlap) {
        // warps 0-3: blocked solve; warps 4-7: prefetch of the next unit's k, u operand
        // (v * w in place), then w operand (in place of k) and kg
        if (warp < 4) {
          solve();
        } else {
          cp_async_wait<0>();  // this thread's copies of v and w
          named_sync(2, 128);  // ... and every staging thread's
          float ng = 0.f;  // next unit's scalars, loaded now, stored after stage_u
          uint32_t nb = 0u;
          if (has_next) {
            const int c2 = static_cast<int>(next / p.H), h2 = static_cast<int>(next % p.H);
            const ChunkDesc d2 = p.table[c2];
            load_scalars(p, d2.tok0, d2.len, h2, 128, ng, nb);
          }
          stage_u<128, 128>(p);
          if (has_next) store_scalars(sPre + (pre ^ 1) * 2 * kTile, 128, ng, nb);
          named_sync(2, 128);
          stage_w_kg<128, 128>(kcur, gKG, gEl, 0);
          if constexpr (kNextFactors) {
            if (has_next && warp == 7) {
              const ChunkDesc d2 = p.table[static_cast<int>(next / p.H)];
              head_factors(sPre + (pre ^ 1) * 2 * kTile, sFac + (pre ^ 1) * Cfg::kSmall, d2.len);
            }
          }
          if constexpr (kEarlyDecay) {
            if (has_next) {
              named_sync(2, 128);  // every staging thread is done with this unit's table
              const int c2 = static_cast<int>(next / p.H), h2 = static_cast<int>(next % p.H);
              const ChunkDesc d2 = p.table[c2];
              load_decay_for(std::integral_constant<int, 128>{}, std::integral_constant<int, 128>{}, 0, d2.tok0,
                             d2.len, h2);
              cp_async_commit();
            }
          }

        }
        __syncthreads();
        // one pass of both products: w = A^-1 . w operand into the w-gate tile (free), u =
        // A^-1 . bf16(v*w) into the score buffer (free once the solve is done)
        __nv_bfloat16* sA16 = reinterpret_cast<__nv_bfloat16*>(sA);
        wy_products(kcur, sW, sA16);
        fence_proxy_async_smem();
        __syncthreads();
        store_tile_async(gW, 0, sW);
        store_tile_async(gU, 0, sA16);
        if (tid == 0) bulk_wait_read();  // before the next unit reloads sW and stores its scores
      } else {
        // ---- D = 256: panel 1's w operand (its keys and decay table are resident) on warps 4-7
        // while warps 0-3 solve; panel 0's is in the value tile sV since the score loop. One pass
        // of both WY products then gives w of both panels ----
        static_assert(Cfg::kPanels == 2, "the panel pair of D = 256");
        __nv_bfloat16* sA16 = reinterpret_cast<__nv_bfloat16*>(sA);  // free once the solve is done
        // the decay table (free once both w operands are staged), or with a per-head decay (no
        // table) the score buffer again: loaded only after the w stores have read it
        __nv_bfloat16* sE16 = reinterpret_cast<__nv_bfloat16*>(sE);
        if (warp < 4)
          solve();
        else
          stage_w_kg<128, 128>(kcur, gKG, gEl, P);
        __syncthreads();
        wy_products(kcur, sW, sA16);  // w of panel 1 -> sW, of panel 0 (sV) -> the score buffer
        fence_proxy_async_smem();
        __syncthreads();
        store_tile_async(gW, P, sW);
        store_tile_async(gW, 0, sA16);
        if (tid == 0) bulk_wait_read();  // before the u pass overwrites sW and the score buffer
        __syncthreads();
        // ---- u of both panels: v and the write gate of panel 0 into the value tiles, of panel 1
        // into the key tile and the decay table; one pass of both products ----
        load_tile(sV, p.v, 0, p.sv);
        if (p.write != nullptr) load_tile(sW, p.write, 0, p.sw);
        load_tile(kcur, p.v, P, p.sv);
        if (p.write != nullptr) load_tile(sE16, p.write, P, p.sw);
        cp_async_commit();
        cp_async_wait<0>();
        __syncthreads();
        stage_u<0, NT>(p);              // sV = bf16(v0 * w0)
        stage_u<0, NT>(p, kcur, sE16);  // kcur = bf16(v1 * w1)
        __syncthreads();
        wy_products(kcur, sW, sA16);  // u of panel 1 -> sW, of panel 0 (sV) -> the score buffer
        fence_proxy_async_smem();
        __syncthreads();
        store_tile_async(gU, P, sW);
        store_tile_async(gU, 0, sA16);
        if (tid == 0) bulk_wait_read();
        __syncthreads();  // the next unit's loads overwrite the tiles the stores read
      }
      if (!has_next) {
        if (tid == 0) bulk_wait_all();
        break;
      }
      unit = next;
      set_unit(p, unit);
      __syncthreads();  // the last tile stores read shared memory the next unit overwrites
      if constexpr (!kOverlap) fetch_scalars(p, tok0, len, h, sPre + (pre ^ 1) * 2 * kTile, 0);
      pre ^= 1;
      load_key_panel(0, !kEarlyDecay);
      cp_async_commit();
    }
  }

  // ---- the persistent loop of the TMA configuration (per-head decay, no erase, D <= 128) ----
  // Thread 0 issues every tile copy: at the top of a unit the unit's v and write tiles and the
  // next unit's k tile (into the spare k buffer), each completing on an mbarrier that the
  // consuming threads wait on; at the end the w and u tiles as bulk stores that are waited for
  // only where their buffers are loaded again. The chunk table entry of the unit after next and
  // the next unit's per-token scalars are loaded into registers at the top as well and consumed
  // one phase or one unit later, so no global-load latency sits on the unit's chain.
  __device__ void run_tma(const IntraParams& p) {
    griddep_wait();               // the chunk table and every input are complete
    griddep_launch_dependents();  // the scan may set up while the last units run
    // units advance by the grid size as (chunk, head) pairs, without divisions
    const int nch = p.hdr->num_chunks;
    const int H = p.H;
    int c = static_cast<int>(blockIdx.x / H);
    h = static_cast<int>(blockIdx.x % H);
    if (c >= nch) return;
    const int dc = static_cast<int>(gridDim.x / H), dh = static_cast<int>(gridDim.x % H);
    auto advance = [&](int& cc, int& hh) {
      hh += dh;
      cc += dc;
      if (hh >= H) {
        hh -= H;
        cc += 1;
      }
    };
    row_stride = (int64_t)H * D;
    auto mb = [&](int i) { return sMb + 8u * i; };
    auto tma_tile = [&](__nv_bfloat16* dst, const CUtensorMap* map, int tk0, int hd, uint32_t bar) {
#pragma unroll
      for (int b = 0; b < P / 64; ++b) tma_load_2d(smem_u32(dst) + b * 8192u, map, hd * D + 64 * b, tk0, bar);
    };
    if (tid == 0) {
      mbar_init(mb(0), 1);
      mbar_init(mb(1), 1);
      mbar_init(mb(2), 1);
      mbar_fence_init();
    }
    __syncthreads();
    __nv_bfloat16* kcur = sK;
    __nv_bfloat16* kspare = sO;
    int kb = 0;         // mbarrier of kcur
    uint32_t kph = 0;   // bit b: phase parity of k buffer b's next completion
    uint32_t vph = 0;   // phase parity of the v + write barrier
    bool ok = true;     // every copy wait of this thread completed
    {
      const ChunkDesc d0 = p.table[c];
      tok0 = d0.tok0;
      len = d0.len;
    }
    int nc = c, nh = h;  // the next unit
    advance(nc, nh);
    ChunkDesc nd{};      // table entry of the next unit
    if (nc < nch) nd = p.table[nc];
    if (tid == 0) {
      mbar_expect_tx(mb(0), kTileBytes);
      tma_tile(kcur, &p.k_map, tok0, h, mb(0));
    }
    pre = 0;
    fetch_scalars(p, tok0, len, h, sPre, 0);
    bool first = true;
    for (;;) {
      const bool has_next = nc < nch;
      const int hn = nh;
      int n2c = nc, n2h = nh;  // the unit after next: its table entry is needed one unit from now
      advance(n2c, n2h);
      ChunkDesc nn{};
      if (n2c < nch) nn = p.table[n2c];
      const int64_t unit = (int64_t)c * H + h;
      __nv_bfloat16* gW = p.W + unit * kTile * D;
      __nv_bfloat16* gU = p.U + unit * kTile * D;
      __nv_bfloat16* gKG = p.KG + unit * kTile * D;
      float* gEl = p.Elast + unit * D;

      if (tid == 0) {
        // sV and sW held the previous unit's WY operands, read before its last barrier
        fence_proxy_async_smem();
        mbar_expect_tx(mb(2), p.write != nullptr ? 2 * kTileBytes : kTileBytes);
        tma_tile(sV, &p.v_map, tok0, h, mb(2));
        if (p.write != nullptr) tma_tile(sW, &p.w_map, tok0, h, mb(2));
      }
      float ng = 0.f;  // next unit's scalars (threads 128..191), stored in the staging
      uint32_t nb = 0u;
      if (has_next) load_scalars(p, nd.tok0, nd.len, hn, 128, ng, nb);
      use_factors(pre);
      if (first) {
        __syncthreads();  // the unit's scalars are visible
        if (warp == 0) head_factors(sPre, sFac, len);
        first = false;
      }

      float acc[3][4];
#pragma unroll
      for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
      // ---- key-key scores: k landed; fold sqrt(beta) (zeroing rows past the chunk) ----
      ok &= mbar_wait(mb(kb), (kph >> kb) & 1u);
      kph ^= 1u << kb;
      if (p.beta_layout != 0)
        fold_beta(p, kcur, 0);
      else if (len < kTile)
        zero_rows<0, NT>(kcur);
      if (tid == 0) {
        // the previous unit's u and w have left the score buffer and kspare: the next unit's k
        bulk_wait_read();
        if (has_next) {
          mbar_expect_tx(mb(kb ^ 1), kTileBytes);
          tma_tile(kspare, &p.k_map, nd.tok0, hn, mb(kb ^ 1));
        }
      }
      __syncthreads();
      scores_panel(acc, kcur);
      store_scores(acc);
      __syncthreads();

      // warps 0-3: blocked solve; warps 4-7: u operand (v * w in place), the next unit's
      // scalars, then w operand (into the write-gate tile, read by the u operand), kg and the
      // next unit's decay factors
      if (warp < 4) {
        solve();
      } else {
        ok &= mbar_wait(mb(2), vph);
        stage_u<128, 128>(p);
        if (has_next) store_scalars(sPre + (pre ^ 1) * 2 * kTile, 128, ng, nb);
        named_sync(2, 128);
        stage_w_kg<128, 128>(kcur, gKG, gEl, 0, sW);
        if (has_next && warp == 7)
          head_factors(sPre + (pre ^ 1) * 2 * kTile, sFac + (pre ^ 1) * Cfg::kSmall, nd.len);
      }
      vph ^= 1u;
      __syncthreads();
      // w into the k tile (read by the scores and the staging), u into the score buffer (free
      // once the solve is done); both leave by bulk copies that nothing waits for before the
      // next unit's fold, after which the k tile of the unit after it is loaded into this buffer
      wy_products(sW, kcur, reinterpret_cast<__nv_bfloat16*>(sA));
      fence_proxy_async_smem();
      __syncthreads();  // every product written, every source tile read
      if (tid == 0) {
        bulk_s2g(gW, smem_u32(kcur), kTileBytes);
        bulk_commit();
        bulk_s2g(gU, smem_u32(sA), kTileBytes);
        bulk_commit();
      }
      if (!has_next) {
        if (tid == 0) bulk_wait_all();
        break;
      }
      c = nc;
      h = nh;
      tok0 = nd.tok0;
      len = nd.len;
      nc = n2c;
      nh = n2h;
      nd = nn;
      pre ^= 1;
      __nv_bfloat16* tmp = kcur;
      kcur = kspare;
      kspare = tmp;
      kb ^= 1;
    }
    if (!ok) atomicOr(&p.hdr->status, 4);  // a tile never arrived: results are not valid
  }
};

template <int D, bool HEAD, bool ERASE>
__global__ void __launch_bounds__(256, 2) intra_kernel(const __grid_constant__ IntraParams p) {
  extern __shared__ __align__(1024) unsigned char smem_intra[];
  using Cfg = IntraCfg<D, HEAD, ERASE>;
  IntraKernel<D, HEAD, ERASE> k;
  constexpr uint32_t kA = Cfg::kAlign;
  unsigned char* base = smem_intra + ((kA - (smem_u32(smem_intra) & (kA - 1))) & (kA - 1));
  k.sK = reinterpret_cast<__nv_bfloat16*>(base + Cfg::offK);
  k.sB = reinterpret_cast<__nv_bfloat16*>(base + Cfg::offB);
  k.sV = reinterpret_cast<__nv_bfloat16*>(base + Cfg::offV);
  k.sW = reinterpret_cast<__nv_bfloat16*>(base + Cfg::offW);
  k.sO = Cfg::kNeedO ? reinterpret_cast<__nv_bfloat16*>(base + Cfg::offO) : nullptr;
  k.sE = reinterpret_cast<float*>(base + Cfg::offE);
  k.sA = reinterpret_cast<float*>(base + Cfg::offA);
  k.sAi = reinterpret_cast<__nv_bfloat16*>(base + Cfg::offAi);
  __shared__ __align__(16) float s_fac[Cfg::kFacFloats];
  __shared__ __align__(16) float s_scr[4 * 256];
  k.sScr = s_scr;
  k.sFac = s_fac;
  k.use_factors(0);
  __shared__ __align__(16) float s_pre[4 * kTile];
  k.sPre = s_pre;
  k.tid = threadIdx.x;
  k.lane = threadIdx.x & 31;
  k.warp = threadIdx.x >> 5;
  k.fast = true;
  if constexpr (Cfg::kTma) {
    __shared__ __align__(8) uint64_t s_mbar[3];
    k.sMb = smem_u32(s_mbar);
    k.run_tma(p);
  } else {
    k.run(p);
  }
}

}  // namespace memt
