// GDN-2 intra-chunk kernel: one CTA per (64-token chunk, head).
//
// Fuses what the reference runs as four launches with HBM round trips between them
// (paths relative to inference/memt_sglang):
//   chunk_local_cumsum                _vendor/fla/ops/utils/cumsum.py:76-133
//   diagonal key-key blocks           _vendor/fla/ops/gdn2/chunk_intra_token_parallel.py:25-132
//   off-diagonal blocks + blocked solve _vendor/fla/ops/gdn2/chunk_intra.py:153-417
//   WY operands u, w, kg              _vendor/fla/ops/gdn2/wy_fast.py:36-142
// and writes only what the state scan consumes: w, u, kg (bf16, [chunk][head][64][D])
// and the chunk's total decay 2^G_last (fp32, [chunk][head][D]).
//
// Numerics follow the reference's GPU rounding points: fp32 cumulative log2 decay;
// exact-fp32 diagonal 16x16 blocks (here: 3xTF32 tensor-core products of the
// factorised operands); tf32 off-diagonal blocks with the per-sub-chunk reference
// point; fp32 forward substitution on the diagonal blocks; tf32 products for the
// off-diagonal inverse blocks; A^-1 stored as bf16; u = A^-1 bf16(v*w),
// w = A^-1 bf16(bf16(k*b) 2^G), kg = bf16(k 2^(G_last-G)), all with fp32 accumulation.
//
// Decay factors: when every cumulative exponent of the panel lies in [-60, 60] the
// kernel tabulates E = 2^G and 1/E once and forms every factor 2^(G_i - G_n) as a
// product (no per-pair exponentials). Otherwise (extreme decays) it evaluates
// exp2(G_i - G_n) directly and computes the diagonal blocks pair by pair, exactly as
// the reference does, so no factor can overflow.
#pragma once

#include "common.cuh"

namespace memt {

template <int D>
struct IntraCfg {
  static constexpr int kPanel = D < 128 ? D : 128;
  static constexpr int kPanels = D / kPanel;
  static constexpr int kThreads = 256;
  static constexpr int kLdE = kPanel + 4;   // fp32 row stride (conflict-free fragment reads)
  static constexpr int kLdK = kPanel + 8;   // bf16 row stride
  static constexpr int kLdA = kTile + 4;    // fp32 64x64
  static constexpr int kLdAi = kTile + 8;   // bf16 64x64
  static constexpr size_t kBytesE = size_t(kTile) * kLdE * 4;
  static constexpr size_t kBytesK = size_t(kTile) * kLdK * 2;
  static constexpr size_t kBytesA = size_t(kTile) * kLdA * 4;
  static constexpr size_t kBytesAi = size_t(kTile) * kLdAi * 2;
  static_assert(size_t(kTile) * kLdK * 2 <= kBytesA, "staging tile must fit in the score buffer");
  static constexpr size_t smem(bool erase) {
    return 2 * kBytesE + kBytesK * (erase ? 2 : 1) + kBytesA + kBytesAi + 16;
  }
};

// 16x16x16 tf32 product on one warp: acc[nt] += A (16x16, row-major, lda) . B (16x16,
// row-major [k][n], ldb); acc[nt] is the C fragment of columns 8*nt..8*nt+7.
__device__ __forceinline__ void warp_tf32_16x16x16(float (&acc)[2][4], const float* A, int lda,
                                                   const float* B, int ldb, int lane) {
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int kk = 0; kk < 16; kk += 8) {
    uint32_t a[4];
    a[0] = to_tf32(A[g * lda + kk + t]);
    a[1] = to_tf32(A[(g + 8) * lda + kk + t]);
    a[2] = to_tf32(A[g * lda + kk + t + 4]);
    a[3] = to_tf32(A[(g + 8) * lda + kk + t + 4]);
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      uint32_t b[2];
      b[0] = to_tf32(B[(kk + t) * ldb + nt * 8 + g]);
      b[1] = to_tf32(B[(kk + t + 4) * ldb + nt * 8 + g]);
      mma_tf32_1688(acc[nt], a, b);
    }
  }
}

__device__ __forceinline__ void warp_store_16x16(float* C, int ldc, const float (&acc)[2][4],
                                                 int lane, float sign) {
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    C[g * ldc + nt * 8 + 2 * t] = sign * acc[nt][0];
    C[g * ldc + nt * 8 + 2 * t + 1] = sign * acc[nt][1];
    C[(g + 8) * ldc + nt * 8 + 2 * t] = sign * acc[nt][2];
    C[(g + 8) * ldc + nt * 8 + 2 * t + 1] = sign * acc[nt][3];
  }
}

__device__ __forceinline__ void zero_acc(float (&acc)[2][4]) {
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
}

template <int D, bool ERASE>
struct IntraKernel {
  using Cfg = IntraCfg<D>;
  static constexpr int P = Cfg::kPanel;

  float* sE;   // E = 2^G (fast) or G (slow)   [64][kLdE]
  float* sEi;  // 1/E (fast)                   [64][kLdE]
  __nv_bfloat16* sK;  // k' (beta folded)      [64][kLdK]
  __nv_bfloat16* sB;  // erase b               [64][kLdK]
  float* sA;          // key-key scores / inverse blocks (fp32) [64][kLdA]
  __nv_bfloat16* sX;  // bf16 staging operand (aliases sA)   [64][kLdK]
  __nv_bfloat16* sAi; // A^-1 bf16              [64][kLdAi]
  int* sFlag;

  int tid, lane, warp, len, tok0, h;
  int64_t row_stride;  // H*D
  bool fast;

  __device__ __forceinline__ float kval(int i, int c) const {
    return __bfloat162float(sK[i * Cfg::kLdK + c]);
  }
  __device__ __forceinline__ float kbval(int i, int c) const {
    float x = kval(i, c);
    if constexpr (ERASE) x *= __bfloat162float(sB[i * Cfg::kLdK + c]);
    return x;
  }
  // 2^(G_i - G_n) for channel c of the panel
  __device__ __forceinline__ float p2d(int i, int n, int c) const {
    if (fast) return sE[i * Cfg::kLdE + c] * sEi[n * Cfg::kLdE + c];
    return fast_exp2(sE[i * Cfg::kLdE + c] - sE[n * Cfg::kLdE + c]);
  }
  // 2^G_i
  __device__ __forceinline__ float p2(int i, int c) const {
    if (fast) return sE[i * Cfg::kLdE + c];
    return fast_exp2(sE[i * Cfg::kLdE + c]);
  }

  // Load k (beta folded), erase and the log-decay of one channel panel; build the
  // cumulative log2 decay and the factor tables. Ends with a barrier.
  __device__ void load_panel(const IntraParams& p, int c0) {
    const int64_t base = (int64_t)tok0 * row_stride + (int64_t)h * D + c0;
    // k, erase: 8 bf16 (16 B) per thread-iteration
    constexpr int kVecPerRow = P / 8;
    for (int idx = tid; idx < kTile * kVecPerRow; idx += Cfg::kThreads) {
      const int i = idx / kVecPerRow, cv = (idx % kVecPerRow) * 8;
      uint4 kv = make_uint4(0, 0, 0, 0), bv = make_uint4(0, 0, 0, 0);
      if (i < len) {
        const int64_t off = base + (int64_t)i * row_stride + cv;
        kv = *reinterpret_cast<const uint4*>(p.k + off);
        if constexpr (ERASE) bv = *reinterpret_cast<const uint4*>(p.erase + off);
        if (p.beta_layout != 0) {
          // k' = bf16( bf16(sqrt(beta)) * k ): stable GDN-2 key scaling
          // (models/qwen/layer.py:81-85, 96)
          float sb[8];
          if (p.beta_layout == 1) {
            float b = __bfloat162float(p.beta[(int64_t)(tok0 + i) * p.H + h]);
            float s = bf16_round(sqrtf(b));
#pragma unroll
            for (int e = 0; e < 8; ++e) sb[e] = s;
          } else {
            uint4 be = *reinterpret_cast<const uint4*>(p.beta + off);
            const uint32_t* bw = reinterpret_cast<const uint32_t*>(&be);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              float2 f = unpack_bf16x2(bw[e]);
              sb[2 * e] = bf16_round(sqrtf(f.x));
              sb[2 * e + 1] = bf16_round(sqrtf(f.y));
            }
          }
          uint32_t* kw = reinterpret_cast<uint32_t*>(&kv);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float2 f = unpack_bf16x2(kw[e]);
            kw[e] = pack_bf16x2(f.x * sb[2 * e], f.y * sb[2 * e + 1]);
          }
        }
      }
      *reinterpret_cast<uint4*>(sK + i * Cfg::kLdK + cv) = kv;
      if constexpr (ERASE) *reinterpret_cast<uint4*>(sB + i * Cfg::kLdK + cv) = bv;
    }
    // cumulative decay: one thread per channel, sequential over the 64 tokens
    // G_t = (sum_{s<=t} g_s) * (1/ln2)  (cumsum.py:126-133; padded tokens add 0)
    bool ok = true;
    if (tid < P) {
      const int c = tid;
      float acc = 0.f;
      for (int i = 0; i < kTile; ++i) {
        float gi = 0.f;
        if (i < len) {
          if (p.g_layout == 2)
            gi = p.g[base + (int64_t)i * row_stride + c];
          else
            gi = p.g[(int64_t)(tok0 + i) * p.H + h];
        }
        acc += gi;
        const float G = acc * kRcpLn2;
        ok = ok && (G >= -60.f) && (G <= 60.f);
        sE[i * Cfg::kLdE + c] = G;
      }
    }
    fast = __syncthreads_and(ok) != 0;
    if (fast) {
      for (int idx = tid; idx < kTile * P; idx += Cfg::kThreads) {
        const int i = idx / P, c = idx % P;
        const float G = sE[i * Cfg::kLdE + c];
        sEi[i * Cfg::kLdE + c] = fast_exp2(-G);
        sE[i * Cfg::kLdE + c] = fast_exp2(G);
      }
    }
    __syncthreads();
  }

  // Accumulate this panel's contribution to the key-key scores of the warp's row block.
  // Warp w: row block r = w/2, n-tiles nt = (w&1), (w&1)+2, ... <= 2r+1.
  __device__ void scores_panel(float (&acc)[4][4]) {
    const int r = warp >> 1, half = warp & 1;
    if (16 * r >= len) return;  // whole row block beyond the chunk (chunk_intra.py:242-278)
    const int g = lane >> 2, t = lane & 3;
    const int n_ref = 16 * r;
    const int i0 = n_ref + g, i1 = n_ref + g + 8;
    const bool v0 = i0 < len, v1 = i1 < len;
#pragma unroll 2
    for (int c0 = 0; c0 < P; c0 += 8) {
      const int ca = c0 + t, cb = c0 + t + 4;
      // left operand: kb_i 2^(G_i - G_n)   (chunk_intra.py:252-256)
      float la[4];
      la[0] = v0 ? kbval(i0, ca) * p2d(i0, n_ref, ca) : 0.f;
      la[1] = v1 ? kbval(i1, ca) * p2d(i1, n_ref, ca) : 0.f;
      la[2] = v0 ? kbval(i0, cb) * p2d(i0, n_ref, cb) : 0.f;
      la[3] = v1 ? kbval(i1, cb) * p2d(i1, n_ref, cb) : 0.f;
      uint32_t ahi[4], alo[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        ahi[q] = to_tf32(la[q]);
        alo[q] = to_tf32(la[q] - __uint_as_float(ahi[q]));
      }
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        const int nt = half + 2 * s;
        if (nt > 2 * r + 1) break;
        const int j = 8 * nt + g;
        // right operand: k_j 2^(G_n - G_j)   (chunk_intra.py:253)
        float rb0 = kval(j, ca) * p2d(n_ref, j, ca);
        float rb1 = kval(j, cb) * p2d(n_ref, j, cb);
        uint32_t bhi[2] = {to_tf32(rb0), to_tf32(rb1)};
        const bool diag = (nt >> 1) == r;
        if (diag) {
          if (!fast) continue;  // exact pairwise evaluation below
          uint32_t blo[2] = {to_tf32(rb0 - __uint_as_float(bhi[0])),
                             to_tf32(rb1 - __uint_as_float(bhi[1]))};
          mma_tf32_1688(acc[s], alo, bhi);
          mma_tf32_1688(acc[s], ahi, blo);
        }
        mma_tf32_1688(acc[s], ahi, bhi);
      }
    }
    if (!fast) {
      // diagonal n-tile: exact per-pair exponents, as the token-parallel kernel
      // (chunk_intra_token_parallel.py:114-123). Lane owns C(g,2t),(g,2t+1),(g+8,2t),(g+8,2t+1).
      // the diagonal n-tile 2r+half sits at position r of this warp's list
      const int nt = 2 * r + half;
      float extra[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int i = n_ref + g + ((q & 2) ? 8 : 0);
        const int j = 8 * nt + 2 * t + (q & 1);
        float sum = 0.f;
        if (i < len && j < i) {
          for (int c = 0; c < P; ++c)
            sum += kbval(i, c) * kval(j, c) *
                   fast_exp2(sE[i * Cfg::kLdE + c] - sE[j * Cfg::kLdE + c]);
        }
        extra[q] = sum;
      }
#pragma unroll
      for (int s = 0; s < 4; ++s)
        if (s == r)
#pragma unroll
          for (int q = 0; q < 4; ++q) acc[s][q] += extra[q];
    }
  }

  // Write the score accumulators to sA (strictly lower on the diagonal blocks).
  __device__ void store_scores(const float (&acc)[4][4]) {
    const int r = warp >> 1, half = warp & 1;
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      const int nt = half + 2 * s;
      if (nt > 2 * r + 1) break;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int i = 16 * r + g + ((q & 2) ? 8 : 0);
        const int j = 8 * nt + 2 * t + (q & 1);
        float x = acc[s][q];
        if (j >= i || i >= len) x = 0.f;
        sA[i * Cfg::kLdA + j] = x;
      }
    }
  }

  // Blocked inverse of (I + A) in place (chunk_intra.py:326-395). Diagonal inverse
  // blocks stay on the diagonal; the off-diagonal inverse block (r, s), r > s, is kept
  // in the unused upper slot (s, r) as a plain 16x16 matrix.
  __device__ void solve() {
    constexpr int LD = Cfg::kLdA;
    // forward substitution on the four diagonal blocks, warp r handles block r
    if (warp < 4) {
      const int r = warp;
      const int c = lane & 15;
      float* blk = sA + (16 * r) * LD + 16 * r;
      float x[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) x[j] = (c < j) ? -blk[j * LD + c] : 0.f;
#pragma unroll
      for (int i = 2; i < 16; ++i) {
        const float a = (c < i) ? -blk[i * LD + c] : 0.f;
        float s = a;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float aj = __shfl_sync(0xffffffffu, a, j);
          if (j < i) s = fmaf(aj, x[j], s);
        }
        x[i] = s;
      }
      __syncwarp();
      if (lane < 16) {
#pragma unroll
        for (int j = 0; j < 16; ++j) blk[j * LD + c] = x[j] + (j == c ? 1.f : 0.f);
      }
    }
    __syncthreads();
    auto D_ = [&](int r) { return sA + (16 * r) * LD + 16 * r; };          // Ai_rr
    auto Ak = [&](int r, int s) { return sA + (16 * r) * LD + 16 * s; };   // Akk_rs, r > s
    auto Ao = [&](int r, int s) { return sA + (16 * s) * LD + 16 * r; };   // Ai_rs stored at (s, r)
    float acc[2][4];
    // stage 1: Ai_{s+1,s} = -(Ai_{s+1,s+1} Akk_{s+1,s}) Ai_{s,s}
    if (warp < 3) {
      const int s = warp;
      // scratch: slots (0,2), (1,3), (0,3) are free until stages 2-3
      float* tmp = (s == 0) ? Ao(2, 0) : (s == 1) ? Ao(3, 1) : Ao(3, 0);
      zero_acc(acc);
      warp_tf32_16x16x16(acc, D_(s + 1), LD, Ak(s + 1, s), LD, lane);
      warp_store_16x16(tmp, LD, acc, lane, 1.f);
      __syncwarp();
      zero_acc(acc);
      warp_tf32_16x16x16(acc, tmp, LD, D_(s), LD, lane);
      warp_store_16x16(Ao(s + 1, s), LD, acc, lane, -1.f);
    }
    __syncthreads();
    // stage 2: Ai20 = -Ai22 (Akk20 Ai00 + Akk21 Ai10); Ai31 = -Ai33 (Akk31 Ai11 + Akk32 Ai21)
    if (warp < 2) {
      const int r = warp + 2;  // 2 or 3
      float* dst = Ao(r, r - 2);
      zero_acc(acc);
      warp_tf32_16x16x16(acc, Ak(r, r - 2), LD, D_(r - 2), LD, lane);
      warp_tf32_16x16x16(acc, Ak(r, r - 1), LD, Ao(r - 1, r - 2), LD, lane);
      warp_store_16x16(dst, LD, acc, lane, 1.f);
      __syncwarp();
      zero_acc(acc);
      warp_tf32_16x16x16(acc, D_(r), LD, dst, LD, lane);
      __syncwarp();
      warp_store_16x16(dst, LD, acc, lane, -1.f);
    }
    __syncthreads();
    // stage 3: Ai30 = -Ai33 (Akk30 Ai00 + Akk31 Ai10 + Akk32 Ai20)
    if (warp == 0) {
      float* dst = Ao(3, 0);
      zero_acc(acc);
      warp_tf32_16x16x16(acc, Ak(3, 0), LD, D_(0), LD, lane);
      warp_tf32_16x16x16(acc, Ak(3, 1), LD, Ao(1, 0), LD, lane);
      warp_tf32_16x16x16(acc, Ak(3, 2), LD, Ao(2, 0), LD, lane);
      warp_store_16x16(dst, LD, acc, lane, 1.f);
      __syncwarp();
      zero_acc(acc);
      warp_tf32_16x16x16(acc, D_(3), LD, dst, LD, lane);
      __syncwarp();
      warp_store_16x16(dst, LD, acc, lane, -1.f);
    }
    __syncthreads();
    // A^-1 -> bf16, rows beyond the chunk zero (chunk_intra.py:408-417)
    for (int idx = tid; idx < kTile * kTile; idx += Cfg::kThreads) {
      const int i = idx / kTile, j = idx % kTile;
      const int r = i >> 4, s = j >> 4;
      float x = 0.f;
      if (i < len) {
        if (r == s)
          x = (j <= i) ? sA[i * LD + j] : 0.f;
        else if (r > s)
          x = sA[(16 * s + (i & 15)) * LD + 16 * r + (j & 15)];
      }
      sAi[i * Cfg::kLdAi + j] = __float2bfloat16_rn(x);
    }
    __syncthreads();
  }

  // out[64][P] (bf16, global rows of stride ld) = A^-1 (64x64 lower) . sX (64 x P).
  // Warp w: row block r = w/2, column half (w&1) of the panel; k-steps 0..r only.
  __device__ void wy_product(__nv_bfloat16* out, int64_t ld) {
    const int r = warp >> 1, half = warp & 1;
    constexpr int NT = P / 16;  // n-tiles per warp (half of P / 8)
    float acc[NT][4];
#pragma unroll
    for (int i = 0; i < NT; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
    const int n_base = half * (P / 2);
    for (int ks = 0; ks <= r; ++ks) {
      uint32_t a[4];
      ldsm_x4(a, smem_u32(sAi + (16 * r + (lane & 15)) * Cfg::kLdAi + 16 * ks + 8 * (lane >> 4)));
#pragma unroll
      for (int np = 0; np < NT; np += 2) {
        uint32_t b[4];
        ldsm_x4_t(b, smem_u32(sX + (16 * ks + (lane & 15)) * Cfg::kLdK + n_base + 8 * np +
                              8 * (lane >> 4)));
        uint32_t b0[2] = {b[0], b[1]}, b1[2] = {b[2], b[3]};
        mma_bf16_16816(acc[np], a, b0);
        mma_bf16_16816(acc[np + 1], a, b1);
      }
    }
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int col = n_base + 8 * nt + 2 * t;
      const int i0 = 16 * r + g;
      *reinterpret_cast<uint32_t*>(out + (int64_t)i0 * ld + col) = pack_bf16x2(acc[nt][0], acc[nt][1]);
      *reinterpret_cast<uint32_t*>(out + (int64_t)(i0 + 8) * ld + col) =
          pack_bf16x2(acc[nt][2], acc[nt][3]);
    }
  }

  __device__ void run(const IntraParams& p) {
    const int c = blockIdx.x;
    if (c >= p.hdr->num_chunks) return;
    const ChunkDesc d = p.table[c];
    tok0 = d.tok0;
    len = d.len;
    h = blockIdx.y;
    row_stride = (int64_t)p.H * D;
    const int64_t chunk_head = (int64_t)c * p.H + h;

    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;

    // ---- key-key scores over all channel panels ----
    for (int pn = 0; pn < Cfg::kPanels; ++pn) {
      load_panel(p, pn * P);
      scores_panel(acc);
      __syncthreads();
    }
    store_scores(acc);
    __syncthreads();
    solve();

    // ---- w and kg per channel panel ----
    const int last = len - 1;
    for (int pn = 0; pn < Cfg::kPanels; ++pn) {
      const int c0 = pn * P;
      if (Cfg::kPanels > 1) load_panel(p, c0);
      // staging operand bf16( bf16(k*b) * 2^G )   (wy_fast.py:110-116)
      for (int idx = tid; idx < kTile * P; idx += Cfg::kThreads) {
        const int i = idx / P, cc = idx % P;
        float kb = kval(i, cc);
        if constexpr (ERASE) kb = bf16_round(kb * __bfloat162float(sB[i * Cfg::kLdK + cc]));
        sX[i * Cfg::kLdK + cc] = __float2bfloat16_rn(kb * p2(i, cc));
      }
      // kg = bf16(k * 2^(G_last - G)) (wy_fast.py:125-139) and 2^G_last
      __nv_bfloat16* kg = p.KG + chunk_head * kTile * D + c0;
      for (int idx = tid; idx < kTile * P / 2; idx += Cfg::kThreads) {
        const int i = idx / (P / 2), cc = (idx % (P / 2)) * 2;
        float x0 = 0.f, x1 = 0.f;
        if (i < len) {
          x0 = kval(i, cc) * p2d(last, i, cc);
          x1 = kval(i, cc + 1) * p2d(last, i, cc + 1);
        }
        *reinterpret_cast<uint32_t*>(kg + (int64_t)i * D + cc) = pack_bf16x2(x0, x1);
      }
      if (tid < P) p.Elast[chunk_head * D + c0 + tid] = p2(last, tid);
      __syncthreads();
      wy_product(p.W + chunk_head * kTile * D + c0, D);
      __syncthreads();
    }

    // ---- u per value panel: A^-1 bf16(v * w)   (wy_fast.py:92-102) ----
    for (int pn = 0; pn < Cfg::kPanels; ++pn) {
      const int c0 = pn * P;
      const int64_t base = (int64_t)tok0 * row_stride + (int64_t)h * D + c0;
      constexpr int kVecPerRow = P / 8;
      for (int idx = tid; idx < kTile * kVecPerRow; idx += Cfg::kThreads) {
        const int i = idx / kVecPerRow, cv = (idx % kVecPerRow) * 8;
        uint4 vv = make_uint4(0, 0, 0, 0);
        if (i < len) {
          const int64_t off = base + (int64_t)i * row_stride + cv;
          vv = *reinterpret_cast<const uint4*>(p.v + off);
          if (p.write != nullptr) {
            uint4 ww = *reinterpret_cast<const uint4*>(p.write + off);
            uint32_t* vw = reinterpret_cast<uint32_t*>(&vv);
            const uint32_t* wg = reinterpret_cast<const uint32_t*>(&ww);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              float2 a = unpack_bf16x2(vw[e]), b = unpack_bf16x2(wg[e]);
              vw[e] = pack_bf16x2(a.x * b.x, a.y * b.y);
            }
          }
        }
        *reinterpret_cast<uint4*>(sX + i * Cfg::kLdK + cv) = vv;
      }
      __syncthreads();
      wy_product(p.U + chunk_head * kTile * D + c0, D);
      __syncthreads();
    }
  }
};

template <int D, bool ERASE>
__global__ void __launch_bounds__(256) intra_kernel(IntraParams p) {
  extern __shared__ __align__(128) unsigned char smem_intra[];
  using Cfg = IntraCfg<D>;
  IntraKernel<D, ERASE> k;
  unsigned char* ptr = smem_intra;
  k.sE = reinterpret_cast<float*>(ptr);
  ptr += Cfg::kBytesE;
  k.sEi = reinterpret_cast<float*>(ptr);
  ptr += Cfg::kBytesE;
  k.sK = reinterpret_cast<__nv_bfloat16*>(ptr);
  ptr += Cfg::kBytesK;
  if constexpr (ERASE) {
    k.sB = reinterpret_cast<__nv_bfloat16*>(ptr);
    ptr += Cfg::kBytesK;
  } else {
    k.sB = nullptr;
  }
  k.sA = reinterpret_cast<float*>(ptr);
  k.sX = reinterpret_cast<__nv_bfloat16*>(ptr);
  ptr += Cfg::kBytesA;
  k.sAi = reinterpret_cast<__nv_bfloat16*>(ptr);
  k.tid = threadIdx.x;
  k.lane = threadIdx.x & 31;
  k.warp = threadIdx.x >> 5;
  k.run(p);
}

}  // namespace memt
