// Shared device helpers for the GDN-2 memory kernels (sm_100a).
//
// Warp-level tensor-core fragments (mma.sync m16n8k16 bf16 and m16n8k8 tf32),
// ldmatrix, cp.async, and the rounding helpers that reproduce the reference's
// bf16 / tf32 cast points.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace memt {

constexpr int kTile = 64;    // tokens per chunk (models/common/constants.py:3)
constexpr int kSub = 16;     // sub-chunk of the blocked solve (gdn2/chunk_intra.py:710)
constexpr float kRcpLn2 = 1.4426950216f;  // _vendor/fla/ops/utils/constant.py:10

// ---------------------------------------------------------------------------
// scalar conversions
// ---------------------------------------------------------------------------
__device__ __forceinline__ float bf16_round(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// bf16x2 product with one round-to-nearest-even of the exact product: the fp32 product of two
// bf16 values is exact, so this equals pack_bf16x2 of the fp32 products.
__device__ __forceinline__ uint32_t mul_bf16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;\n" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
// Two fp32 values in one 64-bit register pair (low word first) and the packed fp32 product,
// rounded to nearest per lane like two separate multiplies.
__device__ __forceinline__ uint64_t bf16x2_to_f32x2(uint32_t u) {  // exact widening
  return (static_cast<uint64_t>(u & 0xffff0000u) << 32) | static_cast<uint64_t>(u << 16);
}
__device__ __forceinline__ uint64_t f32x2_splat(float x) {
  return (static_cast<uint64_t>(__float_as_uint(x)) << 32) | __float_as_uint(x);
}
__device__ __forceinline__ uint64_t f32x2_pack(float lo, float hi) {
  return (static_cast<uint64_t>(__float_as_uint(hi)) << 32) | __float_as_uint(lo);
}
__device__ __forceinline__ uint64_t mul_f32x2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;\n" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t fma_f32x2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;\n" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t sub_f32x2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;\n" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float f32x2_lo(uint64_t v) { return __uint_as_float(static_cast<uint32_t>(v)); }
__device__ __forceinline__ float f32x2_hi(uint64_t v) { return __uint_as_float(static_cast<uint32_t>(v >> 32)); }
__device__ __forceinline__ uint32_t f32x2_to_bf16x2(uint64_t v) {
  return pack_bf16x2(__uint_as_float(static_cast<uint32_t>(v)), __uint_as_float(static_cast<uint32_t>(v >> 32)));
}
// four 8x8 bf16 matrices from mma accumulator fragments into shared memory; lane l gives the
// address of row l % 8 of matrix l / 8
__device__ __forceinline__ void stsm_x4(uint32_t addr, uint32_t r0, uint32_t r1, uint32_t r2, uint32_t r3) {
  asm volatile("stmatrix.sync.aligned.m8n8.x4.shared.b16 [%0], {%1, %2, %3, %4};\n" ::"r"(addr), "r"(r0), "r"(r1),
               "r"(r2), "r"(r3)
               : "memory");
}
__device__ __forceinline__ float2 unpack_bf16x2(uint32_t u) {
  __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162*>(&u);
  return __bfloat1622float2(v);
}

// fp32 -> tf32, round to nearest, ties away from zero (the rounding Triton applies to the
// fp32 operands of its tf32 dots). On the sign-magnitude bit pattern, adding half a tf32 ulp
// (bit 12) and clearing the 13 dropped bits rounds the magnitude half away from zero; the
// carry into the exponent is the correct rounding, infinities are unchanged. Two integer
// ops instead of a conversion instruction.
__device__ __forceinline__ uint32_t to_tf32(float x) {
  return (__float_as_uint(x) + 0x1000u) & 0xffffe000u;
}

__device__ __forceinline__ float fast_exp2(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// ---------------------------------------------------------------------------
// tensor-core fragments
//   A (16 x k, row-major), B (k x 8, "col"), C/D (16 x 8) per the PTX ISA layouts:
//   g = lane / 4, t = lane % 4;  C: c0 (g, 2t) c1 (g, 2t+1) c2 (g+8, 2t) c3 (g+8, 2t+1)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4],
                                               const uint32_t (&b)[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// A: a0 (g, t) a1 (g+8, t) a2 (g, t+4) a3 (g+8, t+4);  B: b0 (k=t, n=g) b1 (k=t+4, n=g)
__device__ __forceinline__ void mma_tf32_1688(float (&d)[4], const uint32_t (&a)[4],
                                              const uint32_t (&b)[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ldmatrix: lane i supplies the address of row (i % 8) of 8x8 matrix (i / 8).
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2(uint32_t (&r)[2], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];\n"
               : "=r"(r[0]), "=r"(r[1])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2_t(uint32_t (&r)[2], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];\n"
               : "=r"(r[0]), "=r"(r[1])
               : "r"(addr));
}

// ---------------------------------------------------------------------------
// async copies (16 bytes per thread, L2-only)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_u32(smem)), "l"(gmem));
}
__device__ __forceinline__ void cp_async16_zfill(void* smem, const void* gmem, bool valid) {
  int src = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(smem)),
               "l"(gmem), "r"(src));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

// ---------------------------------------------------------------------------
// mbarrier + bulk (TMA, untiled) copies global -> shared, each into this CTA only.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t mbar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(mbar), "r"(count));
}
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;\n" ::);
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t mbar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(mbar), "r"(bytes));
}
__device__ __forceinline__ void mbar_arrive(uint32_t mbar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(mbar) : "memory");
}
// Bounded wait for the phase with the given parity; false after 2^24 polls (about a second).
// Plain polling: a thread suspended by a try_wait time hint resumes measurably later than a
// polling one, which lengthens the scan's dependent chain.
__device__ __forceinline__ bool mbar_wait(uint32_t mbar, uint32_t parity) {
  for (int i = 0; i < (1 << 24); ++i) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(mbar), "r"(parity)
        : "memory");
    if (ok) return true;
  }
  return false;
}
// 1-D bulk copy; addresses 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t mbar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(mbar)
      : "memory");
}

// Programmatic dependent launch: a kernel launched with programmatic stream serialization
// may start while the previous kernel of the stream is still running. It must call
// griddep_wait() before touching global memory that any earlier work produces (it returns
// once the previous grid has completed and its writes are visible; a no-op otherwise);
// griddep_launch_dependents() lets the next such kernel start its own prologue early.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;\n" :::); }

// Bulk (TMA engine) copy shared -> global; both addresses 16-byte aligned, bytes % 16 == 0.
__device__ __forceinline__ void bulk_s2g(void* dst, uint32_t src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;\n" ::"l"(dst), "r"(src), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;\n" ::: "memory"); }
// the shared-memory sources of this thread's committed bulk stores may be overwritten
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;\n" ::: "memory"); }
// ... for all but the most recent group
__device__ __forceinline__ void bulk_wait_read_but1() { asm volatile("cp.async.bulk.wait_group.read 1;\n" ::: "memory"); }
// this thread's committed bulk stores have completed
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory"); }
// make this thread's generic-proxy shared-memory writes visible to the async proxy
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }

// XOR-swizzled bf16 tile with RL elements per row (RL % 64 == 0): the low three bits of the
// 16-byte chunk index are XORed with (row & 7), so ldmatrix over 8 consecutive rows and
// fragment-wise 4-byte accesses are bank-conflict free. The intra kernel writes its outputs in
// this layout so the scan can move whole tiles with one bulk copy.
template <int RL>
__device__ __forceinline__ int swz(int row, int col) {
  return row * RL + ((((col >> 3) ^ row) & 7) | ((col >> 3) & ~7)) * 8 + (col & 7);
}

// Element offset in a bf16 [64][D] tile stored as D/64 panels of [64][64], each swz<64>:
// 128-byte rows whose 16-byte chunks are XOR-permuted by (row & 7). With a 1024-byte aligned
// base this is the canonical SWIZZLE_128B operand layout of tcgen05 shared-memory
// descriptors (K-major when the 64 columns are the reduction index, MN-major otherwise).
__device__ __forceinline__ int pswz(int row, int col) {
  return (col >> 6) * (kTile * 64) + swz<64>(row, col & 63);
}

// ---------------------------------------------------------------------------
// chunk table entry written by the plan kernel
// ---------------------------------------------------------------------------
struct ChunkDesc {
  int32_t sample;  // owning sample
  int32_t tok0;    // first packed token
  int32_t len;     // 1..64 valid tokens
  int32_t pad;
};

// Workspace header (first 256 bytes of every update workspace).
struct WsHeader {
  int32_t num_chunks;  // chunks written by the plan kernel
  int32_t status;      // bit 0: clamped offsets, bit 1: chunk table overflow, bit 2: copy wait timed out,
                       // bit 3: a state slot outside its pool
  int32_t reserved[62];
};

// chunks a sample of `len` tokens produces: full events of chunk_tokens plus the remainder
__host__ __device__ inline int64_t chunks_for_length(int64_t len, int32_t chunk_tokens) {
  if (len <= 0) return 0;
  const int64_t per_event = (chunk_tokens + kTile - 1) / kTile;
  const int64_t full = len / chunk_tokens;
  const int64_t rem = len % chunk_tokens;
  return full * per_event + (rem + kTile - 1) / kTile;
}

// Upper bound on the chunk count for any split of L tokens into N samples.
__host__ __device__ inline int64_t max_chunks_bound(int64_t L, int32_t N, int32_t chunk_tokens) {
  return (L + kTile - 1) / kTile + (L + chunk_tokens - 1) / chunk_tokens + N;
}

// ---------------------------------------------------------------------------
// kernel parameter blocks
// ---------------------------------------------------------------------------
struct IntraParams {
  WsHeader* hdr;
  const ChunkDesc* table;
  int64_t L;  // packed tokens
  int32_t H;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  const float* g;
  int32_t g_layout;  // 1 per head, 2 per channel
  const __nv_bfloat16* beta;
  int32_t beta_layout;  // 0 none, 1 per head, 2 per channel
  const __nv_bfloat16* erase;  // per channel or null
  const __nv_bfloat16* write;  // per channel or null
  int64_t sk, sv, sw;          // elements per token row of k, v and write (>= H*D)
  __nv_bfloat16* W;
  __nv_bfloat16* U;
  __nv_bfloat16* KG;
  float* Elast;
  // TMA maps over k, v and write ([L][H*D] bf16, boxes of 64 channels x 64 tokens, 128-byte
  // swizzle); encoded by the launcher for the kernels that load their tiles by TMA
  CUtensorMap k_map, v_map, w_map;
};

// Slot of sample n in a state pool addressed by optional slot indices: n itself when slots is
// null, slots[n] when it lies in [0, num), and -1 otherwise (the caller skips that state).
__device__ __forceinline__ int64_t pool_slot(const int32_t* slots, int32_t num, int n) {
  if (slots == nullptr) return n;
  const int s = slots[n];
  return (s >= 0 && s < num) ? s : -1;
}

struct ScanParams {
  WsHeader* hdr;
  const int32_t* sample_off;  // [N+1] chunk offsets per sample
  int32_t N, H;
  const __nv_bfloat16* W;
  const __nv_bfloat16* U;
  const __nv_bfloat16* KG;
  const float* Elast;
  const float* h0;
  float* ht;
  // optional pools: sample n starts from h0[slots_in[n]] and ends in ht[slots_out[n]]
  const int32_t* slots_in;
  const int32_t* slots_out;
  int32_t num_in, num_out;
};

struct ReadParams {
  int32_t num_blocks, H;
  int64_t L;
  const int32_t* cu;
  const void* q;        // bf16 or fp32 [L,H,D]
  const float* states;  // [num_blocks,H,D,D]
  float scale;
  void* out;            // plain read: [L,H,D] (bf16 or fp32)
  int32_t out_bf16;
  // fused readout
  int32_t fused;
  int32_t normalize_q;
  float q_eps;
  const __nv_bfloat16* gate;
  const __nv_bfloat16* norm_w;
  float norm_eps, softcap;
  const __nv_bfloat16* residual;
  int64_t row_stride;
  int32_t head_offset;
  // optional: block n reads states[slots[n]] of a pool of num_slots snapshots (null: states[n])
  const int32_t* slots;
  int32_t num_slots;
};

struct RecurrentParams {
  const int32_t* cu;
  int32_t N, H;
  int64_t L;
  const float* k;
  const float* v;
  const float* g;
  int32_t g_layout;
  const float* beta;
  int32_t beta_layout;
  const float* erase;
  const float* write;
  const float* h0;
  float* ht;
  const int32_t* slots_in;  // optional pools, as in ScanParams
  const int32_t* slots_out;
  int32_t num_in, num_out;
};

}  // namespace memt
