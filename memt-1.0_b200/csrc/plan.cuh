// Varlen scheduling: device-side chunk table for the GDN-2 update.
//
// The reference builds its ChunkPlan on the host (models/qwen/ops/packed.py:16-31,
// models/qwen/ops/layout.py:128-189): each sample is cut into write events of at
// most chunk_tokens tokens and every event into 64-token tiles (the last one
// partial), in scan order. Here one CTA computes the same table on the device from
// cu_seqlens, so the update needs no host round trip (the Qwen builder copies the
// boundaries device -> host -> device on every new batch).
#pragma once

#include "common.cuh"

namespace memt {

// One CTA of 1024 threads. Offsets outside [0, L] are clamped (status bit 0); a table
// that would overflow max_chunks is truncated (status bit 1). Every write stays in bounds.
__global__ void __launch_bounds__(1024) plan_kernel(const int32_t* __restrict__ cu_seqlens,
                                                    int32_t N, int64_t L, int32_t chunk_tokens,
                                                    int32_t max_chunks, WsHeader* __restrict__ hdr,
                                                    ChunkDesc* __restrict__ table,
                                                    int32_t* __restrict__ sample_off) {
  __shared__ long long s_warp[32];
  __shared__ int32_t s_base;
  __shared__ int32_t s_status;
  const int tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  griddep_launch_dependents();  // the intra kernel waits for this grid before it reads the table
  if (tid == 0) {
    s_base = 0;
    s_status = 0;
  }
  __syncthreads();
  for (int32_t base = 0; base < N; base += blockDim.x) {
    const int32_t n = base + tid;
    int64_t bos = 0, eos = 0;
    int32_t cnt = 0;
    if (n < N) {
      int64_t a = cu_seqlens[n], b = cu_seqlens[n + 1];
      int64_t lo = a < 0 ? 0 : (a > L ? L : a);
      int64_t hi = b < lo ? lo : (b > L ? L : b);
      if (lo != a || hi != b) atomicOr(&s_status, 1);
      bos = lo;
      eos = hi;
      int64_t c = chunks_for_length(eos - bos, chunk_tokens);
      cnt = c > max_chunks ? max_chunks : static_cast<int32_t>(c);
    }
    // block-wide exclusive scan of cnt
    long long x = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      long long y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) s_warp[warp] = x;
    __syncthreads();
    if (warp == 0) {
      long long w = lane < (int)(blockDim.x >> 5) ? s_warp[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        long long y = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += y;
      }
      s_warp[lane] = w;  // inclusive warp totals
    }
    __syncthreads();
    const long long excl = x - cnt + (warp > 0 ? s_warp[warp - 1] : 0);
    const long long total = s_warp[(blockDim.x >> 5) - 1];
    int64_t off = static_cast<int64_t>(s_base) + excl;
    if (n < N) {
      int64_t room = max_chunks - off;
      if (room < 0) room = 0;
      if (cnt > room) atomicOr(&s_status, 2);
      sample_off[n] = static_cast<int32_t>(off < max_chunks ? off : max_chunks);
    }
    __syncthreads();
    if (tid == 0) {
      int64_t nb = static_cast<int64_t>(s_base) + total;
      s_base = static_cast<int32_t>(nb < max_chunks ? nb : max_chunks);
    }
    __syncthreads();
  }
  if (tid == 0) sample_off[N] = s_base;
  __syncthreads();
  // Table entries, one chunk per thread: the sample owning chunk c is the last n with
  // sample_off[n] <= c (binary search; empty samples share their offset with the next one);
  // inside a sample, chunk j is tile j % per_event of write event j / per_event.
  const int32_t total = s_base;
  const int32_t per_event = (chunk_tokens + kTile - 1) / kTile;
  for (int32_t c = tid; c < total; c += blockDim.x) {
    int32_t lo = 0, hi = N - 1;
    while (lo < hi) {
      const int32_t mid = (lo + hi + 1) >> 1;
      if (sample_off[mid] <= c) lo = mid; else hi = mid - 1;
    }
    const int32_t n = lo;
    int64_t a = cu_seqlens[n], b = cu_seqlens[n + 1];
    const int64_t bos = a < 0 ? 0 : (a > L ? L : a);
    const int64_t eos = b < bos ? bos : (b > L ? L : b);
    const int32_t j = c - sample_off[n];
    const int64_t e0 = bos + static_cast<int64_t>(j / per_event) * chunk_tokens;
    const int64_t e1 = (e0 + chunk_tokens < eos) ? e0 + chunk_tokens : eos;
    const int64_t t0 = e0 + static_cast<int64_t>(j % per_event) * kTile;
    ChunkDesc d;
    d.sample = n;
    d.tok0 = static_cast<int32_t>(t0);
    d.len = static_cast<int32_t>((e1 - t0) < kTile ? (e1 - t0) : kTile);
    d.pad = 0;
    table[c] = d;
  }
  if (tid == 0) {
    hdr->num_chunks = s_base;
    hdr->status = s_status;
  }
}

}  // namespace memt
