// Launchers for the snapshot readout kernels (read.cuh).
#include "launch.h"
#include "read.cuh"
#include "read_tc.cuh"

namespace memt {

constexpr int kGemvTokens = 4;     // tokens per GEMV CTA
constexpr int kGemvMaxBlock = 16;  // blocks up to this many tokens use the GEMV kernel

// decode (one token per block) uses a one-token CTA; otherwise kGemvTokens per CTA
template <int D, bool EXACT>
static int launch_gemv(const ReadParams& p, int64_t maxlen, cudaStream_t s) {
  const int tq = maxlen <= 1 ? 1 : kGemvTokens;
  int64_t groups = (maxlen + tq - 1) / tq;
  if (groups < 1) groups = 1;
  if (groups > 65535) return MEMT_ERR_UNSUPPORTED;
  dim3 grid(static_cast<unsigned>(p.num_blocks) * p.H, static_cast<unsigned>(groups));
  ProfScope prof(kProfReadGemv, s);
  if (tq == 1)
    read_gemv_kernel<D, 1, EXACT><<<grid, 256, 0, s>>>(p);
  else
    read_gemv_kernel<D, kGemvTokens, EXACT><<<grid, 256, 0, s>>>(p);
  return cuda_status(cudaGetLastError());
}

template <int D>
static int launch_tile(const ReadParams& p, int64_t maxlen, cudaStream_t s) {
  using Cfg = ReadTileCfg<D>;
  cudaError_t e = ensure_smem(read_tile_kernel<D>, Cfg::kSmem);
  if (e != cudaSuccess) return cuda_status(e);
  const int64_t per = int64_t(read_tiles_per_cta<D>()) * kTile;
  int64_t groups = (maxlen + per - 1) / per;
  if (groups < 1) groups = 1;
  if (groups > 65535) return MEMT_ERR_UNSUPPORTED;
  dim3 grid(static_cast<unsigned>(p.num_blocks) * p.H, static_cast<unsigned>(groups));
  ProfScope prof(kProfReadTile, s);
  read_tile_kernel<D><<<grid, Cfg::kNW * 32, Cfg::kSmem, s>>>(p);
  return cuda_status(cudaGetLastError());
}

// d = 128 / 256, bf16 queries, plain read: tcgen05 kernel with TMA query tiles. A CTA reads
// runs of RUN tiles of one block (16, or 32 for a d = 128 read on its own), converting the
// block's snapshot first. By default a block's runs are spread over as many CTAs as it has
// runs: short CTAs balance over the SMs as they free up. With WAVE (d = 256, whose 128 KB snapshot costs a CTA about as much as a few tiles),
// the runs are spread over one resident wave instead, at most 8 runs a CTA (long or ragged
// blocks still spread over the SMs) — unless the read runs beside the commit's scan on the
// caller's stream, where long CTAs could hold SMs the scan is waiting for. PDL: launched
// after the scan on its stream (kReadAfterScan); the kernel never waits on it.
template <int D, int RUN>
static int launch_read_tc(const ReadParams& p, int64_t maxlen, bool wave, bool pdl, cudaStream_t s) {
  using Cfg = ReadTcCfg<D>;
  auto kernel = read_tc_kernel<D, RUN>;
  ReadTcParams P;
  P.p = p;
  const uint64_t row = static_cast<uint64_t>(p.H) * D;
  cudaError_t e = make_tmap_bf16_2d(&P.q_map, p.q, row, static_cast<uint64_t>(p.L), row * 2, 64, Cfg::kTok);
  if (e == cudaSuccess && p.out_bf16 && Cfg::kTmaOut)
    e = make_tmap_bf16_2d(&P.o_map, p.out, row, static_cast<uint64_t>(p.L), row * 2, 64, Cfg::kTok);
  if (e == cudaSuccess) e = ensure_smem(kernel, Cfg::kSmem);
  if (e != cudaSuccess) return cuda_status(e);
  const int64_t per = int64_t(RUN) * Cfg::kTok;
  int64_t groups = (maxlen + per - 1) / per;
  if (groups < 1) groups = 1;
  const int64_t blocks = int64_t(p.num_blocks) * p.H;
  int64_t gy = groups;
  if (wave) {
    constexpr int64_t kMaxRuns = 8;
    int slots = 0;
    e = resident_slots(kernel, Cfg::kThreads, Cfg::kSmem, &slots);
    if (e != cudaSuccess) return cuda_status(e);
    gy = slots / blocks;
    const int64_t gy_min = (groups + kMaxRuns - 1) / kMaxRuns;
    if (gy < gy_min) gy = gy_min;
    if (gy > groups) gy = groups;
    if (gy < 1) gy = 1;
  }
  if (gy > 65535) return MEMT_ERR_UNSUPPORTED;
  dim3 grid(static_cast<unsigned>(blocks), static_cast<unsigned>(gy));
  ProfScope prof(kProfReadTile, s);
  if (pdl) return cuda_status(launch_pdl(kernel, grid, dim3(Cfg::kThreads), Cfg::kSmem, s, P));
  kernel<<<grid, Cfg::kThreads, Cfg::kSmem, s>>>(P);
  return cuda_status(cudaGetLastError());
}

bool read_uses_tc(const ReadParams& p, int D, bool exact, int64_t maxlen) {
  return !exact && !p.fused && maxlen > kGemvMaxBlock && (D == 128 || D == 256);
}

int launch_read(const ReadParams& p, int D, bool exact, int64_t maxlen, cudaStream_t s, int placement) {
  if (read_uses_tc(p, D, exact, maxlen)) {
    const bool pdl = placement == kReadAfterScan;
    if (D == 128) {
      if (placement == kReadAlone) return launch_read_tc<128, kReadTcTilesAlone>(p, maxlen, false, false, s);
      return launch_read_tc<128, kReadTcTiles>(p, maxlen, false, pdl, s);
    }
    return launch_read_tc<256, kReadTcTiles>(p, maxlen, placement != kReadBeside, pdl, s);
  }
  if (exact || maxlen <= kGemvMaxBlock) {
    switch (D) {
      case 64: return exact ? launch_gemv<64, true>(p, maxlen, s) : launch_gemv<64, false>(p, maxlen, s);
      case 128: return exact ? launch_gemv<128, true>(p, maxlen, s) : launch_gemv<128, false>(p, maxlen, s);
      case 256: return exact ? launch_gemv<256, true>(p, maxlen, s) : launch_gemv<256, false>(p, maxlen, s);
      default: return MEMT_ERR_UNSUPPORTED;
    }
  }
  switch (D) {
    case 64: return launch_tile<64>(p, maxlen, s);
    case 128: return launch_tile<128>(p, maxlen, s);
    case 256: return launch_tile<256>(p, maxlen, s);
    default: return MEMT_ERR_UNSUPPORTED;
  }
}

}  // namespace memt

// Status of the one-token decode kernel on the current device (g_read_status), then cleared.
extern "C" int memt_read_status(memt_stream_t stream, int32_t* status_out) {
  if (status_out == nullptr) return MEMT_ERR_INVALID_ARGUMENT;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int32_t v = 0;
  const int32_t zero = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&v, memt::g_read_status, sizeof(v), 0, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e == cudaSuccess) e = cudaMemcpyToSymbolAsync(memt::g_read_status, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return memt::cuda_status(e);
  *status_out = v;
  return MEMT_OK;
}
