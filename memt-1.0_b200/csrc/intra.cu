// Launcher for the intra-chunk WY kernel (intra.cuh): a persistent grid of
// (SM count x resident CTAs per SM) CTAs striding over the (chunk, head) units.
#include "intra.cuh"
#include "launch.h"

namespace memt {

template <int D, bool HEAD, bool ERASE>
static int launch_intra_t(const IntraParams& p0, int64_t max_chunks, cudaStream_t s) {
  using Cfg = IntraCfg<D, HEAD, ERASE>;
  auto kernel = intra_kernel<D, HEAD, ERASE>;
  IntraParams p = p0;
  cudaError_t e = cudaSuccess;
  if constexpr (Cfg::kTma) {  // [L][H*D] bf16 rows, boxes of 64 channels x 64 tokens
    const uint64_t row = static_cast<uint64_t>(p.H) * D, rows = static_cast<uint64_t>(p.L);
    e = make_tmap_bf16_2d(&p.k_map, p.k, row, rows, static_cast<uint64_t>(p.sk) * 2, 64, kTile);
    if (e == cudaSuccess) e = make_tmap_bf16_2d(&p.v_map, p.v, row, rows, static_cast<uint64_t>(p.sv) * 2, 64, kTile);
    if (e == cudaSuccess && p.write != nullptr)
      e = make_tmap_bf16_2d(&p.w_map, p.write, row, rows, static_cast<uint64_t>(p.sw) * 2, 64, kTile);
    if (e != cudaSuccess) return cuda_status(e);
  }
  e = ensure_smem(kernel, Cfg::kSmem);
  if (e != cudaSuccess) return cuda_status(e);
  int slots = 0;
  e = resident_slots(kernel, Cfg::kThreads, Cfg::kSmem, &slots);
  if (e != cudaSuccess) return cuda_status(e);
  const int64_t units = max_chunks * p.H;
  const unsigned grid = static_cast<unsigned>(units < slots ? units : slots);
  ProfScope prof(kProfIntra, s);
  return cuda_status(launch_pdl(kernel, dim3(grid), dim3(Cfg::kThreads), Cfg::kSmem, s, p));
}

template <int D>
static int launch_intra_d(bool erase, const IntraParams& p, int64_t max_chunks, cudaStream_t s) {
  const bool head = p.g_layout == 1;
  if (head) return erase ? launch_intra_t<D, true, true>(p, max_chunks, s) : launch_intra_t<D, true, false>(p, max_chunks, s);
  return erase ? launch_intra_t<D, false, true>(p, max_chunks, s) : launch_intra_t<D, false, false>(p, max_chunks, s);
}

int launch_intra(int D, bool erase, const IntraParams& p, int64_t max_chunks, cudaStream_t s) {
  switch (D) {
    case 64: return launch_intra_d<64>(erase, p, max_chunks, s);
    case 128: return launch_intra_d<128>(erase, p, max_chunks, s);
    case 256: return launch_intra_d<256>(erase, p, max_chunks, s);
    default: return MEMT_ERR_UNSUPPORTED;
  }
}

}  // namespace memt
