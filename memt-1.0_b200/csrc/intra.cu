// Launcher for the intra-chunk WY kernel (intra.cuh).
#include "intra.cuh"
#include "launch.h"

namespace memt {

template <int D, bool HEAD, bool ERASE>
static int launch_intra_t(const IntraParams& p, int64_t max_chunks, cudaStream_t s) {
  using Cfg = IntraCfg<D, HEAD, ERASE>;
  cudaError_t e = ensure_smem(intra_kernel<D, HEAD, ERASE>, Cfg::kSmem);
  if (e != cudaSuccess) return cuda_status(e);
  dim3 grid(static_cast<unsigned>(max_chunks), p.H);
  ProfScope prof(kProfIntra, s);
  intra_kernel<D, HEAD, ERASE><<<grid, Cfg::kThreads, Cfg::kSmem, s>>>(p);
  return cuda_status(cudaGetLastError());
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
