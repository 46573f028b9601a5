// Launcher for the intra-chunk WY kernel (intra.cuh).
#include "intra.cuh"
#include "launch.h"

namespace memt {

template <int D, bool ERASE>
static int launch_intra_t(const IntraParams& p, int64_t max_chunks, cudaStream_t s) {
  const size_t smem = IntraCfg<D>::smem(ERASE);
  cudaError_t e = ensure_smem(intra_kernel<D, ERASE>, smem);
  if (e != cudaSuccess) return cuda_status(e);
  dim3 grid(static_cast<unsigned>(max_chunks), p.H);
  ProfScope prof(kProfIntra, s);
  intra_kernel<D, ERASE><<<grid, IntraCfg<D>::kThreads, smem, s>>>(p);
  return cuda_status(cudaGetLastError());
}

int launch_intra(int D, bool erase, const IntraParams& p, int64_t max_chunks, cudaStream_t s) {
  switch (D) {
    case 64: return erase ? launch_intra_t<64, true>(p, max_chunks, s) : launch_intra_t<64, false>(p, max_chunks, s);
    case 128: return erase ? launch_intra_t<128, true>(p, max_chunks, s) : launch_intra_t<128, false>(p, max_chunks, s);
    case 256: return erase ? launch_intra_t<256, true>(p, max_chunks, s) : launch_intra_t<256, false>(p, max_chunks, s);
    default: return MEMT_ERR_UNSUPPORTED;
  }
}

}  // namespace memt
