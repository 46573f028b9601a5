// Launcher for the exact fp32 recurrence (recurrent.cuh).
#include "launch.h"
#include "recurrent.cuh"

namespace memt {

template <int D>
static int launch_recurrent_t(const RecurrentParams& p, cudaStream_t s) {
  const unsigned grid = static_cast<unsigned>(p.N) * p.H * (D / 32);
  ProfScope prof(kProfRecurrent, s);
  recurrent_kernel<D><<<grid, 128, 0, s>>>(p);
  return cuda_status(cudaGetLastError());
}

int launch_recurrent(int D, const RecurrentParams& p, cudaStream_t s) {
  switch (D) {
    case 64: return launch_recurrent_t<64>(p, s);
    case 128: return launch_recurrent_t<128>(p, s);
    case 256: return launch_recurrent_t<256>(p, s);
    default: return MEMT_ERR_UNSUPPORTED;
  }
}

}  // namespace memt
