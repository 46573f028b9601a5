// Launcher for the inter-chunk state scan (scan.cuh).
#include "launch.h"
#include "scan.cuh"
#include "scan_tc.cuh"
#include "scan_tc256.cuh"

namespace memt {

template <int D>
static int launch_scan_t(const ScanParams& p, cudaStream_t s) {
  using Cfg = ScanCfg<D>;
  cudaError_t e = ensure_smem(scan_kernel<D>, Cfg::kSmem);
  if (e != cudaSuccess) return cuda_status(e);
  const unsigned grid = static_cast<unsigned>(p.N) * p.H * (D / Cfg::BV);
  ProfScope prof(kProfScan, s);
  return cuda_status(launch_pdl(scan_kernel<D>, dim3(grid), dim3(Cfg::kThreads), Cfg::kSmem, s, p));
}

// d = 128: tcgen05 kernel, one CTA per (sample, head), or per (sample, head, 64-value half)
// when that many CTAs are resident at once (few chains, e.g. a head-sharded rank's slice): the
// chain step is the same, each CTA's share of it halves
template <int VB>
static int launch_scan_tc_vb(const ScanParams& p, cudaStream_t s) {
  using Cfg = ScanTcCfg<VB>;
  cudaError_t e = ensure_smem(scan_tc_kernel<VB>, Cfg::kSmem);
  if (e != cudaSuccess) return cuda_status(e);
  const unsigned grid = static_cast<unsigned>(p.N) * p.H * VB;
  ProfScope prof(kProfScan, s);
  return cuda_status(launch_pdl(scan_tc_kernel<VB>, dim3(grid), dim3(Cfg::kThreads), Cfg::kSmem, s, p));
}

static int launch_scan_tc(const ScanParams& p, cudaStream_t s) {
  int slots = 0;
  cudaError_t e = ensure_smem(scan_tc_kernel<2>, ScanTcCfg<2>::kSmem);
  if (e == cudaSuccess) e = resident_slots(scan_tc_kernel<2>, ScanTcCfg<2>::kThreads, ScanTcCfg<2>::kSmem, &slots);
  if (e != cudaSuccess) return cuda_status(e);
  if (int64_t(p.N) * p.H * 2 <= slots) return launch_scan_tc_vb<2>(p, s);
  return launch_scan_tc_vb<1>(p, s);
}

// d = 256: tcgen05 kernel, one CTA per (sample, head, 128-value block)
static int launch_scan_tc256(const ScanParams& p, cudaStream_t s) {
  using Cfg = ScanTc256Cfg;
  cudaError_t e = ensure_smem(scan_tc256_kernel, Cfg::kSmem);
  if (e != cudaSuccess) return cuda_status(e);
  const unsigned grid = static_cast<unsigned>(p.N) * p.H * Cfg::kBlocks;
  ProfScope prof(kProfScan, s);
  return cuda_status(launch_pdl(scan_tc256_kernel, dim3(grid), dim3(Cfg::kThreads), Cfg::kSmem, s, p));
}

int launch_scan(int D, const ScanParams& p, cudaStream_t s) {
  switch (D) {
    case 64: return launch_scan_t<64>(p, s);
    case 128: return launch_scan_tc(p, s);
    case 256: return launch_scan_tc256(p, s);
    default: return MEMT_ERR_UNSUPPORTED;
  }
}

}  // namespace memt
