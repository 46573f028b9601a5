// memt_qwen_prologue: argument checks and launch of the Qwen memory-block prologue
// (prologue.cuh). Declared, with the reference code it replaces, in include/memt_gdn2.h.
#include "launch.h"
#include "prologue.cuh"

namespace {

using namespace memt;

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <int D>
int launch_prologue(const PrologueParams& p, cudaStream_t s) {
  constexpr int kThreads = 256, kRowsPerCta = (kThreads / 32) * (32 / (D / 8));
  int slots = 0;
  cudaError_t e = resident_slots(qwen_prologue_kernel<D>, kThreads, 0, &slots);
  if (e != cudaSuccess) return cuda_status(e);
  const int64_t rows = p.L * p.H;
  int64_t grid = (rows + kRowsPerCta - 1) / kRowsPerCta;
  if (grid > slots) grid = slots;  // grid-stride over the rows beyond one resident wave
  ProfScope prof(kProfPrologue, s);
  qwen_prologue_kernel<D><<<static_cast<unsigned>(grid), kThreads, 0, s>>>(p);
  return cuda_status(cudaGetLastError());
}

}  // namespace

extern "C" int memt_qwen_prologue(const memt_qwen_prologue_args* a, memt_stream_t stream) {
  if (a == nullptr || a->struct_size != sizeof(memt_qwen_prologue_args)) return MEMT_ERR_INVALID_ARGUMENT;
  const int D = a->head_dim;
  if (D != 64 && D != 128 && D != 256) return MEMT_ERR_UNSUPPORTED;
  if (a->num_heads < 1 || a->total_tokens < 0 || (a->norm_kind != 0 && a->norm_kind != 1))
    return MEMT_ERR_INVALID_ARGUMENT;
  const void* ptrs[] = {a->q, a->k, a->erase_latent, a->write_latent, a->decay_latent, a->decay_bias,
                        a->decay_scale_log, a->q_out, a->k_out, a->write_out, a->log_decay_out};
  for (const void* ptr : ptrs)
    if (ptr == nullptr) return MEMT_ERR_INVALID_ARGUMENT;
  const int64_t row = int64_t(a->num_heads) * D;
  const int64_t strides[] = {a->q_stride, a->k_stride, a->erase_stride, a->write_stride, a->decay_stride};
  for (int64_t st : strides)
    if (st < row) return MEMT_ERR_INVALID_ARGUMENT;
  for (const void* ptr : ptrs)
    if (ptr != a->decay_scale_log && !aligned16(ptr)) return MEMT_ERR_MISALIGNED;
  for (int64_t st : strides)
    if (st % 8 != 0) return MEMT_ERR_MISALIGNED;  // 16-byte aligned token rows
  if (a->total_tokens == 0) return MEMT_OK;
  PrologueParams p{};
  p.H = a->num_heads;
  p.L = a->total_tokens;
  p.q = static_cast<const __nv_bfloat16*>(a->q);
  p.k = static_cast<const __nv_bfloat16*>(a->k);
  p.erase = static_cast<const __nv_bfloat16*>(a->erase_latent);
  p.write = static_cast<const __nv_bfloat16*>(a->write_latent);
  p.decay = static_cast<const __nv_bfloat16*>(a->decay_latent);
  p.sq = a->q_stride;
  p.sk = a->k_stride;
  p.se = a->erase_stride;
  p.sw = a->write_stride;
  p.sd = a->decay_stride;
  p.bias = static_cast<const __nv_bfloat16*>(a->decay_bias);
  p.scale_log = static_cast<const __nv_bfloat16*>(a->decay_scale_log);
  p.eps = a->eps;
  p.rsqrt_norm = a->norm_kind;
  p.q_out = static_cast<__nv_bfloat16*>(a->q_out);
  p.k_out = static_cast<__nv_bfloat16*>(a->k_out);
  p.w_out = static_cast<__nv_bfloat16*>(a->write_out);
  p.g_out = a->log_decay_out;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (D) {
    case 64: return launch_prologue<64>(p, s);
    case 128: return launch_prologue<128>(p, s);
    default: return launch_prologue<256>(p, s);
  }
}
