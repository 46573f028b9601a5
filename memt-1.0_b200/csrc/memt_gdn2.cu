// C ABI of the B200 GDN-2 memory hot path: argument checks, workspace layout and
// kernel dispatch. The entry points are declared (with the reference interfaces they
// replace) in include/memt_gdn2.h.
#include <cuda_runtime.h>

#include <mutex>

#include "memt_gdn2.h"
#include "common.cuh"
#include "launch.h"

namespace memt {

thread_local int g_last_cuda_error = 0;

int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return MEMT_OK;
  g_last_cuda_error = static_cast<int>(e);
  return MEMT_ERR_CUDA;
}

}  // namespace memt

namespace {

using namespace memt;

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct WsLayout {
  int64_t max_chunks;
  size_t sample_off, table, W, KG, U, Elast, total;
};

// Workspace of the bf16 update: header | sample offsets | chunk table | w | kg | u | 2^G_last
WsLayout ws_layout(int32_t N, int64_t L, int32_t H, int32_t K, int32_t V, int32_t ct) {
  WsLayout w{};
  w.max_chunks = max_chunks_bound(L, N, ct);
  size_t off = 256;  // WsHeader
  w.sample_off = off;
  off += align256(size_t(N + 1) * 4);
  w.table = off;
  off += align256(size_t(w.max_chunks) * sizeof(ChunkDesc));
  const size_t ch = size_t(w.max_chunks) * H;
  w.W = off;
  off += align256(ch * kTile * K * 2);
  w.KG = off;
  off += align256(ch * kTile * K * 2);
  w.U = off;
  off += align256(ch * kTile * V * 2);
  w.Elast = off;
  off += align256(ch * K * 4);
  w.total = off;
  return w;
}

bool dim_ok(int32_t d) { return d == 64 || d == 128 || d == 256; }

int check_update(const memt_gdn2_update_args* a) {
  if (a == nullptr || a->struct_size != sizeof(memt_gdn2_update_args)) return MEMT_ERR_INVALID_ARGUMENT;
  if (a->num_samples < 1 || a->num_heads < 1 || a->total_tokens < 0 || a->total_tokens > INT32_MAX - 1 ||
      a->chunk_tokens < 1)
    return MEMT_ERR_INVALID_ARGUMENT;
  if (!dim_ok(a->key_dim) || a->value_dim != a->key_dim) return MEMT_ERR_UNSUPPORTED;
  if (a->dtype != MEMT_BF16 && a->dtype != MEMT_F32) return MEMT_ERR_INVALID_ARGUMENT;
  if (a->cu_seqlens == nullptr || a->k == nullptr || a->v == nullptr || a->g == nullptr ||
      a->initial_state == nullptr || a->final_state == nullptr)
    return MEMT_ERR_INVALID_ARGUMENT;
  if (a->g_layout != MEMT_GATE_PER_HEAD && a->g_layout != MEMT_GATE_PER_CHANNEL) return MEMT_ERR_INVALID_ARGUMENT;
  if (a->beta_layout < MEMT_GATE_NONE || a->beta_layout > MEMT_GATE_PER_CHANNEL) return MEMT_ERR_INVALID_ARGUMENT;
  if ((a->beta_layout == MEMT_GATE_NONE) != (a->beta == nullptr)) return MEMT_ERR_INVALID_ARGUMENT;
  if (a->erase_layout == MEMT_GATE_PER_HEAD || a->write_layout == MEMT_GATE_PER_HEAD) return MEMT_ERR_UNSUPPORTED;
  if (a->erase_layout != MEMT_GATE_NONE && a->erase_layout != MEMT_GATE_PER_CHANNEL) return MEMT_ERR_INVALID_ARGUMENT;
  if (a->write_layout != MEMT_GATE_NONE && a->write_layout != MEMT_GATE_PER_CHANNEL) return MEMT_ERR_INVALID_ARGUMENT;
  if ((a->erase_layout == MEMT_GATE_NONE) != (a->erase == nullptr)) return MEMT_ERR_INVALID_ARGUMENT;
  if ((a->write_layout == MEMT_GATE_NONE) != (a->write == nullptr)) return MEMT_ERR_INVALID_ARGUMENT;
  if (!aligned16(a->k) || !aligned16(a->v) || !aligned16(a->g) || !aligned16(a->initial_state) ||
      !aligned16(a->final_state) || !aligned16(a->erase) || !aligned16(a->write) ||
      (a->beta_layout == MEMT_GATE_PER_CHANNEL && !aligned16(a->beta)))
    return MEMT_ERR_MISALIGNED;
  if ((a->initial_slots != nullptr && a->num_initial_slots < 1) || (a->final_slots != nullptr && a->num_final_slots < 1))
    return MEMT_ERR_INVALID_ARGUMENT;
  const int64_t row = int64_t(a->num_heads) * a->key_dim;
  const int64_t strides[] = {a->k_stride, a->v_stride, a->write_stride};
  for (int64_t st : strides) {
    if (st == 0) continue;
    if (st < row) return MEMT_ERR_INVALID_ARGUMENT;
    if (a->dtype != MEMT_BF16) return MEMT_ERR_UNSUPPORTED;  // the fp32 recurrence reads contiguous rows
    if (st % 8 != 0) return MEMT_ERR_MISALIGNED;              // 16-byte token rows
  }
  return MEMT_OK;
}

// plan and intra kernels of the bf16 update on stream s; *sp receives the scan's parameters
int update_bf16_front(const memt_gdn2_update_args* a, void* ws, cudaStream_t s, ScanParams* sp) {
  const int D = a->key_dim;
  const WsLayout w = ws_layout(a->num_samples, a->total_tokens, a->num_heads, D, D, a->chunk_tokens);
  unsigned char* base = static_cast<unsigned char*>(ws);
  WsHeader* hdr = reinterpret_cast<WsHeader*>(base);
  int32_t* sample_off = reinterpret_cast<int32_t*>(base + w.sample_off);
  ChunkDesc* table = reinterpret_cast<ChunkDesc*>(base + w.table);
  int st = launch_plan(a->cu_seqlens, a->num_samples, a->total_tokens, a->chunk_tokens,
                       static_cast<int32_t>(w.max_chunks), hdr, table, sample_off, s);
  if (st != MEMT_OK) return st;

  IntraParams ip{};
  ip.hdr = hdr;
  ip.table = table;
  ip.L = a->total_tokens;
  ip.H = a->num_heads;
  ip.k = static_cast<const __nv_bfloat16*>(a->k);
  ip.v = static_cast<const __nv_bfloat16*>(a->v);
  ip.g = a->g;
  ip.g_layout = a->g_layout;
  ip.beta = static_cast<const __nv_bfloat16*>(a->beta);
  ip.beta_layout = a->beta_layout;
  ip.erase = static_cast<const __nv_bfloat16*>(a->erase);
  ip.write = static_cast<const __nv_bfloat16*>(a->write);
  const int64_t row = int64_t(a->num_heads) * D;
  ip.sk = a->k_stride > 0 ? a->k_stride : row;
  ip.sv = a->v_stride > 0 ? a->v_stride : row;
  ip.sw = a->write_stride > 0 ? a->write_stride : row;
  ip.W = reinterpret_cast<__nv_bfloat16*>(base + w.W);
  ip.KG = reinterpret_cast<__nv_bfloat16*>(base + w.KG);
  ip.U = reinterpret_cast<__nv_bfloat16*>(base + w.U);
  ip.Elast = reinterpret_cast<float*>(base + w.Elast);
  if (w.max_chunks > 0) {
    st = launch_intra(D, a->erase != nullptr, ip, w.max_chunks, s);
    if (st != MEMT_OK) return st;
  }
  *sp = ScanParams{};
  sp->hdr = hdr;
  sp->sample_off = sample_off;
  sp->N = a->num_samples;
  sp->H = a->num_heads;
  sp->W = ip.W;
  sp->U = ip.U;
  sp->KG = ip.KG;
  sp->Elast = ip.Elast;
  sp->h0 = a->initial_state;
  sp->ht = a->final_state;
  sp->slots_in = a->initial_slots;
  sp->num_in = a->num_initial_slots;
  sp->slots_out = a->final_slots;
  sp->num_out = a->num_final_slots;
  return MEMT_OK;
}

int update_bf16(const memt_gdn2_update_args* a, void* ws, cudaStream_t s) {
  ScanParams sp;
  const int st = update_bf16_front(a, ws, s, &sp);
  if (st != MEMT_OK) return st;
  return launch_scan(a->key_dim, sp, s);
}

// A non-blocking stream of the device's highest priority, created once per device, for the
// state scan of memt_gdn2_update_read.
int scan_stream(cudaStream_t* out) {
  static std::mutex m;
  static cudaStream_t streams[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e);
  if (dev < 0 || dev >= 64) return MEMT_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(m);
  if (streams[dev] == nullptr) {
    int least = 0, greatest = 0;
    e = cudaDeviceGetStreamPriorityRange(&least, &greatest);
    if (e == cudaSuccess) e = cudaStreamCreateWithPriority(&streams[dev], cudaStreamNonBlocking, greatest);
    if (e != cudaSuccess) {
      streams[dev] = nullptr;
      return cuda_status(e);
    }
  }
  *out = streams[dev];
  return MEMT_OK;
}

// The fork/join event pair of memt_gdn2_update_read, created once per (host thread, device)
// and reused by every later call of that thread on that device. Per thread, because an event
// re-recorded by another thread between this thread's record and its wait would make the wait
// follow the other thread's stream. The events live until the process exits.
int fork_join_events(cudaEvent_t* fork, cudaEvent_t* join) {
  thread_local cudaEvent_t events[64][2] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e);
  if (dev < 0 || dev >= 64) return MEMT_ERR_UNSUPPORTED;
  for (int i = 0; i < 2; ++i) {
    if (events[dev][i] == nullptr) {
      e = cudaEventCreateWithFlags(&events[dev][i], cudaEventDisableTiming);
      if (e != cudaSuccess) {
        events[dev][i] = nullptr;
        return cuda_status(e);
      }
    }
  }
  *fork = events[dev][0];
  *join = events[dev][1];
  return MEMT_OK;
}

bool ranges_overlap(const void* a, size_t na, const void* b, size_t nb) {
  const uintptr_t x = reinterpret_cast<uintptr_t>(a), y = reinterpret_cast<uintptr_t>(b);
  return x < y + nb && y < x + na;
}

int update_f32(const memt_gdn2_update_args* a, cudaStream_t s) {
  RecurrentParams p{};
  p.cu = a->cu_seqlens;
  p.N = a->num_samples;
  p.H = a->num_heads;
  p.L = a->total_tokens;
  p.k = static_cast<const float*>(a->k);
  p.v = static_cast<const float*>(a->v);
  p.g = a->g;
  p.g_layout = a->g_layout;
  p.beta = static_cast<const float*>(a->beta);
  p.beta_layout = a->beta_layout;
  p.erase = static_cast<const float*>(a->erase);
  p.write = static_cast<const float*>(a->write);
  p.h0 = a->initial_state;
  p.ht = a->final_state;
  p.slots_in = a->initial_slots;
  p.num_in = a->num_initial_slots;
  p.slots_out = a->final_slots;
  p.num_out = a->num_final_slots;
  return launch_recurrent(a->key_dim, p, s);
}

int check_read(const memt_gdn2_read_args* a) {
  if (a == nullptr || a->struct_size != sizeof(memt_gdn2_read_args)) return MEMT_ERR_INVALID_ARGUMENT;
  if (a->num_blocks < 1 || a->num_heads < 1 || a->total_tokens < 0 ||
      a->cu_seqlens == nullptr || a->q == nullptr || a->states == nullptr || a->out == nullptr)
    return MEMT_ERR_INVALID_ARGUMENT;
  if (!dim_ok(a->key_dim) || a->value_dim != a->key_dim) return MEMT_ERR_UNSUPPORTED;
  if ((a->q_dtype != MEMT_BF16 && a->q_dtype != MEMT_F32) || (a->out_dtype != MEMT_BF16 && a->out_dtype != MEMT_F32))
    return MEMT_ERR_INVALID_ARGUMENT;
  if (!aligned16(a->q) || !aligned16(a->states) || !aligned16(a->out)) return MEMT_ERR_MISALIGNED;
  if (a->state_slots != nullptr && a->num_slots < 1) return MEMT_ERR_INVALID_ARGUMENT;
  if (a->max_block_tokens < 0 || (a->max_block_tokens > 0 && int64_t(a->max_block_tokens) * a->num_blocks < a->total_tokens))
    return MEMT_ERR_INVALID_ARGUMENT;  // a bound the blocks cannot satisfy
  return MEMT_OK;
}

// the read's kernels for arguments check_read accepted
// side: the stream of the commit's scan (null for a read on its own): a tcgen05 tile read then
// runs on it right after the scan, any other read on the caller's stream beside the scan
int read_launch(const memt_gdn2_read_args* a, memt_stream_t stream, cudaStream_t side = nullptr) {
  if (a->total_tokens == 0) return MEMT_OK;
  ReadParams p{};
  p.num_blocks = a->num_blocks;
  p.H = a->num_heads;
  p.L = a->total_tokens;
  p.cu = a->cu_seqlens;
  p.q = a->q;
  p.states = a->states;
  p.scale = a->scale;
  p.out = a->out;
  p.out_bf16 = a->out_dtype == MEMT_BF16;
  p.slots = a->state_slots;
  p.num_slots = a->num_slots;
  const int64_t maxlen = a->max_block_tokens > 0 ? a->max_block_tokens : a->total_tokens;
  const bool exact = a->q_dtype == MEMT_F32;
  if (side == nullptr) return launch_read(p, a->key_dim, exact, maxlen, reinterpret_cast<cudaStream_t>(stream));
  if (read_uses_tc(p, a->key_dim, exact, maxlen)) return launch_read(p, a->key_dim, exact, maxlen, side, kReadAfterScan);
  return launch_read(p, a->key_dim, exact, maxlen, reinterpret_cast<cudaStream_t>(stream), kReadBeside);
}

}  // namespace

extern "C" {

int memt_version(void) { return 300; }

const char* memt_status_string(int status) {
  switch (status) {
    case MEMT_OK: return "ok";
    case MEMT_ERR_INVALID_ARGUMENT: return "invalid argument";
    case MEMT_ERR_UNSUPPORTED: return "unsupported shape or dtype";
    case MEMT_ERR_MISALIGNED: return "pointer not 16-byte aligned";
    case MEMT_ERR_WORKSPACE: return "workspace missing or too small";
    case MEMT_ERR_CUDA: return "CUDA error";
    default: return "unknown status";
  }
}

int memt_last_cuda_error(void) { return memt::g_last_cuda_error; }

int64_t memt_gdn2_count_chunks(const int32_t* cu, int32_t N, int32_t chunk_tokens) {
  if (cu == nullptr || N < 1 || chunk_tokens < 1) return -1;
  int64_t total = 0;
  for (int32_t n = 0; n < N; ++n) {
    if (cu[n + 1] < cu[n] || cu[n] < 0) return -1;
    total += chunks_for_length(int64_t(cu[n + 1]) - cu[n], chunk_tokens);
  }
  return total;
}

size_t memt_gdn2_update_workspace_size(int32_t N, int64_t L, int32_t H, int32_t K, int32_t V,
                                       int32_t chunk_tokens, int32_t dtype) {
  if (N < 1 || L < 0 || H < 1 || chunk_tokens < 1 || !dim_ok(K) || V != K) return 0;
  if (dtype == MEMT_F32) return 256;
  if (dtype != MEMT_BF16) return 0;
  return ws_layout(N, L, H, K, V, chunk_tokens).total;
}

int memt_gdn2_update(const memt_gdn2_update_args* a, void* workspace, size_t workspace_bytes,
                     memt_stream_t stream) {
  int st = check_update(a);
  if (st != MEMT_OK) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (a->dtype == MEMT_F32) return update_f32(a, s);
  const size_t need = memt_gdn2_update_workspace_size(a->num_samples, a->total_tokens, a->num_heads,
                                                      a->key_dim, a->value_dim, a->chunk_tokens, a->dtype);
  if (workspace == nullptr || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return MEMT_ERR_WORKSPACE;
  return update_bf16(a, workspace, s);
}

int memt_gdn2_workspace_status(const void* workspace, memt_stream_t stream, int32_t* status_out) {
  if (workspace == nullptr || status_out == nullptr) return MEMT_ERR_INVALID_ARGUMENT;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int32_t v = 0;
  cudaError_t e = cudaMemcpyAsync(&v, &static_cast<const WsHeader*>(workspace)->status, sizeof(v),
                                  cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_status(e);
  *status_out = v;
  return MEMT_OK;
}

int memt_gdn2_read(const memt_gdn2_read_args* a, memt_stream_t stream) {
  const int st = check_read(a);
  if (st != MEMT_OK) return st;
  return read_launch(a, stream);
}

int memt_gdn2_update_read(const memt_gdn2_update_args* u, void* workspace, size_t workspace_bytes,
                          const memt_gdn2_read_args* r, memt_stream_t stream) {
  int st = check_update(u);
  if (st == MEMT_OK) st = check_read(r);
  if (st != MEMT_OK) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const size_t state_bytes = size_t(u->final_slots != nullptr ? u->num_final_slots : u->num_samples) * u->num_heads *
                             u->key_dim * u->value_dim * sizeof(float);
  const size_t read_state_bytes = size_t(r->state_slots != nullptr ? r->num_slots : r->num_blocks) * r->num_heads *
                                  r->key_dim * r->value_dim * sizeof(float);
  const bool overlap_ok = u->dtype == MEMT_BF16 && r->total_tokens > 0 &&
                          !ranges_overlap(r->states, read_state_bytes, u->final_state, state_bytes);
  if (!overlap_ok) {
    // the fp32 recurrence, or a read of states the update writes (e.g. one pool updated in
    // place): in order, the read first, as it reads the incoming snapshot
    st = read_launch(r, stream);
    return st != MEMT_OK ? st : memt_gdn2_update(u, workspace, workspace_bytes, stream);
  }
  const size_t need = memt_gdn2_update_workspace_size(u->num_samples, u->total_tokens, u->num_heads,
                                                      u->key_dim, u->value_dim, u->chunk_tokens, u->dtype);
  if (workspace == nullptr || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return MEMT_ERR_WORKSPACE;
  cudaStream_t side = nullptr;
  st = scan_stream(&side);
  cudaEvent_t fork = nullptr, join = nullptr;
  if (st == MEMT_OK) st = fork_join_events(&fork, &join);
  if (st != MEMT_OK) return st;
  ScanParams sp;
  st = update_bf16_front(u, workspace, s, &sp);
  if (st != MEMT_OK) return st;
  // fork after the intra kernel: the scan on the high-priority stream; the read after it on the
  // same stream by programmatic launch (tcgen05 tile read) or on the caller's stream
  cudaError_t e = cudaEventRecord(fork, s);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(side, fork, 0);
  if (e == cudaSuccess) {
    st = launch_scan(u->key_dim, sp, side);
    const int st_read = read_launch(r, stream, side);
    e = cudaEventRecord(join, side);  // recorded even after a failed launch, so the join below holds
    if (e == cudaSuccess) e = cudaStreamWaitEvent(s, join, 0);
    if (st == MEMT_OK) st = st_read;
  }
  if (e != cudaSuccess) return cuda_status(e);
  return st;
}

int memt_memory_readout(const memt_memory_readout_args* a, memt_stream_t stream) {
  if (a == nullptr || a->struct_size != sizeof(memt_memory_readout_args)) return MEMT_ERR_INVALID_ARGUMENT;
  if (a->num_blocks < 1 || a->num_heads < 1 || a->total_tokens < 0 || a->head_offset < 0 ||
      a->cu_seqlens == nullptr || a->q == nullptr || a->states == nullptr || a->gate == nullptr ||
      a->norm_weight == nullptr || a->out == nullptr)
    return MEMT_ERR_INVALID_ARGUMENT;
  if (!dim_ok(a->head_dim)) return MEMT_ERR_UNSUPPORTED;
  if (a->row_stride < int64_t(a->head_offset + a->num_heads) * a->head_dim || (a->row_stride & 1))
    return MEMT_ERR_INVALID_ARGUMENT;
  if (!aligned16(a->q) || !aligned16(a->states) || !aligned16(a->gate) || !aligned16(a->out) ||
      !aligned16(a->residual) || !aligned16(a->norm_weight))
    return MEMT_ERR_MISALIGNED;
  if (a->state_slots != nullptr && a->num_slots < 1) return MEMT_ERR_INVALID_ARGUMENT;
  if (a->max_block_tokens < 0 || (a->max_block_tokens > 0 && int64_t(a->max_block_tokens) * a->num_blocks < a->total_tokens))
    return MEMT_ERR_INVALID_ARGUMENT;  // a bound the blocks cannot satisfy
  if (a->total_tokens == 0) return MEMT_OK;
  ReadParams p{};
  p.num_blocks = a->num_blocks;
  p.H = a->num_heads;
  p.L = a->total_tokens;
  p.cu = a->cu_seqlens;
  p.q = a->q;
  p.states = a->states;
  p.scale = a->scale;
  p.out = a->out;
  p.out_bf16 = 1;
  p.fused = 1;
  p.normalize_q = a->normalize_q;
  p.q_eps = a->q_eps;
  p.gate = static_cast<const __nv_bfloat16*>(a->gate);
  p.norm_w = static_cast<const __nv_bfloat16*>(a->norm_weight);
  p.norm_eps = a->norm_eps;
  p.softcap = a->softcap;
  p.residual = static_cast<const __nv_bfloat16*>(a->residual);
  p.row_stride = a->row_stride;
  p.head_offset = a->head_offset;
  p.slots = a->state_slots;
  p.num_slots = a->num_slots;
  const int64_t maxlen = a->max_block_tokens > 0 ? a->max_block_tokens : a->total_tokens;
  return launch_read(p, a->head_dim, false, maxlen, reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"
