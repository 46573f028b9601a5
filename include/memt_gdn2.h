/*
 * memt_gdn2.h — C ABI of the B200 (sm_100a) GDN-2 memory hot path.
 *
 * The functions below replace the operator layer of the MemT-1.0 SGLang plugin
 * (package inference/memt_sglang of the reference). Paths in the comments are
 * relative to that package:
 *
 *   token_memory_packed   models/qwen/ops/packed.py:34-81, models/deepseek/ops/packed.py:70-108
 *                         = memt_gdn2_update (write path) + memt_gdn2_read (read of the incoming
 *                           snapshot)
 *   memt_gdn2_fwd_h and the intra-chunk WY kernels it consumes
 *                         models/qwen/ops/_triton/state.py:127-174, _vendor/fla/ops/gdn2/
 *                         chunk_intra.py:693-787, wy_fast.py:145-196, utils/cumsum.py:446-486
 *                         = memt_gdn2_update
 *   memt_gdn2_read_fwd    models/qwen/ops/read.py:10-39  = memt_gdn2_read
 *   snapshot_read         models/deepseek/ops/read.py:6-31 = memt_gdn2_read
 *   l2norm(q) + read + MemTRMSNormGated + residual injection
 *                         models/qwen/layer.py:15-31,112-131, models/qwen/integration.py:61-64
 *                         = memt_memory_readout
 *   packed_plan / build_chunk_plan (write events + 64-token tiles)
 *                         models/qwen/ops/packed.py:16-31, models/qwen/ops/layout.py:128-189
 *                         = built on the device inside memt_gdn2_update;
 *                           memt_gdn2_count_chunks gives the host the same count
 *
 * Conventions
 *   - All tensor pointers are device pointers to contiguous row-major arrays.
 *     Token-major activations are [L, H, D] (the reference's [1, L, H, D] without
 *     the leading 1). States are fp32 [N, H, K, V], V fastest, the reference's pool
 *     layout (runtime/state.py:47-51).
 *   - Samples are given by cu_seqlens (int32 device array of N+1 offsets), the
 *     reference's boundaries(lengths) (models/common/packed.py:8-9).
 *   - Every entry point is asynchronous on the given stream, never synchronises the
 *     host, allocates nothing (scratch comes from the caller's workspace) and returns a
 *     status. Arguments are checked on the host before any launch; a bad argument
 *     returns a negative status and launches nothing (the reference raises ValueError
 *     before launch: models/common/packed.py:12-34).
 *   - Device-side data that the host cannot see without a sync (cu_seqlens contents)
 *     is clamped on the device so that every access stays in bounds; the plan kernel
 *     records the problem in the workspace status word (memt_gdn2_workspace_status).
 */
#ifndef MEMT_GDN2_H
#define MEMT_GDN2_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* cudaStream_t without including the CUDA headers. */
typedef struct CUstream_st *memt_stream_t;

/* ---- status codes ---------------------------------------------------- */
#define MEMT_OK 0
#define MEMT_ERR_INVALID_ARGUMENT (-1) /* null pointer, bad count, bad enum value      */
#define MEMT_ERR_UNSUPPORTED (-2)      /* head dim / dtype combination not compiled   */
#define MEMT_ERR_MISALIGNED (-3)       /* pointer not 16-byte aligned                 */
#define MEMT_ERR_WORKSPACE (-4)        /* workspace null or smaller than required     */
#define MEMT_ERR_CUDA (-5)             /* a CUDA launch failed; see memt_last_cuda_error */

/* ---- element types ---------------------------------------------------- */
#define MEMT_F32 0
#define MEMT_BF16 1

/* ---- gate layouts ------------------------------------------------------
 * NONE:        gate absent (log-decay 0 / factor 1)
 * PER_HEAD:    one value per (token, head): [L, H]          (BASELINE's g, beta)
 * PER_CHANNEL: one value per (token, head, channel): [L, H, D] (the reference's layout)
 */
#define MEMT_GATE_NONE 0
#define MEMT_GATE_PER_HEAD 1
#define MEMT_GATE_PER_CHANNEL 2

/* Library version (major*10000 + minor*100 + patch).
 *   0.2.0  state pools by slot index (fields appended to the update, read and readout args)
 *   0.3.0  every argument struct starts with struct_size; the memory-block prologue; the
 *          DeepSeek grouped latent RMS norm; memt_gdn2_noalloc_status, memt_read_status */
int memt_version(void);  /* 300 */

/* Argument structs start with `uint32_t struct_size`, which the caller sets to
 * sizeof(the struct) as declared in this header (MEMT_ARGS_INIT does it). An entry point
 * returns MEMT_ERR_INVALID_ARGUMENT and launches nothing when struct_size is not the size this
 * library was built with, so a binding written against another version of a struct cannot
 * make the library read fields the caller never set. */
#define MEMT_ARGS_INIT(type) {(uint32_t)sizeof(type)}

/* Human-readable name of a status code. */
const char *memt_status_string(int status);

/* The cudaError_t of the last MEMT_ERR_CUDA returned on this thread (0 if none). */
int memt_last_cuda_error(void);

/* Number of 64-token chunks the update scans for these samples: the reference's
 * plan.num_chunk (models/qwen/ops/layout.py:142-149). Host array, N+1 entries.
 * Returns -1 on invalid input (non-monotonic offsets, chunk_tokens < 1). */
int64_t memt_gdn2_count_chunks(const int32_t *cu_seqlens_host, int32_t num_samples,
                               int32_t chunk_tokens);

/* ---- GDN-2 chunked update (the writer) ---------------------------------
 *
 * Replaces the write half of token_memory_packed: chunk_local_cumsum ->
 * chunk_gdn2_fwd_intra (token-parallel diagonal, inter-solve, WY recompute) ->
 * memt_gdn2_fwd_h (models/qwen/ops/packed.py:49-79).
 *
 * Per sample, starting from initial_state, for each token t and head h
 * (a_t = exp(g_t), k'_t = sqrt(beta_t) * k_t, b = erase, w = write):
 *     S  <- diag(a_t) S
 *     d  <- w_t*v_t - S^T (b_t*k'_t)
 *     S  <- S + k'_t d^T
 * computed with the chunked WY algorithm (64-token chunks). final_state receives S.
 *
 * dtype BF16: k, v, beta, erase, write are bf16; the tensor-core path reproduces the
 *   reference GPU rounding points (bf16 A^-1, u, w, kg; bf16 state and v_new operands;
 *   tf32 solve). dtype F32: all inputs fp32, exact fp32 token recurrence on CUDA cores.
 * g is always fp32 natural-log decay (<= 0).
 * initial_state may alias final_state (in-place update).
 */
typedef struct memt_gdn2_update_args {
  uint32_t struct_size;    /* sizeof(memt_gdn2_update_args)                     */
  int32_t num_samples;     /* N >= 1                                            */
  int32_t num_heads;       /* H >= 1                                            */
  int32_t key_dim;         /* K: 64, 128 or 256                                 */
  int32_t value_dim;       /* V: equal to K                                     */
  int64_t total_tokens;    /* L = cu_seqlens[N]                                 */
  int32_t chunk_tokens;    /* write-event length (reference chunk_tokens), >= 1 */
  int32_t dtype;           /* MEMT_BF16 or MEMT_F32                             */
  const int32_t *cu_seqlens; /* device [N+1]                                    */
  const void *k;           /* [L,H,K] (already L2-normalised), rows of k_stride  */
  const void *v;           /* [L,H,V], rows of v_stride                         */
  const float *g;          /* log-decay, layout g_layout (PER_HEAD or PER_CHANNEL) */
  int32_t g_layout;
  const void *beta;        /* sqrt(beta) folded into k; NONE / PER_HEAD / PER_CHANNEL */
  int32_t beta_layout;
  const void *erase;       /* FLA channel-wise erase factor b; NONE or PER_CHANNEL  */
  int32_t erase_layout;
  const void *write;       /* write gate on V; NONE or PER_CHANNEL ([L,H,V])        */
  int32_t write_layout;
  const float *initial_state; /* [N,H,K,V] fp32                                  */
  float *final_state;         /* [N,H,K,V] fp32                                  */
  /* Optional state pools (replace the executor's gather before and index_copy_ after the
   * update, runtime/executor.py:84-110): NULL, or device int32 [N] slot indices. Sample n then
   * starts from initial_state[initial_slots[n]] of a pool [num_initial_slots,H,K,V] and/or
   * ends in final_state[final_slots[n]] of a pool [num_final_slots,H,K,V] (the two pools may
   * be one tensor; distinct samples need distinct final slots). An input slot outside its
   * pool starts from a zero state, an output slot outside its pool is not written; both set
   * bit 3 of the workspace status word (bf16 update). */
  const int32_t *initial_slots;
  int32_t num_initial_slots;
  const int32_t *final_slots;
  int32_t num_final_slots;
  /* Elements per token row of k, v and write (0: H*K, the contiguous layout). A larger stride
   * (a multiple of 8, bf16 update only) reads k, v or the write gate in place from a wider
   * buffer, e.g. the split views of one q/k/v projection output. */
  int64_t k_stride;
  int64_t v_stride;
  int64_t write_stride;
} memt_gdn2_update_args;

/* Workspace bytes memt_gdn2_update needs for these sizes (0 on invalid sizes). */
size_t memt_gdn2_update_workspace_size(int32_t num_samples, int64_t total_tokens, int32_t num_heads,
                                       int32_t key_dim, int32_t value_dim, int32_t chunk_tokens,
                                       int32_t dtype);

/* Run the update. workspace: device memory of at least the size above, 256-byte aligned. */
int memt_gdn2_update(const memt_gdn2_update_args *args, void *workspace, size_t workspace_bytes,
                     memt_stream_t stream);

/* ---- the update without any allocation ---------------------------------
 *
 * No counterpart in the reference: it exists for callers that cannot allocate device memory
 * when they call the update, for example serving engines that size their device memory pool
 * once at start-up and forbid allocations inside a step, or hosts that reach this library
 * through a C FFI without a caching allocator, where a cudaMalloc/cudaFree pair around every
 * call would be slow (cudaFree synchronises the device). It runs the same kernels as
 * memt_gdn2_update but takes its scratch from a static device array of
 * MEMT_NOALLOC_SCRATCH_BYTES (64 MiB) that the library holds on each device where this entry
 * point has been called, until the process exits. Nothing is allocated: no cudaMalloc,
 * cudaFree or allocating library routine is called.
 *
 * Limits and rules:
 *   - problems whose memt_gdn2_update_workspace_size exceeds MEMT_NOALLOC_SCRATCH_BYTES are
 *     rejected with MEMT_ERR_WORKSPACE before any launch (at d = 128 that is about 1,300
 *     (64-token chunk, head) tiles, e.g. 5,000 tokens of 16 heads);
 *   - the first call on a device looks up the array's device address (cudaGetSymbolAddress)
 *     with that device current; make that first call before any stream capture;
 *   - all calls on a device share the one array: calls that overlap on the GPU (different
 *     streams, or different host threads without ordering) race. Every byte a call reads from
 *     the array it has written earlier in the same call, so nothing needs clearing between
 *     calls. */
#define MEMT_NOALLOC_SCRATCH_BYTES (64u << 20)
int memt_gdn2_update_noalloc(const memt_gdn2_update_args *args, memt_stream_t stream);

/* Status word the last memt_gdn2_update_noalloc on the current device left in the static
 * scratch (the bits of memt_gdn2_workspace_status), for callers that never see the scratch's
 * address. Synchronises the stream; intended for tests and debugging. */
int memt_gdn2_noalloc_status(memt_stream_t stream, int32_t *status_out);

/* Device status word the last update left in this workspace (0 = clean; bit 0: a sample
 * had negative length or offsets outside [0, L]; bit 1: chunk table overflow; bit 2: a copy
 * wait timed out; bit 3: a state slot outside its pool). Reading it
 * synchronises the stream; intended for tests and debugging. */
int memt_gdn2_workspace_status(const void *workspace, memt_stream_t stream, int32_t *status_out);

/* ---- snapshot read -----------------------------------------------------
 *
 * Replaces memt_gdn2_read_fwd (models/qwen/ops/read.py:10-39, kernel
 * models/qwen/ops/_triton/read.py:22-71) and snapshot_read
 * (models/deepseek/ops/read.py:6-31): every token reads the snapshot of its block,
 *     out[t,h,:] = cast_out( scale * q[t,h,:] . cast_q(states[block(t),h]) )
 * q_dtype BF16: the state is rounded to bf16 before the product and accumulated in
 * fp32 (the reference's rounding); F32: exact fp32.
 */
typedef struct memt_gdn2_read_args {
  uint32_t struct_size;    /* sizeof(memt_gdn2_read_args)                       */
  int32_t num_blocks;      /* number of snapshots / token blocks                */
  int32_t num_heads;
  int32_t key_dim;         /* 64, 128, 256                                      */
  int32_t value_dim;       /* equal to key_dim                                  */
  int64_t total_tokens;    /* L                                                 */
  int32_t max_block_tokens;/* bound on tokens per block that sizes the grid and selects the
                              kernel; 0 = L. A bound with bound * num_blocks < L is rejected.
                              Above 1, a bound below the longest block costs speed, not tokens:
                              the kernels walk every token of a block. A bound of 1 selects the
                              one-token decode kernel, which reads only the first token of a
                              longer block and records that in memt_read_status */
  const int32_t *cu_seqlens; /* device [num_blocks+1]                           */
  const void *q;           /* [L,H,K]                                           */
  int32_t q_dtype;         /* MEMT_BF16 or MEMT_F32                             */
  const float *states;     /* [num_blocks,H,K,V] fp32                           */
  float scale;
  void *out;               /* [L,H,V]                                           */
  int32_t out_dtype;       /* MEMT_BF16 or MEMT_F32                             */
  /* Optional state pool (replaces the executor's gather of the step's states,
   * runtime/executor.py:84-91): NULL, or device [num_blocks] slot indices; block n then
   * reads states[state_slots[n]] of a pool states[num_slots,H,K,V]. A block whose slot lies
   * outside [0, num_slots) is skipped and its output rows are left unwritten. */
  const int32_t *state_slots;
  int32_t num_slots;
} memt_gdn2_read_args;

int memt_gdn2_read(const memt_gdn2_read_args *args, memt_stream_t stream);

/* Status of the reads on the current device since the last call, then cleared: bit 0 = the
 * one-token decode kernel met a block of more than one token (possible only with empty blocks
 * beside it, as bounds with bound * num_blocks < L are rejected) and read only its first token.
 * Synchronises the stream; intended for tests and debugging. */
int memt_read_status(memt_stream_t stream, int32_t *status_out);

/* ---- one memory layer's commit: update and read together ---------------
 *
 * Replaces token_memory_packed (models/qwen/ops/packed.py:34-81, models/deepseek/ops/
 * packed.py:70-108), whose write path and read of the incoming snapshot are independent:
 * the same work as memt_gdn2_update followed by memt_gdn2_read, with the same arguments,
 * results and errors, but the read overlaps the update's sequential state scan. After the
 * update's intra-chunk kernel the scan runs on a library-owned stream of the device's highest
 * priority while the read runs on the caller's stream; the caller's stream then waits for the
 * scan, so everything issued to it afterwards sees both results. When the read's states
 * overlap the update's final_state (for example one state pool read and updated in place),
 * or for the fp32 (exact recurrence) update, the two run in order on the caller's stream
 * instead, the read first: it reads the incoming snapshot.
 * The library-owned stream is one per device, shared by all callers: scans issued from
 * different caller streams of one device run one after another on it. */
int memt_gdn2_update_read(const memt_gdn2_update_args *update, void *workspace, size_t workspace_bytes,
                          const memt_gdn2_read_args *read, memt_stream_t stream);

/* ---- fused memory readout (decode / query path) -----------------------
 *
 * One pass over the fp32 state for:
 *   q_hat = l2norm(q) (optional, FLA l2norm eps)        models/qwen/layer.py:116
 *   o     = bf16(scale * q_hat . bf16(S))               models/qwen/ops/_triton/read.py:51-71
 *   y     = bf16(w * bf16(o * rsqrt(mean o^2 + eps))) * L tanh(SiLU(gate)/L)
 *                                                       models/qwen/layer.py:22-31
 *   out[t, (head_offset+h)*D + v] = bf16(residual[...] + y)   (or y when residual is NULL)
 *                                                       models/qwen/integration.py:61-64
 * All activations bf16. residual may alias out (in-place add into the attention output).
 */
typedef struct memt_memory_readout_args {
  uint32_t struct_size;    /* sizeof(memt_memory_readout_args)                  */
  int32_t num_blocks;
  int32_t num_heads;       /* heads read by this call                           */
  int32_t head_dim;        /* 64, 128, 256                                      */
  int64_t total_tokens;
  int32_t max_block_tokens;/* bound on tokens per block (as in memt_gdn2_read_args); 0 = L */
  const int32_t *cu_seqlens; /* device [num_blocks+1]                           */
  const void *q;           /* bf16 [L,H,D]                                      */
  int32_t normalize_q;     /* 1: apply l2norm to q first                        */
  float q_eps;             /* l2norm epsilon (1e-6 in the reference)            */
  const float *states;     /* [num_blocks,H,D,D] fp32                           */
  float scale;
  const void *gate;        /* bf16 [L,H,D] output-gate pre-activation           */
  const void *norm_weight; /* bf16 [D]                                          */
  float norm_eps;
  float softcap;           /* L in L*tanh(SiLU(g)/L); <= 0 disables the softcap  */
  const void *residual;    /* bf16 [L, row_stride] or NULL                      */
  void *out;               /* bf16 [L, row_stride]                              */
  int64_t row_stride;      /* elements per token row of residual/out (>= (head_offset+H)*D) */
  int32_t head_offset;     /* first head column written                         */
  const int32_t *state_slots; /* optional state pool, as in memt_gdn2_read_args  */
  int32_t num_slots;
} memt_memory_readout_args;

int memt_memory_readout(const memt_memory_readout_args *args, memt_stream_t stream);

/* ---- Qwen memory-block prologue -----------------------------------------
 *
 * Replaces what QwenMemoryBlock.packed computes between its input projection and
 * token_memory_packed (models/qwen/layer.py:71-97): _write_gates (erase and write gates),
 * _log_decay (softplus decay) and _symmetric_inputs (the FLA Triton l2norm of q and k,
 * _vendor/fla/modules/l2norm.py:84-109, and the sqrt-erase fold into the key). For every token
 * t, head h and channel c, in fp32 with the reference's rounding points:
 *   q_out[t,h,:]     = bf16(q / sqrt(sum q^2 + eps))
 *   k_out[t,h,c]     = bf16(bf16(exp(0.5 logsigmoid(erase[t,h,c]))) * bf16(k / sqrt(sum k^2 + eps)))
 *   write_out[t,h,c] = bf16(sigmoid(write[t,h,c]))
 *   log_decay_out[t,h,c] = -exp(decay_scale_log[h]) * softplus(decay[t,h,c] + decay_bias[h*D+c])
 * The reference then passes erase = ones to the update; with these outputs the update is
 * called with no erase factor (erase NULL), which is the same computation. The DeepSeek block's
 * gate and q/k preparation (expand_write_gates and prepare_stable_qk,
 * models/deepseek/ops/compiled_tensor_ops.py:54-78,102-107) is the same arithmetic with its
 * rsqrt l2norm (norm_kind 1); its erase, write and decay pre-activations are the b_up, w_up and
 * f_down projections.
 * The bf16 inputs are token rows of *_stride elements (>= H*D, a multiple of 8), head h at
 * column h*D, so the q/k/v and gate projections' split views need no copy. Outputs are
 * contiguous [L, H, D]. */
typedef struct memt_qwen_prologue_args {
  uint32_t struct_size;    /* sizeof(memt_qwen_prologue_args)                   */
  int32_t num_heads;       /* H                                                 */
  int32_t head_dim;        /* D: 64, 128 or 256                                 */
  int64_t total_tokens;    /* L                                                 */
  const void *q;            int64_t q_stride;      /* bf16 query projection      */
  const void *k;            int64_t k_stride;      /* bf16 key projection        */
  const void *erase_latent; int64_t erase_stride;  /* bf16 erase-gate pre-activation (write_gates[0]) */
  const void *write_latent; int64_t write_stride;  /* bf16 write-gate pre-activation (write_gates[1]) */
  const void *decay_latent; int64_t decay_stride;  /* bf16 f_down(decay latent), [L, H*D] */
  const void *decay_bias;       /* bf16 [H*D]                                    */
  const void *decay_scale_log;  /* bf16 [H]                                      */
  float eps;                    /* l2norm epsilon (1e-6 in the reference)        */
  int32_t norm_kind;            /* 0: x / sqrt(sum x^2 + eps), the FLA l2norm of the Qwen block;
                                   1: x * rsqrt(sum x^2 + eps), the DeepSeek block's l2norm
                                   (models/deepseek/ops/normalization.py:6-8, compiled_tensor_ops.py:102-107) */
  void *q_out;                  /* bf16 [L,H,D]                                  */
  void *k_out;                  /* bf16 [L,H,D]                                  */
  void *write_out;              /* bf16 [L,H,D]                                  */
  float *log_decay_out;         /* fp32 [L,H,D]                                  */
} memt_qwen_prologue_args;

int memt_qwen_prologue(const memt_qwen_prologue_args *args, memt_stream_t stream);

/* ---- DeepSeek grouped latent RMS norm ------------------------------------
 *
 * Replaces _latent_norm as the DeepSeek memory block's low-rank q/k/v expansion applies it
 * (models/deepseek/ops/compiled_tensor_ops.py:12-41, expand_grouped_qkv): for every token t and
 * group g of a row of `groups` latents of `rank` values,
 *   out[t, g, :] = bf16( (x * rsqrt(mean(x^2) + eps[g])) * weight[g, :] ),  x = fp32(x[t, g, :])
 * The q latent is one group. The up-projections that follow are plain (grouped) GEMMs. */
typedef struct memt_latent_norm_args {
  uint32_t struct_size;    /* sizeof(memt_latent_norm_args)                     */
  int32_t groups;          /* G >= 1                                            */
  int32_t rank;            /* R, a multiple of 8                                */
  int64_t total_tokens;    /* L                                                 */
  const void *x;           /* bf16 token rows, group g at column g*R            */
  int64_t x_stride;        /* elements per token row (>= G*R, a multiple of 8)  */
  const void *weight;      /* bf16 [G, R] gains                                 */
  const float *eps;        /* device fp32 [G] epsilons, or NULL: eps_scalar     */
  float eps_scalar;
  void *out;               /* bf16 [L, G, R]                                    */
} memt_latent_norm_args;

int memt_latent_rms_norm(const memt_latent_norm_args *args, memt_stream_t stream);

/* ---- kernel timing (benchmarks) ----------------------------------------
 *
 * No counterpart in the reference (its kernels are timed from Python). When enabled,
 * every kernel this library launches is bracketed by CUDA events on its own stream and
 * its device time is accumulated per kernel family; disabled (the default) it costs
 * nothing. Families: 0 plan, 1 intra (WY operands), 2 scan, 3 read (GEMV),
 * 4 read (tensor-core tiles), 5 fp32 recurrence, 6 prologue and latent norm.
 */
#define MEMT_PROF_FAMILIES 7
int memt_profiler_enable(int on);
int memt_profiler_reset(void);
/* Synchronises the recorded events, then fills ms[i] (total device milliseconds) and
 * launches[i] for i < min(n, MEMT_PROF_FAMILIES). */
int memt_profiler_read(double *ms, int64_t *launches, int n);

#ifdef __cplusplus
}
#endif

#endif /* MEMT_GDN2_H */
