/*
 * nested_ssm.h -- C ABI of the B200 tiered Mamba2 decode state op.
 *
 * The op keeps each head's SSM state S[P][N] split along N: the first pb
 * columns ("hot") are fp32 and updated every token; the remaining N-pb
 * columns ("cold") are stored in fp8 e4m3 (one fp32 scale per headdim row),
 * bf16 or fp32, read stale with an exp(sum dt*A) decay correction, and folded
 * forward every c tokens by a rank-c replay of a per-slot ring of the chunk's
 * (x, dt, B) followed by requantisation.  Slots are addressed through a
 * continuous-batching index (state_batch_indices); rows whose slot equals
 * pad_slot_id are skipped on the GPU.
 *
 * Conventions
 *  - Every pointer is a DEVICE pointer owned by the caller; entry points never
 *    allocate and never synchronise the stream.  `stream` is a cudaStream_t
 *    (NULL = legacy default stream).
 *  - Return value: 0 (NSSM_OK) or an nssm_status; nssm_last_error() gives a
 *    message for the calling thread.  Errors found on the device (a slot
 *    index outside [0, num_slots)) are OR-ed into *status when status != NULL
 *    (bit 0: bad slot) and the row is skipped.
 *  - Strides are in elements.  The innermost dimension of every tensor is
 *    contiguous.
 *
 * Reference interfaces replaced (paths inside omin-Kwon/nested_ssm, plus the
 * third-party call the reference drives):
 *  - nssm_tiered_step  : the tiered decode of one layer = vLLM
 *        selective_state_update (vllm/model_executor/layers/mamba/ops/mamba_ssm.py:493,
 *        called at mamba_mixer2.py:1030-1046) followed by decode_readout
 *        (scale/vllm_v4_patch.py:140-179); equivalently the state-op part of
 *        _v4_fused_decode (scale/v4_fused_decode.py:45-93) and of
 *        _v4_decode (scale/v4_native_decode.py:49-169).
 *  - nssm_fresh_step   : untiered selective_state_update (the fresh control,
 *        scale/bench_v4_decode.py:241-254).
 *  - nssm_prefill_split: prefill_snapshot (scale/vllm_v4_patch.py:123-137) and the
 *        prefill capture of scale/v4_fused_decode.py:121-159.
 *  - nssm_rot_flat     : rot_flat (scale/vllm_v4_patch.py:41-45) / the fp32
 *        rotation of scale/v4_fused_decode.py:45-48.
 *  - nssm_materialize  : no single reference function; returns the exact full
 *        state the native path keeps in cache (scale/v4_native_decode.py:65-67).
 *  - nssm_gated_rmsnorm: the mixer's norm(y, gate) after the state op
 *        (scale/v4_native_decode.py:171; scale/nemotron_retrofit.py:146-161).
 *  - nssm_chunk_scan   : the prefill chunked scan of the lean prefill
 *        (scale/v4_native_decode.py:175-220), i.e. mamba_ssm's
 *        mamba_chunk_scan_combined (called at scale/v4_native_decode.py:209-216)
 *        with z = NULL and the final states returned; its final state feeds
 *        nssm_prefill_split.
 *  - nssm_draft_step / nssm_verify_step / nssm_commit_step: the hot-only self-speculative
 *        draft (install(cold="off"), scale/v4_fused_decode.py:49-55 and :140-142) and the
 *        draft -> verify -> accept cycle that scale/bench_selfspec_e2e.py:1-83 times, on the
 *        tiered state (the reference verifies against a full fp32 state it keeps besides).
 *  - nssm_conv_step    : causal_conv1d_update + split + the post-conv R rotation of
 *        _v4_fused_decode (scale/v4_fused_decode.py:39-48); the HF decode branch's
 *        conv-state roll + weighted sum + act (scale/v4_native_decode.py:36-49).
 */
#ifndef NESTED_SSM_H_
#define NESTED_SSM_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NSSM_ABI_VERSION 3

#if defined(__GNUC__)
#define NSSM_API __attribute__((visibility("default")))
#else
#define NSSM_API
#endif

typedef enum {
  NSSM_OK = 0,
  NSSM_ERR_INVALID = 1,     /* bad argument (shape, pointer, alignment, dtype) */
  NSSM_ERR_UNSUPPORTED = 2, /* valid but not compiled (e.g. hot width)        */
  NSSM_ERR_CUDA = 3         /* a CUDA runtime call failed                     */
} nssm_status;

typedef enum {
  NSSM_F32 = 0,
  NSSM_BF16 = 1,
  NSSM_F8E4M3 = 2
} nssm_dtype;

typedef enum {
  NSSM_MODE_STALE = 0,   /* y_cold = exp(glog) C.cold, glog lags one token (default) */
  NSSM_MODE_CORR = 1,    /* exact rank-c correction (scale/v4_native_decode.py:81-117) */
  NSSM_MODE_COLDOFF = 2  /* hot-only readout, cold still maintained (draft)          */
} nssm_mode;

/* One layer's tiered slot pool.  Layouts (row-major, innermost last):
 *   hot        f32        [num_slots][nheads][headdim][hot_dim]
 *   cold       cold_dtype [num_slots][nheads][headdim][dstate-hot_dim]
 *   cold_scale f32        [num_slots][nheads][headdim]   (fp8 only, else NULL)
 *   glog       f32        [num_slots][nheads]     sum of dt*A since the last flush
 *   t          i32        [num_slots][nheads]     decode tokens since prefill
 *   ring_x     io_dtype   [num_slots][nheads][chunk][headdim]
 *   ring_dt    f32        [num_slots][nheads][round_up(chunk, 4)]
 *   ring_b     f32        [num_slots][ngroups][chunk][dstate-hot_dim]
 * All base pointers must be 16-byte aligned. */
typedef struct {
  int32_t num_slots, nheads, headdim, dstate, ngroups, hot_dim, chunk;
  int32_t cold_dtype; /* nssm_dtype */
  int32_t io_dtype;   /* nssm_dtype of x / B / C / ring (F32 or BF16) */
  int32_t _pad0;
  float* hot;
  void* cold;
  float* cold_scale;
  float* glog;
  int32_t* t;
  void* ring_x;
  float* ring_dt;
  float* ring_b;
} nssm_pool;

/* Per-token inputs of one layer, in the argument order of
 * selective_state_update(state, x, dt, A, B, C, D, z, dt_bias, dt_softplus,
 * state_batch_indices, pad_slot_id, out). */
typedef struct {
  int32_t batch;          /* rows in this call                                   */
  int32_t io_dtype;       /* dtype of x, B, C (F32 or BF16)                     */
  const void* x;          /* [batch][nheads][headdim]                           */
  int64_t x_stride_b, x_stride_h;
  const void* dt;         /* [batch][nheads], pre-softplus                      */
  int64_t dt_stride_b, dt_stride_h;
  int32_t dt_dtype;       /* F32 or BF16                                        */
  int32_t dt_softplus;    /* 1: dt = softplus(dt + dt_bias)                     */
  const float* A;         /* [nheads] (negative)                               */
  const void* B;          /* [batch][ngroups][dstate]  (rotated unless R given) */
  int64_t B_stride_b;
  const void* C;          /* [batch][ngroups][dstate]                           */
  int64_t C_stride_b;
  const float* D;         /* [nheads] or NULL                                   */
  const float* dt_bias;   /* [nheads] or NULL                                   */
  float dt_min;           /* dt = max(dt, dt_min) after softplus (<=0: none)    */
  int32_t mode;           /* nssm_mode                                          */
  const float* R;         /* [ngroups][dstate][dstate] or NULL: rotate B and C first */
  const int32_t* state_batch_indices; /* [batch] slot of each row; NULL = row */
  int32_t pad_slot_id;    /* rows with this slot are skipped                    */
  int32_t out_dtype;      /* F32 or BF16                                        */
  void* out;              /* [batch][nheads][headdim]                           */
  int64_t out_stride_b, out_stride_h;
  void* workspace;        /* >= nssm_step_workspace_bytes() when R != NULL      */
  size_t workspace_bytes;
  int32_t* status;        /* optional device word, error bits OR-ed in          */
  /* Optional gated RMS norm of y, fused into the step (the mixer's norm(y, gate) after the
   * state op, scale/v4_native_decode.py:171): when norm_gate != NULL, out receives
   * weight * round_io(h / sqrt(mean_group(h^2) + eps)) with h = round_out(y) * silu(gate)
   * instead of y, exactly as nssm_gated_rmsnorm applied to the step's y.  A norm group must be
   * one SSM group of one row: norm_group_size == (nheads / ngroups) * headdim. */
  const void* norm_gate;  /* [batch][nheads*headdim] in out_dtype, or NULL         */
  int64_t norm_gate_stride_b;
  const void* norm_weight; /* [nheads*headdim]                                     */
  int32_t norm_weight_dtype; /* F32 or BF16                                        */
  int32_t norm_group_size;
  float norm_eps;
  int32_t _pad1;
} nssm_step_args;

/* Decode-token conv ahead of the state update, for one layer: the causal conv1d update of
 * the in_proj slice [x | B | C] with the per-slot conv state, the activation, the split and
 * the per-group rotation of B and C, in one launch.  Replaces causal_conv1d_update + split +
 * the R einsums of scale/v4_fused_decode.py:39-48 (HF decode branch:
 * scale/v4_native_decode.py:36-49).  Per row b (slot s) and channel d, with width K and a
 * state of L >= K-1 columns: window = last K of [state[s][d][0..L), xbc[b][d]],
 * out = act(bias[d] + sum_k weight[d][k] window[k]) (fp32, k in order), state[s][d] <- last
 * L of [state[s][d], xbc[b][d]]; B and C are rounded to io_dtype, then rotated like
 * nssm_rot_flat. */
typedef struct {
  int32_t batch;
  int32_t nheads, headdim, ngroups, dstate; /* conv_dim = nheads*headdim + 2*ngroups*dstate */
  int32_t width;          /* K (<= 8)                                             */
  int32_t state_len;      /* L, K-1 <= L <= 8                                     */
  int32_t num_slots;
  int32_t io_dtype;       /* dtype of xbc, conv_state and the outputs (F32 / BF16) */
  int32_t weight_dtype;   /* dtype of weight and bias (F32 / BF16)               */
  int32_t activation;     /* 0: none, 1: SiLU                                     */
  int32_t pad_slot_id;
  const void* xbc;        /* [batch][conv_dim]                                    */
  int64_t xbc_stride_b;
  void* conv_state;       /* element (s, d, l) at s*stride_s + d*stride_d + l*stride_l: */
  int64_t state_stride_s; /* [num_slots][conv_dim][state_len] (stride_d = L, stride_l = 1) */
  int64_t state_stride_d; /* or the HF / vLLM cache layout (stride_d = 1,               */
  int64_t state_stride_l; /*   stride_l = conv_dim)                                    */
  const void* weight;     /* [conv_dim][width]                                    */
  const void* bias;       /* [conv_dim] or NULL                                   */
  const float* R;         /* [ngroups][dstate][dstate] or NULL (no rotation)      */
  const int32_t* state_batch_indices; /* [batch] or NULL = row                   */
  void* x_out;            /* [batch][nheads*headdim]                              */
  int64_t x_out_stride_b;
  void* B_out;            /* [batch][ngroups*dstate]                              */
  void* C_out;
  int64_t bc_out_stride_b;
  int32_t* status;        /* optional device word, bit 0 = slot outside [0, num_slots) */
} nssm_conv_args;

NSSM_API int nssm_conv_step(const nssm_conv_args* args, void* stream);
NSSM_API size_t nssm_sizeof_conv_args(void);

/* Gated RMS norm of the mixer output (the step after the state op), one launch:
 * h = y * silu(gate) in fp32; per group of group_size channels h *= 1/sqrt(mean(h^2) + eps);
 * out = weight * (h rounded to io_dtype).  Replaces the NemotronH mixer's norm(y, gate)
 * (transformers Zamba2RMSNormGated; scale/v4_native_decode.py:171, restated by the reference
 * in scale/nemotron_retrofit.py:146-161).  y, gate, out: [batch][dim] in io_dtype (F32 /
 * BF16); weight: [dim] in weight_dtype; group_size divides dim and is <= 2048. */
NSSM_API int nssm_gated_rmsnorm(const void* y, int64_t y_stride, const void* gate, int64_t gate_stride,
                                const void* weight, int32_t weight_dtype, float eps, int32_t batch,
                                int32_t dim, int32_t group_size, int32_t io_dtype, void* out,
                                int64_t out_stride, void* stream);

/* Prefill chunked scan of one layer (the SSD chunk scan of mamba_ssm 2.3.2.post1
 * mamba_chunk_scan_combined with z = NULL and return_final_states; the reference's lean
 * prefill, scale/v4_native_decode.py:209-216).  Per (sequence, head), chunks of chunk_size
 * tokens: dt = clamp(softplus(dt + dt_bias), dt_min, dt_max) (softplus only if dt_softplus),
 * dA_cs = cumsum(dt * A) inside the chunk, y = C.S_prev * exp(dA_cs) + sum_{s<=l} M x_s + D x
 * with M = bf16(C_l.B_s exp(dA_cs_l - dA_cs_s) dt_s), S_chunk = sum_s x_s bf16(B_s
 * exp(dA_cs_last - dA_cs_s) dt_s), S = exp(dA_cs_last) S + S_chunk (fp32; S_prev is S entering
 * the chunk rounded to bf16).  x, B, C, y in bf16 with fp32 accumulation on the tensor cores;
 * head h uses group h / (nheads / ngroups).  Compiled for chunk_size 128, dstate 128 and
 * headdim 64 or 80.  Strides in elements; x / B / C / y 16-byte aligned with strides that are
 * multiples of 8. */
typedef struct {
  int32_t batch, seqlen, nheads, headdim, ngroups, dstate, chunk_size;
  int32_t io_dtype;       /* BF16                                                   */
  const void* x;          /* [batch][seqlen][nheads][headdim]                       */
  int64_t x_stride_b, x_stride_t;
  const void* dt;         /* [batch][seqlen][nheads], before dt_bias / softplus     */
  int64_t dt_stride_b, dt_stride_t;
  int32_t dt_dtype;       /* F32 or BF16                                            */
  int32_t dt_softplus;
  float dt_min, dt_max;   /* dt_limit; (0, +inf) is no clamp                         */
  const float* A;         /* [nheads] (negative)                                    */
  const float* D;         /* [nheads] or NULL                                       */
  const float* dt_bias;   /* [nheads] or NULL                                       */
  const void* B;          /* [batch][seqlen][ngroups][dstate]                       */
  int64_t B_stride_b, B_stride_t;
  const void* C;
  int64_t C_stride_b, C_stride_t;
  const float* initial_states; /* [batch][nheads][headdim][dstate] fp32 or NULL     */
  int64_t init_stride_b;
  void* y;                /* [batch][seqlen][nheads][headdim] bf16                  */
  int64_t y_stride_b, y_stride_t;
  float* final_states;    /* [batch][nheads][headdim][dstate] fp32 or NULL          */
  int64_t final_stride_b;
  int32_t* status;        /* optional device word, bit 1 = a tensor-core wait timed out */
} nssm_scan_args;

NSSM_API int nssm_chunk_scan(const nssm_scan_args* args, void* stream);
NSSM_API size_t nssm_sizeof_scan_args(void);

/* Bytes of workspace nssm_tiered_step / nssm_fresh_step need for `batch` rows
 * when R != NULL (the rotated B and C), 0 otherwise. */
NSSM_API size_t nssm_step_workspace_bytes(int32_t batch, int32_t ngroups, int32_t dstate,
                                 int32_t io_dtype, int32_t has_rotation);

/* Tiered decode of one token for one layer (replaces selective_state_update +
 * decode_readout, see the header comment).  Updates the pool in place and
 * writes y = C_hot.h_hot + exp(glog) C_cold.cold + D x to out. */
NSSM_API int nssm_tiered_step(const nssm_pool* pool, const nssm_step_args* args, void* stream);

/* Bytes of the library's static rotation scratch (one copy per device). */
#define NSSM_STATIC_SCRATCH_BYTES (4u << 20)

/* nssm_tiered_step without a caller workspace: for hosts that cannot allocate
 * device memory on the library's behalf (a server whose memory planner owns
 * every allocation, or an FFI binding that passes only the model's tensors).
 * No counterpart in the reference, which always allocates through torch.
 *  - args->workspace / workspace_bytes are ignored; the rotated B and C go to
 *    a fixed NSSM_STATIC_SCRATCH_BYTES array in the library's own device
 *    memory.  Nothing is allocated and nothing has to start at zero.
 *  - Limit: nssm_step_workspace_bytes(batch, ngroups, dstate, io_dtype, 1)
 *    must not exceed NSSM_STATIC_SCRATCH_BYTES (batch <= 1024 for bf16 and
 *    <= 512 for f32 at ngroups 8, dstate 128); larger calls return
 *    NSSM_ERR_INVALID.  Without R no scratch is used and there is no limit.
 *  - The first call on each device looks the array up (a one-time set-up, on
 *    the current device); make that call before any stream capture begins.
 *    The address is kept for the life of the process: after cudaDeviceReset on
 *    a device (which unloads the library's device memory there) this entry
 *    point must not be called on that device again.
 *  - All calls on one device share the array: two calls with R that may run
 *    at the same time (different streams, or different host threads) race and
 *    corrupt each other's B and C.  Issue them on one stream. */
NSSM_API int nssm_tiered_step_static(const nssm_pool* pool, const nssm_step_args* args, void* stream);

/* Untiered fp32 update of a full state [num_slots][nheads][headdim][dstate]
 * (replaces selective_state_update; the fresh control). */
NSSM_API int nssm_fresh_step(float* state, int32_t num_slots, int32_t nheads, int32_t headdim,
                    int32_t dstate, int32_t ngroups, const nssm_step_args* args,
                    void* stream);

/* Split full fp32 states (row i at state + i*state_stride_b, layout
 * [nheads][headdim][dstate]) into pool slots[i]: hot <- [:hot_dim],
 * cold <- quantise([hot_dim:]), glog <- 0, t <- 0.  Replaces prefill_snapshot. */
NSSM_API int nssm_prefill_split(const nssm_pool* pool, const float* state, int64_t state_stride_b,
                       const int32_t* slots, int32_t batch, int32_t pad_slot_id,
                       void* stream);

/* Write the exact current full fp32 state of slots[i] to out + i*out_stride_b
 * ([nheads][headdim][dstate]): hot, and cold replayed through the ring entries
 * since the last flush.  Read-only on the pool. */
NSSM_API int nssm_materialize(const nssm_pool* pool, const float* A, const int32_t* slots,
                     int32_t batch, int32_t pad_slot_id, float* out, int64_t out_stride_b,
                     void* stream);

/* out[t][g][m] = sum_n R[g][m][n] x[t][g][n] with fp32 accumulation, rounded
 * to `dtype` (F32 or BF16).  Replaces rot_flat. */
NSSM_API int nssm_rot_flat(const void* x, int64_t x_stride, int32_t dtype, const float* R,
                  int32_t T, int32_t ngroups, int32_t dstate, void* out,
                  int64_t out_stride, void* stream);

/* Hot widths compiled into this library for a given dstate, written to
 * widths[0..n) (n <= cap); returns n. */
NSSM_API int32_t nssm_supported_hot_dims(int32_t dstate, int32_t* widths, int32_t cap);

/* Upper bound on the polls of every bounded wait inside the persistent decode kernels
 * (nssm_tiered_step / nssm_tiered_step_static); 0 restores the default (2^26, seconds).
 * A wait that runs out sets bit 1 of *status, lets the copies already issued land and
 * returns without finishing its items (outputs and pool rows of that call are then
 * undefined).  Process-wide; read at each launch.  For failure-detection tests and
 * callers that want a shorter watchdog.  Returns the previous value.  No counterpart in
 * the reference (its torch ops have no device-side waits). */
NSSM_API uint32_t nssm_set_wait_polls(uint32_t polls);

/* Failure injection for tests of the timeout path; never enable it in production.  While
 * enabled, every persistent STEP launch makes its first CTA announce 16 bytes more than
 * the copies of its first item deliver, so that item's pipeline wait can never complete:
 * the CTA's waits run out after the nssm_set_wait_polls limit, bit 1 of *status is set and
 * the call returns (that call's outputs and pool rows are undefined).  No device fault,
 * trap or unbounded wait is involved.  Returns the previous setting.  No counterpart in
 * the reference. */
NSSM_API int32_t nssm_test_inject_stuck_copy(int32_t enable);

/* ---- self-speculative decoding ----------------------------------------------------------
 * A cycle per layer: nssm_draft_step for each draft token (the hot-only model), then one
 * nssm_verify_step over the n drafted tokens (the y the tiered model gives each of them),
 * then nssm_commit_step with the number of tokens each row accepted.  Verify is read-only on
 * the pool; commit of k tokens leaves the pool exactly as k nssm_tiered_step calls with the
 * same inputs would (the same kernels' arithmetic, FLUSH included when the k tokens complete a
 * chunk).  A verify / commit window may end on a chunk boundary but not cross it:
 * (t % chunk) + ntok <= chunk for every row, so a cycle drafts chunk - t % chunk tokens at most.
 * Rows that break this, or whose accept count is outside [0, ntok], are skipped and set bit 2
 * of *status. */

/* Token strides of the multi-token inputs: with nssm_step_args describing token 0 of every
 * row (x_stride_b etc. between rows), token j of row b is at + b*stride_b + j*stride_t. */
typedef struct {
  int32_t ntok;          /* tokens per row (>= 1)                                       */
  int32_t _pad0;
  int64_t x_stride_t;    /* x   [batch][ntok][nheads][headdim]                          */
  int64_t dt_stride_t;   /* dt  [batch][ntok][nheads]                                   */
  int64_t B_stride_t;    /* B   [batch][ntok][ngroups][dstate]                          */
  int64_t C_stride_t;    /* C   [batch][ntok][ngroups][dstate] (verify)                 */
  int64_t out_stride_t;  /* out [batch][ntok][nheads][headdim] (verify)                 */
  const int32_t* accept; /* commit: [batch] tokens each row keeps, 0..ntok (device)     */
} nssm_token_args;

/* Workspace of nssm_verify_step / nssm_commit_step: the rotated B and C of batch*ntok rows
 * when R != NULL, and (commit) one int32 per row. */
NSSM_API size_t nssm_spec_workspace_bytes(int32_t batch, int32_t ntok, int32_t ngroups, int32_t dstate,
                                          int32_t io_dtype, int32_t has_rotation);

/* One draft token of the hot-only model: draft [num_slots][nheads][headdim][hot_dim] fp32
 * (indexed by slot like the pool) <- h exp(dt A) + (dt B_hot) x, with h read from the pool's
 * hot slice when from_pool != 0 (the cycle's first draft token) and from draft otherwise;
 * out <- C_hot . h + D x.  The pool is not written.  args->mode and the norm are not used
 * (norm_gate must be NULL); R, dt_softplus, dt_bias and dt_min as in nssm_tiered_step. */
NSSM_API int nssm_draft_step(const nssm_pool* pool, float* draft, int32_t from_pool, const nssm_step_args* args,
                             void* stream);

/* y of tok->ntok tokens per row from the committed tiered state, exactly as that many
 * successive nssm_tiered_step calls would read them (modes STALE and COLDOFF; CORR is not
 * supported).  Read-only on the pool.  args->batch rows; args->workspace of
 * nssm_spec_workspace_bytes() when R != NULL (B and C rows must then be token-contiguous:
 * B_stride_b == ntok * B_stride_t, likewise C). */
NSSM_API int nssm_verify_step(const nssm_pool* pool, const nssm_step_args* args, const nssm_token_args* tok,
                              void* stream);

/* Make the first tok->accept[b] of tok->ntok tokens of row b permanent (hot slice, ring, glog,
 * t, and the FLUSH of rows whose chunk they complete).  Inputs x, dt, B (and R) as given to
 * nssm_verify_step; C, D, out and mode are not used.  args->workspace of
 * nssm_spec_workspace_bytes() bytes is always needed. */
NSSM_API int nssm_commit_step(const nssm_pool* pool, const nssm_step_args* args, const nssm_token_args* tok,
                              void* stream);

/* sizeof of the argument structs, for binding checks. */
NSSM_API size_t nssm_sizeof_pool(void);
NSSM_API size_t nssm_sizeof_step_args(void);
NSSM_API size_t nssm_sizeof_token_args(void);

NSSM_API int32_t nssm_abi_version(void);
NSSM_API const char* nssm_last_error(void);

#ifdef __cplusplus
}
#endif

#endif /* NESTED_SSM_H_ */
