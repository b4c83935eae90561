/*
 * ema_ssd_b200.h -- C ABI of the B200 (sm_100a) EMA / Mamba-2 SSD chunked-scan library
 * (libema_ssd_b200.so).
 *
 * Plain pointers and sizes only: no framework types cross this boundary.  Every
 * launcher is asynchronous on the given CUDA stream (a cudaStream_t passed as
 * void*; NULL = legacy default stream), allocates nothing, and returns an
 * EMA_* status code.  Device pointers must be 16-byte aligned; tensors are
 * row-major with the innermost (headdim / channel) stride equal to 1 unless a
 * stride array says otherwise.
 *
 * Scratch ("workspace"): the single-pass kernels publish per-chunk aggregates
 * to later CTAs (decoupled look-back).  The caller provides a device buffer of
 * at least ema_scan_workspace_size() bytes, ZERO-FILLED ONCE when allocated.
 * The kernels keep it consistent across calls by themselves (a generation
 * counter in its header tags every flag; the last CTA of each launch resets
 * the counters), so no per-call clearing is needed.  Two launches that may run
 * at the same time on the device must use different workspaces.  Bit flags in
 * the header's status word report device-side wait timeouts
 * (EMA_DEVSTATUS_*); read them with ema_workspace_status().
 */
#ifndef EMA_SSD_B200_H_
#define EMA_SSD_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define EMA_API __attribute__((visibility("default")))
#else
#define EMA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- codes -------------------------------------------------------------- */
#define EMA_DTYPE_F32 0
#define EMA_DTYPE_BF16 1
#define EMA_DTYPE_F16 2

#define EMA_IDX_NONE 0
#define EMA_IDX_I8 1
#define EMA_IDX_I32 2
#define EMA_IDX_I64 3

#define EMA_OK 0
#define EMA_ERR_INVALID_ARGUMENT 1 /* null pointer, bad shape, misaligned stride */
#define EMA_ERR_UNSUPPORTED 2      /* shape/dtype combination without a kernel */
#define EMA_ERR_WORKSPACE 3        /* workspace missing, too small or misaligned */
#define EMA_ERR_CUDA 4             /* CUDA runtime/driver call failed */

#define EMA_DEVSTATUS_LOOKBACK_TIMEOUT 1u /* a look-back wait gave up */
#define EMA_DEVSTATUS_TMA_TIMEOUT 2u      /* a TMA completion wait gave up */
#define EMA_DEVSTATUS_BAD_TICKET 4u       /* workspace counters not reset: overlapping launches */

/* ---- EMA forward ----------------------------------------------------------
 * Z[t] = a[t] * Z[t-1] + w[t] * x[t] per (batch, head, channel), Z[-1] = initial_state or 0.
 * Decay, one of:
 *   reference form: dA (B,H,L) float32 log2 decay, a = exp2(dA), w = 1;
 *   dt form:        dt (B,L,H) float32 and A (H,) float32, a = exp(dt*A), w = dt.
 * seq_idx (B,L) restarts the state where the id differs from the previous token.
 * Outputs other than `out` are optional (NULL).
 * Replaces the launch of `ema_fwd_kernel` in `ema_fwd_triton`
 * (kernels/forward/ema_ssd_fwd.py:474-500; kernel :236-398).
 */
typedef struct EmaFwdArgs {
  int64_t batch, seqlen, nheads, headdim, chunk_size;
  int32_t dtype;         /* EMA_DTYPE_* of x and out */
  int32_t seq_idx_type;  /* EMA_IDX_* (EMA_IDX_NONE when seq_idx is NULL) */
  const void* x;         /* (B,L,H,P) */
  int64_t x_stride[3];   /* element strides of batch, seqlen, head */
  void* out;             /* (B,L,H,P), dtype; NULL = state-only pass (needs final_state) */
  int64_t out_stride[3];
  const float* dA;       /* reference form, (B,H,L) contiguous, or NULL */
  const float* dt;       /* dt form, (B,L,H) contiguous, or NULL */
  const float* A;        /* dt form, (H,) */
  const void* seq_idx;   /* (B,L) contiguous or NULL */
  const float* initial_state; /* (B,H,P) contiguous or NULL */
  float* states;         /* chunk START states or NULL; element strides below */
  int64_t states_stride[4]; /* batch, chunk, head, channel */
  float* da_cs;          /* reference form only: (B,H,L) within-chunk cumsum of dA, or NULL */
  float* da_cs_sum;      /* reference form only: (B,H,nchunks) chunk totals of dA, or NULL */
  float* final_state;    /* (B,H,P) contiguous or NULL */
  void* workspace;
  size_t workspace_bytes;
  /* Not in the reference interface: the state entering token chunk_size / 2 of
   * every chunk, or NULL (dt form only, no seq_idx).  Interleaved with `states`
   * (chunk c at index 2c, its mid state at 2c + 1) it is the chunk-start state
   * array of chunk_size / 2, so the backward can run on half-size chunks. */
  float* mid_states;
  int64_t mid_states_stride[4];
  /* Not in the reference interface: dt form only, a (B,H,L) float32 buffer or
   * NULL.  When given, the launcher first copies dt into it transposed (one
   * contiguous row of seqlen values per (batch, head)), and the kernel loads
   * each tile's dt as one row instead of gathering a column strided by nheads;
   * the buffer then holds what EmaBwdArgs.dt_rows takes. */
  float* dt_rows;
} EmaFwdArgs;

/* ---- EMA backward ---------------------------------------------------------
 * Adjoint of the forward.  G[t] = dout[t] + a[t+1] G[t+1], G[L-1] seeded with
 * d_final_state; dx = w * G (+ d_last_token at t = L-1); the per-token gradient
 * of the natural-log decay is dl[t] = sum_p G[t] a[t] Z[t-1].
 * Decay, one of:
 *   reference form: da_cs (B,H,L) within-chunk cumsum of the log2 decay and
 *                   da_cs_sum (B,H,nchunks), as the forward stores them;
 *                   output dl (B,H,L) float32;
 *   dt form:        dt (B,L,H), A (H,); outputs ddt (B,L,H) and dA_out (H,)
 *                   (= sum over batch and tokens of dt * dl).
 * `states` are the forward's chunk START states (chunk 0 = the initial state).
 * Replaces the launch of `ema_ssd_bwd_kernel_dpx` in `compute_dpx`
 * (kernels/backward/ema_ssd_combined.py:128-167; kernel
 * kernels/backward/ema_ssd_bwd.py:38-295).
 */
typedef struct EmaBwdArgs {
  int64_t batch, seqlen, nheads, headdim, chunk_size;
  int32_t dtype;          /* EMA_DTYPE_* of x, dout, dx */
  int32_t reserved;
  const void* x;
  int64_t x_stride[3];
  const void* dout;
  int64_t dout_stride[3];
  void* dx;              /* NULL = state-only pass: only d_initial_state is written */
  int64_t dx_stride[3];
  const float* da_cs;     /* reference form */
  const float* da_cs_sum; /* reference form */
  const float* dt;        /* dt form */
  const float* A;         /* dt form */
  const float* states;    /* chunk start states */
  int64_t states_stride[4]; /* batch, chunk, head, channel */
  const float* d_final_state; /* (B,H,P) contiguous or NULL */
  const float* d_last_token;  /* (B,H,P) contiguous or NULL; added to dx[:, L-1] */
  float* dl;              /* reference form output (B,H,L) */
  float* ddt;             /* dt form output (B,L,H) */
  float* dA_out;          /* dt form output (H,) */
  float* d_initial_state; /* (B,H,P) contiguous or NULL */
  void* workspace;
  size_t workspace_bytes;
  /* Not in the reference interface: dt form only, dt transposed to (B,H,L)
   * (as EmaFwdArgs.dt_rows leaves it) or NULL; when given, each tile's dt is
   * read from it as one contiguous row (`dt` is still required). */
  const float* dt_rows;
} EmaBwdArgs;

/* Bytes of workspace the EMA launchers need for this shape. */
EMA_API size_t ema_scan_workspace_size(int64_t batch, int64_t seqlen, int64_t nheads, int64_t headdim,
                               int64_t chunk_size);

EMA_API int ema_fwd_launch(const EmaFwdArgs* args, void* stream);
EMA_API int ema_bwd_launch(const EmaBwdArgs* args, void* stream);

/* ---- chunk cumsum ----------------------------------------------------------
 * dA (B,H,L) float32 with element strides dA_stride[3];
 * dA_cs[t]     = sum of dA over [chunk start, t]           (inclusive);
 * dA_cs_rev[t] = sum of dA over (t, chunk end]              (exclusive, 0 at the chunk's last token);
 * with exp2 != 0 both are exponentiated (the last token's reverse value is then 1).
 * Replaces the launch of `chunk_cumsum_kernel` in `chunk_cumsum_triton`
 * (kernels/forward/ema_ssd_fwd.py:194-211; kernel :109-157).
 */
EMA_API int chunk_cumsum_launch(const float* dA, const int64_t dA_stride[3], float* dA_cs,
                        const int64_t cs_stride[3], float* dA_cs_rev, const int64_t rev_stride[3],
                        int64_t batch, int64_t nheads, int64_t seqlen, int64_t chunk_size, int32_t exp2,
                        void* stream);

/* ---- EMA forward without a caller-provided workspace ------------------------
 * No counterpart in the reference.  For callers that cannot allocate device
 * memory (an FFI host with no device allocator, a runtime whose memory plan is
 * fixed after start-up): same arguments and results as ema_fwd_launch, but the
 * look-back scratch is a static device array of EMA_NOALLOC_SCRATCH_BYTES
 * compiled into the library (held on every GPU that loads it until exit);
 * args->workspace / workspace_bytes are ignored.  Shapes needing more scratch
 * than that (ema_scan_workspace_size) are rejected with EMA_ERR_WORKSPACE.
 * The first call on a device looks up the array's address and clears it, so
 * make it before any stream capture.  Every call on a device shares the array:
 * calls that overlap on the GPU race.  Allocates nothing.
 */
#define EMA_NOALLOC_SCRATCH_BYTES (4u << 20)
EMA_API int ema_fwd_launch_noalloc(const EmaFwdArgs* args, void* stream);
/* Status word of that static scratch on the current device (the counterpart of
 * ema_workspace_status for callers that never see the array): copies it to
 * *status, synchronising with `stream`, and clears it afterwards when `clear`
 * is non-zero.  Non-zero bits (EMA_DEVSTATUS_*) mean a device-side wait gave
 * up or two calls overlapped on the array, and the results are invalid.  0
 * before the first ema_fwd_launch_noalloc on the device.  No counterpart in
 * the reference.
 */
EMA_API int ema_noalloc_status(uint32_t* status, int32_t clear, void* stream);

/* ---- dt rows ----------------------------------------------------------------
 * No counterpart in the reference.  Copies dt (B,L,H) float32 into dt_rows
 * transposed, (B,H,L): one contiguous row of seqlen values per (batch, head),
 * the layout EmaFwdArgs.dt_rows / EmaBwdArgs.dt_rows hold.  The forward fills
 * its dt_rows buffer itself; this is for a backward whose caller kept only dt.
 */
EMA_API int ema_dt_rows_launch(const float* dt, float* dt_rows, int64_t batch, int64_t seqlen, int64_t nheads,
                               void* stream);

/* ---- sequence-parallel sub-span folds -------------------------------------
 * No counterpart in the reference (its sequence-parallel hooks are the
 * d_ossm_state / d_issm_state terms of compute_dpx, ema_ssd_bwd.py:111-117,
 * 293-295).  A rank's span of every (batch, head) chain is cut into
 * `subspans` sub-spans run as batch rows; `log_decay` (batch, subspans,
 * nheads) float64 holds ld_k = A_h * sum of dt over sub-span k, `values`
 * (batch * subspans, nheads, headdim) each sub-span's boundary value from its
 * own inputs -- direction 0: its end state from a zero start; direction 1: the
 * gradient w.r.t. its start state from its own dy.  With cl_k = sum_{j<k} ld_j
 * and tot = sum_k ld_k (all folds in float64):
 *   ema_span_summary: out (batch, nheads, headdim) = the span's boundary value
 *     -- direction 0: sum_k exp(tot - cl_k - ld_k) V_k; direction 1:
 *     sum_k exp(cl_k) V_k -- and span_decay (batch, nheads) = exp(tot), or NULL.
 *   ema_span_expand: out (batch * subspans, nheads, headdim) = every
 *     sub-span's boundary value given the span's `boundary` (batch, nheads,
 *     headdim) -- direction 0 (the state entering the span): the state entering
 *     sub-span k, exp(cl_k) S + sum_{q<k} exp(cl_k - cl_q - ld_q) V_q;
 *     direction 1 (the gradient arriving at the span's end): the gradient
 *     arriving at sub-span k's end, exp(tot - cl_k - ld_k) G +
 *     sum_{q>k} exp(cl_q - cl_k - ld_k) V_q.
 * All tensors contiguous; at most 64 sub-spans.  Nothing is allocated. */
typedef struct EmaSpanFoldArgs {
  int64_t batch, subspans, nheads, headdim;
  int32_t direction;
  int32_t reserved;
  const double* log_decay;
  const float* values;
  const float* boundary;  /* expansion input */
  float* out;
  float* span_decay;      /* summary output, or NULL */
} EmaSpanFoldArgs;
EMA_API int ema_span_summary(const EmaSpanFoldArgs* args, void* stream);
EMA_API int ema_span_expand(const EmaSpanFoldArgs* args, void* stream);

/* The state-only passes of the sequence-parallel EMA (dt form) as weighted
 * column sums, per (row, head) of a (rows, seqlen, nheads, headdim) tensor
 * with cs_t = A_h * sum_{u <= t} dt_u over the row:
 *   direction 0: out = sum_t exp(cs_end - cs_t) dt_t x_t  (the row's end state
 *                from a zero start; `x` is the input x);
 *   direction 1: out = sum_t exp(cs_t) dy_t               (the gradient w.r.t. the
 *                row's start state from the row's own dy; `x` is dy).
 * out (rows, nheads, headdim) float32; headdim 32, 64 or 128; x channel stride 1,
 * other strides multiples of 16 bytes, 16-byte aligned; dt (rows, seqlen,
 * nheads) float32 contiguous.  Same results as ema_fwd_launch /
 * ema_bwd_launch in their state-only modes, without their look-back.
 * log_decay (optional, (rows, nheads) float64): A_h * sum_t dt_t per row, the
 * log of the row's decay, summed in float64 (what the sub-span folds take). */
typedef struct EmaSpanStateArgs {
  int64_t rows, seqlen, nheads, headdim;
  int32_t dtype;      /* EMA_DTYPE_* of x */
  int32_t direction;
  const void* x;
  int64_t x_stride[3];  /* element strides of row, token, head */
  const float* dt;
  const float* A;
  float* out;
  double* log_decay;  /* or NULL */
} EmaSpanStateArgs;
EMA_API int ema_span_state_launch(const EmaSpanStateArgs* args, void* stream);

/* The span exchange of the sequence-parallel EMA over NVLink peer memory, in
 * one kernel: each rank's span summary from its sub-spans (as
 * ema_span_summary), the summaries written into every rank's exchange buffer
 * with a flag per (rank, batch x head), a bounded wait for every rank's flags,
 * the fold of the spans before this one (direction 0) / after it (direction
 * 1) into `span_in`, and its expansion into every sub-span (as
 * ema_span_expand) into `out`.  No counterpart in the reference (its
 * sequence-parallel hooks are the d_ossm_state / d_issm_state arguments of
 * compute_dpx, kernels/backward/ema_ssd_bwd.py:111-117, :293-295); it replaces
 * the NCCL exchange of kernels/ema_sp.py for groups whose ranks are on
 * different GPUs of one NVLink domain.
 * Collective: every rank of the group calls it with the same shapes in the
 * same order.  `buffers[q]` is rank q's exchange buffer as mapped in this
 * process (buffers[rank] its own, from ema_p2p_alloc; the others from
 * ema_p2p_open of the owners' ema_p2p_handle), all of `buffer_bytes` >=
 * ema_span_exchange_bytes(world, batch * nheads, headdim), zeroed before the
 * group's first call.  `boundary` (optional, (batch, nheads, headdim)): the
 * sequence's initial state (direction 0, used on rank 0) or the gradient
 * w.r.t. its final state (direction 1, used on the last rank).  headdim <=
 * 128, at most 64 sub-spans, at most EMA_SPAN_EXCHANGE_MAX_RANKS ranks, and
 * batch * nheads CTAs that fit on the GPU at once (refused otherwise).  A wait
 * that passes 1 s sets bit 1 of the buffer's status word
 * (ema_span_exchange_status) and the kernel finishes with wrong values. */
#define EMA_SPAN_EXCHANGE_MAX_RANKS 8
#define EMA_P2P_HANDLE_BYTES 64
typedef struct EmaSpanExchangeArgs {
  int64_t batch, subspans, nheads, headdim;
  int32_t direction, rank, world, reserved;
  const double* log_decay; /* (batch, subspans, nheads) */
  const float* values;     /* (batch subspans, nheads, headdim): the sub-spans' boundary values */
  const float* boundary;   /* or NULL */
  float* span_in;          /* (batch, nheads, headdim) */
  float* out;              /* (batch subspans, nheads, headdim) */
  uint64_t buffer_bytes;
  void* buffers[EMA_SPAN_EXCHANGE_MAX_RANKS];
} EmaSpanExchangeArgs;
EMA_API size_t ema_span_exchange_bytes(int64_t world, int64_t batch_heads, int64_t headdim);
EMA_API int ema_span_exchange(const EmaSpanExchangeArgs* args, void* stream);
EMA_API int ema_span_exchange_status(void* own_buffer, uint32_t* status, int32_t clear);
/* Exchange buffers: cudaMalloc + zero (ema_p2p_alloc / ema_p2p_free) and their
 * CUDA IPC handles (ema_p2p_handle fills EMA_P2P_HANDLE_BYTES bytes; a peer
 * process maps the buffer with ema_p2p_open and unmaps it with ema_p2p_close). */
EMA_API int ema_p2p_alloc(size_t bytes, void** ptr);
EMA_API int ema_p2p_free(void* ptr);
EMA_API int ema_p2p_handle(void* ptr, unsigned char* handle);
EMA_API int ema_p2p_open(const unsigned char* handle, void** ptr);
EMA_API int ema_p2p_close(void* ptr);

/* ---- utilities ------------------------------------------------------------ */
/* Copies the workspace status word to *status (synchronises with `stream`). */
EMA_API int ema_workspace_status(const void* workspace, uint32_t* status, void* stream);
/* Clears the workspace status word (asynchronously on `stream`). */
EMA_API int ema_workspace_clear_status(void* workspace, void* stream);
/* Selects whether the launchers use their tensor-core (tcgen05) kernels where
 * one applies or always the CUDA-core kernels; process-wide, default 0 (the
 * CUDA-core kernels).  Bit 0 (1): the backward, for bf16, headdim 64,
 * chunk_size 128, dx requested.  Bit 1 (2): the forward, for the dt form, bf16,
 * headdim 64, chunk_size 128, out given, no seq_idx and no mid_states; it
 * rounds the decay matrix and dt x to bf16 once for y, as the reference's
 * forward does (kernels/forward/ema_ssd_fwd.py:361-368), while the states
 * stay fp32.  Returns the previous setting.  No counterpart in the reference:
 * the kernels agree within the bf16 tolerance, and this switch lets a caller
 * pick one.
 */
EMA_API int ema_set_tensor_core_path(int32_t enable);
/* Human-readable detail of the last error returned on the calling thread. */
EMA_API const char* ema_last_error(void);
/* Library version string. */
EMA_API const char* ema_version(void);

#ifdef __cplusplus
}
#endif

#endif /* EMA_SSD_B200_H_ */
