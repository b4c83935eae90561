/*
 * ssd_b200.h -- C ABI of the Mamba-2 SSD chunked scan in libema_ssd_b200.so (sm_100a).
 *
 * The reference benchmarks the EMA against the third-party
 * mamba_ssm.ops.triton.ssd_combined.mamba_chunk_scan_combined(x, dt, A, B, C,
 * chunk_size, seq_idx=None) (kernels/benchmarks/bench_ema_total.py:72-76); it has no
 * SSD kernel of its own.  These entry points replace that call (forward: its
 * _chunk_cumsum_fwd / _chunk_state_fwd / _state_passing_fwd / _bmm_chunk_fwd /
 * _chunk_scan_fwd launches; backward: the mirror launches of
 * _mamba_chunk_scan_combined_bwd), with the same layouts:
 *
 *   x, y, dx        (batch, seqlen, nheads, headdim)      bf16, headdim stride 1
 *   dt, ddt         (batch, seqlen, nheads)               fp32 contiguous (dt > 0 after the optional
 *                                                          bias / softplus / clamp map in the args)
 *   A, dA, D, dD    (nheads,)                             fp32
 *   B, C            (batch, seqlen, ngroups, dstate)      bf16, dstate stride 1
 *   dB, dC          (batch, seqlen, ngroups, dstate)      fp32 contiguous (summed over the heads of a group)
 *   states          (batch, nheads, headdim, dstate)      fp32 contiguous
 *
 * s_t = exp(dt_t A_h) s_{t-1} + dt_t x_t B_t^T,  y_t = s_t C_t + D_h x_t.
 *
 * Supported: headdim 64, dstate 128, nheads a multiple of ngroups.  The forward
 * runs on the tcgen05 tensor cores (128-token chunks, two heads per CTA) when
 * every group has an even number of heads, else on mma.sync tiles; whatever
 * chunk_size is given (the result does not depend on it), it saves the state
 * entering every 64-token internal chunk for the backward in `chunk_states`,
 * fp32 (batch, ssd_internal_chunks, nheads, headdim, dstate), and the backward
 * walks those 64-token chunks.  Launchers allocate nothing and return an EMA_*
 * status code (ema_ssd_b200.h); ema_last_error() holds the message.
 */
#ifndef SSD_B200_H_
#define SSD_B200_H_

#include "ema_ssd_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct SsdFwdArgs {
  int64_t batch, seqlen, nheads, headdim, dstate, ngroups;
  int32_t dtype;                 /* EMA_DTYPE_BF16 */
  int32_t reserved;
  const void* x;                 /* (B,L,H,P) */
  int64_t x_stride[3];           /* element strides of b, l, h */
  const float* dt;               /* (B,L,H) contiguous */
  const float* A;                /* (H,) */
  const void* B;                 /* (B,L,G,N) */
  int64_t B_stride[3];           /* element strides of b, l, g */
  const void* C;                 /* (B,L,G,N) */
  int64_t C_stride[3];
  const float* D;                /* (H,) or NULL */
  const float* initial_state;    /* (B,H,P,N) contiguous or NULL */
  void* out;                     /* (B,L,H,P) */
  int64_t out_stride[3];
  float* chunk_states;           /* (B, ssd_internal_chunks(L), H, P, N) or NULL (no backward) */
  float* final_state;            /* (B,H,P,N) or NULL */
  /* dt pre-processing inside the kernels (mamba_chunk_scan_combined's dt_bias,
   * dt_softplus and dt_limit): dt <- clamp(softplus(dt + dt_bias), dt_min, dt_max),
   * each step optional; all zero (the default of a zero-filled struct): dt as given.
   * softplus(v) = log(1 + exp(v)), and v itself above 20 (torch's threshold). */
  const float* dt_bias;          /* (H,) or NULL */
  int32_t dt_softplus;           /* non-zero: apply the softplus */
  int32_t dt_clamp;              /* non-zero: clamp to [dt_min, dt_max] */
  float dt_min, dt_max;
} SsdFwdArgs;

typedef struct SsdBwdArgs {
  int64_t batch, seqlen, nheads, headdim, dstate, ngroups;
  int32_t dtype;
  int32_t reserved;
  const void* x;
  int64_t x_stride[3];
  const float* dt;
  const float* A;
  const void* B;
  int64_t B_stride[3];
  const void* C;
  int64_t C_stride[3];
  const float* D;                /* (H,) or NULL */
  const float* chunk_states;     /* from the forward */
  const void* dout;              /* (B,L,H,P) */
  int64_t dout_stride[3];
  const float* d_final_state;    /* (B,H,P,N) or NULL */
  void* dx;                      /* (B,L,H,P) */
  int64_t dx_stride[3];
  float* ddt;                    /* (B,L,H) */
  float* dA;                     /* (H,) */
  float* dB;                     /* (B,L,G,N) fp32 */
  float* dC;                     /* (B,L,G,N) fp32 */
  float* dD;                     /* (H,) or NULL (required when D is given) */
  float* d_initial_state;        /* (B,H,P,N) or NULL */
  /* dt pre-processing inside the kernels (mamba_chunk_scan_combined's dt_bias,
   * dt_softplus and dt_limit): dt <- clamp(softplus(dt + dt_bias), dt_min, dt_max),
   * each step optional; all zero (the default of a zero-filled struct): dt as given.
   * softplus(v) = log(1 + exp(v)), and v itself above 20 (torch's threshold). */
  const float* dt_bias;          /* (H,) or NULL */
  int32_t dt_softplus;           /* non-zero: apply the softplus */
  int32_t dt_clamp;              /* non-zero: clamp to [dt_min, dt_max] */
  float dt_min, dt_max;
  /* With a dt map, ddt is the gradient of the dt given (before the bias), and
   * ddt_bias (H,) -- zero-filled by the launcher, then accumulated -- the
   * gradient of dt_bias; NULL to skip it. */
  float* ddt_bias;
} SsdBwdArgs;

/* The output gate of mamba_chunk_scan_combined's `z` argument, out = y * silu(z),
 * and its gradient, one pass each over (batch, seqlen, nheads, headdim) tensors
 * of one element type (EMA_DTYPE_*), channel stride 1, fp32 arithmetic:
 *   ssd_gate_fwd_launch:  out = y * z * sigmoid(z)
 *   ssd_gate_bwd_launch:  out = dout * z * sigmoid(z)                        (dy)
 *                         dz  = dout * y * sigmoid(z) * (1 + z (1 - sigmoid(z)))
 * Replaces the gate mamba_ssm applies in its chunk-scan kernels (no counterpart
 * in the reference, whose benchmark call passes no z: bench_ema_total.py:72-76). */
typedef struct SsdGateArgs {
  int64_t batch, seqlen, nheads, headdim;
  int32_t dtype;
  int32_t reserved;
  const void* y;    int64_t y_stride[3];     /* element strides of b, l, h */
  const void* z;    int64_t z_stride[3];
  void* out;        int64_t out_stride[3];   /* forward: the gated output; backward: dy */
  const void* dout; int64_t dout_stride[3];  /* backward only */
  void* dz;         int64_t dz_stride[3];    /* backward only */
} SsdGateArgs;
EMA_API int ssd_gate_fwd_launch(const SsdGateArgs* args, void* stream);
EMA_API int ssd_gate_bwd_launch(const SsdGateArgs* args, void* stream);

/* Number of 64-token internal chunks of a sequence: ceil(seqlen / 64). */
EMA_API int64_t ssd_internal_chunks(int64_t seqlen);
EMA_API int ssd_fwd_launch(const SsdFwdArgs* args, void* stream);
/* dB, dC, dA and dD are accumulated over heads / tokens: the launcher zero-fills
 * them on the stream first.  Their summation order is not fixed (atomics), so
 * they are not bitwise reproducible run to run. */
EMA_API int ssd_bwd_launch(const SsdBwdArgs* args, void* stream);
/* Error word of the tensor-core SSD kernels (0: none; 2: a bounded wait on the
 * device timed out; 0x100: misaligned shared memory), read on `stream` after
 * the work queued before it; zeroed afterwards when `clear` is non-zero. */
EMA_API int ssd_device_status(uint32_t* status, int clear, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SSD_B200_H_ */
