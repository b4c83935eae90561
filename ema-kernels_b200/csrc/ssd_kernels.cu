// Mamba-2 SSD chunked scan, forward and backward, for sm_100a.
//
//   s_t = exp(dt_t A_h) s_{t-1} + dt_t x_t B_t^T   (headdim P x dstate N per head)
//   y_t = s_t C_t + D_h x_t
//
// One CTA per (batch, head) chain walks the sequence in 64-token chunks and
// keeps the chain's fp32 state (64 x 128) in registers as tensor-core
// accumulator fragments.  Per chunk, with cs the within-chunk cumsum of dt A:
//
//   forward   CB = C B^T;  M_ij = CB_ij exp(cs_i - cs_j) dt_j  (j <= i)
//             y  = M x + exp(cs) (C s^T) + D x
//             s  = exp(cs_end) s + (x^T diag(exp(cs_end - cs) dt)) B
//   backward  the adjoint of the same four contractions, chunks in reverse,
//             the state gradient in registers, the saved chunk states read
//             back (see ssd_bwd_kernel).
//
// Every contraction is a 16 x 8 x 16 bf16 tensor-core MMA (mma.sync) with fp32
// accumulation over operands staged in shared memory, both K-contiguous
// ("A B^T" form), rows padded by 8 elements so the fragment loads hit 32
// distinct banks.  Decay factors, scans and the state stay fp32; operands are
// rounded to bf16 only at the MMA inputs, as the Triton SSD kernels do.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <string>

#include "ema_common.cuh"
#include "ema_scan_dispatch.h"
#include "ssd_b200.h"

namespace emab {
void set_last_error(const char* msg);  // ema_scan_host.cu: text returned by ema_last_error()
int ssd_fwd_tc_launch(const SsdFwdArgs* a, cudaStream_t stream);  // ssd_fwd_tc.cu
int ssd_tc_status(uint32_t* out, bool clear, cudaStream_t stream);
int ssd_bwd_tc_launch(const SsdBwdArgs* a, cudaStream_t stream);  // ssd_bwd_tc.cu

namespace ssd {

using bf16 = __nv_bfloat16;

constexpr int Q = 64;     // tokens per internal chunk
constexpr int P = 64;     // headdim
constexpr int N = 128;    // dstate
constexpr int NTHR = 256;  // 8 warps
constexpr int PAD = 8;
constexpr int LQ = Q + PAD, LP = P + PAD, LN = N + PAD;  // padded row lengths (elements)

struct Params {
  int B, L, H, G, nc;
  const bf16* x;
  long long sx_b, sx_l, sx_h;
  const float* dt;
  const float* A;
  const bf16* Bm;
  long long sb_b, sb_l, sb_g;
  const bf16* Cm;
  long long sc_b, sc_l, sc_g;
  const float* D;
  const float* s0;       // initial state (B,H,P,N) or null
  bf16* y;
  long long sy_b, sy_l, sy_h;
  float* chunk_states;   // (B,nc,H,P,N) or null
  float* s_final;        // (B,H,P,N) or null
  // backward
  const bf16* dy;
  long long sdy_b, sdy_l, sdy_h;
  const float* ds_final;  // (B,H,P,N) or null
  bf16* dx;
  long long sdx_b, sdx_l, sdx_h;
  float* ddt;
  float* dA;
  float* dB;
  float* dC;
  float* dD;
  float* ds0;
  DtMap dtm;        // dt <- clamp(softplus(dt + bias)), applied as dt is staged
  float* ddt_bias;  // (H,) or null: the gradient of the bias, accumulated
};

__device__ __forceinline__ uint32_t ld32(const bf16* p) { return *reinterpret_cast<const uint32_t*>(p); }

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  uint32_t w;
  memcpy(&w, &v, 4);
  return w;
}

// c += a * b for one 16x8x16 tile (bf16 in, fp32 accumulate).
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// acc[nt] (16 x 8 each) += A[16 x K] * Bm[8 NT x K]^T; A row r at A + r * lda,
// Bm row n at Bm + n * ldb, both K-contiguous bf16 in shared memory.
// Fragment of acc[nt]: element r of lane (g, q) = (lane / 4, lane % 4) is
// row g + 8 (r / 2), column 8 nt + 2 q + (r % 2).
template <int NT, int K>
__device__ __forceinline__ void warp_gemm(const bf16* A, int lda, const bf16* Bm, int ldb, float (&acc)[NT][4],
                                          int lane) {
  const int g = lane >> 2, q = lane & 3;
#pragma unroll
  for (int k0 = 0; k0 < K; k0 += 16) {
    const uint32_t a[4] = {ld32(A + g * lda + k0 + 2 * q), ld32(A + (g + 8) * lda + k0 + 2 * q),
                           ld32(A + g * lda + k0 + 8 + 2 * q), ld32(A + (g + 8) * lda + k0 + 8 + 2 * q)};
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const bf16* b = Bm + (nt * 8 + g) * ldb + k0 + 2 * q;
      mma16816(acc[nt], a, ld32(b), ld32(b + 8));
    }
  }
}

// The same with the B operand split into a bf16 head and a bf16 residual
// (Bhi + Blo carries 16 significant bits): for the fp32 state operands whose
// products feed the cancelling decay-gradient sums.
template <int NT, int K>
__device__ __forceinline__ void warp_gemm_split(const bf16* A, int lda, const bf16* Bhi, const bf16* Blo, int ldb,
                                                float (&acc)[NT][4], int lane) {
  const int g = lane >> 2, q = lane & 3;
#pragma unroll
  for (int k0 = 0; k0 < K; k0 += 16) {
    const uint32_t a[4] = {ld32(A + g * lda + k0 + 2 * q), ld32(A + (g + 8) * lda + k0 + 2 * q),
                           ld32(A + g * lda + k0 + 8 + 2 * q), ld32(A + (g + 8) * lda + k0 + 8 + 2 * q)};
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int o = (nt * 8 + g) * ldb + k0 + 2 * q;
      mma16816(acc[nt], a, ld32(Bhi + o), ld32(Bhi + o + 8));
      mma16816(acc[nt], a, ld32(Blo + o), ld32(Blo + o + 8));
    }
  }
}
// ... and with the A operand split.
template <int NT, int K>
__device__ __forceinline__ void warp_gemm_splitA(const bf16* Ahi, const bf16* Alo, int lda, const bf16* Bm, int ldb,
                                                 float (&acc)[NT][4], int lane) {
  const int g = lane >> 2, q = lane & 3;
#pragma unroll
  for (int k0 = 0; k0 < K; k0 += 16) {
    const int o0 = g * lda + k0 + 2 * q, o1 = (g + 8) * lda + k0 + 2 * q;
    const uint32_t ah[4] = {ld32(Ahi + o0), ld32(Ahi + o1), ld32(Ahi + o0 + 8), ld32(Ahi + o1 + 8)};
    const uint32_t al[4] = {ld32(Alo + o0), ld32(Alo + o1), ld32(Alo + o0 + 8), ld32(Alo + o1 + 8)};
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const bf16* b = Bm + (nt * 8 + g) * ldb + k0 + 2 * q;
      const uint32_t b0 = ld32(b), b1 = ld32(b + 8);
      mma16816(acc[nt], ah, b0, b1);
      mma16816(acc[nt], al, b0, b1);
    }
  }
}

// bf16 head of v and the bf16 rounding of the rest.
__device__ __forceinline__ void split_bf16(float v, bf16& hi, bf16& lo) {
  hi = __float2bfloat16_rn(v);
  lo = __float2bfloat16_rn(v - __bfloat162float(hi));
}

template <int NT>
__device__ __forceinline__ void zero(float (&acc)[NT][4]) {
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
}

// Load `rows` x `cols` bf16 (cols a multiple of 8) from global rows spaced
// `gstride` apart into `dst` (row-major, leading dim ld), and optionally its
// transpose into `dstT` (leading dim ldT); rows >= nvalid are zero.
__device__ __forceinline__ void load_tile(const bf16* src, long long gstride, int rows, int cols, int nvalid,
                                          bf16* dst, int ld, bf16* dstT, int ldT) {
  const int per_row = cols / 8;
  for (int idx = threadIdx.x; idx < rows * per_row; idx += NTHR) {
    const int r = idx / per_row, c8 = (idx - r * per_row) * 8;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (r < nvalid) v = __ldg(reinterpret_cast<const uint4*>(src + r * gstride + c8));
    *reinterpret_cast<uint4*>(dst + r * ld + c8) = v;
    if (dstT != nullptr) {
      const bf16* e = reinterpret_cast<const bf16*>(&v);
#pragma unroll
      for (int k = 0; k < 8; ++k) dstT[(c8 + k) * ldT + r] = e[k];
    }
  }
}

// The same for a tile whose shape is known at compile time: every load of the
// thread is issued before any store, so the tile costs one memory round trip.
template <int ROWS, int COLS>
__device__ __forceinline__ void load_tile_batched(const bf16* src, long long gstride, int nvalid, bf16* dst, int ld,
                                                  bf16* dstT, int ldT) {
  constexpr int PER_ROW = COLS / 8, PER = ROWS * PER_ROW / NTHR;
  static_assert(ROWS * PER_ROW % NTHR == 0, "whole iterations");
  uint4 v[PER];
#pragma unroll
  for (int it = 0; it < PER; ++it) {
    const int idx = threadIdx.x + it * NTHR, r = idx / PER_ROW, c8 = (idx - r * PER_ROW) * 8;
    v[it] = (r < nvalid) ? __ldg(reinterpret_cast<const uint4*>(src + r * gstride + c8)) : make_uint4(0u, 0u, 0u, 0u);
  }
#pragma unroll
  for (int it = 0; it < PER; ++it) {
    const int idx = threadIdx.x + it * NTHR, r = idx / PER_ROW, c8 = (idx - r * PER_ROW) * 8;
    *reinterpret_cast<uint4*>(dst + r * ld + c8) = v[it];
    if (dstT != nullptr) {
      const bf16* e = reinterpret_cast<const bf16*>(&v[it]);
#pragma unroll
      for (int k = 0; k < 8; ++k) dstT[(c8 + k) * ldT + r] = e[k];
    }
  }
}

// L2 prefetch of `rows` rows of `bytes_per_row` (a multiple of 128) from `src`
// with stride `gstride_bytes`, spread over the CTA's threads.
__device__ __forceinline__ void prefetch_rows_l2(const void* src, long long gstride_bytes, int rows, int nvalid,
                                                 int bytes_per_row) {
  const int lines = bytes_per_row / 128;
  for (int idx = threadIdx.x; idx < rows * lines; idx += NTHR) {
    const int r = idx / lines, l = idx - r * lines;
    if (r < nvalid)
      asm volatile("prefetch.global.L2 [%0];" ::"l"(static_cast<const char*>(src) + r * gstride_bytes + l * 128));
  }
}

// Inclusive cumsum of v[0..63] by one warp (two elements per lane).
__device__ __forceinline__ void warp_cumsum64(float* cs, const float* v, float scale, int lane) {
  float a = v[lane] * scale, b = v[32 + lane] * scale;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float na = __shfl_up_sync(0xffffffffu, a, o), nb = __shfl_up_sync(0xffffffffu, b, o);
    if (lane >= o) {
      a += na;
      b += nb;
    }
  }
  b += __shfl_sync(0xffffffffu, a, 31);
  cs[lane] = a;
  cs[32 + lane] = b;
}

// ---------------------------------------------------------------------------
// Forward
// ---------------------------------------------------------------------------
struct FwdSmem {
  bf16 x[Q * LP];     // x chunk, token-major
  bf16 xT[P * LQ];    // x^T
  bf16 xw[P * LQ];    // x^T scaled by w_j = exp(cs_end - cs_j) dt_j
  bf16 Bm[Q * LN];    // B chunk
  bf16 BT[N * LQ];    // B^T
  bf16 Cm[Q * LN];    // C chunk
  bf16 M[Q * LQ];     // decay-masked C B^T, scaled by dt_j
  bf16 S[P * LN];     // state entering the chunk (bf16 MMA operand)
  float cs[Q];
  float dtv[Q];
};

__global__ void __launch_bounds__(NTHR, 2) ssd_fwd_kernel(const Params p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  FwdSmem& sm = *reinterpret_cast<FwdSmem*>(smem_raw);
  const int h = blockIdx.x, b = blockIdx.y;
  const int grp = h / (p.H / p.G);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, q4 = lane & 3;
  const float Ah = p.A[h];
  const float Dh = (p.D != nullptr) ? p.D[h] : 0.f;

  // state fragment of this warp: rows (headdim) p0 + [0,16), columns (dstate) n0 + [0,64)
  const int p0 = 16 * (warp & 3), n0 = 64 * (warp >> 2);
  float st[8][4];
  const size_t bh = static_cast<size_t>(b) * p.H + h;
#pragma unroll
  for (int nt = 0; nt < 8; ++nt)
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int pp = p0 + gq + 8 * (r >> 1), nn = n0 + nt * 8 + 2 * q4 + (r & 1);
      st[nt][r] = (p.s0 != nullptr) ? p.s0[(bh * P + pp) * N + nn] : 0.f;
    }
  // bf16 copy of the state for the first chunk's C s^T
#pragma unroll
  for (int nt = 0; nt < 8; ++nt)
#pragma unroll
    for (int r = 0; r < 4; r += 2) {
      const int pp = p0 + gq + 8 * (r >> 1), nn = n0 + nt * 8 + 2 * q4;
      *reinterpret_cast<uint32_t*>(&sm.S[pp * LN + nn]) = pack_bf16(st[nt][r], st[nt][r + 1]);
    }

  for (int c = 0; c < p.nc; ++c) {
    const int t0 = c * Q;
    const int nq = min(Q, p.L - t0);
    // ---- stage the chunk -------------------------------------------------
    load_tile(p.x + b * p.sx_b + static_cast<long long>(t0) * p.sx_l + h * p.sx_h, p.sx_l, Q, P, nq, sm.x, LP,
              sm.xT, LQ);
    load_tile(p.Bm + b * p.sb_b + static_cast<long long>(t0) * p.sb_l + grp * p.sb_g, p.sb_l, Q, N, nq, sm.Bm,
              LN, sm.BT, LQ);
    load_tile(p.Cm + b * p.sc_b + static_cast<long long>(t0) * p.sc_l + grp * p.sc_g, p.sc_l, Q, N, nq, sm.Cm,
              LN, nullptr, 0);
    if (tid < Q)
      sm.dtv[tid] = (tid < nq) ? dt_map(p.dtm, h, p.dt[(static_cast<size_t>(b) * p.L + t0 + tid) * p.H + h], nullptr)
                               : 0.f;
    // chunk start state, saved for the backward
    if (p.chunk_states != nullptr) {
      float* cs_out = p.chunk_states + ((static_cast<size_t>(b) * p.nc + c) * p.H + h) * P * N;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int r = 0; r < 4; r += 2) {
          const int pp = p0 + gq + 8 * (r >> 1), nn = n0 + nt * 8 + 2 * q4;
          *reinterpret_cast<float2*>(cs_out + pp * N + nn) = make_float2(st[nt][r], st[nt][r + 1]);
        }
    }
    __syncthreads();
    if (warp == 0) warp_cumsum64(sm.cs, sm.dtv, Ah, lane);
    __syncthreads();
    const float cs_end = sm.cs[Q - 1];
    // x^T scaled by the chunk-end weights
    for (int idx = tid; idx < P * Q / 2; idx += NTHR) {
      const int pp = idx / (Q / 2), j = (idx - pp * (Q / 2)) * 2;
      const float w0 = __expf(cs_end - sm.cs[j]) * sm.dtv[j], w1 = __expf(cs_end - sm.cs[j + 1]) * sm.dtv[j + 1];
      const __nv_bfloat162 xv = *reinterpret_cast<const __nv_bfloat162*>(&sm.xT[pp * LQ + j]);
      *reinterpret_cast<uint32_t*>(&sm.xw[pp * LQ + j]) =
          pack_bf16(__bfloat162float(xv.x) * w0, __bfloat162float(xv.y) * w1);
    }
    // ---- C B^T -> decay-masked M ---------------------------------------------
    {
      const int i0 = 16 * (warp & 3), j0 = 32 * (warp >> 2);
      float acc[4][4];
      zero(acc);
      warp_gemm<4, N>(sm.Cm + i0 * LN, LN, sm.Bm + j0 * LN, LN, acc, lane);
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int r = 0; r < 4; r += 2) {
          const int i = i0 + gq + 8 * (r >> 1), j = j0 + nt * 8 + 2 * q4;
          const float ci = sm.cs[i];
          const float m0 = (j <= i) ? acc[nt][r] * __expf(ci - sm.cs[j]) * sm.dtv[j] : 0.f;
          const float m1 = (j + 1 <= i) ? acc[nt][r + 1] * __expf(ci - sm.cs[j + 1]) * sm.dtv[j + 1] : 0.f;
          *reinterpret_cast<uint32_t*>(&sm.M[i * LQ + j]) = pack_bf16(m0, m1);
        }
    }
    __syncthreads();
    // ---- y = M x + exp(cs) C s^T + D x ----------------------------------------
    {
      const int i0 = 16 * (warp & 3), c0 = 32 * (warp >> 2);
      float yacc[4][4], iacc[4][4];
      zero(yacc);
      zero(iacc);
      warp_gemm<4, Q>(sm.M + i0 * LQ, LQ, sm.xT + c0 * LQ, LQ, yacc, lane);
      warp_gemm<4, N>(sm.Cm + i0 * LN, LN, sm.S + c0 * LN, LN, iacc, lane);
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int r = 0; r < 4; r += 2) {
          const int i = i0 + gq + 8 * (r >> 1), pp = c0 + nt * 8 + 2 * q4;
          if (i < nq) {
            const float e = __expf(sm.cs[i]);
            const __nv_bfloat162 xv = *reinterpret_cast<const __nv_bfloat162*>(&sm.x[i * LP + pp]);
            const float y0 = yacc[nt][r] + e * iacc[nt][r] + Dh * __bfloat162float(xv.x);
            const float y1 = yacc[nt][r + 1] + e * iacc[nt][r + 1] + Dh * __bfloat162float(xv.y);
            bf16* dst = p.y + b * p.sy_b + static_cast<long long>(t0 + i) * p.sy_l + h * p.sy_h + pp;
            *reinterpret_cast<uint32_t*>(dst) = pack_bf16(y0, y1);
          }
        }
    }
    // ---- s = exp(cs_end) s + (x^T W) B -----------------------------------------
    {
      const float dec = __expf(cs_end);
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int r = 0; r < 4; ++r) st[nt][r] *= dec;
      warp_gemm<8, Q>(sm.xw + p0 * LQ, LQ, sm.BT + n0 * LQ, LQ, st, lane);
    }
    __syncthreads();  // every warp is done with this chunk's operands (and with sm.S)
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int r = 0; r < 4; r += 2) {
        const int pp = p0 + gq + 8 * (r >> 1), nn = n0 + nt * 8 + 2 * q4;
        *reinterpret_cast<uint32_t*>(&sm.S[pp * LN + nn]) = pack_bf16(st[nt][r], st[nt][r + 1]);
      }
  }
  if (p.s_final != nullptr) {
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int r = 0; r < 4; r += 2) {
        const int pp = p0 + gq + 8 * (r >> 1), nn = n0 + nt * 8 + 2 * q4;
        *reinterpret_cast<float2*>(p.s_final + (bh * P + pp) * N + nn) = make_float2(st[nt][r], st[nt][r + 1]);
      }
  }
}

// ---------------------------------------------------------------------------
// Backward
// ---------------------------------------------------------------------------
// Chunks in reverse; dS (registers, fp32) is the gradient w.r.t. the state
// after the chunk.  With a_ij = exp(cs_i - cs_j) (j <= i), e_i = exp(cs_i),
// w_j = dt_j exp(cs_end - cs_j), CB = C B^T and DX_ij = dy_i . x_j:
//   dx_j  = sum_i CB_ij a_ij dt_j dy_i + w_j dS B_j + D dy_j
//   dB_j  = dt_j sum_i a_ij DX_ij C_i + w_j dS^T x_j            (atomics over heads)
//   dC_i  = sum_j a_ij DX_ij dt_j B_j + e_i Sin^T dy_i           (atomics over heads)
//   dS   <- exp(cs_end) dS + sum_i e_i dy_i C_i^T
//   dcs_i = sum_j T_ij - sum_k T_ki + e_i dy_i^T Sin C_i - U_i (+ state terms at the end)
//           with T_ij = CB_ij a_ij dt_j DX_ij and U_j = w_j x_j^T dS B_j
//   ddt_j = sum_i CB_ij a_ij DX_ij + U_j / dt_j + A sum_{m >= j} dcs_m
//   dA   += sum_j dt_j sum_{m >= j} dcs_m,  dD += sum dy . x
struct BwdSmem {
  bf16 x[Q * LP];
  bf16 dy[Q * LP];
  bf16 dyT[P * LQ];    // dy^T; later e_i dy_i transposed (head)
  bf16 Bm[Q * LN];
  bf16 BT[N * LQ];
  bf16 Cm[Q * LN];
  bf16 CT[N * LQ];
  bf16 dS[P * LN];     // state gradient after the chunk: head ...
  bf16 dSlo[P * LN];   // ... and residual
  bf16 dST[N * LP];    // its head, transposed
  bf16 SinT[N * LP];   // state entering the chunk, transposed: head ...
  bf16 SinTlo[N * LP]; // ... and residual
  bf16 MtT[Q * LQ];    // (CB a dt)^T; later the residual of e_i dy_i transposed
  bf16 ET[Q * LQ];     // (a DX)^T
  bf16 Ed[Q * LQ];     // a DX dt
  float cs[Q];
  float dtv[Q];
  float der[Q];        // d dt / d (dt given) per token
  float rowT[Q], colT[Q], colR[Q], inter[Q], V[Q];
  float misc[4];       // [0] sum dS_out . Sin, [1] sum dy . x
};

__device__ __forceinline__ void store_T(bf16* dstT, int ldT, int r, int c, float v) { dstT[c * ldT + r] = __float2bfloat16_rn(v); }

__global__ void __launch_bounds__(NTHR, 1) ssd_bwd_kernel(const Params p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  BwdSmem& sm = *reinterpret_cast<BwdSmem*>(smem_raw);
  const int h = blockIdx.x, b = blockIdx.y;
  const int grp = h / (p.H / p.G);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, q4 = lane & 3;
  const unsigned FULL = 0xffffffffu;
  const float Ah = p.A[h];
  const float Dh = (p.D != nullptr) ? p.D[h] : 0.f;
  const int p0 = 16 * (warp & 3), n0 = 64 * (warp >> 2);  // state-shaped tiles (rows p, columns n)
  const int r0 = 16 * (warp & 3);                          // token-row tiles
  const size_t bh = static_cast<size_t>(b) * p.H + h;

  float ds[8][4];
#pragma unroll
  for (int nt = 0; nt < 8; ++nt)
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int pp = p0 + gq + 8 * (r >> 1), nn = n0 + nt * 8 + 2 * q4 + (r & 1);
      ds[nt][r] = (p.ds_final != nullptr) ? p.ds_final[(bh * P + pp) * N + nn] : 0.f;
    }
  float dA_acc = 0.f, dD_acc = 0.f, dbias_acc = 0.f;

  for (int c = p.nc - 1; c >= 0; --c) {
    const int t0 = c * Q;
    const int nq = min(Q, p.L - t0);
    // ---- stage the chunk (one memory round trip per tile) -----------------
    load_tile_batched<Q, P>(p.x + b * p.sx_b + static_cast<long long>(t0) * p.sx_l + h * p.sx_h, p.sx_l, nq, sm.x,
                            LP, nullptr, 0);
    load_tile_batched<Q, P>(p.dy + b * p.sdy_b + static_cast<long long>(t0) * p.sdy_l + h * p.sdy_h, p.sdy_l, nq,
                            sm.dy, LP, sm.dyT, LQ);
    load_tile_batched<Q, N>(p.Bm + b * p.sb_b + static_cast<long long>(t0) * p.sb_l + grp * p.sb_g, p.sb_l, nq,
                            sm.Bm, LN, sm.BT, LQ);
    load_tile_batched<Q, N>(p.Cm + b * p.sc_b + static_cast<long long>(t0) * p.sc_l + grp * p.sc_g, p.sc_l, nq,
                            sm.Cm, LN, sm.CT, LQ);
    if (tid < Q) {
      float der = 0.f;
      sm.dtv[tid] = (tid < nq) ? dt_map(p.dtm, h, p.dt[(static_cast<size_t>(b) * p.L + t0 + tid) * p.H + h], &der)
                               : 0.f;
      sm.der[tid] = der;
      sm.rowT[tid] = sm.colT[tid] = sm.colR[tid] = sm.inter[tid] = sm.V[tid] = 0.f;
    }
    if (tid < 4) sm.misc[tid] = 0.f;
    {
      // the state entering the chunk (transposed bf16) and sum dS . Sin over this thread's fragment
      const float* sin = p.chunk_states + ((static_cast<size_t>(b) * p.nc + c) * p.H + h) * P * N;
      float part = 0.f;
      float2 svs[8][2];  // all of this thread's loads first: one round trip
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int r = 0; r < 4; r += 2) {
          const int pp = p0 + gq + 8 * (r >> 1), nn = n0 + nt * 8 + 2 * q4;
          svs[nt][r >> 1] = __ldg(reinterpret_cast<const float2*>(sin + pp * N + nn));
        }
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int r = 0; r < 4; r += 2) {
          const int pp = p0 + gq + 8 * (r >> 1), nn = n0 + nt * 8 + 2 * q4;
          const float2 sv = svs[nt][r >> 1];
          part = fmaf(ds[nt][r], sv.x, fmaf(ds[nt][r + 1], sv.y, part));
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            bf16 hi, lo;
            split_bf16(e ? sv.y : sv.x, hi, lo);
            sm.SinT[(nn + e) * LP + pp] = hi;
            sm.SinTlo[(nn + e) * LP + pp] = lo;
            split_bf16(ds[nt][r + e], hi, lo);
            sm.dS[pp * LN + nn + e] = hi;
            sm.dSlo[pp * LN + nn + e] = lo;
            sm.dST[(nn + e) * LP + pp] = hi;
          }
        }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(FULL, part, o);
      __syncthreads();  // misc zeroed
      if (lane == 0) atomicAdd(&sm.misc[0], part);
    }
    __syncthreads();
    if (warp == 0) warp_cumsum64(sm.cs, sm.dtv, Ah, lane);
    if (c > 0) {  // the next chunk (towards 0) into L2 while this one computes
      const int tp = t0 - Q;
      prefetch_rows_l2(p.x + b * p.sx_b + static_cast<long long>(tp) * p.sx_l + h * p.sx_h, p.sx_l * 2, Q, Q, P * 2);
      prefetch_rows_l2(p.dy + b * p.sdy_b + static_cast<long long>(tp) * p.sdy_l + h * p.sdy_h, p.sdy_l * 2, Q, Q,
                       P * 2);
      prefetch_rows_l2(p.Bm + b * p.sb_b + static_cast<long long>(tp) * p.sb_l + grp * p.sb_g, p.sb_l * 2, Q, Q,
                       N * 2);
      prefetch_rows_l2(p.Cm + b * p.sc_b + static_cast<long long>(tp) * p.sc_l + grp * p.sc_g, p.sc_l * 2, Q, Q,
                       N * 2);
      prefetch_rows_l2(p.chunk_states + ((static_cast<size_t>(b) * p.nc + c - 1) * p.H + h) * P * N, 512, P, P,
                       N * 4);
    }
    __syncthreads();
    const float cs_end = sm.cs[Q - 1];
    // ---- CB = C B^T and DX = dy x^T -> MtT, ET, Ed and the dcs / ddt sums ---------
    {
      const int j0 = 32 * (warp >> 2);
      float cb[4][4], dxm[4][4];
      zero(cb);
      zero(dxm);
      warp_gemm<4, N>(sm.Cm + r0 * LN, LN, sm.Bm + j0 * LN, LN, cb, lane);
      warp_gemm<4, P>(sm.dy + r0 * LP, LP, sm.x + j0 * LP, LP, dxm, lane);
      float rsum[2] = {0.f, 0.f};
      float csum[4][2], rcol[4][2];
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) csum[nt][e] = rcol[nt][e] = 0.f;
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const int i = r0 + gq + 8 * (r >> 1), j = j0 + nt * 8 + 2 * q4 + (r & 1);
          float mt = 0.f, ev = 0.f, tv = 0.f, rv = 0.f;
          if (j <= i) {
            const float a = __expf(sm.cs[i] - sm.cs[j]);
            const float dtj = sm.dtv[j];
            mt = cb[nt][r] * a * dtj;
            ev = a * dxm[nt][r];
            rv = cb[nt][r] * ev;
            tv = rv * dtj;
          }
          store_T(sm.MtT, LQ, i, j, mt);
          store_T(sm.ET, LQ, i, j, ev);
          sm.Ed[i * LQ + j] = __float2bfloat16_rn(ev * sm.dtv[j]);
          rsum[r >> 1] += tv;
          csum[nt][r & 1] += tv;
          rcol[nt][r & 1] += rv;
        }
      // row sums: over this lane's columns, then the 4 lanes of a row
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float v = rsum[e];
        v += __shfl_xor_sync(FULL, v, 1);
        v += __shfl_xor_sync(FULL, v, 2);
        if (q4 == 0) atomicAdd(&sm.rowT[r0 + gq + 8 * e], v);
      }
      // column sums: over this lane's two rows, then the 8 lanes of a column
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          float v = csum[nt][e], w = rcol[nt][e];
#pragma unroll
          for (int o = 4; o < 32; o <<= 1) {
            v += __shfl_xor_sync(FULL, v, o);
            w += __shfl_xor_sync(FULL, w, o);
          }
          if (gq == 0) {
            atomicAdd(&sm.colT[j0 + nt * 8 + 2 * q4 + e], v);
            atomicAdd(&sm.colR[j0 + nt * 8 + 2 * q4 + e], w);
          }
        }
    }
    __syncthreads();
    // ---- dx = (CB a dt)^T dy + w (B dS^T) + D dy -----------------------------------
    {
      const int c0 = 32 * (warp >> 2);
      float ax[4][4], as[4][4];
      zero(ax);
      zero(as);
      warp_gemm<4, Q>(sm.MtT + r0 * LQ, LQ, sm.dyT + c0 * LQ, LQ, ax, lane);
      warp_gemm_split<4, N>(sm.Bm + r0 * LN, LN, sm.dS + c0 * LN, sm.dSlo + c0 * LN, LN, as, lane);
      float dd = 0.f, vpart[2] = {0.f, 0.f};
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int r = 0; r < 4; r += 2) {
          const int j = r0 + gq + 8 * (r >> 1), pp = c0 + nt * 8 + 2 * q4;
          if (j < nq) {
            const float wj = sm.dtv[j] * __expf(cs_end - sm.cs[j]);
            const __nv_bfloat162 dv = *reinterpret_cast<const __nv_bfloat162*>(&sm.dy[j * LP + pp]);
            const __nv_bfloat162 xv = *reinterpret_cast<const __nv_bfloat162*>(&sm.x[j * LP + pp]);
            const float dy0 = __bfloat162float(dv.x), dy1 = __bfloat162float(dv.y);
            const float g0 = ax[nt][r] + wj * as[nt][r] + Dh * dy0;
            const float g1 = ax[nt][r + 1] + wj * as[nt][r + 1] + Dh * dy1;
            bf16* dst = p.dx + b * p.sdx_b + static_cast<long long>(t0 + j) * p.sdx_l + h * p.sdx_h + pp;
            *reinterpret_cast<uint32_t*>(dst) = pack_bf16(g0, g1);
            dd = fmaf(dy0, __bfloat162float(xv.x), fmaf(dy1, __bfloat162float(xv.y), dd));
          }
          // V_j = exp(cs_end - cs_j) x_j . (dS B_j), from the split-precision product
          const __nv_bfloat162 xv2 = *reinterpret_cast<const __nv_bfloat162*>(&sm.x[j * LP + pp]);
          vpart[r >> 1] = fmaf(as[nt][r], __bfloat162float(xv2.x),
                               fmaf(as[nt][r + 1], __bfloat162float(xv2.y), vpart[r >> 1]));
        }
      dD_acc += dd;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float v = vpart[e];
        v += __shfl_xor_sync(FULL, v, 1);
        v += __shfl_xor_sync(FULL, v, 2);
        const int j = r0 + gq + 8 * e;
        if (q4 == 0) atomicAdd(&sm.V[j], v * __expf(cs_end - sm.cs[j]));
      }
    }
    // ---- dB = dt (a DX)^T C + w x dS --------------------------------------------------
    {
      float a1[8][4], a2[8][4];
      zero(a1);
      zero(a2);
      warp_gemm<8, Q>(sm.ET + r0 * LQ, LQ, sm.CT + n0 * LQ, LQ, a1, lane);
      warp_gemm<8, P>(sm.x + r0 * LP, LP, sm.dST + n0 * LP, LP, a2, lane);
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int r = 0; r < 4; r += 2) {
          const int j = r0 + gq + 8 * (r >> 1), nn = n0 + nt * 8 + 2 * q4;
          if (j < nq) {
            const float dtj = sm.dtv[j], wj = dtj * __expf(cs_end - sm.cs[j]);
            float* dst = p.dB + ((static_cast<size_t>(b) * p.L + t0 + j) * p.G + grp) * N + nn;
            atomicAdd(reinterpret_cast<float2*>(dst),
                      make_float2(dtj * a1[nt][r] + wj * a2[nt][r], dtj * a1[nt][r + 1] + wj * a2[nt][r + 1]));
          }
        }
    }
    // ---- dC = (a DX dt) B + e dy Sin ;  inter_i = e_i (dy_i Sin) . C_i ---------------------
    {
      float a1[8][4], a2[8][4];
      zero(a1);
      zero(a2);
      warp_gemm<8, Q>(sm.Ed + r0 * LQ, LQ, sm.BT + n0 * LQ, LQ, a1, lane);
      warp_gemm_split<8, P>(sm.dy + r0 * LP, LP, sm.SinT + n0 * LP, sm.SinTlo + n0 * LP, LP, a2, lane);
      float ipart[2] = {0.f, 0.f};
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int r = 0; r < 4; r += 2) {
          const int i = r0 + gq + 8 * (r >> 1), nn = n0 + nt * 8 + 2 * q4;
          const __nv_bfloat162 cv = *reinterpret_cast<const __nv_bfloat162*>(&sm.Cm[i * LN + nn]);
          ipart[r >> 1] = fmaf(a2[nt][r], __bfloat162float(cv.x), fmaf(a2[nt][r + 1], __bfloat162float(cv.y),
                                                                       ipart[r >> 1]));
          if (i < nq) {
            const float ei = __expf(sm.cs[i]);
            float* dst = p.dC + ((static_cast<size_t>(b) * p.L + t0 + i) * p.G + grp) * N + nn;
            atomicAdd(reinterpret_cast<float2*>(dst),
                      make_float2(a1[nt][r] + ei * a2[nt][r], a1[nt][r + 1] + ei * a2[nt][r + 1]));
          }
        }
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float v = ipart[e];
        v += __shfl_xor_sync(FULL, v, 1);
        v += __shfl_xor_sync(FULL, v, 2);
        const int i = r0 + gq + 8 * e;
        if (q4 == 0) atomicAdd(&sm.inter[i], v * __expf(sm.cs[i]));
      }
    }
    // ---- dS <- exp(cs_end) dS + (e dy)^T C --------------------------------------------
    __syncthreads();  // dy^T and MtT are no longer read: they take e_i dy_i (head, residual)
    for (int idx = tid; idx < P * Q; idx += NTHR) {
      const int pp = idx / Q, i = idx - pp * Q;
      bf16 hi, lo;
      split_bf16(__expf(sm.cs[i]) * __bfloat162float(sm.dyT[pp * LQ + i]), hi, lo);
      sm.dyT[pp * LQ + i] = hi;
      sm.MtT[pp * LQ + i] = lo;
    }
    __syncthreads();
    {
      const float dec = __expf(cs_end);
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int r = 0; r < 4; ++r) ds[nt][r] *= dec;
      warp_gemm_splitA<8, Q>(sm.dyT + p0 * LQ, sm.MtT + p0 * LQ, LQ, sm.CT + n0 * LQ, LQ, ds, lane);
    }
    __syncthreads();  // the shared sums are complete
    // ---- per token: dcs, its reverse cumsum, ddt and dA -------------------------------
    if (warp == 0) {
      float dcs[2], dir[2], dtk[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int i = lane + 32 * e;
        dtk[e] = sm.dtv[i];
        const float U = dtk[e] * sm.V[i];
        dcs[e] = sm.rowT[i] - sm.colT[i] + sm.inter[i] - U;
        dir[e] = sm.colR[i] + sm.V[i];
      }
      // the chunk-end terms: sum_j U_j and exp(cs_end) dS . Sin
      float usum = dtk[0] * sm.V[lane] + dtk[1] * sm.V[lane + 32];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) usum += __shfl_xor_sync(FULL, usum, o);
      if (lane == 31) dcs[1] += usum + __expf(cs_end) * sm.misc[0];
      // reverse inclusive cumsum over the 64 tokens
      float r1 = dcs[1], r0v = dcs[0];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float n1 = __shfl_down_sync(FULL, r1, o), n0v = __shfl_down_sync(FULL, r0v, o);
        if (lane + o < 32) {
          r1 += n1;
          r0v += n0v;
        }
      }
      r0v += __shfl_sync(FULL, r1, 0);
      const float R[2] = {r0v, r1};
      float da = 0.f, db = 0.f;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int i = lane + 32 * e;
        if (i < nq) {
          const float g = (dir[e] + Ah * R[e]) * sm.der[i];
          p.ddt[(static_cast<size_t>(b) * p.L + t0 + i) * p.H + h] = g;
          db += g;
        }
        da = fmaf(dtk[e], R[e], da);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        da += __shfl_xor_sync(FULL, da, o);
        db += __shfl_xor_sync(FULL, db, o);
      }
      dA_acc += da;
      dbias_acc += db;
    }
    __syncthreads();  // before the next chunk overwrites the staged operands
  }
  // dA, dD per (batch, head) summed over batches by atomics
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) dD_acc += __shfl_xor_sync(FULL, dD_acc, o);
  if (lane == 0 && p.dD != nullptr) atomicAdd(&p.dD[h], dD_acc);
  if (tid == 0) atomicAdd(&p.dA[h], dA_acc);
  if (tid == 0 && p.ddt_bias != nullptr) atomicAdd(&p.ddt_bias[h], dbias_acc);
  if (p.ds0 != nullptr) {
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int r = 0; r < 4; r += 2) {
        const int pp = p0 + gq + 8 * (r >> 1), nn = n0 + nt * 8 + 2 * q4;
        *reinterpret_cast<float2*>(p.ds0 + (bh * P + pp) * N + nn) = make_float2(ds[nt][r], ds[nt][r + 1]);
      }
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
namespace {

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  set_last_error(buf);
  return code;
}

bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0u; }

int check_common(int64_t B, int64_t L, int64_t H, int64_t Pd, int64_t Nd, int64_t G, int dtype, const void* x,
                 const int64_t xs[3], const void* Bm, const int64_t bs[3], const void* Cm, const int64_t cs[3],
                 const float* dt, const float* A) {
  if (B < 0 || L < 0 || H <= 0 || G <= 0) return fail(EMA_ERR_INVALID_ARGUMENT, "ssd: bad shape");
  if (Pd != P || Nd != N)
    return fail(EMA_ERR_UNSUPPORTED, "ssd: headdim must be %d and dstate %d (got %lld, %lld)", P, N,
                static_cast<long long>(Pd), static_cast<long long>(Nd));
  if (H % G != 0) return fail(EMA_ERR_INVALID_ARGUMENT, "ssd: nheads must be a multiple of ngroups");
  if (dtype != EMA_DTYPE_BF16) return fail(EMA_ERR_UNSUPPORTED, "ssd: only bf16 x / B / C are supported");
  if (B > 65535 || H > 2147483647 || L > 2147483647) return fail(EMA_ERR_UNSUPPORTED, "ssd: shape too large");
  if (x == nullptr || Bm == nullptr || Cm == nullptr || dt == nullptr || A == nullptr)
    return fail(EMA_ERR_INVALID_ARGUMENT, "ssd: x, dt, A, B and C are required");
  if (!aligned16(x) || !aligned16(Bm) || !aligned16(Cm))
    return fail(EMA_ERR_INVALID_ARGUMENT, "ssd: x, B and C must be 16-byte aligned");
  for (int i = 0; i < 3; ++i)
    if (xs[i] % 8 != 0 || bs[i] % 8 != 0 || cs[i] % 8 != 0)
      return fail(EMA_ERR_INVALID_ARGUMENT, "ssd: strides of x, B and C must be multiples of 8 elements");
  return EMA_OK;
}

int launch_check(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(EMA_ERR_CUDA, "%s launch failed: %s", what, cudaGetErrorString(e));
  return EMA_OK;
}

}  // namespace
}  // namespace ssd
}  // namespace emab

using emab::ssd::Params;

extern "C" EMA_API int64_t ssd_internal_chunks(int64_t seqlen) {
  return seqlen <= 0 ? 0 : (seqlen + emab::ssd::Q - 1) / emab::ssd::Q;
}

extern "C" EMA_API int ssd_fwd_launch(const SsdFwdArgs* a, void* stream) {
  using namespace emab::ssd;
  if (a == nullptr) return fail(EMA_ERR_INVALID_ARGUMENT, "ssd_fwd: args is NULL");
  int r = check_common(a->batch, a->seqlen, a->nheads, a->headdim, a->dstate, a->ngroups, a->dtype, a->x,
                       a->x_stride, a->B, a->B_stride, a->C, a->C_stride, a->dt, a->A);
  if (r) return r;
  if (a->out == nullptr || !aligned16(a->out)) return fail(EMA_ERR_INVALID_ARGUMENT, "ssd_fwd: out is required");
  for (int i = 0; i < 3; ++i)
    if (a->out_stride[i] % 2 != 0) return fail(EMA_ERR_INVALID_ARGUMENT, "ssd_fwd: out strides must be even");
  if (a->batch == 0 || a->seqlen == 0) return EMA_OK;
  // the tensor-core kernel covers an even number of heads per group
  r = emab::ssd_fwd_tc_launch(a, static_cast<cudaStream_t>(stream));
  if (r != EMA_ERR_UNSUPPORTED) return r;
  Params p{};
  p.B = static_cast<int>(a->batch);
  p.L = static_cast<int>(a->seqlen);
  p.H = static_cast<int>(a->nheads);
  p.G = static_cast<int>(a->ngroups);
  p.nc = static_cast<int>(ssd_internal_chunks(a->seqlen));
  p.x = static_cast<const bf16*>(a->x);
  p.sx_b = a->x_stride[0];
  p.sx_l = a->x_stride[1];
  p.sx_h = a->x_stride[2];
  p.dt = a->dt;
  p.A = a->A;
  p.Bm = static_cast<const bf16*>(a->B);
  p.sb_b = a->B_stride[0];
  p.sb_l = a->B_stride[1];
  p.sb_g = a->B_stride[2];
  p.Cm = static_cast<const bf16*>(a->C);
  p.sc_b = a->C_stride[0];
  p.sc_l = a->C_stride[1];
  p.sc_g = a->C_stride[2];
  p.D = a->D;
  p.s0 = a->initial_state;
  p.y = static_cast<bf16*>(a->out);
  p.sy_b = a->out_stride[0];
  p.sy_l = a->out_stride[1];
  p.sy_h = a->out_stride[2];
  p.chunk_states = a->chunk_states;
  p.s_final = a->final_state;
  p.dtm = emab::dt_map_of(a);
  static unsigned long long attr_mask = 0;
  r = emab::ensure_smem_attr(reinterpret_cast<const void*>(ssd_fwd_kernel), static_cast<int>(sizeof(FwdSmem)),
                             &attr_mask);
  if (r) return fail(EMA_ERR_CUDA, "ssd_fwd: %s", cudaGetErrorString(static_cast<cudaError_t>(r)));
  ssd_fwd_kernel<<<dim3(p.H, p.B), NTHR, sizeof(FwdSmem), static_cast<cudaStream_t>(stream)>>>(p);
  return launch_check("ssd_fwd");
}

extern "C" EMA_API int ssd_device_status(uint32_t* status, int clear, void* stream) {
  if (status == nullptr) return emab::ssd::fail(EMA_ERR_INVALID_ARGUMENT, "ssd_device_status: status is NULL");
  return emab::ssd_tc_status(status, clear != 0, static_cast<cudaStream_t>(stream));
}

extern "C" EMA_API int ssd_bwd_launch(const SsdBwdArgs* a, void* stream) {
  using namespace emab::ssd;
  if (a == nullptr) return fail(EMA_ERR_INVALID_ARGUMENT, "ssd_bwd: args is NULL");
  int r = check_common(a->batch, a->seqlen, a->nheads, a->headdim, a->dstate, a->ngroups, a->dtype, a->x,
                       a->x_stride, a->B, a->B_stride, a->C, a->C_stride, a->dt, a->A);
  if (r) return r;
  if (a->dout == nullptr || a->dx == nullptr || a->chunk_states == nullptr || a->ddt == nullptr ||
      a->dA == nullptr || a->dB == nullptr || a->dC == nullptr)
    return fail(EMA_ERR_INVALID_ARGUMENT, "ssd_bwd: dout, chunk_states, dx, ddt, dA, dB and dC are required");
  if (a->D != nullptr && a->dD == nullptr) return fail(EMA_ERR_INVALID_ARGUMENT, "ssd_bwd: dD is required with D");
  if (!aligned16(a->dout) || !aligned16(a->dx) || (reinterpret_cast<uintptr_t>(a->dB) & 7u) ||
      (reinterpret_cast<uintptr_t>(a->dC) & 7u) || (reinterpret_cast<uintptr_t>(a->chunk_states) & 7u))
    return fail(EMA_ERR_INVALID_ARGUMENT, "ssd_bwd: misaligned dout / dx / dB / dC / chunk_states");
  for (int i = 0; i < 3; ++i)
    if (a->dout_stride[i] % 8 != 0 || a->dx_stride[i] % 2 != 0)
      return fail(EMA_ERR_INVALID_ARGUMENT, "ssd_bwd: dout strides must be multiples of 8, dx strides even");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t bl = static_cast<size_t>(a->batch) * a->seqlen;
  cudaError_t e = cudaMemsetAsync(a->dA, 0, a->nheads * sizeof(float), s);
  if (e == cudaSuccess) e = cudaMemsetAsync(a->dB, 0, bl * a->ngroups * N * sizeof(float), s);
  if (e == cudaSuccess) e = cudaMemsetAsync(a->dC, 0, bl * a->ngroups * N * sizeof(float), s);
  if (e == cudaSuccess && a->dD != nullptr) e = cudaMemsetAsync(a->dD, 0, a->nheads * sizeof(float), s);
  if (e == cudaSuccess && a->ddt_bias != nullptr) e = cudaMemsetAsync(a->ddt_bias, 0, a->nheads * sizeof(float), s);
  if (e != cudaSuccess) return fail(EMA_ERR_CUDA, "ssd_bwd: %s", cudaGetErrorString(e));
  if (a->batch == 0 || a->seqlen == 0) return EMA_OK;
  // the tensor-core kernel, wherever its TMA and vector-store alignment holds
  r = emab::ssd_bwd_tc_launch(a, s);
  if (r != EMA_ERR_UNSUPPORTED) return r;
  Params p{};
  p.B = static_cast<int>(a->batch);
  p.L = static_cast<int>(a->seqlen);
  p.H = static_cast<int>(a->nheads);
  p.G = static_cast<int>(a->ngroups);
  p.nc = static_cast<int>(ssd_internal_chunks(a->seqlen));
  p.x = static_cast<const bf16*>(a->x);
  p.sx_b = a->x_stride[0];
  p.sx_l = a->x_stride[1];
  p.sx_h = a->x_stride[2];
  p.dt = a->dt;
  p.A = a->A;
  p.Bm = static_cast<const bf16*>(a->B);
  p.sb_b = a->B_stride[0];
  p.sb_l = a->B_stride[1];
  p.sb_g = a->B_stride[2];
  p.Cm = static_cast<const bf16*>(a->C);
  p.sc_b = a->C_stride[0];
  p.sc_l = a->C_stride[1];
  p.sc_g = a->C_stride[2];
  p.D = a->D;
  p.chunk_states = const_cast<float*>(a->chunk_states);
  p.dy = static_cast<const bf16*>(a->dout);
  p.sdy_b = a->dout_stride[0];
  p.sdy_l = a->dout_stride[1];
  p.sdy_h = a->dout_stride[2];
  p.ds_final = a->d_final_state;
  p.dx = static_cast<bf16*>(a->dx);
  p.sdx_b = a->dx_stride[0];
  p.sdx_l = a->dx_stride[1];
  p.sdx_h = a->dx_stride[2];
  p.ddt = a->ddt;
  p.dA = a->dA;
  p.dB = a->dB;
  p.dC = a->dC;
  p.dD = a->dD;
  p.ds0 = a->d_initial_state;
  p.dtm = emab::dt_map_of(a);
  p.ddt_bias = a->ddt_bias;
  static unsigned long long attr_mask = 0;
  r = emab::ensure_smem_attr(reinterpret_cast<const void*>(ssd_bwd_kernel), static_cast<int>(sizeof(BwdSmem)),
                             &attr_mask);
  if (r) return fail(EMA_ERR_CUDA, "ssd_bwd: %s", cudaGetErrorString(static_cast<cudaError_t>(r)));
  ssd_bwd_kernel<<<dim3(p.H, p.B), NTHR, sizeof(BwdSmem), s>>>(p);
  return launch_check("ssd_bwd");
}
