// EMA chunked scan, forward and backward, as single-pass decoupled look-back
// kernels for sm_100a.
//
// Work unit ("tile"): one chunk of Q tokens x one (batch, head) -- a [Q, P]
// slab of x, fetched with one TMA box {P, 1, Q, 1} of the (B, L, H, P) tensor.
// CTAs take tiles from a ticket counter in chunk-major order (forward: chunk
// 0 first; backward: last chunk first), so every tile a CTA waits on belongs
// to a CTA that already started: the look-back cannot deadlock.
//
// Inside a tile, warp w owns the token segment [w*SEG, (w+1)*SEG) and lane l
// owns channels [l*CPT, (l+1)*CPT).  Each thread runs the recurrence
// sequentially over its segment (one FMA per element), segments are chained
// in shared memory, tiles are chained through global memory:
//
//   forward  z_t = a_t z_{t-1} + w_t x_t          (reference form: w = 1)
//   backward G_t = dy_t + a_{t+1} G_{t+1},  dx = w G,
//            dl_t = sum_p G_t a_t z_{t-1}   (gradient of the natural-log decay)
//
// HBM traffic is the algorithmic minimum: the forward reads x and the decay
// once and writes y once; the backward reads x, dy and the decay once and
// writes dx and the per-token decay gradient once.  The only extra traffic is
// the per-chunk start states (P floats per tile) and the look-back slots.
#pragma once

#include "ema_common.cuh"

namespace emab {

enum FwdMode : int { kFwdLog2 = 0, kFwdDt = 1 };
enum BwdMode : int { kBwdCumsum = 0, kBwdDt = 1 };

template <int BP, int Q>
struct ScanGeo {
  static constexpr int CPT = BP / 32;              // channels per lane
  static constexpr int SEG = (BP <= 64) ? 32 : 16;  // tokens per warp segment
  static constexpr int NW = Q / SEG;                // warps per CTA
  static constexpr int NT = NW * 32;                // threads per CTA
  static constexpr int RB = 8;                      // backward recompute block
  // Backward CTAs hold two [Q, BP] tiles; aim for >= 768 resident threads per
  // SM so several tiles stream at once (caps registers at ~85 per thread).
  static constexpr int BWD_MIN_BLOCKS = (768 / NT) > 0 ? (768 / NT) : 1;
  static_assert(BP % 32 == 0 && BP <= 128, "block headdim");
  static_assert(Q % SEG == 0 && NT >= Q && NT >= BP, "geometry");
};

struct ScanWorkspace {
  uint32_t* hdr;    // kHdrWords header words
  float* partial;   // [tiles] per-tile dA partial sums (dt-form backward)
  uint32_t* flags;  // [tiles] look-back flags: (epoch << 2) | {0, AGG, INCL}
  float* decay;     // [tiles] tile aggregate decay
  float* vals;      // [tiles][2][BP] aggregate / inclusive vectors
};

struct FwdParams {
  int B, L, H, P, nc;
  const float* dA;  // (B,H,L)
  const float* dt;  // (B,L,H)
  const float* A;   // (H,)
  const void* seq_idx;
  int seq_idx_type;
  const float* init;  // (B,H,P)
  float* states;
  long long st_b, st_c, st_h, st_p;
  float* da_cs;      // (B,H,L)
  float* da_cs_sum;  // (B,H,nc)
  float* final_state;
  ScanWorkspace ws;
};

struct BwdParams {
  int B, L, H, P, nc;
  const float* da_cs;      // (B,H,L)
  const float* da_cs_sum;  // (B,H,nc) (unused by the kernel; chunk decay is the token product)
  const float* dt;         // (B,L,H)
  const float* A;          // (H,)
  const float* states;
  long long st_b, st_c, st_h, st_p;
  const float* d_final;  // (B,H,P)
  const float* d_last;   // (B,H,P)
  float* dl;             // (B,H,L)
  float* ddt;            // (B,L,H)
  float* dA_out;         // (H,)
  float* d_init;         // (B,H,P)
  ScanWorkspace ws;
};

__device__ __forceinline__ long long load_seq_id(const void* base, int type, size_t i) {
  switch (type) {
    case 1: return static_cast<const int8_t*>(base)[i];
    case 2: return static_cast<const int32_t*>(base)[i];
    default: return static_cast<const long long*>(base)[i];
  }
}

// Walk the chain from tile `c` in direction `step` (-1: towards chunk 0,
// +1: towards the last chunk), combining published aggregates until an
// inclusive prefix (or the chain end) is found.  Executed by one full warp;
// lane l returns channels [l*CPT, (l+1)*CPT) of the incoming vector in `run`
// and the accumulated decay in `rdec`.  Returns true when the chain end was
// reached (the caller then adds rdec * boundary value).  Waits are bounded.
template <int BP>
__device__ __forceinline__ bool lookback_warp(const ScanWorkspace& ws, uint32_t epoch, int bh, int BH,
                                              int c, int step, int nc, int lane,
                                              float (&run)[BP / 32], float& rdec) {
  constexpr int CPT = BP / 32;
#pragma unroll
  for (int k = 0; k < CPT; ++k) run[k] = 0.f;
  rdec = 1.f;
  const unsigned FULL = 0xffffffffu;
  for (int j = c + step; j >= 0 && j < nc; j += step) {
    const size_t slot = static_cast<size_t>(j) * BH + bh;
    uint32_t st = 0;
    bool timed_out = false;
    unsigned long long t_start = 0;
    for (int it = 0;; ++it) {
      const uint32_t f = ld_acquire_gpu(&ws.flags[slot]);
      st = ((f >> 2) == epoch) ? (f & 3u) : 0u;
      if (__all_sync(FULL, st != 0u)) break;
      if (it == 0) t_start = global_timer_ns();
      // the give-up decision is warp-uniform so every lane leaves together
      if (__any_sync(FULL, global_timer_ns() - t_start > kWaitLimitNs)) {
        timed_out = true;
        break;
      }
      __nanosleep(40);
    }
    if (timed_out) {
      if (lane == 0) atomicOr(&ws.hdr[kHdrStatus], kStatusLookbackTimeout);
      return false;  // leave run as accumulated so far; result is flagged invalid
    }
    // Every lane acquired at least the aggregate; use the inclusive prefix only
    // when every lane acquired it (each lane reads only what it acquired).
    const bool incl = __all_sync(FULL, st == kFlagIncl);
    const float* v = ws.vals + slot * (2 * BP) + (incl ? BP : 0) + lane * CPT;
#pragma unroll
    for (int k = 0; k < CPT; ++k) run[k] = fmaf(rdec, ld_relaxed_gpu(v + k), run[k]);
    if (incl) return false;
    rdec *= ld_relaxed_gpu(&ws.decay[slot]);
  }
  return true;
}

// Publish a vector (BP floats from smem) + optional decay into the tile's
// slot, then raise the flag.  Called by all threads of the CTA.
template <int BP>
__device__ __forceinline__ void publish_cta(const ScanWorkspace& ws, size_t slot, int which,
                                            const float* s_vec, float dec, uint32_t flag, int tid) {
  if (tid < BP) {
    ws.vals[slot * (2 * BP) + which * BP + tid] = s_vec[tid];
    if (tid == 0 && which == 0) ws.decay[slot] = dec;
    __threadfence();
  }
  __syncthreads();
  if (tid == 0) st_release_gpu(&ws.flags[slot], flag);
}

// Last-CTA bookkeeping: count this CTA as finished; the final one resets the
// ticket/done counters and advances the epoch for the next launch.  Returns
// true in the last CTA (all threads), after a block barrier.
__device__ __forceinline__ bool finish_cta(const ScanWorkspace& ws, uint32_t epoch, int tid,
                                           uint32_t* s_flag) {
  if (tid == 0) {
    __threadfence();
    const uint32_t prev = atomicAdd(&ws.hdr[kHdrDone], 1u);
    *s_flag = (prev == gridDim.x - 1) ? 1u : 0u;
  }
  __syncthreads();
  return *s_flag != 0u;
}
__device__ __forceinline__ void reset_counters(const ScanWorkspace& ws, uint32_t epoch) {
  __threadfence();
  ws.hdr[kHdrTicket] = 0u;
  ws.hdr[kHdrDone] = 0u;
  __threadfence();
  ws.hdr[kHdrEpoch] = (epoch + 1u) & kEpochMask;
}

// Sum of v[j] over the 32 lanes, transposed: after the call lane l holds the
// total of index j = (l >> 2) & 7 (lanes 4j..4j+3 agree).  9 shuffles for 8 values.
__device__ __forceinline__ float transpose_reduce8(float (&v)[8], int lane) {
  const unsigned FULL = 0xffffffffu;
  {
    const bool up = lane & 16;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float send = up ? v[k] : v[k + 4];
      const float keep = up ? v[k + 4] : v[k];
      v[k] = keep + __shfl_xor_sync(FULL, send, 16);
    }
  }
  {
    const bool up = lane & 8;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const float send = up ? v[k] : v[k + 2];
      const float keep = up ? v[k + 2] : v[k];
      v[k] = keep + __shfl_xor_sync(FULL, send, 8);
    }
  }
  {
    const bool up = lane & 4;
    const float send = up ? v[0] : v[1];
    const float keep = up ? v[1] : v[0];
    v[0] = keep + __shfl_xor_sync(FULL, send, 4);
  }
  float r = v[0];
  r += __shfl_xor_sync(FULL, r, 2);
  r += __shfl_xor_sync(FULL, r, 1);
  return r;
}

// ---------------------------------------------------------------------------
// Forward
// ---------------------------------------------------------------------------
template <typename T, int BP, int Q>
struct FwdSmem {
  using G = ScanGeo<BP, Q>;
  static constexpr int kX = 0;
  static constexpr int kXBytes = Q * BP * static_cast<int>(sizeof(T));
  static constexpr int kA = kXBytes;                 // float[Q]
  static constexpr int kW = kA + Q * 4;              // float[Q]
  static constexpr int kL2 = kW + Q * 4;             // float[Q]
  static constexpr int kE = kL2 + Q * 4;             // float[NW][BP]
  static constexpr int kD = kE + G::NW * BP * 4;     // float[NW]
  static constexpr int kG0 = kD + G::NW * 4;         // float[NW]
  static constexpr int kSin = kG0 + G::NW * 4;       // float[BP]
  static constexpr int kEt = kSin + BP * 4;          // float[BP]
  static constexpr int kMisc = kEt + BP * 4;         // float[32]
  static constexpr int kBar = (kMisc + 32 * 4 + 15) / 16 * 16;  // uint64
  static constexpr int kBytes = kBar + 16;
};

template <typename T, int BP, int Q, int MODE, bool SEQ>
__global__ void __launch_bounds__(ScanGeo<BP, Q>::NT)
    ema_fwd_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_y,
                   const FwdParams p) {
  using G = ScanGeo<BP, Q>;
  using S = FwdSmem<T, BP, Q>;
  constexpr int CPT = G::CPT, SEG = G::SEG, NW = G::NW;
  extern __shared__ __align__(128) unsigned char smem[];
  T* s_x = reinterpret_cast<T*>(smem + S::kX);
  float* s_a = reinterpret_cast<float*>(smem + S::kA);
  float* s_w = reinterpret_cast<float*>(smem + S::kW);
  float* s_l2 = reinterpret_cast<float*>(smem + S::kL2);
  float* s_E = reinterpret_cast<float*>(smem + S::kE);
  float* s_D = reinterpret_cast<float*>(smem + S::kD);
  float* s_G0 = reinterpret_cast<float*>(smem + S::kG0);
  float* s_Sin = reinterpret_cast<float*>(smem + S::kSin);
  float* s_Et = reinterpret_cast<float*>(smem + S::kEt);
  float* s_misc = reinterpret_cast<float*>(smem + S::kMisc);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + S::kBar);
  __shared__ uint32_t s_tile, s_epoch, s_last;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const ScanWorkspace& ws = p.ws;
  if (tid == 0) {
    tma_prefetch_desc(&tm_x);
    s_tile = atomicAdd(&ws.hdr[kHdrTicket], 1u);
    s_epoch = ld_volatile_u32(&ws.hdr[kHdrEpoch]) & kEpochMask;
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (s_tile >= gridDim.x) {  // counters not reset: workspace shared by overlapping launches
    if (tid == 0) atomicOr(&ws.hdr[kHdrStatus], kStatusBadTicket);
    return;
  }
  const uint32_t epoch = s_epoch;
  const int BH = p.B * p.H;
  const int c = static_cast<int>(s_tile) / BH;
  const int bh = static_cast<int>(s_tile) % BH;
  const int b = bh / p.H, h = bh % p.H;
  const int t0 = c * Q;
  const size_t slot = static_cast<size_t>(c) * BH + bh;
  if (tid == 0) {
    mbar_arrive_expect_tx(bar, S::kXBytes);
    tma_load_4d(s_x, &tm_x, bar, 0, h, t0, b);
  }

  // ---- per-token decay a_t and input weight w_t -------------------------
  if (tid < Q) {
    const int t = t0 + tid;
    float a = 1.f, w = 0.f, l2 = 0.f;
    if (t < p.L) {
      if (MODE == kFwdLog2) {
        l2 = p.dA[(static_cast<size_t>(b) * p.H + h) * p.L + t];
        w = 1.f;
      } else {
        const float d = p.dt[(static_cast<size_t>(b) * p.L + t) * p.H + h];
        l2 = d * p.A[h] * kLog2e;
        w = d;
      }
      a = exp2f(l2);
      if (SEQ && t > 0) {
        const size_t i = static_cast<size_t>(b) * p.L + t;
        if (load_seq_id(p.seq_idx, p.seq_idx_type, i) != load_seq_id(p.seq_idx, p.seq_idx_type, i - 1))
          a = 0.f;
      }
    }
    s_a[tid] = a;
    s_w[tid] = w;
    s_l2[tid] = l2;
  }
  // within-chunk cumsum of the log2 decay (reference outputs da_cs / da_cs_sum)
  if (MODE == kFwdLog2 && (p.da_cs != nullptr || p.da_cs_sum != nullptr)) {
    float v = (tid < Q) ? s_l2[tid] : 0.f;
    // (s_l2 written by this same thread above)
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float n = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += n;
    }
    if (lane == 31) s_misc[warp] = v;
    __syncthreads();
    float pre = 0.f;
    for (int k = 0; k < warp; ++k) pre += s_misc[k];
    v += pre;
    if (tid < Q && t0 + tid < p.L && p.da_cs != nullptr)
      p.da_cs[(static_cast<size_t>(b) * p.H + h) * p.L + t0 + tid] = v;
    if (tid == Q - 1 && p.da_cs_sum != nullptr)
      p.da_cs_sum[(static_cast<size_t>(b) * p.H + h) * p.nc + c] = v;
  }
  __syncthreads();

  mbar_wait_bounded(bar, 0, &ws.hdr[kHdrStatus]);

  // ---- pass 1: per-segment end state from zero input, and segment decay ----
  const int s0 = warp * SEG;
  const int ch = lane * CPT;
  {
    float z[CPT];
#pragma unroll
    for (int k = 0; k < CPT; ++k) z[k] = 0.f;
    float D = 1.f;
#pragma unroll
    for (int i = 0; i < SEG; ++i) {
      const float a = s_a[s0 + i], w = s_w[s0 + i];
      float xv[CPT];
      load_pack<T, CPT>(s_x + (s0 + i) * BP + ch, xv);
#pragma unroll
      for (int k = 0; k < CPT; ++k) z[k] = fmaf(a, z[k], w * xv[k]);
      D *= a;
    }
#pragma unroll
    for (int k = 0; k < CPT; ++k) s_E[warp * BP + ch + k] = z[k];
    if (lane == 0) s_D[warp] = D;
  }
  __syncthreads();

  // ---- chain the segments of this tile --------------------------------------
  if (tid < BP) {
    float Sv = 0.f, Gd = 1.f;
#pragma unroll
    for (int s = 0; s < NW; ++s) {
      const float e = s_E[s * BP + tid];
      s_E[s * BP + tid] = Sv;  // state before segment s (zero tile input)
      if (tid == 0) s_G0[s] = Gd;
      Sv = fmaf(s_D[s], Sv, e);
      Gd *= s_D[s];
    }
    s_Et[tid] = Sv;
    if (tid == 0) s_misc[0] = Gd;
  }
  __syncthreads();
  const float Dtile = s_misc[0];
  const bool has_succ = (c + 1 < p.nc);
  if (c > 0 && has_succ) publish_cta<BP>(ws, slot, 0, s_Et, Dtile, (epoch << 2) | kFlagAgg, tid);

  // ---- look-back for the state entering this tile ---------------------------
  if (warp == 0) {
    float run[CPT], rdec = 1.f;
    bool at_start = true;
    if (c > 0) {
      at_start = lookback_warp<BP>(ws, epoch, bh, BH, c, -1, p.nc, lane, run, rdec);
    } else {
#pragma unroll
      for (int k = 0; k < CPT; ++k) run[k] = 0.f;
    }
    if (at_start && p.init != nullptr) {
      const float* iv = p.init + (static_cast<size_t>(b) * p.H + h) * p.P;
#pragma unroll
      for (int k = 0; k < CPT; ++k)
        if (ch + k < p.P) run[k] = fmaf(rdec, iv[ch + k], run[k]);
    }
#pragma unroll
    for (int k = 0; k < CPT; ++k) {
      s_Sin[ch + k] = run[k];
      run[k] = fmaf(Dtile, run[k], s_Et[ch + k]);  // inclusive (state at the tile end)
    }
    if (has_succ) {
#pragma unroll
      for (int k = 0; k < CPT; ++k) ws.vals[slot * (2 * BP) + BP + ch + k] = run[k];
      __threadfence();
      __syncwarp();
      if (lane == 0) st_release_gpu(&ws.flags[slot], (epoch << 2) | kFlagIncl);
    } else if (p.final_state != nullptr) {
      float* fo = p.final_state + (static_cast<size_t>(b) * p.H + h) * p.P;
#pragma unroll
      for (int k = 0; k < CPT; ++k)
        if (ch + k < p.P) fo[ch + k] = run[k];
    }
  }
  __syncthreads();

  if (p.states != nullptr && tid < p.P)
    p.states[b * p.st_b + static_cast<long long>(c) * p.st_c + h * p.st_h + tid * p.st_p] = s_Sin[tid];

  // ---- pass 2: exact outputs, written over the x tile -----------------------
  {
    const float g0 = s_G0[warp];
    float z[CPT];
#pragma unroll
    for (int k = 0; k < CPT; ++k) z[k] = fmaf(g0, s_Sin[ch + k], s_E[warp * BP + ch + k]);
#pragma unroll
    for (int i = 0; i < SEG; ++i) {
      const float a = s_a[s0 + i], w = s_w[s0 + i];
      T* px = s_x + (s0 + i) * BP + ch;
      float xv[CPT];
      load_pack<T, CPT>(px, xv);
#pragma unroll
      for (int k = 0; k < CPT; ++k) z[k] = fmaf(a, z[k], w * xv[k]);
      store_pack<T, CPT>(px, z);
    }
  }
  fence_proxy_async_smem();
  __syncthreads();
  if (tid == 0) {
    tma_store_4d(&tm_y, s_x, 0, h, t0, b);
    bulk_commit();
    bulk_wait_read_all();
  }
  if (finish_cta(ws, epoch, tid, &s_last) && tid == 0) reset_counters(ws, epoch);
}

// ---------------------------------------------------------------------------
// Backward
// ---------------------------------------------------------------------------
template <typename T, int BP, int Q>
struct BwdSmem {
  using G = ScanGeo<BP, Q>;
  static constexpr int kXBytes = Q * BP * static_cast<int>(sizeof(T));
  static constexpr int kX = 0;
  static constexpr int kDy = kXBytes;
  static constexpr int kA = 2 * kXBytes;          // float[Q]
  static constexpr int kW = kA + Q * 4;           // float[Q]
  static constexpr int kE = kW + Q * 4;           // float[NW][BP]  forward prefix -> Zin
  static constexpr int kR = kE + G::NW * BP * 4;  // float[NW][BP]  reverse aggregate -> Rloc
  static constexpr int kD = kR + G::NW * BP * 4;  // float[NW]
  static constexpr int kHs = kD + G::NW * 4;      // float[NW]
  static constexpr int kSin = kHs + G::NW * 4;    // float[BP]
  static constexpr int kGn = kSin + BP * 4;       // float[BP]
  static constexpr int kRt = kGn + BP * 4;        // float[BP]
  static constexpr int kMisc = kRt + BP * 4;      // float[32]
  static constexpr int kCk = kMisc + 32 * 4;      // float[NW][SEG/RB][BP] recompute checkpoints
  static constexpr int kBar = (kCk + G::NW * (G::SEG / G::RB) * BP * 4 + 15) / 16 * 16;
  static constexpr int kBytes = kBar + 16;
};

template <typename T, int BP, int Q, int MODE>
__global__ void __launch_bounds__(ScanGeo<BP, Q>::NT, ScanGeo<BP, Q>::BWD_MIN_BLOCKS)
    ema_bwd_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_dy,
                   const __grid_constant__ CUtensorMap tm_dx, const BwdParams p) {
  using G = ScanGeo<BP, Q>;
  using S = BwdSmem<T, BP, Q>;
  constexpr int CPT = G::CPT, SEG = G::SEG, NW = G::NW, RB = G::RB, NB = SEG / RB;
  static_assert(SEG % RB == 0, "recompute block");
  extern __shared__ __align__(128) unsigned char smem[];
  T* s_x = reinterpret_cast<T*>(smem + S::kX);
  T* s_dy = reinterpret_cast<T*>(smem + S::kDy);
  float* s_a = reinterpret_cast<float*>(smem + S::kA);
  float* s_w = reinterpret_cast<float*>(smem + S::kW);
  float* s_E = reinterpret_cast<float*>(smem + S::kE);
  float* s_R = reinterpret_cast<float*>(smem + S::kR);
  float* s_D = reinterpret_cast<float*>(smem + S::kD);
  float* s_Hs = reinterpret_cast<float*>(smem + S::kHs);
  float* s_Sin = reinterpret_cast<float*>(smem + S::kSin);
  float* s_Gn = reinterpret_cast<float*>(smem + S::kGn);
  float* s_Rt = reinterpret_cast<float*>(smem + S::kRt);
  float* s_misc = reinterpret_cast<float*>(smem + S::kMisc);
  float* s_ck = reinterpret_cast<float*>(smem + S::kCk);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + S::kBar);
  __shared__ uint32_t s_tile, s_epoch, s_last;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const ScanWorkspace& ws = p.ws;
  if (tid == 0) {
    tma_prefetch_desc(&tm_x);
    tma_prefetch_desc(&tm_dy);
    s_tile = atomicAdd(&ws.hdr[kHdrTicket], 1u);
    s_epoch = ld_volatile_u32(&ws.hdr[kHdrEpoch]) & kEpochMask;
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (s_tile >= gridDim.x) {  // counters not reset: workspace shared by overlapping launches
    if (tid == 0) atomicOr(&ws.hdr[kHdrStatus], kStatusBadTicket);
    return;
  }
  const uint32_t epoch = s_epoch;
  const int BH = p.B * p.H;
  const int c = p.nc - 1 - static_cast<int>(s_tile) / BH;
  const int bh = static_cast<int>(s_tile) % BH;
  const int b = bh / p.H, h = bh % p.H;
  const int t0 = c * Q;
  const size_t slot = static_cast<size_t>(c) * BH + bh;
  if (tid == 0) {
    mbar_arrive_expect_tx(bar, 2 * S::kXBytes);
    tma_load_4d(s_x, &tm_x, bar, 0, h, t0, b);
    tma_load_4d(s_dy, &tm_dy, bar, 0, h, t0, b);
  }

  // ---- per-token decay / weight; chunk start state ---------------------------
  float Ah = 0.f;
  if (MODE == kBwdDt) Ah = p.A[h];
  if (tid < Q) {
    const int t = t0 + tid;
    float a = 1.f, w = 0.f;
    if (t < p.L) {
      if (MODE == kBwdCumsum) {
        const float* cs = p.da_cs + (static_cast<size_t>(b) * p.H + h) * p.L;
        const float prev = (tid == 0) ? 0.f : cs[t - 1];
        a = exp2f(cs[t] - prev);
        w = 1.f;
      } else {
        const float d = p.dt[(static_cast<size_t>(b) * p.L + t) * p.H + h];
        a = exp2f(d * Ah * kLog2e);
        w = d;
      }
    }
    s_a[tid] = a;
    s_w[tid] = w;
  }
  if (tid < BP) {
    s_Sin[tid] = (tid < p.P) ? p.states[b * p.st_b + static_cast<long long>(c) * p.st_c + h * p.st_h +
                                        tid * p.st_p]
                             : 0.f;
  }
  __syncthreads();
  mbar_wait_bounded(bar, 0, &ws.hdr[kHdrStatus]);

  const int s0 = warp * SEG;
  const int ch = lane * CPT;
  // ---- pass 1: forward end state (zero input) and reverse aggregate ---------
  {
    float z[CPT], g[CPT];
#pragma unroll
    for (int k = 0; k < CPT; ++k) z[k] = g[k] = 0.f;
    float D = 1.f;
#pragma unroll
    for (int i = 0; i < SEG; ++i) {
      const float a = s_a[s0 + i], w = s_w[s0 + i];
      float xv[CPT];
      load_pack<T, CPT>(s_x + (s0 + i) * BP + ch, xv);
#pragma unroll
      for (int k = 0; k < CPT; ++k) z[k] = fmaf(a, z[k], w * xv[k]);
      D *= a;
      const int r = SEG - 1 - i;
      const float ar = s_a[s0 + r];
      float dv[CPT];
      load_pack<T, CPT>(s_dy + (s0 + r) * BP + ch, dv);
#pragma unroll
      for (int k = 0; k < CPT; ++k) g[k] = ar * (dv[k] + g[k]);
    }
#pragma unroll
    for (int k = 0; k < CPT; ++k) {
      s_E[warp * BP + ch + k] = z[k];
      s_R[warp * BP + ch + k] = g[k];
    }
    if (lane == 0) s_D[warp] = D;
  }
  __syncthreads();

  // ---- chain segments: Zin (forward) and Rloc (reverse) ---------------------
  if (tid < BP) {
    float Sv = s_Sin[tid];
#pragma unroll
    for (int s = 0; s < NW; ++s) {
      const float e = s_E[s * BP + tid];
      s_E[s * BP + tid] = Sv;  // true state before segment s
      Sv = fmaf(s_D[s], Sv, e);
    }
    float r = 0.f, Hd = 1.f;
#pragma unroll
    for (int s = NW - 1; s >= 0; --s) {
      const float rr = s_R[s * BP + tid];
      s_R[s * BP + tid] = r;  // gradient w.r.t. z at segment end, from later segments of this tile
      if (tid == 0) s_Hs[s] = Hd;
      r = fmaf(s_D[s], r, rr);
      Hd *= s_D[s];
    }
    s_Rt[tid] = r;  // gradient w.r.t. the state entering the tile, from this tile's dy
    if (tid == 0) s_misc[0] = Hd;
  }
  __syncthreads();
  const float Dtile = s_misc[0];
  const bool has_succ = (c > 0);  // the reverse chain continues towards chunk 0
  if (c + 1 < p.nc && has_succ) publish_cta<BP>(ws, slot, 0, s_Rt, Dtile, (epoch << 2) | kFlagAgg, tid);

  // ---- look-back: gradient arriving at the tile end from later chunks -------
  if (warp == 0) {
    float run[CPT], rdec = 1.f;
    bool at_end = true;
    if (c + 1 < p.nc) {
      at_end = lookback_warp<BP>(ws, epoch, bh, BH, c, +1, p.nc, lane, run, rdec);
    } else {
#pragma unroll
      for (int k = 0; k < CPT; ++k) run[k] = 0.f;
    }
    if (at_end && p.d_final != nullptr) {
      const float* dv = p.d_final + (static_cast<size_t>(b) * p.H + h) * p.P;
#pragma unroll
      for (int k = 0; k < CPT; ++k)
        if (ch + k < p.P) run[k] = fmaf(rdec, dv[ch + k], run[k]);
    }
#pragma unroll
    for (int k = 0; k < CPT; ++k) {
      s_Gn[ch + k] = run[k];
      run[k] = fmaf(Dtile, run[k], s_Rt[ch + k]);  // gradient w.r.t. the state before the tile
    }
    if (has_succ) {
#pragma unroll
      for (int k = 0; k < CPT; ++k) ws.vals[slot * (2 * BP) + BP + ch + k] = run[k];
      __threadfence();
      __syncwarp();
      if (lane == 0) st_release_gpu(&ws.flags[slot], (epoch << 2) | kFlagIncl);
    } else if (p.d_init != nullptr) {
      float* di = p.d_init + (static_cast<size_t>(b) * p.H + h) * p.P;
#pragma unroll
      for (int k = 0; k < CPT; ++k)
        if (ch + k < p.P) di[ch + k] = run[k];
    }
  }
  __syncthreads();

  // ---- pass 2: exact gradients -----------------------------------------------
  float dap = 0.f;  // dt-form: sum_t dt_t * dl_t over this lane's tokens
  {
    float g[CPT];
    const float hs = s_Hs[warp];
#pragma unroll
    for (int k = 0; k < CPT; ++k) g[k] = fmaf(hs, s_Gn[ch + k], s_R[warp * BP + ch + k]);
    // forward recompute of the segment; the state entering every RB-token
    // block is kept (per thread) in shared memory for the reverse sweep
    float* ck = s_ck + warp * NB * BP + ch;
    {
      float z[CPT];
#pragma unroll
      for (int k = 0; k < CPT; ++k) z[k] = s_E[warp * BP + ch + k];
#pragma unroll
      for (int i = 0; i < SEG; ++i) {
        if (i % RB == 0) {
#pragma unroll
          for (int k = 0; k < CPT; ++k) ck[(i / RB) * BP + k] = z[k];
        }
        const float a = s_a[s0 + i], w = s_w[s0 + i];
        float xv[CPT];
        load_pack<T, CPT>(s_x + (s0 + i) * BP + ch, xv);
#pragma unroll
        for (int k = 0; k < CPT; ++k) z[k] = fmaf(a, z[k], w * xv[k]);
      }
    }
    const bool last_tile = (t0 + Q >= p.L);
    const float* dlast = (p.d_last != nullptr && last_tile)
                             ? p.d_last + (static_cast<size_t>(b) * p.H + h) * p.P
                             : nullptr;
#pragma unroll 1
    for (int blk = NB - 1; blk >= 0; --blk) {
      float zz[RB][CPT];
      {
        float z[CPT];
#pragma unroll
        for (int k = 0; k < CPT; ++k) z[k] = ck[blk * BP + k];
#pragma unroll
        for (int j = 0; j < RB; ++j) {
          const int t = s0 + blk * RB + j;
          const float a = s_a[t], w = s_w[t];
          float xv[CPT];
          load_pack<T, CPT>(s_x + t * BP + ch, xv);
#pragma unroll
          for (int k = 0; k < CPT; ++k) {
            zz[j][k] = z[k];
            z[k] = fmaf(a, z[k], w * xv[k]);
          }
        }
      }
      float p1[RB], p2[RB];
#pragma unroll
      for (int j = RB - 1; j >= 0; --j) {
        const int t = s0 + blk * RB + j;
        const float a = s_a[t], w = s_w[t];
        float dv[CPT];
        T* pd = s_dy + t * BP + ch;
        load_pack<T, CPT>(pd, dv);
        float Gv[CPT], dxv[CPT];
#pragma unroll
        for (int k = 0; k < CPT; ++k) {
          Gv[k] = dv[k] + g[k];
          dxv[k] = w * Gv[k];
        }
        if (dlast != nullptr && t0 + t == p.L - 1) {
#pragma unroll
          for (int k = 0; k < CPT; ++k)
            if (ch + k < p.P) dxv[k] += dlast[ch + k];
        }
        store_pack<T, CPT>(pd, dxv);
        float q1 = 0.f, q2 = 0.f;
        if (MODE == kBwdDt) {
          float xv[CPT];
          load_pack<T, CPT>(s_x + t * BP + ch, xv);
#pragma unroll
          for (int k = 0; k < CPT; ++k) q2 = fmaf(Gv[k], xv[k], q2);
        }
#pragma unroll
        for (int k = 0; k < CPT; ++k) {
          q1 = fmaf(Gv[k], zz[j][k], q1);
          g[k] = a * Gv[k];
        }
        p1[j] = a * q1;
        p2[j] = q2;
      }
      const float P1 = transpose_reduce8(p1, lane);
      float P2 = 0.f;
      if (MODE == kBwdDt) P2 = transpose_reduce8(p2, lane);
      if ((lane & 3) == 0) {
        const int t = s0 + blk * RB + (lane >> 2);
        const int gt = t0 + t;
        if (gt < p.L) {
          if (MODE == kBwdCumsum) {
            p.dl[(static_cast<size_t>(b) * p.H + h) * p.L + gt] = P1;
          } else {
            p.ddt[(static_cast<size_t>(b) * p.L + gt) * p.H + h] = fmaf(Ah, P1, P2);
            dap = fmaf(s_w[t], P1, dap);
          }
        }
      }
    }
  }

  // ---- dt-form: per-tile partial of dA (deterministic order) ----------------
  if (MODE == kBwdDt) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) dap += __shfl_xor_sync(0xffffffffu, dap, o);
    if (lane == 0) s_misc[1 + warp] = dap;
  }
  fence_proxy_async_smem();
  __syncthreads();
  if (tid == 0) {
    tma_store_4d(&tm_dx, s_dy, 0, h, t0, b);
    bulk_commit();
    if (MODE == kBwdDt) {
      float tot = 0.f;
      for (int w = 0; w < NW; ++w) tot += s_misc[1 + w];
      ws.partial[slot] = tot;
    }
    bulk_wait_read_all();
  }
  if (finish_cta(ws, epoch, tid, &s_last)) {
    if (MODE == kBwdDt) {
      __threadfence();
      for (int hh = tid; hh < p.H; hh += G::NT) {
        float acc = 0.f;
        for (int cc = 0; cc < p.nc; ++cc)
          for (int bb = 0; bb < p.B; ++bb)
            acc += ld_relaxed_gpu(&ws.partial[static_cast<size_t>(cc) * BH + bb * p.H + hh]);
        p.dA_out[hh] = acc;
      }
      __syncthreads();
    }
    if (tid == 0) reset_counters(ws, epoch);
  }
}

// ---------------------------------------------------------------------------
// Within-chunk cumsums (chunk_cumsum_triton)
// ---------------------------------------------------------------------------
// One CTA of NTH >= Q threads per (chunk, head, batch); thread i owns token i.
template <int NTH>
__global__ void __launch_bounds__(NTH)
    chunk_cumsum_kernel(const float* __restrict__ dA, long long sa_b, long long sa_h, long long sa_l,
                        float* __restrict__ cs, long long sc_b, long long sc_h, long long sc_l,
                        float* __restrict__ rev, long long sr_b, long long sr_h, long long sr_l, int L,
                        int Q, int exp2_out) {
  __shared__ float s_tot[2][NTH / 32];
  __shared__ float s_rev[NTH + 1];
  const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int t = c * Q + tid;
  const bool valid = (tid < Q) && (t < L);
  const float v = valid ? dA[b * sa_b + h * sa_h + static_cast<long long>(t) * sa_l] : 0.f;
  // inclusive forward scan and inclusive reverse scan over the chunk
  float f = v, r = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float n = __shfl_up_sync(0xffffffffu, f, o);
    if (lane >= o) f += n;
    const float m = __shfl_down_sync(0xffffffffu, r, o);
    if (lane + o < 32) r += m;
  }
  if (lane == 31) s_tot[0][warp] = f;
  if (lane == 0) s_tot[1][warp] = r;
  __syncthreads();
  for (int k = 0; k < warp; ++k) f += s_tot[0][k];
  for (int k = warp + 1; k < NTH / 32; ++k) r += s_tot[1][k];
  s_rev[tid] = r;
  if (tid == 0) s_rev[NTH] = 0.f;
  __syncthreads();
  if (!valid) return;
  // The exclusive reverse sum of token t is the inclusive reverse sum of token
  // t+1 of the same chunk; the chunk's last token gets 0 (1 after exp2).
  const bool last = (tid == Q - 1) || (t == L - 1);
  const float ex = last ? 0.f : s_rev[tid + 1];
  cs[b * sc_b + h * sc_h + static_cast<long long>(t) * sc_l] = exp2_out ? exp2f(f) : f;
  rev[b * sr_b + h * sr_h + static_cast<long long>(t) * sr_l] = exp2_out ? exp2f(ex) : ex;
}

}  // namespace emab
