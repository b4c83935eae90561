// EMA chunked scan, forward and backward, for sm_100a: persistent,
// warp-specialised, single-pass decoupled look-back kernels.
//
// Work unit ("tile"): one chunk of Q tokens x one (batch, head) -- a [Q, P]
// slab of x (and dy), fetched with one TMA box {BP, 1, Q, 1} of the
// (B, L, H, P) tensor.  Each CTA is persistent:
//
//   producer warp   takes tiles from a ticket counter (chunk-major: forward
//                   from chunk 0, backward from the last chunk) and streams
//                   them into an S-stage shared-memory ring -- TMA for the
//                   x / dy tiles, cp.async for the per-token decay row, the
//                   head's A and (backward) the chunk start state -- with one
//                   "full" mbarrier per stage;
//   look-back warp  follows the ring and fetches each tile's incoming state
//                   (forward) or arriving gradient (backward) from the tiles
//                   before it while the compute warps run the tile's first pass;
//   compute warps   scan the tile in the stage: warp w owns a token segment,
//                   lane l owns BP/32 channels; the recurrence runs
//                   sequentially per thread (one FMA per element), segments
//                   are chained in shared memory, tiles through global memory;
//                   outputs go straight from registers to global memory
//                   (coalesced 128-byte rows), so a stage is free as soon as
//                   the tile's second pass has read it.
//
// The tile's incoming state (forward) or outgoing gradient (backward) comes
// from a decoupled look-back over earlier tiles of the same (batch, head)
// chain.  Records are arrays of self-validating 64-bit words {value, tag},
// tag = launch generation + 1, so a reader that sees the tag sees the value:
// no flags, no fences, one round trip per hop.  Every wait is bounded.
//
//   forward  z_t = a_t z_{t-1} + w_t x_t          (reference form: w = 1)
//   backward G_t = dy_t + a_{t+1} G_{t+1},  dx = w G,
//            dl_t = sum_p G_t a_t z_{t-1}   (gradient of the natural-log decay)
//
// HBM traffic is the algorithmic minimum: the forward reads x and the decay
// once and writes y once; the backward reads x, dy and the decay once and
// writes dx and the per-token decay gradient once.
#pragma once

#include "ema_common.cuh"

namespace emab {

enum FwdMode : int { kFwdLog2 = 0, kFwdDt = 1 };
enum BwdMode : int { kBwdCumsum = 0, kBwdDt = 1 };

constexpr int kSmemPerSM = 233472;      // 228 KB of shared memory per SM
constexpr int kSmemPerCtaMax = 232448;  // 227 KB opt-in per CTA
constexpr int kCtaReserve = 1024;       // per-CTA system reservation
constexpr int kMaxStages = 8;

constexpr int align_up(int x, int a) { return (x + a - 1) / a * a; }

// Stage count and CTAs per SM for a ring of `stage`-byte stages plus `priv`
// bytes of per-CTA state: two CTAs per SM when each still gets >= 3 stages
// (one computing, two loading), else one CTA with as many stages as fit.
template <int STAGE, int PRIV>
struct Ring {
  static constexpr int S2 = ((kSmemPerSM / 2 - kCtaReserve) - PRIV) / STAGE;
  static constexpr int S1 = (kSmemPerCtaMax - PRIV) / STAGE;
  static constexpr bool TWO = S2 >= 3;
  static constexpr int S = TWO ? (S2 > kMaxStages ? kMaxStages : S2) : (S1 > kMaxStages ? kMaxStages : S1);
  static constexpr int CTAS = TWO ? 2 : 1;
  static constexpr bool OK = S >= 1;
};

// n / d for 0 <= n < 2^31 without a division: q = umulhi(n, m) >> sh with
// m = ceil(2^(31+l) / d), sh = l - 1, l = ceil(log2 d) (Granlund-Montgomery);
// m == 0 marks d == 1.  Built on the host by make_fast_div.
struct FastDiv {
  uint32_t m, sh;
};
__device__ __forceinline__ int fast_div(int n, FastDiv f) {
  return f.m ? static_cast<int>(__umulhi(static_cast<uint32_t>(n), f.m) >> f.sh) : n;
}
inline FastDiv make_fast_div(uint32_t d) {
  FastDiv f{0u, 0u};
  if (d >= 2) {
    uint32_t l = 0;
    while ((1ull << l) < d) ++l;
    f.sh = l - 1;
    f.m = static_cast<uint32_t>(((1ull << (31 + l)) + d - 1) / d);
  }
  return f;
}

struct ScanWorkspace {
  uint32_t* hdr;   // kHdrWords header words
  float* partial;  // [tiles] per-tile dA partial sums (dt-form backward)
  uint64_t* agg;   // [tiles][BP + 1] aggregate words (index BP: decay)
  uint64_t* incl;  // [tiles][BP] inclusive words
};

struct FwdParams {
  int B, L, H, P, nc;
  FastDiv div_bh, div_h;  // division by B*H and by H
  const float* rows;  // (B,H,L) per-token decay rows: log2 decay dA, or dt (transposed)
  const float* A;     // (H,)
  const void* seq_idx;
  int seq_idx_type;
  const float* init;  // (B,H,P)
  float* states;
  long long st_b, st_c, st_h, st_p;
  float* da_cs;      // (B,H,L)
  float* da_cs_sum;  // (B,H,nc)
  float* final_state;
  void* y;                      // (B,L,H,P) output
  long long sy_b, sy_l, sy_h;   // its element strides
  ScanWorkspace ws;
};

struct BwdParams {
  int B, L, H, P, nc;
  FastDiv div_bh, div_h;
  const float* rows;  // (B,H,L) per-token rows: within-chunk log2 cumsum da_cs, or dt (transposed)
  const float* A;     // (H,)
  const float* states;
  long long st_b, st_c, st_h, st_p;
  const float* d_final;  // (B,H,P)
  const float* d_last;   // (B,H,P)
  float* dl;             // (B,H,L) reference form
  float* ddt_rows;       // (B,H,L) dt form (transposed to (B,L,H) by the launcher)
  float* dA_out;         // (H,)
  float* d_init;         // (B,H,P)
  void* dx;                     // (B,L,H,P) output
  long long sdx_b, sdx_l, sdx_h;
  ScanWorkspace ws;
};

__device__ __forceinline__ long long load_seq_id(const void* base, int type, size_t i) {
  switch (type) {
    case 1: return static_cast<const int8_t*>(base)[i];
    case 2: return static_cast<const int32_t*>(base)[i];
    default: return static_cast<const long long*>(base)[i];
  }
}

// Walk the chain from tile `c` in direction `step` (-1: towards chunk 0, +1:
// towards the last chunk), combining published aggregates until an inclusive
// record (or the chain end).  One full warp; lane l returns channels
// [l*CPT, (l+1)*CPT) of the incoming vector in `run` and the accumulated
// decay in `rdec`.  Returns true when the chain end was reached (the caller
// adds rdec * boundary value).  A record is used only when every lane saw all
// of its words.  Waits are bounded.
template <int BP>
__device__ __forceinline__ bool lookback_warp(const ScanWorkspace& ws, uint32_t tag, int bh, int BH, int c,
                                              int step, int nc, int lane, float (&run)[BP / 32],
                                              float& rdec) {
  constexpr int CPT = BP / 32;
  const unsigned FULL = 0xffffffffu;
#pragma unroll
  for (int k = 0; k < CPT; ++k) run[k] = 0.f;
  rdec = 1.f;
  for (int j = c + step; j >= 0 && j < nc; j += step) {
    const size_t slot = static_cast<size_t>(j) * BH + bh;
    const uint64_t* inc = ws.incl + slot * BP;
    const uint64_t* agg = ws.agg + slot * (BP + 1);
    unsigned long long t_start = 0;
    uint32_t backoff = 32;
    for (int it = 0;; ++it) {
      // cheap probe: one word of each record, read by lane 0
      uint32_t seen = 0;
      if (lane == 0)
        seen = (word_tag(ld_relaxed_u64(inc)) == tag ? 2u : 0u) | (word_tag(ld_relaxed_u64(agg + BP)) == tag ? 1u : 0u);
      seen = __shfl_sync(FULL, seen, 0);
      if (seen != 0u) {
        // a record is (being) published: read and validate all of its words
        const uint64_t* src = (seen & 2u) ? inc : agg;
        uint64_t wv[CPT];
        bool ok = true;
#pragma unroll
        for (int k = 0; k < CPT; ++k) {
          wv[k] = ld_relaxed_u64(src + lane * CPT + k);
          ok &= word_tag(wv[k]) == tag;
        }
        if (__all_sync(FULL, ok)) {
#pragma unroll
          for (int k = 0; k < CPT; ++k) run[k] = fmaf(rdec, word_val(wv[k]), run[k]);
          if (seen & 2u) return false;
          rdec *= word_val(ld_relaxed_u64(agg + BP));
          break;
        }
        backoff = 32;  // words still landing: retry soon
      }
      if (it == 0) t_start = global_timer_ns();
      // the give-up decision is warp-uniform so every lane leaves together
      if (__any_sync(FULL, global_timer_ns() - t_start > kWaitLimitNs)) {
        if (lane == 0) atomicOr(&ws.hdr[kHdrStatus], kStatusLookbackTimeout);
        return false;
      }
      __nanosleep(backoff);
      backoff = backoff < 2048 ? backoff * 2 : 2048;
    }
  }
  return true;
}

// Transposed warp sum: v[j] summed over the 32 lanes lands in lanes 4j..4j+3.
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

// Completion bookkeeping, by consumer thread 0 after all of its CTA's stores:
// true in the last CTA of the launch.
__device__ __forceinline__ bool count_cta_done(const ScanWorkspace& ws) {
  __threadfence();
  const uint32_t prev = atomicAdd(&ws.hdr[kHdrDone], 1u);
  return prev == gridDim.x - 1;
}
// Every CTA's producer draws exactly one ticket past the last tile, so a
// launch that started from reset counters ends at total + gridDim.x; anything
// else means the workspace was shared by overlapping launches.
__device__ __forceinline__ void reset_counters(const ScanWorkspace& ws, uint32_t epoch, int total) {
  __threadfence();
  if (ld_volatile_u32(&ws.hdr[kHdrTicket]) != static_cast<uint32_t>(total) + gridDim.x)
    atomicOr(&ws.hdr[kHdrStatus], kStatusBadTicket);
  ws.hdr[kHdrTicket] = 0u;
  ws.hdr[kHdrDone] = 0u;
  __threadfence();
  ws.hdr[kHdrEpoch] = (epoch + 1u) & kEpochMask;
}

// Producer-side end of stream: mark the stage as "no more tiles" with the
// 33 arrivals its full barrier expects.
__device__ __forceinline__ void post_sentinel(uint64_t* full_s, uint64_t* tid_s, int* tile_s, int lane) {
  if (lane == 0) {
    *tile_s = -1;
    mbar_arrive(tid_s);
    mbar_arrive(full_s);
  }
  mbar_arrive(full_s);
}

// Compute-warp wait on an mbarrier phase: warp 0 waits on the barrier, the
// other compute warps block in a named barrier (which issues nothing), so a
// wait costs one warp's polling instead of all of theirs.  Returns false on a
// timeout (then every compute thread sees false).
__device__ __forceinline__ bool compute_wait(uint64_t* bar, uint32_t parity, uint32_t* status, int warp,
                                             int nc, volatile uint32_t* s_fail) {
  if (warp == 0) {
    const bool ok = mbar_wait_bounded(bar, parity, status);
    if (!ok && (threadIdx.x & 31) == 0) *s_fail = 1u;
  }
  named_sync(1, nc);
  return *s_fail == 0u;
}

// ---------------------------------------------------------------------------
// Warp roles shared by the forward and backward kernels
// ---------------------------------------------------------------------------
// Producer warp, one tile: bring `n` floats of a contiguous global row into
// shared memory -- one bulk copy (counted on `bar` by lane 0, which must
// include `*bulk_bytes` in its expect_tx) when the row is 16-byte aligned and
// a whole number of 16-byte units, else one 4-byte cp.async per element.
__device__ __forceinline__ uint32_t row_bulk_bytes(const float* src, int n) {
  return ((reinterpret_cast<uintptr_t>(src) & 15u) == 0u && (n & 3) == 0) ? static_cast<uint32_t>(n) * 4u : 0u;
}
__device__ __forceinline__ void load_row(float* dst, const float* src, int n, uint32_t bulk_bytes, uint64_t* bar,
                                         int lane) {
  if (bulk_bytes) {
    if (lane == 0) bulk_g2s(dst, src, bulk_bytes, bar);
  } else {
    for (int i = lane; i < n; i += 32) cp_async_4(dst + i, src + i);
  }
}

// Producer warp: tickets -> tiles -> loads into the ring.  `issue(s, ticket)`
// sets s_tile[s] and issues the stage's TMA (lane 0) and cp.async (all lanes).
template <int S, class Issue>
__device__ __forceinline__ void producer_loop(uint64_t* full, uint64_t* empty, uint64_t* tid_full, int* s_tile,
                                              uint32_t* hdr, int total, int lane, Issue&& issue) {
  uint32_t* status = &hdr[kHdrStatus];
  for (int k = 0;; ++k) {
    const int s = k % S;
    if (k >= S && !mbar_wait_bounded(&empty[s], ((k / S) - 1) & 1, status, 512)) break;
    uint32_t ticket = 0;
    if (lane == 0) ticket = atomicAdd(&hdr[kHdrTicket], 1u);
    ticket = __shfl_sync(0xffffffffu, ticket, 0);
    if (ticket >= static_cast<uint32_t>(total)) {
      post_sentinel(&full[s], &tid_full[s], &s_tile[s], lane);
      break;
    }
    issue(s, static_cast<int>(ticket));
    cp_async_mbar_arrive_noinc(&full[s]);
    if (lane == 0) mbar_arrive(&tid_full[s]);  // tile id known: the look-back warp may start
  }
  cp_async_wait_all();
}

// Look-back warp: follows the ring in tile order -- starting as soon as the
// producer has assigned a tile, before its data lands -- and leaves the
// incoming vector (forward: state entering the tile; backward: gradient
// arriving at its end) in vec[k % 2][BP] for the compute warps, while they
// run the tile's first pass.  `body(tile, run)` fills this lane's channels.
template <int S, int BP, class Body>
__device__ __forceinline__ void lookback_loop(uint64_t* tid_full, const int* s_tile, uint64_t* vec_full,
                                              uint64_t* vec_empty, float* vec, uint32_t* status, int lane,
                                              Body&& body) {
  constexpr int CPT = BP / 32;
  for (int k = 0;; ++k) {
    const int s = k % S;
    if (!mbar_wait_bounded(&tid_full[s], (k / S) & 1, status, 512)) break;
    const int tile = s_tile[s];
    if (tile < 0) break;
    if (k >= 2 && !mbar_wait_bounded(&vec_empty[k & 1], ((k >> 1) - 1) & 1, status, 512)) break;
    float run[CPT];
    body(tile, run);
#pragma unroll
    for (int q = 0; q < CPT; ++q) vec[(k & 1) * BP + lane * CPT + q] = run[q];
    __syncwarp();
    if (lane == 0) mbar_arrive(&vec_full[k & 1]);
  }
}

// ---------------------------------------------------------------------------
// Forward
// ---------------------------------------------------------------------------
template <typename T, int BP, int Q>
struct FwdCfg {
  static constexpr int CPT = BP / 32;
  static constexpr int SEG = (BP <= 64) ? 32 : 16;
  static constexpr int NW = Q / SEG;  // compute warps
  static constexpr int NC = NW * 32;  // compute threads
  static constexpr int NT = NC + 64;  // + producer warp + look-back warp
  static_assert(BP % 32 == 0 && BP <= 128 && Q % SEG == 0 && NC >= Q && NC >= BP, "geometry");
  static constexpr int kX = Q * BP * static_cast<int>(sizeof(T));
  static constexpr int kStage = align_up(kX + (Q + 4) * 4, 128);  // x tile | decay row | A_h
  // per-CTA state after the ring
  static constexpr int oAW = 0;                  // float2[Q] (token decay, token weight)
  static constexpr int oG = oAW + Q * 8;         // float[Q]  decay from the segment start through t
  static constexpr int oL2 = oG + Q * 4;         // float[Q]  log2 decay
  static constexpr int oE = oL2 + Q * 4;         // float[NW][BP]
  static constexpr int oD = oE + NW * BP * 4;    // float[NW]
  static constexpr int oG0 = oD + NW * 4;        // float[NW]
  static constexpr int oSin = oG0 + NW * 4;      // float[2][BP]  from the look-back warp
  static constexpr int oEt = oSin + 2 * BP * 4;  // float[BP]
  static constexpr int oMisc = oEt + BP * 4;     // float[32]
  static constexpr int oTile = oMisc + 32 * 4;   // int[kMaxStages]
  static constexpr int oBar = align_up(oTile + kMaxStages * 4, 16);  // full, empty, tid_full, vec_full/empty
  static constexpr int kPriv = oBar + (3 * kMaxStages + 4) * 8;
  using R = Ring<kStage, kPriv>;
  static constexpr int S = R::S;
  static constexpr int CTAS = R::CTAS;
  static constexpr int kPrivBase = S * kStage;
  static constexpr int kBytes = kPrivBase + kPriv;
};

template <typename T, int BP, int Q, int MODE, bool SEQ>
__global__ void __launch_bounds__(FwdCfg<T, BP, Q>::NT, FwdCfg<T, BP, Q>::CTAS)
    ema_fwd_kernel(const __grid_constant__ CUtensorMap tm_x, const FwdParams p) {
  using C = FwdCfg<T, BP, Q>;
  constexpr int CPT = C::CPT, SEG = C::SEG, NW = C::NW, NC = C::NC, S = C::S;
  extern __shared__ __align__(128) unsigned char smem[];
  unsigned char* priv = smem + C::kPrivBase;
  float2* s_aw = reinterpret_cast<float2*>(priv + C::oAW);
  float* s_g = reinterpret_cast<float*>(priv + C::oG);
  float* s_l2 = reinterpret_cast<float*>(priv + C::oL2);
  float* s_E = reinterpret_cast<float*>(priv + C::oE);
  float* s_D = reinterpret_cast<float*>(priv + C::oD);
  float* s_G0 = reinterpret_cast<float*>(priv + C::oG0);
  float* s_Sin2 = reinterpret_cast<float*>(priv + C::oSin);
  float* s_Et = reinterpret_cast<float*>(priv + C::oEt);
  float* s_misc = reinterpret_cast<float*>(priv + C::oMisc);
  int* s_tile = reinterpret_cast<int*>(priv + C::oTile);
  uint64_t* full = reinterpret_cast<uint64_t*>(priv + C::oBar);
  uint64_t* empty = full + kMaxStages;
  uint64_t* tid_full = empty + kMaxStages;
  uint64_t* vec_full = tid_full + kMaxStages;
  uint64_t* vec_empty = vec_full + 2;
  __shared__ uint32_t s_epoch, s_fail;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const ScanWorkspace& ws = p.ws;
  uint32_t* status = &ws.hdr[kHdrStatus];
  if (tid == 0) {
    s_fail = 0u;
    s_epoch = ld_volatile_u32(&ws.hdr[kHdrEpoch]) & kEpochMask;
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 33);     // producer lane 0 (expect_tx) + 32 cp.async arrivals
      mbar_init(&empty[s], 1);     // compute thread 0
      mbar_init(&tid_full[s], 1);  // producer lane 0, once the tile id is written
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&vec_full[i], 1);   // look-back lane 0
      mbar_init(&vec_empty[i], 1);  // compute thread 0
    }
    fence_mbar_init();
  }
  __syncthreads();
  const uint32_t epoch = s_epoch;
  const uint32_t tag = epoch + 1u;
  const int BH = p.B * p.H;
  const int total = BH * p.nc;

  if (warp == NW) {
    // ------------------------------ producer ------------------------------
    if (lane == 0) tma_prefetch_desc(&tm_x);
    producer_loop<S>(full, empty, tid_full, s_tile, ws.hdr, total, lane, [&](int s, int ticket) {
      const int c = fast_div(ticket, p.div_bh), bh = ticket - c * BH;
      const int b = fast_div(bh, p.div_h), h = bh - b * p.H, t0 = c * Q;
      unsigned char* st = smem + s * C::kStage;
      float* raw = reinterpret_cast<float*>(st + C::kX);
      const float* src = p.rows + static_cast<size_t>(bh) * p.L + t0;
      const int n = min(Q, p.L - t0);
      const uint32_t bulk = row_bulk_bytes(src, n);
      if (lane == 0) {
        s_tile[s] = ticket;
        mbar_arrive_expect_tx(&full[s], C::kX + bulk);
        tma_load_4d(st, &tm_x, &full[s], 0, h, t0, b);
      }
      load_row(raw, src, n, bulk, &full[s], lane);
      if (MODE == kFwdDt && lane == 0) cp_async_4(raw + Q, p.A + h);
    });
    return;
  }
  if (warp == NW + 1) {
    // ------------------------------ look-back ------------------------------
    lookback_loop<S, BP>(tid_full, s_tile, vec_full, vec_empty, s_Sin2, status, lane,
                         [&](int tile, float(&run)[CPT]) {
                           const int c = fast_div(tile, p.div_bh), bh = tile - c * BH;
                           float rdec = 1.f;
                           bool at_start = true;
                           if (c > 0) {
                             at_start = lookback_warp<BP>(ws, tag, bh, BH, c, -1, p.nc, lane, run, rdec);
                           } else {
#pragma unroll
                             for (int q = 0; q < CPT; ++q) run[q] = 0.f;
                           }
                           if (at_start && p.init != nullptr) {
                             const float* iv = p.init + static_cast<size_t>(bh) * p.P;
#pragma unroll
                             for (int q = 0; q < CPT; ++q)
                               if (lane * CPT + q < p.P) run[q] = fmaf(rdec, iv[lane * CPT + q], run[q]);
                           }
                         });
    return;
  }

  // ------------------------------ compute warps ---------------------------
  const int s0 = warp * SEG;
  const int ch = lane * CPT;
  const bool ch_ok = ch < p.P;  // P is a multiple of CPT: a pack is wholly in or out
  const unsigned FULL = 0xffffffffu;
  for (int k = 0;; ++k) {
    const int s = k % S;
    if (!compute_wait(&full[s], (k / S) & 1, status, warp, NC, &s_fail)) break;
    const int tile = s_tile[s];
    if (tile < 0) break;
    const int c = fast_div(tile, p.div_bh), bh = tile - c * BH;
    const int b = fast_div(bh, p.div_h), h = bh - b * p.H, t0 = c * Q;
    const size_t slot = static_cast<size_t>(tile);
    const T* s_x = reinterpret_cast<const T*>(smem + s * C::kStage);
    const float* raw = reinterpret_cast<const float*>(smem + s * C::kStage + C::kX);

    // ---- per-token decay and weight; decay products within each segment -----
    if (tid < Q) {
      const int t = t0 + tid;
      float a = 1.f, w = 0.f, l2 = 0.f;
      if (t < p.L) {
        if (MODE == kFwdLog2) {
          l2 = raw[tid];
          w = 1.f;
        } else {
          const float d = raw[tid];
          l2 = d * raw[Q] * kLog2e;
          w = d;
        }
        a = exp2f(l2);
        if (SEQ && t > 0) {
          const size_t i = static_cast<size_t>(b) * p.L + t;
          if (load_seq_id(p.seq_idx, p.seq_idx_type, i) != load_seq_id(p.seq_idx, p.seq_idx_type, i - 1))
            a = 0.f;
        }
      }
      float g = a;  // product of the decays from the segment start through t
#pragma unroll
      for (int o = 1; o < SEG; o <<= 1) {
        const float n = __shfl_up_sync(FULL, g, o, SEG);
        if ((lane & (SEG - 1)) >= o) g *= n;
      }
      s_aw[tid] = make_float2(a, w);
      s_g[tid] = g;
      if ((lane & (SEG - 1)) == SEG - 1) s_D[tid / SEG] = g;
      s_l2[tid] = l2;
    }
    if (MODE == kFwdLog2 && (p.da_cs != nullptr || p.da_cs_sum != nullptr)) {
      // within-chunk cumsum of the log2 decay (reference outputs da_cs / da_cs_sum)
      float v = (tid < Q) ? s_l2[tid] : 0.f;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float n = __shfl_up_sync(FULL, v, o);
        if (lane >= o) v += n;
      }
      if (lane == 31) s_misc[warp] = v;
      named_sync(1, NC);
      float pre = 0.f;
      for (int w = 0; w < warp; ++w) pre += s_misc[w];
      v += pre;
      if (tid < Q && t0 + tid < p.L && p.da_cs != nullptr) p.da_cs[static_cast<size_t>(bh) * p.L + t0 + tid] = v;
      if (tid == Q - 1 && p.da_cs_sum != nullptr) p.da_cs_sum[static_cast<size_t>(bh) * p.nc + c] = v;
    }
    named_sync(1, NC);

    // ---- pass 1: local scan of the segment from zero, kept in registers -------
    float zl[SEG][CPT];
    {
      float z[CPT];
#pragma unroll
      for (int q = 0; q < CPT; ++q) z[q] = 0.f;
#pragma unroll
      for (int i = 0; i < SEG; ++i) {
        const float2 aw = s_aw[s0 + i];
        float xv[CPT];
        load_pack<T, CPT>(s_x + (s0 + i) * BP + ch, xv);
#pragma unroll
        for (int q = 0; q < CPT; ++q) {
          z[q] = (MODE == kFwdLog2) ? fmaf(aw.x, z[q], xv[q]) : fmaf(aw.x, z[q], aw.y * xv[q]);
          zl[i][q] = z[q];
        }
      }
#pragma unroll
      for (int q = 0; q < CPT; ++q) s_E[warp * BP + ch + q] = z[q];
    }
    named_sync(1, NC);

    // ---- chain the segments; publish the tile aggregate ---------------------
    const bool has_succ = (c + 1 < p.nc);
    if (tid < BP) {
      float Sv = 0.f, Gd = 1.f;
#pragma unroll
      for (int q = 0; q < NW; ++q) {
        const float e = s_E[q * BP + tid];
        s_E[q * BP + tid] = Sv;  // state before segment q (zero tile input)
        if (tid == 0) s_G0[q] = Gd;
        Sv = fmaf(s_D[q], Sv, e);
        Gd *= s_D[q];
      }
      s_Et[tid] = Sv;
      if (tid == 0) s_misc[0] = Gd;
      if (c > 0 && has_succ) {
        uint64_t* agg = ws.agg + slot * (BP + 1);
        st_relaxed_u64(agg + tid, tag_word(Sv, tag));
        if (tid == 0) st_relaxed_u64(agg + BP, tag_word(Gd, tag));
      }
    }
    named_sync(1, NC);

    // ---- state entering the tile (from the look-back warp) -------------------
    if (!compute_wait(&vec_full[k & 1], (k >> 1) & 1, status, warp, NC, &s_fail)) break;
    // the x stage is no longer read (and the look-back warp has taken the tile id)
    if (tid == 0) mbar_arrive(&empty[s]);
    const float* s_Sin = s_Sin2 + (k & 1) * BP;
    if (tid < BP) {
      const float incl = fmaf(s_misc[0], s_Sin[tid], s_Et[tid]);  // state at the tile end
      if (has_succ) {
        st_relaxed_u64(ws.incl + slot * BP + tid, tag_word(incl, tag));
      } else if (p.final_state != nullptr && tid < p.P) {
        p.final_state[static_cast<size_t>(bh) * p.P + tid] = incl;
      }
      if (p.states != nullptr && tid < p.P)
        p.states[b * p.st_b + static_cast<long long>(c) * p.st_c + h * p.st_h + tid * p.st_p] = s_Sin[tid];
    }

    // ---- pass 2: y = local scan + (segment decay so far) x (incoming state) ---
    {
      const float g0 = s_G0[warp];
      float tin[CPT];
#pragma unroll
      for (int q = 0; q < CPT; ++q) tin[q] = fmaf(g0, s_Sin[ch + q], s_E[warp * BP + ch + q]);
      // running row pointer: one 64-bit add per token
      T* yp = static_cast<T*>(p.y) + b * p.sy_b + static_cast<long long>(t0 + s0) * p.sy_l + h * p.sy_h + ch;
      const long long ystep = p.sy_l;
      const int nv = ch_ok ? p.L - (t0 + s0) : 0;
#pragma unroll
      for (int i = 0; i < SEG; ++i) {
        const float g = s_g[s0 + i];
        float yv[CPT];
#pragma unroll
        for (int q = 0; q < CPT; ++q) yv[q] = fmaf(g, tin[q], zl[i][q]);
        if (i < nv) store_pack_global_cs<T, CPT>(yp, yv);
        yp += ystep;
      }
    }
    named_sync(1, NC);
    if (tid == 0) mbar_arrive(&vec_empty[k & 1]);
  }
  if (tid == 0 && count_cta_done(ws)) reset_counters(ws, epoch, total);
}

// ---------------------------------------------------------------------------
// Backward
// ---------------------------------------------------------------------------
template <typename T, int BP, int Q>
struct BwdCfg {
  static constexpr int CPT = BP / 32;
  static constexpr int SEG = 16;  // tokens per warp segment
  static constexpr int RB = 8;    // tokens per transposed reduction
  static constexpr int NW = Q / SEG;
  static constexpr int NC = NW * 32;
  static constexpr int NT = NC + 64;
  static_assert(BP % 32 == 0 && BP <= 128 && Q % SEG == 0 && NC >= Q && NC >= BP && NT <= 1024, "geometry");
  static constexpr int kX = Q * BP * static_cast<int>(sizeof(T));
  // stage: x tile | dy tile | decay row [Q] | A_h [4] | chunk start state [BP]
  static constexpr int oRaw = 2 * kX;
  static constexpr int oSt = oRaw + (Q + 4) * 4;
  static constexpr int kStage = align_up(oSt + BP * 4, 128);
  static constexpr int oAW = 0;                  // float2[Q] (token decay, token weight)
  static constexpr int oGf = oAW + Q * 8;        // float[Q]  decay from the segment start through t
  static constexpr int oE = oGf + Q * 4;         // float[NW][BP]  forward prefix -> Zin
  static constexpr int oR = oE + NW * BP * 4;    // float[NW][BP]  reverse aggregate -> Rloc
  static constexpr int oD = oR + NW * BP * 4;    // float[NW]
  static constexpr int oHs = oD + NW * 4;        // float[NW]
  static constexpr int oGn = oHs + NW * 4;       // float[2][BP]  from the look-back warp
  static constexpr int oRt = oGn + 2 * BP * 4;   // float[BP]
  static constexpr int oMisc = oRt + BP * 4;     // float[48]
  static constexpr int oTile = oMisc + 48 * 4;   // int[kMaxStages]
  static constexpr int oBar = align_up(oTile + kMaxStages * 4, 16);  // full, empty, tid_full, vec_full/empty
  static constexpr int kPriv = oBar + (3 * kMaxStages + 4) * 8;
  using R = Ring<kStage, kPriv>;
  static constexpr int S = R::S;
  static constexpr int CTAS = R::CTAS;
  static constexpr int kPrivBase = S * kStage;
  static constexpr int kBytes = kPrivBase + kPriv;
};

template <typename T, int BP, int Q, int MODE>
__global__ void __launch_bounds__(BwdCfg<T, BP, Q>::NT, BwdCfg<T, BP, Q>::CTAS)
    ema_bwd_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_dy,
                   const BwdParams p) {
  using C = BwdCfg<T, BP, Q>;
  constexpr int CPT = C::CPT, SEG = C::SEG, NW = C::NW, NC = C::NC, S = C::S, RB = C::RB;
  extern __shared__ __align__(128) unsigned char smem[];
  unsigned char* priv = smem + C::kPrivBase;
  float2* s_aw = reinterpret_cast<float2*>(priv + C::oAW);
  float* s_gf = reinterpret_cast<float*>(priv + C::oGf);
  float* s_E = reinterpret_cast<float*>(priv + C::oE);
  float* s_R = reinterpret_cast<float*>(priv + C::oR);
  float* s_D = reinterpret_cast<float*>(priv + C::oD);
  float* s_Hs = reinterpret_cast<float*>(priv + C::oHs);
  float* s_Gn2 = reinterpret_cast<float*>(priv + C::oGn);
  float* s_Rt = reinterpret_cast<float*>(priv + C::oRt);
  float* s_misc = reinterpret_cast<float*>(priv + C::oMisc);
  int* s_tile = reinterpret_cast<int*>(priv + C::oTile);
  uint64_t* full = reinterpret_cast<uint64_t*>(priv + C::oBar);
  uint64_t* empty = full + kMaxStages;
  uint64_t* tid_full = empty + kMaxStages;
  uint64_t* vec_full = tid_full + kMaxStages;
  uint64_t* vec_empty = vec_full + 2;
  __shared__ uint32_t s_epoch, s_last, s_fail;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const ScanWorkspace& ws = p.ws;
  uint32_t* status = &ws.hdr[kHdrStatus];
  if (tid == 0) {
    s_fail = 0u;
    s_epoch = ld_volatile_u32(&ws.hdr[kHdrEpoch]) & kEpochMask;
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 33);
      mbar_init(&empty[s], 1);
      mbar_init(&tid_full[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&vec_full[i], 1);
      mbar_init(&vec_empty[i], 1);
    }
    fence_mbar_init();
  }
  __syncthreads();
  const uint32_t epoch = s_epoch;
  const uint32_t tag = epoch + 1u;
  const int BH = p.B * p.H;
  const int total = BH * p.nc;

  if (warp == NW) {
    // ------------------------------ producer ------------------------------
    if (lane == 0) {
      tma_prefetch_desc(&tm_x);
      tma_prefetch_desc(&tm_dy);
    }
    producer_loop<S>(full, empty, tid_full, s_tile, ws.hdr, total, lane, [&](int s, int ticket) {
      const int cr = fast_div(ticket, p.div_bh), bh = ticket - cr * BH;
      const int c = p.nc - 1 - cr;
      const int b = fast_div(bh, p.div_h), h = bh - b * p.H, t0 = c * Q;
      unsigned char* st = smem + s * C::kStage;
      float* raw = reinterpret_cast<float*>(st + C::oRaw);
      float* sst = reinterpret_cast<float*>(st + C::oSt);
      const float* src = p.rows + static_cast<size_t>(bh) * p.L + t0;
      const int n = min(Q, p.L - t0);
      const uint32_t bulk = row_bulk_bytes(src, n);
      const float* srow = p.states + b * p.st_b + static_cast<long long>(c) * p.st_c + h * p.st_h;
      const uint32_t sbulk = (p.st_p == 1) ? row_bulk_bytes(srow, p.P) : 0u;
      if (lane == 0) {
        s_tile[s] = c * BH + bh;
        mbar_arrive_expect_tx(&full[s], 2 * C::kX + bulk + sbulk);
        tma_load_4d(st, &tm_x, &full[s], 0, h, t0, b);
        tma_load_4d(st + C::kX, &tm_dy, &full[s], 0, h, t0, b);
      }
      load_row(raw, src, n, bulk, &full[s], lane);
      if (MODE == kBwdDt && lane == 0) cp_async_4(raw + Q, p.A + h);
      if (sbulk) {
        if (lane == 0) bulk_g2s(sst, srow, sbulk, &full[s]);
      } else {
        for (int i = lane; i < p.P; i += 32) cp_async_4(sst + i, srow + static_cast<long long>(i) * p.st_p);
      }
    });
    return;
  }
  if (warp == NW + 1) {
    // ------------------------------ look-back ------------------------------
    lookback_loop<S, BP>(tid_full, s_tile, vec_full, vec_empty, s_Gn2, status, lane,
                         [&](int tile, float(&run)[CPT]) {
                           const int c = fast_div(tile, p.div_bh), bh = tile - c * BH;
                           float rdec = 1.f;
                           bool at_end = true;
                           if (c + 1 < p.nc) {
                             at_end = lookback_warp<BP>(ws, tag, bh, BH, c, +1, p.nc, lane, run, rdec);
                           } else {
#pragma unroll
                             for (int q = 0; q < CPT; ++q) run[q] = 0.f;
                           }
                           if (at_end && p.d_final != nullptr) {
                             const float* dv = p.d_final + static_cast<size_t>(bh) * p.P;
#pragma unroll
                             for (int q = 0; q < CPT; ++q)
                               if (lane * CPT + q < p.P) run[q] = fmaf(rdec, dv[lane * CPT + q], run[q]);
                           }
                         });
    return;
  }

  // ------------------------------ compute warps ---------------------------
  const int s0 = warp * SEG;
  const int ch = lane * CPT;
  const bool ch_ok = ch < p.P;
  const unsigned FULL = 0xffffffffu;
  for (int k = 0;; ++k) {
    const int s = k % S;
    if (!compute_wait(&full[s], (k / S) & 1, status, warp, NC, &s_fail)) break;
    const int tile = s_tile[s];
    if (tile < 0) break;
    const int c = fast_div(tile, p.div_bh), bh = tile - c * BH;
    const int b = fast_div(bh, p.div_h), h = bh - b * p.H, t0 = c * Q;
    const size_t slot = static_cast<size_t>(tile);
    const unsigned char* st = smem + s * C::kStage;
    const T* s_x = reinterpret_cast<const T*>(st);
    const T* s_dy = reinterpret_cast<const T*>(st + C::kX);
    const float* raw = reinterpret_cast<const float*>(st + C::oRaw);
    const float* s_Sin = reinterpret_cast<const float*>(st + C::oSt);
    const float Ah = (MODE == kBwdDt) ? raw[Q] : 0.f;

    // ---- per-token decay / weight; decay products within each segment ---------
    if (tid < Q) {
      const int t = t0 + tid;
      float a = 1.f, w = 0.f;
      if (t < p.L) {
        if (MODE == kBwdCumsum) {
          const float prev = (tid == 0) ? 0.f : raw[tid - 1];
          a = exp2f(raw[tid] - prev);
          w = 1.f;
        } else {
          const float d = raw[tid];
          a = exp2f(d * Ah * kLog2e);
          w = d;
        }
      }
      float g = a;
#pragma unroll
      for (int o = 1; o < SEG; o <<= 1) {
        const float n = __shfl_up_sync(FULL, g, o, SEG);
        if ((lane & (SEG - 1)) >= o) g *= n;
      }
      s_aw[tid] = make_float2(a, w);
      s_gf[tid] = g;
      if ((lane & (SEG - 1)) == SEG - 1) s_D[tid / SEG] = g;
    }
    named_sync(1, NC);

    // ---- pass 1: local forward scan (kept in registers) and reverse aggregate --
    float zl[SEG][CPT];
    {
      float z[CPT], r[CPT];
#pragma unroll
      for (int q = 0; q < CPT; ++q) z[q] = r[q] = 0.f;
#pragma unroll
      for (int i = 0; i < SEG; ++i) {
        const float2 aw = s_aw[s0 + i];
        float xv[CPT];
        load_pack<T, CPT>(s_x + (s0 + i) * BP + ch, xv);
#pragma unroll
        for (int q = 0; q < CPT; ++q) {
          z[q] = (MODE == kBwdCumsum) ? fmaf(aw.x, z[q], xv[q]) : fmaf(aw.x, z[q], aw.y * xv[q]);
          zl[i][q] = z[q];
        }
        const int j = SEG - 1 - i;
        const float aj = s_aw[s0 + j].x;
        float dv[CPT];
        load_pack<T, CPT>(s_dy + (s0 + j) * BP + ch, dv);
#pragma unroll
        for (int q = 0; q < CPT; ++q) r[q] = aj * (dv[q] + r[q]);
      }
#pragma unroll
      for (int q = 0; q < CPT; ++q) {
        s_E[warp * BP + ch + q] = z[q];
        s_R[warp * BP + ch + q] = r[q];
      }
    }
    named_sync(1, NC);

    // ---- chain segments: Zin (forward) and Rloc (reverse); publish ----------
    const bool has_succ = (c > 0);  // the reverse chain continues towards chunk 0
    if (tid < BP) {
      float Sv = (tid < p.P) ? s_Sin[tid] : 0.f;
#pragma unroll
      for (int q = 0; q < NW; ++q) {
        const float e = s_E[q * BP + tid];
        s_E[q * BP + tid] = Sv;  // true state before segment q
        Sv = fmaf(s_D[q], Sv, e);
      }
      float r = 0.f, Hd = 1.f;
#pragma unroll
      for (int q = NW - 1; q >= 0; --q) {
        const float rr = s_R[q * BP + tid];
        s_R[q * BP + tid] = r;  // gradient w.r.t. z at the segment end, from later segments
        if (tid == 0) s_Hs[q] = Hd;
        r = fmaf(s_D[q], r, rr);
        Hd *= s_D[q];
      }
      s_Rt[tid] = r;  // gradient w.r.t. the state entering the tile, from this tile's dy
      if (tid == 0) s_misc[0] = Hd;
      if (c + 1 < p.nc && has_succ) {
        uint64_t* agg = ws.agg + slot * (BP + 1);
        st_relaxed_u64(agg + tid, tag_word(r, tag));
        if (tid == 0) st_relaxed_u64(agg + BP, tag_word(Hd, tag));
      }
    }
    named_sync(1, NC);

    // ---- gradient arriving at the tile end (from the look-back warp) ----------
    if (!compute_wait(&vec_full[k & 1], (k >> 1) & 1, status, warp, NC, &s_fail)) break;
    const float* s_Gn = s_Gn2 + (k & 1) * BP;
    if (tid < BP) {
      const float incl = fmaf(s_misc[0], s_Gn[tid], s_Rt[tid]);  // gradient w.r.t. the state before the tile
      if (has_succ) {
        st_relaxed_u64(ws.incl + slot * BP + tid, tag_word(incl, tag));
      } else if (p.d_init != nullptr && tid < p.P) {
        p.d_init[static_cast<size_t>(bh) * p.P + tid] = incl;
      }
    }

    // ---- pass 2: reverse sweep with exact gradients ------------------------------
    float dap = 0.f;  // dt form: sum over this lane's tokens of dt * dl
    {
      float zin[CPT], g[CPT];
      const float hs = s_Hs[warp];
#pragma unroll
      for (int q = 0; q < CPT; ++q) {
        zin[q] = s_E[warp * BP + ch + q];
        g[q] = fmaf(hs, s_Gn[ch + q], s_R[warp * BP + ch + q]);  // gradient w.r.t. z at the segment end
      }
      const float* dlast = (p.d_last != nullptr && t0 + Q >= p.L) ? p.d_last + static_cast<size_t>(bh) * p.P
                                                                 : nullptr;
      // running row pointer (reverse order): one 64-bit add per token
      const long long dxstep = p.sdx_l;
      T* dxp = static_cast<T*>(p.dx) + b * p.sdx_b + static_cast<long long>(t0 + s0 + SEG - 1) * dxstep +
               h * p.sdx_h + ch;
      const int nv = ch_ok ? p.L - (t0 + s0) : 0;
#pragma unroll
      for (int blk = SEG / RB - 1; blk >= 0; --blk) {
        float p1[RB], p2[RB];
#pragma unroll
        for (int j = RB - 1; j >= 0; --j) {
          const int i = blk * RB + j;
          const int t = s0 + i;
          const float2 aw = s_aw[t];
          float dv[CPT];
          load_pack<T, CPT>(s_dy + t * BP + ch, dv);
          float Gv[CPT], dxv[CPT];
#pragma unroll
          for (int q = 0; q < CPT; ++q) {
            Gv[q] = dv[q] + g[q];
            dxv[q] = (MODE == kBwdCumsum) ? Gv[q] : aw.y * Gv[q];
          }
          if (dlast != nullptr && t0 + t == p.L - 1) {
#pragma unroll
            for (int q = 0; q < CPT; ++q)
              if (ch + q < p.P) dxv[q] += dlast[ch + q];
          }
          if (i < nv) store_pack_global_cs<T, CPT>(dxp, dxv);
          dxp -= dxstep;
          // state before token t: local scan of the previous token + decay so far x Zin
          const float gprev = (i > 0) ? s_gf[t - 1] : 1.f;
          float q1 = 0.f, q2 = 0.f;
#pragma unroll
          for (int q = 0; q < CPT; ++q) {
            const float zp = (i > 0) ? fmaf(gprev, zin[q], zl[i > 0 ? i - 1 : 0][q]) : zin[q];
            q1 = fmaf(Gv[q], zp, q1);
            g[q] = aw.x * Gv[q];
          }
          if (MODE == kBwdDt) {
            float xv[CPT];
            load_pack<T, CPT>(s_x + t * BP + ch, xv);
#pragma unroll
            for (int q = 0; q < CPT; ++q) q2 = fmaf(Gv[q], xv[q], q2);
          }
          p1[j] = aw.x * q1;
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
              p.dl[static_cast<size_t>(bh) * p.L + gt] = P1;
            } else {
              p.ddt_rows[static_cast<size_t>(bh) * p.L + gt] = fmaf(Ah, P1, P2);
              dap = fmaf(s_aw[t].y, P1, dap);
            }
          }
        }
      }
    }

    // ---- dt form: per-tile partial of dA (fixed order) -------------------------
    if (MODE == kBwdDt) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) dap += __shfl_xor_sync(FULL, dap, o);
      if (lane == 0) s_misc[1 + warp] = dap;
    }
    named_sync(1, NC);
    if (tid == 0) {
      if (MODE == kBwdDt) {
        float tot = 0.f;
        for (int w = 0; w < NW; ++w) tot += s_misc[1 + w];
        ws.partial[slot] = tot;
      }
      mbar_arrive(&empty[s]);
      mbar_arrive(&vec_empty[k & 1]);
    }
  }
  if (tid == 0) s_last = count_cta_done(ws) ? 1u : 0u;
  named_sync(1, NC);
  if (s_last) {
    if (MODE == kBwdDt) {
      __threadfence();
      for (int hh = tid; hh < p.H; hh += NC) {
        float acc = 0.f;
        for (int cc = 0; cc < p.nc; ++cc)
          for (int bb = 0; bb < p.B; ++bb)
            acc += ld_relaxed_gpu(&ws.partial[static_cast<size_t>(cc) * BH + bb * p.H + hh]);
        p.dA_out[hh] = acc;
      }
      named_sync(1, NC);
    }
    if (tid == 0) reset_counters(ws, epoch, total);
  }
}

// ---------------------------------------------------------------------------
// (B, X, Y) -> (B, Y, X) float32 transpose through 32x32 shared-memory tiles
// (per-token rows for the scan kernels: dt (B,L,H) <-> rows (B,H,L)).
// ---------------------------------------------------------------------------
static __global__ void __launch_bounds__(256) transpose_f32_kernel(const float* __restrict__ src, float* __restrict__ dst,
                                                            int X, int Y) {
  __shared__ float tile[32][33];
  const int b = blockIdx.z;
  const int x0 = blockIdx.x * 32, y0 = blockIdx.y * 32;
  const float* s = src + static_cast<size_t>(b) * X * Y;
  float* d = dst + static_cast<size_t>(b) * X * Y;
#pragma unroll
  for (int r = threadIdx.y; r < 32; r += 8) {
    const int x = x0 + r, y = y0 + threadIdx.x;
    if (x < X && y < Y) tile[r][threadIdx.x] = s[static_cast<size_t>(x) * Y + y];
  }
  __syncthreads();
#pragma unroll
  for (int r = threadIdx.y; r < 32; r += 8) {
    const int y = y0 + r, x = x0 + threadIdx.x;
    if (x < X && y < Y) d[static_cast<size_t>(y) * X + x] = tile[threadIdx.x][r];
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
