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
//   compute warps   scan the tile in the stage: warp w owns a token segment
//                   of it.  Forward: lane l owns a channel pair (BP / 32
//                   channels) over the whole segment, so the local scan needs
//                   no shuffles; backward: lane (run, group) owns a channel
//                   group over a run of tokens, runs chained with shuffles.
//                   The local scan (and, backward, the local gradient) runs
//                   sequentially per thread and stays in registers; segments
//                   are chained in shared memory (two block barriers per
//                   tile), tiles through global memory; outputs go straight
//                   from registers to global memory (coalesced rows, streaming
//                   stores).  Each warp releases the stage with its own
//                   mbarrier arrival as soon as it no longer reads it.
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
template <int STAGE, int PRIV, int MAXC = 2>
struct Ring {
  static constexpr int stages(int n) {
    return n == 1 ? (kSmemPerCtaMax - PRIV) / STAGE : ((kSmemPerSM / n - kCtaReserve) - PRIV) / STAGE;
  }
  static constexpr int pick() {
    for (int n = MAXC; n >= 2; --n)
      if (stages(n) >= 3) return n;
    return 1;
  }
  static constexpr int CTAS = pick();
  static constexpr int S = stages(CTAS) > kMaxStages ? kMaxStages : stages(CTAS);
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
  float* partial;  // dA partial sums, head-major: one per tile (dt-form backward), 4 per tile (tensor-core backward); room for 32
  uint64_t* agg;   // [tiles][BP + 1] aggregate words (index BP: decay)
  uint64_t* incl;  // [tiles][BP] inclusive words
  uint64_t* rec_end;  // one past the workspace's last whole word: records live in [agg, rec_end)
};

// A ring stage's tile, decoded once by the producer for the compute warps.
struct __align__(16) TileInfo {
  int c, b, h, t0;      // chunk, batch, head, first token
  int bh, pad0;         // batch * H + head
  long long out_off;    // element offset of (b, t0, h, 0) in the (B, L, H, P) output
};

struct FwdParams {
  int B, L, H, P, nc;
  FastDiv div_bh, div_h;  // division by B*H and by H
  const float* rows;  // (B,H,L) log2 decay dA (reference form)
  const float* dt;    // (B,L,H) dt (dt form)
  const float* A;     // (H,)
  int dt_rows;        // dt laid out (B,H,L): one contiguous row per tile
  const void* seq_idx;
  int seq_idx_type;
  const float* init;  // (B,H,P)
  float* states;
  long long st_b, st_c, st_h, st_p;
  float* mid_states;  // state entering token Q/2 of each chunk, or null
  long long sm_b, sm_c, sm_h, sm_p;
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
  const float* rows;  // (B,H,L) within-chunk log2 cumsum da_cs (reference form)
  const float* dt;    // (B,L,H) dt (dt form)
  const float* A;     // (H,)
  int dt_rows;        // dt laid out (B,H,L): one contiguous row per tile
  const float* states;
  long long st_b, st_c, st_h, st_p;
  const float* d_final;  // (B,H,P)
  const float* d_last;   // (B,H,P)
  float* dl;             // (B,H,L) reference form
  float* ddt;            // (B,L,H) dt form
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
      backoff = backoff < 128 ? backoff * 2 : 128;
    }
  }
  return true;
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
// `tickets`: the ticket counter as read after a fence that follows this CTA's
// done count (kTicketsUnread: read it here).
constexpr uint32_t kTicketsUnread = 0xffffffffu;
__device__ __forceinline__ void reset_counters(const ScanWorkspace& ws, uint32_t epoch, int total,
                                               uint32_t tickets = kTicketsUnread) {
  if (tickets == kTicketsUnread) {
    __threadfence();
    tickets = ld_volatile_u32(&ws.hdr[kHdrTicket]);
  }
  if (tickets != static_cast<uint32_t>(total) + gridDim.x) atomicOr(&ws.hdr[kHdrStatus], kStatusBadTicket);
  ws.hdr[kHdrTicket] = 0u;
  ws.hdr[kHdrDone] = 0u;
  __threadfence();
  ws.hdr[kHdrEpoch] = (epoch + 1u) & kEpochMask;
}

// End of a launch, in the last CTA only, by `nthreads` threads that share named
// barrier `bar`: resets the counters and advances the epoch.  Tags are the
// epoch + 1 and the epoch wraps to 0 after 2^30 launches, so a record slot
// that no launch since rewrote (a larger shape's slot, say) could carry the
// tag the next launch takes for current; the launch whose reset wraps the
// epoch therefore clears every record word of the workspace first (a few
// microseconds, once per 2^30 launches).
__device__ __forceinline__ void finish_launch(const ScanWorkspace& ws, uint32_t epoch, int total, int tid,
                                              int nthreads, int bar, uint32_t tickets = kTicketsUnread) {
  if (((epoch + 1u) & kEpochMask) == 0u) {
    const size_t n = static_cast<size_t>(ws.rec_end - ws.agg);
    for (size_t i = tid; i < n; i += nthreads) ws.agg[i] = 0ull;
    __threadfence();
    named_sync(bar, nthreads);
  }
  if (tid == 0) reset_counters(ws, epoch, total, tickets);
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

// Producer warp, one tile: gather `n` floats spaced `stride` apart (a column
// of a (B, L, H) tensor) with 4-byte cp.async; the neighbouring heads' tiles
// read the same sectors at about the same time, so DRAM sees each once.
__device__ __forceinline__ void gather_col(float* dst, const float* src, int stride, int n, int lane) {
  for (int i = lane; i < n; i += 32) cp_async_4(dst + i, src + static_cast<size_t>(i) * stride);
}

// Producer warp: tickets -> tiles -> loads into the ring.  `issue(s, ticket)`
// sets s_tile[s] and issues the stage's TMA (lane 0) and cp.async (all lanes).
// The next ticket is drawn as soon as the current one is taken, so the
// counter's round trip (a microsecond or more under contention) overlaps the
// wait for a free stage instead of adding to every refill.  Tickets are
// still taken in increasing order per CTA, and each producer still draws
// exactly one ticket past the last tile.  Before waiting for a free stage the
// producer asks for the upcoming tile's data in L2 (`prefetch(ticket)`, lane
// 0): its DRAM reads then start a stage earlier than the ring alone allows.
template <int S, class Issue, class Prefetch>
__device__ __forceinline__ void producer_loop(uint64_t* full, uint64_t* empty, uint64_t* tid_full, int* s_tile,
                                              uint32_t* hdr, int total, int lane, Issue&& issue,
                                              Prefetch&& prefetch) {
  uint32_t* status = &hdr[kHdrStatus];
  uint32_t next = 0;
  if (lane == 0) next = atomicAdd(&hdr[kHdrTicket], 1u);
  for (int k = 0;; ++k) {
    const int s = k % S;
    if (k >= S) {
      if (lane == 0 && next < static_cast<uint32_t>(total)) prefetch(static_cast<int>(next));
      if (!mbar_wait_bounded(&empty[s], ((k / S) - 1) & 1, status, 128)) break;
    }
    const uint32_t ticket = __shfl_sync(0xffffffffu, next, 0);
    if (ticket < static_cast<uint32_t>(total) && lane == 0) next = atomicAdd(&hdr[kHdrTicket], 1u);
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
// `pre(k, s)` runs first, once slot k % 2 is free (it may prepare other
// per-tile tables in that slot and signal them itself); returning false ends
// the loop.  Having read the tile id the warp arrives on the stage's empty
// barrier (which counts the compute warps and this warp): the compute warps
// arrive only after `pre`'s consumers have finished, so `pre` may still read
// the stage.
template <int S, int BP, class Pre, class Body>
__device__ __forceinline__ void lookback_loop(uint64_t* tid_full, const int* s_tile, uint64_t* empty,
                                              uint64_t* vec_full, uint64_t* vec_empty, float* vec,
                                              uint32_t* status, int lane, Pre&& pre, Body&& body) {
  constexpr int CPT = BP / 32;
  for (int k = 0;; ++k) {
    const int s = k % S;
    if (!mbar_wait_bounded(&tid_full[s], (k / S) & 1, status, 512)) break;
    const int tile = s_tile[s];
    if (tile < 0) break;
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    if (k >= 2 && !mbar_wait_bounded(&vec_empty[k & 1], ((k >> 1) - 1) & 1, status, 512)) break;
    if (!pre(k, s)) break;
    float run[CPT];
    body(tile, run);
#pragma unroll
    for (int q = 0; q < CPT; ++q) vec[(k & 1) * BP + lane * CPT + q] = run[q];
    __syncwarp();
    if (lane == 0) mbar_arrive(&vec_full[k & 1]);
  }
}

// ---------------------------------------------------------------------------
// Compute-warp lane layout shared by both kernels
// ---------------------------------------------------------------------------
// A compute warp owns a segment of SEG consecutive tokens of the tile.  Lane
// (ts, cg) = (lane / CG, lane % CG) owns channels [CPL cg, CPL cg + CPL) of
// the 8-token run ts of that segment: the recurrence runs sequentially over
// the run's tokens on CPL / 2 independent fp32x2 pairs, every shared-memory
// access is a vector, and per-token sums over channels reduce across only the
// CG lanes of a run.  Runs are chained inside the warp with shuffles,
// segments inside the CTA through shared memory, tiles through the look-back.
template <int BP, int CPL, int RUN_>
struct Lanes {
  static_assert(CPL == 4 || CPL == 8, "4 or 8 channels per lane");
  static_assert(RUN_ == 8 || RUN_ == 16, "8 or 16 tokens per run");
  static constexpr int NPR = CPL / 2;   // fp32x2 pairs per lane
  static constexpr int CG = BP / CPL;   // lanes per token (channel groups)
  static constexpr int TS = 32 / CG;    // runs per warp
  static constexpr int RUN = RUN_;      // tokens per run
  static constexpr int SEG = TS * RUN;  // tokens per warp
  static_assert(CG >= RUN, "a run's tokens reduce over its channel-group lanes");
};

// Padded index of per-token shared arrays: the runs of a warp (RUN tokens
// apart) then fall in different banks, and tix(r0 + u) = tix(r0) + u for a
// run start r0 and u < RUN.
template <int RUN>
__device__ __forceinline__ constexpr int tix(int t) { return t + t / RUN; }
template <int RUN>
constexpr int tix_size(int q) { return q + q / RUN; }

// Scan of the affine maps z -> D z + E over the TS runs of a warp, in token
// order (inclusive and exclusive).  E holds this lane's 8 channels; lanes of
// one channel group are CG apart.
template <int CG, int TS, int NPR>
__device__ __forceinline__ void runs_scan_fwd(float D, const float2 (&E)[NPR], int ts, float& Dinc,
                                              float2 (&Einc)[NPR], float& Dexc, float2 (&Eexc)[NPR]) {
  const unsigned FULL = 0xffffffffu;
  Dinc = D;
#pragma unroll
  for (int q = 0; q < NPR; ++q) Einc[q] = E[q];
#pragma unroll
  for (int o = 1; o < TS; o <<= 1) {
    const float Dp = __shfl_up_sync(FULL, Dinc, o * CG);
    float2 Ep[NPR];
#pragma unroll
    for (int q = 0; q < NPR; ++q) {
      Ep[q].x = __shfl_up_sync(FULL, Einc[q].x, o * CG);
      Ep[q].y = __shfl_up_sync(FULL, Einc[q].y, o * CG);
    }
    if (ts >= o) {
#pragma unroll
      for (int q = 0; q < NPR; ++q) Einc[q] = f2_fma(f2_bcast(Dinc), Ep[q], Einc[q]);
      Dinc *= Dp;
    }
  }
  Dexc = __shfl_up_sync(FULL, Dinc, CG);
#pragma unroll
  for (int q = 0; q < NPR; ++q) {
    Eexc[q].x = __shfl_up_sync(FULL, Einc[q].x, CG);
    Eexc[q].y = __shfl_up_sync(FULL, Einc[q].y, CG);
  }
  if (ts == 0) {
    Dexc = 1.f;
#pragma unroll
    for (int q = 0; q < NPR; ++q) Eexc[q] = make_float2(0.f, 0.f);
  }
}
// The same in reverse token order: g -> D g + R, composed from the last run.
template <int CG, int TS, int NPR>
__device__ __forceinline__ void runs_scan_rev(float D, const float2 (&R)[NPR], int ts, float& Dinc,
                                              float2 (&Rinc)[NPR], float& Dexc, float2 (&Rexc)[NPR]) {
  const unsigned FULL = 0xffffffffu;
  Dinc = D;
#pragma unroll
  for (int q = 0; q < NPR; ++q) Rinc[q] = R[q];
#pragma unroll
  for (int o = 1; o < TS; o <<= 1) {
    const float Dn = __shfl_down_sync(FULL, Dinc, o * CG);
    float2 Rn[NPR];
#pragma unroll
    for (int q = 0; q < NPR; ++q) {
      Rn[q].x = __shfl_down_sync(FULL, Rinc[q].x, o * CG);
      Rn[q].y = __shfl_down_sync(FULL, Rinc[q].y, o * CG);
    }
    if (ts + o < TS) {
#pragma unroll
      for (int q = 0; q < NPR; ++q) Rinc[q] = f2_fma(f2_bcast(Dinc), Rn[q], Rinc[q]);
      Dinc *= Dn;
    }
  }
  Dexc = __shfl_down_sync(FULL, Dinc, CG);
#pragma unroll
  for (int q = 0; q < NPR; ++q) {
    Rexc[q].x = __shfl_down_sync(FULL, Rinc[q].x, CG);
    Rexc[q].y = __shfl_down_sync(FULL, Rinc[q].y, CG);
  }
  if (ts == TS - 1) {
    Dexc = 1.f;
#pragma unroll
    for (int q = 0; q < NPR; ++q) Rexc[q] = make_float2(0.f, 0.f);
  }
}

// Sum of v[j] over the CG lanes of a channel-group run, transposed: lane cg
// returns the total of v[cg % RUN] (RUN - 1 shuffles for the transposition,
// then one per further doubling up to CG).
template <int RUN, int CG>
__device__ __forceinline__ float group_reduce(float (&v)[RUN], int cg) {
  const unsigned FULL = 0xffffffffu;
#pragma unroll
  for (int half = RUN / 2; half >= 1; half /= 2) {
    const bool up = cg & half;
#pragma unroll
    for (int k = 0; k < half; ++k) {
      const float send = up ? v[k] : v[k + half];
      const float keep = up ? v[k + half] : v[k];
      v[k] = keep + __shfl_xor_sync(FULL, send, half);
    }
  }
  float r = v[0];
#pragma unroll
  for (int o = RUN; o < CG; o <<= 1) r += __shfl_xor_sync(FULL, r, o);
  return r;
}

template <int NPR>
__device__ __forceinline__ void st_row(float* dst, const float2 (&v)[NPR]) {
#pragma unroll
  for (int q = 0; q < NPR; q += 2)
    reinterpret_cast<float4*>(dst)[q / 2] = make_float4(v[q].x, v[q].y, v[q + 1].x, v[q + 1].y);
}
template <int NPR>
__device__ __forceinline__ void ld_row(const float* src, float2 (&v)[NPR]) {
#pragma unroll
  for (int q = 0; q < NPR; q += 2) {
    const float4 a = reinterpret_cast<const float4*>(src)[q / 2];
    v[q] = make_float2(a.x, a.y);
    v[q + 1] = make_float2(a.z, a.w);
  }
}

// Per-segment rows of channel values (s_E, s_R) are padded by 4 floats: the
// chain below reads one channel of every segment at once, and unpadded rows
// of BP floats would put all of them in one bank.
constexpr int kRowPad = 4;

// Chain the NW segments of a tile: thread c < BP runs channel c's chain over
// the segments.  All of the chain's shared-memory operands are loaded before
// the first FMA, so the chain costs NW dependent FMAs, not NW load latencies.
//
// Forward chain.  In: s_E[q][c] = end state of segment q from a zero start,
// s_D[q] = its decay.  Out: s_E[q][c] = state before segment q from the tile
// start state s0 (zero when s0 is null), s_G0[q] = decay from the tile start
// to segment q, s_Et[c] / *Gd = the tile's end state from zero and its decay;
// `agg` (if non-null) receives them as tagged words.
template <int BP, int NW>
__device__ __forceinline__ void chain_segments_fwd(float* s_E, const float* s_D, float* s_G0, float* s_Et,
                                                   float* Gd, const float* s0, int P, uint64_t* agg, uint32_t tag,
                                                   int tid) {
  if (tid >= BP) return;
  constexpr int RS = BP + kRowPad;
  float e[NW], d[NW];
#pragma unroll
  for (int q = 0; q < NW; ++q) {
    e[q] = s_E[q * RS + tid];
    d[q] = s_D[q];
  }
  float Sv = (s0 != nullptr && tid < P) ? s0[tid] : 0.f, Z = 0.f, G = 1.f;
#pragma unroll
  for (int q = 0; q < NW; ++q) {
    const float before = Sv;
    if (tid == 0 && s_G0 != nullptr) s_G0[q] = G;
    Sv = fmaf(d[q], Sv, e[q]);
    Z = fmaf(d[q], Z, e[q]);
    G *= d[q];
    e[q] = before;
  }
#pragma unroll
  for (int q = 0; q < NW; ++q) s_E[q * RS + tid] = e[q];
  if (s_Et != nullptr) s_Et[tid] = Z;
  if (tid == 0) *Gd = G;
  if (agg != nullptr) {
    st_relaxed_u64(agg + tid, tag_word(Z, tag));
    if (tid == 0) st_relaxed_u64(agg + BP, tag_word(G, tag));
  }
}
// Reverse chain.  In: s_R[q][c] = what segment q's own dy contributes to the
// gradient of the state before it, s_D[q] its decay.  Out: s_R[q][c] = the
// gradient w.r.t. z at the end of segment q from later segments of the tile,
// s_Hs[q] = decay of the segments after q, s_Rt[c] / *Hd = the tile's total
// and its decay; `agg` as above.  Threads 0 .. BP-1 of `tid` work (the
// caller may offset tid to run this beside the forward chain).
template <int BP, int NW>
__device__ __forceinline__ void chain_segments_rev(float* s_R, const float* s_D, float* s_Hs, float* s_Rt,
                                                   float* Hd, uint64_t* agg, uint32_t tag, int tid) {
  if (static_cast<unsigned>(tid) >= static_cast<unsigned>(BP)) return;
  constexpr int RS = BP + kRowPad;
  float r[NW], d[NW];
#pragma unroll
  for (int q = 0; q < NW; ++q) {
    r[q] = s_R[q * RS + tid];
    d[q] = s_D[q];
  }
  float g = 0.f, H = 1.f;
#pragma unroll
  for (int q = NW - 1; q >= 0; --q) {
    const float after = g;
    if (tid == 0) s_Hs[q] = H;
    g = fmaf(d[q], g, r[q]);
    H *= d[q];
    r[q] = after;
  }
#pragma unroll
  for (int q = 0; q < NW; ++q) s_R[q * RS + tid] = r[q];
  s_Rt[tid] = g;
  if (tid == 0) *Hd = H;
  if (agg != nullptr) {
    st_relaxed_u64(agg + tid, tag_word(g, tag));
    if (tid == 0) st_relaxed_u64(agg + BP, tag_word(H, tag));
  }
}

// ---------------------------------------------------------------------------
// Forward
// ---------------------------------------------------------------------------
// Compute-warp layout of the forward ("channel-pair lanes"): warp w owns the
// SEG consecutive tokens [w SEG, (w + 1) SEG) of the tile and all of its BP
// channels; lane l owns channels [l CPL, (l + 1) CPL) (CPL = BP / 32: one
// bf16x2 / f16x2 word or a float2 at headdim 64) and runs the recurrence
// sequentially over the SEG tokens.  A warp reads one whole tile row per
// shared-memory instruction (consecutive 4- or 8-byte words: conflict-free
// without swizzle) and writes one whole row of y per store instruction (a
// full 128-byte line at headdim 64, bf16); a segment's end state needs no
// shuffles, only the per-token decay table (one exp per token).
// Tokens per compute warp: 32 at headdim <= 64 (one token per lane in the
// per-token table), 16 at headdim <= 128 (4 channels per lane: the local
// results of 16 tokens fill the same 64 registers).
constexpr int fwd_segment_tokens(int BP) { return BP == 64 ? 32 : 16; }

// CPL consecutive elements of this lane as CPL / 2 float pairs (shared memory).
template <typename T, int CPL>
__device__ __forceinline__ void lane_load(const T* p, float2 (&v)[CPL / 2]) {
  float f[CPL];
  load_pack<T, CPL>(p, f);
#pragma unroll
  for (int q = 0; q < CPL / 2; ++q) v[q] = make_float2(f[2 * q], f[2 * q + 1]);
}
// Streaming store of CPL elements to global memory.
template <typename T, int CPL>
__device__ __forceinline__ void lane_store_cs(T* p, const float2 (&v)[CPL / 2]) {
  float f[CPL];
#pragma unroll
  for (int q = 0; q < CPL / 2; ++q) {
    f[2 * q] = v[q].x;
    f[2 * q + 1] = v[q].y;
  }
  store_pack_global_cs<T, CPL>(p, f);
}
// v rounded to T and back (the value a store of T keeps).
template <typename T>
__device__ __forceinline__ float round_to(float v) {
  return to_f32(from_f32<T>(v));
}

template <int CPL>
__device__ __forceinline__ void lane_st_f32(float* p, const float2 (&v)[CPL / 2]) {
  if constexpr (CPL == 2) {
    *reinterpret_cast<float2*>(p) = v[0];
  } else {
    *reinterpret_cast<float4*>(p) = make_float4(v[0].x, v[0].y, v[1].x, v[1].y);
  }
}
template <int CPL>
__device__ __forceinline__ void lane_ld_f32(const float* p, float2 (&v)[CPL / 2]) {
  if constexpr (CPL == 2) {
    v[0] = *reinterpret_cast<const float2*>(p);
  } else {
    const float4 a = *reinterpret_cast<const float4*>(p);
    v[0] = make_float2(a.x, a.y);
    v[1] = make_float2(a.z, a.w);
  }
}

// ---------------------------------------------------------------------------
// Forward
// ---------------------------------------------------------------------------
template <typename T, int BP, int Q>
struct FwdCfg {
  static constexpr int CPL = BP / 32;  // channels per lane
  static constexpr int NPL = CPL / 2;  // float pairs per lane
  static constexpr int SEG = fwd_segment_tokens(BP);
  static constexpr int CPT = BP / 32;  // channels per lane of the look-back warp
  static constexpr int NW = Q / SEG;   // compute warps
  static constexpr int NC = NW * 32;   // compute threads
  static constexpr int NT = NC + 64;   // + producer warp + look-back warp
  static_assert((BP == 64 || BP == 128) && Q % SEG == 0 && NC >= BP && NC >= Q && NW <= 32, "geometry");
  static constexpr int kX = Q * BP * static_cast<int>(sizeof(T));
  static constexpr int kStage = align_up(kX + (Q + 4) * 4, 128);  // x tile | decay row | A_h
  static constexpr int oTok = 0;                               // float4[Q]  (a, w, g, log2 decay)
  static constexpr int oE = align_up(oTok + Q * 16, 16);       // float[NW][BP + pad]
  static constexpr int oD = oE + NW * (BP + kRowPad) * 4;      // float[NW]
  static constexpr int oG0 = oD + NW * 4;                      // float[NW]
  static constexpr int oSin = align_up(oG0 + NW * 4, 16);      // float[2][BP]  from the look-back warp
  static constexpr int oEt = oSin + 2 * BP * 4;                // float[BP]
  static constexpr int oMisc = oEt + BP * 4;                   // float[32]
  static constexpr int oTile = oMisc + 32 * 4;                 // int[kMaxStages]
  static constexpr int oInfo = align_up(oTile + kMaxStages * 4, 16);  // TileInfo[kMaxStages]
  static constexpr int oBar = oInfo + kMaxStages * static_cast<int>(sizeof(TileInfo));
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
  constexpr int CPT = C::CPT, SEG = C::SEG, NW = C::NW, NC = C::NC, S = C::S, CPL = C::CPL, NPL = C::NPL;
  extern __shared__ __align__(128) unsigned char smem[];
  unsigned char* priv = smem + C::kPrivBase;
  float4* s_tok = reinterpret_cast<float4*>(priv + C::oTok);
  float* s_E = reinterpret_cast<float*>(priv + C::oE);
  float* s_D = reinterpret_cast<float*>(priv + C::oD);
  float* s_G0 = reinterpret_cast<float*>(priv + C::oG0);
  float* s_Sin2 = reinterpret_cast<float*>(priv + C::oSin);
  float* s_Et = reinterpret_cast<float*>(priv + C::oEt);
  float* s_misc = reinterpret_cast<float*>(priv + C::oMisc);
  int* s_tile = reinterpret_cast<int*>(priv + C::oTile);
  TileInfo* s_info = reinterpret_cast<TileInfo*>(priv + C::oInfo);
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
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 33);       // producer lane 0 (expect_tx) + 32 cp.async arrivals
      mbar_init(&empty[s], NW + 1);  // every compute warp + the look-back warp
      mbar_init(&tid_full[s], 1);    // producer lane 0, once the tile id is written
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&vec_full[i], 1);    // look-back lane 0
      mbar_init(&vec_empty[i], NW);  // every compute warp
    }
    fence_mbar_init();
  }
  __syncthreads();  // barriers initialised (under programmatic launch this overlaps the previous kernel)
  const int BH = p.B * p.H;
  const int total = BH * p.nc;
  auto prefetch_tile = [&](int ticket) {
    const int c = fast_div(ticket, p.div_bh), bh = ticket - c * BH;
    const int b = fast_div(bh, p.div_h), h = bh - b * p.H;
    tma_prefetch_l2_4d(&tm_x, 0, h, c * Q, b);
  };
  if (warp == NW && lane == 0) {
    // The first tickets' x tiles, asked into L2 while the previous kernel
    // drains: a hint only (L2 is coherent with that kernel's writes), so it
    // needs no ordering; the CTA's first tickets are about blockIdx.x and
    // blockIdx.x + gridDim.x.
    tma_prefetch_desc(&tm_x);
    for (int t = blockIdx.x; t < total && t < 2 * static_cast<int>(gridDim.x); t += gridDim.x) prefetch_tile(t);
  }
  grid_dep_wait();  // the previous kernel's writes (and its workspace reset) are visible from here
  grid_dep_release();

  if (warp == NW) {
    // ------------------------------ producer ------------------------------
    // (needs no epoch: its first ticket round trip overlaps the epoch read below)
    producer_loop<S>(full, empty, tid_full, s_tile, ws.hdr, total, lane, [&](int s, int ticket) {
      const int c = fast_div(ticket, p.div_bh), bh = ticket - c * BH;
      const int b = fast_div(bh, p.div_h), h = bh - b * p.H, t0 = c * Q;
      unsigned char* st = smem + s * C::kStage;
      float* raw = reinterpret_cast<float*>(st + C::kX);
      const int n = min(Q, p.L - t0);
      const bool rows = (MODE != kFwdDt) || p.dt_rows;
      const float* src = (MODE != kFwdDt) ? p.rows + static_cast<size_t>(bh) * p.L + t0
                         : rows ? p.dt + static_cast<size_t>(bh) * p.L + t0
                                : p.dt + (static_cast<size_t>(b) * p.L + t0) * p.H + h;
      const uint32_t bulk = rows ? row_bulk_bytes(src, n) : 0u;
      if (lane == 0) {
        s_tile[s] = ticket;
        s_info[s] = TileInfo{c, b, h, t0, bh, 0, b * p.sy_b + static_cast<long long>(t0) * p.sy_l + h * p.sy_h};
        mbar_arrive_expect_tx(&full[s], C::kX + bulk);
        tma_load_4d(st, &tm_x, &full[s], 0, h, t0, b);
      }
      if (rows) {
        load_row(raw, src, n, bulk, &full[s], lane);
      } else {
        gather_col(raw, src, p.H, n, lane);  // dt column of head h (stride H)
      }
      if (MODE == kFwdDt && lane == 0) cp_async_4(raw + Q, p.A + h);
    }, prefetch_tile);
    return;
  }
  // the look-back and compute warps tag their records with the launch epoch
  if (tid == 0) s_epoch = ld_volatile_u32(&ws.hdr[kHdrEpoch]) & kEpochMask;
  named_sync(2, NC + 32);  // every warp but the producer
  const uint32_t epoch = s_epoch;
  const uint32_t tag = epoch + 1u;
  if (warp == NW + 1) {
    // ------------------------------ look-back ------------------------------
    lookback_loop<S, BP>(tid_full, s_tile, empty, vec_full, vec_empty, s_Sin2, status, lane,
                         [](int, int) { return true; },
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
  const int s0 = warp * SEG;  // this warp's first token in the tile
  const int ch = lane * CPL;  // this lane's first channel
  const unsigned FULL = 0xffffffffu;
  const float4* tok_w = s_tok + s0;
  for (int k = 0;; ++k) {
    const int s = k % S;
    if (!compute_wait(&full[s], (k / S) & 1, status, warp, NC, &s_fail)) break;
    const int tile = s_tile[s];
    if (tile < 0) break;
    const TileInfo ti = s_info[s];
    const int c = ti.c, bh = ti.bh, b = ti.b, h = ti.h, t0 = ti.t0;
    const size_t slot = static_cast<size_t>(tile);
    const T* s_x = reinterpret_cast<const T*>(smem + s * C::kStage);
    const float* raw = reinterpret_cast<const float*>(smem + s * C::kStage + C::kX);

    // ---- this warp's tokens: decay, weight, decay products from the segment start
    {
      const int i = lane & (SEG - 1);
      const int t = t0 + s0 + i;
      float a = 1.f, w = 0.f, l2 = 0.f;
      if (t < p.L) {
        if (MODE == kFwdLog2) {
          l2 = raw[s0 + i];
          w = 1.f;
        } else {
          const float d = raw[s0 + i];
          l2 = d * raw[Q] * kLog2e;
          w = d;
        }
        a = exp2f(l2);
        if (SEQ && t > 0) {
          const size_t gi = static_cast<size_t>(b) * p.L + t;
          if (load_seq_id(p.seq_idx, p.seq_idx_type, gi) != load_seq_id(p.seq_idx, p.seq_idx_type, gi - 1))
            a = 0.f;
        }
      }
      float g = a;  // product of the decays from the segment start through t
#pragma unroll
      for (int o = 1; o < SEG; o <<= 1) {
        const float n = __shfl_up_sync(FULL, g, o, SEG);
        if (i >= o) g *= n;
      }
      if (lane < SEG) s_tok[s0 + i] = make_float4(a, w, g, l2);
    }
    if (MODE == kFwdLog2 && (p.da_cs != nullptr || p.da_cs_sum != nullptr)) {
      // within-chunk cumsum of the log2 decay (reference outputs da_cs / da_cs_sum)
      named_sync(1, NC);
      float v = (tid < Q) ? s_tok[tid].w : 0.f;
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
    __syncwarp();

    // ---- pass 1: the segment's scan from zero, kept in registers -------------
    const T* x_l = s_x + s0 * BP + ch;
    float2 zl[SEG][NPL];
    {
      float2 z[NPL];
#pragma unroll
      for (int q = 0; q < NPL; ++q) z[q] = make_float2(0.f, 0.f);
#pragma unroll
      for (int u = 0; u < SEG; ++u) {
        const float4 tk = tok_w[u];
        float2 xv[NPL];
        lane_load<T, CPL>(x_l + u * BP, xv);
#pragma unroll
        for (int q = 0; q < NPL; ++q) {
          z[q] = (MODE == kFwdLog2) ? f2_fma(f2_bcast(tk.x), z[q], xv[q])
                                    : f2_fma(f2_bcast(tk.x), z[q], f2_mul(f2_bcast(tk.y), xv[q]));
          zl[u][q] = z[q];
        }
      }
      lane_st_f32<CPL>(s_E + warp * (BP + kRowPad) + ch, z);  // the segment's end state from zero
      if (lane == 0) s_D[warp] = tok_w[SEG - 1].z;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);  // this warp no longer reads the x stage
    named_sync(1, NC);                      // every segment's end state and decay

    // ---- chain the segments; publish the tile aggregate ---------------------
    const bool has_succ = (c + 1 < p.nc);
    chain_segments_fwd<BP, NW>(s_E, s_D, s_G0, s_Et, &s_misc[0], nullptr, p.P,
                               (c > 0 && has_succ) ? ws.agg + slot * (BP + 1) : nullptr, tag, tid);
    if (warp == NW - 1 && !mbar_wait_bounded(&vec_full[k & 1], (k >> 1) & 1, status) && lane == 0) s_fail = 1u;
    named_sync(1, NC);  // chained segments + the state entering the tile
    if (s_fail) break;
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
      if (p.mid_states != nullptr && tid < p.P)  // the state entering segment NW/2 = token Q/2
        p.mid_states[b * p.sm_b + static_cast<long long>(c) * p.sm_c + h * p.sm_h + tid * p.sm_p] =
            fmaf(s_G0[NW / 2], s_Sin[tid], s_E[(NW / 2) * (BP + kRowPad) + tid]);
    }

    // ---- pass 2: y = local scan + (decay from the segment start) x (state entering it)
    float2 tin[NPL];
    {
      const float2 g0 = f2_bcast(s_G0[warp]);
      float2 sin[NPL], sw[NPL];
      lane_ld_f32<CPL>(s_Sin + ch, sin);
      lane_ld_f32<CPL>(s_E + warp * (BP + kRowPad) + ch, sw);
#pragma unroll
      for (int q = 0; q < NPL; ++q) tin[q] = f2_fma(g0, sin[q], sw[q]);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&vec_empty[k & 1]);  // this warp no longer reads the incoming state
    if (p.y != nullptr && ch < p.P) {  // (a state-only pass computes just the chunk and final states)
      T* yp = static_cast<T*>(p.y) + ti.out_off + static_cast<long long>(s0) * p.sy_l + ch;
      const long long ystep = p.sy_l;
      const int nv = p.L - (t0 + s0);
#pragma unroll
      for (int u = 0; u < SEG; ++u) {
        const float2 g = f2_bcast(tok_w[u].z);
        float2 yv[NPL];
#pragma unroll
        for (int q = 0; q < NPL; ++q) yv[q] = f2_fma(g, tin[q], zl[u][q]);
        if (u < nv) lane_store_cs<T, CPL>(yp, yv);
        yp += ystep;
      }
    }
  }
  __shared__ uint32_t s_last;
  named_sync(1, NC);  // every compute thread is past its last store
  if (tid == 0) s_last = count_cta_done(ws) ? 1u : 0u;
  named_sync(1, NC);
  if (s_last) finish_launch(ws, epoch, total, tid, NC, 1);
}

// ---------------------------------------------------------------------------
// Backward
// ---------------------------------------------------------------------------
// Per-token table of one backward tile, built by a single warp (the
// look-back warp, off the compute warps' path): for token t of the tile,
// tok[tix(t)] = (a_t, w_t, A_h a_t, w_t a_t) and g[tix(t)] = the product of
// the decays after t through the end of its RUN-token run (1 at the run end).
// dt form: a_t = exp(dt_t A_h), w_t = dt_t; reference form: a_t =
// 2^(cs_t - cs_{t-1}), w_t = 1 (ema_fwd_triton's decay between rows,
// kernels/ema_kernels/ema_fused.py).  Tokens at or past `n` get a = 1, w = 0.
// Each lane owns Q / 32 consecutive tokens; the suffix product crosses the
// lanes of a run with shuffles.
template <int Q, int RUN, int MODE>
__device__ __forceinline__ void bwd_token_table(const float* raw, float Ah, int n, float4* tok, float2* g,
                                                int lane) {
  constexpr int TPL = Q / 32;                          // tokens per lane
  constexpr int LPR = RUN > TPL ? RUN / TPL : 1;       // lanes per run
  static_assert(TPL >= 1 && TPL <= RUN && RUN % TPL == 0, "a lane's tokens lie in one run");
  const int j0 = lane * TPL;
  float a[TPL], w[TPL];
#pragma unroll
  for (int j = 0; j < TPL; ++j) {
    const int t = j0 + j;
    a[j] = 1.f;
    w[j] = 0.f;
    if (t < n) {
      if (MODE == kBwdCumsum) {
        const float prev = (t == 0) ? 0.f : raw[t - 1];
        a[j] = exp2f(raw[t] - prev);
        w[j] = 1.f;
      } else {
        const float d = raw[t];
        a[j] = exp2f(d * Ah * kLog2e);
        w[j] = d;
      }
    }
  }
  float suf[TPL];  // product of this lane's decays after token j
  float prod = 1.f;
#pragma unroll
  for (int j = TPL - 1; j >= 0; --j) {
    suf[j] = prod;
    prod *= a[j];
  }
  // product of the decays of the later lanes of the same run
  float incl = prod;
#pragma unroll
  for (int o = 1; o < LPR; o <<= 1) {
    const float m = __shfl_down_sync(0xffffffffu, incl, o, LPR);
    if ((lane % LPR) + o < LPR) incl *= m;
  }
  float after = __shfl_down_sync(0xffffffffu, incl, 1, LPR);
  if (lane % LPR == LPR - 1) after = 1.f;
#pragma unroll
  for (int j = 0; j < TPL; ++j) {
    tok[tix<RUN>(j0 + j)] = make_float4(a[j], w[j], Ah * a[j], w[j] * a[j]);
    g[tix<RUN>(j0 + j)] = f2_bcast(suf[j] * after);
  }
}

// dA[h] = the sum of the n per-tile partials of head h (`part`, head-major,
// contiguous), by the NT threads of the last CTA.  Each head gets G
// consecutive lanes (the largest power of two <= 32 with G * H <= NT, else 1);
// lane g of a head sums elements g, g + G, ... in that order with 16 loads in
// flight (float4 loads when the head's run is 16-byte aligned), and the G lanes
// combine in a fixed shuffle tree: the result does not depend on timing, and
// the whole tail costs one or two L2 round trips instead of one per head.
template <int NT>
__device__ __forceinline__ void sum_head_partials(const float* part, int H, int n, float* out, int tid) {
  static_assert(NT % 32 == 0, "whole warps");
  const unsigned FULL = 0xffffffffu;
  int G = 32;
  while (G > 1 && G * H > NT) G >>= 1;
  const bool vec = (n & 3) == 0 && (reinterpret_cast<uintptr_t>(part) & 15u) == 0;
  for (int base = 0; base < H * G; base += NT) {  // warp-uniform trip count
    const int slot = base + tid;
    const int hh = slot / G, g = slot % G;
    float acc = 0.f;
    if (slot < H * G) {
      const float* src = part + static_cast<size_t>(hh) * n;
      if (vec) {
        const float4* s4 = reinterpret_cast<const float4*>(src);
        const int nq = n >> 2;
        float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int j = g; j < nq; j += 16 * G) {
          float4 v[16];
#pragma unroll
          for (int u = 0; u < 16; ++u) v[u] = (j + u * G < nq) ? __ldcg(s4 + j + u * G) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
          for (int u = 0; u < 16; ++u) {
            a.x += v[u].x;
            a.y += v[u].y;
            a.z += v[u].z;
            a.w += v[u].w;
          }
        }
        acc = (a.x + a.y) + (a.z + a.w);
      } else {
        for (int j = g; j < n; j += 16 * G) {
          float v[16];
#pragma unroll
          for (int u = 0; u < 16; ++u) v[u] = (j + u * G < n) ? __ldcg(src + j + u * G) : 0.f;
#pragma unroll
          for (int u = 0; u < 16; ++u) acc += v[u];
        }
      }
    }
    for (int o = G >> 1; o > 0; o >>= 1) acc += __shfl_xor_sync(FULL, acc, o);
    if (slot < H * G && g == 0) out[hh] = acc;
  }
}

// Tokens per compute-warp segment of the backward at block headdim BP: the
// height of the box the host's dx tensor map stores per warp.
constexpr int bwd_segment_tokens(int BP) { return BP == 64 ? 32 : 16; }

template <typename T, int BP, int Q>
struct BwdCfg {
  // 4 channels x 16 tokens per lane at BP = 64 (32-token segments: the
  // per-tile work of a lane amortised over 16 tokens), 8 x 8 at BP = 128
  static constexpr int CPL = (BP == 64) ? 4 : 8;
  using Ln = Lanes<BP, CPL, (BP == 64) ? 16 : 8>;
  static constexpr int CG = Ln::CG, TS = Ln::TS, SEG = Ln::SEG, NPR = Ln::NPR, RUN = Ln::RUN;
  static constexpr int CPT = BP / 32;
  static constexpr int NW = Q / SEG;
  static constexpr int NC = NW * 32;
  static constexpr int NT = NC + 64;
  static_assert((BP == 64 || BP == 128) && Q % SEG == 0 && NC >= BP && NT <= 1024 && NW <= 32 && NW % 2 == 0,
                "geometry");
  static_assert(SEG == bwd_segment_tokens(BP), "the host's dx map stores SEG-token boxes");
  static constexpr int kX = Q * BP * static_cast<int>(sizeof(T));
  // stage: x tile | dy tile | decay row [Q] | A_h [4] | chunk start state [BP]
  static constexpr int oRaw = 2 * kX;
  static constexpr int oSt = oRaw + (Q + 4) * 4;
  static constexpr int kStage = align_up(oSt + BP * 4, 128);
  static constexpr int kTix = tix_size<RUN>(Q);
  // token tables, one per look-back slot (k % 2): built by the look-back warp
  static constexpr int oTok = 0;                           // float4[2][tix]  (a, a, w, w)
  static constexpr int oG = oTok + 2 * kTix * 16;          // float2[2][tix]  decay after t through the run end
  static constexpr int oE = align_up(oG + 2 * kTix * 8, 16);  // float[NW][BP + pad]  forward prefix -> Zin
  static constexpr int oR = oE + NW * (BP + kRowPad) * 4;  // float[NW][BP + pad]  reverse aggregate -> Rloc
  static constexpr int oD = oR + NW * (BP + kRowPad) * 4;  // float[NW]
  static constexpr int oHs = oD + NW * 4;                  // float[NW]
  static constexpr int oGn = align_up(oHs + NW * 4, 16);   // float[2][BP]  from the look-back warp
  static constexpr int oRt = oGn + 2 * BP * 4;             // float[BP]
  static constexpr int oMisc = oRt + BP * 4;               // float[8]
  static constexpr int oTile = oMisc + 8 * 4;              // int[kMaxStages]
  static constexpr int oInfo = align_up(oTile + kMaxStages * 4, 16);  // TileInfo[kMaxStages]
  // full, empty, tid_full, vec_full/empty, tok_full
  static constexpr int oBar = oInfo + kMaxStages * static_cast<int>(sizeof(TileInfo));
  static constexpr int kPriv = oBar + (3 * kMaxStages + 6) * 8;
  using R = Ring<kStage, kPriv>;
  static constexpr int S = R::S;
  static constexpr int CTAS = R::CTAS;
  static constexpr int kPrivBase = S * kStage;
  static constexpr int kBytes = kPrivBase + kPriv;
};

template <typename T, int BP, int Q, int MODE>
__global__ void __launch_bounds__(BwdCfg<T, BP, Q>::NT, BwdCfg<T, BP, Q>::CTAS)
    ema_bwd_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_dy,
                   const __grid_constant__ CUtensorMap tm_dx, const BwdParams p) {
  using C = BwdCfg<T, BP, Q>;
  constexpr int CPT = C::CPT, CG = C::CG, TS = C::TS, SEG = C::SEG, NW = C::NW, NC = C::NC, S = C::S;
  constexpr int CPL = C::CPL, NPR = C::NPR, RUN = C::RUN;
  extern __shared__ __align__(128) unsigned char smem[];
  unsigned char* priv = smem + C::kPrivBase;
  float4* s_tok = reinterpret_cast<float4*>(priv + C::oTok);
  float2* s_g = reinterpret_cast<float2*>(priv + C::oG);
  float* s_E = reinterpret_cast<float*>(priv + C::oE);
  float* s_R = reinterpret_cast<float*>(priv + C::oR);
  float* s_D = reinterpret_cast<float*>(priv + C::oD);
  float* s_Hs = reinterpret_cast<float*>(priv + C::oHs);
  float* s_Gn2 = reinterpret_cast<float*>(priv + C::oGn);
  float* s_Rt = reinterpret_cast<float*>(priv + C::oRt);
  float* s_misc = reinterpret_cast<float*>(priv + C::oMisc);
  int* s_tile = reinterpret_cast<int*>(priv + C::oTile);
  TileInfo* s_info = reinterpret_cast<TileInfo*>(priv + C::oInfo);
  uint64_t* full = reinterpret_cast<uint64_t*>(priv + C::oBar);
  uint64_t* empty = full + kMaxStages;
  uint64_t* tid_full = empty + kMaxStages;
  uint64_t* vec_full = tid_full + kMaxStages;
  uint64_t* vec_empty = vec_full + 2;
  uint64_t* tok_full = vec_empty + 2;
  __shared__ uint32_t s_epoch, s_last, s_fail;
  __shared__ float s_dap[2][NW];  // dt form: each compute warp's dA partial of tile k, slot k % 2

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const ScanWorkspace& ws = p.ws;
  uint32_t* status = &ws.hdr[kHdrStatus];
  if (tid == 0) {
    s_fail = 0u;
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 33);
      mbar_init(&empty[s], NW + 1);
      mbar_init(&tid_full[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&vec_full[i], 1);
      mbar_init(&vec_empty[i], NW);  // released once a compute warp's last pass is done with slot i
      mbar_init(&tok_full[i], 1);
    }
    fence_mbar_init();
  }
  __syncthreads();  // barriers initialised (under programmatic launch this overlaps the previous kernel)
  const int BH = p.B * p.H;
  const int total = BH * p.nc;
  auto prefetch_tile = [&](int ticket) {
    const int cr = fast_div(ticket, p.div_bh), bh = ticket - cr * BH;
    const int c = p.nc - 1 - cr;
    const int b = fast_div(bh, p.div_h), h = bh - b * p.H, t0 = c * Q;
    if (p.dx != nullptr) tma_prefetch_l2_4d(&tm_x, 0, h, t0, b);
    tma_prefetch_l2_4d(&tm_dy, 0, h, t0, b);
  };
  if (warp == NW && lane == 0) {
    // The first tickets' x and dy tiles, asked into L2 while the previous
    // kernel drains: a hint only (L2 is coherent with that kernel's writes),
    // so it needs no ordering; the CTA's first tickets are about blockIdx.x
    // and blockIdx.x + gridDim.x.
    tma_prefetch_desc(&tm_x);
    tma_prefetch_desc(&tm_dy);
    for (int t = blockIdx.x; t < total && t < 2 * static_cast<int>(gridDim.x); t += gridDim.x) prefetch_tile(t);
  }
  grid_dep_wait();  // the previous kernel's writes (and its workspace reset) are visible from here
  grid_dep_release();

  if (warp == NW) {
    // ------------------------------ producer ------------------------------
    // (needs no epoch: its first ticket round trip overlaps the epoch read below)
    producer_loop<S>(full, empty, tid_full, s_tile, ws.hdr, total, lane, [&](int s, int ticket) {
      const int cr = fast_div(ticket, p.div_bh), bh = ticket - cr * BH;
      const int c = p.nc - 1 - cr;
      const int b = fast_div(bh, p.div_h), h = bh - b * p.H, t0 = c * Q;
      unsigned char* st = smem + s * C::kStage;
      float* raw = reinterpret_cast<float*>(st + C::oRaw);
      float* sst = reinterpret_cast<float*>(st + C::oSt);
      const int n = min(Q, p.L - t0);
      const bool rows = (MODE != kBwdDt) || p.dt_rows;
      const float* src = (MODE != kBwdDt) ? p.rows + static_cast<size_t>(bh) * p.L + t0
                         : rows ? p.dt + static_cast<size_t>(bh) * p.L + t0
                                : p.dt + (static_cast<size_t>(b) * p.L + t0) * p.H + h;
      const uint32_t bulk = rows ? row_bulk_bytes(src, n) : 0u;
      // a state-only pass (no dx) needs only the reverse chain: dy and the decays,
      // not x or the chunk start state (pass 1 then scans stale x; nothing uses it)
      const bool full_pass = p.dx != nullptr;
      const float* srow = p.states + b * p.st_b + static_cast<long long>(c) * p.st_c + h * p.st_h;
      const uint32_t sbulk = (full_pass && p.st_p == 1) ? row_bulk_bytes(srow, p.P) : 0u;
      if (lane == 0) {
        s_tile[s] = c * BH + bh;
        s_info[s] = TileInfo{c, b, h, t0, bh, 0, b * p.sdx_b + static_cast<long long>(t0) * p.sdx_l + h * p.sdx_h};
        mbar_arrive_expect_tx(&full[s], (full_pass ? 2 : 1) * C::kX + bulk + sbulk);
        if (full_pass) tma_load_4d(st, &tm_x, &full[s], 0, h, t0, b);
        tma_load_4d(st + C::kX, &tm_dy, &full[s], 0, h, t0, b);
      }
      if (rows) {
        load_row(raw, src, n, bulk, &full[s], lane);
      } else {
        gather_col(raw, src, p.H, n, lane);  // dt column of head h (stride H)
      }
      if (MODE == kBwdDt && lane == 0) cp_async_4(raw + Q, p.A + h);
      if (sbulk) {
        if (lane == 0) bulk_g2s(sst, srow, sbulk, &full[s]);
      } else if (full_pass) {
        for (int i = lane; i < p.P; i += 32) cp_async_4(sst + i, srow + static_cast<long long>(i) * p.st_p);
      }
    }, prefetch_tile);
    return;
  }
  // the look-back and compute warps tag their records with the launch epoch
  if (tid == 0) s_epoch = ld_volatile_u32(&ws.hdr[kHdrEpoch]) & kEpochMask;
  named_sync(2, NC + 32);  // every warp but the producer
  const uint32_t epoch = s_epoch;
  const uint32_t tag = epoch + 1u;
  if (warp == NW + 1) {
    // ------------------------------ look-back ------------------------------
    lookback_loop<S, BP>(tid_full, s_tile, empty, vec_full, vec_empty, s_Gn2, status, lane,
                         [&](int k, int s) {
                           // the tile's token table, once its data has landed
                           if (!mbar_wait_bounded(&full[s], (k / S) & 1, status)) return false;
                           const float* raw = reinterpret_cast<const float*>(smem + s * C::kStage + C::oRaw);
                           const int n = min(Q, p.L - s_info[s].t0);
                           bwd_token_table<Q, RUN, MODE>(raw, (MODE == kBwdDt) ? raw[Q] : 0.f, n,
                                                         s_tok + (k & 1) * C::kTix, s_g + (k & 1) * C::kTix, lane);
                           __syncwarp();
                           if (lane == 0) mbar_arrive(&tok_full[k & 1]);
                           return true;
                         },
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
  const int ts = lane / CG, cg = lane % CG;
  const int s0 = warp * SEG;
  const int r0 = s0 + ts * RUN;
  const int ch = cg * CPL;
  const int nch = min(CPL, p.P - ch);
  const unsigned FULL = 0xffffffffu;
  // stage whose dx store (issued at the end of the previous tile) may still be
  // reading it: released once this tile's first pass is done, so the store's
  // read of shared memory overlaps that pass instead of stalling the warp.  A
  // one-stage ring cannot defer (the next tile's data needs that stage).
  constexpr bool kDefer = S >= 2;
  int pend = -1;
  // dt form: the previous tile's dA partial slot, written by thread 0 once the
  // block barrier below has seen every warp's share (the sum over warps is
  // taken in warp order, so it does not depend on timing)
  size_t pslot = ~size_t{0};
  for (int k = 0;; ++k) {
    const int s = k % S;
    if (!compute_wait(&full[s], (k / S) & 1, status, warp, NC, &s_fail)) break;
    if (MODE == kBwdDt && tid == 0 && pslot != ~size_t{0}) {
      const float* d = s_dap[(k - 1) & 1];
      float t = d[0];
#pragma unroll
      for (int w = 1; w < NW; ++w) t += d[w];
      ws.partial[pslot] = t;
      pslot = ~size_t{0};
    }
    const int tile = s_tile[s];
    if (tile < 0) break;
    const TileInfo ti = s_info[s];
    const int c = ti.c, bh = ti.bh, b = ti.b, h = ti.h, t0 = ti.t0;
    const size_t slot = static_cast<size_t>(tile);
    const unsigned char* st = smem + s * C::kStage;
    const T* s_x = reinterpret_cast<const T*>(st);
    const T* s_dy = reinterpret_cast<const T*>(st + C::kX);
    const float* raw = reinterpret_cast<const float*>(st + C::oRaw);
    const float* s_Sin = reinterpret_cast<const float*>(st + C::oSt);
    const float Ah = (MODE == kBwdDt) ? raw[Q] : 0.f;
    // this run's per-token entries (built by the look-back warp in slot k % 2):
    // r0 is a multiple of RUN, so tix(r0 + u) = tix(r0) + u
    const float4* tok_r = s_tok + (k & 1) * C::kTix + tix<RUN>(r0);
    const float2* g_r = s_g + (k & 1) * C::kTix + tix<RUN>(r0);
    // a timeout is recorded and acted on at the next block barrier, together
    if (!mbar_wait_bounded(&tok_full[k & 1], (k >> 1) & 1, status) && lane == 0) s_fail = 1u;

    // ---- pass 1: forward aggregate; local gradients kept in registers ---------
    //   z  <- a_u z + w_u x_u                      (u ascending; only the end value)
    //   gc <- a_{u+1} gc + dy_u,  gl[u] = gc       (u descending; gradient from
    //                                               this run's dy only)
    const T* x_r = s_x + r0 * BP + ch;
    const T* dy_r = s_dy + r0 * BP + ch;
    float2 gl[RUN][NPR];
    float Dexc, Dsuf;
    float2 Eexc[NPR], Gexc[NPR];
    {
      float2 z[NPR], gc[NPR];
#pragma unroll
      for (int q = 0; q < NPR; ++q) z[q] = gc[q] = make_float2(0.f, 0.f);
      float2 an = make_float2(0.f, 0.f);  // a_{u+1}; nothing beyond the run end
#pragma unroll
      for (int i = 0; i < RUN; ++i) {
        const float4 tk = tok_r[i];
        float2 xv[NPR];
        load_grp<T, NPR>(x_r + i * BP, xv);
#pragma unroll
        for (int q = 0; q < NPR; ++q)
          z[q] = (MODE == kBwdCumsum) ? f2_fma(f2_bcast(tk.x), z[q], xv[q])
                                      : f2_fma(f2_bcast(tk.x), z[q], f2_mul(f2_bcast(tk.y), xv[q]));
        const int u = RUN - 1 - i;
        float2 dv[NPR];
        load_grp<T, NPR>(dy_r + u * BP, dv);
#pragma unroll
        for (int q = 0; q < NPR; ++q) {
          gc[q] = f2_fma(an, gc[q], dv[q]);
          gl[u][q] = gc[q];
        }
        const float4 tu = tok_r[u];
        an = f2_bcast(tu.x);
      }
      // an = a at the run start: the run's dy reaches the state before it as a_r0 gc
      float2 Rr[NPR];
#pragma unroll
      for (int q = 0; q < NPR; ++q) Rr[q] = f2_mul(an, gc[q]);
      const float Drun = an.x * g_r[0].x;
      float Dinc, Drinc;
      float2 Einc[NPR], Rinc[NPR];
      runs_scan_fwd<CG, TS, NPR>(Drun, z, ts, Dinc, Einc, Dexc, Eexc);
      runs_scan_rev<CG, TS, NPR>(Drun, Rr, ts, Drinc, Rinc, Dsuf, Gexc);
      if (ts == TS - 1) {
        st_row<NPR>(s_E + warp * (BP + kRowPad) + ch, Einc);
        if (cg == 0) s_D[warp] = Dinc;
      }
      if (ts == 0) st_row<NPR>(s_R + warp * (BP + kRowPad) + ch, Rinc);
    }
    named_sync(1, NC);  // every segment's aggregates
    if (pend >= 0 && lane == 0) {
      bulk_wait_read<0>();
      mbar_arrive(&empty[pend]);
    }
    pend = -1;

    // ---- chain segments: Zin (forward, true states) and Rloc (reverse); publish
    const bool has_succ = (c > 0);  // the reverse chain continues towards chunk 0
    // the two chains run side by side on different warps where there are enough
    constexpr int kRevTid = (NC >= 2 * BP) ? BP : 0;
    chain_segments_fwd<BP, NW>(s_E, s_D, nullptr, nullptr, &s_misc[1], s_Sin, p.P, nullptr, 0u, tid);
    chain_segments_rev<BP, NW>(s_R, s_D, s_Hs, s_Rt, &s_misc[0],
                               (c + 1 < p.nc && has_succ) ? ws.agg + slot * (BP + 1) : nullptr, tag, tid - kRevTid);
    if (warp == NW - 1 && !mbar_wait_bounded(&vec_full[k & 1], (k >> 1) & 1, status) && lane == 0) s_fail = 1u;
    named_sync(1, NC);  // chained segments + the gradient arriving at the tile end
    if (s_fail) break;
    const float* s_Gn = s_Gn2 + (k & 1) * BP;
    if (tid < BP) {
      const float incl = fmaf(s_misc[0], s_Gn[tid], s_Rt[tid]);  // gradient w.r.t. the state before the tile
      if (has_succ) {
        st_relaxed_u64(ws.incl + slot * BP + tid, tag_word(incl, tag));
      } else if (p.d_init != nullptr && tid < p.P) {
        p.d_init[static_cast<size_t>(bh) * p.P + tid] = incl;
      }
    }

    // ---- pass 2: exact gradients, first token first ---------------------------
    //   G_t = gl_t + (decay after t in the run) x (gradient at the run end)
    //   z_{t-1} runs forward from the true state before the run
    float2 zp[NPR], gend[NPR];
    {
      float2 zw[NPR], gn[NPR], rw[NPR];
      ld_row<NPR>(s_E + warp * (BP + kRowPad) + ch, zw);
      ld_row<NPR>(s_Gn + ch, gn);
      ld_row<NPR>(s_R + warp * (BP + kRowPad) + ch, rw);
      const float2 hs = f2_bcast(s_Hs[warp]), de = f2_bcast(Dexc), ds = f2_bcast(Dsuf);
#pragma unroll
      for (int q = 0; q < NPR; ++q) {
        zp[q] = f2_fma(de, zw[q], Eexc[q]);
        gend[q] = f2_fma(ds, f2_fma(hs, gn[q], rw[q]), Gexc[q]);
      }
    }
    float dsum = 0.f;  // dt form: sum over this lane's tokens of dt a sum_p G z_{t-1}
    if (p.dx != nullptr) {  // (a state-only pass computes just the gradient at the span start)
      {
        // dx goes over this run's rows of the dy tile (dy is no longer read:
        // gl holds it), then one TMA store per warp segment (it clips the
        // rows past seqlen and the channels past headdim)
        T* const dx_s = const_cast<T*>(s_dy) + r0 * BP + ch;
        float pr[RUN];
        // token u + 1's shared-memory operands are read before token u's dx is
        // stored: the store may alias them as far as the compiler knows, so
        // loads written after it would wait for it, one latency per token
        float4 tk_n = tok_r[0];
        float2 gr_n = g_r[0];
        float2 xv_n[NPR];
        load_grp<T, NPR>(x_r, xv_n);
#pragma unroll
        for (int u = 0; u < RUN; ++u) {
          const float4 tk = tk_n;
          const float2 gr = gr_n;
          float2 G[NPR], dxv[NPR], xv[NPR];
#pragma unroll
          for (int q = 0; q < NPR; ++q) xv[q] = xv_n[q];
          if (u + 1 < RUN) {
            tk_n = tok_r[u + 1];
            gr_n = g_r[u + 1];
            load_grp<T, NPR>(x_r + (u + 1) * BP, xv_n);
          }
          const float2 aa = f2_bcast(tk.x), ww = f2_bcast(tk.y);
#pragma unroll
          for (int q = 0; q < NPR; ++q) {
            G[q] = f2_fma(gr, gend[q], gl[u][q]);
            dxv[q] = (MODE == kBwdCumsum) ? G[q] : f2_mul(ww, G[q]);
          }
          store_grp<T, NPR>(dx_s + u * BP, dxv);
          if (MODE == kBwdCumsum) {
            // dl_t = a_t sum_p G_t z_{t-1}
            float2 m = f2_mul(G[0], zp[0]);
#pragma unroll
            for (int q = 1; q < NPR; ++q) m = f2_fma(G[q], zp[q], m);
            pr[u] = tk.x * (m.x + m.y);
#pragma unroll
            for (int q = 0; q < NPR; ++q) zp[q] = f2_fma(aa, zp[q], xv[q]);
          } else {
            // with S1 = sum_p G_t x_t and S2 = sum_p G_t z_{t-1} (this lane's channels):
            // ddt_t = S1 + A a_t S2;  dA += dt_t a_t S2
            float2 s1 = f2_mul(G[0], xv[0]), s2 = f2_mul(G[0], zp[0]);
#pragma unroll
            for (int q = 1; q < NPR; ++q) {
              s1 = f2_fma(G[q], xv[q], s1);
              s2 = f2_fma(G[q], zp[q], s2);
            }
#pragma unroll
            for (int q = 0; q < NPR; ++q) zp[q] = f2_fma(aa, zp[q], f2_mul(ww, xv[q]));
            const float S2 = s2.x + s2.y;
            pr[u] = fmaf(tk.z, S2, s1.x + s1.y);
            dsum = fmaf(tk.w, S2, dsum);
          }
        }
        // the last token's extra gradient is added to the rounded dx, as the
        // reference does after its kernel (dx[:, -1] += d_ox_state)
        if (p.d_last != nullptr && nch > 0) {
          const int ul = p.L - 1 - (t0 + r0);
          if (ul >= 0 && ul < RUN) {
            T* q_dx = dx_s + ul * BP;
            const float* dl = p.d_last + static_cast<size_t>(bh) * p.P + ch;
            float2 v[NPR];
            load_grp<T, NPR>(q_dx, v);
#pragma unroll
            for (int q = 0; q < NPR; ++q) {
              if (2 * q < nch) {
                v[q].x += dl[2 * q];
                v[q].y += dl[2 * q + 1];
              }
            }
            store_grp<T, NPR>(q_dx, v);
          }
        }
        fence_proxy_async_smem();  // this lane's dx rows, for the TMA store

        const float Pr = group_reduce<RUN, CG>(pr, cg);
        if (cg < RUN) {
          const int gt = t0 + r0 + cg;
          if (gt < p.L) {
            if (MODE == kBwdCumsum) p.dl[static_cast<size_t>(bh) * p.L + gt] = Pr;
            else p.ddt[(static_cast<size_t>(b) * p.L + gt) * p.H + h] = Pr;
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) {
      if (p.dx != nullptr) {
        tma_store_4d(&tm_dx, s_dy + s0 * BP, 0, h, t0 + s0, b);
        bulk_commit();
      }
      mbar_arrive(&vec_empty[k & 1]);  // this warp no longer reads slot k % 2 (arriving gradient, token table)
    }
    // the stage is released once the dx store has read it (next tile, or below)
    if (kDefer && p.dx != nullptr) {
      pend = s;
    } else if (lane == 0) {
      if (p.dx != nullptr) bulk_wait_read<0>();
      mbar_arrive(&empty[s]);
    }
    if (MODE == kBwdDt && p.dx != nullptr) {
      // this tile's dA partial: per warp here, summed over the warps by thread
      // 0 at the next tile's first barrier into slot (h, c, b) -- head-major,
      // so that the last CTA reads each head's partials as one contiguous run
      float dap = dsum;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) dap += __shfl_xor_sync(FULL, dap, o);
      if (lane == 0) s_dap[k & 1][warp] = dap;
      if (tid == 0) pslot = (static_cast<size_t>(h) * p.nc + c) * p.B + b;
    }
  }
  // this warp's dx stores have read their stage (nothing in this launch reads dx
  // back; the stores complete with the grid)
  if (lane == 0 && p.dx != nullptr) bulk_wait_read<0>();
  if (pend >= 0 && lane == 0) mbar_arrive(&empty[pend]);
  named_sync(1, NC);
  if (tid == 0) s_last = count_cta_done(ws) ? 1u : 0u;
  named_sync(1, NC);
  if (s_last) {
    if (MODE == kBwdDt && p.dx != nullptr) {
      // dA[h] = sum of head h's nc * B per-tile partials.  The ticket count
      // (checked by the counter reset) is read behind the same fence, so its
      // round trip overlaps the sums; the reset touches neither the partials
      // nor dA, so it follows without a barrier.
      __threadfence();
      const uint32_t tickets = tid == 0 ? ld_volatile_u32(&ws.hdr[kHdrTicket]) : kTicketsUnread;
      sum_head_partials<NC>(ws.partial, p.H, p.nc * p.B, p.dA_out, tid);
      finish_launch(ws, epoch, total, tid, NC, 1, tickets);
    } else {
      finish_launch(ws, epoch, total, tid, NC, 1);
    }
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
