// EMA chunked scan, backward, on the 5th-generation tensor cores (tcgen05 +
// tensor memory), for sm_100a: bf16 x / dy / dx, headdim 64, 128-token tiles.
//
// Same work units, ring, ticket order and decoupled look-back as the
// CUDA-core backward (ema_scan_kernels.cuh); only the tile's arithmetic
// differs.  Within a tile of Q = 128 tokens, with cs_t the inclusive cumsum
// of the natural-log decay l_t (l_t = dt_t A_h, or the reference form's
// log2 cumsum times ln 2) and the strict lower-triangular decay matrix
//
//   L[i][j] = exp(cs_i - cs_j)   for j < i,   0 otherwise,
//
// the recurrences G_t = dy_t + a_{t+1} G_{t+1} and z_t = a_t z_{t-1} + w_t x_t
// become 128 x 64 x 128 MMAs plus rank-one corrections:
//
//   G  = L^T dy + dy + exp(cs_end - cs) Gn     (Gn: gradient arriving at the tile end)
//   Zs = L X        + exp(cs) Sin              (X = w x; Zs_t = a_t z_{t-1}; Sin: state entering the tile)
//
//   dx_t = w_t G_t,   dl_t = sum_p G_t Zs_t,   ddt_t = sum_p G_t x_t + A_h dl_t
//
// Precision.  dl and ddt are sums over the channels of products that cancel,
// so a bf16 rounding of L or X (2^-9 relative) would show through them.  L
// and X are therefore split into bf16 pairs hi + lo (2^-14 relative) and
//
//   L^T dy = L_hi^T dy + L_lo^T dy,   L X = L_hi [X_hi | X_lo] + L_lo X_hi
//
// (the L_lo X_lo term is below fp32 rounding of the result).  dy and x are
// bf16 inputs and enter exactly; sums, scans and accumulators are fp32.  In
// the reference form X = x exactly and X_lo vanishes.
//
// The tile publishes a_0 G_0 (its reverse aggregate from the local G, then
// its inclusive value as soon as the arriving gradient is known) exactly
// like the CUDA-core kernel.  One L buffer serves both products: its rows
// are the K index of L^T dy (MN-major A) and the M index of L X (K-major A).
// An element of L is exp(cs_i - cs_g) exp(cs_g - cs_j) for its 16-key group
// g (cs_g: the group's first key), or one exp where the group's cumsum spans
// more than kWideSpan.
//
// Warp roles (one CTA per SM; tiles flow builder -> MMA -> epilogue):
//   warps 0-7  builders: the tile's cumsum and key factors (warps 0-3, one
//              token per thread), then L (the 8-key chunks of rows i and
//              128 - i split over a quad of threads, so every thread has about
//              the same share of the triangle) and X (a thread pair per row).
//              L_hi of tile k+1 is written once the MMAs of tile k that read
//              L_hi are done, L_lo and X once all of them are;
//   warps 8-11 epilogue: thread i reads lane i of the accumulators and writes
//              dx (into a staging tile, then one TMA store), dl / ddt,
//              the dA partials and the tile's look-back records;
//   warp 12    producer (TMA ring, as the CUDA-core kernel);
//   warp 13    look-back warp (the gradient arriving at each tile's end);
//   warp 14    MMA issue: two commits per tile (the L_hi products, then the
//              L_lo ones) into one of two tensor-memory accumulator sets.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "ema_scan_dispatch.h"
#include "ema_ssd_b200.h"
#include "tc_common.cuh"

namespace emab {
namespace ematc {

using bf16 = __nv_bfloat16;

constexpr int Q = 128;             // tokens per tile
constexpr int BP = 64;             // channels per tile (headdim)
constexpr int NBT = 256;           // builder threads (warps 0-7)
constexpr int NET = 128;           // epilogue threads (warps 8-11): thread i owns token i
constexpr int kProdWarp = 12, kLbWarp = 13, kMmaWarp = 14;
constexpr int NT = 480;
constexpr int S = 3;               // ring stages
constexpr int kTile = Q * BP * 2;  // one 128-row x 128-byte swizzled bf16 tile
constexpr float kWideSpan = 60.f;
constexpr int kBarBuild = 1, kBarEpi = 2, kBarBoth = 3;  // named barriers

// ring stage: x | dy | raw[Q] | A_h | Sin[BP]
constexpr int oSx = 0;
constexpr int oSdy = kTile;
constexpr int oSraw = 2 * kTile;
constexpr int oSA = oSraw + Q * 4;
constexpr int oSst = oSA + 16;
constexpr int kStage = align_up(oSst + BP * 4, 1024);
// operand buffers after the ring (1024-byte aligned)
constexpr int oLh = S * kStage;        // L_hi: 2 key regions of [128 rows x 64 bf16]
constexpr int oLl = oLh + 2 * kTile;   // L_lo
constexpr int oXh = oLl + 2 * kTile;   // X_hi [128 tokens x 64 channels]
constexpr int oXl = oXh + kTile;       // X_lo, right after X_hi: [X_hi | X_lo] is one N = 128 operand
// small state
constexpr int oDx = oXl + kTile;       // dx staging for the TMA store [128 tokens x 64 channels]
constexpr int oCs = oDx + kTile;       // float[2][Q]  cs per accumulator set
constexpr int oW = oCs + 2 * Q * 4;    // float[2][Q]  w
constexpr int oV = oW + 2 * Q * 4;     // float[Q]     key factors exp(cs_g - cs_j)
constexpr int oRef = oV + Q * 4;       // float[8]     cs_g per key group
constexpr int oWsum = oRef + 32;       // float[4]     per-warp scan totals
constexpr int oWide = oWsum + 16;      // u32[4]       per-warp wide-group bits
constexpr int oAgg = oWide + 16;       // float[BP]    local reverse aggregate, staged by epilogue lane 0
constexpr int oGn = oAgg + BP * 4;     // float[2][BP] from the look-back warp
constexpr int oTile = oGn + 2 * BP * 4;                            // int[S]
constexpr int oInfo = align_up(oTile + S * 4, 16);                 // TileInfo[S]
constexpr int oBar = oInfo + S * static_cast<int>(sizeof(TileInfo));
// barriers: full, empty, tid_full [S]; vec_full, vec_empty, mma_b, tmem_empty [2]; op_ready, mma_a
constexpr int oMisc = oBar + (3 * S + 10) * 8;  // u32: taddr, fail (builders), fail (epilogue), epoch, last
constexpr int kSmem = oMisc + 32;
constexpr int kSmemAlloc = kSmem + 1024;  // room to align the base to 1024 bytes
static_assert(kSmemAlloc <= kSmemPerCtaMax, "shared memory");
// tensor memory: two accumulator sets of 256 columns:
//   +0 G (64) | +64 L X_hi (64) | +128 L_hi X_lo (64, dt form)
constexpr uint32_t kCols = 512;
constexpr uint32_t kSetCols = 256;

using tc::chunk_off;
using tc::group_wait;

// 8 floats -> bf16 hi (4 words) and bf16 lo (4 words), hi + lo = v to 2^-14
// relative: hi is v truncated to bf16, lo the (exact) remainder v - hi
// truncated again.  Integer and fp32 add only: no conversion instructions.
__device__ __forceinline__ void split8(const float (&v)[8], uint4& hi, uint4& lo) {
  uint32_t h[4], l[4];
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    const uint32_t ua = __float_as_uint(v[2 * m]), ub = __float_as_uint(v[2 * m + 1]);
    h[m] = __byte_perm(ua, ub, 0x7632);  // the high halves: element 2m in the low 16 bits
    const float2 r = f2_add(make_float2(v[2 * m], v[2 * m + 1]),
                            make_float2(__uint_as_float((ua & 0xffff0000u) ^ 0x80000000u),
                                        __uint_as_float((ub & 0xffff0000u) ^ 0x80000000u)));
    l[m] = __byte_perm(__float_as_uint(r.x), __float_as_uint(r.y), 0x7632);
  }
  hi = make_uint4(h[0], h[1], h[2], h[3]);
  lo = make_uint4(l[0], l[1], l[2], l[3]);
}

template <int MODE>
__global__ void __launch_bounds__(NT, 1)
    ema_bwd_tc_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_dy,
                      const __grid_constant__ CUtensorMap tm_dx, const BwdParams p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  float* s_cs2 = reinterpret_cast<float*>(smem + oCs);
  float* s_w2 = reinterpret_cast<float*>(smem + oW);
  float* s_v = reinterpret_cast<float*>(smem + oV);
  float* s_ref = reinterpret_cast<float*>(smem + oRef);
  float* s_wsum = reinterpret_cast<float*>(smem + oWsum);
  uint32_t* s_wide = reinterpret_cast<uint32_t*>(smem + oWide);
  float* s_agg = reinterpret_cast<float*>(smem + oAgg);
  float* s_Gn2 = reinterpret_cast<float*>(smem + oGn);
  int* s_tile = reinterpret_cast<int*>(smem + oTile);
  TileInfo* s_info = reinterpret_cast<TileInfo*>(smem + oInfo);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + oBar);
  uint64_t* empty = full + S;
  uint64_t* tid_full = empty + S;
  uint64_t* vec_full = tid_full + S;
  uint64_t* vec_empty = vec_full + 2;
  uint64_t* mma_b = vec_empty + 2;
  uint64_t* tmem_empty = mma_b + 2;
  uint64_t* op_ready = tmem_empty + 2;
  uint64_t* mma_a = op_ready + 1;
  uint32_t* s_taddr = reinterpret_cast<uint32_t*>(smem + oMisc);
  volatile uint32_t* s_fail_b = s_taddr + 1;
  volatile uint32_t* s_fail_e = s_taddr + 2;
  uint32_t* s_epoch = s_taddr + 3;
  volatile uint32_t* s_last = s_taddr + 4;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const ScanWorkspace& ws = p.ws;
  uint32_t* status = &ws.hdr[kHdrStatus];
  const unsigned FULL = 0xffffffffu;
  if (tid == 0) {
    *s_fail_b = 0u;
    *s_fail_e = 0u;
    *s_epoch = ld_volatile_u32(&ws.hdr[kHdrEpoch]) & kEpochMask;
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 33);  // producer lane 0 (expect_tx) + 32 cp.async arrivals
      mbar_init(&empty[s], 2);  // epilogue thread 0 + the look-back warp
      mbar_init(&tid_full[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&vec_full[i], 1);
      mbar_init(&vec_empty[i], 1);   // epilogue thread 0
      mbar_init(&mma_b[i], 1);       // tcgen05.commit after the L_lo products
      mbar_init(&tmem_empty[i], 1);  // epilogue thread 0
    }
    mbar_init(op_ready, 1);  // builder thread 0
    mbar_init(mma_a, 1);     // tcgen05.commit after the L_hi products
    fence_mbar_init();
  }
  // L's strict upper triangle is never written again: zero both L buffers once
  for (int o = tid * 16; o < 4 * kTile; o += NT * 16)
    *reinterpret_cast<uint4*>(smem + oLh + o) = make_uint4(0u, 0u, 0u, 0u);
  fence_proxy_async_smem();
  if (warp == 0) {
    tc::tmem_alloc(s_taddr, kCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t epoch = *s_epoch;
  const uint32_t tag = epoch + 1u;
  const int BH = p.B * p.H;
  const int total = BH * p.nc;
  const uint32_t tb = *s_taddr;

  if (warp == kProdWarp) {
    // ------------------------------ producer ------------------------------
    if (lane == 0) {
      tma_prefetch_desc(&tm_x);
      tma_prefetch_desc(&tm_dy);
    }
    producer_loop<S>(full, empty, tid_full, s_tile, ws.hdr, total, lane, [&](int s, int ticket) {
      const int cr = fast_div(ticket, p.div_bh), bh = ticket - cr * BH;
      const int c = p.nc - 1 - cr;
      const int b = fast_div(bh, p.div_h), h = bh - b * p.H, t0 = c * Q;
      unsigned char* st = smem + s * kStage;
      float* raw = reinterpret_cast<float*>(st + oSraw);
      float* sst = reinterpret_cast<float*>(st + oSst);
      const int n = min(Q, p.L - t0);
      const float* src = (MODE == kBwdDt) ? p.dt + (static_cast<size_t>(b) * p.L + t0) * p.H + h
                                          : p.rows + static_cast<size_t>(bh) * p.L + t0;
      const uint32_t bulk = (MODE == kBwdDt) ? 0u : row_bulk_bytes(src, n);
      const float* srow = p.states + b * p.st_b + static_cast<long long>(c) * p.st_c + h * p.st_h;
      const uint32_t sbulk = (p.st_p == 1) ? row_bulk_bytes(srow, BP) : 0u;
      if (lane == 0) {
        s_tile[s] = c * BH + bh;
        s_info[s] = TileInfo{c, b, h, t0, bh, 0, 0};
        mbar_arrive_expect_tx(&full[s], 2 * kTile + bulk + sbulk);
        tma_load_4d(st + oSx, &tm_x, &full[s], 0, h, t0, b);
        tma_load_4d(st + oSdy, &tm_dy, &full[s], 0, h, t0, b);
      }
      if (MODE == kBwdDt) {
        gather_col(raw, src, p.H, n, lane);
        if (lane == 0) cp_async_4(raw + Q, p.A + h);
      } else {
        load_row(raw, src, n, bulk, &full[s], lane);
      }
      if (sbulk) {
        if (lane == 0) bulk_g2s(sst, srow, sbulk, &full[s]);
      } else {
        for (int i = lane; i < BP; i += 32) cp_async_4(sst + i, srow + static_cast<long long>(i) * p.st_p);
      }
    }, [&](int ticket) {
      const int cr = fast_div(ticket, p.div_bh), bh = ticket - cr * BH;
      const int c = p.nc - 1 - cr;
      const int b = fast_div(bh, p.div_h), h = bh - b * p.H, t0 = c * Q;
      tma_prefetch_l2_4d(&tm_x, 0, h, t0, b);
      tma_prefetch_l2_4d(&tm_dy, 0, h, t0, b);
    });
    return;
  }
  if (warp == kLbWarp) {
    // ------------------------------ look-back ------------------------------
    lookback_loop<S, BP>(tid_full, s_tile, empty, vec_full, vec_empty, s_Gn2, status, lane,
                         [](int, int) { return true; },
                         [&](int tile, float(&run)[BP / 32]) {
                           const int c = fast_div(tile, p.div_bh), bh = tile - c * BH;
                           float rdec = 1.f;
                           bool at_end = true;
                           if (c + 1 < p.nc) {
                             at_end = lookback_warp<BP>(ws, tag, bh, BH, c, +1, p.nc, lane, run, rdec);
                           } else {
#pragma unroll
                             for (int q = 0; q < BP / 32; ++q) run[q] = 0.f;
                           }
                           if (at_end && p.d_final != nullptr) {
                             const float* dv = p.d_final + static_cast<size_t>(bh) * BP;
#pragma unroll
                             for (int q = 0; q < BP / 32; ++q) run[q] = fmaf(rdec, dv[lane * (BP / 32) + q], run[q]);
                           }
                         });
    return;
  }

  if (warp == kMmaWarp) {
    // ------------------------------ MMA issue ------------------------------
    const uint32_t sb = smem_u32(smem);
    const uint64_t dKLh = tc::smem_desc_sw128(sb + oLh, 16, 1024);     // L_hi, K-major (M = query row)
    const uint64_t dKLl = tc::smem_desc_sw128(sb + oLl, 16, 1024);     // L_lo, K-major
    const uint64_t dNLh = tc::smem_desc_sw128(sb + oLh, kTile, 1024);  // L_hi^T, MN-major (M = key)
    const uint64_t dNLl = tc::smem_desc_sw128(sb + oLl, kTile, 1024);  // L_lo^T, MN-major
    const uint64_t dNXh = tc::smem_desc_sw128(sb + oXh, kTile, 1024);  // [X_hi | X_lo], MN-major, N = 128
    const uint32_t id64mn = tc::idesc_bf16(128, 64, true, true);
    const uint32_t id64 = tc::idesc_bf16(128, 64, false, true);
    const uint32_t id128 = tc::idesc_bf16(128, 128, false, true);
    auto kstep = [](int s) { return static_cast<uint64_t>(((s >> 2) * kTile + (s & 3) * 32) >> 4); };
    auto nstep = [](int s) { return static_cast<uint64_t>((s * 2048) >> 4); };
    int last = -1;
    for (int k = 0;; ++k) {
      const int s = k % S, kb = k & 1;
      if (!mbar_wait_bounded(&full[s], (k / S) & 1, status)) break;
      if (s_tile[s] < 0) break;
      if (!mbar_wait_bounded(op_ready, k & 1, status)) break;
      if (k >= 2 && !mbar_wait_bounded(&tmem_empty[kb], ((k - 2) >> 1) & 1, status)) break;
      tc::fence_after_sync();
      if (lane == 0) {
        const uint32_t d = tb + kb * kSetCols;
        const uint64_t dNdy = tc::smem_desc_sw128(sb + s * kStage + oSdy, kTile, 1024);
        const uint64_t dNx = tc::smem_desc_sw128(sb + s * kStage + oSx, kTile, 1024);
        // the L_hi products
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) tc::mma_bf16(d, dNLh + nstep(ks), dNdy + nstep(ks), id64mn, ks > 0);
        if (MODE == kBwdDt) {
#pragma unroll
          for (int ks = 0; ks < 8; ++ks) tc::mma_bf16(d + 64, dKLh + kstep(ks), dNXh + nstep(ks), id128, ks > 0);
        } else {
#pragma unroll
          for (int ks = 0; ks < 8; ++ks) tc::mma_bf16(d + 64, dKLh + kstep(ks), dNx + nstep(ks), id64, ks > 0);
        }
        tc::mma_commit(mma_a);
        // the L_lo products
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) tc::mma_bf16(d, dNLl + nstep(ks), dNdy + nstep(ks), id64mn, true);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          tc::mma_bf16(d + 64, dKLl + kstep(ks), (MODE == kBwdDt ? dNXh : dNx) + nstep(ks), id64, true);
        tc::mma_commit(&mma_b[kb]);
      }
      __syncwarp();
      last = k;
    }
    // leave only once the last products have landed
    if (last >= 0) mbar_wait_bounded(&mma_b[last & 1], (last >> 1) & 1, status);
    return;
  }

  if (warp < 8) {
    // ------------------------------ builders ------------------------------
    const bool tok = tid < Q;  // warps 0-3 own one token each for the cumsum
    const int i = tid;
    for (int k = 0;; ++k) {
      const int s = k % S, kb = k & 1;
      if (!group_wait(&full[s], (k / S) & 1, status, warp == 0, kBarBuild, NBT, s_fail_b)) break;
      const int tile = s_tile[s];
      if (tile < 0) break;
      unsigned char* st = smem + s * kStage;
      const float* raw = reinterpret_cast<const float*>(st + oSraw);
      const int n = min(Q, p.L - s_info[s].t0);
      const bool valid = i < n;
      // the epilogue of tile k - 2 is done with set kb's cs / w
      if (k >= 2 && !group_wait(&tmem_empty[kb], ((k - 2) >> 1) & 1, status, warp == 0, kBarBuild, NBT, s_fail_b))
        break;

      // ---- per-token decay, weight and within-tile cumsum (warps 0-3) ----------
      float* csb = s_cs2 + kb * Q;
      float w = 0.f, cs = 0.f;
      if (MODE == kBwdDt) {
        float d = 0.f, v = 0.f;
        if (tok) {
          const float Ah = *reinterpret_cast<const float*>(st + oSA);
          d = valid ? raw[i] : 0.f;
          v = d * Ah;
#pragma unroll
          for (int o = 1; o < 32; o <<= 1) {
            const float nv = __shfl_up_sync(FULL, v, o);
            if (lane >= o) v += nv;
          }
          if (lane == 31) s_wsum[warp] = v;
        }
        named_sync(kBarBuild, NBT);
        float pre = 0.f;
#pragma unroll
        for (int ww = 0; ww < 3; ++ww)
          if (ww < warp) pre += s_wsum[ww];
        w = d;
        cs = v + pre;
      } else if (tok) {
        w = valid ? 1.f : 0.f;
        cs = raw[valid ? i : n - 1] * kLn2;
      }
      if (tok) {
        const float cref = __shfl_sync(FULL, cs, lane & ~15);
        float span = fabsf(cref - cs);
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) span = fmaxf(span, __shfl_xor_sync(FULL, span, o));
        const bool wide = span > kWideSpan;
        csb[i] = cs;
        s_w2[kb * Q + i] = w;
        s_v[i] = wide ? 0.f : __expf(cref - cs);
        if ((lane & 15) == 0) s_ref[i >> 4] = cref;
        const uint32_t wb = __ballot_sync(FULL, wide);
        if (lane == 0) s_wide[warp] = ((wb & 1u) | ((wb >> 15) & 2u)) << (2 * warp);
      }
      named_sync(kBarBuild, NBT);
      const uint32_t wmask = s_wide[0] | s_wide[1] | s_wide[2] | s_wide[3];

      // ---- L: hi once tile k-1's L_hi products are done, lo once all are ---------
      if (k >= 1 && !group_wait(mma_a, (k - 1) & 1, status, warp == 0, kBarBuild, NBT, s_fail_b)) break;
      // a quad of threads builds rows pr + 1 and 127 - pr (row 64 alone for the
      // last quad): about 17.5 chunks per quad, interleaved over its threads
      // (at most five each); lo stays in registers until it may be written
      const int pr = tid >> 2, sub = tid & 3;
      const int ra = pr + 1, rb = 127 - pr;
      const int na = ((ra - 1) >> 3) + 1;
      const int nab = na + ((pr == Q / 2 - 1) ? 0 : ((rb - 1) >> 3) + 1);
      const float csa = csb[ra], csr = csb[rb];
      uint4 lo[5];
      uint32_t offs[5];
#pragma unroll
      for (int q = 0; q < 5; ++q) {
        const int idx = sub + 4 * q;
        offs[q] = 0u;
        lo[q] = make_uint4(0u, 0u, 0u, 0u);
        if (idx < nab) {
          const bool ina = idx < na;
          const int ri = ina ? ra : rb;
          const int cc = ina ? idx : idx - na;
          const float ci = ina ? csa : csr;
          const int j0 = 8 * cc, g = cc >> 1;
          float v8[8];
          if (!((wmask >> g) & 1u)) {
            const float uu = __expf(ci - s_ref[g]);
            const float4 a = *reinterpret_cast<const float4*>(s_v + j0);
            const float4 bq = *reinterpret_cast<const float4*>(s_v + j0 + 4);
            v8[0] = uu * a.x; v8[1] = uu * a.y; v8[2] = uu * a.z; v8[3] = uu * a.w;
            v8[4] = uu * bq.x; v8[5] = uu * bq.y; v8[6] = uu * bq.z; v8[7] = uu * bq.w;
          } else {
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) v8[kk] = __expf(ci - csb[j0 + kk]);
          }
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            if (j0 + kk >= ri) v8[kk] = 0.f;
          uint4 hi;
          split8(v8, hi, lo[q]);
          offs[q] = (j0 >> 6) * kTile + chunk_off(ri, (j0 & 63) >> 3);
          *reinterpret_cast<uint4*>(smem + oLh + offs[q]) = hi;
        }
      }
      if (k >= 1 && !group_wait(&mma_b[kb ^ 1], ((k - 1) >> 1) & 1, status, warp == 0, kBarBuild, NBT, s_fail_b))
        break;
#pragma unroll
      for (int q = 0; q < 5; ++q)
        if (sub + 4 * q < nab) *reinterpret_cast<uint4*>(smem + oLl + offs[q]) = lo[q];
      // ---- X = w x, hi and lo (dt form; the reference form's X is x itself) ------
      // thread pair per token row, four 8-channel chunks each
      if (MODE == kBwdDt) {
        const int xr = tid >> 1, c0 = 4 * (tid & 1);
        const float wx = s_w2[kb * Q + xr];
#pragma unroll
        for (int cc = c0; cc < c0 + 4; ++cc) {
          const uint4 a = *reinterpret_cast<const uint4*>(st + oSx + chunk_off(xr, cc));
          const uint32_t xw[4] = {a.x, a.y, a.z, a.w};
          float v8[8];
#pragma unroll
          for (int m = 0; m < 4; ++m) {
            const float2 f = cvt_pair<bf16>(xw[m]);
            v8[2 * m] = wx * f.x;
            v8[2 * m + 1] = wx * f.y;
          }
          uint4 hi, xlo;
          split8(v8, hi, xlo);
          *reinterpret_cast<uint4*>(smem + oXh + chunk_off(xr, cc)) = hi;
          *reinterpret_cast<uint4*>(smem + oXl + chunk_off(xr, cc)) = xlo;
        }
      }
      fence_proxy_async_smem();
      tc::fence_before_sync();
      named_sync(kBarBuild, NBT);
      if (tid == 0) mbar_arrive(op_ready);
    }
  } else {
    // ------------------------------ epilogue ------------------------------
    const int et = tid - NBT;  // 0..127: token row of the tile = tensor-memory lane
    const int ew = warp - 8;   // = warp % 4: the lane quarter this warp may read
    const int i = et;
    for (int k = 0;; ++k) {
      const int s = k % S, kb = k & 1;
      if (!group_wait(&full[s], (k / S) & 1, status, ew == 0, kBarEpi, NET, s_fail_e)) break;
      const int tile = s_tile[s];
      if (tile < 0) break;
      const TileInfo ti = s_info[s];
      const int c = ti.c, b = ti.b, h = ti.h, t0 = ti.t0, bh = ti.bh;
      const size_t slot = static_cast<size_t>(tile);
      unsigned char* st = smem + s * kStage;
      const float* s_Sin = reinterpret_cast<const float*>(st + oSst);
      const int n = min(Q, p.L - t0);
      const bool valid = i < n;
      if (!group_wait(&mma_b[kb], (k >> 1) & 1, status, ew == 0, kBarEpi, NET, s_fail_e)) break;
      tc::fence_after_sync();
      const uint32_t lane_base = tc::tmem_at(tb, 32 * ew, kb * kSetCols);
      const float cs = s_cs2[kb * Q + i], w = s_w2[kb * Q + i];
      const float cs_end = s_cs2[kb * Q + Q - 1];
      const float e = __expf(cs);           // decay from the tile start through token i
      const float f = __expf(cs_end - cs);  // decay after token i through the tile end

      // ---- reverse aggregate a_0 G_0 from this tile's dy alone -------------------
      // (published for the look-back of earlier chunks when the tile is mid-chain;
      // kept for the inclusive record below in any case)
      const bool mid = (c > 0) && (c + 1 < p.nc);
      if (ew == 0) {
        float g4[4][16];
#pragma unroll
        for (int gq = 0; gq < 4; ++gq) tc::tmem_ld16(lane_base + 16 * gq, g4[gq]);
        tc::tmem_wait_ld();
        if (lane == 0) {
          const float2 e2 = f2_bcast(e);
#pragma unroll
          for (int cc = 0; cc < 8; ++cc) {
            const uint4 d4 = *reinterpret_cast<const uint4*>(st + oSdy + chunk_off(0, cc));
            const float* gv = &g4[cc >> 1][8 * (cc & 1)];
            const float2 a0 = f2_mul(e2, f2_add(make_float2(gv[0], gv[1]), cvt_pair<bf16>(d4.x)));
            const float2 a1 = f2_mul(e2, f2_add(make_float2(gv[2], gv[3]), cvt_pair<bf16>(d4.y)));
            const float2 a2 = f2_mul(e2, f2_add(make_float2(gv[4], gv[5]), cvt_pair<bf16>(d4.z)));
            const float2 a3 = f2_mul(e2, f2_add(make_float2(gv[6], gv[7]), cvt_pair<bf16>(d4.w)));
            reinterpret_cast<float4*>(s_agg)[2 * cc] = make_float4(a0.x, a0.y, a1.x, a1.y);
            reinterpret_cast<float4*>(s_agg)[2 * cc + 1] = make_float4(a2.x, a2.y, a3.x, a3.y);
          }
        }
        __syncwarp();
        if (mid) {
          uint64_t* agg = ws.agg + slot * (BP + 1);
          st_relaxed_u64(agg + 2 * lane, tag_word(s_agg[2 * lane], tag));
          st_relaxed_u64(agg + 2 * lane + 1, tag_word(s_agg[2 * lane + 1], tag));
          if (lane == 0) st_relaxed_u64(agg + BP, tag_word(__expf(cs_end), tag));
        }
      }

      // ---- the gradient arriving at the tile end ------------------------------------
      if (!group_wait(&vec_full[kb], (k >> 1) & 1, status, ew == 0, kBarEpi, NET, s_fail_e)) break;
      const float* Gn = s_Gn2 + kb * BP;
      // ---- inclusive record a_0 G_0 = aggregate + exp(cs_end) Gn, published at once ----
      if (ew == 0) {
        const float dec = __expf(cs_end);
        const float v0 = fmaf(dec, Gn[2 * lane], s_agg[2 * lane]);
        const float v1 = fmaf(dec, Gn[2 * lane + 1], s_agg[2 * lane + 1]);
        if (c > 0) {
          uint64_t* inc = ws.incl + slot * BP;
          st_relaxed_u64(inc + 2 * lane, tag_word(v0, tag));
          st_relaxed_u64(inc + 2 * lane + 1, tag_word(v1, tag));
        } else if (p.d_init != nullptr) {
          p.d_init[static_cast<size_t>(bh) * BP + 2 * lane] = v0;
          p.d_init[static_cast<size_t>(bh) * BP + 2 * lane + 1] = v1;
        }
      }

      // ---- dx into the staging buffer, dl, ddt -----------------------------------------
      // (the previous tile's store has long read the buffer; confirmed before any row is written)
      if (et == 0) bulk_wait_read<0>();
      named_sync(kBarEpi, NET);
      float2 dl2 = make_float2(0.f, 0.f), xs2 = make_float2(0.f, 0.f);
      const float2 e2 = f2_bcast(e), f2 = f2_bcast(f), w2 = f2_bcast(w);
#pragma unroll 1
      for (int gq = 0; gq < 4; ++gq) {
        float dg[16], z0[16], z1[16];
        tc::tmem_ld16(lane_base + 16 * gq, dg);
        tc::tmem_ld16(lane_base + 64 + 16 * gq, z0);
        if (MODE == kBwdDt) tc::tmem_ld16(lane_base + 128 + 16 * gq, z1);
        const uint4 d0 = *reinterpret_cast<const uint4*>(st + oSdy + chunk_off(i, 2 * gq));
        const uint4 d1 = *reinterpret_cast<const uint4*>(st + oSdy + chunk_off(i, 2 * gq + 1));
        const uint32_t dyw[8] = {d0.x, d0.y, d0.z, d0.w, d1.x, d1.y, d1.z, d1.w};
        uint32_t xw[8];
        if (MODE == kBwdDt) {
          const uint4 a0 = *reinterpret_cast<const uint4*>(st + oSx + chunk_off(i, 2 * gq));
          const uint4 a1 = *reinterpret_cast<const uint4*>(st + oSx + chunk_off(i, 2 * gq + 1));
          xw[0] = a0.x; xw[1] = a0.y; xw[2] = a0.z; xw[3] = a0.w;
          xw[4] = a1.x; xw[5] = a1.y; xw[6] = a1.z; xw[7] = a1.w;
        }
        tc::tmem_wait_ld();
        uint32_t o[8];
#pragma unroll
        for (int kk = 0; kk < 16; kk += 4) {
          const int pc = 16 * gq + kk;
          const float4 gn = *reinterpret_cast<const float4*>(Gn + pc);
          const float4 sn = *reinterpret_cast<const float4*>(s_Sin + pc);
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const int q2 = kk + 2 * hh;
            const float2 gnv = hh ? make_float2(gn.z, gn.w) : make_float2(gn.x, gn.y);
            const float2 snv = hh ? make_float2(sn.z, sn.w) : make_float2(sn.x, sn.y);
            const float2 G = f2_fma(f2, gnv, f2_add(make_float2(dg[q2], dg[q2 + 1]), cvt_pair<bf16>(dyw[q2 / 2])));
            float2 zl = make_float2(z0[q2], z0[q2 + 1]);
            if (MODE == kBwdDt) zl = f2_add(zl, make_float2(z1[q2], z1[q2 + 1]));
            const float2 Zs = f2_fma(e2, snv, zl);
            dl2 = f2_fma(G, Zs, dl2);
            float2 dxv = G;
            if (MODE == kBwdDt) {
              xs2 = f2_fma(G, cvt_pair<bf16>(xw[q2 / 2]), xs2);
              dxv = f2_mul(w2, G);
            }
            o[q2 / 2] = pack_pair<bf16>(dxv);
          }
        }
        *reinterpret_cast<uint4*>(smem + oDx + chunk_off(i, 2 * gq)) = make_uint4(o[0], o[1], o[2], o[3]);
        *reinterpret_cast<uint4*>(smem + oDx + chunk_off(i, 2 * gq + 1)) = make_uint4(o[4], o[5], o[6], o[7]);
      }
      // the last token's extra gradient, added to the rounded dx as the reference does
      if (p.d_last != nullptr && t0 + i == p.L - 1) {
        const float* dlv = p.d_last + static_cast<size_t>(bh) * BP;
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
          uint4* q4 = reinterpret_cast<uint4*>(smem + oDx + chunk_off(i, cc));
          uint4 v = *q4;
          uint32_t* vw = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
          for (int m = 0; m < 4; ++m) {
            const float2 a = cvt_pair<bf16>(vw[m]);
            vw[m] = pack_pair<bf16>(make_float2(a.x + dlv[8 * cc + 2 * m], a.y + dlv[8 * cc + 2 * m + 1]));
          }
          *q4 = v;
        }
      }
      const float dl = dl2.x + dl2.y;
      if (MODE == kBwdDt) {
        const float Ah = *reinterpret_cast<const float*>(st + oSA);
        if (valid) p.ddt[(static_cast<size_t>(b) * p.L + t0 + i) * p.H + h] = (xs2.x + xs2.y) + Ah * dl;
        float dap = w * dl;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) dap += __shfl_xor_sync(FULL, dap, o);
        if (lane == 0) ws.partial[((static_cast<size_t>(h) * p.nc + c) * p.B + b) * 4 + ew] = dap;
      } else {
        if (valid) p.dl[static_cast<size_t>(bh) * p.L + t0 + i] = dl;
      }
      fence_proxy_async_smem();  // dx rows, for the TMA store
      tc::fence_before_sync();
      named_sync(kBarEpi, NET);
      if (et == 0) {
        tma_store_4d(&tm_dx, smem + oDx, 0, h, t0, b);
        bulk_commit();
        mbar_arrive(&tmem_empty[kb]);  // accumulator set kb and its cs / w are free
        mbar_arrive(&vec_empty[kb]);   // so is the arriving-gradient slot
        mbar_arrive(&empty[s]);        // and the stage: dx went to the staging buffer
      }
    }
    if (et == 0) bulk_wait_all();
    named_sync(kBarEpi, NET);
    if (et == 0) *s_last = count_cta_done(ws) ? 1u : 0u;
    named_sync(kBarEpi, NET);
    if (*s_last) {
      if (MODE == kBwdDt) {
        // dA[h]: the sum of head h's nc * B * 4 partials, in a fixed order
        __threadfence();
        const int n2 = p.nc * p.B * 4 / 2;
        for (int hh = ew; hh < p.H; hh += 4) {
          const float2* part = reinterpret_cast<const float2*>(ws.partial + static_cast<size_t>(hh) * p.nc * p.B * 4);
          float2 acc = make_float2(0.f, 0.f);
          int q = lane;
          for (; q + 7 * 32 < n2; q += 8 * 32) {
            float2 v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) v[u] = __ldcg(part + q + u * 32);
#pragma unroll
            for (int u = 0; u < 8; ++u) acc = f2_add(acc, v[u]);
          }
          for (; q < n2; q += 32) acc = f2_add(acc, __ldcg(part + q));
          float a = acc.x + acc.y;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(FULL, a, o);
          if (lane == 0) p.dA_out[hh] = a;
        }
        named_sync(kBarEpi, NET);
      }
      finish_launch(ws, epoch, total, et, NET, kBarEpi);
    }
  }
  // builders and epilogue meet before the tensor memory is released
  tc::fence_before_sync();
  named_sync(kBarBoth, NBT + NET);
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tb, kCols);
  }
}

}  // namespace ematc


// Launch the tensor-core backward when it applies: bf16, headdim 64,
// 128-token chunks, dx requested.  Returns 1 when the case is not covered
// (the caller runs the CUDA-core kernel), 0 when launched, -3 when a tensor
// map could not be encoded, otherwise a cudaError_t.
int bwd_tc_launch(const BwdLaunch& l, int dtype, const void* x, const int64_t xs[3], const void* dy,
                  const int64_t dys[3], void* dx, const int64_t dxs[3]) {
  using namespace ematc;
  const BwdParams& p = l.params;
  if (dtype != EMA_DTYPE_BF16 || p.P != BP || l.chunk != Q || p.dx == nullptr) return 1;
  if (l.mode != kBwdDt && l.mode != kBwdCumsum) return 1;
  CUtensorMap mx, mdy, mdx;
  const uint64_t dims[4] = {static_cast<uint64_t>(p.P), static_cast<uint64_t>(p.H), static_cast<uint64_t>(p.L),
                            static_cast<uint64_t>(p.B)};
  const uint32_t box[4] = {64u, 1u, static_cast<uint32_t>(Q), 1u};
  auto enc = [&](CUtensorMap* m, const void* ptr, const int64_t st[3]) {
    const uint64_t sb[3] = {static_cast<uint64_t>(st[2]) * 2u, static_cast<uint64_t>(st[1]) * 2u,
                            static_cast<uint64_t>(st[0]) * 2u};
    return encode_map(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, ptr, dims, sb, box, true);
  };
  if (enc(&mx, x, xs) || enc(&mdy, dy, dys) || enc(&mdx, dx, dxs)) return -3;
  static unsigned long long mask_dt = 0, mask_cs = 0;
  const unsigned grid = static_cast<unsigned>(l.tiles < l.num_sms ? l.tiles : l.num_sms);
  if (l.mode == kBwdDt) {
    auto fn = ema_bwd_tc_kernel<kBwdDt>;
    int e = ensure_smem_attr(reinterpret_cast<const void*>(fn), kSmemAlloc, &mask_dt);
    if (e) return e;
    fn<<<grid, NT, kSmemAlloc, l.stream>>>(mx, mdy, mdx, p);
  } else {
    auto fn = ema_bwd_tc_kernel<kBwdCumsum>;
    int e = ensure_smem_attr(reinterpret_cast<const void*>(fn), kSmemAlloc, &mask_cs);
    if (e) return e;
    fn<<<grid, NT, kSmemAlloc, l.stream>>>(mx, mdy, mdx, p);
  }
  return static_cast<int>(cudaGetLastError());
}

}  // namespace emab
