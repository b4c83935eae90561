// EMA chunked scan, forward, on the 5th-generation tensor cores (tcgen05 +
// tensor memory), for sm_100a: dt form, bf16 x / y, headdim 64, 128-token
// tiles.
//
// Same work units, ticket order and decoupled look-back as the CUDA-core
// forward (ema_scan_kernels.cuh); the tile's arithmetic differs.  With cs_t
// the inclusive within-tile cumsum of dt_t A_h and the lower-triangular decay
// matrix (diagonal included)
//
//   L[i][j] = exp(cs_i - cs_j)   for j <= i,   0 otherwise,
//
// the recurrence z_t = exp(dt_t A_h) z_{t-1} + dt_t x_t over a tile becomes
//
//   y = L X + exp(cs) Sin          (X = dt x; Sin: the state entering the tile)
//
// one 128 x 64 x 128 MMA per tile.  L and X enter the MMA rounded once to
// bf16 (round to nearest), as the reference's forward rounds its decay matrix
// before tl.dot (kernels/forward/ema_ssd_fwd.py:361-368); the sums are fp32.
// The tile's end state from zero -- the look-back aggregate, and so every
// state handed to the next tile and saved for the backward -- is summed on
// the CUDA cores in fp32 from x (sum_j exp(cs_end - cs_j) dt_j x_j), so the
// chunk states match the CUDA-core kernel's; only y carries the bf16
// rounding.  An element of L is exp(cs_i - cs_g) exp(cs_g - cs_j) for the
// key's 16-key group g (cs_g: the group's first key), or one exp where the
// group's cumsum spans more than kWideSpan.
//
// Warp roles (one CTA per SM; tiles flow builder -> MMA -> epilogue):
//   warps 0-7  builders: the tile's cumsum and key factors (warps 0-3, one
//              token per thread), the fp32 end state from zero (published as
//              the look-back aggregate at once), then L (rows i and 127 - i
//              per thread quad) and X (a thread pair per token row), written
//              once the MMA of the previous tile has read L and X;
//   warps 8-11 epilogue: the inclusive record and the chunk start state as
//              soon as the incoming state is known, then thread i reads lane
//              i of the accumulator, adds exp(cs_i) Sin and stages the y row;
//              one TMA store per tile;
//   warp 12    producer (TMA ring, as the CUDA-core kernel);
//   warp 13    look-back warp (the state entering each tile);
//   warp 14    MMA issue, into one of two tensor-memory accumulators.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "ema_scan_dispatch.h"
#include "ema_ssd_b200.h"
#include "tc_common.cuh"

namespace emab {
namespace ematcf {

using bf16 = __nv_bfloat16;
using tc::chunk_off;
using tc::group_wait;

constexpr int Q = 128;             // tokens per tile
constexpr int BP = 64;             // channels per tile (headdim)
constexpr int NBT = 256;           // builder threads (warps 0-7)
constexpr int NET = 128;           // epilogue threads (warps 8-11): thread i owns token i
constexpr int kProdWarp = 12, kLbWarp = 13, kMmaWarp = 14;
constexpr int NT = 480;
constexpr int S = 4;               // ring stages
constexpr int kTile = Q * BP * 2;  // one 128-row x 128-byte swizzled bf16 tile
constexpr float kWideSpan = 60.f;
constexpr int kBarBuild = 1, kBarEpi = 2, kBarBoth = 3;  // named barriers

// ring stage: x | raw dt[Q] | A_h
constexpr int oSx = 0;
constexpr int oSraw = kTile;
constexpr int oSA = oSraw + Q * 4;
constexpr int kStage = align_up(oSA + 16, 1024);
// operand and staging buffers after the ring (1024-byte aligned)
constexpr int oLh = S * kStage;       // L: 2 key regions of [128 rows x 64 bf16]
constexpr int oXh = oLh + 2 * kTile;  // X [128 tokens x 64 channels]
constexpr int oY = oXh + kTile;       // y staging for the TMA store
constexpr int oCs = oY + kTile;       // float[2][Q]   cs per accumulator set
constexpr int oW = oCs + 2 * Q * 4;   // float[Q]      dt (0 past the sequence end)
constexpr int oFw = oW + Q * 4;       // float[Q]      exp(cs_end - cs_j) dt_j
constexpr int oV = oFw + Q * 4;       // float[Q]      key factors exp(cs_g - cs_j)
constexpr int oRef = oV + Q * 4;      // float[8]      cs_g per key group
constexpr int oWsum = oRef + 32;      // float[4]      per-warp scan totals
constexpr int oWide = oWsum + 16;     // u32[4]        per-warp wide-group bits
constexpr int oAggP = oWide + 16;     // float[4][BP]  end-state partials by token quarter
constexpr int oAgg = oAggP + 4 * BP * 4;  // float[2][BP] the tile's end state from zero, per set
constexpr int oSin = oAgg + 2 * BP * 4;   // float[2][BP] from the look-back warp
constexpr int oETile = oSin + 2 * BP * 4;                          // int[2]: tile per set (-1: end)
constexpr int oEInfo = align_up(oETile + 8, 16);                   // TileInfo[2] per set
constexpr int oTile = oEInfo + 2 * static_cast<int>(sizeof(TileInfo));  // int[S]
constexpr int oInfo = align_up(oTile + S * 4, 16);                 // TileInfo[S]
constexpr int oBar = oInfo + S * static_cast<int>(sizeof(TileInfo));
// barriers: full, empty, tid_full [S]; vec_full, vec_empty, mma_done, tmem_empty, agg_ready [2]; op_ready
constexpr int oMisc = oBar + (3 * S + 11) * 8;  // u32: taddr, fail (builders), fail (epilogue), epoch, last
constexpr int kSmem = oMisc + 32;
constexpr int kSmemAlloc = kSmem + 1024;  // room to align the base to 1024 bytes
static_assert(kSmemAlloc <= kSmemPerCtaMax, "shared memory");
// tensor memory: two accumulator sets of 64 columns (y = L X of one tile)
constexpr uint32_t kCols = 128;
constexpr uint32_t kSetCols = 64;

// 8 floats -> 8 bf16 (round to nearest), one 16-byte chunk.
__device__ __forceinline__ uint4 pack8(const float (&v)[8]) {
  return make_uint4(pack_pair<bf16>(make_float2(v[0], v[1])), pack_pair<bf16>(make_float2(v[2], v[3])),
                    pack_pair<bf16>(make_float2(v[4], v[5])), pack_pair<bf16>(make_float2(v[6], v[7])));
}

__global__ void __launch_bounds__(NT, 1)
    ema_fwd_tc_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_y,
                      const FwdParams p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  float* s_cs2 = reinterpret_cast<float*>(smem + oCs);
  float* s_w = reinterpret_cast<float*>(smem + oW);
  float* s_fw = reinterpret_cast<float*>(smem + oFw);
  float* s_v = reinterpret_cast<float*>(smem + oV);
  float* s_ref = reinterpret_cast<float*>(smem + oRef);
  float* s_wsum = reinterpret_cast<float*>(smem + oWsum);
  uint32_t* s_wide = reinterpret_cast<uint32_t*>(smem + oWide);
  float* s_aggp = reinterpret_cast<float*>(smem + oAggP);
  float* s_agg2 = reinterpret_cast<float*>(smem + oAgg);
  float* s_Sin2 = reinterpret_cast<float*>(smem + oSin);
  int* s_etile = reinterpret_cast<int*>(smem + oETile);
  TileInfo* s_einfo = reinterpret_cast<TileInfo*>(smem + oEInfo);
  int* s_tile = reinterpret_cast<int*>(smem + oTile);
  TileInfo* s_info = reinterpret_cast<TileInfo*>(smem + oInfo);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + oBar);
  uint64_t* empty = full + S;
  uint64_t* tid_full = empty + S;
  uint64_t* vec_full = tid_full + S;
  uint64_t* vec_empty = vec_full + 2;
  uint64_t* mma_done = vec_empty + 2;
  uint64_t* tmem_empty = mma_done + 2;
  uint64_t* agg_ready = tmem_empty + 2;
  uint64_t* op_ready = agg_ready + 2;
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
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 33);  // producer lane 0 (expect_tx) + 32 cp.async arrivals
      mbar_init(&empty[s], 2);  // builder thread 0 + the look-back warp
      mbar_init(&tid_full[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&vec_full[i], 1);    // look-back lane 0
      mbar_init(&vec_empty[i], 1);   // epilogue thread 0
      mbar_init(&mma_done[i], 1);    // tcgen05.commit
      mbar_init(&tmem_empty[i], 1);  // epilogue thread 0
      mbar_init(&agg_ready[i], 1);   // builder thread 0
    }
    mbar_init(op_ready, 1);  // builder thread 0
    fence_mbar_init();
  }
  // L's strict upper triangle is never written: zero the L buffer once
  for (int o = tid * 16; o < 2 * kTile; o += NT * 16)
    *reinterpret_cast<uint4*>(smem + oLh + o) = make_uint4(0u, 0u, 0u, 0u);
  fence_proxy_async_smem();
  if (warp == 0) {
    tc::tmem_alloc(s_taddr, kCols);
    tc::tmem_relinquish();
  }
  grid_dep_wait();  // the previous kernel's writes (dt rows, workspace reset) are visible from here
  grid_dep_release();
  if (tid == 0) *s_epoch = ld_volatile_u32(&ws.hdr[kHdrEpoch]) & kEpochMask;
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
    if (lane == 0) tma_prefetch_desc(&tm_x);
    producer_loop<S>(full, empty, tid_full, s_tile, ws.hdr, total, lane, [&](int s, int ticket) {
      const int c = fast_div(ticket, p.div_bh), bh = ticket - c * BH;
      const int b = fast_div(bh, p.div_h), h = bh - b * p.H, t0 = c * Q;
      unsigned char* st = smem + s * kStage;
      float* raw = reinterpret_cast<float*>(st + oSraw);
      const int n = min(Q, p.L - t0);
      const float* src = p.dt_rows ? p.dt + static_cast<size_t>(bh) * p.L + t0
                                   : p.dt + (static_cast<size_t>(b) * p.L + t0) * p.H + h;
      const uint32_t bulk = p.dt_rows ? row_bulk_bytes(src, n) : 0u;
      if (lane == 0) {
        s_tile[s] = ticket;
        s_info[s] = TileInfo{c, b, h, t0, bh, 0, 0};
        mbar_arrive_expect_tx(&full[s], kTile + bulk);
        tma_load_4d(st + oSx, &tm_x, &full[s], 0, h, t0, b);
      }
      if (p.dt_rows) {
        load_row(raw, src, n, bulk, &full[s], lane);
      } else {
        gather_col(raw, src, p.H, n, lane);
      }
      if (lane == 0) cp_async_4(raw + Q, p.A + h);
    }, [&](int ticket) {
      const int c = fast_div(ticket, p.div_bh), bh = ticket - c * BH;
      const int b = fast_div(bh, p.div_h), h = bh - b * p.H;
      tma_prefetch_l2_4d(&tm_x, 0, h, c * Q, b);
    });
    return;
  }
  if (warp == kLbWarp) {
    // ------------------------------ look-back ------------------------------
    lookback_loop<S, BP>(tid_full, s_tile, empty, vec_full, vec_empty, s_Sin2, status, lane,
                         [](int, int) { return true; },
                         [&](int tile, float(&run)[BP / 32]) {
                           const int c = fast_div(tile, p.div_bh), bh = tile - c * BH;
                           float rdec = 1.f;
                           bool at_start = true;
                           if (c > 0) {
                             at_start = lookback_warp<BP>(ws, tag, bh, BH, c, -1, p.nc, lane, run, rdec);
                           } else {
#pragma unroll
                             for (int q = 0; q < BP / 32; ++q) run[q] = 0.f;
                           }
                           if (at_start && p.init != nullptr) {
                             const float* iv = p.init + static_cast<size_t>(bh) * BP;
#pragma unroll
                             for (int q = 0; q < BP / 32; ++q)
                               run[q] = fmaf(rdec, iv[lane * (BP / 32) + q], run[q]);
                           }
                         });
    return;
  }

  if (warp == kMmaWarp) {
    // ------------------------------ MMA issue ------------------------------
    const uint32_t sb = smem_u32(smem);
    const uint64_t dKL = tc::smem_desc_sw128(sb + oLh, 16, 1024);     // L, K-major (M = query row, K = key)
    const uint64_t dNX = tc::smem_desc_sw128(sb + oXh, kTile, 1024);  // X, MN-major (K = token, N = channel)
    const uint32_t id64 = tc::idesc_bf16(128, 64, false, true);
    auto kstep = [](int s) { return static_cast<uint64_t>(((s >> 2) * kTile + (s & 3) * 32) >> 4); };
    auto nstep = [](int s) { return static_cast<uint64_t>((s * 2048) >> 4); };
    for (int k = 0;; ++k) {
      const int kb = k & 1;
      if (!mbar_wait_bounded(op_ready, k & 1, status)) break;
      if (s_etile[kb] < 0) break;
      if (k >= 2 && !mbar_wait_bounded(&tmem_empty[kb], ((k - 2) >> 1) & 1, status)) break;
      tc::fence_after_sync();
      if (lane == 0) {
        const uint32_t d = tb + kb * kSetCols;
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) tc::mma_bf16(d, dKL + kstep(ks), dNX + nstep(ks), id64, ks > 0);
        tc::mma_commit(&mma_done[kb]);
      }
      __syncwarp();
    }
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
      // set kb (cs, end state, tile id) is free once the epilogue of tile k - 2 is done
      if (k >= 2 && !group_wait(&tmem_empty[kb], ((k - 2) >> 1) & 1, status, warp == 0, kBarBuild, NBT, s_fail_b))
        break;
      if (tile < 0) {
        // the MMA warp must have taken op_ready's previous phase before this arrival
        if (k >= 1 && !group_wait(&mma_done[kb ^ 1], ((k - 1) >> 1) & 1, status, warp == 0, kBarBuild, NBT,
                                  s_fail_b))
          break;
        if (tid == 0) {
          s_etile[kb] = -1;
          mbar_arrive(&agg_ready[kb]);
          mbar_arrive(op_ready);
        }
        break;
      }
      unsigned char* st = smem + s * kStage;
      const float* raw = reinterpret_cast<const float*>(st + oSraw);
      const TileInfo ti = s_info[s];
      const int n = min(Q, p.L - ti.t0);
      const bool has_succ = ti.c + 1 < p.nc;

      // ---- per-token cumsum of dt A, dt, key factors (warps 0-3) ----------------
      float* csb = s_cs2 + kb * Q;
      float d = 0.f, cs = 0.f;
      if (tok) {
        const float Ah = *reinterpret_cast<const float*>(st + oSA);
        d = (i < n) ? raw[i] : 0.f;
        float v = d * Ah;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float nv = __shfl_up_sync(FULL, v, o);
          if (lane >= o) v += nv;
        }
        if (lane == 31) s_wsum[warp] = v;
        cs = v;
      }
      named_sync(kBarBuild, NBT);
      if (tok) {
#pragma unroll
        for (int ww = 0; ww < 3; ++ww)
          if (ww < warp) cs += s_wsum[ww];
        const float cref = __shfl_sync(FULL, cs, lane & ~15);
        float span = fabsf(cref - cs);
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) span = fmaxf(span, __shfl_xor_sync(FULL, span, o));
        const bool wide = span > kWideSpan;
        csb[i] = cs;
        s_w[i] = d;
        s_v[i] = wide ? 0.f : __expf(cref - cs);
        if ((lane & 15) == 0) s_ref[i >> 4] = cref;
        const uint32_t wb = __ballot_sync(FULL, wide);
        if (lane == 0) s_wide[warp] = ((wb & 1u) | ((wb >> 15) & 2u)) << (2 * warp);
      }
      named_sync(kBarBuild, NBT);
      const float cs_end = csb[Q - 1];  // tokens past the sequence end add nothing: cs_end is the last token's
      if (tok) s_fw[i] = __expf(cs_end - cs) * d;
      named_sync(kBarBuild, NBT);

      // ---- the tile's end state from zero, fp32: sum_j exp(cs_end - cs_j) dt_j x_j ----
      {
        const int ch = tid & (BP - 1), qq = tid >> 6;
        const unsigned char* xcol = st + oSx + 2 * (ch & 7);
        float acc = 0.f;
#pragma unroll 8
        for (int u = 0; u < Q / 4; ++u) {
          const int j = (Q / 4) * qq + u;
          const bf16 xv = *reinterpret_cast<const bf16*>(xcol + chunk_off(j, ch >> 3));
          acc = fmaf(s_fw[j], __bfloat162float(xv), acc);
        }
        s_aggp[qq * BP + ch] = acc;
      }
      named_sync(kBarBuild, NBT);
      if (tid < BP) {
        const float agg = (s_aggp[tid] + s_aggp[BP + tid]) + (s_aggp[2 * BP + tid] + s_aggp[3 * BP + tid]);
        s_agg2[kb * BP + tid] = agg;
        if (ti.c > 0 && has_succ) {  // mid-chain: later tiles may combine it before this tile's inclusive lands
          uint64_t* rec = ws.agg + static_cast<size_t>(tile) * (BP + 1);
          st_relaxed_u64(rec + tid, tag_word(agg, tag));
          if (tid == 0) st_relaxed_u64(rec + BP, tag_word(__expf(cs_end), tag));
        }
      }
      if (tid == 0) {
        s_etile[kb] = tile;
        s_einfo[kb] = ti;
      }
      named_sync(kBarBuild, NBT);
      if (tid == 0) mbar_arrive(&agg_ready[kb]);
      const uint32_t wmask = s_wide[0] | s_wide[1] | s_wide[2] | s_wide[3];

      // ---- L and X, once the MMA of tile k - 1 has read them ---------------------------
      if (k >= 1 && !group_wait(&mma_done[kb ^ 1], ((k - 1) >> 1) & 1, status, warp == 0, kBarBuild, NBT, s_fail_b))
        break;
      // a quad of threads builds rows pr and 127 - pr: 17 chunks of 8 keys, at most 5 each
      {
        const int pr = tid >> 2, sub = tid & 3;
        const int ra = pr, rb = Q - 1 - pr;
        const int na = (ra >> 3) + 1;
        const int nab = na + (rb >> 3) + 1;
        const float csa = csb[ra], csr = csb[rb];
#pragma unroll
        for (int q = 0; q < 5; ++q) {
          const int idx = sub + 4 * q;
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
              if (j0 + kk > ri) v8[kk] = 0.f;
            *reinterpret_cast<uint4*>(smem + oLh + (j0 >> 6) * kTile + chunk_off(ri, (j0 & 63) >> 3)) = pack8(v8);
          }
        }
      }
      // X = dt x: a thread pair per token row, four 8-channel chunks each
      {
        const int xr = tid >> 1, c0 = 4 * (tid & 1);
        const float wx = s_w[xr];
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
          *reinterpret_cast<uint4*>(smem + oXh + chunk_off(xr, cc)) = pack8(v8);
        }
      }
      fence_proxy_async_smem();
      tc::fence_before_sync();
      named_sync(kBarBuild, NBT);
      if (tid == 0) {
        mbar_arrive(op_ready);
        mbar_arrive(&empty[s]);  // the builders were the stage's only compute readers
      }
    }
  } else {
    // ------------------------------ epilogue ------------------------------
    const int et = tid - NBT;  // 0..127: token row of the tile = tensor-memory lane
    const int ew = warp - 8;   // = warp % 4: the lane quarter this warp may read
    const int i = et;
    for (int k = 0;; ++k) {
      const int kb = k & 1;
      if (!group_wait(&agg_ready[kb], (k >> 1) & 1, status, ew == 0, kBarEpi, NET, s_fail_e)) break;
      const int tile = s_etile[kb];
      if (tile < 0) break;
      const TileInfo ti = s_einfo[kb];
      const int c = ti.c, b = ti.b, h = ti.h, t0 = ti.t0, bh = ti.bh;
      const float* csb = s_cs2 + kb * Q;
      const float cs_end = csb[Q - 1];

      // ---- the incoming state: inclusive record, chunk start state ---------------------
      if (!group_wait(&vec_full[kb], (k >> 1) & 1, status, ew == 0, kBarEpi, NET, s_fail_e)) break;
      const float* Sin = s_Sin2 + kb * BP;
      if (et < BP) {
        const float incl = fmaf(__expf(cs_end), Sin[et], s_agg2[kb * BP + et]);  // state at the tile end
        if (c + 1 < p.nc) {
          st_relaxed_u64(ws.incl + static_cast<size_t>(tile) * BP + et, tag_word(incl, tag));
        } else if (p.final_state != nullptr) {
          p.final_state[static_cast<size_t>(bh) * BP + et] = incl;
        }
        if (p.states != nullptr)
          p.states[b * p.st_b + static_cast<long long>(c) * p.st_c + h * p.st_h + et * p.st_p] = Sin[et];
      }

      // ---- y = L X + exp(cs) Sin into the staging tile ------------------------------------
      if (!group_wait(&mma_done[kb], (k >> 1) & 1, status, ew == 0, kBarEpi, NET, s_fail_e)) break;
      tc::fence_after_sync();
      if (et == 0) bulk_wait_read<0>();  // the previous tile's store has read the staging tile
      named_sync(kBarEpi, NET);
      const uint32_t lane_base = tc::tmem_at(tb, 32 * ew, kb * kSetCols);
      const float2 e2 = f2_bcast(__expf(csb[i]));
#pragma unroll 1
      for (int gq = 0; gq < 4; ++gq) {
        float acc[16];
        tc::tmem_ld16(lane_base + 16 * gq, acc);
        tc::tmem_wait_ld();
        uint32_t o[8];
#pragma unroll
        for (int kk = 0; kk < 16; kk += 4) {
          const float4 sn = *reinterpret_cast<const float4*>(Sin + 16 * gq + kk);
          o[kk / 2] = pack_pair<bf16>(f2_fma(e2, make_float2(sn.x, sn.y), make_float2(acc[kk], acc[kk + 1])));
          o[kk / 2 + 1] = pack_pair<bf16>(f2_fma(e2, make_float2(sn.z, sn.w), make_float2(acc[kk + 2], acc[kk + 3])));
        }
        *reinterpret_cast<uint4*>(smem + oY + chunk_off(i, 2 * gq)) = make_uint4(o[0], o[1], o[2], o[3]);
        *reinterpret_cast<uint4*>(smem + oY + chunk_off(i, 2 * gq + 1)) = make_uint4(o[4], o[5], o[6], o[7]);
      }
      fence_proxy_async_smem();  // y rows, for the TMA store
      tc::fence_before_sync();
      named_sync(kBarEpi, NET);
      if (et == 0) {
        tma_store_4d(&tm_y, smem + oY, 0, h, t0, b);  // rows past the sequence end are clipped
        bulk_commit();
        mbar_arrive(&tmem_empty[kb]);  // accumulator set kb and its cs / end state are free
        mbar_arrive(&vec_empty[kb]);   // so is the incoming-state slot
      }
    }
    if (et == 0) bulk_wait_all();
    named_sync(kBarEpi, NET);
    if (et == 0) *s_last = count_cta_done(ws) ? 1u : 0u;
    named_sync(kBarEpi, NET);
    if (*s_last) finish_launch(ws, epoch, total, et, NET, kBarEpi);
  }
  // builders and epilogue meet before the tensor memory is released
  tc::fence_before_sync();
  named_sync(kBarBoth, NBT + NET);
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tb, kCols);
  }
}

}  // namespace ematcf

// Launch the tensor-core forward when it applies: dt form, bf16, headdim 64,
// 128-token chunks, y requested, no seq_idx and no mid-chunk states.
// Returns 1 when the case is not covered (the caller runs the CUDA-core
// kernel), 0 when launched, -3 when a tensor map could not be encoded
// (message set), otherwise a cudaError_t.
int fwd_tc_launch(const FwdLaunch& l, int dtype, const void* x, const int64_t xs[3], void* y,
                  const int64_t ys[3]) {
  using namespace ematcf;
  const FwdParams& p = l.params;
  if (dtype != EMA_DTYPE_BF16 || p.P != BP || l.chunk != Q || l.mode != kFwdDt || l.seq) return 1;
  if (y == nullptr || p.mid_states != nullptr) return 1;
  CUtensorMap mx, my;
  const uint64_t dims[4] = {static_cast<uint64_t>(p.P), static_cast<uint64_t>(p.H), static_cast<uint64_t>(p.L),
                            static_cast<uint64_t>(p.B)};
  const uint32_t box[4] = {64u, 1u, static_cast<uint32_t>(Q), 1u};
  auto enc = [&](CUtensorMap* m, const void* ptr, const int64_t st[3]) {
    const uint64_t sb[3] = {static_cast<uint64_t>(st[2]) * 2u, static_cast<uint64_t>(st[1]) * 2u,
                            static_cast<uint64_t>(st[0]) * 2u};
    return encode_map(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, ptr, dims, sb, box, true);
  };
  if (enc(&mx, x, xs) || enc(&my, y, ys)) return -3;
  static unsigned long long mask = 0;
  const int e = ensure_smem_attr(reinterpret_cast<const void*>(ema_fwd_tc_kernel), kSmemAlloc, &mask);
  if (e) return e;
  const unsigned grid = static_cast<unsigned>(l.tiles < l.num_sms ? l.tiles : l.num_sms);
  return static_cast<int>(
      launch_programmatic(ema_fwd_tc_kernel, dim3(grid), dim3(NT), kSmemAlloc, l.stream, mx, my, p));
}

}  // namespace emab
