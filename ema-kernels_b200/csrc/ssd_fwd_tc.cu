// Mamba-2 SSD chunked scan, forward, on the 5th-generation tensor cores
// (tcgen05 + tensor memory), for sm_100a.
//
//   s_t = exp(dt_t A_h) s_{t-1} + dt_t x_t B_t^T   (headdim 64 x dstate 128 per head)
//   y_t = s_t C_t + D_h x_t
//
// One CTA per (batch, pair of heads of one group) walks the sequence in
// 128-token chunks.  Per chunk, with cs_h the within-chunk cumsum of dt A_h:
//
//   CB     = C B^T                                     128x128x128, shared by both heads
//   M_h    = CB o exp(cs_h,i - cs_h,j) dt_h,j (j <= i)  (epilogue, bf16 into shared memory)
//   Y_h    = M_h x_h                                   128x64x128 per head
//   Yi_h   = C S_h^T                                   128x64x128 per head (S_h: state entering the chunk, bf16)
//   y_h    = Y_h + exp(cs_h,i) Yi_h + D_h x_h           (epilogue)
//   dS     = [x_w,h0 ; x_w,h1]^T B                     128x128 per token half, both heads stacked as M
//   S      = exp(cs_h,end) S + dS                       (epilogue; S fp32 in tensor memory)
//
// with x_w,h,j = exp(cs_h,half end - cs_h,j) dt_h,j x_h,j.  The state GEMM runs
// per 64-token half so that the state at every 64-token boundary -- the
// chunk_states the backward reads -- is exact.  Thread 0 issues the TMA loads,
// the MMAs and the TMA stores: y is written over the consumed x tile and the
// saved states are staged (fp32, swizzled) in the M buffer once its MMA is
// done, so no epilogue thread stores to global memory.  All sixteen warps run
// the epilogues (warp w owns tensor-memory
// lanes 32 (w % 4) .. + 31 and a quarter of the columns).  Operands are rounded to
// bf16 at the MMA inputs only, as in the mma.sync kernels (ssd_kernels.cu):
// the decay factors, scans, accumulators and the state stay fp32.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>

#include "ema_scan_dispatch.h"
#include "ssd_b200.h"
#include "tc_common.cuh"

namespace emab {
void set_last_error(const char* msg);

namespace ssdtc {

using bf16 = __nv_bfloat16;

constexpr int Q = 128;       // tokens per chunk
constexpr int QH = 64;       // tokens per state half (the saved-state granularity)
constexpr int P = 64;        // headdim
constexpr int N = 128;       // dstate
constexpr int NW = 16;       // warps: four per tensor-memory lane quarter
constexpr int NT = NW * 32;
constexpr int CWS = NW / 4;          // warps sharing a lane quarter (they split the columns)
constexpr int CPW = 128 / CWS;       // columns per warp of a 128-column epilogue
constexpr int GPW = CPW / 16;        // 16-column groups per warp
constexpr int XPT = 64 / (NT / 256); // x_w channels per thread
constexpr int kReg = 128 * 128;  // one 128-row x 128-byte swizzled region
constexpr int kReg64 = 64 * 128;  // one 64-row region

// shared-memory layout (from a 1024-byte-aligned base)
constexpr int oX = 0;                   // x: 2 heads x [128 tokens x 64 channels]
constexpr int oB = oX + 2 * kReg;       // B: 2 dstate halves x [128 tokens x 64]
constexpr int oC = oB + 2 * kReg;       // C: the same
constexpr int oM = oC + 2 * kReg;       // M: 2 heads x 2 key halves x [128 queries x 64 keys]
constexpr int oXw = oM + 4 * kReg;      // x_w: 2 heads x [128 tokens x 64 channels]
constexpr int oS = oXw + 2 * kReg;      // S (bf16): 2 heads x 2 dstate halves x [64 channels x 64]
constexpr int oCs = oS + 4 * kReg64;    // float cs[2][128]
constexpr int oDt = oCs + 2 * Q * 4;    // float dt[2][128], then the key factors (see the cumsum step)
constexpr int oBar = oDt + 2 * Q * 4;   // full, mma (u64); taddr, fail, wide[2] (u32)
constexpr int kSmem = oBar + 32;
// exp(cs_i - cs_j) is factored per 16-key group g as exp(cs_i - cs_g) exp(cs_g - cs_j)
// (cs_g: the group's first key) unless the cumsum spans more than this inside the group
constexpr float kWideSpan = 60.f;

// tensor-memory columns
constexpr uint32_t cCB = 0;    // C B^T, then the state increment dS
constexpr uint32_t cY = 128;   // Y_h at cY + 64 h
constexpr uint32_t cYi = 256;  // Yi_h at cYi + 64 h
constexpr uint32_t cS = 384;   // fp32 state: lane (h, p) = 64 h + p, column n
constexpr uint32_t kCols = 512;

constexpr uint32_t kStatusAlign = 0x100u;  // (kStatusTmaTimeout from a bounded wait: 2)

struct Params {
  int B, L, H, G, ncq, nc64;
  const float* dt;
  const float* A;
  const float* D;
  const float* s0;
  bf16* y;
  long long sy_b, sy_l, sy_h;
  float* chunk_states;  // (B, nc64, H, P, N) or null
  float* s_final;       // (B, H, P, N) or null
  uint32_t* status;
  DtMap dtm;            // dt <- clamp(softplus(dt + bias)), applied as dt lands in shared memory
};

__device__ uint32_t g_status;

__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, uint32_t* status) {
  return mbar_wait_bounded(bar, parity, status);
}

using tc::st_sw16;
using tc::ld_sw16;

// Stage 16 floats of state row `row` (columns n0 .. n0 + 15) into four
// 128-row x 32-float regions (128-byte swizzle), the layout a TMA store with
// 32-float boxes reads.
__device__ __forceinline__ void stage_f32(unsigned char* base, int row, int n0, const float (&v)[16]) {
  unsigned char* region = base + (n0 / 32) * kReg;
#pragma unroll
  for (int k4 = 0; k4 < 4; ++k4) {
    const int c = (n0 % 32) / 4 + k4;  // 16-byte chunk of the 128-byte row
    *reinterpret_cast<float4*>(region + row * 128 + ((c ^ (row & 7)) << 4)) =
        make_float4(v[4 * k4], v[4 * k4 + 1], v[4 * k4 + 2], v[4 * k4 + 3]);
  }
}

template <bool SAVE>
__global__ void __launch_bounds__(NT, 1)
    ssd_fwd_tc_kernel(const __grid_constant__ CUtensorMap mx, const __grid_constant__ CUtensorMap mb,
                      const __grid_constant__ CUtensorMap mc, const __grid_constant__ CUtensorMap my,
                      const __grid_constant__ CUtensorMap ms, const Params p) {
  extern __shared__ __align__(1024) unsigned char smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint32_t* status = p.status;
  if ((smem_u32(smem) & 1023u) != 0u) {  // the swizzled tiles need a 1024-byte-aligned base
    if (tid == 0) atomicOr(status, kStatusAlign);
    return;
  }
  const int h0 = 2 * blockIdx.x, b = blockIdx.y;
  const int grp = h0 / (p.H / p.G);
  const int q = warp & 3, cw = warp >> 2;  // lane quarter, column share
  float* s_cs = reinterpret_cast<float*>(smem + oCs);
  float* s_dt = reinterpret_cast<float*>(smem + oDt);
  uint64_t* bar_full = reinterpret_cast<uint64_t*>(smem + oBar);
  uint64_t* bar_mma = bar_full + 1;
  uint32_t* s_taddr = reinterpret_cast<uint32_t*>(bar_full + 2);
  volatile uint32_t* s_fail = s_taddr + 1;  // a timed-out wait, acted on together after the next barrier
  uint32_t* s_wide = s_taddr + 2;            // per head: bit g = key group g is not factored
  const uint32_t sbase = smem_u32(smem);

  if (tid == 0) {
    mbar_init(bar_full, 1);
    mbar_init(bar_mma, 1);
    *s_fail = 0u;
    fence_mbar_init();
  }
  if (warp == 0) tc::tmem_alloc(s_taddr, kCols);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tb = *s_taddr;
  uint32_t mma_phase = 0;
  // operand descriptors of the fixed shared-memory tiles; a K step or region
  // offset is added to the start-address field (bytes >> 4, no carry out of it)
  const uint64_t dKC = tc::smem_desc_sw128(sbase + oC, 16, 1024);    // C, K-major
  const uint64_t dKB = tc::smem_desc_sw128(sbase + oB, 16, 1024);    // B, K-major
  const uint64_t dKM = tc::smem_desc_sw128(sbase + oM, 16, 1024);    // M_h, K-major
  const uint64_t dKS = tc::smem_desc_sw128(sbase + oS, 16, 1024);    // S_h (bf16), K-major
  const uint64_t dNX = tc::smem_desc_sw128(sbase + oX, kReg, 1024);  // x_h, MN-major
  const uint64_t dNW = tc::smem_desc_sw128(sbase + oXw, kReg, 1024); // [x_w,h0 ; x_w,h1], MN-major
  const uint64_t dNB = tc::smem_desc_sw128(sbase + oB, kReg, 1024);  // B, MN-major
  auto kstep = [](int s) { return static_cast<uint64_t>(((s >> 2) * kReg + (s & 3) * 32) >> 4); };  // K-major
  auto nstep = [](int s) { return static_cast<uint64_t>((s * 2048) >> 4); };                         // MN-major

  auto issue_loads = [&](int cc) {
    const int t0 = cc * Q;
    mbar_arrive_expect_tx(bar_full, 6u * kReg);
    tma_load_4d(smem + oX, &mx, bar_full, 0, h0, t0, b);
    tma_load_4d(smem + oX + kReg, &mx, bar_full, 0, h0 + 1, t0, b);
    tma_load_4d(smem + oB, &mb, bar_full, 0, grp, t0, b);
    tma_load_4d(smem + oB + kReg, &mb, bar_full, 64, grp, t0, b);
    tma_load_4d(smem + oC, &mc, bar_full, 0, grp, t0, b);
    tma_load_4d(smem + oC + kReg, &mc, bar_full, 64, grp, t0, b);
  };
  // all threads: wait for the MMAs committed last, then order tensor-memory reads after them
  // the staged state of 64-token chunk k (both heads: 128 rows of 128 floats)
  auto store_state = [&](int k) {
    const int row0 = ((b * p.nc64 + k) * p.H + h0) * P;
#pragma unroll 1
    for (int r = 0; r < 4; ++r) tc::tma_store_2d(&ms, smem + oM + r * kReg, 32 * r, row0);
    bulk_commit();
  };
  auto wait_mma = [&]() {
    if (!wait_bar(bar_mma, mma_phase & 1u, status)) *s_fail = 1u;
    ++mma_phase;
    tc::fence_after_sync();
  };

  // ---- initial state: fp32 into tensor memory, bf16 into the Yi operand ----
  const int srow = 32 * q + lane;        // tensor-memory lane of this thread: (head, channel)
  const int sh = srow >> 6, sp = srow & 63;
  const size_t bh_s = static_cast<size_t>(b) * p.H + h0 + sh;
  {
#pragma unroll
    for (int g = 0; g < GPW; ++g) {
      const int n0 = CPW * cw + 16 * g;
      float v[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = (p.s0 != nullptr) ? p.s0[(bh_s * P + sp) * N + n0 + i] : 0.f;
      tc::tmem_st16(tc::tmem_at(tb, 32 * q, cS + n0), v);
      st_sw16(smem + oS + (2 * sh + n0 / 64) * kReg64, sp, n0 % 64, v);
      if (SAVE) stage_f32(smem + oM, srow, n0, v);
    }
    tc::tmem_wait_st();
  }
  fence_proxy_async_smem();
  tc::fence_before_sync();
  __syncthreads();

  if (tid == 0) {
    tma_prefetch_desc(&mx);
    tma_prefetch_desc(&mb);
    tma_prefetch_desc(&mc);
    issue_loads(0);
    if (SAVE) store_state(0);
  }

  const float A0 = p.A[h0], A1 = p.A[h0 + 1];
  // warps 0 and 1 fetch dt of head h0 + warp for a chunk into s_dt (4 tokens
  // per lane) with cp.async, so no register waits on it: the coming chunk's as
  // soon as this chunk's last reader (x_w) is done
  auto fetch_dt = [&](int tc0) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int j = 4 * lane + k, tj = tc0 + j;
      float* dst = s_dt + warp * Q + j;
      if (tj < p.L) cp_async_4(dst, p.dt + (static_cast<size_t>(b) * p.L + tj) * p.H + h0 + warp);
      else *dst = 0.f;
    }
  };
  if (warp < 2) fetch_dt(0);
  const float D0 = (p.D != nullptr) ? p.D[h0] : 0.f, D1 = (p.D != nullptr) ? p.D[h0 + 1] : 0.f;

  for (int cc = 0; cc < p.ncq; ++cc) {
    const int t0 = cc * Q;
    const int nq = min(Q, p.L - t0);
    // ---- dt and the within-chunk cumsum of dt A, one warp per head ----------
    if (warp < 2) {
      const float Ah = warp == 0 ? A0 : A1;
      float d[4], c[4];
      float run = 0.f;
      cp_async_wait_all();
      __syncwarp();
      const bool mapped = dt_map_active(p.dtm);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        d[k] = s_dt[warp * Q + 4 * lane + k];
        if (mapped && t0 + 4 * lane + k < p.L) d[k] = dt_map(p.dtm, h0 + warp, d[k], nullptr);  // padding stays 0
        run += d[k];
        c[k] = run;
      }
      float incl = run;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      const float excl = incl - run;
      float cv[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) cv[k] = Ah * (excl + c[k]);
      // key factors of the 16-token group (4 lanes): exp(cs_g - cs_j) dt_j, or dt_j
      // itself where the group's cumsum span is too wide to factor in fp32
      const float cg = __shfl_sync(0xffffffffu, cv[0], lane & ~3);
      const float ce = __shfl_sync(0xffffffffu, cv[3], lane | 3);
      const bool wide = fabsf(cg - ce) > kWideSpan;
      const uint32_t wb = __ballot_sync(0xffffffffu, wide);
      uint32_t gm = 0;
#pragma unroll
      for (int g = 0; g < 8; ++g) gm |= ((wb >> (4 * g)) & 1u) << g;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        s_cs[warp * Q + 4 * lane + k] = cv[k];
        s_dt[warp * Q + 4 * lane + k] = wide ? d[k] : __expf(cg - cv[k]) * d[k];
      }
      if (lane == 0) s_wide[warp] = gm;
    }
    if (tid == 0) bulk_wait_read_all();  // the states staged in the M buffer have been read
    if (tid == 0 && cc + 1 < p.ncq) {  // the next chunk's tiles towards L2
      const int tn = t0 + Q;
      tma_prefetch_l2_4d(&mx, 0, h0, tn, b);
      tma_prefetch_l2_4d(&mx, 0, h0 + 1, tn, b);
      tma_prefetch_l2_4d(&mb, 0, grp, tn, b);
      tma_prefetch_l2_4d(&mb, 64, grp, tn, b);
      tma_prefetch_l2_4d(&mc, 0, grp, tn, b);
      tma_prefetch_l2_4d(&mc, 64, grp, tn, b);
    }
    __syncthreads();

    // ---- CB = C B^T (committed alone), then Yi_h = C S_h^T ------------------------
    // Yi needs only C and the carried state, so it runs while the epilogue
    // builds M; the next commit covers it.
    if (tid == 0) {
      if (wait_bar(bar_full, cc & 1, status)) {
        tc::fence_after_sync();
        const uint32_t id = tc::idesc_bf16(128, 128, false, false);
        const uint32_t idi = tc::idesc_bf16(128, 64, false, false);
#pragma unroll
        for (int s = 0; s < 8; ++s) tc::mma_bf16(tb + cCB, dKC + kstep(s), dKB + kstep(s), id, s > 0);
        tc::mma_commit(bar_mma);
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const uint64_t sh = static_cast<uint64_t>((2 * hh * kReg64) >> 4);
#pragma unroll
          for (int s = 0; s < 8; ++s) {
            const uint64_t so = static_cast<uint64_t>(((s >> 2) * kReg64 + (s & 3) * 32) >> 4);
            tc::mma_bf16(tb + cYi + 64 * hh, dKC + kstep(s), dKS + sh + so, idi, s > 0);
          }
        }
      } else {
        *s_fail = 1u;
        mbar_arrive(bar_mma);  // nothing issued: release the others
      }
    }
    // the TMA tiles are read by every thread below: observe their completion too
    if (tid != 0 && !wait_bar(bar_full, cc & 1, status)) *s_fail = 1u;

    // ---- x_w (needs only x), while C B^T runs ----------------------------------------
    {
      constexpr int TPP = NT / 256;  // threads per (token, head)
      const int pr = tid / TPP, j = pr >> 1, hh = pr & 1, xc0 = (tid % TPP) * XPT;
      const int jend = SAVE ? ((j < QH) ? QH - 1 : Q - 1) : Q - 1;
      const int jref = ((s_wide[hh] >> (j >> 4)) & 1u) ? j : (j & ~15);  // s_dt: dt_j or exp(cs_g - cs_j) dt_j
      const float w = __expf(s_cs[hh * Q + jend] - s_cs[hh * Q + jref]) * s_dt[hh * Q + j];
#pragma unroll
      for (int g = 0; g < XPT / 16; ++g) {
        float xv[16];
        ld_sw16(smem + oX + hh * kReg, j, xc0 + 16 * g, xv);
#pragma unroll
        for (int k = 0; k < 16; ++k) xv[k] *= w;
        st_sw16(smem + oXw + hh * kReg, j, xc0 + 16 * g, xv);
      }
    }
    wait_mma();

    // ---- M_h (both heads) ------------------------------------------------------------
    {
      const int i = 32 * q + lane;  // query row
      const float ci0 = s_cs[i], ci1 = s_cs[Q + i];
      const uint32_t wide0 = s_wide[0], wide1 = s_wide[1];
#pragma unroll 1
      for (int g = 0; g < GPW; ++g) {
        const int j0 = CPW * cw + 16 * g;
        float v[16], m0[16], m1[16];
        if (j0 <= 32 * q + 31) {  // warp-uniform: some key of the group is causal for some row of the warp
          tc::tmem_ld16(tc::tmem_at(tb, 32 * q, cCB + j0), v);
          tc::tmem_wait_ld();
          const int jg = j0 >> 4;
          if (((wide0 | wide1) >> jg) & 1u) {  // warp-uniform: a wide group, one exp per element
#pragma unroll
            for (int k = 0; k < 16; ++k) {
              const int j = j0 + k;
              const bool causal = j <= i;
              const float f0 = ((wide0 >> jg) & 1u) ? __expf(ci0 - s_cs[j]) : __expf(ci0 - s_cs[j0]);
              const float f1 = ((wide1 >> jg) & 1u) ? __expf(ci1 - s_cs[Q + j]) : __expf(ci1 - s_cs[Q + j0]);
              m0[k] = causal ? v[k] * f0 * s_dt[j] : 0.f;
              m1[k] = causal ? v[k] * f1 * s_dt[Q + j] : 0.f;
            }
          } else {  // one row factor per head: exp(cs_i - cs_j0); the key factors are in s_dt
            const float r0 = __expf(ci0 - s_cs[j0]), r1 = __expf(ci1 - s_cs[Q + j0]);
#pragma unroll
            for (int k = 0; k < 16; ++k) {
              const int j = j0 + k;
              const bool causal = j <= i;
              m0[k] = causal ? v[k] * r0 * s_dt[j] : 0.f;
              m1[k] = causal ? v[k] * r1 * s_dt[Q + j] : 0.f;
            }
          }
        } else {
#pragma unroll
          for (int k = 0; k < 16; ++k) m0[k] = m1[k] = 0.f;
        }
        st_sw16(smem + oM + (0 * 2 + j0 / 64) * kReg, i, j0 % 64, m0);
        st_sw16(smem + oM + (1 * 2 + j0 / 64) * kReg, i, j0 % 64, m1);
      }
    }
    fence_proxy_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    if (*s_fail) break;
    if (warp < 2 && cc + 1 < p.ncq) fetch_dt(t0 + Q);  // s_dt has no reader left in this chunk

    // ---- Y_h = M_h x_h, dS (first half or all); the commit also covers Yi --------
    if (tid == 0) {
      tc::fence_after_sync();
      const uint32_t idy = tc::idesc_bf16(128, 64, false, true);
      const uint32_t ids = tc::idesc_bf16(128, 128, true, true);
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const uint64_t mh = static_cast<uint64_t>((hh * 2 * kReg) >> 4), xh = static_cast<uint64_t>((hh * kReg) >> 4);
#pragma unroll
        for (int s = 0; s < 8; ++s) tc::mma_bf16(tb + cY + 64 * hh, dKM + mh + kstep(s), dNX + xh + nstep(s), idy, s > 0);
      }
      constexpr int sN = SAVE ? 4 : 8;
#pragma unroll
      for (int s = 0; s < sN; ++s) tc::mma_bf16(tb + cCB, dNW + nstep(s), dNB + nstep(s), ids, s > 0);
      tc::mma_commit(bar_mma);
    }
    wait_mma();

    // ---- y = Y + exp(cs) Yi + D x ----------------------------------------------
    {
      const int i = 32 * q + lane, hh = (CPW * cw) / 64, yc0 = (CPW * cw) % 64;
      const float e = __expf(s_cs[hh * Q + i]);
      const float Dh = hh ? D1 : D0;
#pragma unroll 1
      for (int g = 0; g < GPW; ++g) {
        const int c0 = yc0 + 16 * g;
        float yv[16], yi[16], xv[16];
        tc::tmem_ld16(tc::tmem_at(tb, 32 * q, cY + 64 * hh + c0), yv);
        tc::tmem_ld16(tc::tmem_at(tb, 32 * q, cYi + 64 * hh + c0), yi);
        tc::tmem_wait_ld();
        ld_sw16(smem + oX + hh * kReg, i, c0, xv);
#pragma unroll
        for (int k = 0; k < 16; ++k) xv[k] = fmaf(e, yi[k], yv[k]) + Dh * xv[k];
        st_sw16(smem + oX + hh * kReg, i, c0, xv);  // y over x; the TMA store drops rows past seqlen
      }
    }

    // ---- state: S = exp(cs_end) S + dS (per half when saving) -------------------
    auto state_update = [&](float dec, bool write_bf16, bool stage, float* final_to) {
#pragma unroll 1
      for (int g = 0; g < GPW; ++g) {
        const int n0 = CPW * cw + 16 * g;
        float ds[16], sv[16];
        tc::tmem_ld16(tc::tmem_at(tb, 32 * q, cCB + n0), ds);
        tc::tmem_ld16(tc::tmem_at(tb, 32 * q, cS + n0), sv);
        tc::tmem_wait_ld();
#pragma unroll
        for (int k = 0; k < 16; ++k) sv[k] = fmaf(dec, sv[k], ds[k]);
        tc::tmem_st16(tc::tmem_at(tb, 32 * q, cS + n0), sv);
        if (write_bf16) st_sw16(smem + oS + (2 * sh + n0 / 64) * kReg64, sp, n0 % 64, sv);
        if (stage) stage_f32(smem + oM, srow, n0, sv);
        if (final_to != nullptr)
#pragma unroll
          for (int k = 0; k < 16; k += 4)
            *reinterpret_cast<float4*>(final_to + sp * N + n0 + k) = make_float4(sv[k], sv[k + 1], sv[k + 2], sv[k + 3]);
      }
      tc::tmem_wait_st();
    };
    const bool last = (cc + 1 == p.ncq);
    float* fin = (last && p.s_final != nullptr) ? p.s_final + bh_s * P * N : nullptr;
    const float* csh = s_cs + sh * Q;
    if (SAVE) {
      const int k1 = 2 * cc + 1, k2 = 2 * cc + 2;
      state_update(__expf(csh[QH - 1]), false, k1 < p.nc64, nullptr);
      fence_proxy_async_smem();  // y and the staged state, for the TMA stores
      tc::fence_before_sync();
      __syncthreads();
      if (*s_fail) break;
      if (tid == 0) {
        tc::fence_after_sync();
        tma_store_4d(&my, smem + oX, 0, h0, t0, b);
        tma_store_4d(&my, smem + oX + kReg, 0, h0 + 1, t0, b);
        if (k1 < p.nc64) store_state(k1);
        else bulk_commit();
        const uint32_t ids = tc::idesc_bf16(128, 128, true, true);
#pragma unroll
        for (int s = 4; s < 8; ++s) tc::mma_bf16(tb + cCB, dNW + nstep(s), dNB + nstep(s), ids, s > 4);
        tc::mma_commit(bar_mma);
        bulk_wait_read_all();  // the M buffer is staged into again below, y has left the x tile
      }
      wait_mma();
      __syncthreads();
      // x, B and C have no reader left in this chunk: the next chunk's tiles load under the state update
      if (tid == 0 && cc + 1 < p.ncq) issue_loads(cc + 1);
      state_update(__expf(csh[Q - 1] - csh[QH - 1]), true, k2 < p.nc64, fin);
      fence_proxy_async_smem();  // the bf16 state for the next chunk's Yi, the staged state
      tc::fence_before_sync();
      __syncthreads();
      if (*s_fail) break;
      if (tid == 0) {
        if (k2 < p.nc64) store_state(k2);
      }
    } else {
      state_update(__expf(csh[Q - 1]), true, false, fin);
      fence_proxy_async_smem();  // y, and the bf16 state for the next chunk's Yi
      tc::fence_before_sync();
      __syncthreads();
      if (*s_fail) break;
      if (tid == 0) {
        tma_store_4d(&my, smem + oX, 0, h0, t0, b);
        tma_store_4d(&my, smem + oX + kReg, 0, h0 + 1, t0, b);
        bulk_commit();
        bulk_wait_read_all();  // the next x tile lands where y was staged
        if (cc + 1 < p.ncq) issue_loads(cc + 1);
      }
    }
  }

  if (tid == 0) bulk_wait_all();  // the last stores have landed
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    tc::tmem_relinquish();
    tc::tmem_dealloc(tb, kCols);
  }
}

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  set_last_error(buf);
  return code;
}

unsigned long long g_mask_save = 0, g_mask_nosave = 0;

}  // namespace ssdtc

// The tensor-core forward for the shapes it covers: headdim 64, dstate 128,
// an even number of heads per group.  EMA_ERR_UNSUPPORTED (message unset)
// means "use the other kernel".
int ssd_fwd_tc_launch(const SsdFwdArgs* a, cudaStream_t stream) {
  using namespace ssdtc;
  if (a->headdim != P || a->dstate != N || a->nheads % 2 != 0 || (a->nheads / a->ngroups) % 2 != 0)
    return EMA_ERR_UNSUPPORTED;
  if (a->batch > 65535 || a->nheads / 2 > 2147483647) return EMA_ERR_UNSUPPORTED;
  for (int i = 0; i < 3; ++i)
    if (a->out_stride[i] % 8 != 0) return EMA_ERR_UNSUPPORTED;  // 16-byte row stores
  if ((reinterpret_cast<uintptr_t>(a->out) & 15u) != 0) return EMA_ERR_UNSUPPORTED;
  CUtensorMap mx{}, mb{}, mc{};
  const uint64_t dx[4] = {static_cast<uint64_t>(P), static_cast<uint64_t>(a->nheads), static_cast<uint64_t>(a->seqlen),
                          static_cast<uint64_t>(a->batch)};
  const uint64_t sx[3] = {static_cast<uint64_t>(a->x_stride[2]) * 2, static_cast<uint64_t>(a->x_stride[1]) * 2,
                          static_cast<uint64_t>(a->x_stride[0]) * 2};
  const uint32_t box[4] = {64, 1, static_cast<uint32_t>(Q), 1};
  int r = encode_map(&mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, a->x, dx, sx, box, true);
  if (r) return r;
  const uint64_t dbc[4] = {static_cast<uint64_t>(N), static_cast<uint64_t>(a->ngroups),
                           static_cast<uint64_t>(a->seqlen), static_cast<uint64_t>(a->batch)};
  const uint64_t sb[3] = {static_cast<uint64_t>(a->B_stride[2]) * 2, static_cast<uint64_t>(a->B_stride[1]) * 2,
                          static_cast<uint64_t>(a->B_stride[0]) * 2};
  const uint64_t sc[3] = {static_cast<uint64_t>(a->C_stride[2]) * 2, static_cast<uint64_t>(a->C_stride[1]) * 2,
                          static_cast<uint64_t>(a->C_stride[0]) * 2};
  r = encode_map(&mb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, a->B, dbc, sb, box, true);
  if (r) return r;
  r = encode_map(&mc, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, a->C, dbc, sc, box, true);
  if (r) return r;
  CUtensorMap my{}, ms{};
  const uint64_t sy[3] = {static_cast<uint64_t>(a->out_stride[2]) * 2, static_cast<uint64_t>(a->out_stride[1]) * 2,
                          static_cast<uint64_t>(a->out_stride[0]) * 2};
  r = encode_map(&my, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, a->out, dx, sy, box, true);
  if (r) return r;
  ms = my;
  if (a->chunk_states != nullptr) {
    const int64_t nc64 = (a->seqlen + QH - 1) / QH;
    const uint64_t ds[2] = {static_cast<uint64_t>(N), static_cast<uint64_t>(a->batch * nc64 * a->nheads * P)};
    const uint64_t ss[1] = {static_cast<uint64_t>(N) * 4};
    const uint32_t sbox[2] = {32, 128};
    r = encode_map(&ms, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, a->chunk_states, ds, ss, sbox, true);
    if (r) return r;
  }
  Params p{};
  p.B = static_cast<int>(a->batch);
  p.L = static_cast<int>(a->seqlen);
  p.H = static_cast<int>(a->nheads);
  p.G = static_cast<int>(a->ngroups);
  p.ncq = static_cast<int>((a->seqlen + Q - 1) / Q);
  p.nc64 = static_cast<int>((a->seqlen + QH - 1) / QH);
  p.dt = a->dt;
  p.A = a->A;
  p.D = a->D;
  p.s0 = a->initial_state;
  p.y = static_cast<bf16*>(a->out);
  p.sy_b = a->out_stride[0];
  p.sy_l = a->out_stride[1];
  p.sy_h = a->out_stride[2];
  p.chunk_states = a->chunk_states;
  p.s_final = a->final_state;
  p.dtm = dt_map_of(a);
  void* st = nullptr;
  if (cudaGetSymbolAddress(&st, g_status) != cudaSuccess) return fail(EMA_ERR_CUDA, "ssd_fwd: status word");
  p.status = static_cast<uint32_t*>(st);
  const dim3 grid(static_cast<unsigned>(a->nheads / 2), static_cast<unsigned>(a->batch));
  if (a->chunk_states != nullptr) {
    r = ensure_smem_attr(reinterpret_cast<const void*>(ssd_fwd_tc_kernel<true>), kSmem, &g_mask_save);
    if (r) return fail(EMA_ERR_CUDA, "ssd_fwd: %s", cudaGetErrorString(static_cast<cudaError_t>(r)));
    ssd_fwd_tc_kernel<true><<<grid, NT, kSmem, stream>>>(mx, mb, mc, my, ms, p);
  } else {
    r = ensure_smem_attr(reinterpret_cast<const void*>(ssd_fwd_tc_kernel<false>), kSmem, &g_mask_nosave);
    if (r) return fail(EMA_ERR_CUDA, "ssd_fwd: %s", cudaGetErrorString(static_cast<cudaError_t>(r)));
    ssd_fwd_tc_kernel<false><<<grid, NT, kSmem, stream>>>(mx, mb, mc, my, ms, p);
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(EMA_ERR_CUDA, "ssd_fwd launch failed: %s", cudaGetErrorString(e));
  return EMA_OK;
}

uint32_t* ssd_tc_status_device_ptr() {
  void* ptr = nullptr;
  return cudaGetSymbolAddress(&ptr, ssdtc::g_status) == cudaSuccess ? static_cast<uint32_t*>(ptr) : nullptr;
}

// Device status of the tensor-core SSD kernels (bit 1: a wait timed out, bit 2:
// misaligned shared memory); cleared when `clear` is set.
int ssd_tc_status(uint32_t* out, bool clear, cudaStream_t stream) {
  uint32_t v = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&v, ssdtc::g_status, 4, 0, cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e == cudaSuccess && clear) {
    const uint32_t z = 0;
    e = cudaMemcpyToSymbolAsync(ssdtc::g_status, &z, 4, 0, cudaMemcpyHostToDevice, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  }
  if (e != cudaSuccess) return ssdtc::fail(EMA_ERR_CUDA, "ssd status: %s", cudaGetErrorString(e));
  *out = v;
  return EMA_OK;
}

}  // namespace emab
