// Mamba-2 SSD chunked scan, backward, on the 5th-generation tensor cores
// (tcgen05 + tensor memory), for sm_100a.
//
// The adjoint of ssd_fwd (the algorithm of ssd_bwd_kernel in ssd_kernels.cu,
// contraction by contraction).  One CTA of eight warps per (batch, head) walks
// the 64-token chunks in reverse with the state gradient dS (headdim 64 x
// dstate 128, fp32) in tensor memory.  With a_ij = exp(cs_i - cs_j) (j <= i),
// e_i = exp(cs_i), w_j = dt_j exp(cs_end - cs_j), per chunk:
//
//   phase 1   CB = C B^T, DX = dy x^T, dXs = B dS^T (dS head + residual),
//             G8 = dy Sin (Sin head + residual)
//             -> Mq = CB a dt, E = a DX, Ed = a DX dt (bf16 operand tiles), the
//                row / column sums of T = CB a dt DX and R = CB a DX, the
//                per-token terms inter_i = e_i G8_i . C_i and V_j, and dC += e G8
//   phase 2   dXi = Mq^T dy, dB = Ed^T C + x_w dS (x_w = w x, one accumulator)
//             -> dx = dXi + w dXs + D dy, dB (one atomic pass)
//   phase 3   G7 = Ed B, G9 = (e dy)^T C (head + residual)
//             -> dC += G7, dS = exp(cs_end) dS + G9
//   then      dcs, its reverse cumsum within the chunk, ddt and dA (one warp).
//
// Every operand is an M = 64 tile (token or headdim rows): D row r lives in
// tensor-memory lane 32 (r / 16) + r % 16, so in the epilogues lanes 0-15 of
// each warp hold rows and the two warps of a lane quarter split the columns.
// No operand is transposed: x, dy, B, C and the saved state come in by TMA
// (128-byte swizzle) and are read K-major or MN-major as each contraction
// needs; the tiles built per chunk are written once in the same layout.  dB and
// dC are summed over the heads of a group with fp32 vector atomics.
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
uint32_t* ssd_tc_status_device_ptr();  // ssd_fwd_tc.cu: the error word both tensor-core SSD kernels share

namespace ssdbtc {

using bf16 = __nv_bfloat16;
using tc::ld_sw16;
using tc::st_sw16;

constexpr int Q = 64;    // tokens per chunk (the saved-state granularity)
constexpr int P = 64;    // headdim
constexpr int N = 128;   // dstate
constexpr int NW = 8;
constexpr int NT = NW * 32;
constexpr int R64 = 64 * 128;  // one 64-row x 128-byte swizzled region

// shared memory (from a 1024-byte-aligned base)
constexpr int oX = 0;               // x  [64 tokens][64 p]
constexpr int oDY = oX + R64;       // dy [64 tokens][64 p]
constexpr int oB = oDY + R64;       // B  [64 tokens][128 n]: 2 regions
constexpr int oC = oB + 2 * R64;    // C  the same
constexpr int oSF = oC + 2 * R64;   // Sin fp32 [64 p][128 n]: 4 regions of 32 floats per row
constexpr int oSH = oSF + 4 * R64;  // Sin bf16 head  [64 p][128 n]: 2 regions
constexpr int oSL = oSH + 2 * R64;  // Sin bf16 residual
constexpr int oDH = oSL + 2 * R64;  // dS bf16 head  [64 p][128 n]
constexpr int oDL = oDH + 2 * R64;  // dS bf16 residual
constexpr int oMq = oDL + 2 * R64;  // CB a dt [64 i][64 j]
constexpr int oXW = oMq + R64;      // x_w = w x [64 tokens][64 p]
constexpr int oEd = oXW + R64;      // a DX dt
constexpr int oYH = oEd + R64;      // e dy head [64 i][64 p]
constexpr int oYL = oYH + R64;      // e dy residual
constexpr int oF = oYL + R64;       // floats below
// float offsets within oF
constexpr int fCs = 0, fDt = 64, fRow = 192, fColT = 320, fColR = 384, fInter = 448, fV = 576, fMisc = 704;
constexpr int fEcol = 712;  // exp(cs_g - cs_j) per key j (g: first key of its 16-key group), and a wide-group mask
constexpr int fDer = 780;   // d dt / d (dt given) per token, where a dt map is active
constexpr int kFloats = 844;
// exp(cs_i - cs_j) is factored per 16-key group unless the cumsum spans more than this inside it
constexpr float kWideSpan = 60.f;
constexpr int kTP = 65;                     // padded row of the staged T / R tiles
constexpr int oT = oF + kFloats * 4;        // float T[64][65] = CB a dt DX (masked), for its column sums
constexpr int oR = oT + 64 * kTP * 4;       // float R[64][65] = CB a DX
constexpr int oBar = oR + 64 * kTP * 4;     // full, mma (u64); taddr, fail (u32)
constexpr int kSmem = oBar + 32;
static_assert(kSmem <= 232448, "shared memory");

// tensor-memory columns (M = 64 accumulators)
constexpr uint32_t cCB = 0, cDX = 64, cXS = 128, cG8 = 192;  // phase 1
constexpr uint32_t cXI = 0, cBI = 192;                       // phase 2
constexpr uint32_t cG7 = 128, cG9 = 256;                     // phase 3
constexpr uint32_t cS = 384;                                 // state gradient, persistent
constexpr uint32_t kCols = 512;

constexpr uint32_t kStatusAlign = 0x100u;

struct Params {
  int B, L, H, G, nc;
  const float* dt;
  const float* A;
  const float* D;
  const float* ds_final;  // (B,H,P,N) or null
  bf16* dx;
  long long sdx_b, sdx_l, sdx_h;
  float* ddt;
  float* dA;
  float* dB;  // (B,L,G,N) fp32 contiguous
  float* dC;
  float* dD;
  float* ds0;  // (B,H,P,N) or null
  uint32_t* status;
  DtMap dtm;        // dt <- clamp(softplus(dt + bias)), applied as dt lands in shared memory
  float* ddt_bias;  // (H,) or null: the gradient of the bias, accumulated
};

__device__ __forceinline__ void split_bf16(float v, float& hi, float& lo) {
  hi = __bfloat162float(__float2bfloat16_rn(v));
  lo = v - hi;
}

// fp32 element (row, n) of a staged 4-region state tile (32 floats per row per region)
__device__ __forceinline__ const float* sf_at(const unsigned char* base, int row, int n) {
  const int c = (n & 31) >> 2;
  return reinterpret_cast<const float*>(base + (n >> 5) * R64 + row * 128 + ((c ^ (row & 7)) << 4)) + (n & 3);
}

__global__ void __launch_bounds__(NT, 1)
    ssd_bwd_tc_kernel(const __grid_constant__ CUtensorMap mx, const __grid_constant__ CUtensorMap mdy,
                      const __grid_constant__ CUtensorMap mb, const __grid_constant__ CUtensorMap mc,
                      const __grid_constant__ CUtensorMap ms, const Params p) {
  extern __shared__ __align__(1024) unsigned char smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint32_t* status = p.status;
  if ((smem_u32(smem) & 1023u) != 0u) {
    if (tid == 0) atomicOr(status, kStatusAlign);
    return;
  }
  const int h = blockIdx.x, b = blockIdx.y;
  const int grp = h / (p.H / p.G);
  const int q = warp & 3, hw = warp >> 2;  // lane quarter, column half
  const bool act = lane < 16;              // lanes holding an M = 64 row
  const int row = 16 * q + (lane & 15);    // that row
  float* F = reinterpret_cast<float*>(smem + oF);
  float* s_cs = F + fCs;
  float* s_dt = F + fDt;  // [2][64]: double buffer by chunk parity
  float* s_row = F + fRow;  // [2][64] per column half
  float* s_colT = F + fColT;
  float* s_colR = F + fColR;
  float* s_inter = F + fInter;  // [2][64]
  float* s_V = F + fV;          // [2][64]
  float* s_misc = F + fMisc;
  float* s_ecol = F + fEcol;
  float* s_der = F + fDer;
  const bool mapped = dt_map_active(p.dtm);
  uint32_t* s_wide = reinterpret_cast<uint32_t*>(F + fEcol + 64);
  uint64_t* bar_full = reinterpret_cast<uint64_t*>(smem + oBar);
  uint64_t* bar_mma = bar_full + 1;
  uint32_t* s_taddr = reinterpret_cast<uint32_t*>(bar_full + 2);
  volatile uint32_t* s_fail = s_taddr + 1;
  const uint32_t sbase = smem_u32(smem);
  const float Ah = p.A[h];
  const float Dh = (p.D != nullptr) ? p.D[h] : 0.f;
  const size_t bh = static_cast<size_t>(b) * p.H + h;

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

  // descriptors of the fixed tiles; steps add to the start-address field
  const uint64_t kX = tc::smem_desc_sw128(sbase + oX, 16, 1024), kDY = tc::smem_desc_sw128(sbase + oDY, 16, 1024);
  const uint64_t kB = tc::smem_desc_sw128(sbase + oB, 16, 1024), kC = tc::smem_desc_sw128(sbase + oC, 16, 1024);
  const uint64_t kDH = tc::smem_desc_sw128(sbase + oDH, 16, 1024), kDL = tc::smem_desc_sw128(sbase + oDL, 16, 1024);
  const uint64_t kEd = tc::smem_desc_sw128(sbase + oEd, 16, 1024);
  const uint64_t nDY = tc::smem_desc_sw128(sbase + oDY, R64, 1024), nB = tc::smem_desc_sw128(sbase + oB, R64, 1024);
  const uint64_t nC = tc::smem_desc_sw128(sbase + oC, R64, 1024);
  const uint64_t nSH = tc::smem_desc_sw128(sbase + oSH, R64, 1024), nSL = tc::smem_desc_sw128(sbase + oSL, R64, 1024);
  const uint64_t nDH = tc::smem_desc_sw128(sbase + oDH, R64, 1024);
  const uint64_t nMq = tc::smem_desc_sw128(sbase + oMq, R64, 1024), nEd = tc::smem_desc_sw128(sbase + oEd, R64, 1024);
  const uint64_t kXW = tc::smem_desc_sw128(sbase + oXW, 16, 1024);
  const uint64_t nYH = tc::smem_desc_sw128(sbase + oYH, R64, 1024), nYL = tc::smem_desc_sw128(sbase + oYL, R64, 1024);
  auto kst = [](int s) { return static_cast<uint64_t>(((s >> 2) * R64 + (s & 3) * 32) >> 4); };  // K-major step
  auto nst = [](int s) { return static_cast<uint64_t>((s * 2048) >> 4); };                        // MN-major step

  auto issue_loads = [&](int c) {
    const int t0 = c * Q;
    const int srow = (static_cast<int>(b * p.nc + c) * p.H + h) * P;
    mbar_arrive_expect_tx(bar_full, 10u * R64);
    tma_load_4d(smem + oX, &mx, bar_full, 0, h, t0, b);
    tma_load_4d(smem + oDY, &mdy, bar_full, 0, h, t0, b);
    tma_load_4d(smem + oB, &mb, bar_full, 0, grp, t0, b);
    tma_load_4d(smem + oB + R64, &mb, bar_full, 64, grp, t0, b);
    tma_load_4d(smem + oC, &mc, bar_full, 0, grp, t0, b);
    tma_load_4d(smem + oC + R64, &mc, bar_full, 64, grp, t0, b);
#pragma unroll
    for (int r = 0; r < 4; ++r) tc::tma_load_2d(smem + oSF + r * R64, &ms, bar_full, 32 * r, srow);
  };
  auto fetch_dt = [&](int c) {  // warp 0: dt of chunk c into s_dt[c & 1] (cp.async)
    const int t0 = c * Q;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int j = lane + 32 * k, t = t0 + j;
      float* dst = s_dt + (c & 1) * Q + j;
      if (t < p.L) cp_async_4(dst, p.dt + (static_cast<size_t>(b) * p.L + t) * p.H + h);
      else *dst = 0.f;
    }
  };
  // Chunk c's saved state: fp32 (landed by TMA) -> bf16 head and residual
  // tiles, and <dS, Sin> (dS from its bf16 head + residual tiles) into
  // s_misc[c & 1].  Run by the 128 threads t0 .. t0 + 127, which first observe
  // the chunk's TMA completion.
  auto stage_state = [&](int c, int t) {
    if (!mbar_wait_bounded(bar_full, (p.nc - 1 - c) & 1, status)) *s_fail = 1u;
    const int pr = t >> 1, n0 = (t & 1) * 64;
    float part = 0.f;
#pragma unroll 1
    for (int g = 0; g < 4; ++g) {
      const int n = n0 + 16 * g;
      float v[16], hi[16], lo[16], dh[16], dl[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) v[k] = *sf_at(smem + oSF, pr, n + k);
#pragma unroll
      for (int k = 0; k < 16; ++k) split_bf16(v[k], hi[k], lo[k]);
      st_sw16(smem + oSH + (n >> 6) * R64, pr, n & 63, hi);
      st_sw16(smem + oSL + (n >> 6) * R64, pr, n & 63, lo);
      ld_sw16(smem + oDH + (n >> 6) * R64, pr, n & 63, dh);
      ld_sw16(smem + oDL + (n >> 6) * R64, pr, n & 63, dl);
#pragma unroll
      for (int k = 0; k < 16; ++k) part = fmaf(dh[k] + dl[k], v[k], part);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
    if ((t & 31) == 0) atomicAdd(&s_misc[c & 1], part);
    fence_proxy_async_smem();  // the bf16 state tiles, for the chunk's MMAs
  };
  auto wait_mma = [&]() {
    if (!mbar_wait_bounded(bar_mma, mma_phase & 1u, status)) *s_fail = 1u;
    ++mma_phase;
    tc::fence_after_sync();
  };

  // ---- the state gradient after the last chunk: tensor memory + bf16 tiles ----
  {
#pragma unroll 1
    for (int g = 0; g < 4; ++g) {
      const int n0 = 64 * hw + 16 * g;
      float v[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) v[k] = (act && p.ds_final != nullptr) ? p.ds_final[(bh * P + row) * N + n0 + k] : 0.f;
      tc::tmem_st16(tc::tmem_at(tb, 32 * q, cS + n0), v);
      if (act) {
        float hi[16], lo[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) split_bf16(v[k], hi[k], lo[k]);
        st_sw16(smem + oDH + (n0 >> 6) * R64, row, n0 & 63, hi);
        st_sw16(smem + oDL + (n0 >> 6) * R64, row, n0 & 63, lo);
      }
    }
    tc::tmem_wait_st();
  }
  fence_proxy_async_smem();
  if (tid == 0) {
    tma_prefetch_desc(&mx);
    tma_prefetch_desc(&mdy);
    tma_prefetch_desc(&mb);
    tma_prefetch_desc(&mc);
    tma_prefetch_desc(&ms);
    issue_loads(p.nc - 1);
  }
  if (warp == 0) fetch_dt(p.nc - 1);
  if (tid < 4) s_misc[tid] = 0.f;
  tc::fence_before_sync();
  __syncthreads();
  if (tid >= 128) stage_state(p.nc - 1, tid - 128);

  float dA_acc = 0.f, dD_acc = 0.f, dbias_acc = 0.f;
  const uint32_t id64 = tc::idesc_bf16(64, 64, false, false);

  for (int c = p.nc - 1; c >= 0; --c) {
    const int t0 = c * Q;
    const int nq = min(Q, p.L - t0);
    const float* dtv = s_dt + (c & 1) * Q;
    // ---- phase 0: cumsum, the state and e dy operand tiles, sum dS . Sin -------
    if (!mbar_wait_bounded(bar_full, (p.nc - 1 - c) & 1, status)) *s_fail = 1u;
    if (warp == 0) {
      cp_async_wait_all();
      __syncwarp();
      if (mapped) {  // the map in place (padding tokens stay 0), its derivative for ddt
        float* dtw = s_dt + (c & 1) * Q;
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int j = lane + 32 * e;
          float der = 0.f;
          if (t0 + j < p.L) dtw[j] = dt_map(p.dtm, h, dtw[j], &der);
          s_der[j] = der;
        }
        __syncwarp();
      }
      float a0 = dtv[lane] * Ah, a1 = dtv[32 + lane] * Ah;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float n0 = __shfl_up_sync(0xffffffffu, a0, o), n1 = __shfl_up_sync(0xffffffffu, a1, o);
        if (lane >= o) {
          a0 += n0;
          a1 += n1;
        }
      }
      a1 += __shfl_sync(0xffffffffu, a0, 31);
      s_cs[lane] = a0;
      s_cs[32 + lane] = a1;
      // key factors per 16-key group: lanes 0-15 / 16-31 hold groups 0 / 1 (a0) and 2 / 3 (a1)
      const float g0 = __shfl_sync(0xffffffffu, a0, lane & ~15), e0 = __shfl_sync(0xffffffffu, a0, lane | 15);
      const float g1 = __shfl_sync(0xffffffffu, a1, lane & ~15), e1 = __shfl_sync(0xffffffffu, a1, lane | 15);
      const bool w0 = fabsf(g0 - e0) > kWideSpan, w1 = fabsf(g1 - e1) > kWideSpan;
      s_ecol[lane] = w0 ? 0.f : __expf(g0 - a0);
      s_ecol[32 + lane] = w1 ? 0.f : __expf(g1 - a1);
      const uint32_t b0 = __ballot_sync(0xffffffffu, w0), b1 = __ballot_sync(0xffffffffu, w1);
      if (lane == 0) *s_wide = (b0 & 1u) | (((b0 >> 16) & 1u) << 1) | ((b1 & 1u) << 2) | (((b1 >> 16) & 1u) << 3);
    }
    if (tid == 0) s_misc[(c + 1) & 1] = 0.f;  // the slot the previous chunk consumed: the next chunk's sum
    __syncthreads();  // the cumsum and this chunk's state tiles are written
    {
      // e_i dy_i -> bf16 head and residual, [i][p]
      const int i = tid >> 2, p0 = (tid & 3) * 16;
      const float e = __expf(s_cs[i]);
      float v[16], hi[16], lo[16];
      ld_sw16(smem + oDY, i, p0, v);
#pragma unroll
      for (int k = 0; k < 16; ++k) split_bf16(e * v[k], hi[k], lo[k]);
      st_sw16(smem + oYH, i, p0, hi);
      st_sw16(smem + oYL, i, p0, lo);
      // x_w = dt exp(cs_end - cs) x (the state part of dB, folded into its operand)
      const float wi = dtv[i] * __expf(s_cs[Q - 1] - s_cs[i]);
      ld_sw16(smem + oX, i, p0, v);
#pragma unroll
      for (int k = 0; k < 16; ++k) v[k] *= wi;
      st_sw16(smem + oXW, i, p0, v);
    }
    if (warp == 0 && c > 0) fetch_dt(c - 1);
    fence_proxy_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    if (*s_fail) break;
    const float cs_end = s_cs[Q - 1];

    // ---- phase 1 -----------------------------------------------------------------
    if (tid == 0) {
      tc::fence_after_sync();
      const uint32_t idKM128 = tc::idesc_bf16(64, 128, false, true);
#pragma unroll
      for (int s = 0; s < 8; ++s) tc::mma_bf16(tb + cCB, kC + kst(s), kB + kst(s), id64, s > 0);       // C B^T
#pragma unroll
      for (int s = 0; s < 4; ++s) tc::mma_bf16(tb + cDX, kDY + kst(s), kX + kst(s), id64, s > 0);     // dy x^T
#pragma unroll
      for (int s = 0; s < 8; ++s) tc::mma_bf16(tb + cXS, kB + kst(s), kDH + kst(s), id64, s > 0);      // B dS^T
#pragma unroll
      for (int s = 0; s < 8; ++s) tc::mma_bf16(tb + cXS, kB + kst(s), kDL + kst(s), id64, true);
#pragma unroll
      for (int s = 0; s < 4; ++s) tc::mma_bf16(tb + cG8, kDY + kst(s), nSH + nst(s), idKM128, s > 0);  // dy Sin
#pragma unroll
      for (int s = 0; s < 4; ++s) tc::mma_bf16(tb + cG8, kDY + kst(s), nSL + nst(s), idKM128, true);
      tc::mma_commit(bar_mma);
    }
    wait_mma();
    {
      const int i = row;
      const float ci = s_cs[i];
      const uint32_t wide = *s_wide;
      // (a) masked products -> Mq, E, Ed tiles; row / column sums of T and R
      float rsum = 0.f;
      float cb2[2][16], dx2[2][16];  // both 16-column groups, loaded before one wait
#pragma unroll
      for (int g = 0; g < 2; ++g) {
        tc::tmem_ld16(tc::tmem_at(tb, 32 * q, cCB + 32 * hw + 16 * g), cb2[g]);
        tc::tmem_ld16(tc::tmem_at(tb, 32 * q, cDX + 32 * hw + 16 * g), dx2[g]);
      }
      tc::tmem_wait_ld();
#pragma unroll
      for (int g = 0; g < 2; ++g) {
        const int j0 = 32 * hw + 16 * g;
        const float (&cb)[16] = cb2[g];
        const float (&dxm)[16] = dx2[g];
        float mq[16], ev[16], ed[16], tv[16], rv[16];
        const bool wg = (wide >> (j0 >> 4)) & 1u;  // warp-uniform
        const float rf = __expf(ci - s_cs[j0]);       // row factor of the group
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          const int j = j0 + k;
          mq[k] = ev[k] = ed[k] = tv[k] = rv[k] = 0.f;
          if (act && j <= i) {
            const float a = wg ? __expf(ci - s_cs[j]) : rf * s_ecol[j];
            const float dtj = dtv[j];
            mq[k] = cb[k] * a * dtj;
            ev[k] = a * dxm[k];
            ed[k] = ev[k] * dtj;
            rv[k] = cb[k] * ev[k];
            tv[k] = rv[k] * dtj;
          }
          rsum += tv[k];
        }
        if (act) {
          st_sw16(smem + oMq, i, j0, mq);
          st_sw16(smem + oEd, i, j0, ed);
          // staged for the column sums (summed by other threads during phase 2)
          float* tr = reinterpret_cast<float*>(smem + oT) + i * kTP + j0;
          float* rr = reinterpret_cast<float*>(smem + oR) + i * kTP + j0;
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            tr[k] = tv[k];
            rr[k] = rv[k];
          }
        }
      }
      if (act) s_row[hw * 64 + i] = rsum;
      // (b) G8 = dy Sin: inter_i = e_i G8_i . C_i, and dC += e G8
      {
        const float e = __expf(ci);
        float ip = 0.f;
        float* dcrow = p.dC + ((static_cast<size_t>(b) * p.L + t0 + i) * p.G + grp) * N;
#pragma unroll 1
        for (int g2 = 0; g2 < 4; g2 += 2) {
          float v2[2][16];
          tc::tmem_ld16(tc::tmem_at(tb, 32 * q, cG8 + 64 * hw + 16 * g2), v2[0]);
          tc::tmem_ld16(tc::tmem_at(tb, 32 * q, cG8 + 64 * hw + 16 * g2 + 16), v2[1]);
          tc::tmem_wait_ld();
#pragma unroll
          for (int gg = 0; gg < 2; ++gg) {
          const int n0 = 64 * hw + 16 * (g2 + gg);
          const float (&v)[16] = v2[gg];
          float cv[16];
          if (act) {
            ld_sw16(smem + oC + (n0 >> 6) * R64, i, n0 & 63, cv);
#pragma unroll
            for (int k = 0; k < 16; ++k) ip = fmaf(v[k], cv[k], ip);
            if (i < nq)
#pragma unroll
              for (int k = 0; k < 16; k += 4)
                atomicAdd(reinterpret_cast<float4*>(dcrow + n0 + k),
                          make_float4(e * v[k], e * v[k + 1], e * v[k + 2], e * v[k + 3]));
          }
          }
        }
        if (act) s_inter[hw * 64 + i] = e * ip;
      }
      // (c) V_j = exp(cs_end - cs_j) x_j . (B_j dS^T)
      {
        float vp = 0.f;
        float vx2[2][16];
        tc::tmem_ld16(tc::tmem_at(tb, 32 * q, cXS + 32 * hw), vx2[0]);
        tc::tmem_ld16(tc::tmem_at(tb, 32 * q, cXS + 32 * hw + 16), vx2[1]);
        tc::tmem_wait_ld();
#pragma unroll
        for (int g = 0; g < 2; ++g) {
          const int p0 = 32 * hw + 16 * g;
          const float (&v)[16] = vx2[g];
          float xv[16];
          if (act) {
            ld_sw16(smem + oX, i, p0, xv);
#pragma unroll
            for (int k = 0; k < 16; ++k) vp = fmaf(v[k], xv[k], vp);
          }
        }
        if (act) s_V[hw * 64 + i] = __expf(cs_end - ci) * vp;
      }
    }
    fence_proxy_async_smem();
    tc::fence_before_sync();
    __syncthreads();

    // ---- phase 2 -----------------------------------------------------------------
    if (tid == 0) {
      tc::fence_after_sync();
      const uint32_t idMM64 = tc::idesc_bf16(64, 64, true, true), idMM128 = tc::idesc_bf16(64, 128, true, true);
#pragma unroll
      for (int s = 0; s < 4; ++s) tc::mma_bf16(tb + cXI, nMq + nst(s), nDY + nst(s), idMM64, s > 0);  // Mq^T dy
      const uint32_t idKM128 = tc::idesc_bf16(64, 128, false, true);
#pragma unroll
      for (int s = 0; s < 4; ++s) tc::mma_bf16(tb + cBI, nEd + nst(s), nC + nst(s), idMM128, s > 0);  // Ed^T C
#pragma unroll
      for (int s = 0; s < 4; ++s) tc::mma_bf16(tb + cBI, kXW + kst(s), nDH + nst(s), idKM128, true);  // x_w dS
      tc::mma_commit(bar_mma);
    }
    if (tid >= 64 && tid < 192) {  // column sums of T and R while the MMAs run
      const int j = tid & 63;
      const float* src = reinterpret_cast<const float*>(smem + (tid < 128 ? oT : oR)) + j;
      float acc = 0.f;
#pragma unroll 8
      for (int i = 0; i < 64; ++i) acc += src[i * kTP];
      (tid < 128 ? s_colT : s_colR)[j] = acc;
    }
    wait_mma();
    {
      const int j = row;
      const float dtj = dtv[j], wj = dtj * __expf(cs_end - s_cs[j]);
      // dx = dXi + w dXs + D dy; dD += dy . x
      bf16* dxrow = p.dx + b * p.sdx_b + static_cast<long long>(t0 + j) * p.sdx_l + h * p.sdx_h;
      float xi2[2][16], xs2[2][16];  // both 16-column groups, loaded before one wait
#pragma unroll
      for (int g = 0; g < 2; ++g) {
        tc::tmem_ld16(tc::tmem_at(tb, 32 * q, cXI + 32 * hw + 16 * g), xi2[g]);
        tc::tmem_ld16(tc::tmem_at(tb, 32 * q, cXS + 32 * hw + 16 * g), xs2[g]);
      }
      tc::tmem_wait_ld();
#pragma unroll
      for (int g = 0; g < 2; ++g) {
        const int p0 = 32 * hw + 16 * g;
        const float (&xi)[16] = xi2[g];
        const float (&xs)[16] = xs2[g];
        float dv[16], xv[16];
        if (act && j < nq) {
          ld_sw16(smem + oDY, j, p0, dv);
          ld_sw16(smem + oX, j, p0, xv);
          uint32_t w[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            w[k] = pack_pair<bf16>(make_float2(xi[2 * k] + wj * xs[2 * k] + Dh * dv[2 * k],
                                               xi[2 * k + 1] + wj * xs[2 * k + 1] + Dh * dv[2 * k + 1]));
            dD_acc = fmaf(dv[2 * k], xv[2 * k], fmaf(dv[2 * k + 1], xv[2 * k + 1], dD_acc));
          }
          *reinterpret_cast<uint4*>(dxrow + p0) = make_uint4(w[0], w[1], w[2], w[3]);
          *reinterpret_cast<uint4*>(dxrow + p0 + 8) = make_uint4(w[4], w[5], w[6], w[7]);
        }
      }
      // dB (both parts, summed over the group's heads by the atomics)
      float* dbrow = p.dB + ((static_cast<size_t>(b) * p.L + t0 + j) * p.G + grp) * N;
#pragma unroll 1
      for (int g2 = 0; g2 < 4; g2 += 2) {
        float v2[2][16];
        tc::tmem_ld16(tc::tmem_at(tb, 32 * q, cBI + 64 * hw + 16 * g2), v2[0]);
        tc::tmem_ld16(tc::tmem_at(tb, 32 * q, cBI + 64 * hw + 16 * g2 + 16), v2[1]);
        tc::tmem_wait_ld();
        if (act && j < nq)
#pragma unroll
          for (int gg = 0; gg < 2; ++gg)
#pragma unroll
            for (int k = 0; k < 16; k += 4)
              atomicAdd(reinterpret_cast<float4*>(dbrow + 64 * hw + 16 * (g2 + gg) + k),
                        make_float4(v2[gg][k], v2[gg][k + 1], v2[gg][k + 2], v2[gg][k + 3]));
      }
    }
    tc::fence_before_sync();
    __syncthreads();

    // ---- phase 3 -----------------------------------------------------------------
    if (tid == 0) {
      tc::fence_after_sync();
      const uint32_t idKM128 = tc::idesc_bf16(64, 128, false, true), idMM128 = tc::idesc_bf16(64, 128, true, true);
#pragma unroll
      for (int s = 0; s < 4; ++s) tc::mma_bf16(tb + cG7, kEd + kst(s), nB + nst(s), idKM128, s > 0);   // Ed B
#pragma unroll
      for (int s = 0; s < 4; ++s) tc::mma_bf16(tb + cG9, nYH + nst(s), nC + nst(s), idMM128, s > 0);   // (e dy)^T C
#pragma unroll
      for (int s = 0; s < 4; ++s) tc::mma_bf16(tb + cG9, nYL + nst(s), nC + nst(s), idMM128, true);
      tc::mma_commit(bar_mma);
    }
    wait_mma();
    // x, dy, B, C and Sin have no reader left: the next chunk's tiles load under the epilogue
    if (tid == 0 && c > 0) issue_loads(c - 1);
    {
      const int r = row;  // token (dC) or headdim row (dS)
      float* dcrow = p.dC + ((static_cast<size_t>(b) * p.L + t0 + r) * p.G + grp) * N;
      const float dec = __expf(cs_end);
#pragma unroll 1
      for (int g = 0; g < 4; ++g) {
        const int n0 = 64 * hw + 16 * g;
        float c7[16], g9[16], sv[16];
        tc::tmem_ld16(tc::tmem_at(tb, 32 * q, cG7 + n0), c7);
        tc::tmem_ld16(tc::tmem_at(tb, 32 * q, cG9 + n0), g9);
        tc::tmem_ld16(tc::tmem_at(tb, 32 * q, cS + n0), sv);
        tc::tmem_wait_ld();
        if (act && r < nq) {
#pragma unroll
          for (int k = 0; k < 16; k += 4)
            atomicAdd(reinterpret_cast<float4*>(dcrow + n0 + k), make_float4(c7[k], c7[k + 1], c7[k + 2], c7[k + 3]));
        }
#pragma unroll
        for (int k = 0; k < 16; ++k) sv[k] = fmaf(dec, sv[k], g9[k]);
        tc::tmem_st16(tc::tmem_at(tb, 32 * q, cS + n0), sv);
        if (act) {
          float hi[16], lo[16];
#pragma unroll
          for (int k = 0; k < 16; ++k) split_bf16(sv[k], hi[k], lo[k]);
          st_sw16(smem + oDH + (n0 >> 6) * R64, r, n0 & 63, hi);
          st_sw16(smem + oDL + (n0 >> 6) * R64, r, n0 & 63, lo);
          if (c == 0 && p.ds0 != nullptr)
#pragma unroll
            for (int k = 0; k < 16; k += 4)
              *reinterpret_cast<float4*>(p.ds0 + (bh * P + r) * N + n0 + k) =
                  make_float4(sv[k], sv[k + 1], sv[k + 2], sv[k + 3]);
        }
      }
      tc::tmem_wait_st();
    }
    fence_proxy_async_smem();  // the bf16 state-gradient tiles for the next chunk
    tc::fence_before_sync();
    __syncthreads();

    // ---- per token: dcs, its reverse cumsum, ddt and dA ---------------------------
    if (warp == 0) {
      float dcs[2], dir[2], dtk[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int i = lane + 32 * e;
        dtk[e] = dtv[i];
        const float Vi = s_V[i] + s_V[64 + i];
        const float U = dtk[e] * Vi;
        dcs[e] = (s_row[i] + s_row[64 + i]) - s_colT[i] + (s_inter[i] + s_inter[64 + i]) - U;
        dir[e] = s_colR[i] + Vi;
      }
      float usum = dtk[0] * (s_V[lane] + s_V[64 + lane]) + dtk[1] * (s_V[32 + lane] + s_V[96 + lane]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) usum += __shfl_xor_sync(0xffffffffu, usum, o);
      if (lane == 31) dcs[1] += usum + __expf(cs_end) * s_misc[c & 1];
      float r1 = dcs[1], r0 = dcs[0];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float n1 = __shfl_down_sync(0xffffffffu, r1, o), n0 = __shfl_down_sync(0xffffffffu, r0, o);
        if (lane + o < 32) {
          r1 += n1;
          r0 += n0;
        }
      }
      r0 += __shfl_sync(0xffffffffu, r1, 0);
      const float R[2] = {r0, r1};
      float da = 0.f, db = 0.f;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int i = lane + 32 * e;
        if (i < nq) {
          float g = dir[e] + Ah * R[e];
          if (mapped) {
            g *= s_der[i];
            db += g;
          }
          p.ddt[(static_cast<size_t>(b) * p.L + t0 + i) * p.H + h] = g;
        }
        da = fmaf(dtk[e], R[e], da);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        da += __shfl_xor_sync(0xffffffffu, da, o);
        db += __shfl_xor_sync(0xffffffffu, db, o);
      }
      dA_acc += da;
      dbias_acc += db;
    } else if (warp >= 4 && c > 0) {
      stage_state(c - 1, tid - 128);  // the next chunk's state tiles, off its critical path
    }
    __syncthreads();  // the per-token sums are read; the next chunk rewrites them
    if (*s_fail) break;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) dD_acc += __shfl_xor_sync(0xffffffffu, dD_acc, o);
  if (lane == 0 && p.dD != nullptr) atomicAdd(&p.dD[h], dD_acc);
  if (tid == 0) atomicAdd(&p.dA[h], dA_acc);
  if (tid == 0 && p.ddt_bias != nullptr) atomicAdd(&p.ddt_bias[h], dbias_acc);
  if (warp == 0) cp_async_wait_all();
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

unsigned long long g_mask = 0;

}  // namespace ssdbtc

// The tensor-core backward for headdim 64 / dstate 128 with TMA-compatible
// strides.  EMA_ERR_UNSUPPORTED (message unset) means "use the other kernel".
// dA, dB, dC and dD must already be zero.
int ssd_bwd_tc_launch(const SsdBwdArgs* a, cudaStream_t stream) {
  using namespace ssdbtc;
  if (a->headdim != P || a->dstate != N || a->batch > 65535) return EMA_ERR_UNSUPPORTED;
  for (int i = 0; i < 3; ++i)
    if (a->dx_stride[i] % 8 != 0) return EMA_ERR_UNSUPPORTED;  // 16-byte row stores
  if ((reinterpret_cast<uintptr_t>(a->dx) & 15u) || (reinterpret_cast<uintptr_t>(a->dB) & 15u) ||
      (reinterpret_cast<uintptr_t>(a->dC) & 15u) || (reinterpret_cast<uintptr_t>(a->chunk_states) & 15u))
    return EMA_ERR_UNSUPPORTED;
  const int64_t nc = (a->seqlen + Q - 1) / Q;
  CUtensorMap mx{}, mdy{}, mb{}, mc{}, ms{};
  const uint64_t dx4[4] = {static_cast<uint64_t>(P), static_cast<uint64_t>(a->nheads),
                           static_cast<uint64_t>(a->seqlen), static_cast<uint64_t>(a->batch)};
  const uint32_t box[4] = {64, 1, static_cast<uint32_t>(Q), 1};
  const uint64_t sx[3] = {static_cast<uint64_t>(a->x_stride[2]) * 2, static_cast<uint64_t>(a->x_stride[1]) * 2,
                          static_cast<uint64_t>(a->x_stride[0]) * 2};
  const uint64_t sy[3] = {static_cast<uint64_t>(a->dout_stride[2]) * 2, static_cast<uint64_t>(a->dout_stride[1]) * 2,
                          static_cast<uint64_t>(a->dout_stride[0]) * 2};
  int r = encode_map(&mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, a->x, dx4, sx, box, true);
  if (r) return r;
  r = encode_map(&mdy, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, a->dout, dx4, sy, box, true);
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
  const uint64_t ds[2] = {static_cast<uint64_t>(N), static_cast<uint64_t>(a->batch * nc * a->nheads * P)};
  const uint64_t ss[1] = {static_cast<uint64_t>(N) * 4};
  const uint32_t sbox[2] = {32, 64};
  r = encode_map(&ms, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, a->chunk_states, ds, ss, sbox, true);
  if (r) return r;
  Params p{};
  p.B = static_cast<int>(a->batch);
  p.L = static_cast<int>(a->seqlen);
  p.H = static_cast<int>(a->nheads);
  p.G = static_cast<int>(a->ngroups);
  p.nc = static_cast<int>(nc);
  p.dt = a->dt;
  p.A = a->A;
  p.D = a->D;
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
  p.dtm = dt_map_of(a);
  p.ddt_bias = a->ddt_bias;
  p.status = ssd_tc_status_device_ptr();
  if (p.status == nullptr) return fail(EMA_ERR_CUDA, "ssd_bwd: status word");
  r = ensure_smem_attr(reinterpret_cast<const void*>(ssd_bwd_tc_kernel), kSmem, &g_mask);
  if (r) return fail(EMA_ERR_CUDA, "ssd_bwd: %s", cudaGetErrorString(static_cast<cudaError_t>(r)));
  ssd_bwd_tc_kernel<<<dim3(static_cast<unsigned>(a->nheads), static_cast<unsigned>(a->batch)), NT, kSmem, stream>>>(
      mx, mdy, mb, mc, ms, p);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(EMA_ERR_CUDA, "ssd_bwd launch failed: %s", cudaGetErrorString(e));
  return EMA_OK;
}

}  // namespace emab
