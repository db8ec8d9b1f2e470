// Tensor-core backward, row-owned half (bf16 / fp16 inputs), sm_100a.
//
// Produces, per query row i and head h: dq (with upstream's host epilogue
// dq = scale (dqp + H W^T + sigma b) fused, backward.py:600-605), D, sigma =
// rowsum(dS) and this CTA's partial of dW = sum qt (x) H + dO (x) G
// (backward.py:607-614). Upstream computes the same quantities in
// flash_spacetime_bwd_rows_kernel (backward.py:316-485) with two sweeps over
// the keys: one for D = sum P dP / sum P, one for dS = P (dP - D).
//
// Here a single sweep suffices. With c_i = dO_i . (out_i - [act] b) (an
// estimate of D from the forward output) and dP'_ij = dP_ij - c_i, the
// sweep accumulates, from the rounded operands that the tensor cores see,
//   X_i  = sum_j [P dP']_ij k_j       Y_i  = sum_j [P]_ij k_j
//   H'_i = sum_j [P dP']_ij E_ij      G_i  = sum_j [P]_ij E_ij
//   a_i  = sum_j [P dP']_ij           p_i  = sum_j [P]_ij
// ([.] = rounded to the 16-bit type), and at the end
//   D'_i = a_i / p_i,   dqp_i = X_i - D'_i Y_i,   H_i = H'_i - D'_i G_i,
//   sigma_i = a_i - D'_i p_i.
// This is dS_ij = [P dP']_ij - D'_i [P]_ij contracted exactly: every sum of
// dS that feeds dq, H and sigma is formed from the same rounded values, so
// rowsum(dS) = a - D' p vanishes up to one fp32 rounding, and D = c + D' is
// the P-weighted mean of dP normalised by sum P as upstream requires
// (backward.py:371-407). Subtracting c first keeps the row's common mode out
// of the 16-bit products.
//
// Layout and warp roles follow the forward kernel (fst_tc_fwd.cu): head
// warps own one head's 16 rows (S = Q K^T, dP = dO V^T, X, Y on the tensor
// cores), E warps own QPE rows for all heads (embedding, the two logit-side
// bias products u.E and w~.E, and H', G), and the per-chunk bias tiles and P
// tiles cross between the two groups through double-buffered shared memory.
// The prologue forms u = (q*scale) W and w~ = dO W on the tensor cores and
// writes them, with qt = [q*scale], to the workspace for the column kernel;
// the epilogue forms this CTA's dW / db partials on the tensor cores.

#include <cuda_runtime.h>

#include "fst_internal.h"
#include "fst_tc_common.cuh"

namespace fst {
namespace tc {

template <int DH, int C>
struct RowShape {
  static constexpr int BM = 16, BN = 16;
  // Queries per E warp: two (eight E warps) at C <= 32 -- the E warps carry
  // the longer dependency chain per key chunk, so they get two warps per
  // scheduler.
  static constexpr int QPE = C <= 32 ? 2 : 1;
  static constexpr int NE = BM / QPE;
  // Heads per CTA: 12 only for the narrowest shapes; with C >= 32 a CTA of 8
  // heads keeps 128 registers a thread (at C = 32: 116 bytes of spills
  // instead of 368 with 12 heads at 96 registers).
  static constexpr int HP = (DH <= 32 && C <= 16) ? 12 : 8;
  // E warps run one chunk ahead (two E fragments live). Their u / w~
  // A-fragments are then re-read from a resident staged tile each chunk
  // instead of being held in registers.
  static constexpr bool AHEAD = C <= 16 && DH <= 32;
  // Loops unrolled by two chunks with literal ring stages where the
  // registers allow it (the wide shapes would spill).
  static constexpr bool LIT = AHEAD;
  static constexpr int NWARPS = HP + NE;
  static constexpr int KSD = DH / 16, NTD = DH / 8;
  static constexpr int KSC = C / 16, NTC = C / 8;
  static constexpr int F = C / 2, FG = F / 8;
  static constexpr int DHP = DH <= 16 ? 16 : (DH <= 32 ? 32 : 64);
  static constexpr int CP = C <= 16 ? 16 : (C <= 32 ? 32 : 64);
  static constexpr int RBD = DHP * 2, RBC = CP * 2;
  // bias tile: per (q, h) 16 keys x (u.E, w~.E) fp32 + 16 pad words.
  static constexpr int BROW = 48;
  static constexpr int BQ = HP * BROW + 16;
  // P tiles: per query 16 head rows of 16 keys (8 words) padded to 12 words,
  // + 4 pad words per query (conflict-free ldmatrix rows and stores).
  static constexpr int PH = 12;
  static constexpr int PQ = 16 * PH + 4;

  // The union region holds, in turn: staged Q and dO (phase 1), staged u and
  // w~ (phase 2), the loop's bias and P tiles, and the epilogue's H and G.
  // The epilogue's R = H W^T goes to the K/V ring, dead by then.
  static constexpr int SZ_QS = HP * BM * RBD;     // staged Q (scaled), and dO
  static constexpr int SZ_US = BM * 16 * RBC;     // staged u, and w~
  static constexpr int SZ_B = BM * BQ * 4;        // one bias stage
  static constexpr int SZ_P = BM * PQ * 4;        // one P tile
  static constexpr int SZ_LOOP = 2 * SZ_B + 4 * SZ_P;  // bias x2, (P, P dP') x2
  static constexpr int SZ_HG = 2 * BM * HP * C * 4;
  static constexpr int SZ_A = 2 * SZ_QS > 2 * SZ_US ? 2 * SZ_QS : 2 * SZ_US;
  static constexpr int SZ_B2 = SZ_LOOP > SZ_HG ? SZ_LOOP : SZ_HG;
  static constexpr int SZ_UNION = SZ_A > SZ_B2 ? SZ_A : SZ_B2;
  static constexpr int OFF_Q = 0, OFF_DO = SZ_QS;
  static constexpr int OFF_B = 0, OFF_P = 2 * SZ_B;
  static constexpr int OFF_H = 0, OFF_G = BM * HP * C * 4;
  static constexpr int OFF_W = SZ_UNION;
  static constexpr int SZ_W = 2 * DH * RBC;
  // K / V rings come by TMA where the box (16 rows x Dh) fills whole swizzled
  // rows (Dh = 16, 32, 64); their stages start on 1024-byte boundaries.
  // At C = 64 the ring's barrier state costs the kernel registers it cannot
  // spare (config 2 measured 27.4 / 30.6 TFLOP/s with TMA against 28.5 / 31.5
  // with cp.async at Dh = 32 / 64), so those shapes keep cp.async.
  static constexpr bool TMA = (DH == 16 || DH == 32 || DH == 64) && C <= 32;
  static constexpr int OFF_K = (OFF_W + SZ_W + 1023) / 1024 * 1024;
  static constexpr int SZ_KV = HP * BN * RBD;
  static constexpr int OFF_V = OFF_K + 2 * SZ_KV;
  static constexpr int OFF_C = OFF_V + 2 * SZ_KV;           // [NE][2][BN][4]
  static constexpr int OFF_QC = OFF_C + NE * 2 * BN * 16;   // [BM][4]
  static constexpr int OFF_ST = OFF_QC + BM * 16;           // lse2, coff, D' : [3][BM][HP]
  static constexpr int OFF_UWR = OFF_ST + 3 * BM * HP * 4;  // resident u, w~ (AHEAD)
  static constexpr int OFF_U = AHEAD ? OFF_UWR : 0;
  static constexpr int OFF_WT = OFF_U + SZ_US;
  static constexpr int END_UW = OFF_UWR + (AHEAD ? 2 * SZ_US : 0);
  // Fast prologue / epilogue (AHEAD shapes that fit): raw q and dO stay
  // resident for the whole kernel (projections, dO fragments, dW partials),
  // and every prologue copy is one batch of cp.async; `out` rows for the row
  // offsets are staged in the union region next to the scaled Q.
  static constexpr int OFF_QR = END_UW, OFF_DOR = OFF_QR + SZ_QS;
  static constexpr int OFF_OS = SZ_QS;
  static constexpr bool FASTPRO = AHEAD && OFF_DOR + SZ_QS + HP * 16 <= 227 * 1024;
  static constexpr int OFF_MB = FASTPRO ? OFF_DOR + SZ_QS : END_UW;  // ring mbarriers [HP][2]
  static constexpr int SMEM = OFF_MB + HP * 16;
  static_assert(!FASTPRO || 2 * SZ_QS <= OFF_P, "staged Q / out do not overlap the P tiles");
  static constexpr int OFF_R = OFF_K;                        // [BM][HP][DH] fp32
  static_assert(BM * HP * DH * 4 <= 4 * SZ_KV, "R fits the K/V ring");
  static_assert(2 * HP * BM * RBD <= 4 * SZ_KV, "staged q, dO fit the K/V ring");
  static constexpr bool kFits = SMEM <= 227 * 1024;
};

__device__ __forceinline__ int rb_bias_full(int s) { return 1 + s; }
__device__ __forceinline__ int rb_bias_empty(int s) { return 3 + s; }
__device__ __forceinline__ int rb_p_full(int s) { return 5 + s; }
__device__ __forceinline__ int rb_p_empty(int s) { return 7 + s; }

template <typename T, int DH, int C>
__global__ void __launch_bounds__(RowShape<DH, C>::NWARPS * 32, 1)
    bwd_rows_tc_kernel(const FstBackwardArgs a, const int* __restrict__ tile_start,
                       int heads_per_group, T* __restrict__ u_ws, T* __restrict__ wt_ws,
                       T* __restrict__ qt_ws, const __grid_constant__ TmaPair kv_maps) {
  using S = RowShape<DH, C>;
  using E = Elem<T>;
  extern __shared__ __align__(1024) unsigned char smem[];
  const FstProblem& p = a.prob;

  const int h0 = blockIdx.z * heads_per_group;
  const int NH = min(heads_per_group, p.heads - h0);
  T* __restrict__ gdq = (T*)a.dq;
  // This CTA's dW / db partial slot: one per CTA of the grid.
  const int64_t part = ((int64_t)blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
  float* dwp = a.dw_partial + part * DH * C;
  float* dbp = a.db_partial + part * DH;

  // Event and row block of this CTA: grid (L / BM, B, groups) over the
  // padded layout, or entry blockIdx.x of the device tile list.
  int b, qb;
  if (uses_tile_list(p)) {
    int t = blockIdx.x;
    if (list_padding(p)) {
      const int writers = pad_ctas(p, DH * 2 + 8);  // padding bytes per (row, head)
      auto fill = [&](int e, int r0, int r1, int nan) {
        const EventSpan es = event_span(p, e);
        fill_rows<T, DH>(gdq, qkv_span(p, e, DH), a.delta, a.sigma, es, r0, r1, h0, NH,
                         nan ? E::kNaN2 : 0u, nan ? __int_as_float(0x7fc00000) : 0.f);
      };
      t = list_padded_role(p, tile_start, S::BM, writers, blockIdx.x, gridDim.x, fill);
    }
    const bool poisoned = t == kRolePoisoned;
    if (t < 0 || !list_tile(p, tile_start, t, b, qb)) {
      // No block to compute: the partial slot holds zeros (NaN when the
      // caller's valid_rows was too small).
      const float v = poisoned ? __int_as_float(0x7fc00000) : 0.f;
      for (int i = threadIdx.x; i < DH * C; i += blockDim.x) dwp[i] = v;
      for (int i = threadIdx.x; i < DH; i += blockDim.x) dbp[i] = v;
      return;
    }
  } else {
    b = p.event_order ? p.event_order[blockIdx.y] : (int)blockIdx.y;
    qb = blockIdx.x;
  }
  const EventSpan ev = event_span(p, b);
  const EventSpan evq = qkv_span(p, b, DH);  // q, k, v, dq (a fused QKV buffer's row stride)
  const int q0 = qb * S::BM;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int NE = S::NE;
  const int nthreads = blockDim.x;
  const bool attn = p.use_attn_bias != 0, act = p.use_act_bias != 0;
  const T* __restrict__ gq = (const T*)a.q;
  const T* __restrict__ gk = (const T*)a.k;
  const T* __restrict__ gv = (const T*)a.v;
  const T* __restrict__ gdo = (const T*)a.dout;
  const T* __restrict__ gout = (const T*)a.out;

  if (q0 >= ev.len) {
    for (int i = threadIdx.x; i < DH * C; i += nthreads) dwp[i] = 0.f;
    for (int i = threadIdx.x; i < DH; i += nthreads) dbp[i] = 0.f;
    if (!is_varlen(p)) {
      constexpr int CH = DH / 8;  // 16-byte chunks per row
      for (int idx = threadIdx.x; idx < NH * S::BM * CH; idx += nthreads) {
        const int c = idx % CH, r = idx / CH;
        const int h = h0 + r / S::BM, q = q0 + r % S::BM;
        if (q >= p.max_len) continue;
        *(uint4*)(gdq + ev_off(evq, q, h, DH) + c * 8) = make_uint4(0, 0, 0, 0);
        if (c == 0) {
          const int64_t so = ev_off(ev, q, h, 1);
          a.delta[so] = 0.f;
          a.sigma[so] = 0.f;
        }
      }
    }
    return;
  }
  const int nvalid_q = min(S::BM, ev.len - q0);
  const int nchunks = (ev.len + S::BN - 1) / S::BN;
  const int NBAR = (NH + NE) * 32;
  const uint32_t sm = smem_u32(smem);
  float* fQC = (float*)(smem + S::OFF_QC);
  float* fLse = (float*)(smem + S::OFF_ST);
  float* fCoff = fLse + S::BM * S::HP;
  float* fDp = fCoff + S::BM * S::HP;

  const int m4 = lane & 3, r8 = lane >> 2;
  const bool idle = warp >= NH + NE;
  uint32_t qa[S::KSD][4], da[S::KSD][4];  // head warps: Q (scaled) and dO, rows on M
  uint32_t ua[S::QPE][S::KSC][4], wa[S::QPE][S::KSC][4];  // E warps: u_q, w~_q
  if constexpr (S::FASTPRO) {
    // --------------------- prologue (one round of copies) ---------------------
    constexpr int QCH = DH / 8;
    const bool proj_u = attn && a.u == nullptr, proj_w = act && a.wt == nullptr;
    for (int idx = threadIdx.x; idx < NH * S::BM * QCH; idx += nthreads) {
      const int c = idx % QCH, q = (idx / QCH) % S::BM, h = idx / (QCH * S::BM);
      const uint32_t off = h * S::BM * S::RBD + swz<S::RBD>(q, c);
      if (q < nvalid_q) {
        const int64_t go = ev_off(ev, q0 + q, h0 + h, DH) + c * 8;
        cp_async16(sm + S::OFF_QR + off, gq + ev_off(evq, q0 + q, h0 + h, DH) + c * 8);
        cp_async16(sm + S::OFF_DOR + off, gdo + go);
        if (gout) cp_async16(sm + S::OFF_OS + off, gout + go);
      } else {
        *(uint4*)(smem + S::OFF_QR + off) = make_uint4(0, 0, 0, 0);
        *(uint4*)(smem + S::OFF_DOR + off) = make_uint4(0, 0, 0, 0);
        *(uint4*)(smem + S::OFF_OS + off) = make_uint4(0, 0, 0, 0);
      }
    }
    for (int idx = threadIdx.x; idx < S::BM * NH; idx += nthreads) {
      const int q = idx / NH, h = idx % NH;
      const uint32_t dst = smem_u32(fLse + q * S::HP + h);
      if (q < nvalid_q)
        cp_async4(dst, a.lse + ev_off(ev, q0 + q, h0 + h, 1));
      else
        fLse[q * S::HP + h] = 0.f;
    }
    for (int q = threadIdx.x; q < S::BM; q += nthreads) {
      const uint32_t dst = smem_u32(fQC + q * 4);
      if (q < nvalid_q)
        cp_async16(dst, p.feats + (ev.row0 + q0 + q) * p.feat_stride);
      else
        *(float4*)(fQC + q * 4) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    cp_async_commit();
    // While the copies are in flight: W as [d][c] split into hi + lo halves,
    // the zero head rows of the projected tiles, the P tiles, and caller-given
    // u / w~ (if any).
    for (int idx = threadIdx.x; idx < DH * (S::CP / 2); idx += nthreads) {
      const int c2 = idx % (S::CP / 2), d = idx / (S::CP / 2);
      float w0 = 0.f, w1 = 0.f;
      if ((attn || act) && 2 * c2 < C) {
        w0 = p.weight[(int64_t)d * C + 2 * c2];
        w1 = p.weight[(int64_t)d * C + 2 * c2 + 1];
      }
      const uint32_t hi = E::pack(w0, w1);
      const uint32_t lo = E::pack(w0 - E::lo(hi), w1 - E::hi(hi));
      const uint32_t off = swz<S::RBC>(d, c2 / 4) + (c2 % 4) * 4;
      *(uint32_t*)(smem + S::OFF_W + off) = hi;
      *(uint32_t*)(smem + S::OFF_W + DH * S::RBC + off) = lo;
    }
    {
      constexpr int UCH = S::CP / 8;
      const int zrows = 16 - NH;
      for (int idx = threadIdx.x; idx < S::BM * zrows * UCH; idx += nthreads) {
        const int c = idx % UCH, h = NH + (idx / UCH) % zrows, q = idx / (UCH * zrows);
        const uint32_t off = swz<S::RBC>(q * 16 + h, c);
        if (proj_u) *(uint4*)(smem + S::OFF_U + off) = make_uint4(0, 0, 0, 0);
        if (proj_w) *(uint4*)(smem + S::OFF_WT + off) = make_uint4(0, 0, 0, 0);
      }
    }
    for (int idx = threadIdx.x; idx < 4 * S::SZ_P / 4; idx += nthreads)
      ((uint32_t*)(smem + S::OFF_P))[idx] = 0u;
    if (attn && !proj_u)
      stage_rows<T, C, S::CP>((const T*)a.u, ev, q0, nvalid_q, S::BM, h0, NH, smem + S::OFF_U);
    if (act && !proj_w)
      stage_rows<T, C, S::CP>((const T*)a.wt, ev, q0, nvalid_q, S::BM, h0, NH,
                              smem + S::OFF_WT);
    cp_async_wait<0>();
    __syncthreads();
    // Per (row, head): LSE in log2 units and the row offset c = dO.(out - [act] b),
    // d in order. Rows past the event were staged as zeros (c = 0, LSE 0).
    for (int idx = threadIdx.x; idx < S::BM * NH; idx += nthreads) {
      const int q = idx / NH, h = idx % NH;
      float c = 0.f;
      if (gout && q < nvalid_q) {
        const unsigned char* orow = smem + S::OFF_OS + h * S::BM * S::RBD;
        const unsigned char* drow = smem + S::OFF_DOR + h * S::BM * S::RBD;
#pragma unroll
        for (int ch = 0; ch < QCH; ++ch) {
          const uint4 ov = *(const uint4*)(orow + swz<S::RBD>(q, ch));
          const uint4 dv = *(const uint4*)(drow + swz<S::RBD>(q, ch));
          const uint32_t* o2 = (const uint32_t*)&ov;
          const uint32_t* d2 = (const uint32_t*)&dv;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float o0 = E::lo(o2[e]), o1 = E::hi(o2[e]);
            if (act && p.bias) {
              o0 -= p.bias[ch * 8 + 2 * e];
              o1 -= p.bias[ch * 8 + 2 * e + 1];
            }
            c = fmaf(E::lo(d2[e]), o0, c);
            c = fmaf(E::hi(d2[e]), o1, c);
          }
        }
      }
      fLse[q * S::HP + h] *= kLog2e;
      fCoff[q * S::HP + h] = c;
    }
    // qt = [q * scale] into the union region (head-warp fragments), its valid
    // rows to the workspace for the column kernel.
    for (int idx = threadIdx.x; idx < NH * S::BM * QCH; idx += nthreads) {
      const int c = idx % QCH, q = (idx / QCH) % S::BM, h = idx / (QCH * S::BM);
      const uint32_t off = h * S::BM * S::RBD + swz<S::RBD>(q, c);
      uint4 v = *(const uint4*)(smem + S::OFF_QR + off);
      uint32_t* w = (uint32_t*)&v;
#pragma unroll
      for (int k = 0; k < 4; ++k) w[k] = E::pack(E::lo(w[k]) * p.scale, E::hi(w[k]) * p.scale);
      *(uint4*)(smem + S::OFF_Q + off) = v;
      if (q < nvalid_q) *(uint4*)(qt_ws + ev_off(ev, q0 + q, h0 + h, DH) + c * 8) = v;
    }
    // u = (q * scale) W and w~ = dO W (one head per warp, tensor cores) into
    // the resident tiles and the workspace (for the column kernel).
    if (warp < NH) {
      const uint32_t sW = sm + S::OFF_W, sWlo = sW + DH * S::RBC;
      if (proj_u)
        project_mma<T, DH, C, S::CP, S::RBD, S::BM>(sm + S::OFF_QR + warp * S::BM * S::RBD, sW,
                                                    sWlo, p.scale, ev, q0, nvalid_q, h0 + warp,
                                                    warp, smem + S::OFF_U, u_ws);
      if (proj_w)
        project_mma<T, DH, C, S::CP, S::RBD, S::BM>(sm + S::OFF_DOR + warp * S::BM * S::RBD, sW,
                                                    sWlo, 1.f, ev, q0, nvalid_q, h0 + warp, warp,
                                                    smem + S::OFF_WT, wt_ws);
    }
    __syncthreads();
    if (warp < NH) {
#pragma unroll
      for (int ks = 0; ks < S::KSD; ++ks) {
        const int mi = lane >> 3;
        const int q = (mi & 1) * 8 + (lane & 7);
        const uint32_t off = warp * S::BM * S::RBD + swz<S::RBD>(q, 2 * ks + (mi >> 1));
        ldsm_x4(sm + S::OFF_Q + off, qa[ks]);
        ldsm_x4(sm + S::OFF_DOR + off, da[ks]);
      }
    }
    __syncthreads();  // the loop's bias tiles reuse the scaled-Q bytes
  } else {
    // ------------------------------- prologue -------------------------------
    {
      constexpr int QCH = DH / 8;
      for (int idx = threadIdx.x; idx < NH * S::BM * QCH; idx += nthreads) {
        const int c = idx % QCH, q = (idx / QCH) % S::BM, h = idx / (QCH * S::BM);
        uint4 vq = make_uint4(0, 0, 0, 0), vd = make_uint4(0, 0, 0, 0);
        if (q < nvalid_q) {  // raw q (scaled in place after the projections)
          const int64_t go = ev_off(ev, q0 + q, h0 + h, DH) + c * 8;
          vq = *(const uint4*)(gq + ev_off(evq, q0 + q, h0 + h, DH) + c * 8);
          vd = *(const uint4*)(gdo + go);
        }
        const uint32_t off = h * S::BM * S::RBD + swz<S::RBD>(q, c);
        *(uint4*)(smem + S::OFF_Q + off) = vq;
        *(uint4*)(smem + S::OFF_DO + off) = vd;
      }
      // W as [d][c], split into hi + lo halves of the 16-bit type: operand of
      // the projections below and of R = H W^T in the epilogue.
      for (int idx = threadIdx.x; idx < DH * (S::CP / 2); idx += nthreads) {
        const int c2 = idx % (S::CP / 2), d = idx / (S::CP / 2);
        float w0 = 0.f, w1 = 0.f;
        if ((attn || act) && 2 * c2 < C) {
          w0 = p.weight[(int64_t)d * C + 2 * c2];
          w1 = p.weight[(int64_t)d * C + 2 * c2 + 1];
        }
        const uint32_t hi = E::pack(w0, w1);
        const uint32_t lo = E::pack(w0 - E::lo(hi), w1 - E::hi(hi));
        const uint32_t off = swz<S::RBC>(d, c2 / 4) + (c2 % 4) * 4;
        *(uint32_t*)(smem + S::OFF_W + off) = hi;
        *(uint32_t*)(smem + S::OFF_W + DH * S::RBC + off) = lo;
      }
    }
    __syncthreads();
    // Per (row, head): LSE in log2 units and the row offset c = dO.(out - [act] b),
    // dO from the staged tile and out with 16-byte loads (d in order).
    for (int idx = threadIdx.x; idx < S::BM * NH; idx += nthreads) {
      const int q = idx / NH, h = idx % NH;
      float l2 = 0.f, c = 0.f;
      if (q < nvalid_q) {
        l2 = a.lse[ev_off(ev, q0 + q, h0 + h, 1)] * kLog2e;
        if (gout) {
          const T* orow = gout + ev_off(ev, q0 + q, h0 + h, DH);
          const unsigned char* drow = smem + S::OFF_DO + h * S::BM * S::RBD;
#pragma unroll
          for (int ch = 0; ch < DH / 8; ++ch) {
            const uint4 ov = *(const uint4*)(orow + ch * 8);
            const uint4 dv = *(const uint4*)(drow + swz<S::RBD>(q, ch));
            const uint32_t* o2 = (const uint32_t*)&ov;
            const uint32_t* d2 = (const uint32_t*)&dv;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              float o0 = E::lo(o2[e]), o1 = E::hi(o2[e]);
              if (act && p.bias) {
                o0 -= p.bias[ch * 8 + 2 * e];
                o1 -= p.bias[ch * 8 + 2 * e + 1];
              }
              c = fmaf(E::lo(d2[e]), o0, c);
              c = fmaf(E::hi(d2[e]), o1, c);
            }
          }
        }
      }
      fLse[q * S::HP + h] = l2;
      fCoff[q * S::HP + h] = c;
    }
    // u = (q * scale) W and w~ = dO W from the staged raw rows (one head per
    // warp, on the tensor cores), unless the caller passed them; they go to the
    // workspace, where phase 2 below and the column kernel read them.
    if (warp < NH) {
      const uint32_t sW = sm + S::OFF_W, sWlo = sW + DH * S::RBC;
      if (attn && a.u == nullptr)
        project_mma<T, DH, C, S::CP, S::RBD, S::BM>(sm + S::OFF_Q + warp * S::BM * S::RBD, sW,
                                                    sWlo, p.scale, ev, q0, nvalid_q, h0 + warp,
                                                    warp, nullptr, u_ws);
      if (act && a.wt == nullptr)
        project_mma<T, DH, C, S::CP, S::RBD, S::BM>(sm + S::OFF_DO + warp * S::BM * S::RBD, sW,
                                                    sWlo, 1.f, ev, q0, nvalid_q, h0 + warp, warp,
                                                    nullptr, wt_ws);
    }
    __syncthreads();
    scale_staged<T, DH, S::RBD>(smem + S::OFF_Q, NH, S::BM, p.scale);  // qt = [q * scale]
    __syncthreads();
    {
      // qt of the valid rows to the workspace, for the column kernel.
      constexpr int QCH = DH / 8;
      for (int idx = threadIdx.x; idx < NH * nvalid_q * QCH; idx += nthreads) {
        const int c = idx % QCH, q = (idx / QCH) % nvalid_q, h = idx / (QCH * nvalid_q);
        *(uint4*)(qt_ws + ev_off(ev, q0 + q, h0 + h, DH) + c * 8) =
            *(const uint4*)(smem + S::OFF_Q + h * S::BM * S::RBD + swz<S::RBD>(q, c));
      }
    }
    if (warp < NH) {
#pragma unroll
      for (int ks = 0; ks < S::KSD; ++ks) {
        const int mi = lane >> 3;
        const int q = (mi & 1) * 8 + (lane & 7);
        const uint32_t off = warp * S::BM * S::RBD + swz<S::RBD>(q, 2 * ks + (mi >> 1));
        ldsm_x4(sm + S::OFF_Q + off, qa[ks]);
        ldsm_x4(sm + S::OFF_DO + off, da[ks]);
      }
    }
    __syncthreads();  // phase 2 of the staging reuses the Q / dO bytes
    {
      if (attn)
        stage_rows<T, C, S::CP>(a.u ? (const T*)a.u : u_ws, ev, q0, nvalid_q, S::BM, h0, NH,
                                smem + S::OFF_U);
      if (act)
        stage_rows<T, C, S::CP>(a.wt ? (const T*)a.wt : wt_ws, ev, q0, nvalid_q, S::BM, h0, NH,
                                smem + S::OFF_WT);
      for (int idx = threadIdx.x; idx < S::BM * 4; idx += nthreads) {
        const int q = idx / 4, k = idx % 4;
        fQC[idx] = q < nvalid_q ? p.feats[(ev.row0 + q0 + q) * p.feat_stride + k] : 0.f;
      }
    }
    __syncthreads();
    if (warp >= NH && !idle) {
      const int qe = (warp - NH) * S::QPE;
#pragma unroll
      for (int t = 0; t < S::QPE; ++t)
#pragma unroll
        for (int ks = 0; ks < S::KSC; ++ks) {
          const int mi = lane >> 3;
          const int h = (mi & 1) * 8 + (lane & 7);
          const uint32_t off = swz<S::RBC>((qe + t) * 16 + h, 2 * ks + (mi >> 1));
          if (!S::AHEAD) {
            ldsm_x4(sm + S::OFF_U + off, ua[t][ks]);
            ldsm_x4(sm + S::OFF_WT + off, wa[t][ks]);
          }
        }
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < 4 * S::SZ_P / 4; idx += nthreads)
      ((uint32_t*)(smem + S::OFF_P))[idx] = 0u;
    __syncthreads();
  }

  if (idle) {
    // Surplus warps of a short head group: no role in the key loop, but they
    // keep the CTA-wide barrier count and help with the cooperative epilogue.
    __syncthreads();  // (A)
  } else if (warp >= NH) {
    // =============================== E warps ==============================
    const int e = warp - NH;
    const int qe = e * S::QPE;
    float fr[S::FG][2], fv[S::FG][2];  // f and f / (2 pi) of this lane's frequencies
#pragma unroll
    for (int g = 0; g < S::FG; ++g) {
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        fr[g][r] = p.freqs[8 * g + 2 * m4 + r];
        fv[g][r] = fr[g][r] * 0.15915494309189535f;
      }
    }
    // Each lane of a quad forms the interval angle of one (query, 8-key
    // tile) pair of the warp's QPE (<= 2) queries and the chunk's two key
    // tiles: lane m4 takes query m4 % QPE and tile m4 / QPE % 2, and the
    // others read it by shuffle (no angle is formed twice).
    static_assert(S::QPE <= 2, "one angle per lane");
    const int my_t = m4 % S::QPE, my_nt = (m4 / S::QPE) & 1;
    const int qx_row = qe + my_t;
    Coord4 cq;
    cq.x = fQC[qx_row * 4 + 0];
    cq.y = fQC[qx_row * 4 + 1];
    cq.z = fQC[qx_row * 4 + 2];
    cq.t = fQC[qx_row * 4 + 3];
    const uint32_t c_ring = sm + S::OFF_C + e * 2 * S::BN * 16;
    const float* __restrict__ fbase = p.feats + ev.row0 * p.feat_stride;
    auto load_coords = [&](int n) {
      if (n < nchunks && lane < S::BN) {
        const int j = n * S::BN + lane;
        const uint32_t dst = c_ring + ((n & 1) * S::BN + lane) * 16;
        if (j < ev.len)
          cp_async16(dst, fbase + j * p.feat_stride);
        else
          asm volatile("st.shared.v4.u32 [%0], {%1,%1,%1,%1};\n" ::"r"(dst), "r"(0));
      }
      cp_async_commit();
    };
    load_coords(0);
    load_coords(1);

    float hacc[S::QPE][S::NTC][4], gacc[S::QPE][S::NTC][4];
#pragma unroll
    for (int t = 0; t < S::QPE; ++t)
#pragma unroll
      for (int nc = 0; nc < S::NTC; ++nc)
#pragma unroll
        for (int i = 0; i < 4; ++i) hacc[t][nc][i] = gacc[t][nc][i] = 0.f;

    // With S::AHEAD the E warps run one chunk ahead: chunk n+1's embedding
    // and bias are produced before waiting for the head warps' P of chunk n,
    // so the head warps' work on chunk n overlaps the embedding of chunk n+1.
    using EFrag = uint32_t[S::QPE][2][S::KSC][2];  // E B-fragments (k = channel, n = key)
    // Embedding of chunk n into eb and its (u.E, w~.E) bias into stage n & 1.
    auto produce = [&](int n, int s, EFrag& eb) {
      cp_async_wait<1>();
      __syncwarp();
      float x1;
      {
        const float4 ck =
            *(const float4*)(smem + S::OFF_C + (e * 2 * S::BN + s * S::BN + my_nt * 8 + r8) * 16);
        Coord4 c4;
        c4.x = ck.x;
        c4.y = ck.y;
        c4.z = ck.z;
        c4.t = ck.w;
        x1 = pair_angle_fast(cq, c4);
      }
      __syncwarp();
      load_coords(n + 2);

      if (n >= 2) named_sync(rb_bias_empty(s), NBAR);
#pragma unroll
      for (int t = 0; t < S::QPE; ++t) {
        float sn[2][S::FG][2], cs[2][S::FG][2];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          const float xt = __shfl_sync(0xffffffffu, x1, (lane & ~3) | (t + S::QPE * nt));
#pragma unroll
          for (int g = 0; g < S::FG; ++g)
            sincos_xf2(xt, fr[g], fv[g], sn[nt][g], cs[nt][g]);
        }
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int ks = 0; ks < S::KSC; ++ks)
#pragma unroll
            for (int hi = 0; hi < 2; ++hi) {
              const int cb = 16 * ks + 8 * hi;
              const int g = (cb % S::F) / 8;
              const bool is_sin = cb < S::F;
              eb[t][nt][ks][hi] = E::pack(is_sin ? sn[nt][g][0] : cs[nt][g][0],
                                          is_sin ? sn[nt][g][1] : cs[nt][g][1]);
            }
        const int q = qe + t;
        if constexpr (S::AHEAD) {
#pragma unroll
          for (int ks = 0; ks < S::KSC; ++ks) {
            const int mi = lane >> 3;
            const int h = (mi & 1) * 8 + (lane & 7);
            const uint32_t off = swz<S::RBC>(q * 16 + h, 2 * ks + (mi >> 1));
            if (attn) ldsm_x4(sm + S::OFF_U + off, ua[t][ks]);
            if (act) ldsm_x4(sm + S::OFF_WT + off, wa[t][ks]);
          }
        }
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          float du[4] = {0.f, 0.f, 0.f, 0.f}, dw[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int ks = 0; ks < S::KSC; ++ks) {
            if (attn) mma16816<T>(du, ua[t][ks], eb[t][nt][ks]);
            if (act) mma16816<T>(dw, wa[t][ks], eb[t][nt][ks]);
          }
          // (u.E, w~.E) pairs for keys 2 m4 and 2 m4 + 1 of this 8-key tile.
          const uint32_t base = sm + S::OFF_B + s * S::SZ_B + (q * S::BQ + nt * 16 + 4 * m4) * 4;
          if (r8 < NH)
            asm volatile("st.shared.v4.f32 [%0], {%1,%2,%3,%4};\n" ::"r"(base + r8 * S::BROW * 4),
                         "f"(du[0]), "f"(dw[0]), "f"(du[1]), "f"(dw[1]));
          if (r8 + 8 < NH)
            asm volatile("st.shared.v4.f32 [%0], {%1,%2,%3,%4};\n" ::"r"(base + (r8 + 8) * S::BROW * 4),
                         "f"(du[2]), "f"(dw[2]), "f"(du[3]), "f"(dw[3]));
        }
      }
      named_arrive(rb_bias_full(s), NBAR);
    };
    // H' += [P dP'] E and G += [P] E for chunk n.
    auto consume = [&](int n, int s, const EFrag& eb) {
      named_sync(rb_p_full(s), NBAR);
#pragma unroll
      for (int t = 0; t < S::QPE; ++t) {
        const int q = qe + t;
        uint32_t pp[4], pd[4];
        const int mi = lane >> 3;
        const int h = (mi & 1) * 8 + (lane & 7);
        const uint32_t po = (q * S::PQ + h * S::PH + (mi >> 1) * 4) * 4;
        ldsm_x4(sm + S::OFF_P + (2 * s) * S::SZ_P + po, pp);
        ldsm_x4(sm + S::OFF_P + (2 * s + 1) * S::SZ_P + po, pd);
#pragma unroll
        for (int nc = 0; nc < S::NTC; ++nc) {
          uint32_t bt[2];
          bt[0] = movm_t(eb[t][0][nc >> 1][nc & 1]);
          bt[1] = movm_t(eb[t][1][nc >> 1][nc & 1]);
          // G is needed for dW when the output term is on, and for the
          // D' correction of H when the logit term is on.
          mma16816<T>(gacc[t][nc], pp, bt);
          if (attn) mma16816<T>(hacc[t][nc], pd, bt);
        }
      }
      if (n + 2 < nchunks) named_arrive(rb_p_empty(s), NBAR);
    };

    if constexpr (S::AHEAD) {
      EFrag eb0, eb1;
      produce(0, 0, eb0);
      for (int n = 0; n < nchunks; n += 2) {
        if (n + 1 < nchunks) produce(n + 1, 1, eb1);
        consume(n, 0, eb0);
        if (n + 1 >= nchunks) break;
        if (n + 2 < nchunks) produce(n + 2, 0, eb0);
        consume(n + 1, 1, eb1);
      }
    } else {
      EFrag eb0;
      for (int n = 0; n < nchunks; ++n) {
        produce(n, n & 1, eb0);
        consume(n, n & 1, eb0);
      }
    }

    __syncthreads();  // (A) head warps published D'
    // H = H' - D' G, stored fp32 [q][h][c] with G for the dW partial; then
    // R = H W^T (hi/lo split of both H and W) into [q][h][d].
    float* fH = (float*)(smem + S::OFF_H);
    float* fG = (float*)(smem + S::OFF_G);
    float* fR = (float*)(smem + S::OFF_R);  // K/V ring, dead after the loop
#pragma unroll
    for (int t = 0; t < S::QPE; ++t) {
      const int q = qe + t;
      const float d0 = r8 < NH ? fDp[q * S::HP + r8] : 0.f;
      const float d1 = r8 + 8 < NH ? fDp[q * S::HP + r8 + 8] : 0.f;
#pragma unroll
      for (int nc = 0; nc < S::NTC; ++nc) {
        hacc[t][nc][0] -= d0 * gacc[t][nc][0];
        hacc[t][nc][1] -= d0 * gacc[t][nc][1];
        hacc[t][nc][2] -= d1 * gacc[t][nc][2];
        hacc[t][nc][3] -= d1 * gacc[t][nc][3];
        const int c = nc * 8 + 2 * m4;
        if (r8 < NH) {
          fH[(q * S::HP + r8) * C + c] = hacc[t][nc][0];
          fH[(q * S::HP + r8) * C + c + 1] = hacc[t][nc][1];
          fG[(q * S::HP + r8) * C + c] = gacc[t][nc][0];
          fG[(q * S::HP + r8) * C + c + 1] = gacc[t][nc][1];
        }
        if (r8 + 8 < NH) {
          fH[(q * S::HP + r8 + 8) * C + c] = hacc[t][nc][2];
          fH[(q * S::HP + r8 + 8) * C + c + 1] = hacc[t][nc][3];
          fG[(q * S::HP + r8 + 8) * C + c] = gacc[t][nc][2];
          fG[(q * S::HP + r8 + 8) * C + c + 1] = gacc[t][nc][3];
        }
      }
      if (attn) {
        uint32_t ah[S::KSC][4], al[S::KSC][4];
#pragma unroll
        for (int ks = 0; ks < S::KSC; ++ks) {
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            const float* hv = hacc[t][2 * ks + half];
            const uint32_t h01 = E::pack(hv[0], hv[1]);
            const uint32_t h23 = E::pack(hv[2], hv[3]);
            ah[ks][2 * half] = h01;
            ah[ks][2 * half + 1] = h23;
            al[ks][2 * half] = E::pack(hv[0] - E::lo(h01), hv[1] - E::hi(h01));
            al[ks][2 * half + 1] = E::pack(hv[2] - E::lo(h23), hv[3] - E::hi(h23));
          }
        }
#pragma unroll
        for (int nd = 0; nd < S::NTD; ++nd) {
          float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int ks = 0; ks < S::KSC; ++ks) {
            uint32_t wh[2], wl[2];
            const int mi = (lane >> 3) & 1;
            const uint32_t wo = swz<S::RBC>(nd * 8 + (lane & 7), 2 * ks + mi);
            ldsm_x2(sm + S::OFF_W + wo, wh);
            ldsm_x2(sm + S::OFF_W + DH * S::RBC + wo, wl);
            mma16816<T>(d, ah[ks], wh);
            mma16816<T>(d, ah[ks], wl);
            mma16816<T>(d, al[ks], wh);
          }
          const int dd = nd * 8 + 2 * m4;
          if (r8 < NH) {
            fR[(q * S::HP + r8) * DH + dd] = d[0];
            fR[(q * S::HP + r8) * DH + dd + 1] = d[1];
          }
          if (r8 + 8 < NH) {
            fR[(q * S::HP + r8 + 8) * DH + dd] = d[2];
            fR[(q * S::HP + r8 + 8) * DH + dd + 1] = d[3];
          }
        }
      }
    }
  } else {
    // ============================== head warps ============================
    const int hl = warp;
    const int h = h0 + hl;
    const uint32_t k_ring = sm + S::OFF_K + hl * S::BN * S::RBD;
    const uint32_t v_ring = sm + S::OFF_V + hl * S::BN * S::RBD;
    // TMA ring (as in the forward): one mbarrier per stage; the box origin is
    // this head's first column and the event's row of key 0 in the row view.
    const uint32_t mbar = sm + S::OFF_MB + hl * 16;
    const int tx = rows_interleaved(p) ? h * DH : 0;
    const int ty = rows_interleaved(p) ? (int)evq.row0 : (int)(evq.base1 + h * evq.hs1);
    bool tma_late = false;
    const bool ring_tma = S::TMA && ((sm + S::OFF_K) & 1023u) == 0;
    if (ring_tma) {
      if (lane == 0) {
        mbar_init(mbar, 1);
        mbar_init(mbar + 8, 1);
        mbar_init_fence();
      }
      __syncwarp();
    }
    auto load_kv = [&](int n) {
      if (ring_tma) {
        if (n < nchunks && lane == 0) {
          const int st = n & 1;
          const uint32_t bar = mbar + 8 * st;
          fence_proxy_async();
          mbar_arrive_tx(bar, 2 * S::BN * DH * (int)sizeof(T));
          tma_load_2d(k_ring + st * S::SZ_KV, &kv_maps.a, bar, tx, ty + n * S::BN);
          tma_load_2d(v_ring + st * S::SZ_KV, &kv_maps.b, bar, tx, ty + n * S::BN);
        }
        return;
      }
      if (n < nchunks) {
        // K / V of this head: event base pointer and row stride (formed here,
        // so they hold no registers across the TMA path's loop).
        const T* __restrict__ kbase = gk + ev_off(evq, 0, h, DH);
        const T* __restrict__ vbase = gv + ev_off(evq, 0, h, DH);
        const int rs = qkv_row_stride(p, DH);
        constexpr int CH = DH / 8;
        const int j0 = n * S::BN;
        const uint32_t ks_ = k_ring + (n & 1) * S::SZ_KV, vs_ = v_ring + (n & 1) * S::SZ_KV;
        for (int idx = lane; idx < S::BN * CH; idx += 32) {
          const int c = idx % CH, j = idx / CH;
          const uint32_t off = swz<S::RBD>(j, c);
          if (j0 + j < ev.len) {
            const int go = (j0 + j) * rs + c * 8;
            cp_async16(ks_ + off, kbase + go);
            cp_async16(vs_ + off, vbase + go);
          } else {
            asm volatile("st.shared.v4.u32 [%0], {%1,%1,%1,%1};\n" ::"r"(ks_ + off), "r"(0));
            asm volatile("st.shared.v4.u32 [%0], {%1,%1,%1,%1};\n" ::"r"(vs_ + off), "r"(0));
          }
        }
      }
      cp_async_commit();
    };
    load_kv(0);
    load_kv(1);
    const float lse0 = fLse[r8 * S::HP + hl], lse1 = fLse[(r8 + 8) * S::HP + hl];
    const float c0 = fCoff[r8 * S::HP + hl], c1 = fCoff[(r8 + 8) * S::HP + hl];
    float X[S::NTD][4], Y[S::NTD][4];
#pragma unroll
    for (int nd = 0; nd < S::NTD; ++nd)
#pragma unroll
      for (int i = 0; i < 4; ++i) X[nd][i] = Y[nd][i] = 0.f;
    // Row sums of [P] and [P dP'] as MMAs against a ones B-fragment: the
    // tensor core adds exactly the rounded values the X / Y products consume,
    // and every lane ends with the full sums of rows r8 (slot 0) and r8 + 8
    // (slot 2).
    float pacc[4] = {0.f, 0.f, 0.f, 0.f}, aacc[4] = {0.f, 0.f, 0.f, 0.f};
    const uint32_t ones[2] = {E::kOnes, E::kOnes};

    // One key chunk; the stage s = n & 1 is passed as a literal.
    auto step = [&](int n, int s) {
      const int j0 = n * S::BN;
      const uint32_t k_st = k_ring + s * S::SZ_KV, v_st = v_ring + s * S::SZ_KV;
      if (ring_tma) {
        if (!mbar_wait(mbar + 8 * s, (n >> 1) & 1)) tma_late = true;
        if (j0 + S::BN > ev.len) {  // keys past the event must be exact zeros
          constexpr int CH = DH / 8;
          for (int idx = lane; idx < S::BN * CH; idx += 32) {
            const int c = idx % CH, j = idx / CH;
            if (j0 + j >= ev.len) {
              asm volatile("st.shared.v4.u32 [%0], {%1,%1,%1,%1};\n" ::"r"(k_st + swz<S::RBD>(j, c)), "r"(0));
              asm volatile("st.shared.v4.u32 [%0], {%1,%1,%1,%1};\n" ::"r"(v_st + swz<S::RBD>(j, c)), "r"(0));
            }
          }
        }
      } else {
        cp_async_wait<1>();
      }
      __syncwarp();
      // S = Q K^T and dP = dO V^T (B fragments: k = head dim, n = key).
      float sc[2][4], dp[2][4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
        for (int i = 0; i < 4; ++i) sc[nt][i] = dp[nt][i] = 0.f;
#pragma unroll
        for (int kp = 0; kp < (S::KSD + 1) / 2; ++kp) {
          const int mi = lane >> 3;
          uint32_t rk[4], rv[4];
          if (S::KSD - 2 * kp >= 2) {
            const uint32_t off = swz<S::RBD>(nt * 8 + (lane & 7), 4 * kp + mi);
            ldsm_x4(k_st + off, rk);
            ldsm_x4(v_st + off, rv);
            mma16816<T>(sc[nt], qa[2 * kp], rk);
            mma16816<T>(sc[nt], qa[2 * kp + 1], rk + 2);
            mma16816<T>(dp[nt], da[2 * kp], rv);
            mma16816<T>(dp[nt], da[2 * kp + 1], rv + 2);
          } else {
            const uint32_t off = swz<S::RBD>(nt * 8 + (lane & 7), 4 * kp + (mi & 1));
            ldsm_x2(k_st + off, rk);
            ldsm_x2(v_st + off, rv);
            mma16816<T>(sc[nt], qa[2 * kp], rk);
            mma16816<T>(dp[nt], da[2 * kp], rv);
          }
        }
      }
      named_sync(rb_bias_full(s), NBAR);
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const uint32_t base = sm + S::OFF_B + s * S::SZ_B + (hl * S::BROW + nt * 16 + 4 * m4) * 4;
        float4 b0, b1;
        asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];\n"
                     : "=f"(b0.x), "=f"(b0.y), "=f"(b0.z), "=f"(b0.w)
                     : "r"(base + r8 * S::BQ * 4));
        asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];\n"
                     : "=f"(b1.x), "=f"(b1.y), "=f"(b1.z), "=f"(b1.w)
                     : "r"(base + (r8 + 8) * S::BQ * 4));
        sc[nt][0] += b0.x;
        dp[nt][0] += b0.y;
        sc[nt][1] += b0.z;
        dp[nt][1] += b0.w;
        sc[nt][2] += b1.x;
        dp[nt][2] += b1.y;
        sc[nt][3] += b1.z;
        dp[nt][3] += b1.w;
      }
      if (n + 2 < nchunks) named_arrive(rb_bias_empty(s), NBAR);

      // P = exp(s - lse), dP' = dP - c; masked keys get P = 0.
      uint32_t pp[4], pd[4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) sc[nt][i] = ex2(fmaf(sc[nt][i], kLog2e, (i >> 1) ? -lse1 : -lse0));
      if (j0 + S::BN > ev.len) {  // keys past the event: last chunk only
        const int lim = ev.len - j0 - 2 * m4;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int i = 0; i < 4; ++i)
            if (nt * 8 + (i & 1) >= lim) sc[nt][i] = 0.f;
      }
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) dp[nt][i] = sc[nt][i] * (dp[nt][i] - ((i >> 1) ? c1 : c0));
      // A fragments (rows on M, keys on K) of [P] and [P dP'].
      pp[0] = E::pack(sc[0][0], sc[0][1]);
      pp[1] = E::pack(sc[0][2], sc[0][3]);
      pp[2] = E::pack(sc[1][0], sc[1][1]);
      pp[3] = E::pack(sc[1][2], sc[1][3]);
      pd[0] = E::pack(dp[0][0], dp[0][1]);
      pd[1] = E::pack(dp[0][2], dp[0][3]);
      pd[2] = E::pack(dp[1][0], dp[1][1]);
      pd[3] = E::pack(dp[1][2], dp[1][3]);
      mma16816<T>(pacc, pp, ones);
      mma16816<T>(aacc, pd, ones);

      if (n >= 2) named_sync(rb_p_empty(s), NBAR);
      {
        const uint32_t pb = sm + S::OFF_P + (2 * s) * S::SZ_P + (hl * S::PH + m4) * 4;
        const uint32_t db = sm + S::OFF_P + (2 * s + 1) * S::SZ_P + (hl * S::PH + m4) * 4;
        sts_u32(pb + r8 * S::PQ * 4, pp[0]);
        sts_u32(pb + r8 * S::PQ * 4 + 16, pp[2]);
        sts_u32(pb + (r8 + 8) * S::PQ * 4, pp[1]);
        sts_u32(pb + (r8 + 8) * S::PQ * 4 + 16, pp[3]);
        sts_u32(db + r8 * S::PQ * 4, pd[0]);
        sts_u32(db + r8 * S::PQ * 4 + 16, pd[2]);
        sts_u32(db + (r8 + 8) * S::PQ * 4, pd[1]);
        sts_u32(db + (r8 + 8) * S::PQ * 4 + 16, pd[3]);
      }
      named_arrive(rb_p_full(s), NBAR);

      // X += [P dP'] K, Y += [P] K (B fragments: k = key, n = head dim).
#pragma unroll
      for (int np = 0; np < (S::NTD + 1) / 2; ++np) {
        const int mi = lane >> 3;
        uint32_t r[4];
        if (S::NTD - 2 * np >= 2) {
          ldsm_x4_t(k_st + swz<S::RBD>((mi & 1) * 8 + (lane & 7), 2 * np + (mi >> 1)), r);
          mma16816<T>(X[2 * np], pd, r);
          mma16816<T>(X[2 * np + 1], pd, r + 2);
          mma16816<T>(Y[2 * np], pp, r);
          mma16816<T>(Y[2 * np + 1], pp, r + 2);
        } else {
          ldsm_x2_t(k_st + swz<S::RBD>((mi & 1) * 8 + (lane & 7), 2 * np), r);
          mma16816<T>(X[2 * np], pd, r);
          mma16816<T>(Y[2 * np], pp, r);
        }
      }
      __syncwarp();
      load_kv(n + 2);
    };
    if constexpr (S::LIT) {
      for (int n = 0; n < nchunks; n += 2) {
        step(n, 0);
        if (n + 1 < nchunks) step(n + 1, 1);
      }
    } else {
      for (int n = 0; n < nchunks; ++n) step(n, n & 1);
    }
    if (ring_tma) {
      // A ring wait that gave up leaves its copy in flight: wait (bounded) for
      // the last copy of each stage before the ring is reused, and flag this
      // warp's rows (delta = NaN) below.
      tma_late = __any_sync(0xffffffffu, tma_late);
      if (tma_late)
        for (int st = 0; st < 2 && st < nchunks; ++st) {
          const int last = nchunks - 1 - ((nchunks - 1 - st) & 1);
          mbar_wait(mbar + 8 * st, (last >> 1) & 1);
        }
    }

    // D' = a / p, sigma = a - D' p, dqp = X - D' Y (rows r8 and r8 + 8).
    float dpr[2], sig[2];
#pragma unroll
    for (int rh = 0; rh < 2; ++rh) {
      const float av = aacc[2 * rh], pv = pacc[2 * rh];
      dpr[rh] = pv > 0.f ? av / pv : 0.f;
      sig[rh] = av - dpr[rh] * pv;
      if (m4 == 0) fDp[(r8 + 8 * rh) * S::HP + hl] = dpr[rh];
    }
#pragma unroll
    for (int nd = 0; nd < S::NTD; ++nd) {
      X[nd][0] -= dpr[0] * Y[nd][0];
      X[nd][1] -= dpr[0] * Y[nd][1];
      X[nd][2] -= dpr[1] * Y[nd][2];
      X[nd][3] -= dpr[1] * Y[nd][3];
    }
    __syncthreads();  // (A) D' published
    __syncthreads();  // (B) E warps published H, G, R
    const float* fR = (const float*)(smem + S::OFF_R);
#pragma unroll
    for (int rh = 0; rh < 2; ++rh) {
      const int q = r8 + 8 * rh;
      const bool valid = q < nvalid_q;
      if (!valid && (uses_tile_list(p) || q0 + q >= p.max_len)) continue;
      T* orow = gdq + ev_off(evq, q0 + q, h, DH);
#pragma unroll
      for (int nd = 0; nd < S::NTD; ++nd) {
        const int d = nd * 8 + 2 * m4;
        float v0 = X[nd][2 * rh], v1 = X[nd][2 * rh + 1];
        if (attn) {
          v0 += fR[(q * S::HP + hl) * DH + d];
          v1 += fR[(q * S::HP + hl) * DH + d + 1];
          if (p.bias) {
            v0 += sig[rh] * p.bias[d];
            v1 += sig[rh] * p.bias[d + 1];
          }
        }
        v0 = valid ? v0 * p.scale : 0.f;
        v1 = valid ? v1 * p.scale : 0.f;
        *(uint32_t*)(orow + d) = E::pack(v0, v1);
      }
      if (m4 == 0) {
        const int64_t so = ev_off(ev, q0 + q, h, 1);
        a.delta[so] = tma_late ? __int_as_float(0x7fc00000)  // a K/V copy never landed
                      : valid  ? fCoff[q * S::HP + hl] + dpr[rh]
                               : 0.f;
        a.sigma[so] = valid ? sig[rh] : 0.f;
      }
    }
  }
  if (warp >= NH) __syncthreads();  // (B) from the E-warp and idle-warp side
  // Raw q and dO as [head][row][DHP] swizzled tiles (rows past the event are
  // zero) for the dW / db partials: resident since the prologue on the fast
  // path; otherwise staged again into the K/V ring once R is consumed.
  const uint32_t sq = S::FASTPRO ? sm + S::OFF_QR : sm + S::OFF_K;
  const uint32_t sdo = S::FASTPRO ? sm + S::OFF_DOR : sq + S::HP * S::BM * S::RBD;
  if constexpr (!S::FASTPRO) {
    __syncthreads();  // (C) head warps are done with R; the K/V ring is free
    constexpr int CH = DH / 8;
    for (int idx = threadIdx.x; idx < NH * S::BM * CH; idx += nthreads) {
      const int c = idx % CH, q = (idx / CH) % S::BM, hl = idx / (CH * S::BM);
      uint4 vq = make_uint4(0, 0, 0, 0), vd = make_uint4(0, 0, 0, 0);
      if (q < nvalid_q) {
        const int64_t go = ev_off(ev, q0 + q, h0 + hl, DH) + c * 8;
        vq = *(const uint4*)(gq + ev_off(evq, q0 + q, h0 + hl, DH) + c * 8);
        vd = *(const uint4*)(gdo + go);
      }
      const uint32_t so = hl * S::BM * S::RBD + swz<S::RBD>(q, c);
      *(uint4*)(smem + (sq - sm) + so) = vq;
      *(uint4*)(smem + (sdo - sm) + so) = vd;
    }
    __syncthreads();  // (D)
  }
  // dW and db partials of this CTA (backward.py:607-622) on the tensor cores,
  // one (16 d x 8 c) output tile per warp, K running over (head, row) in a
  // fixed order:
  //   dW = scale * sum q^T H + sum dO^T G,   db = sum dO  (= dO^T 1),
  // with q, dO exact in T and H, G split into hi + lo halves of T.
  {
    constexpr int MT = DH / 16, NTW = C / 8;
    const float* fH = (const float*)(smem + S::OFF_H);
    const float* fG = (const float*)(smem + S::OFF_G);
    const int nwarps = nthreads >> 5;
    const int mi = lane >> 3;
    const uint32_t ones[2] = {E::kOnes, E::kOnes};
    // On the fast path the tiles go to the last warps (E and idle warps), which
    // run them while the head warps write dq.
    const int first = S::FASTPRO ? nwarps - 1 - warp : warp;
    for (int tile = first; tile < MT * NTW; tile += nwarps) {
      const int mt = tile / NTW, nt = tile % NTW;
      const int c = nt * 8 + r8;  // this lane's B column
      // A = x^T (m = d, k = row) from the [row][d] tile by transposed loads.
      const uint32_t aoff = swz<S::RBD>((mi >> 1) * 8 + (lane & 7), 2 * mt + (mi & 1));
      float aq[4] = {0.f, 0.f, 0.f, 0.f}, ad[4] = {0.f, 0.f, 0.f, 0.f};
      float ab[4] = {0.f, 0.f, 0.f, 0.f};
      for (int hl = 0; hl < NH; ++hl) {
        uint32_t fq[4], fd[4];
        ldsm_x4_t(sq + hl * S::BM * S::RBD + aoff, fq);
        ldsm_x4_t(sdo + hl * S::BM * S::RBD + aoff, fd);
        // B (k = row, n = channel): rows 2 m4 (+1) and 2 m4 + 8 (+1).
        float hv[4], gv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int q = 2 * m4 + (i & 1) + 8 * (i >> 1);
          const bool ok = q < nvalid_q;
          hv[i] = ok ? fH[(q * S::HP + hl) * C + c] : 0.f;
          gv[i] = ok ? fG[(q * S::HP + hl) * C + c] : 0.f;
        }
        if (attn) {
          uint32_t bh[2], bl[2];
#pragma unroll
          for (int r = 0; r < 2; ++r) {
            bh[r] = E::pack(hv[2 * r], hv[2 * r + 1]);
            bl[r] = E::pack(hv[2 * r] - E::lo(bh[r]), hv[2 * r + 1] - E::hi(bh[r]));
          }
          mma16816<T>(aq, fq, bh);
          mma16816<T>(aq, fq, bl);
        }
        if (act) {
          uint32_t bh[2], bl[2];
#pragma unroll
          for (int r = 0; r < 2; ++r) {
            bh[r] = E::pack(gv[2 * r], gv[2 * r + 1]);
            bl[r] = E::pack(gv[2 * r] - E::lo(bh[r]), gv[2 * r + 1] - E::hi(bh[r]));
          }
          mma16816<T>(ad, fd, bh);
          mma16816<T>(ad, fd, bl);
        }
        if (nt == 0) mma16816<T>(ab, fd, ones);
      }
#pragma unroll
      for (int rh = 0; rh < 2; ++rh) {
        const int d = mt * 16 + r8 + 8 * rh;
        const int c0 = nt * 8 + 2 * m4;
        dwp[d * C + c0] = aq[2 * rh] * p.scale + ad[2 * rh];
        dwp[d * C + c0 + 1] = aq[2 * rh + 1] * p.scale + ad[2 * rh + 1];
        if (nt == 0 && m4 == 0) dbp[d] = ab[2 * rh];
      }
    }
  }
}

// ---------------------------------------------------------------------------

// Grid of the row kernel for one (Dh, C) shape: (row tiles, events, head
// groups). Every CTA writes one dW / db partial, so this also sizes the
// partial buffers (rows_partials).
template <int DH, int C>
static dim3 rows_grid(const FstProblem& p) {
  using S = RowShape<DH, C>;
  const int groups = (p.heads + S::HP - 1) / S::HP;
  if (uses_tile_list(p)) {
    const int64_t upper = (list_rows(p) + S::BM - 1) / S::BM + p.batch +
        pad_ctas(p, DH * 2 + 8);
    return dim3((unsigned)upper, 1, groups);
  }
  return dim3((p.max_len + S::BM - 1) / S::BM, p.batch, groups);
}

template <typename T, int DH, int C>
static int launch_rows_shape(const FstBackwardArgs& a, cudaStream_t st, int* tile_start,
                             void* u_ws, void* wt_ws, void* qt_ws) {
  using S = RowShape<DH, C>;
  const FstProblem& p = a.prob;
  if constexpr (!S::kFits) {
    return FST_ERR_UNSUPPORTED;
  }
  static std::atomic<uint64_t> configured{0};
  if (allow_dynamic_smem((const void*)bwd_rows_tc_kernel<T, DH, C>, S::SMEM, configured))
    return api_fail(FST_ERR_CUDA, "cannot allow %d bytes of dynamic shared memory", S::SMEM);
  TmaPair maps{};
  if constexpr (S::TMA) {
    const int rs = p.qkv_row_stride ? p.qkv_row_stride : p.heads * DH;
    int rc = make_head_map(&maps.a, p, a.k, rs);
    if (!rc) rc = make_head_map(&maps.b, p, a.v, rs);
    if (rc) return rc;
  }
  const dim3 grid = rows_grid<DH, C>(p);
  const int groups = (int)grid.z;
  const int per_group = (p.heads + groups - 1) / groups;
  const int threads = (per_group + S::NE) * 32;
  // The tile list (and a self-ordered problem's event order, which the
  // kernels then read) for this kernel and the column kernel after it.
  if (uses_tile_list(p) || self_ordered(p)) tile_prefix(p, S::BM, tile_start, st);
  FstBackwardArgs ka = a;
  if (self_ordered(p)) ka.prob.event_order = tile_start + order_offset(p);
  if (grid.x == 0 || grid.y == 0) return FST_OK;
  bwd_rows_tc_kernel<T, DH, C><<<grid, threads, S::SMEM, st>>>(
      ka, tile_start, per_group, (T*)u_ws, (T*)wt_ws, (T*)qt_ws, maps);
  count_launch();
  return FST_OK;
}

int64_t rows_partials(const FstProblem& p) {
  const int D = p.head_dim, C = p.channels;
  dim3 g(0, 0, 0);
#define FST_ROWS_CASE(DD, CC) \
  if (D == DD && C == CC) g = rows_grid<DD, CC>(p);
  FST_ROWS_CASE(32, 16)
  FST_ROWS_CASE(32, 32)
  FST_ROWS_CASE(32, 64)
  FST_ROWS_CASE(64, 32)
  FST_ROWS_CASE(64, 64)
  FST_ROWS_CASE(16, 16)
  FST_ROWS_CASE(48, 48)
#undef FST_ROWS_CASE
  return (int64_t)g.x * g.y * g.z;
}

template <typename T>
static int launch_rows_t(const FstBackwardArgs& a, cudaStream_t st, int* ts, void* u_ws,
                         void* wt_ws, void* qt_ws) {
  const int D = a.prob.head_dim, C = a.prob.channels;
#define FST_ROWS_CASE(DD, CC) \
  if (D == DD && C == CC) return launch_rows_shape<T, DD, CC>(a, st, ts, u_ws, wt_ws, qt_ws);
  FST_ROWS_CASE(32, 16)
  FST_ROWS_CASE(32, 32)
  FST_ROWS_CASE(32, 64)
  FST_ROWS_CASE(64, 32)
  FST_ROWS_CASE(64, 64)
  FST_ROWS_CASE(16, 16)
  FST_ROWS_CASE(48, 48)
#undef FST_ROWS_CASE
  return FST_ERR_UNSUPPORTED;
}

int launch_bwd_rows(const FstBackwardArgs& a, cudaStream_t st, int* tile_start, void* u_ws,
                    void* wt_ws, void* qt_ws) {
  if (a.prob.dtype == FST_BF16)
    return launch_rows_t<__nv_bfloat16>(a, st, tile_start, u_ws, wt_ws, qt_ws);
  if (a.prob.dtype == FST_F16)
    return launch_rows_t<__half>(a, st, tile_start, u_ws, wt_ws, qt_ws);
  return FST_ERR_UNSUPPORTED;
}

}  // namespace tc
}  // namespace fst
