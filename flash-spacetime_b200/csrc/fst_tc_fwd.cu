// Tensor-core forward kernel (bf16 / fp16 inputs) of fused spacetime-bias
// attention for sm_100a.
//
// What it computes is upstream's flash_spacetime_fwd_kernel
// (src/flash_spacetime/forward.py:63-219) plus the host epilogue of
// flash_spacetime_forward (forward.py:333-345):
//   s_ij = qt_i . k_j + u_i . E_ij           (u = (q*scale) W, formed in the prologue)
//   P    = online softmax over the event's keys
//   out  = sum_j P v_j / l + (sum_j P E_ij / l) W^T + b,  lse = log sum_j exp s
//
// How it is laid out on B200 (one CTA = one event x BM queries x <= 12 heads):
//
//   head warps  (one per head): own BM query rows of their head. They form
//               u = (q*scale) W for their head in the prologue, run QK^T and
//               PV on the tensor cores (m16n8k16, fp32 accumulate, O in
//               registers), add the pair bias, and do the online softmax with
//               exp2 on the MUFU pipe (the reference max of a row moves only
//               when it grows by more than 2^8).
//   E warps     (BM / QPE of them): own QPE query rows each, all heads. They
//               evaluate the C-channel embedding E_ij of every pair once (not
//               once per head) directly in mma B-fragment order, form the
//               logit bias u_q . E_qj for all heads with one MMA per query
//               (heads on M), and accumulate A'_q = sum_j P_qj E_qj per query
//               (heads on M, keys on K) from the head warps' P.
//
// Each head warp streams its own head's K and V 16-key chunks into a
// 2-stage shared-memory ring with cp.async (prefetch distance one chunk);
// each E warp streams its own copy of the key coordinates the same way. No
// operand stage is shared between warps, so no cross-warp barrier guards
// the ring.
//
// The two consumer groups exchange, per chunk, the fp32 bias tile (E warps
// -> head warps) and the bf16/fp16 P tile plus the online-softmax rescale
// factors (head warps -> E warps) through double-buffered shared memory,
// handed over with named barriers (full/empty pairs). At Dh <= 32, C <= 16
// the E warps run one chunk ahead (the bias of chunk n+1 is ready before the
// head warps finish chunk n). The embedding is never written to memory and
// nothing of size O(L^2) exists anywhere.
//
// There are no spin waits: cp.async completion is awaited per thread and
// every named barrier is reached by all head and E warps in the same order.

#include <cuda_runtime.h>

#include "fst_internal.h"
#include "fst_tc_common.cuh"

namespace fst {
namespace tc {

constexpr int kHeadsPerCta = 12;
// A row's reference max moves only when a chunk exceeds it by more than this
// (log2 units), so the P values the MMAs see are at most 2^kLazyMax.
constexpr float kLazyMax = 8.f;

template <int DH, int C>
struct FwdShape {
  // 32 query rows per CTA only for the narrowest shapes: at C = 32 the
  // 16-row block keeps 96 registers a thread (4 bytes of spills instead of
  // 352 with 32 rows at 72 registers).
  static constexpr int BM = (DH <= 32 && C <= 16) ? 32 : 16;  // query rows per CTA
  static constexpr int RG = BM / 16;                          // 16-row groups
  static constexpr int BN = 16;                               // keys per chunk
  static constexpr int QPE = C <= 16 ? 4 : (C <= 32 ? 2 : 1); // queries per E warp
  static constexpr int NE = BM / QPE;                         // E warps
  // E warps run one chunk ahead (two E fragments live) where the registers
  // allow it without spilling.
  static constexpr bool AHEAD = C <= 16 && DH <= 32;
  // Loops unrolled by two chunks with literal ring stages where the
  // registers allow it (the wide shapes would spill).
  static constexpr bool LIT = AHEAD;
  static constexpr int HP = kHeadsPerCta;
  static constexpr int NWARPS = HP + NE;                      // max warps per CTA
  static constexpr int KSD = DH / 16, NTD = DH / 8;
  static constexpr int KSC = C / 16, NTC = C / 8;
  static constexpr int F = C / 2;                             // frequencies
  static constexpr int FG = F / 8;                            // frequency groups per lane
  static constexpr int DHP = DH <= 16 ? 16 : (DH <= 32 ? 32 : 64);
  static constexpr int CP = C <= 16 ? 16 : (C <= 32 ? 32 : 64);
  static constexpr int RBD = DHP * 2;                         // bytes per Q/K/V smem row
  static constexpr int RBC = CP * 2;                          // bytes per u / W smem row
  // fp32 bias tile: row (q, h) holds 16 keys + 8 pad floats; q stride padded
  // to 8 (mod 32) words so both the E-warp stores and head-warp loads are
  // free of bank conflicts.
  static constexpr int BROW = 24;
  static constexpr int BQ = ((HP * BROW + 31) / 32) * 32 + 8;
  // P tile: per query 16 head rows of 16 keys (8 words) padded to 12 words,
  // + 4 pad words per query: the E warps' ldmatrix rows (one per head) then
  // fall in distinct bank groups, and the head warps' stores stay
  // conflict-free.
  static constexpr int PH = 12;
  static constexpr int PQ = 16 * PH + 4;

  // Shared memory carve-up (bytes). The Q and u staging tiles are read into
  // registers once, before the key loop; the bias / P / alpha exchange tiles
  // of the loop then reuse the same bytes.
  static constexpr int SZ_Q = HP * BM * RBD;
  static constexpr int SZ_U = BM * 16 * RBC;
  static constexpr int SZ_B = BM * BQ * 4;                    // one bias stage
  static constexpr int SZ_R = BM * HP * DH * 4;               // epilogue R reuses bias
  static constexpr int SZ_BR = (2 * SZ_B > SZ_R) ? 2 * SZ_B : SZ_R;
  static constexpr int SZ_P = BM * PQ * 4;                    // one P stage
  static constexpr int SZ_A = 2 * BM * HP * 4;                // alpha, both stages
  static constexpr int SZ_STAGE = SZ_Q + SZ_U;
  static constexpr int SZ_LOOP = SZ_BR + 2 * SZ_P + SZ_A;
  static constexpr int SZ_UNION = SZ_STAGE > SZ_LOOP ? SZ_STAGE : SZ_LOOP;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_U = OFF_Q + SZ_Q;
  static constexpr int OFF_B = 0;                             // bias [2][BM][BQ] fp32
  static constexpr int OFF_P = OFF_B + SZ_BR;                 // P [2][BM][PQ] words
  static constexpr int OFF_A = OFF_P + 2 * SZ_P;              // alpha [2][BM][HP]
  static constexpr int OFF_W = SZ_UNION;                      // W hi, W lo: [DH][CP]
  static constexpr int SZ_W = 2 * DH * RBC;
  // K / V rings come by TMA where the box (16 rows x Dh) fills whole swizzled
  // rows (Dh = 16, 32, 64); their stages start on 1024-byte boundaries, as
  // the TMA swizzle patterns (32/64/128 B) require.
  // At C = 64 the ring's barrier state costs the kernel registers it cannot
  // spare (config 2 measured 27.4 / 30.6 TFLOP/s with TMA against 28.5 / 31.5
  // with cp.async at Dh = 32 / 64), so those shapes keep cp.async.
  static constexpr bool TMA = (DH == 16 || DH == 32 || DH == 64) && C <= 32;
  static constexpr int OFF_K = (OFF_W + SZ_W + 1023) / 1024 * 1024;
  static constexpr int SZ_KV = HP * BN * RBD;                 // one stage of K (or V)
  static constexpr int OFF_V = OFF_K + 2 * SZ_KV;
  static constexpr int OFF_C = OFF_V + 2 * SZ_KV;             // key coords [NE][2][BN][4]
  static constexpr int OFF_QC = OFF_C + NE * 2 * BN * 16;     // query coords [BM][4]
  static constexpr int OFF_L = OFF_QC + BM * 16;              // row sums [BM][HP]
  static constexpr int OFF_F = OFF_L + BM * HP * 4;           // rescale flags [2][16] int
  static constexpr int OFF_MB = OFF_F + 2 * 16 * 4;           // K/V ring mbarriers [HP][2]
  static constexpr int SMEM = OFF_MB + HP * 16;
  // Whether the P tiles lie clear of the staging bytes (then they are zeroed
  // while Q and u are staged, saving a barrier).
  static constexpr bool P_CLEAR = OFF_P >= SZ_STAGE;
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
};

// Named barrier ids (0 is __syncthreads).
__device__ __forceinline__ int bar_bias_full(int s) { return 1 + s; }
__device__ __forceinline__ int bar_bias_empty(int s) { return 3 + s; }
__device__ __forceinline__ int bar_p_full(int s) { return 5 + s; }
__device__ __forceinline__ int bar_p_empty(int s) { return 7 + s; }

template <typename T, int DH, int C>
__global__ void __launch_bounds__(FwdShape<DH, C>::NWARPS * 32, 1)
    fwd_tc_kernel(const FstForwardArgs a, const int* __restrict__ tile_start, int heads_per_group,
                  const __grid_constant__ TmaPair kv_maps) {
  using S = FwdShape<DH, C>;
  using E = Elem<T>;
  extern __shared__ __align__(1024) unsigned char smem[];
  const FstProblem& p = a.prob;

  // Heads are split into gridDim.z groups of heads_per_group (<= HP); the
  // block is sized for heads_per_group head warps, so in a shorter last group
  // the surplus warps idle (they only join the CTA-wide barriers).
  const int h0 = blockIdx.z * heads_per_group;
  const int NH = min(heads_per_group, p.heads - h0);
  T* __restrict__ gout = (T*)a.out;

  // Event and query block of this CTA: grid (L / BM, B, groups) over the
  // padded layout, or entry blockIdx.x of the device tile list.
  int b, qb;
  if (uses_tile_list(p)) {
    int t = blockIdx.x;
    if (list_padding(p)) {
      const int writers = pad_ctas(p, DH * 2 + 4);  // padding bytes per (row, head)
      auto fill = [&](int e, int r0, int r1, int nan) {
        const EventSpan es = event_span(p, e);
        fill_rows<T, DH>(gout, es, a.lse, nullptr, es, r0, r1, h0, NH, nan ? E::kNaN2 : 0u,
                         nan ? __int_as_float(0x7fc00000) : 0.f);
      };
      t = list_padded_role(p, tile_start, S::BM, writers, blockIdx.x, gridDim.x, fill);
      if (t < 0) return;
    }
    if (!list_tile(p, tile_start, t, b, qb)) return;
  } else {
    b = p.event_order ? p.event_order[blockIdx.y] : (int)blockIdx.y;
    qb = blockIdx.x;
  }
  const EventSpan ev = event_span(p, b);
  const EventSpan evq = qkv_span(p, b, DH);  // q, k, v (a fused QKV buffer's row stride)
  const int q0 = qb * S::BM;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int NE = S::NE;
  const int nthreads = blockDim.x;
  const T* __restrict__ gq = (const T*)a.q;
  const T* __restrict__ gk = (const T*)a.k;
  const T* __restrict__ gv = (const T*)a.v;
  const T* __restrict__ gu = (const T*)a.u;
  const bool attn = p.use_attn_bias != 0;
  const bool act = p.use_act_bias != 0;

  // A query block entirely past the event's end: padding rows (padded
  // layout) get zeros; nothing else to do.
  if (q0 >= ev.len) {
    if (!is_varlen(p)) {
      constexpr int CH = DH / 8;  // 16-byte chunks per row
      for (int idx = threadIdx.x; idx < NH * S::BM * CH; idx += nthreads) {
        const int c = idx % CH, r = idx / CH;
        const int h = h0 + r / S::BM, q = q0 + r % S::BM;
        if (q >= p.max_len) continue;
        *(uint4*)(gout + ev_off(ev, q, h, DH) + c * 8) = make_uint4(0, 0, 0, 0);
        if (c == 0) a.lse[ev_off(ev, q, h, 1)] = 0.f;
      }
    }
    return;
  }
  const int nvalid_q = min(S::BM, ev.len - q0);
  const int nchunks = (ev.len + S::BN - 1) / S::BN;
  const int NBAR = (NH + NE) * 32;  // threads in the head/E-warp hand-offs

  const uint32_t sm = smem_u32(smem);
  const uint32_t sQ = sm + S::OFF_Q, sU = sm + S::OFF_U, sW = sm + S::OFF_W;
  const uint32_t sK = sm + S::OFF_K, sV = sm + S::OFF_V, sC = sm + S::OFF_C;
  const uint32_t sB = sm + S::OFF_B, sP = sm + S::OFF_P, sA = sm + S::OFF_A;
  const uint32_t sL = sm + S::OFF_L;
  float* fQC = (float*)(smem + S::OFF_QC);

  // ---------------- prologue: stage Q, u, W, query coords ----------------
  // One round of copies: raw q and the query coordinates by cp.async; while
  // they are in flight, W (hi + lo), the u tile's zero rows (or a caller's u),
  // the rescale flags and, where they lie clear of the staging bytes, the
  // zeroed P tiles.
  {
    constexpr int QCH = DH / 8;  // 16-byte chunks per q row
    for (int idx = threadIdx.x; idx < NH * S::BM * QCH; idx += nthreads) {
      const int c = idx % QCH, q = (idx / QCH) % S::BM, h = idx / (QCH * S::BM);
      const uint32_t off = S::OFF_Q + h * S::BM * S::RBD + swz<S::RBD>(q, c);
      if (q < nvalid_q)
        cp_async16(sm + off, gq + ev_off(evq, q0 + q, h0 + h, DH) + c * 8);
      else
        *(uint4*)(smem + off) = make_uint4(0, 0, 0, 0);
    }
    for (int q = threadIdx.x; q < S::BM; q += nthreads) {
      if (q < nvalid_q)
        cp_async16(smem_u32(fQC + q * 4), p.feats + (ev.row0 + q0 + q) * p.feat_stride);
      else
        *(float4*)(fQC + q * 4) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    cp_async_commit();
    if (attn && gu == nullptr) {
      // u is projected by the head warps below; the tile's head rows past the
      // CTA's heads (the heads-on-M MMA reads 16) are zero.
      constexpr int UCH = S::CP / 8;
      const int zrows = 16 - NH;
      for (int idx = threadIdx.x; idx < S::BM * zrows * UCH; idx += nthreads) {
        const int c = idx % UCH, h = NH + (idx / UCH) % zrows, q = idx / (UCH * zrows);
        *(uint4*)(smem + S::OFF_U + swz<S::RBC>(q * 16 + h, c)) = make_uint4(0, 0, 0, 0);
      }
    } else {
      constexpr int UCH = S::CP / 8;
      for (int idx = threadIdx.x; idx < S::BM * 16 * UCH; idx += nthreads) {
        const int c = idx % UCH, h = (idx / UCH) % 16, q = idx / (UCH * 16);
        uint4 v = make_uint4(0, 0, 0, 0);
        if (attn && q < nvalid_q && h < NH && c * 8 < C)
          v = *(const uint4*)(gu + ev_off(ev, q0 + q, h0 + h, C) + c * 8);
        *(uint4*)(smem + S::OFF_U + swz<S::RBC>(q * 16 + h, c)) = v;
      }
    }
    // W as [d][c], split into hi + lo halves of the 16-bit type so that the
    // projection u = (q * scale) W and the epilogue's (A'/l) W^T keep W at
    // ~fp32 accuracy.
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
    if constexpr (S::P_CLEAR) {
      for (int idx = threadIdx.x; idx < 2 * S::SZ_P / 4; idx += nthreads)
        ((uint32_t*)(smem + S::OFF_P))[idx] = 0u;
    }
    if (threadIdx.x < 32) ((int*)(smem + S::OFF_F))[threadIdx.x] = 0;
    cp_async_wait<0>();
  }
  __syncthreads();

  const int m4 = lane & 3, r8 = lane >> 2;
  // Operand fragments that stay in registers for the whole key loop.
  uint32_t qa[S::RG][S::KSD][4];   // head warps: scaled Q (queries on M)
  uint32_t ua[S::QPE][S::KSC][4];  // E warps: u_q (heads on M)
  const bool idle = warp >= NH + NE;
  if (warp < NH) {
    // u = (q * scale) W from the raw rows (one head per warp), then this
    // head's qt = [q * scale] fragments, scaled in registers.
    if (attn && gu == nullptr)
      project_mma<T, DH, C, S::CP, S::RBD, S::BM>(sQ + warp * S::BM * S::RBD, sW,
                                                  sW + DH * S::RBC, p.scale, ev, q0, nvalid_q,
                                                  h0 + warp, warp, smem + S::OFF_U, nullptr);
#pragma unroll
    for (int rg = 0; rg < S::RG; ++rg)
#pragma unroll
      for (int ks = 0; ks < S::KSD; ++ks) {
        const int mi = lane >> 3;
        const int q = rg * 16 + (mi & 1) * 8 + (lane & 7);
        ldsm_x4(sQ + warp * S::BM * S::RBD + swz<S::RBD>(q, 2 * ks + (mi >> 1)), qa[rg][ks]);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          qa[rg][ks][k] = E::pack(E::lo(qa[rg][ks][k]) * p.scale, E::hi(qa[rg][ks][k]) * p.scale);
      }
  }
  __syncthreads();  // u tile complete
  if (warp >= NH && !idle) {
    const int qe = (warp - NH) * S::QPE;
#pragma unroll
    for (int t = 0; t < S::QPE; ++t)
#pragma unroll
      for (int ks = 0; ks < S::KSC; ++ks) {
        const int mi = lane >> 3;
        const int h = (mi & 1) * 8 + (lane & 7);
        ldsm_x4(sU + swz<S::RBC>((qe + t) * 16 + h, 2 * ks + (mi >> 1)), ua[t][ks]);
      }
  }
  __syncthreads();  // the staging tiles are dead; the exchange tiles take their place
  if constexpr (!S::P_CLEAR) {
    for (int idx = threadIdx.x; idx < 2 * S::SZ_P / 4; idx += nthreads)
      ((uint32_t*)(smem + S::OFF_P))[idx] = 0u;
    __syncthreads();
  }

  if (idle) {
    __syncthreads();
    __syncthreads();
    return;
  }
  if (warp >= NH) {
    // ======================= E warps ======================================
    const int e = warp - NH;
    const int qe = e * S::QPE;  // first query row owned by this warp
    // This lane evaluates frequencies 8g + 2*m4 + r (g < FG, r < 2).
    float fr[S::FG][2], fv[S::FG][2];  // f and f / (2 pi) of this lane's frequencies
#pragma unroll
    for (int g = 0; g < S::FG; ++g) {
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        fr[g][r] = p.freqs[8 * g + 2 * m4 + r];
        fv[g][r] = fr[g][r] * 0.15915494309189535f;
      }
    }
    // The interval angles of the warp's QPE queries and the chunk's two
    // 8-key tiles: with QPE = 4 lane m4 of a quad forms query m4's angles
    // for both tiles; with QPE <= 2 (wide shapes) each lane forms one
    // (query m4 % QPE, tile m4 / QPE % 2) angle, so that none is formed
    // twice. The others read them by shuffle. (64, 64), whose forward
    // already spills, measured 3 % slower with it and keeps both per lane.
    constexpr bool kOneAngle = S::QPE <= 2 && DH * C < 64 * 64;
    const int my_t = kOneAngle ? m4 % S::QPE : m4;
    const int my_nt = kOneAngle ? (m4 / S::QPE) & 1 : 0;
    const int qx_row = qe + my_t;
    Coord4 cq;
    cq.x = fQC[qx_row * 4 + 0];
    cq.y = fQC[qx_row * 4 + 1];
    cq.z = fQC[qx_row * 4 + 2];
    cq.t = fQC[qx_row * 4 + 3];

    // Private ring of key coordinates: [2 stages][BN][4] fp32.
    const uint32_t c_ring = sC + e * 2 * S::BN * 16;
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

    float acc[S::QPE][S::NTC][4];
#pragma unroll
    for (int t = 0; t < S::QPE; ++t)
#pragma unroll
      for (int nc = 0; nc < S::NTC; ++nc)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[t][nc][i] = 0.f;

    // With S::AHEAD the E warps run one chunk ahead of the P.E products: chunk n+1's
    // embedding and logit bias are produced before waiting for the head
    // warps' P of chunk n, so the head warps' softmax of chunk n overlaps the
    // embedding of chunk n+1 instead of following it.
    using EFrag = uint32_t[S::QPE][2][S::KSC][2];  // E B-fragments (k = channel, n = key)
    // Embedding of chunk n into eb and (attn) its logit bias into bias stage n & 1.
    auto produce = [&](int n, int s, EFrag& eb) {
      cp_async_wait<1>();
      __syncwarp();
      // x for (query qx_row, key nt*8 + r8): both tiles, or tile my_nt.
      float xl[2];
#pragma unroll
      for (int nt = 0; nt < (kOneAngle ? 1 : 2); ++nt) {
        const int kt = kOneAngle ? my_nt : nt;
        const float4 ck = *(const float4*)(smem + S::OFF_C + (e * 2 * S::BN + s * S::BN + kt * 8 + r8) * 16);
        Coord4 c4;
        c4.x = ck.x;
        c4.y = ck.y;
        c4.z = ck.z;
        c4.t = ck.w;
        xl[nt] = pair_angle_fast(cq, c4);
      }
      __syncwarp();
      load_coords(n + 2);  // stage s is free again
      if (attn && n >= 2) named_sync(bar_bias_empty(s), NBAR);
#pragma unroll
      for (int t = 0; t < S::QPE; ++t) {
        float sn[2][S::FG][2], cs[2][S::FG][2];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          const float xt =
              kOneAngle ? __shfl_sync(0xffffffffu, xl[0], (lane & ~3) | (t + S::QPE * nt))
                        : __shfl_sync(0xffffffffu, xl[nt], (lane & ~3) | t);
#pragma unroll
          for (int g = 0; g < S::FG; ++g)
            sincos_xf2(xt, fr[g], fv[g], sn[nt][g], cs[nt][g]);
        }
        // Channel c < F is sin(x f_c); c >= F is cos(x f_{c-F}). The lane's
        // fragment slots are channels 16 ks + 8 hi + 2 m4 + r.
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int ks = 0; ks < S::KSC; ++ks)
#pragma unroll
            for (int hi = 0; hi < 2; ++hi) {
              const int cb = 16 * ks + 8 * hi;
              const int g = (cb % S::F) / 8;
              const bool is_sin = cb < S::F;
              const float v0 = is_sin ? sn[nt][g][0] : cs[nt][g][0];
              const float v1 = is_sin ? sn[nt][g][1] : cs[nt][g][1];
              eb[t][nt][ks][hi] = E::pack(v0, v1);
            }
        if (attn) {
          const int q = qe + t;
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) {
            float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int ks = 0; ks < S::KSC; ++ks) mma16816<T>(d, ua[t][ks], eb[t][nt][ks]);
            const uint32_t base = sB + s * S::SZ_B + (q * S::BQ + nt * 8 + 2 * m4) * 4;
            if (r8 < NH) sts_v2(base + r8 * S::BROW * 4, d[0], d[1]);
            if (r8 + 8 < NH) sts_v2(base + (r8 + 8) * S::BROW * 4, d[2], d[3]);
          }
        }
      }
      if (attn) named_arrive(bar_bias_full(s), NBAR);
    };
    // A'_q += P_q E_q for chunk n, after the online-softmax rescale.
    auto consume = [&](int n, int s, const EFrag& eb) {
      named_sync(bar_p_full(s), NBAR);
      // Did any head move a reference max this chunk? Otherwise every
      // rescale factor is exactly 1 and A' is left as it is.
      const int4* fl = (const int4*)(smem + S::OFF_F + s * 64);
      const int4 f0 = fl[0], f1 = fl[1], f2 = fl[2];
      const bool resc = (f0.x | f0.y | f0.z | f0.w | f1.x | f1.y | f1.z | f1.w | f2.x | f2.y |
                         f2.z | f2.w) != 0;
#pragma unroll
      for (int t = 0; t < S::QPE; ++t) {
        const int q = qe + t;
        if (resc) {
          // Heads whose warp moved no reference left their factors unwritten: 1.
          const float* alph = (const float*)(smem + S::OFF_A + (s * S::BM + q) * S::HP * 4);
          const int* flg = (const int*)(smem + S::OFF_F + s * 64);
          const float a0 = (r8 < NH && flg[r8]) ? alph[r8] : 1.f;
          const float a1 = (r8 + 8 < NH && flg[r8 + 8]) ? alph[r8 + 8] : 1.f;
#pragma unroll
          for (int nc = 0; nc < S::NTC; ++nc) {
            acc[t][nc][0] *= a0;
            acc[t][nc][1] *= a0;
            acc[t][nc][2] *= a1;
            acc[t][nc][3] *= a1;
          }
        }
        uint32_t pa[4];
        {
          const int mi = lane >> 3;
          const int h = (mi & 1) * 8 + (lane & 7);
          ldsm_x4(sP + s * S::SZ_P + (q * S::PQ + h * S::PH + (mi >> 1) * 4) * 4, pa);
        }
#pragma unroll
        for (int nc = 0; nc < S::NTC; ++nc) {
          // E^T B-fragment (k = key, n = channel) by transposing the 8x8
          // blocks of the (k = channel, n = key) fragment in registers.
          uint32_t bt[2];
          bt[0] = movm_t(eb[t][0][nc >> 1][nc & 1]);
          bt[1] = movm_t(eb[t][1][nc >> 1][nc & 1]);
          mma16816<T>(acc[t][nc], pa, bt);
        }
      }
      if (n + 2 < nchunks) named_arrive(bar_p_empty(s), NBAR);
    };

    if (attn || act) {
      if constexpr (S::AHEAD) {
        EFrag eb0, eb1;
        produce(0, 0, eb0);
        for (int n = 0; n < nchunks; n += 2) {
          if (n + 1 < nchunks) produce(n + 1, 1, eb1);
          if (act) consume(n, 0, eb0);
          if (n + 1 >= nchunks) break;
          if (n + 2 < nchunks) produce(n + 2, 0, eb0);
          if (act) consume(n + 1, 1, eb1);
        }
      } else {
        EFrag eb0;
        for (int n = 0; n < nchunks; ++n) {
          produce(n, n & 1, eb0);
          if (act) consume(n, n & 1, eb0);
        }
      }
    }

    __syncthreads();  // head warps published their row sums
    if (act) {
      // R_q = (A'_q / l) W^T  (heads on M, channels on K, head dim on N),
      // with W split into hi + lo halves. Stored fp32 as [q][h][d].
#pragma unroll
      for (int t = 0; t < S::QPE; ++t) {
        const int q = qe + t;
        const float* lsum = (const float*)(smem + S::OFF_L + q * S::HP * 4);
        const float il0 = r8 < NH ? 1.f / lsum[r8] : 0.f;
        const float il1 = r8 + 8 < NH ? 1.f / lsum[r8 + 8] : 0.f;
        uint32_t aa[S::KSC][4];
#pragma unroll
        for (int ks = 0; ks < S::KSC; ++ks) {
          aa[ks][0] = E::pack(acc[t][2 * ks][0] * il0, acc[t][2 * ks][1] * il0);
          aa[ks][1] = E::pack(acc[t][2 * ks][2] * il1, acc[t][2 * ks][3] * il1);
          aa[ks][2] = E::pack(acc[t][2 * ks + 1][0] * il0, acc[t][2 * ks + 1][1] * il0);
          aa[ks][3] = E::pack(acc[t][2 * ks + 1][2] * il1, acc[t][2 * ks + 1][3] * il1);
        }
#pragma unroll
        for (int nd = 0; nd < S::NTD; ++nd) {
          float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int ks = 0; ks < S::KSC; ++ks) {
#pragma unroll
            for (int part = 0; part < 2; ++part) {
              // B (k = channel, n = d) = W[d][c]: rows d, 8 channels per row.
              uint32_t wb[2];
              const int mi = (lane >> 3) & 1;
              ldsm_x2(sW + part * DH * S::RBC + swz<S::RBC>(nd * 8 + (lane & 7), 2 * ks + mi), wb);
              mma16816<T>(d, aa[ks], wb);
            }
          }
          float* rs = (float*)(smem + S::OFF_B);
          if (r8 < NH) {
            rs[(q * S::HP + r8) * DH + nd * 8 + 2 * m4] = d[0];
            rs[(q * S::HP + r8) * DH + nd * 8 + 2 * m4 + 1] = d[1];
          }
          if (r8 + 8 < NH) {
            rs[(q * S::HP + r8 + 8) * DH + nd * 8 + 2 * m4] = d[2];
            rs[(q * S::HP + r8 + 8) * DH + nd * 8 + 2 * m4 + 1] = d[3];
          }
        }
      }
    }
    __syncthreads();  // R published
    return;
  } else {
    // ======================= head warps ===================================
    const int hl = warp;  // local head
    const int h = h0 + hl;
    // Private ring of this head's K and V chunks: [2 stages][BN][DHP].
    // TMA ring: one mbarrier per stage; box (x = this head's first column,
    // y = the event's row index of key 0 in the 2D row view).
    const uint32_t mbar = sm + S::OFF_MB + hl * 16;
    const int tx = rows_interleaved(p) ? h * DH : 0;
    const int ty = rows_interleaved(p) ? (int)evq.row0 : (int)(evq.base1 + h * evq.hs1);
    bool tma_late = false;  // a ring wait gave up (the copy never landed)
    // The swizzled TMA boxes need their stages on 1024-byte boundaries of the
    // shared window; the copy ring falls back to cp.async otherwise.
    const bool ring_tma = S::TMA && (sK & 1023u) == 0;
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
          const uint32_t off = st * S::SZ_KV + hl * S::BN * S::RBD;
          fence_proxy_async();  // the stage's earlier reads precede the async writes
          mbar_arrive_tx(bar, 2 * S::BN * DH * (int)sizeof(T));
          tma_load_2d(sK + off, &kv_maps.a, bar, tx, ty + n * S::BN);
          tma_load_2d(sV + off, &kv_maps.b, bar, tx, ty + n * S::BN);
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
        const uint32_t k_st = sK + (n & 1) * S::SZ_KV + hl * S::BN * S::RBD;
        const uint32_t v_st = sV + (n & 1) * S::SZ_KV + hl * S::BN * S::RBD;
        for (int idx = lane; idx < S::BN * CH; idx += 32) {
          const int c = idx % CH, j = idx / CH;
          const uint32_t off = swz<S::RBD>(j, c);
          if (j0 + j < ev.len) {
            const int go = (j0 + j) * rs + c * 8;
            cp_async16(k_st + off, kbase + go);
            cp_async16(v_st + off, vbase + go);
          } else {
            asm volatile("st.shared.v4.u32 [%0], {%1,%1,%1,%1};\n" ::"r"(k_st + off), "r"(0));
            asm volatile("st.shared.v4.u32 [%0], {%1,%1,%1,%1};\n" ::"r"(v_st + off), "r"(0));
          }
        }
      }
      cp_async_commit();
    };
    load_kv(0);
    load_kv(1);

    float o[S::RG][S::NTD][4];
    float mrun[S::RG][2], lrun[S::RG][2];
#pragma unroll
    for (int rg = 0; rg < S::RG; ++rg) {
#pragma unroll
      for (int nd = 0; nd < S::NTD; ++nd)
#pragma unroll
        for (int i = 0; i < 4; ++i) o[rg][nd][i] = 0.f;
      mrun[rg][0] = mrun[rg][1] = -INFINITY;
      lrun[rg][0] = lrun[rg][1] = 0.f;
    }

    // One key chunk; s = n & 1 is passed as a literal so that every stage
    // offset folds into the shared-memory instructions.
    auto step = [&](int n, int s) {
      const int j0 = n * S::BN;
      const uint32_t k_st = sK + s * S::SZ_KV + hl * S::BN * S::RBD;
      const uint32_t v_st = sV + s * S::SZ_KV + hl * S::BN * S::RBD;
      if (ring_tma) {
        if (!mbar_wait(mbar + 8 * s, (n >> 1) & 1)) tma_late = true;
        if (j0 + S::BN > ev.len) {
          // Keys past the event: the box brought whatever lies there (the
          // next event's rows or padding); they must be exact zeros.
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

      // K B-fragments (k = head dim, n = key): kb[nt][ks][2].
      uint32_t kb[2][S::KSD][2];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int kp = 0; kp < (S::KSD + 1) / 2; ++kp) {
          const int mi = lane >> 3;
          const int chunk = 4 * kp + mi;  // d chunk (8 elements)
          uint32_t r[4];
          if (S::KSD - 2 * kp >= 2) {
            ldsm_x4(k_st + swz<S::RBD>(nt * 8 + (lane & 7), chunk), r);
            kb[nt][2 * kp][0] = r[0];
            kb[nt][2 * kp][1] = r[1];
            kb[nt][2 * kp + 1][0] = r[2];
            kb[nt][2 * kp + 1][1] = r[3];
          } else {
            ldsm_x2(k_st + swz<S::RBD>(nt * 8 + (lane & 7), 4 * kp + (mi & 1)), r);
            kb[nt][2 * kp][0] = r[0];
            kb[nt][2 * kp][1] = r[1];
          }
        }

      // Logits s = u.E + qt.k. Where the E warps run a chunk ahead (AHEAD),
      // the fp32 pair bias is usually ready, and it starts the MMA
      // accumulators (no separate additions; forward -0.7 % on config 1).
      // Elsewhere the QK^T MMAs go first, so that they overlap the wait for
      // the bias, which is added after (waiting first cost the row and column
      // kernels 4 % and config 2 (64, 64) 7 %).
      float sc[S::RG][2][4];
      if (S::AHEAD && attn) {
        named_sync(bar_bias_full(s), NBAR);
#pragma unroll
        for (int rg = 0; rg < S::RG; ++rg)
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) {
            const int q = rg * 16 + r8;
            const uint32_t base = sB + s * S::SZ_B + (hl * S::BROW + nt * 8 + 2 * m4) * 4;
            const float2 b0 = lds_v2(base + q * S::BQ * 4);
            const float2 b1 = lds_v2(base + (q + 8) * S::BQ * 4);
            sc[rg][nt][0] = b0.x;
            sc[rg][nt][1] = b0.y;
            sc[rg][nt][2] = b1.x;
            sc[rg][nt][3] = b1.y;
          }
        if (n + 2 < nchunks) named_arrive(bar_bias_empty(s), NBAR);
      } else {
#pragma unroll
        for (int rg = 0; rg < S::RG; ++rg)
#pragma unroll
          for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int i = 0; i < 4; ++i) sc[rg][nt][i] = 0.f;
      }
#pragma unroll
      for (int rg = 0; rg < S::RG; ++rg)
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int ks = 0; ks < S::KSD; ++ks) mma16816<T>(sc[rg][nt], qa[rg][ks], kb[nt][ks]);
      if (!S::AHEAD && attn) {
        named_sync(bar_bias_full(s), NBAR);
#pragma unroll
        for (int rg = 0; rg < S::RG; ++rg)
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) {
            const int q = rg * 16 + r8;
            const uint32_t base = sB + s * S::SZ_B + (hl * S::BROW + nt * 8 + 2 * m4) * 4;
            const float2 b0 = lds_v2(base + q * S::BQ * 4);
            const float2 b1 = lds_v2(base + (q + 8) * S::BQ * 4);
            sc[rg][nt][0] += b0.x;
            sc[rg][nt][1] += b0.y;
            sc[rg][nt][2] += b1.x;
            sc[rg][nt][3] += b1.y;
          }
        if (n + 2 < nchunks) named_arrive(bar_bias_empty(s), NBAR);
      }

      // Online softmax in the log2 domain (upstream forward.py:170-185).
      // Keys past the event exist only in the last chunk; only that chunk
      // pays for the mask.
      if (j0 + S::BN > ev.len) {
        const int lim = ev.len - j0 - 2 * m4;
#pragma unroll
        for (int rg = 0; rg < S::RG; ++rg)
#pragma unroll
          for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int i = 0; i < 4; ++i)
              if (nt * 8 + (i & 1) >= lim) sc[rg][nt][i] = -INFINITY;
      }
      uint32_t pa[S::RG][4];
      float alpha[S::RG][2];
      float mnew[S::RG][2];
      bool grew = false;
#pragma unroll
      for (int rg = 0; rg < S::RG; ++rg)
#pragma unroll
        for (int rh = 0; rh < 2; ++rh) {
          float mx = fmaxf(fmaxf(sc[rg][0][2 * rh], sc[rg][0][2 * rh + 1]),
                           fmaxf(sc[rg][1][2 * rh], sc[rg][1][2 * rh + 1])) * kLog2e;
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
          // The reference max of a row moves only when the chunk's max
          // exceeds it by more than kLazyMax (log2 units), so P <= 2^kLazyMax;
          // the final 1/l and the LSE use the same reference, so the result
          // does not depend on when it moved.
          const bool up = mx > mrun[rg][rh] + kLazyMax;
          mnew[rg][rh] = up ? mx : mrun[rg][rh];
          grew |= up;
        }
      // After the first chunk a reference rarely moves; when it moved for no
      // row of the warp, every rescale factor is exactly 1.
      const bool rescale = __any_sync(0xffffffffu, grew);
#pragma unroll
      for (int rg = 0; rg < S::RG; ++rg) {
#pragma unroll
        for (int rh = 0; rh < 2; ++rh) {
          const float muse = mnew[rg][rh] == -INFINITY ? 0.f : mnew[rg][rh];
          float ps = 0.f;
#pragma unroll
          for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int c = 0; c < 2; ++c) {
              const float pv = ex2(fmaf(sc[rg][nt][2 * rh + c], kLog2e, -muse));
              sc[rg][nt][2 * rh + c] = pv;
              ps += pv;
            }
          float al = 1.f;
          if (rescale) {
            al = mnew[rg][rh] != mrun[rg][rh] ? ex2(mrun[rg][rh] - muse) : 1.f;
#pragma unroll
            for (int nd = 0; nd < S::NTD; ++nd) {
              o[rg][nd][2 * rh] *= al;
              o[rg][nd][2 * rh + 1] *= al;
            }
          }
          lrun[rg][rh] = lrun[rg][rh] * al + ps;
          mrun[rg][rh] = mnew[rg][rh];
          alpha[rg][rh] = al;
        }
        pa[rg][0] = E::pack(sc[rg][0][0], sc[rg][0][1]);
        pa[rg][1] = E::pack(sc[rg][0][2], sc[rg][0][3]);
        pa[rg][2] = E::pack(sc[rg][1][0], sc[rg][1][1]);
        pa[rg][3] = E::pack(sc[rg][1][2], sc[rg][1][3]);
      }

      if (act) {
        if (n >= 2) named_sync(bar_p_empty(s), NBAR);
        const uint32_t pbase = sP + s * S::SZ_P + (hl * S::PH + m4) * 4;
#pragma unroll
        for (int rg = 0; rg < S::RG; ++rg) {
          const int q = rg * 16 + r8;
          sts_u32(pbase + q * S::PQ * 4, pa[rg][0]);
          sts_u32(pbase + q * S::PQ * 4 + 16, pa[rg][2]);
          sts_u32(pbase + (q + 8) * S::PQ * 4, pa[rg][1]);
          sts_u32(pbase + (q + 8) * S::PQ * 4 + 16, pa[rg][3]);
          if (m4 == 0 && rescale) {
            float* al = (float*)(smem + S::OFF_A + s * S::BM * S::HP * 4);
            al[q * S::HP + hl] = alpha[rg][0];
            al[(q + 8) * S::HP + hl] = alpha[rg][1];
          }
        }
        if (lane == 0) ((int*)(smem + S::OFF_F))[s * 16 + hl] = rescale ? 1 : 0;
        named_arrive(bar_p_full(s), NBAR);
      }

      // O += P V (V B-fragments: k = key, n = head dim, via ldmatrix.trans).
#pragma unroll
      for (int np = 0; np < (S::NTD + 1) / 2; ++np) {
        const int mi = lane >> 3;
        uint32_t r[4];
        if (S::NTD - 2 * np >= 2) {
          ldsm_x4_t(v_st + swz<S::RBD>((mi & 1) * 8 + (lane & 7), 2 * np + (mi >> 1)), r);
#pragma unroll
          for (int rg = 0; rg < S::RG; ++rg) {
            mma16816<T>(o[rg][2 * np], pa[rg], r);
            mma16816<T>(o[rg][2 * np + 1], pa[rg], r + 2);
          }
        } else {
          ldsm_x2_t(v_st + swz<S::RBD>((mi & 1) * 8 + (lane & 7), 2 * np), r);
#pragma unroll
          for (int rg = 0; rg < S::RG; ++rg) mma16816<T>(o[rg][2 * np], pa[rg], r);
        }
      }
      __syncwarp();
      load_kv(n + 2);  // stage s is free again
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
      // the last copy of each stage before the shared memory is released, and
      // flag this warp's rows (lse = NaN) below.
      tma_late = __any_sync(0xffffffffu, tma_late);
      if (tma_late)
        for (int st = 0; st < 2 && st < nchunks; ++st) {
          const int last = nchunks - 1 - ((nchunks - 1 - st) & 1);
          mbar_wait(mbar + 8 * st, (last >> 1) & 1);
        }
    }

    // Row sums over the quad, published for the E warps' A' normalisation.
#pragma unroll
    for (int rg = 0; rg < S::RG; ++rg)
#pragma unroll
      for (int rh = 0; rh < 2; ++rh) {
        float l = lrun[rg][rh];
        l += __shfl_xor_sync(0xffffffffu, l, 1);
        l += __shfl_xor_sync(0xffffffffu, l, 2);
        lrun[rg][rh] = l;
        if (m4 == 0) ((float*)(smem + S::OFF_L))[(rg * 16 + r8 + 8 * rh) * S::HP + hl] = l;
      }
    __syncthreads();
    __syncthreads();  // E warps published R = (A'/l) W^T

    const float* rsm = (const float*)(smem + S::OFF_B);
#pragma unroll
    for (int rg = 0; rg < S::RG; ++rg)
#pragma unroll
      for (int rh = 0; rh < 2; ++rh) {
        const int q = rg * 16 + r8 + 8 * rh;
        const bool valid = q < nvalid_q;
        if (!valid && (uses_tile_list(p) || q0 + q >= p.max_len)) continue;
        const float il = valid ? 1.f / lrun[rg][rh] : 0.f;
        T* orow = gout + ev_off(ev, q0 + q, h, DH);
#pragma unroll
        for (int nd = 0; nd < S::NTD; ++nd) {
          const int d = nd * 8 + 2 * m4;
          float v0 = o[rg][nd][2 * rh] * il, v1 = o[rg][nd][2 * rh + 1] * il;
          if (act && valid) {
            v0 += rsm[(q * S::HP + hl) * DH + d];
            v1 += rsm[(q * S::HP + hl) * DH + d + 1];
            if (p.bias) {
              v0 += p.bias[d];
              v1 += p.bias[d + 1];
            }
          }
          if (!valid) v0 = v1 = 0.f;
          *(uint32_t*)(orow + d) = E::pack(v0, v1);
        }
        if (m4 == 0)
          a.lse[ev_off(ev, q0 + q, h, 1)] =
              tma_late ? __int_as_float(0x7fc00000)  // a K/V copy never landed
              : valid  ? (mrun[rg][rh] + __log2f(lrun[rg][rh])) * 0.6931471805599453f
                       : 0.f;
      }
    return;
  }
}

// ---------------------------------------------------------------------------

__device__ __forceinline__ int event_len(const FstProblem& p, int b) {
  return is_varlen(p) ? p.cu_seqlens[b + 1] - p.cu_seqlens[b]
                      : min(max(p.seqlens[b], 0), p.max_len);
}

__global__ void tile_prefix_kernel(const FstProblem p, int bm, int* __restrict__ tile_start) {
  // Single-CTA exclusive scans over the events: of ceil(len_b / bm), the
  // events taken in p.event_order (position k holds event order[k]) or the
  // natural one, into tile_start[0..B]; for a padded layout walked by the
  // tile list, also of the padding row counts max_len - len_b in natural
  // order, into tile_start[B+1 .. 2B+1].
  //
  // A self-ordered problem (FST_FLAG_LONGEST_FIRST, B <= kMaxSelfOrdered)
  // first ranks its events: the rank of event i is the number of events
  // longer than it plus the number of equally long ones before it (a stable
  // longest-first sort by counting, B^2 / 1024 comparisons a thread), and
  // order[rank] = i goes to tile_start[order_offset ..] for the kernels.
  __shared__ int2 warp_sums[32];
  __shared__ int2 carry;
  __shared__ int s_len[kMaxSelfOrdered];
  __shared__ int s_ord[kMaxSelfOrdered];
  const bool pad = list_padding(p);
  const int batch = p.batch;
  const bool ranked = self_ordered(p);
  if (ranked) {
    for (int i = threadIdx.x; i < batch; i += blockDim.x) s_len[i] = event_len(p, i);
    __syncthreads();
    int* order = tile_start + order_offset(p);
    for (int i = threadIdx.x; i < batch; i += blockDim.x) {
      const int li = s_len[i];
      int rank = 0;
      for (int j = 0; j < batch; ++j) {
        const int lj = s_len[j];
        rank += (lj > li) || (lj == li && j < i);
      }
      s_ord[rank] = i;
      order[rank] = i;
    }
  }
  if (threadIdx.x == 0) carry = make_int2(0, 0);
  __syncthreads();
  for (int base = 0; base < batch; base += blockDim.x) {
    const int k = base + threadIdx.x;
    int2 v = make_int2(0, 0);
    if (k < batch) {
      const int ev = ranked ? s_ord[k] : (p.event_order ? p.event_order[k] : k);
      const int len = event_len(p, ev);
      v.x = (len + bm - 1) / bm;
      if (pad) v.y = p.max_len - min(max(p.seqlens[k], 0), p.max_len);
    }
    int2 x = v;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int yx = __shfl_up_sync(0xffffffffu, x.x, o);
      const int yy = __shfl_up_sync(0xffffffffu, x.y, o);
      if (lane >= o) {
        x.x += yx;
        x.y += yy;
      }
    }
    if (lane == 31) warp_sums[w] = x;
    __syncthreads();
    if (w == 0) {
      int2 ws = lane < (int)(blockDim.x >> 5) ? warp_sums[lane] : make_int2(0, 0);
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int yx = __shfl_up_sync(0xffffffffu, ws.x, o);
        const int yy = __shfl_up_sync(0xffffffffu, ws.y, o);
        if (lane >= o) {
          ws.x += yx;
          ws.y += yy;
        }
      }
      warp_sums[lane] = ws;
    }
    __syncthreads();
    const int2 before = w > 0 ? warp_sums[w - 1] : make_int2(0, 0);
    const int2 incl = make_int2(x.x + before.x + carry.x, x.y + before.y + carry.y);
    if (k < batch) {
      tile_start[k] = incl.x - v.x;
      if (pad) tile_start[batch + 1 + k] = incl.y - v.y;
    }
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) carry = incl;
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    tile_start[batch] = carry.x;
    if (pad) tile_start[2 * batch + 1] = carry.y;
  }
}

void tile_prefix(const FstProblem& p, int bm, int* tile_start, cudaStream_t st) {
  tile_prefix_kernel<<<1, 1024, 0, st>>>(p, bm, tile_start);
  count_launch();
}

template <typename T, int DH, int C>
static int launch_fwd_shape(const FstForwardArgs& a, cudaStream_t st, int* tile_start) {
  using S = FwdShape<DH, C>;
  const FstProblem& p = a.prob;
  TmaPair maps{};
  if constexpr (S::TMA) {
    const int rs = p.qkv_row_stride ? p.qkv_row_stride : p.heads * DH;
    int rc = make_head_map(&maps.a, p, a.k, rs);
    if (!rc) rc = make_head_map(&maps.b, p, a.v, rs);
    if (rc) return rc;
  }
  static std::atomic<uint64_t> configured{0};  // per template instance, one bit per device
  if (allow_dynamic_smem((const void*)fwd_tc_kernel<T, DH, C>, S::SMEM, configured))
    return api_fail(FST_ERR_CUDA, "cannot allow %d bytes of dynamic shared memory", S::SMEM);
  const int groups = (p.heads + S::HP - 1) / S::HP;
  const int per_group = (p.heads + groups - 1) / groups;  // balanced, <= HP
  const int threads = (per_group + S::NE) * 32;
  // A self-ordered problem's kernels read the order tile_prefix ranks.
  FstForwardArgs ka = a;
  if (self_ordered(p)) ka.prob.event_order = tile_start + order_offset(p);
  dim3 grid;
  if (self_ordered(p) && !uses_tile_list(p)) tile_prefix(p, S::BM, tile_start, st);
  if (uses_tile_list(p)) {
    tile_prefix(p, S::BM, tile_start, st);
    const int64_t upper = (list_rows(p) + S::BM - 1) / S::BM + p.batch +
        pad_ctas(p, DH * 2 + 4);
    grid = dim3((unsigned)upper, 1, groups);
  } else {
    grid = dim3((p.max_len + S::BM - 1) / S::BM, p.batch, groups);
  }
  if (grid.x == 0 || grid.y == 0) return FST_OK;
  fwd_tc_kernel<T, DH, C><<<grid, threads, S::SMEM, st>>>(ka, tile_start, per_group, maps);
  count_launch();
  return FST_OK;
}

template <typename T>
static int launch_fwd_t(const FstForwardArgs& a, cudaStream_t st, int* ts) {
  const int D = a.prob.head_dim, C = a.prob.channels;
#define FST_FWD_CASE(DD, CC) \
  if (D == DD && C == CC) return launch_fwd_shape<T, DD, CC>(a, st, ts);
  FST_FWD_CASE(32, 16)
  FST_FWD_CASE(32, 32)
  FST_FWD_CASE(32, 64)
  FST_FWD_CASE(64, 32)
  FST_FWD_CASE(64, 64)
  FST_FWD_CASE(16, 16)
  FST_FWD_CASE(48, 48)
#undef FST_FWD_CASE
  return FST_ERR_UNSUPPORTED;
}

bool fwd_supported(const FstProblem& p) {
  if (p.dtype == FST_F32) return false;
  const int D = p.head_dim, C = p.channels;
  return (D == 32 && (C == 16 || C == 32 || C == 64)) || (D == 64 && (C == 32 || C == 64)) ||
         (D == 16 && C == 16) || (D == 48 && C == 48);
}

// Workspace: the tile list's prefixes (tile_list_ints).
size_t fwd_workspace(const FstProblem& p) {
  return ((size_t)tile_list_ints(p) * sizeof(int) + 15) / 16 * 16;
}

int launch_fwd(const FstForwardArgs& a, cudaStream_t st) {
  int* tile_start = (int*)a.workspace;
  if (a.prob.dtype == FST_BF16) return launch_fwd_t<__nv_bfloat16>(a, st, tile_start);
  if (a.prob.dtype == FST_F16) return launch_fwd_t<__half>(a, st, tile_start);
  return FST_ERR_UNSUPPORTED;
}

}  // namespace tc
}  // namespace fst
