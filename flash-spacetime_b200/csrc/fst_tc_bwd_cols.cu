// Tensor-core backward, column-owned half (bf16 / fp16 inputs), sm_100a.
//
// Produces dk_j = sum_i dS_ij qt_i and dv_j = sum_i P_ij dO_i for the 16 keys
// j of one event this CTA owns, for up to HP heads, looping over the event's
// queries in chunks of 16 -- upstream's flash_spacetime_bwd_cols_kernel
// (src/flash_spacetime/backward.py:209-313): every key row has exactly one
// writer and the loop order is fixed, so the result is deterministic without
// atomics. P and dS are recomputed from the saved LSE and from D written by
// the row kernel: P_ij = exp(s_ij - lse_i), dS_ij = P_ij (dP_ij - D_i) with
// dP_ij = dO_i . v_j + [act] w~_i . E_ij (the dO.b row constant is left out of
// both dP and D, where it cancels).
//
// Orientation: keys on the MMA M axis. Head warps hold K and V of their head
// as A fragments, compute S^T = K Q^T and dP^T = V dO^T (queries on N), and
// accumulate dV += P^T dO and dK += dS^T Q with P^T / dS^T reused directly as
// A fragments. E warps evaluate E_ij once per pair for all heads and form
// the two bias products u_i . E_ij and w~_i . E_ij per query (heads on M),
// handing them to the head warps through a double-buffered shared tile laid
// out [head][key][query] so that each head warp reads its slice with 16-byte
// loads.
//
// With ds_absmax given, the kernel also reports rowmax_j |dS_ij| per (i, h)
// through atomicMax on the float bit pattern (max is order independent, so
// the result is still deterministic).

#include <cuda_runtime.h>

#include "fst_internal.h"
#include "fst_tc_common.cuh"

namespace fst {
namespace tc {

template <int DH, int C>
struct ColShape {
  static constexpr int BK = 16;   // keys per CTA
  static constexpr int BQ = 16;   // queries per chunk
  // Queries per E warp and heads per CTA: 8 heads from C = 32 on, and two
  // queries per E warp at (64, 64), keep 128 registers a thread (spills at
  // (64, 64): 68 bytes instead of 568; config 2 measured 30.6 instead of
  // 28.8 TFLOP/s). At (32, 64) one query per E warp stays faster (28.8 vs
  // 27.2) despite its spills: the E side needs the extra warps there.
  static constexpr int QPE = C <= 16 ? 4 : ((C <= 32 || DH >= 64) ? 2 : 1);
  static constexpr int NE = BQ / QPE;
  static constexpr int HP = (DH <= 32 && C <= 16) ? 12 : 8;
  static constexpr int NWARPS = HP + NE;
  // Loops unrolled by two chunks with literal ring stages where the
  // registers allow it (the wide shapes would spill).
  static constexpr bool LIT = C <= 16 && DH <= 32;
  static constexpr int KSD = DH / 16, NTD = DH / 8;
  static constexpr int KSC = C / 16;
  static constexpr int F = C / 2, FG = F / 8;
  static constexpr int DHP = DH <= 16 ? 16 : (DH <= 32 ? 32 : 64);
  static constexpr int CP = C <= 16 ? 16 : (C <= 32 ? 32 : 64);
  static constexpr int RBD = DHP * 2, RBC = CP * 2;
  // bias tile [head][key][query] of (u.E, w~.E) pairs: 32 words per key row,
  // 8 pad words per head, and the 16-byte chunk of a query pair XOR-swizzled
  // by the key (bias_chunk) -- a layout searched so that the E-warp stores
  // are at most 2-way bank conflicted and the head-warp 16-byte loads are
  // conflict free.
  static constexpr int JS = 32;
  static constexpr int HS = BK * JS + 8;
  static constexpr int SZ_BIAS = HP * HS * 4;                 // one stage
  // head-warp ring stage: qt chunk, dO chunk [BQ][DHP] by cp.async, and their
  // LSE and D [BQ] in a separate stats ring. (A TMA ring for the tiles, as in
  // the forward and row kernels, doubled this kernel's spills at 128
  // registers a thread and measured 7 % slower on config 1: 1124 vs 1049 us.)
  static constexpr int SZ_HR = 2 * BQ * RBD;
  static constexpr int SZ_HS = 2 * BQ * 4;
  // E-warp ring stage: u and w~ rows [QPE][HP][CP] + query coords [QPE][4].
  // The MMA's head rows past the CTA's heads read a shared zero row instead.
  static constexpr int UW = QPE * HP * RBC;                   // one of u / w~
  static constexpr int SZ_ER = 2 * UW + QPE * 16;

  static constexpr int SZ_KVS = HP * BK * RBD;                // staged K (and V)
  static constexpr int OFF_KS = 0, OFF_VS = SZ_KVS;           // prologue only
  static constexpr int OFF_BIAS = 0;                          // loop: [2][HP][BK][JS]
  static constexpr int SZ_U = (2 * SZ_KVS > 2 * SZ_BIAS) ? 2 * SZ_KVS : 2 * SZ_BIAS;
  static constexpr int OFF_HR = SZ_U;                         // [HP][2] tile stages
  static constexpr int OFF_HS = OFF_HR + HP * 2 * SZ_HR;      // [HP][2] LSE, D stages
  static constexpr int OFF_ER = OFF_HS + HP * 2 * SZ_HS;      // [NE][2] stages
  static constexpr int OFF_KC = OFF_ER + NE * 2 * SZ_ER;      // key coords [BK][4]
  static constexpr int OFF_ZR = OFF_KC + BK * 16;             // zero row [CP]
  static constexpr int SMEM = OFF_ZR + RBC;
  static constexpr bool kFits = SMEM <= 227 * 1024;
};

// Word offset of the (u, w) pair of (key j, query q) inside one head's tile.
__device__ __forceinline__ int bias_word(int j, int q, int js) {
  const int g = ((j >> 1) & 3) | ((j & 1) << 2);
  return j * js + 4 * ((q >> 1) ^ g) + 2 * (q & 1);
}

__device__ __forceinline__ int cb_bias_full(int s) { return 1 + s; }
__device__ __forceinline__ int cb_bias_empty(int s) { return 3 + s; }

template <typename T, int DH, int C>
__device__ __forceinline__ void bwd_cols_body(const FstBackwardArgs& a,
                                              const int* __restrict__ tile_start,
                                              int heads_per_group, const T* __restrict__ gu,
                                              const T* __restrict__ gwt,
                                              const T* __restrict__ gqt) {
  using S = ColShape<DH, C>;
  using E = Elem<T>;
  extern __shared__ __align__(128) unsigned char smem[];
  const FstProblem& p = a.prob;

  const int h0 = blockIdx.z * heads_per_group;
  const int NH = min(heads_per_group, p.heads - h0);
  T* __restrict__ gdk = (T*)a.dk;
  T* __restrict__ gdv = (T*)a.dv;

  // Event and key block of this CTA: grid (L / BK, B, groups) over the
  // padded layout, or entry blockIdx.x of the device tile list (the row
  // kernel's, whose blocks are also BK rows).
  int b, kb;
  if (uses_tile_list(p)) {
    int t = blockIdx.x;
    if (list_padding(p)) {
      const int writers = pad_ctas(p, DH * 4);  // padding bytes per (row, head)
      auto fill = [&](int e, int r0, int r1, int nan) {
        const EventSpan es = qkv_span(p, e, DH);
        const uint32_t v2 = nan ? E::kNaN2 : 0u;
        fill_rows<T, DH>(gdk, es, nullptr, nullptr, es, r0, r1, h0, NH, v2, 0.f);
        fill_rows<T, DH>(gdv, es, nullptr, nullptr, es, r0, r1, h0, NH, v2, 0.f);
      };
      t = list_padded_role(p, tile_start, S::BK, writers, blockIdx.x, gridDim.x, fill);
      if (t < 0) return;
    }
    if (!list_tile(p, tile_start, t, b, kb)) return;
  } else {
    b = p.event_order ? p.event_order[blockIdx.y] : (int)blockIdx.y;
    kb = blockIdx.x;
  }
  const EventSpan ev = event_span(p, b);
  const EventSpan evq = qkv_span(p, b, DH);  // k, v, dk, dv (a fused QKV buffer's row stride)
  const int k0 = kb * S::BK;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int NE = S::NE;
  const int nthreads = blockDim.x;
  const bool attn = p.use_attn_bias != 0, act = p.use_act_bias != 0;
  const T* __restrict__ gk = (const T*)a.k;
  const T* __restrict__ gv = (const T*)a.v;
  const T* __restrict__ gdo = (const T*)a.dout;

  if (k0 >= ev.len) {
    if (!is_varlen(p)) {
      constexpr int CH = DH / 8;  // 16-byte chunks per row
      for (int idx = threadIdx.x; idx < NH * S::BK * CH; idx += nthreads) {
        const int c = idx % CH, r = idx / CH;
        const int h = h0 + r / S::BK, j = k0 + r % S::BK;
        if (j >= p.max_len) continue;
        const int64_t off = ev_off(evq, j, h, DH) + c * 8;
        *(uint4*)(gdk + off) = make_uint4(0, 0, 0, 0);
        *(uint4*)(gdv + off) = make_uint4(0, 0, 0, 0);
      }
    }
    return;
  }
  const int nvalid_k = min(S::BK, ev.len - k0);
  const int nchunks = (ev.len + S::BQ - 1) / S::BQ;
  const int NBAR = (NH + NE) * 32;
  const uint32_t sm = smem_u32(smem);
  float* fKC = (float*)(smem + S::OFF_KC);

  // ------------------------------ prologue ---------------------------------
  {
    // One round of copies (cp.async) for K, V and the key coordinates.
    constexpr int CH = DH / 8;
    for (int idx = threadIdx.x; idx < NH * S::BK * CH; idx += nthreads) {
      const int c = idx % CH, j = (idx / CH) % S::BK, h = idx / (CH * S::BK);
      const uint32_t off = h * S::BK * S::RBD + swz<S::RBD>(j, c);
      if (j < nvalid_k) {
        const int64_t go = ev_off(evq, k0 + j, h0 + h, DH) + c * 8;
        cp_async16(sm + S::OFF_KS + off, gk + go);
        cp_async16(sm + S::OFF_VS + off, gv + go);
      } else {
        *(uint4*)(smem + S::OFF_KS + off) = make_uint4(0, 0, 0, 0);
        *(uint4*)(smem + S::OFF_VS + off) = make_uint4(0, 0, 0, 0);
      }
    }
    for (int j = threadIdx.x; j < S::BK; j += nthreads) {
      if (j < nvalid_k)
        cp_async16(smem_u32(fKC + j * 4), p.feats + (ev.row0 + k0 + j) * p.feat_stride);
      else
        *(float4*)(fKC + j * 4) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    cp_async_commit();
    for (int idx = threadIdx.x; idx < S::RBC / 4; idx += nthreads)
      ((uint32_t*)(smem + S::OFF_ZR))[idx] = 0u;
    cp_async_wait<0>();
  }
  __syncthreads();
  const int m4 = lane & 3, r8 = lane >> 2;
  const bool idle = warp >= NH + NE;
  uint32_t ka[S::KSD][4], va[S::KSD][4];  // head warps: K, V with keys on M
  if (warp < NH) {
#pragma unroll
    for (int ks = 0; ks < S::KSD; ++ks) {
      const int mi = lane >> 3;
      const int j = (mi & 1) * 8 + (lane & 7);
      const uint32_t off = warp * S::BK * S::RBD + swz<S::RBD>(j, 2 * ks + (mi >> 1));
      ldsm_x4(sm + S::OFF_KS + off, ka[ks]);
      ldsm_x4(sm + S::OFF_VS + off, va[ks]);
    }
  }
  __syncthreads();  // staging bytes become the bias tiles

  if (idle) return;

  if (warp >= NH) {
    // =============================== E warps ==============================
    const int e = warp - NH;
    float fr[S::FG][2], fv[S::FG][2];  // f and f / (2 pi) of this lane's frequencies
#pragma unroll
    for (int g = 0; g < S::FG; ++g) {
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        fr[g][r] = p.freqs[8 * g + 2 * m4 + r];
        fv[g][r] = fr[g][r] * 0.15915494309189535f;
      }
    }
    // The interval angles of the warp's QPE queries and the two 8-key tiles:
    // with QPE = 4 lane m4 of a quad forms query m4's angles for both tiles;
    // with QPE <= 2 each lane forms one (query m4 % QPE, tile m4 / QPE % 2)
    // angle, so that none is formed twice. The others read them by shuffle.
    constexpr bool kOneAngle = S::QPE <= 2;
    const int my_t = kOneAngle ? m4 % S::QPE : (m4 < S::QPE ? m4 : 0);
    const int my_nt = kOneAngle ? (m4 / S::QPE) & 1 : 0;
    // Coordinates of the keys this lane pairs with (both n-tiles, or my_nt).
    Coord4 ck[2];
#pragma unroll
    for (int nt = 0; nt < (kOneAngle ? 1 : 2); ++nt) {
      const int j = (kOneAngle ? my_nt : nt) * 8 + r8;
      ck[nt].x = fKC[j * 4 + 0];
      ck[nt].y = fKC[j * 4 + 1];
      ck[nt].z = fKC[j * 4 + 2];
      ck[nt].t = fKC[j * 4 + 3];
    }
    // Bias-tile addressing of this lane's keys j = nt*8 + 2 m4 + r (bias_word
    // split into its per-lane and per-query parts): byte offset of head r8's
    // row of key j, and the key's swizzle group.
    uint32_t krow[2][2];
    int kgrp[2][2];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int j = nt * 8 + 2 * m4 + r;
        krow[nt][r] = (r8 * S::HS + j * S::JS) * 4;
        kgrp[nt][r] = ((j >> 1) & 3) | ((j & 1) << 2);
      }
    const uint32_t ring = sm + S::OFF_ER + e * 2 * S::SZ_ER;
    const float* __restrict__ fbase = p.feats + ev.row0 * p.feat_stride;
    auto load_ring = [&](int n) {
      if (n < nchunks) {
        const uint32_t st = ring + (n & 1) * S::SZ_ER;
        constexpr int CC = C / 8;  // 16-byte chunks per (q, h) row
        constexpr int NIT = (S::QPE * S::HP * CC + 31) / 32;
#pragma unroll
        for (int it = 0; it < NIT; ++it) {
          const int idx = it * 32 + lane;
          const int c = idx % CC, h = (idx / CC) % S::HP, t = idx / (CC * S::HP);
          if (t >= S::QPE || h >= NH) continue;
          const int i = n * S::BQ + e * S::QPE + t;
          const uint32_t off = swz<S::RBC>(t * S::HP + h, c);
          if (i < ev.len) {
            const int64_t go = ev_off(ev, i, h0 + h, C) + c * 8;
            if (attn) cp_async16(st + off, gu + go);
            if (act) cp_async16(st + S::UW + off, gwt + go);
          } else {
            asm volatile("st.shared.v4.u32 [%0], {%1,%1,%1,%1};\n" ::"r"(st + off), "r"(0));
            asm volatile("st.shared.v4.u32 [%0], {%1,%1,%1,%1};\n" ::"r"(st + S::UW + off),
                         "r"(0));
          }
        }
        if (lane < S::QPE) {
          const int i = n * S::BQ + e * S::QPE + lane;
          const uint32_t dst = st + 2 * S::UW + lane * 16;
          if (i < ev.len)
            cp_async16(dst, fbase + i * p.feat_stride);
          else
            asm volatile("st.shared.v4.u32 [%0], {%1,%1,%1,%1};\n" ::"r"(dst), "r"(0));
        }
      }
      cp_async_commit();
    };
    load_ring(0);
    load_ring(1);

    // One query chunk; the stage s = n & 1 is passed as a literal.
    auto estep = [&](int n, int s) {
      cp_async_wait<1>();
      __syncwarp();
      const uint32_t st = ring + s * S::SZ_ER;
      uint32_t ua[S::QPE][S::KSC][4], wa[S::QPE][S::KSC][4];
#pragma unroll
      for (int t = 0; t < S::QPE; ++t)
#pragma unroll
        for (int ks = 0; ks < S::KSC; ++ks) {
          const int mi = lane >> 3;
          const int h = (mi & 1) * 8 + (lane & 7);
          const int chunk = 2 * ks + (mi >> 1);
          const bool real = h < NH;
          const uint32_t au = real ? st + swz<S::RBC>(t * S::HP + h, chunk)
                                   : sm + S::OFF_ZR + chunk * 16;
          const uint32_t aw = real ? au + S::UW : au;
          ldsm_x4(au, ua[t][ks]);
          ldsm_x4(aw, wa[t][ks]);
        }
      // x for (query my_t of this warp, key nt*8 + r8): both tiles, or my_nt.
      float xl[2];
      {
        const float4 c4 =
            *(const float4*)(smem + S::OFF_ER + (e * 2 + s) * S::SZ_ER + 2 * S::UW + my_t * 16);
        Coord4 cq;
        cq.x = c4.x;
        cq.y = c4.y;
        cq.z = c4.z;
        cq.t = c4.w;
        xl[0] = pair_angle_fast(cq, ck[0]);
        if (!kOneAngle) xl[1] = pair_angle_fast(cq, ck[1]);
      }
      __syncwarp();
      load_ring(n + 2);

      if (n >= 2) named_sync(cb_bias_empty(s), NBAR);
      const uint32_t base = sm + S::OFF_BIAS + s * S::SZ_BIAS;
      // Queries are taken two at a time (when QPE is even), so that the (u.E,
      // w~.E) pairs of queries 2k and 2k + 1 -- adjacent in the tile -- go out
      // in one 16-byte store.
      constexpr int TG = S::QPE % 2 == 0 ? 2 : 1;
#pragma unroll
      for (int tp = 0; tp < S::QPE; tp += TG) {
        float du[TG][2][4], dw[TG][2][4];  // [query of the group][nt][fragment]
#pragma unroll
        for (int tt = 0; tt < TG; ++tt) {
          const int t = tp + tt;
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
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) {
            uint32_t eb[S::KSC][2];
#pragma unroll
            for (int ks = 0; ks < S::KSC; ++ks)
#pragma unroll
              for (int hi = 0; hi < 2; ++hi) {
                const int cb = 16 * ks + 8 * hi;
                const int g = (cb % S::F) / 8;
                const bool is_sin = cb < S::F;
                eb[ks][hi] = E::pack(is_sin ? sn[nt][g][0] : cs[nt][g][0],
                                     is_sin ? sn[nt][g][1] : cs[nt][g][1]);
              }
#pragma unroll
            for (int i = 0; i < 4; ++i) du[tt][nt][i] = dw[tt][nt][i] = 0.f;
#pragma unroll
            for (int ks = 0; ks < S::KSC; ++ks) {
              if (attn) mma16816<T>(du[tt][nt], ua[t][ks], eb[ks]);
              if (act) mma16816<T>(dw[tt][nt], wa[t][ks], eb[ks]);
            }
          }
        }
        // D[h][key]: h = r8 (+8), keys nt*8 + 2 m4 (+1). Tile [h][key][q].
        const int qq = e * S::QPE + tp;  // query index within the chunk
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int r = 0; r < 2; ++r) {
            const uint32_t a0 =
                base + krow[nt][r] + 16 * ((qq >> 1) ^ kgrp[nt][r]) + 8 * (qq & 1);
            if constexpr (TG == 2) {
              if (r8 < NH)
                asm volatile("st.shared.v4.f32 [%0], {%1,%2,%3,%4};\n" ::"r"(a0),
                             "f"(du[0][nt][r]), "f"(dw[0][nt][r]), "f"(du[1][nt][r]),
                             "f"(dw[1][nt][r]));
              if (r8 + 8 < NH)
                asm volatile("st.shared.v4.f32 [%0], {%1,%2,%3,%4};\n" ::"r"(a0 + 8 * S::HS * 4),
                             "f"(du[0][nt][2 + r]), "f"(dw[0][nt][2 + r]), "f"(du[1][nt][2 + r]),
                             "f"(dw[1][nt][2 + r]));
            } else {
              if (r8 < NH) sts_v2(a0, du[0][nt][r], dw[0][nt][r]);
              if (r8 + 8 < NH) sts_v2(a0 + 8 * S::HS * 4, du[0][nt][2 + r], dw[0][nt][2 + r]);
            }
          }
      }
      named_arrive(cb_bias_full(s), NBAR);
    };
    if constexpr (S::LIT) {
      for (int n = 0; n < nchunks; n += 2) {
        estep(n, 0);
        if (n + 1 < nchunks) estep(n + 1, 1);
      }
    } else {
      for (int n = 0; n < nchunks; ++n) estep(n, n & 1);
    }
    return;
  }

  // ================================ head warps ===============================
  const int hl = warp;
  const int h = h0 + hl;
  const uint32_t ring = sm + S::OFF_HR + hl * 2 * S::SZ_HR;
  const uint32_t sring = sm + S::OFF_HS + hl * 2 * S::SZ_HS;
  const float* __restrict__ lse_h = a.lse + ev_off(ev, 0, h, 1);  // row qi at qi * ev.rs1
  const float* __restrict__ delta_h = a.delta + ev_off(ev, 0, h, 1);
  auto load_ring = [&](int n) {
    if (n < nchunks) {
      const uint32_t st = ring + (n & 1) * S::SZ_HR;
      constexpr int CH = DH / 8;
      // qt = [q * scale] and dO of this head: event base pointers and row stride.
      const T* __restrict__ qbase = gqt + ev_off(ev, 0, h, DH);
      const T* __restrict__ dobase = gdo + ev_off(ev, 0, h, DH);
      const int rs = row_stride(p, DH);
      for (int idx = lane; idx < S::BQ * CH; idx += 32) {
        const int c = idx % CH, i = idx / CH;
        const uint32_t off = swz<S::RBD>(i, c);
        const int qi = n * S::BQ + i;
        if (qi < ev.len) {
          const int go = qi * rs + c * 8;
          cp_async16(st + off, qbase + go);
          cp_async16(st + S::BQ * S::RBD + off, dobase + go);
        } else {
          asm volatile("st.shared.v4.u32 [%0], {%1,%1,%1,%1};\n" ::"r"(st + off), "r"(0));
          asm volatile("st.shared.v4.u32 [%0], {%1,%1,%1,%1};\n" ::"r"(st + S::BQ * S::RBD + off),
                       "r"(0));
        }
      }
      if (lane < S::BQ) {  // LSE (natural log) and D of the chunk's queries
        const int qi = n * S::BQ + lane;
        const uint32_t f = sring + (n & 1) * S::SZ_HS + lane * 4;
        if (qi < ev.len) {
          cp_async4(f, lse_h + qi * ev.rs1);
          cp_async4(f + S::BQ * 4, delta_h + qi * ev.rs1);
        } else {
          asm volatile("st.shared.u32 [%0], %1;\n" ::"r"(f), "r"(0));
          asm volatile("st.shared.u32 [%0], %1;\n" ::"r"(f + S::BQ * 4), "r"(0));
        }
      }
    }
    cp_async_commit();
  };
  load_ring(0);
  load_ring(1);

  // This lane's (u, w) words in its head's bias tile: keys r8 (+8), queries
  // nt*8 + 2 m4 (+1), 16 bytes per key -- the same every chunk.
  uint32_t boff[2][2];
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int rh = 0; rh < 2; ++rh)
      boff[nt][rh] = (hl * S::HS + bias_word(r8 + 8 * rh, nt * 8 + 2 * m4, S::JS)) * 4;

  float dk[S::NTD][4], dv[S::NTD][4];
#pragma unroll
  for (int nd = 0; nd < S::NTD; ++nd)
#pragma unroll
    for (int i = 0; i < 4; ++i) dk[nd][i] = dv[nd][i] = 0.f;

  // One query chunk; the stage s = n & 1 is passed as a literal.
  auto step = [&](int n, int s) {
    const int i0 = n * S::BQ;
    const uint32_t st = ring + s * S::SZ_HR;
    const uint32_t q_st = st, do_st = st + S::BQ * S::RBD;
    const float* stat = (const float*)(smem + (sring - sm) + s * S::SZ_HS);
    cp_async_wait<1>();
    __syncwarp();

    // S^T = K Q^T, dP^T = V dO^T (B fragments: k = head dim, n = query).
    float sc[2][4], dp[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int i = 0; i < 4; ++i) sc[nt][i] = dp[nt][i] = 0.f;
#pragma unroll
      for (int kp = 0; kp < (S::KSD + 1) / 2; ++kp) {
        const int mi = lane >> 3;
        uint32_t rq[4], rd[4];
        if (S::KSD - 2 * kp >= 2) {
          const uint32_t off = swz<S::RBD>(nt * 8 + (lane & 7), 4 * kp + mi);
          ldsm_x4(q_st + off, rq);
          ldsm_x4(do_st + off, rd);
          mma16816<T>(sc[nt], ka[2 * kp], rq);
          mma16816<T>(sc[nt], ka[2 * kp + 1], rq + 2);
          mma16816<T>(dp[nt], va[2 * kp], rd);
          mma16816<T>(dp[nt], va[2 * kp + 1], rd + 2);
        } else {
          const uint32_t off = swz<S::RBD>(nt * 8 + (lane & 7), 4 * kp + (mi & 1));
          ldsm_x2(q_st + off, rq);
          ldsm_x2(do_st + off, rd);
          mma16816<T>(sc[nt], ka[2 * kp], rq);
          mma16816<T>(dp[nt], va[2 * kp], rd);
        }
      }
    }
    named_sync(cb_bias_full(s), NBAR);
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const uint32_t base = sm + S::OFF_BIAS + s * S::SZ_BIAS;
      float4 b0, b1;
      asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];\n"
                   : "=f"(b0.x), "=f"(b0.y), "=f"(b0.z), "=f"(b0.w)
                   : "r"(base + boff[nt][0]));
      asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];\n"
                   : "=f"(b1.x), "=f"(b1.y), "=f"(b1.z), "=f"(b1.w)
                   : "r"(base + boff[nt][1]));
      sc[nt][0] += b0.x;
      dp[nt][0] += b0.y;
      sc[nt][1] += b0.z;
      dp[nt][1] += b0.w;
      sc[nt][2] += b1.x;
      dp[nt][2] += b1.y;
      sc[nt][3] += b1.z;
      dp[nt][3] += b1.w;
    }
    if (n + 2 < nchunks) named_arrive(cb_bias_empty(s), NBAR);

    // P^T and dS^T; queries past the event (last chunk only) get P = dS = 0.
    uint32_t pt[4], dt[4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int qi = nt * 8 + 2 * m4 + c;
        const float l2 = stat[qi] * kLog2e, dl = stat[S::BQ + qi];
#pragma unroll
        for (int hi = 0; hi < 2; ++hi) {
          const int i = 2 * hi + c;
          const float pv = ex2(fmaf(sc[nt][i], kLog2e, -l2));
          dp[nt][i] = pv * (dp[nt][i] - dl);
          sc[nt][i] = pv;
        }
      }
    if (i0 + S::BQ > ev.len) {
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (i0 + nt * 8 + 2 * m4 + (i & 1) >= ev.len) sc[nt][i] = dp[nt][i] = 0.f;
    }
    pt[0] = E::pack(sc[0][0], sc[0][1]);
    pt[1] = E::pack(sc[0][2], sc[0][3]);
    pt[2] = E::pack(sc[1][0], sc[1][1]);
    pt[3] = E::pack(sc[1][2], sc[1][3]);
    dt[0] = E::pack(dp[0][0], dp[0][1]);
    dt[1] = E::pack(dp[0][2], dp[0][3]);
    dt[2] = E::pack(dp[1][0], dp[1][1]);
    dt[3] = E::pack(dp[1][2], dp[1][3]);
    if (a.ds_absmax) {
      // max over this warp's 16 keys (lanes with equal m4), then one atomic
      // per (query, head) from the r8 == 0 lanes.
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          float v = 0.f;
          if (r8 < nvalid_k) v = fabsf(dp[nt][c]);
          if (r8 + 8 < nvalid_k) v = fmaxf(v, fabsf(dp[nt][2 + c]));
          v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 4));
          v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 8));
          v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 16));
          const int qi = i0 + nt * 8 + 2 * m4 + c;
          if (r8 == 0 && qi < ev.len)
            atomicMax((int*)&a.ds_absmax[ev_off(ev, qi, h, 1)], __float_as_int(v));
        }
    }
    // dV += P^T dO, dK += dS^T qt (B fragments: k = query, n = head dim).
#pragma unroll
    for (int np = 0; np < (S::NTD + 1) / 2; ++np) {
      const int mi = lane >> 3;
      uint32_t rdo[4], rq[4];
      if (S::NTD - 2 * np >= 2) {
        const uint32_t off = swz<S::RBD>((mi & 1) * 8 + (lane & 7), 2 * np + (mi >> 1));
        ldsm_x4_t(do_st + off, rdo);
        ldsm_x4_t(q_st + off, rq);
        mma16816<T>(dv[2 * np], pt, rdo);
        mma16816<T>(dv[2 * np + 1], pt, rdo + 2);
        mma16816<T>(dk[2 * np], dt, rq);
        mma16816<T>(dk[2 * np + 1], dt, rq + 2);
      } else {
        const uint32_t off = swz<S::RBD>((mi & 1) * 8 + (lane & 7), 2 * np);
        ldsm_x2_t(do_st + off, rdo);
        ldsm_x2_t(q_st + off, rq);
        mma16816<T>(dv[2 * np], pt, rdo);
        mma16816<T>(dk[2 * np], dt, rq);
      }
    }
    __syncwarp();
    load_ring(n + 2);
  };
  if constexpr (S::LIT) {
    for (int n = 0; n < nchunks; n += 2) {
      step(n, 0);
      if (n + 1 < nchunks) step(n + 1, 1);
    }
  } else {
    for (int n = 0; n < nchunks; ++n) step(n, n & 1);
  }
#pragma unroll
  for (int rh = 0; rh < 2; ++rh) {
    const int j = r8 + 8 * rh;
    const bool valid = j < nvalid_k;
    if (!valid && (uses_tile_list(p) || k0 + j >= p.max_len)) continue;
    const int64_t off = ev_off(evq, k0 + j, h, DH);
#pragma unroll
    for (int nd = 0; nd < S::NTD; ++nd) {
      const int d = nd * 8 + 2 * m4;
      *(uint32_t*)(gdk + off + d) =
          valid ? E::pack(dk[nd][2 * rh], dk[nd][2 * rh + 1]) : 0u;
      *(uint32_t*)(gdv + off + d) =
          valid ? E::pack(dv[nd][2 * rh], dv[nd][2 * rh + 1]) : 0u;
    }
  }
}

// ---------------------------------------------------------------------------

template <typename T, int DH, int C>
__global__ void __launch_bounds__(ColShape<DH, C>::NWARPS * 32, 1)
    bwd_cols_tc_kernel(const FstBackwardArgs a, const int* __restrict__ tile_start,
                       int heads_per_group, const T* __restrict__ gu,
                       const T* __restrict__ gwt, const T* __restrict__ gqt) {
  bwd_cols_body<T, DH, C>(a, tile_start, heads_per_group, gu, gwt, gqt);
}

// The same kernel held to 120 registers a thread (a few bytes of spills):
// 512 x 120 registers leave 4096 of an SM's 65536 free, room for a small
// kernel running beside it on every SM -- the host-to-device row gather of a
// training loop's next batch (fst_upload_rows, 128 threads x <= 32 registers),
// which cannot start on an SM that this kernel fills. Chosen when the caller
// sets FST_FLAG_SHARE_SMS; costs about 7 % of the backward when nothing runs
// beside it. Only the narrow shapes have the variant.
template <typename T, int DH, int C>
__global__ void __maxnreg__(120)
    bwd_cols_tc_shared_kernel(const FstBackwardArgs a, const int* __restrict__ tile_start,
                              int heads_per_group, const T* __restrict__ gu,
                              const T* __restrict__ gwt, const T* __restrict__ gqt) {
  bwd_cols_body<T, DH, C>(a, tile_start, heads_per_group, gu, gwt, gqt);
}

template <int DH, int C>
constexpr bool has_shared_variant() {
  return DH <= 32 && C <= 16 && ColShape<DH, C>::NWARPS * 32 * 120 <= 65536 - 4096;
}

template <typename T, int DH, int C>
static int launch_cols_shape(const FstBackwardArgs& a, cudaStream_t st, int* tile_start,
                             const void* gu, const void* gwt, const void* gqt) {
  using S = ColShape<DH, C>;
  const FstProblem& p = a.prob;
  if constexpr (!S::kFits) {
    return FST_ERR_UNSUPPORTED;
  } else {
    bool shared = false;
    const void* fn = (const void*)bwd_cols_tc_kernel<T, DH, C>;
    if constexpr (has_shared_variant<DH, C>()) {
      shared = (p.flags & FST_FLAG_SHARE_SMS) != 0;
      if (shared) fn = (const void*)bwd_cols_tc_shared_kernel<T, DH, C>;
    }
    static std::atomic<uint64_t> configured{0}, configured_shared{0};
    if (allow_dynamic_smem(fn, S::SMEM, shared ? configured_shared : configured))
      return api_fail(FST_ERR_CUDA, "cannot allow %d bytes of dynamic shared memory", S::SMEM);
    const int groups = (p.heads + S::HP - 1) / S::HP;
    const int per_group = (p.heads + groups - 1) / groups;
    const int threads = (per_group + S::NE) * 32;
    dim3 grid;
    if (uses_tile_list(p)) {
      // tile_start (16-row tiles) was built by the row kernel's launch.
      const int64_t upper = (list_rows(p) + S::BK - 1) / S::BK + p.batch +
          pad_ctas(p, DH * 4);
      grid = dim3((unsigned)upper, 1, groups);
    } else {
      grid = dim3((p.max_len + S::BK - 1) / S::BK, p.batch, groups);
    }
    if (grid.x == 0 || grid.y == 0) return FST_OK;
    // A self-ordered problem's event order, ranked by the row kernel's launch.
    FstBackwardArgs ka = a;
    if (self_ordered(p)) ka.prob.event_order = tile_start + order_offset(p);
    if constexpr (has_shared_variant<DH, C>()) {
      if (shared) {
        bwd_cols_tc_shared_kernel<T, DH, C><<<grid, threads, S::SMEM, st>>>(
            ka, tile_start, per_group, (const T*)gu, (const T*)gwt, (const T*)gqt);
        count_launch();
        return FST_OK;
      }
    }
    bwd_cols_tc_kernel<T, DH, C><<<grid, threads, S::SMEM, st>>>(
        ka, tile_start, per_group, (const T*)gu, (const T*)gwt, (const T*)gqt);
    count_launch();
    return FST_OK;
  }
}

template <typename T>
static int launch_cols_t(const FstBackwardArgs& a, cudaStream_t st, int* ts, const void* gu,
                         const void* gwt, const void* gqt) {
  const int D = a.prob.head_dim, C = a.prob.channels;
#define FST_COLS_CASE(DD, CC) \
  if (D == DD && C == CC) return launch_cols_shape<T, DD, CC>(a, st, ts, gu, gwt, gqt);
  FST_COLS_CASE(32, 16)
  FST_COLS_CASE(32, 32)
  FST_COLS_CASE(32, 64)
  FST_COLS_CASE(64, 32)
  FST_COLS_CASE(64, 64)
  FST_COLS_CASE(16, 16)
  FST_COLS_CASE(48, 48)
#undef FST_COLS_CASE
  return FST_ERR_UNSUPPORTED;
}

int launch_bwd_cols(const FstBackwardArgs& a, cudaStream_t st, int* tile_start, const void* gu,
                    const void* gwt, const void* gqt) {
  if (a.prob.dtype == FST_BF16)
    return launch_cols_t<__nv_bfloat16>(a, st, tile_start, gu, gwt, gqt);
  if (a.prob.dtype == FST_F16) return launch_cols_t<__half>(a, st, tile_start, gu, gwt, gqt);
  return FST_ERR_UNSUPPORTED;
}

bool bwd_supported(const FstProblem& p) {
  return fwd_supported(p);  // same (Dh, C) list; every shape fits both kernels
}

// Workspace: [tile list prefixes, tile_list_ints][u and w~, rows x H x C each
// in the 16-bit type, 256-byte aligned][qt = [q * scale], rows x H x Dh in
// the 16-bit type] -- the row kernel writes the two projections there (when
// the caller did not pass them) and the scaled q, the column kernel reads
// them back.
static size_t ws_proj_offset(const FstProblem& p) {
  return ((size_t)tile_list_ints(p) * sizeof(int) + 255) / 256 * 256;
}
static size_t ws_proj_bytes(const FstProblem& p) {
  return ((size_t)p.total_rows * p.heads * p.channels * 2 + 255) / 256 * 256;
}
static size_t ws_qt_bytes(const FstProblem& p) {
  return ((size_t)p.total_rows * p.heads * p.head_dim * 2 + 255) / 256 * 256;
}

size_t bwd_workspace(const FstProblem& p) {
  return ws_proj_offset(p) + 2 * ws_proj_bytes(p) + ws_qt_bytes(p);
}

int launch_bwd(const FstBackwardArgs& a, cudaStream_t st) {
  const FstProblem& p = a.prob;
  int* tile_start = (int*)a.workspace;
  unsigned char* proj = (unsigned char*)a.workspace + ws_proj_offset(p);
  void* u_ws = proj;
  void* wt_ws = proj + ws_proj_bytes(p);
  void* qt_ws = proj + 2 * ws_proj_bytes(p);
  if (a.ds_absmax) {
    const int64_t n = p.total_rows * p.heads;
    if (cudaMemsetAsync(a.ds_absmax, 0, n * sizeof(float), st) != cudaSuccess) return FST_ERR_CUDA;
  }
  int rc = launch_bwd_rows(a, st, tile_start, u_ws, wt_ws, qt_ws);
  if (rc) return rc;
  return launch_bwd_cols(a, st, tile_start, a.u ? a.u : u_ws, a.wt ? a.wt : wt_ws, qt_ws);
}

}  // namespace tc
}  // namespace fst
