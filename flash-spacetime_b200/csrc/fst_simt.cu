// CUDA-core (SIMT) kernels: the fp32 path, and any shape the tensor-core
// kernels do not cover (Dh, C <= 64).
//
// One thread owns one (row, head). Every product and accumulation is fp32
// FMA with accurate sincosf/expf, which is what upstream's fp32 path does
// with ieee-precision dots (upstream forward.py:268-270). The algorithm is
// the upstream one, restated per thread:
//   forward  -- online softmax over the event's keys (forward.py:136-219);
//   backward -- rows: D_i = sum P dP / sum P from the same recomputed P and
//               dP, then dS = P (dP - D) and dq, H = sum dS E, G = sum P E,
//               sigma = sum dS (backward.py:316-485);
//               cols: dk = sum_i dS qt_i, dv = sum_i P dO_i (backward.py:209-313);
//               dW partials: fixed-order sums of qt (x) H + dO (x) G
//               (backward.py:607-614).
// Epilogues that upstream runs on the host as separate GEMMs
// (forward.py:333-345, backward.py:600-605) are fused per row here.

#include <cuda_runtime.h>

#include "fst_common.cuh"
#include "fst_internal.h"

namespace fst {
namespace simt {

constexpr int kMax = 64;  // max Dh and max C on this path

struct RowTask {
  int64_t row;  // flat row
  int h;
  int b;
  EventSpan ev;
  int i;  // row inside its event
};

// Maps a flat thread index over [rows, H] to its (row, head, event).
__device__ __forceinline__ bool row_task(const FstProblem& p, int64_t gid, RowTask& t) {
  int64_t rows = p.total_rows;
  if (gid >= rows * p.heads) return false;
  t.row = gid / p.heads;
  t.h = (int)(gid - t.row * p.heads);
  if (is_varlen(p)) {
    t.b = packed_event_of(p.cu_seqlens, p.batch, t.row);
  } else {
    t.b = (int)(t.row / p.max_len);
  }
  t.ev = event_span(p, t.b);
  t.i = (int)(t.row - t.ev.row0);
  return true;
}

// E_ij into e[0..C): sin(x f_k) for k < C/2, cos(x f_k) after.
__device__ __forceinline__ void embed(float x, const float* freqs, int C, float* e) {
  int half = C >> 1;
#pragma unroll
  for (int k = 0; k < kMax / 2; ++k) {
    if (k < half) {
      float sn, cs;
      sincosf(reduce_2pi(x, freqs[k]), &sn, &cs);  // accurate sin/cos of the exact x*f
      e[k] = sn;
      e[k + half] = cs;
    }
  }
}

// sum_d (x[off + d] * mul) W[d][c] in fp32, rounded to T as the host-side
// projection is. x is read from global memory with a rolled loop: inlined
// into the unrolled channel loops of the callers, a fully unrolled d loop
// would make the compiler process Dh x C (64 x 64) bodies per call site.
template <typename T>
__device__ __forceinline__ float project(const FstProblem& p, const T* __restrict__ x, int64_t off,
                                         float mul, int c, int D, int C) {
  float acc = 0.f;
#pragma unroll 1
  for (int d = 0; d < D; ++d) acc = fmaf(to_f<T>(x[off + d]) * mul, p.weight[(int64_t)d * C + c], acc);
  return to_f<T>(from_f<T>(acc));
}

template <typename T>
__global__ void __launch_bounds__(128) fwd_kernel(FstForwardArgs a) {
  const FstProblem& p = a.prob;
  RowTask t;
  if (!row_task(p, (int64_t)blockIdx.x * blockDim.x + threadIdx.x, t)) return;
  const int D = p.head_dim, C = p.channels;
  const T* q = (const T*)a.q;
  const T* k = (const T*)a.k;
  const T* v = (const T*)a.v;
  const T* u = (const T*)a.u;
  T* out = (T*)a.out;
  const int64_t off = vec_off(p, t.row, t.h, D);
  const int64_t qoff = qkv_off(p, t.row, t.h, D);
  if (t.i >= t.ev.len) {  // padding row (padded layout only)
    for (int d = 0; d < D; ++d) out[off + d] = from_f<T>(0.f);
    a.lse[stat_off(p, t.row, t.h)] = 0.f;
    return;
  }
  const bool pair = p.use_attn_bias || p.use_act_bias;
  float qt[kMax], uu[kMax], acc[kMax], ae[kMax], e[kMax];
#pragma unroll
  for (int d = 0; d < kMax; ++d) {
    qt[d] = d < D ? to_f<T>(q[qoff + d]) * p.scale : 0.f;
    acc[d] = 0.f;
  }
  const int64_t uoff = vec_off(p, t.row, t.h, C);
#pragma unroll
  for (int c = 0; c < kMax; ++c) {
    uu[c] = (p.use_attn_bias && c < C)
                ? (u ? to_f<T>(u[uoff + c]) : project<T>(p, q, qoff, p.scale, c, D, C))
                : 0.f;
    ae[c] = 0.f;
    e[c] = 0.f;
  }
  const Coord4 ci = load_coord(p, t.row);
  float m = -INFINITY, l = 0.f;
  for (int j = 0; j < t.ev.len; ++j) {
    const int64_t krow = t.ev.row0 + j;
    const int64_t koff = qkv_off(p, krow, t.h, D);
    float s = 0.f;
#pragma unroll
    for (int d = 0; d < kMax; ++d)
      if (d < D) s = fmaf(qt[d], to_f<T>(k[koff + d]), s);
    if (pair) embed(pair_angle(ci, load_coord(p, krow)), p.freqs, C, e);
    if (p.use_attn_bias) {
#pragma unroll
      for (int c = 0; c < kMax; ++c)
        if (c < C) s = fmaf(uu[c], e[c], s);
    }
    const float mn = fmaxf(m, s);
    const float alpha = expf(m - mn);  // exp(-inf) = 0 on the first key
    const float pj = expf(s - mn);
    l = l * alpha + pj;
    m = mn;
#pragma unroll
    for (int d = 0; d < kMax; ++d)
      if (d < D) acc[d] = fmaf(pj, to_f<T>(v[koff + d]), acc[d] * alpha);
    if (p.use_act_bias) {
#pragma unroll
      for (int c = 0; c < kMax; ++c)
        if (c < C) ae[c] = fmaf(pj, e[c], ae[c] * alpha);
    }
  }
  const float inv = 1.f / l;
  for (int d = 0; d < D; ++d) {
    float o = acc[d] * inv;
    if (p.use_act_bias) {
      float r = p.bias ? p.bias[d] : 0.f;
      const float* w = p.weight + (int64_t)d * C;
#pragma unroll
      for (int c = 0; c < kMax; ++c)
        if (c < C) r = fmaf(ae[c] * inv, w[c], r);
      o += r;
    }
    out[off + d] = from_f<T>(o);
  }
  a.lse[stat_off(p, t.row, t.h)] = m + logf(l);
}

// Shared by the row and column backward kernels: P_ij and dP_ij.
// Per-row operands of the backward. `off` is a row offset subtracted from dP
// before any sum is formed: c_i = dO_i . (out_i - [act] b) = sum_j P_ij dP_ij
// up to the forward's rounding, so the sums below see dP - D (no common
// mode) and their rounding stays relative to |dS|. The dO . b term of dP
// (upstream backward.py:164-168) is a row constant that cancels in dP - D
// and is left out for the same reason.
template <typename T>
struct BwdRow {
  float qt[kMax], dov[kMax], uu[kMax], wt[kMax];
  float lse, off;
  Coord4 c;
};

template <typename T>
__device__ __forceinline__ void load_bwd_row(const FstBackwardArgs& a, int64_t row, int h,
                                             BwdRow<T>& r) {
  const FstProblem& p = a.prob;
  const int D = p.head_dim, C = p.channels;
  const int64_t off = vec_off(p, row, h, D), coff = vec_off(p, row, h, C);
  const int64_t qoff = qkv_off(p, row, h, D);
  const T* q = (const T*)a.q;
  const T* dout = (const T*)a.dout;
  const T* o = (const T*)a.out;
  float c = 0.f;
#pragma unroll
  for (int d = 0; d < kMax; ++d) {
    r.qt[d] = d < D ? to_f<T>(q[qoff + d]) * p.scale : 0.f;
    r.dov[d] = d < D ? to_f<T>(dout[off + d]) : 0.f;
    if (d < D && o) {
      float od = to_f<T>(o[off + d]);
      if (p.use_act_bias && p.bias) od -= p.bias[d];
      c = fmaf(r.dov[d], od, c);
    }
  }
#pragma unroll
  for (int c = 0; c < kMax; ++c) {
    r.uu[c] = 0.f;
    r.wt[c] = 0.f;
    if (c < C && p.use_attn_bias)
      r.uu[c] = a.u ? to_f<T>(((const T*)a.u)[coff + c]) : project<T>(p, q, qoff, p.scale, c, D, C);
    if (c < C && p.use_act_bias)
      r.wt[c] = a.wt ? to_f<T>(((const T*)a.wt)[coff + c]) : project<T>(p, dout, off, 1.f, c, D, C);
  }
  r.off = c;
  r.lse = a.lse[stat_off(p, row, h)];
  r.c = load_coord(p, row);
}

// P and dP for the pair (row r, key krow); e receives E_ij.
template <typename T>
__device__ __forceinline__ void p_dp(const FstBackwardArgs& a, const BwdRow<T>& r, int64_t krow,
                                     int h, const float* kv, const float* vv, float* e,
                                     float& P, float& dP) {
  const FstProblem& p = a.prob;
  const int D = p.head_dim, C = p.channels;
  float s = 0.f, dp = 0.f;
#pragma unroll
  for (int d = 0; d < kMax; ++d) {
    if (d < D) {
      s = fmaf(r.qt[d], kv[d], s);
      dp = fmaf(r.dov[d], vv[d], dp);
    }
  }
  if (p.use_attn_bias || p.use_act_bias)
    embed(pair_angle(r.c, load_coord(p, krow)), p.freqs, C, e);
  if (p.use_attn_bias) {
#pragma unroll
    for (int c = 0; c < kMax; ++c)
      if (c < C) s = fmaf(r.uu[c], e[c], s);
  }
  if (p.use_act_bias) {
#pragma unroll
    for (int c = 0; c < kMax; ++c)
      if (c < C) dp = fmaf(r.wt[c], e[c], dp);
  }
  P = expf(s - r.lse);
  dP = dp - r.off;
}

template <typename T>
__device__ __forceinline__ void load_vec(const T* x, int64_t off, int D, float* out) {
#pragma unroll
  for (int d = 0; d < kMax; ++d) out[d] = d < D ? to_f<T>(x[off + d]) : 0.f;
}

// Row-owned backward: D, dq (with its host-side epilogue fused), H, G, sigma.
template <typename T>
__global__ void __launch_bounds__(128) bwd_rows_kernel(FstBackwardArgs a, float* hbuf,
                                                       float* gbuf) {
  const FstProblem& p = a.prob;
  RowTask t;
  if (!row_task(p, (int64_t)blockIdx.x * blockDim.x + threadIdx.x, t)) return;
  const int D = p.head_dim, C = p.channels;
  const int64_t off = qkv_off(p, t.row, t.h, D), coff = vec_off(p, t.row, t.h, C);
  const int64_t so = stat_off(p, t.row, t.h);
  T* dq = (T*)a.dq;
  if (t.i >= t.ev.len) {
    for (int d = 0; d < D; ++d) dq[off + d] = from_f<T>(0.f);
    for (int c = 0; c < C; ++c) hbuf[coff + c] = gbuf[coff + c] = 0.f;
    a.delta[so] = 0.f;
    a.sigma[so] = 0.f;
    return;
  }
  const T* k = (const T*)a.k;
  const T* v = (const T*)a.v;
  BwdRow<T> r;
  load_bwd_row<T>(a, t.row, t.h, r);
  float kv[kMax], vv[kMax], e[kMax];
#pragma unroll
  for (int c = 0; c < kMax; ++c) e[c] = 0.f;

  // One sweep over the keys, accumulating the dS contractions with D left
  // symbolic (dS_ij = P_ij dP'_ij - D'_i P_ij): X = sum P dP' k, Y = sum P k,
  // Hn = sum P dP' E, G = sum P E, a = sum P dP', ps = sum P. At the end
  // D' = a / ps, so every sum of dS below is formed from the same P and dP'
  // values and rowsum(dS) = a - D' ps vanishes up to one rounding.
  float X[kMax], Y[kMax], Hn[kMax], G[kMax];
#pragma unroll
  for (int d = 0; d < kMax; ++d) X[d] = Y[d] = Hn[d] = G[d] = 0.f;
  float acc_a = 0.f, acc_p = 0.f;
  for (int j = 0; j < t.ev.len; ++j) {
    const int64_t krow = t.ev.row0 + j;
    const int64_t koff = qkv_off(p, krow, t.h, D);
    load_vec<T>(k, koff, D, kv);
    load_vec<T>(v, koff, D, vv);
    float P, dP;
    p_dp<T>(a, r, krow, t.h, kv, vv, e, P, dP);
    const float pd = P * dP;
    acc_a += pd;
    acc_p += P;
#pragma unroll
    for (int d = 0; d < kMax; ++d) {
      if (d < D) {
        X[d] = fmaf(pd, kv[d], X[d]);
        Y[d] = fmaf(P, kv[d], Y[d]);
      }
    }
#pragma unroll
    for (int c = 0; c < kMax; ++c) {
      if (c < C) {
        Hn[c] = fmaf(pd, e[c], Hn[c]);
        G[c] = fmaf(P, e[c], G[c]);
      }
    }
  }
  const float Dr = acc_p > 0.f ? acc_a / acc_p : 0.f;
  float sig = acc_a - Dr * acc_p;
  float dqp[kMax], H[kMax];
#pragma unroll
  for (int d = 0; d < kMax; ++d) {
    dqp[d] = X[d] - Dr * Y[d];
    H[d] = Hn[d] - Dr * G[d];
  }
  const float sig_out = sig;
  if (!p.use_attn_bias) sig = 0.f;  // sigma only enters dq through b (attn)
  // dq = scale (dqp + [attn] (H W^T + sigma b))  (upstream backward.py:600-605)
  for (int d = 0; d < D; ++d) {
    float g = dqp[d];
    if (p.use_attn_bias) {
      const float* w = p.weight + (int64_t)d * C;
      float hw = p.bias ? sig * p.bias[d] : 0.f;
#pragma unroll
      for (int c = 0; c < kMax; ++c)
        if (c < C) hw = fmaf(H[c], w[c], hw);
      g += hw;
    }
    dq[off + d] = from_f<T>(g * p.scale);
  }
  for (int c = 0; c < C; ++c) {
    hbuf[coff + c] = p.use_attn_bias ? H[c] : 0.f;
    gbuf[coff + c] = p.use_act_bias ? G[c] : 0.f;
  }
  a.delta[so] = r.off + Dr;
  a.sigma[so] = sig_out;
}

// Column-owned backward: dk_j = sum_i dS_ij qt_i, dv_j = sum_i P_ij dO_i.
template <typename T>
__global__ void __launch_bounds__(128) bwd_cols_kernel(FstBackwardArgs a) {
  const FstProblem& p = a.prob;
  RowTask t;
  if (!row_task(p, (int64_t)blockIdx.x * blockDim.x + threadIdx.x, t)) return;
  const int D = p.head_dim;
  const int64_t off = qkv_off(p, t.row, t.h, D);
  T* dk = (T*)a.dk;
  T* dv = (T*)a.dv;
  if (t.i >= t.ev.len) {
    for (int d = 0; d < D; ++d) dk[off + d] = dv[off + d] = from_f<T>(0.f);
    return;
  }
  float kv[kMax], vv[kMax], e[kMax], dkv[kMax], dvv[kMax];
  load_vec<T>((const T*)a.k, off, D, kv);
  load_vec<T>((const T*)a.v, off, D, vv);
#pragma unroll
  for (int d = 0; d < kMax; ++d) dkv[d] = dvv[d] = e[d] = 0.f;
  BwdRow<T> r;
  for (int i = 0; i < t.ev.len; ++i) {
    const int64_t qrow = t.ev.row0 + i;
    load_bwd_row<T>(a, qrow, t.h, r);
    float P, dP;
    p_dp<T>(a, r, t.row, t.h, kv, vv, e, P, dP);
    const float ds = P * (dP - (a.delta[stat_off(p, qrow, t.h)] - r.off));
    if (a.ds_absmax)
      atomicMax((int*)&a.ds_absmax[stat_off(p, qrow, t.h)], __float_as_int(fabsf(ds)));
#pragma unroll
    for (int d = 0; d < kMax; ++d) {
      if (d < D) {
        dkv[d] = fmaf(ds, r.qt[d], dkv[d]);
        dvv[d] = fmaf(P, r.dov[d], dvv[d]);
      }
    }
  }
  for (int d = 0; d < D; ++d) {
    dk[off + d] = from_f<T>(dkv[d]);
    dv[off + d] = from_f<T>(dvv[d]);
  }
}

// dW partials: CTA c sums rows [c*chunk, (c+1)*chunk) of qt (x) H + dO (x) G
// in a fixed order. Thread (d, c') owns one output element.
template <typename T>
__global__ void __launch_bounds__(256) dw_partial_kernel(FstBackwardArgs a, const float* hbuf,
                                                         const float* gbuf, int64_t chunk) {
  const FstProblem& p = a.prob;
  const int D = p.head_dim, C = p.channels;
  const int64_t n = p.total_rows * p.heads;
  const int64_t r0 = (int64_t)blockIdx.x * chunk;
  const int64_t r1 = min(n, r0 + chunk);
  const T* q = (const T*)a.q;
  const T* dout = (const T*)a.dout;
  for (int o = threadIdx.x; o < D * C; o += blockDim.x) {
    const int d = o / C, c = o - d * C;
    float acc = 0.f;
    for (int64_t g = r0; g < r1; ++g) {
      const int64_t row = g / p.heads;
      const int h = (int)(g - row * p.heads);
      if (!is_varlen(p)) {  // padding rows carry no gradient, whatever dout holds
        const int64_t b = row / p.max_len;
        if (row - b * p.max_len >= p.seqlens[b]) continue;
      }
      const int64_t off = vec_off(p, row, h, D), coff = vec_off(p, row, h, C);
      if (p.use_attn_bias)
        acc = fmaf(to_f<T>(q[qkv_off(p, row, h, D) + d]) * p.scale, hbuf[coff + c], acc);
      if (p.use_act_bias) acc = fmaf(to_f<T>(dout[off + d]), gbuf[coff + c], acc);
    }
    a.dw_partial[(int64_t)blockIdx.x * D * C + o] = acc;
  }
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float acc = 0.f;
    for (int64_t g = r0; g < r1; ++g) {
      const int64_t row = g / p.heads;
      const int h = (int)(g - row * p.heads);
      if (!is_varlen(p)) {
        const int64_t b = row / p.max_len;
        if (row - b * p.max_len >= p.seqlens[b]) continue;
      }
      acc += to_f<T>(dout[vec_off(p, row, h, D) + d]);
    }
    a.db_partial[(int64_t)blockIdx.x * D + d] = acc;
  }
}

constexpr int kDwParts = 512;

int64_t dw_parts(const FstProblem& p) { return kDwParts; }

size_t bwd_workspace(const FstProblem& p) {
  return (size_t)p.total_rows * p.heads * p.channels * sizeof(float) * 2;
}

template <typename T>
static int launch_fwd_t(const FstForwardArgs& a, cudaStream_t st) {
  const int64_t n = a.prob.total_rows * a.prob.heads;
  if (n == 0) return FST_OK;
  fwd_kernel<T><<<(unsigned)((n + 127) / 128), 128, 0, st>>>(a);
  count_launch();
  return FST_OK;
}

template <typename T>
static int launch_bwd_t(const FstBackwardArgs& a, cudaStream_t st) {
  const FstProblem& p = a.prob;
  const int64_t n = p.total_rows * p.heads;
  float* hbuf = (float*)a.workspace;
  float* gbuf = hbuf + (size_t)n * p.channels;
  if (a.ds_absmax) cudaMemsetAsync(a.ds_absmax, 0, (size_t)n * sizeof(float), st);
  if (n > 0) {
    const unsigned grid = (unsigned)((n + 127) / 128);
    bwd_rows_kernel<T><<<grid, 128, 0, st>>>(a, hbuf, gbuf);
    bwd_cols_kernel<T><<<grid, 128, 0, st>>>(a);
    count_launch(2);
  }
  const int64_t chunk = (n + kDwParts - 1) / kDwParts;
  dw_partial_kernel<T><<<kDwParts, 256, 0, st>>>(a, hbuf, gbuf, chunk > 0 ? chunk : 1);
  count_launch();
  return FST_OK;
}

int launch_fwd(const FstForwardArgs& a, cudaStream_t st) {
  switch (a.prob.dtype) {
    case FST_F32: return launch_fwd_t<float>(a, st);
    case FST_BF16: return launch_fwd_t<__nv_bfloat16>(a, st);
    case FST_F16: return launch_fwd_t<__half>(a, st);
  }
  return FST_ERR_INVALID;
}

int launch_bwd(const FstBackwardArgs& a, cudaStream_t st) {
  switch (a.prob.dtype) {
    case FST_F32: return launch_bwd_t<float>(a, st);
    case FST_BF16: return launch_bwd_t<__nv_bfloat16>(a, st);
    case FST_F16: return launch_bwd_t<__half>(a, st);
  }
  return FST_ERR_INVALID;
}

}  // namespace simt
}  // namespace fst
