// Shared device helpers for the fused spacetime-bias attention kernels.
//
// Layout addressing (padded [B,H,L,*] vs packed [T,H,*]), dtype conversion and
// the pair angle x_ij of the spacetime interval. The angle follows upstream
// src/flash_spacetime/_tiles.py:25-42 (itself the encoder definition of
// reference.py:75-81): I = |dp|^2 - (dt * 18)^2, x = 1024 clip(sign(I)
// sqrt|I|, -4, 4), with sign(0) = 0.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/flash_spacetime.h"

namespace fst {

constexpr float kTimeScale = 18.0f;    // 3e4 / 500 * 0.3, exact in fp32
constexpr float kInputScale = 1024.0f;
constexpr float kClip = 4.0f;
constexpr float kLog2e = 1.4426950408889634f;

template <typename T> __device__ __forceinline__ float to_f(T x);
template <> __device__ __forceinline__ float to_f<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) {
  return __bfloat162float(x);
}
template <> __device__ __forceinline__ float to_f<__half>(__half x) { return __half2float(x); }

template <typename T> __device__ __forceinline__ T from_f(float x);
template <> __device__ __forceinline__ float from_f<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}
template <> __device__ __forceinline__ __half from_f<__half>(float x) {
  return __float2half_rn(x);
}

// Layouts (FstProblem::packed): 0 padded [B, H, L, *]; 1 packed (varlen)
// [T, H, *] with cu_seqlens; 2 padded row-major [B, L, H, *] with seqlens --
// the caller's [B, L, H*Dh] projections without a head split. Layouts 1 and 2
// interleave heads within a row; only layout 1 uses the event tile list.
__host__ __device__ __forceinline__ bool is_varlen(const FstProblem& p) { return p.packed == 1; }
__host__ __device__ __forceinline__ bool rows_interleaved(const FstProblem& p) {
  return p.packed != 0;
}

// Whether the 16-bit kernels take their CTAs' (event, block) pairs from the
// device tile list (tile_prefix) rather than from a (L / BM, B) grid: always
// in the packed layout, and in the padded ones when the caller gave the
// valid row count (FstProblem::valid_rows) below B*L. The list then holds the
// live blocks only and the kernels launch about valid_rows / BM + B CTAs.
__host__ __device__ __forceinline__ bool uses_tile_list(const FstProblem& p) {
  return is_varlen(p) ||
         (p.valid_rows > 0 && p.valid_rows < p.total_rows && p.total_rows < (1ll << 31));
}
// A padded layout walked by the tile list: no CTA lies past an event's end,
// so a few CTAs at the head of the grid write the zero padding rows
// (pad_ctas), and the workspace holds a second prefix (of the padding row
// counts) after the tile prefix.
__host__ __device__ __forceinline__ bool list_padding(const FstProblem& p) {
  return !is_varlen(p) && uses_tile_list(p);
}
// Upper bound on the rows the tile list covers.
__host__ __device__ __forceinline__ int64_t list_rows(const FstProblem& p) {
  return is_varlen(p) ? p.total_rows : p.valid_rows;
}
// CTAs that write the zero padding rows of a padded tile-list grid, for a
// kernel that writes row_bytes per padding (row, head): one per 4 MiB of
// padding (B*L minus the valid rows), at least 1 and at most 32. A CTA
// stores at ~0.1 TB/s, so 32 of them leave most of the HBM bandwidth and
// every other SM to the live blocks; the launch adds them to the grid.
__host__ __device__ __forceinline__ int pad_ctas(const FstProblem& p, int row_bytes) {
  if (!list_padding(p)) return 0;
  const int64_t bytes = (p.total_rows - p.valid_rows) * p.heads * (int64_t)row_bytes;
  const int64_t z = bytes >> 22;
  return z < 1 ? 1 : (z > 32 ? 32 : (int)z);
}
// Whether the library ranks the events longest first itself
// (FST_FLAG_LONGEST_FIRST, at most kMaxSelfOrdered events) into the workspace.
constexpr int kMaxSelfOrdered = 1024;
__host__ __device__ __forceinline__ bool self_ordered(const FstProblem& p) {
  return (p.flags & FST_FLAG_LONGEST_FIRST) && !p.event_order && p.batch > 0;
}
// The tile-list workspace, in int32s: the tile prefix [B + 1]; for a padded
// layout walked by the list, the padding-row prefix [B + 1]; for a
// self-ordered problem, the event order [B] (order_offset).
__host__ __device__ __forceinline__ int64_t order_offset(const FstProblem& p) {
  return (int64_t)(p.batch + 1) * (list_padding(p) ? 2 : 1);
}
__host__ __device__ __forceinline__ int64_t tile_list_ints(const FstProblem& p) {
  return order_offset(p) + (self_ordered(p) ? p.batch : 0);
}

// Where one event lives. `row0` is the flat row of the event's first token in
// the [rows] index space (padded: b*L, packed: cu[b]); `len` its valid length.
// `base1`, `hs1` and `rs1` address its rows without any division: element
// (i, h, 0) of a per-row-per-head tensor with `dim` elements per (row, head)
// sits at (base1 + h*hs1 + i*rs1) * dim (ev_off).
struct EventSpan {
  int64_t row0;
  int len;
  int64_t base1;  // (event, head 0, row 0) in units of dim
  int64_t hs1;    // head stride in units of dim: packed 1, padded L
  int rs1;        // row stride in units of dim: packed H, padded 1
};

__device__ __forceinline__ EventSpan event_span(const FstProblem& p, int b) {
  EventSpan e;
  if (is_varlen(p)) {
    int s0 = p.cu_seqlens[b];
    e.row0 = s0;
    e.len = p.cu_seqlens[b + 1] - s0;
  } else {
    e.row0 = (int64_t)b * p.max_len;
    e.len = p.seqlens[b];
  }
  if (rows_interleaved(p)) {
    e.base1 = e.row0 * p.heads;
    e.hs1 = 1;
    e.rs1 = p.heads;
  } else {
    e.base1 = (int64_t)b * p.heads * p.max_len;
    e.hs1 = p.max_len;
    e.rs1 = 1;
  }
  return e;
}

// The span of the q, k, v inputs and the dq, dk, dv outputs of event b: as
// event_span, with the caller's row stride (a fused QKV buffer) in the
// row-interleaved layouts. `dim` is the head dimension.
__device__ __forceinline__ EventSpan qkv_span(const FstProblem& p, int b, int dim) {
  EventSpan e = event_span(p, b);
  if (rows_interleaved(p) && p.qkv_row_stride) {
    e.rs1 = p.qkv_row_stride / dim;
    e.base1 = e.row0 * e.rs1;
  }
  return e;
}

// Element offset of (row i of the event, head h, 0) in a [*, H, dim] (packed)
// or [B, H, L, dim] (padded) tensor.
__device__ __forceinline__ int64_t ev_off(const EventSpan& e, int i, int h, int dim) {
  return (e.base1 + h * e.hs1 + (int64_t)i * e.rs1) * dim;
}

// Event that owns packed row t: the largest b with cu[b] <= t (binary search).
__device__ __forceinline__ int packed_event_of(const int32_t* cu, int batch, int64_t t) {
  int lo = 0, hi = batch - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if ((int64_t)cu[mid] <= t) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// Element offset of (row, head, 0) in a [*, H, D] (packed) or [B, H, L, D]
// (padded) tensor, where `row` is a flat row index as in EventSpan.
__device__ __forceinline__ int64_t vec_off(const FstProblem& p, int64_t row, int h, int dim) {
  if (rows_interleaved(p)) return (row * p.heads + h) * (int64_t)dim;
  int64_t b = row / p.max_len;
  int64_t i = row - b * p.max_len;
  return ((b * p.heads + h) * p.max_len + i) * (int64_t)dim;
}

// Element stride between consecutive rows of one event for a fixed head:
// packed [T, H, D] rows are H*D apart, padded [B, H, L, D] rows D apart.
__device__ __forceinline__ int row_stride(const FstProblem& p, int dim) {
  return rows_interleaved(p) ? p.heads * dim : dim;
}

// row_stride for q, k, v, dq, dk, dv (the caller's qkv_row_stride if set).
__device__ __forceinline__ int qkv_row_stride(const FstProblem& p, int dim) {
  return (rows_interleaved(p) && p.qkv_row_stride) ? p.qkv_row_stride : row_stride(p, dim);
}

// vec_off for q, k, v, dq, dk, dv.
__device__ __forceinline__ int64_t qkv_off(const FstProblem& p, int64_t row, int h, int dim) {
  if (rows_interleaved(p) && p.qkv_row_stride) return row * p.qkv_row_stride + (int64_t)h * dim;
  return vec_off(p, row, h, dim);
}

// Offset of (row, head) in a per-row-per-head fp32 vector (LSE, D, sigma).
__device__ __forceinline__ int64_t stat_off(const FstProblem& p, int64_t row, int h) {
  return vec_off(p, row, h, 1);
}

struct Coord4 {
  float x, y, z, t;
};

__device__ __forceinline__ Coord4 load_coord(const FstProblem& p, int64_t row) {
  const float* f = p.feats + row * p.feat_stride;
  Coord4 c;
  c.x = f[0];
  c.y = f[1];
  c.z = f[2];
  c.t = f[3];
  return c;
}

// x_ij in fp32 (upstream _tiles.py:25-42).
__device__ __forceinline__ float pair_angle(const Coord4& a, const Coord4& b) {
  float dx = a.x - b.x, dy = a.y - b.y, dz = a.z - b.z;
  float dt = (a.t - b.t) * kTimeScale;
  float iv = dx * dx + dy * dy + dz * dz - dt * dt;
  float d = iv > 0.f ? sqrtf(iv) : -sqrtf(-iv);
  d = iv == 0.f ? 0.f : d;
  return kInputScale * fminf(fmaxf(d, -kClip), kClip);
}

// x * f - n * 2pi in [-pi, pi], with the product x*f taken exactly: Cody-Waite
// argument reduction (W. J. Cody and W. Waite, "Software Manual for the
// Elementary Functions", 1980) with 2*pi = C1 + C2 + C3, C1 = 6.28125 (8
// significant bits, so n * C1 is exact for |n| < 2^16) and the first FMA
// forming x*f - n*C1 from the unrounded product. |x*f| <= 4096 here.
__device__ __forceinline__ float reduce_2pi(float x, float f) {
  const float kInv2Pi = 0.15915494309189535f;
  const float kC1 = 6.28125f;
  const float kC2 = 1.9353071795864769e-03f;  // 2*pi - C1, rounded
  const float kC3 = 1.0253377e-11f;           // 2*pi - C1 - C2
  const float n = rintf(x * f * kInv2Pi);
  float r = fmaf(x, f, -n * kC1);
  r = fmaf(-n, kC2, r);
  return fmaf(-n, kC3, r);
}

}  // namespace fst
