// Device building blocks of the tensor-core kernels (sm_100a):
// warp-level bf16/fp16 MMA, ldmatrix/movmatrix, cp.async, named barriers,
// the sin/cos of the pair embedding and the tensor-core projection.
#pragma once

#include <cuda.h>  // CUtensorMap (the type only; maps are encoded on the host)
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "fst_common.cuh"

namespace fst {
namespace tc {

// The two TMA tensor maps a kernel streams per head: K and V (forward, row
// kernel) or qt and dO (column kernel). Each describes a 2D row view of a
// 16-bit tensor -- [B*H*L, Dh] for the padded layout, [rows, H*Dh] (row
// stride as given) for the row-interleaved ones -- with a [16 rows x Dh] box
// and the shared-memory swizzle that equals swz<Dh * 2> below. Passed by
// value as a __grid_constant__ kernel parameter.
struct __align__(64) TmaPair {
  CUtensorMap a, b;
};

// ---- element types ---------------------------------------------------------

template <typename T> struct Elem;
template <> struct Elem<__nv_bfloat16> {
  static constexpr uint32_t kOnes = 0x3f803f80u;  // (1.0, 1.0)
  static constexpr uint32_t kNaN2 = 0x7fc07fc0u;  // (NaN, NaN)
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
  }
  static __device__ __forceinline__ float lo(uint32_t v) { return __uint_as_float(v << 16); }
  static __device__ __forceinline__ float hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }
};
template <> struct Elem<__half> {
  static constexpr uint32_t kOnes = 0x3c003c00u;  // (1.0, 1.0)
  static constexpr uint32_t kNaN2 = 0x7e007e00u;  // (NaN, NaN)
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
  }
  static __device__ __forceinline__ float lo(uint32_t v) {
    return __half2float(__ushort_as_half((unsigned short)(v & 0xffff)));
  }
  static __device__ __forceinline__ float hi(uint32_t v) {
    return __half2float(__ushort_as_half((unsigned short)(v >> 16)));
  }
};

// D += A(16x16) * B(16x8), fp32 accumulate. A/B are both bf16 or both fp16.
template <typename T>
__device__ __forceinline__ void mma16816(float* d, const uint32_t* a, const uint32_t* b);
template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float* d, const uint32_t* a,
                                                        const uint32_t* b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
template <>
__device__ __forceinline__ void mma16816<__half>(float* d, const uint32_t* a, const uint32_t* b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// ---- shared memory access --------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];\n"
               : "=r"(r[0]), "=r"(r[1])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2_t(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];\n"
               : "=r"(r[0]), "=r"(r[1])
               : "r"(addr));
}

// In-register transpose of an 8x8 b16 tile held in mma fragment order.
__device__ __forceinline__ uint32_t movm_t(uint32_t x) {
  uint32_t r;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;\n" : "=r"(r) : "r"(x));
  return r;
}

__device__ __forceinline__ void sts_v2(uint32_t addr, float a, float b) {
  asm volatile("st.shared.v2.f32 [%0], {%1, %2};\n" ::"r"(addr), "f"(a), "f"(b) : "memory");
}
__device__ __forceinline__ void sts_u32(uint32_t addr, uint32_t v) {
  asm volatile("st.shared.u32 [%0], %1;\n" ::"r"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ float2 lds_v2(uint32_t addr) {
  float2 r;
  asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];\n" : "=f"(r.x), "=f"(r.y) : "r"(addr) : "memory");
  return r;
}

// Row swizzle of a tile whose rows are `RB` bytes (a power of two, 32..128):
// the 16-byte chunk c of row r moves to chunk c ^ ((r / (128/RB)) % (RB/16)),
// so 8 consecutive rows read at the same logical chunk hit 8 distinct
// 16-byte bank groups (conflict-free ldmatrix).
template <int RB>
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  static_assert(RB == 32 || RB == 64 || RB == 128, "row bytes");
  constexpr int kChunks = RB / 16;
  constexpr int kRowsPerLine = 128 / RB;
  return (uint32_t)(row * RB + ((chunk ^ ((row / kRowsPerLine) % kChunks)) << 4));
}

// ---- async copies and barriers --------------------------------------------

__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}
// Wait until at most N of this thread's committed cp.async groups are pending.
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}
__device__ __forceinline__ void named_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(nthreads) : "memory");
}
__device__ __forceinline__ void named_arrive(int id, int nthreads) {
  asm volatile("bar.arrive %0, %1;\n" ::"r"(id), "r"(nthreads) : "memory");
}

// ---- mbarriers and TMA (cp.async.bulk.tensor) -------------------------------

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
}
// Makes initialised barriers visible to the async proxy (the TMA unit).
__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}
// One arrival that also expects `bytes` of TMA transactions on this phase.
__device__ __forceinline__ void mbar_arrive_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}
// Waits for the phase of parity `parity` to complete, giving up after a
// bounded number of polls (each try_wait itself suspends for a while), so a
// transfer that never lands cannot hang the GPU. Returns false on give-up.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  for (int i = 0; i < (1 << 22); ++i)
    if (mbar_test(bar, parity)) return true;
  return false;
}
// Orders this thread's earlier generic-proxy accesses of shared memory before
// its later async-proxy (TMA) writes to it.
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}
// 2D tiled TMA load of the box at (x = column, y = row) of `map` into `dst`,
// completing `bar`'s transaction count. x * 2 bytes is a multiple of 16 (x is
// a multiple of Dh); rows past the tensor's end read as zeros.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];\n" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
      : "memory");
}

// ---- math ------------------------------------------------------------------

__device__ __forceinline__ float ex2(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// sin and cos of x*f for the 16-bit kernels. Exact-product Cody-Waite
// reduction to [-pi, pi] (as reduce_2pi, with the third constant dropped: its
// contribution is < 1e-8 rad for |n| <= 652), the nearest integer n formed on
// the FMA pipe by the 1.5*2^23 rounding constant instead of rintf, and the
// hardware sin.approx / cos.approx (absolute error ~1e-6 on [-pi, pi], far
// below the 16-bit rounding of E). f_rev = f / (2 pi) is precomputed.
__device__ __forceinline__ void sincos_xf(float x, float f, float f_rev, float& s, float& c) {
  const float kRound = 12582912.f;            // 1.5 * 2^23
  const float kC1 = 6.28125f;
  const float kC2 = 1.9353071795864769e-03f;
  const float n = fmaf(x, f_rev, kRound) - kRound;
  float r = fmaf(x, f, -n * kC1);
  r = fmaf(-n, kC2, r);
  s = __sinf(r);
  c = __cosf(r);
}

// sincos_xf for two frequencies at once: the same operations, issued as the
// packed two-lane fp32 instructions of sm_100 (fma/sub/mul .rn.f32x2), so the
// reduction of both arguments costs the issue slots of one.
__device__ __forceinline__ uint64_t f2pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ void sincos_xf2(float x, const float (&f)[2], const float (&f_rev)[2],
                                           float (&s)[2], float (&c)[2]) {
  const uint64_t x2 = f2pack(x, x);
  const uint64_t fr2 = f2pack(f_rev[0], f_rev[1]), f2 = f2pack(f[0], f[1]);
  const uint64_t kRound2 = f2pack(12582912.f, 12582912.f);  // 1.5 * 2^23
  const uint64_t kNegC1 = f2pack(-6.28125f, -6.28125f);
  const uint64_t kNegC2 = f2pack(-1.9353071795864769e-03f, -1.9353071795864769e-03f);
  uint64_t n2, m2, r2;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(n2) : "l"(x2), "l"(fr2), "l"(kRound2));
  asm("sub.rn.f32x2 %0, %0, %1;" : "+l"(n2) : "l"(kRound2));
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(m2) : "l"(n2), "l"(kNegC1));
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r2) : "l"(x2), "l"(f2), "l"(m2));
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(r2) : "l"(n2), "l"(kNegC2));
  float r0, r1;
  f2unpack(r2, r0, r1);
  s[0] = __sinf(r0);
  c[0] = __cosf(r0);
  s[1] = __sinf(r1);
  c[1] = __cosf(r1);
}

// x_ij for the 16-bit kernels: as pair_angle, with the square root taken by
// sqrt.approx (one MUFU op) and the clip applied before it -- |I| >= 16 maps
// straight to +-4096, the exact value the clipped branch takes.
__device__ __forceinline__ float pair_angle_fast(const Coord4& a, const Coord4& b) {
  const float dx = a.x - b.x, dy = a.y - b.y, dz = a.z - b.z;
  const float dt = (a.t - b.t) * kTimeScale;
  const float iv = dx * dx + dy * dy + dz * dz - dt * dt;
  const float m = fabsf(iv);
  float r;
  asm("sqrt.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(m));
  const float x = m >= 16.f ? 4096.f : kInputScale * r;
  return copysignf(x, iv);
}

// Projection of one head's block of BM rows through the encoder weight on the
// tensor cores, the arithmetic of the host-side ((x.float() * mul) @ W).to(T)
// of upstream forward.py:279-286 and backward.py:546-547:
//   out[q][c] = [ mul * sum_d x[q][d] W[d][c] ]
// x comes from the staged swizzled tile of this head ([BM][DHP], 16-bit, as
// the kernels stage Q and dO), W from the staged [DH][CP] tiles of its hi and
// lo halves in T (W = W_hi + W_lo to ~16 significant bits; x is exact in T),
// the products are accumulated in fp32 and rounded once to T. One warp per
// head: rows q < nvalid go to gdst (rows i0 + q of event ev, head h), and, if
// tile is given, all BM rows go to row (q * 16 + hl) of the swizzled
// [BM][16][CP] tile the heads-on-M MMAs read.
template <typename T, int DH, int C, int CP, int RBD, int BM>
__device__ __forceinline__ void project_mma(uint32_t x_tile, uint32_t w_hi, uint32_t w_lo,
                                            float mul, const EventSpan& ev, int i0, int nvalid,
                                            int h, int hl, unsigned char* tile,
                                            T* __restrict__ gdst) {
  using E = Elem<T>;
  constexpr int RG = BM / 16, KSD = DH / 16, NTC = C / 8, RBC = CP * 2;
  static_assert(NTC % 2 == 0, "n-tiles come in pairs");
  const int lane = threadIdx.x & 31, m4 = lane & 3, r8 = lane >> 2, mi = lane >> 3;
  float acc[RG][NTC][4];
#pragma unroll
  for (int rg = 0; rg < RG; ++rg)
#pragma unroll
    for (int nc = 0; nc < NTC; ++nc)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[rg][nc][i] = 0.f;
#pragma unroll
  for (int ks = 0; ks < KSD; ++ks) {
    // W B-fragments (k = d, n = c) from the [d][c] tiles by transposed loads.
    uint32_t bh[NTC][2], bl[NTC][2];
#pragma unroll
    for (int np = 0; np < NTC / 2; ++np) {
      const uint32_t off = swz<RBC>(ks * 16 + (mi & 1) * 8 + (lane & 7), 2 * np + (mi >> 1));
      uint32_t r[4];
      ldsm_x4_t(w_hi + off, r);
      bh[2 * np][0] = r[0];
      bh[2 * np][1] = r[1];
      bh[2 * np + 1][0] = r[2];
      bh[2 * np + 1][1] = r[3];
      ldsm_x4_t(w_lo + off, r);
      bl[2 * np][0] = r[0];
      bl[2 * np][1] = r[1];
      bl[2 * np + 1][0] = r[2];
      bl[2 * np + 1][1] = r[3];
    }
#pragma unroll
    for (int rg = 0; rg < RG; ++rg) {
      uint32_t xa[4];
      ldsm_x4(x_tile + swz<RBD>(rg * 16 + (mi & 1) * 8 + (lane & 7), 2 * ks + (mi >> 1)), xa);
#pragma unroll
      for (int nc = 0; nc < NTC; ++nc) {
        mma16816<T>(acc[rg][nc], xa, bh[nc]);
        mma16816<T>(acc[rg][nc], xa, bl[nc]);
      }
    }
  }
#pragma unroll
  for (int rg = 0; rg < RG; ++rg)
#pragma unroll
    for (int rh = 0; rh < 2; ++rh) {
      const int q = rg * 16 + r8 + 8 * rh;
      T* grow = (gdst != nullptr && q < nvalid) ? gdst + ev_off(ev, i0 + q, h, C) : nullptr;
#pragma unroll
      for (int nc = 0; nc < NTC; ++nc) {
        const int c = nc * 8 + 2 * m4;
        const uint32_t v = E::pack(acc[rg][nc][2 * rh] * mul, acc[rg][nc][2 * rh + 1] * mul);
        if (grow) *(uint32_t*)(grow + c) = v;
        if (tile) *(uint32_t*)(tile + swz<RBC>(q * 16 + hl, nc) + m4 * 4) = v;
      }
    }
}

// Multiply a staged [h][q][DHP] 16-bit tile by `mul` in place, rounding once.
template <typename T, int DH, int RBD>
__device__ __forceinline__ void scale_staged(unsigned char* xs, int nheads, int rows_per_head,
                                             float mul) {
  using E = Elem<T>;
  constexpr int CH = DH / 8;
  for (int idx = threadIdx.x; idx < nheads * rows_per_head * CH; idx += blockDim.x) {
    const int c = idx % CH, q = (idx / CH) % rows_per_head, h = idx / (CH * rows_per_head);
    uint4* ptr = (uint4*)(xs + h * rows_per_head * RBD + swz<RBD>(q, c));
    uint4 v = *ptr;
    uint32_t* w = (uint32_t*)&v;
#pragma unroll
    for (int k = 0; k < 4; ++k) w[k] = E::pack(E::lo(w[k]) * mul, E::hi(w[k]) * mul);
    *ptr = v;
  }
}

// Copy [rows, H, C] rows given by the caller into the same swizzled tile
// layout project_staged produces.
template <typename T, int C, int CP>
__device__ __forceinline__ void stage_rows(const T* __restrict__ src, const EventSpan& ev,
                                           int i0, int nvalid, int nrows, int h0, int NH,
                                           unsigned char* tile) {
  constexpr int RBC = CP * 2, UCH = CP / 8;
  for (int idx = threadIdx.x; idx < nrows * 16 * UCH; idx += blockDim.x) {
    const int c = idx % UCH, h = (idx / UCH) % 16, q = idx / (UCH * 16);
    uint4 v = make_uint4(0, 0, 0, 0);
    if (q < nvalid && h < NH && c * 8 < C)
      v = *(const uint4*)(src + ev_off(ev, i0 + q, h0 + h, C) + c * 8);
    *(uint4*)(tile + swz<RBC>(q * 16 + h, c)) = v;
  }
}

// ---- the device tile list ---------------------------------------------------

// Entry t of the tile list (tile_prefix: the exclusive prefix tile_start[0..B]
// of each event's block count, events in p.event_order): its event b and the
// block's index within the event. False past the list's end.
__host__ __device__ __forceinline__ bool list_tile(const FstProblem& p,
                                                   const int* __restrict__ tile_start, int t,
                                                   int& b, int& blk) {
  if (t >= tile_start[p.batch]) return false;
  int lo = 0, hi = p.batch - 1;
  while (lo < hi) {  // last position with tile_start[pos] <= t
    const int mid = (lo + hi + 1) >> 1;
    if (tile_start[mid] <= t) lo = mid; else hi = mid - 1;
  }
  blk = t - tile_start[lo];
  b = p.event_order ? p.event_order[lo] : lo;
  return true;
}

// Writes the 16-bit pair `v2` to rows [r0, r1) of heads [h0, h0 + nh) of event
// e in a [*, H, DIM]-addressed tensor (16-byte stores; DIM a multiple of 8),
// and `s` to the same (row, head) entries of the fp32 vectors s0 and s1 (each
// may be NULL) addressed by es.
template <typename T, int DIM>
__device__ __forceinline__ void fill_rows(T* __restrict__ base, const EventSpan& e,
                                          float* __restrict__ s0, float* __restrict__ s1,
                                          const EventSpan& es, int r0, int r1, int h0, int nh,
                                          uint32_t v2, float s) {
  constexpr int CH = DIM / 8;
  const int per_row = nh * CH;
  const int n = (r1 - r0) * per_row;
  for (int idx = threadIdx.x; idx < n; idx += blockDim.x) {
    const int r = idx / per_row, rem = idx - r * per_row;
    const int h = h0 + rem / CH, c = rem % CH;
    // Streaming stores: nothing reads these rows again in the kernel, so they
    // should not push the live blocks' K / V out of L2.
    __stcs((uint4*)(base + ev_off(e, r0 + r, h, DIM) + c * 8), make_uint4(v2, v2, v2, v2));
    if (c == 0) {
      if (s0) __stcs(s0 + ev_off(es, r0 + r, h, 1), s);
      if (s1) __stcs(s1 + ev_off(es, r0 + r, h, 1), s);
    }
  }
}

// A padded layout walked by the tile list has no CTA past an event's end, so
// the padding rows [len_b, max_len) of all events are split evenly into n
// shares (pad_start: the exclusive prefix of max_len - len_b in natural event
// order, written by tile_prefix). For share t, fn(b, r0, r1) is called for
// each row range it holds -- one or a few, in ascending rows. (Host-
// callable, like list_tile and list_padded_role, so that a CPU test can check
// the row arithmetic of the padding writers.)
#pragma nv_exec_check_disable
template <typename F>
__host__ __device__ __forceinline__ void padding_share(const FstProblem& p,
                                                       const int* __restrict__ pad_start, int t,
                                                       int n, F&& fn) {
  const int64_t total = pad_start[p.batch];
  int64_t r = total * t / n;
  const int64_t r1 = total * (t + 1) / n;
  if (r >= r1) return;
  int lo = 0, hi = p.batch - 1;
  while (lo < hi) {  // the event whose padding holds row r
    const int mid = (lo + hi + 1) >> 1;
    if (pad_start[mid] <= r) lo = mid; else hi = mid - 1;
  }
  for (int b = lo; b < p.batch && r < r1; ++b) {
    const int64_t s0 = pad_start[b];
    const int64_t s1 = r1 < pad_start[b + 1] ? r1 : (int64_t)pad_start[b + 1];
    if (s1 <= r) continue;                                 // no padding rows in event b
    const int len = p.max_len - (pad_start[b + 1] - pad_start[b]);  // clamped seqlens[b]
    fn(b, len + (int)(r - s0), len + (int)(s1 - s0));
    r = s1;
  }
}

// Role of CTA t of a grid of g (blockIdx.x, gridDim.x) in a padded layout
// walked by the tile list (list_padding). Such a grid is n_tiles live blocks
// after zc = g - n_tiles CTAs.
// The first nz = min(zc, writers) of those write the zero padding rows,
// split evenly between them, while the live blocks run beside them
// (`writers` = pad_ctas, which the launch adds to the grid); the others exit.
// Returns the tile-list entry this CTA computes, or kRoleDone. When the
// caller's valid_rows was too small for the grid to hold every live block
// (zc < 1), every CTA writes its share of the padding and NaN in every valid
// row of the blocks t, t + g, ..., and returns kRolePoisoned. fill(b, r0, r1,
// nan) writes rows [r0, r1) of event b: zeros, or NaN when nan != 0.
constexpr int kRoleDone = -1, kRolePoisoned = -2;
#pragma nv_exec_check_disable
template <typename F>
__host__ __device__ __forceinline__ int list_padded_role(const FstProblem& p,
                                                         const int* __restrict__ tile_start,
                                                         int bm, int writers, int t, int g,
                                                         F&& fill) {
  const int n_tiles = tile_start[p.batch];
  const int zc = g - n_tiles;
  const int* pad_start = tile_start + p.batch + 1;
  auto zero = [&](int b, int r0, int r1) { fill(b, r0, r1, 0); };
  if (zc >= 1) {
    if (t >= zc) return t - zc;
    const int nz = zc < writers ? zc : writers;
    if (t < nz) padding_share(p, pad_start, t, nz, zero);
    return kRoleDone;
  }
  padding_share(p, pad_start, t, g, zero);
  for (int tt = t; tt < n_tiles; tt += g) {
    int b, blk;
    list_tile(p, tile_start, tt, b, blk);
    const int sl = p.seqlens[b] < 0 ? 0 : p.seqlens[b];
    const int len = sl < p.max_len ? sl : p.max_len;
    fill(b, blk * bm, len < (blk + 1) * bm ? len : (blk + 1) * bm, 1);
  }
  return kRolePoisoned;
}

}  // namespace tc
}  // namespace fst
