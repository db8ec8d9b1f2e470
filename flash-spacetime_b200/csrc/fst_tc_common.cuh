// Device building blocks of the tensor-core kernels (sm_100a):
// warp-level bf16/fp16 MMA, ldmatrix/movmatrix, cp.async with mbarrier
// completion, named barriers, bounded mbarrier waits and the sin/cos of the
// pair embedding.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "fst_common.cuh"

namespace fst {
namespace tc {

// ---- element types ---------------------------------------------------------

template <typename T> struct Elem;
template <> struct Elem<__nv_bfloat16> {
  static constexpr uint32_t kOnes = 0x3f803f80u;  // (1.0, 1.0)
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
// Arrive on `bar` once all of this thread's prior cp.async copies completed.
__device__ __forceinline__ void cp_async_arrive(uint32_t bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];\n" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_init(uint32_t bar, int count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("{ .reg .b64 st; mbarrier.arrive.shared::cta.b64 st, [%0]; }\n" ::"r"(bar)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Error bits a kernel ORs into the caller's status word.
constexpr int kErrTimeout = 1;

// Spin on an mbarrier phase with an iteration cap (each try_wait already
// suspends for a hardware-chosen interval). On timeout the status word gets
// kErrTimeout and the caller carries on with whatever is in shared memory:
// the kernel always terminates and the host reports the error.
constexpr long kSpinLimit = 1L << 26;
__device__ __forceinline__ void mbar_wait(uint32_t bar, uint32_t parity, int* status) {
  long it = 0;
  while (!mbar_try_wait(bar, parity)) {
    if (++it > kSpinLimit) {
      if (status) atomicOr(status, kErrTimeout);
      return;
    }
  }
}

__device__ __forceinline__ void named_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(nthreads) : "memory");
}
__device__ __forceinline__ void named_arrive(int id, int nthreads) {
  asm volatile("bar.arrive %0, %1;\n" ::"r"(id), "r"(nthreads) : "memory");
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

// Projection of a block of rows through the encoder weight, in fp32:
//   out[q][h][c] = [ sum_d (x[q, h0+h, d] * mul) W[d][c] ]
// rounded once to T -- the same arithmetic as the host-side
// ((x.float() * mul) @ W).to(dtype) of upstream forward.py:279-286 and
// backward.py:546-547, up to the order of the DH-term sum. x is read from a
// staged shared tile [h][q][DHP] (the swizzled 16-bit layout the kernels
// stage Q and dO in); W comes from global memory (it is tiny and stays in
// L1). The result goes to a swizzled shared tile [q][16][CP] (head rows >= NH,
// channels >= C and rows >= nvalid are written as zeros) and, if gdst is
// given, to global memory in the [rows, H, C] layout, rows i0 + q of event ev.
template <typename T, int DH, int C, int CP, int RBD>
__device__ __forceinline__ void project_staged(const FstProblem& p, const unsigned char* xs,
                                               int rows_per_head, float mul, const EventSpan& ev,
                                               int i0, int nvalid, int nrows, int h0, int NH,
                                               unsigned char* tile, T* __restrict__ gdst) {
  using E = Elem<T>;
  constexpr int RBC = CP * 2;
  for (int idx = threadIdx.x; idx < nrows * 16 * (CP / 2); idx += blockDim.x) {
    const int c2 = idx % (CP / 2), h = (idx / (CP / 2)) % 16, q = idx / (16 * (CP / 2));
    uint32_t packed = 0u;
    if (q < nvalid && h < NH && 2 * c2 < C) {
      const unsigned char* xr = xs + h * rows_per_head * RBD;
      float a0 = 0.f, a1 = 0.f;
#pragma unroll
      for (int ch = 0; ch < DH / 8; ++ch) {
        const uint4 raw = *(const uint4*)(xr + swz<RBD>(q, ch));
        const uint32_t* w2 = (const uint32_t*)&raw;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int d = ch * 8 + 2 * e;
          const float x0 = E::lo(w2[e]) * mul, x1 = E::hi(w2[e]) * mul;
          const float2 wa = *(const float2*)(p.weight + (int64_t)d * C + 2 * c2);
          const float2 wb = *(const float2*)(p.weight + (int64_t)(d + 1) * C + 2 * c2);
          a0 = fmaf(x0, wa.x, a0);
          a1 = fmaf(x0, wa.y, a1);
          a0 = fmaf(x1, wb.x, a0);
          a1 = fmaf(x1, wb.y, a1);
        }
      }
      packed = E::pack(a0, a1);
      if (gdst) *(uint32_t*)(gdst + ev_off(ev, i0 + q, h0 + h, C) + 2 * c2) = packed;
    }
    if (tile) *(uint32_t*)(tile + swz<RBC>(q * 16 + h, c2 / 4) + (c2 % 4) * 4) = packed;
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

}  // namespace tc
}  // namespace fst
