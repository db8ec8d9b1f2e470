// Fixed-order sums of the backward's per-CTA dW / db partials.
//
// fst_backward leaves one [Dh, C] dW partial and one [Dh] db partial per
// row-kernel CTA (thousands of them), so that dW and db never need atomics.
// Upstream forms the same sums on the host side of its backward
// (backward.py:607-622). Here one launch reduces both: a thread-block cluster
// of kSplit CTAs per 32 output columns, each CTA summing 1/kSplit of the
// rows (16 warps, eight 128-byte row loads in flight per warp), and the
// cluster's rank-0 CTA adding the kSplit segment sums from the others' shared
// memory (DSMEM) in rank order. Which partials a warp adds, and in which
// order, depends only on the problem's partial count, so the sums are
// bitwise reproducible.

#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include "fst_internal.h"

namespace fst {
namespace {

namespace cg = cooperative_groups;

constexpr int kSplit = 8;     // CTAs of a cluster (row segments); portable cluster size
constexpr int kWarps = 16;    // warps of a CTA
constexpr int kInFlight = 8;  // row loads a warp keeps in flight

// blockIdx.x: a 32-column block of [dW columns | db columns]; blockIdx.y:
// the row segment (rank in the cluster).
__global__ void __cluster_dims__(1, kSplit, 1) __launch_bounds__(kWarps * 32)
    sum_partials_kernel(const float* __restrict__ dwp, const float* __restrict__ dbp,
                        int64_t rows, int ncw, int ncb, float* __restrict__ dw,
                        float* __restrict__ db) {
  __shared__ float acc[kWarps][32];
  __shared__ float seg[32];
  cg::cluster_group cluster = cg::this_cluster();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nbw = (ncw + 31) / 32;
  const bool is_w = (int)blockIdx.x < nbw;
  const float* part = is_w ? dwp : dbp;
  float* out = is_w ? dw : db;
  const int cols = is_w ? ncw : ncb;
  const int col = ((int)blockIdx.x - (is_w ? 0 : nbw)) * 32 + lane;
  const int rank = (int)cluster.block_rank();
  const int64_t r0 = rows * rank / kSplit, r1 = rows * (rank + 1) / kSplit;
  float s = 0.f;
  if (out && col < cols) {
    int64_t r = r0 + warp;
    constexpr int kStep = kWarps * kInFlight;
    for (; r + (kInFlight - 1) * kWarps < r1; r += kStep) {
      float v[kInFlight];
#pragma unroll
      for (int i = 0; i < kInFlight; ++i) v[i] = part[(r + i * kWarps) * cols + col];
#pragma unroll
      for (int i = 0; i < kInFlight; ++i) s += v[i];
    }
    for (; r < r1; r += kWarps) s += part[r * cols + col];
  }
  acc[warp][lane] = s;
  __syncthreads();
  if (warp == 0) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) t += acc[w][lane];
    seg[lane] = t;
  }
  cluster.sync();  // every CTA's segment sum is in its shared memory
  if (rank == 0 && warp == 0 && out && col < cols) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < kSplit; ++k) t += cluster.map_shared_rank(seg, k)[lane];
    out[col] = t;
  }
  cluster.sync();  // the others' shared memory stays until rank 0 has read it
}

}  // namespace

int launch_sum_partials(const float* dw_partial, const float* db_partial, int64_t rows, int ncw,
                        int ncb, float* dw, float* db, cudaStream_t st) {
  const dim3 grid((ncw + 31) / 32 + (ncb + 31) / 32, kSplit);
  sum_partials_kernel<<<grid, kWarps * 32, 0, st>>>(dw_partial, db_partial, rows, ncw, ncb, dw,
                                                      db);
  const cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess)
    return api_fail(FST_ERR_CUDA, "sum_partials: launch: %s", cudaGetErrorString(err));
  count_launch();
  return FST_OK;
}
}  // namespace fst
