// Host -> device transfer of the valid rows of a padded batch.
//
// A padded batch of variable-length events ([B, G, L, row] with event b's
// rows i >= len_b being padding) is mostly padding when the events are short
// next to L: on the workload the benchmark runs, 75 % of the rows. The kernels
// never read a padding row of an input (they zero-fill the shared-memory
// tiles past the event's end instead), so a data loader only has to ship the
// valid rows. In each (event, group) those are one contiguous span of
// len_b * row bytes.
//
// Page-locked (pinned) sources are gathered by a kernel that reads the host
// memory directly over the host link (mapped pinned memory): a few 128-thread
// CTAs walk the spans with 16-byte loads, four in flight per thread. A copy
// engine would need one descriptor per span and row, and moving ~3000 spans
// of ~12 KB that way is bound by the per-copy cost, not by the link. Each CTA
// holds 4096 registers and no shared memory, so it fits beside a resident
// forward or row-kernel CTA, and a copy issued on a side stream overlaps the
// step before.
// Pageable sources, or rows that are not a multiple of 16 bytes, fall back to
// one cudaMemcpy2DAsync per event.

#include <cuda_runtime.h>

#include "fst_internal.h"

namespace fst {
namespace io {

// Event lengths travel in the kernel's parameter block (no device buffer,
// no extra copy): at most kMaxEvents events per launch.
constexpr int kMaxEvents = 960;
struct EventLengths {
  int32_t len[kMaxEvents];
};
constexpr int kThreads = 128;

// A few CTAs keep the host link busy (each has 8 KB of loads in flight); a
// grid as wide as the spans would fill every SM and hold off the attention
// kernels of the step it is meant to overlap. Measured on the benchmark's
// config-1 batch: 8 CTAs are link-starved, 16-24 saturate it, 48 and more
// slow the overlapped step.
constexpr int kCtas = 24;

__global__ void __launch_bounds__(kThreads) gather_rows_kernel(
    uint4* __restrict__ dst, const uint4* __restrict__ src, const EventLengths lens, int groups,
    int spans, int64_t span_stride, int row_chunks) {
  for (int span = blockIdx.x; span < spans; span += gridDim.x) {
    // Span (event b, group g) of this launch's events; both tensors hold it
    // at the same offset.
    const int b = span / groups;
    const int64_t base = (int64_t)span * span_stride;
    const int64_t n = (int64_t)lens.len[b] * row_chunks;  // 16-byte chunks of valid rows
    const uint4* s = src + base;
    uint4* d = dst + base;
    for (int64_t i0 = threadIdx.x; i0 < n; i0 += 4 * kThreads) {
      uint4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t i = i0 + u * kThreads;
        if (i < n) v[u] = s[i];
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t i = i0 + u * kThreads;
        if (i < n) d[i] = v[u];
      }
    }
  }
}

// Whether the kernel may read `p` at the same address: page-locked host
// memory mapped into the device's address space at its host address (as
// cudaHostAlloc / cudaHostRegister memory is under unified addressing). The
// query leaves no CUDA error state behind.
bool mapped_host(const void* p) {
  cudaPointerAttributes at;
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return at.type == cudaMemoryTypeHost && at.devicePointer == p;
}
// Whether `p` is memory of the current device (or managed memory).
bool device_memory(const void* p) {
  cudaPointerAttributes at;
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return (at.type == cudaMemoryTypeDevice && at.device == dev) || at.type == cudaMemoryTypeManaged;
}

}  // namespace io
}  // namespace fst

extern "C" int fst_upload_rows(void* dst, const void* src, const int32_t* lens, int64_t batch,
                               int64_t groups, int64_t max_len, int64_t row_bytes,
                               void* stream) {
  using namespace fst::io;
  if (batch < 0 || groups < 1 || max_len < 0 || row_bytes < 1)
    return fst::api_fail(FST_ERR_INVALID,
                         "fst_upload_rows: batch %lld, groups %lld, max_len %lld, row_bytes %lld",
                         (long long)batch, (long long)groups, (long long)max_len,
                         (long long)row_bytes);
  if (batch == 0) return FST_OK;
  if (!dst || !src || !lens) return fst::api_fail(FST_ERR_INVALID, "fst_upload_rows: null pointer");
  // Every length is checked before the first copy is issued, so an invalid
  // request copies nothing; the gather kernel's spans then stay inside both
  // [batch][groups][max_len][row_bytes] tensors.
  for (int64_t b = 0; b < batch; ++b)
    if (lens[b] < 0 || lens[b] > max_len)
      return fst::api_fail(FST_ERR_INVALID,
                           "fst_upload_rows: lens[%lld] = %d outside [0, max_len = %lld]",
                           (long long)b, lens[b], (long long)max_len);
  cudaStream_t st = (cudaStream_t)stream;
  const size_t pitch = (size_t)max_len * (size_t)row_bytes;
  const size_t event_bytes = pitch * (size_t)groups;

  if (!device_memory(dst))
    return fst::api_fail(FST_ERR_INVALID,
                         "fst_upload_rows: dst is not memory of the current device");
  const bool vec = row_bytes % 16 == 0 && (uintptr_t)dst % 16 == 0 &&
                   (uintptr_t)src % 16 == 0 && mapped_host(src);
  if (vec && groups <= 65535) {
    const int row_chunks = (int)(row_bytes / 16);
    const int64_t span_stride = max_len * row_chunks;  // in 16-byte chunks
    for (int64_t b0 = 0; b0 < batch; b0 += kMaxEvents) {
      const int nev = (int)(batch - b0 < kMaxEvents ? batch - b0 : kMaxEvents);
      EventLengths el;
      for (int i = 0; i < nev; ++i) el.len[i] = lens[b0 + i];
      const size_t off = (size_t)b0 * event_bytes;
      const int spans = nev * (int)groups;
      gather_rows_kernel<<<spans < kCtas ? spans : kCtas, kThreads, 0, st>>>(
          (uint4*)((char*)dst + off), (const uint4*)((const char*)src + off), el, (int)groups,
          spans, span_stride, row_chunks);
      fst::count_launch();
      const cudaError_t e = cudaGetLastError();
      if (e != cudaSuccess)
        return fst::api_fail(FST_ERR_CUDA, "fst_upload_rows: gather launch: %s",
                             cudaGetErrorString(e));
    }
    return FST_OK;
  }
  for (int64_t b = 0; b < batch; ++b) {
    if (lens[b] == 0) continue;
    char* d = (char*)dst + (size_t)b * event_bytes;
    const char* s = (const char*)src + (size_t)b * event_bytes;
    const size_t width = (size_t)lens[b] * (size_t)row_bytes;
    cudaError_t e;
    if (groups == 1 || width == pitch)
      e = cudaMemcpyAsync(d, s, width + (size_t)(groups - 1) * pitch, cudaMemcpyHostToDevice, st);
    else
      e = cudaMemcpy2DAsync(d, pitch, s, pitch, width, (size_t)groups, cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess)
      return fst::api_fail(FST_ERR_CUDA, "fst_upload_rows: event %lld: %s", (long long)b,
                           cudaGetErrorString(e));
  }
  return FST_OK;
}
