// fst_forward_noalloc: the fused forward for callers that cannot allocate
// device memory.
//
// fst_forward takes its scratch (for the tensor-core kernels, the per-event
// tile prefix of a packed batch) from a workspace the caller allocates. Some
// callers cannot do that on the calling path: inference servers and plugin
// hosts that run with a fixed, pre-reserved memory pool, code running under a
// memory manager that forbids allocation after start-up, and real-time loops
// where a cudaMalloc (which can synchronise the device) is not allowed. This
// entry point runs the same kernels with that scratch taken from a file-scope
// device array instead, so it allocates nothing; the caller still passes the
// inputs and outputs.
//
// The array is kScratchBytes (256 KiB) per GPU. A problem whose workspace
// (fst_forward_workspace_size) exceeds it -- a 16-bit batch of more than
// 65535 events, or 32767 in a padded layout given valid_rows (whose tile list
// holds two prefixes) -- is rejected with FST_ERR_INVALID; problems that need no
// workspace (fp32 inputs) are not limited. Every GPU that loads the library
// holds the array until the process exits.
//
// Set-up: the first call on a device looks up the array's device address
// with cudaGetSymbolAddress (with that device current) and caches it for the
// life of the process; make that first call before any stream capture. A
// cudaDeviceReset on that device invalidates the cached address, so the entry
// point must not be used on a device after it was reset. Every call shares
// the one array and it keeps the last call's contents, so calls that overlap
// on the GPU (different streams, no ordering between them) race on it;
// serialise them on one stream or with events. The tile prefix is rewritten
// in full by every packed call before it is read, so nothing needs clearing.

#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "fst_internal.h"

namespace {

constexpr size_t kScratchBytes = 256 * 1024;

__device__ __align__(256) unsigned char g_fst_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_fst_scratch on the current device (looked up once per
// device; in host code the symbol itself is only a host-side stand-in).
int scratch_for_current_device(void** out, char* err, size_t errlen) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    snprintf(err, errlen, "fst_forward_noalloc: no usable current CUDA device");
    return FST_ERR_CUDA;
  }
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch_ptr[dev]) {
    void* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_fst_scratch);
    if (e != cudaSuccess || !ptr) {
      snprintf(err, errlen, "fst_forward_noalloc: cudaGetSymbolAddress failed: %s",
               cudaGetErrorString(e));
      return FST_ERR_CUDA;
    }
    g_scratch_ptr[dev] = ptr;
  }
  *out = g_scratch_ptr[dev];
  return FST_OK;
}

}  // namespace

extern "C" int fst_forward_noalloc(const FstForwardArgs* args, void* stream) {
  char err[256];
  if (!args) return fst::api_fail(FST_ERR_INVALID, "fst_forward_noalloc: null args");
  // The tensor-core forward's workspace is the int32 tile-list prefixes
  // (fst::tc::fwd_workspace); the fp32 kernels need none.
  const size_t need = fst_forward_workspace_size(&args->prob);
  if (need > kScratchBytes)
    return fst::api_fail(FST_ERR_INVALID,
                         "fst_forward_noalloc: %d events need %zu bytes of scratch, above the "
                         "built-in scratch limit of %zu bytes (at most 65535 events, 32767 padded with "
                         "valid_rows; use "
                         "fst_forward with a caller workspace)",
                         args->prob.batch, need, kScratchBytes);
  void* scratch = nullptr;
  const int rc = scratch_for_current_device(&scratch, err, sizeof(err));
  if (rc) return fst::api_fail(rc, "%s", err);
  FstForwardArgs a = *args;
  a.workspace = scratch;
  a.workspace_bytes = kScratchBytes;
  return fst_forward(&a, stream);
}
