// fst_forward_noalloc: the fused forward for callers that cannot allocate
// device memory.
//
// fst_forward takes its scratch (a status word and, for packed batches, the
// per-event tile prefix) from a workspace the caller allocates. Some callers
// cannot do that on the calling path: inference servers and plugin hosts that
// run with a fixed, pre-reserved memory pool, code running under a memory
// manager that forbids allocation after start-up, and real-time loops where a
// cudaMalloc (which can synchronise the device) is not allowed. This entry
// point runs the same kernels with that scratch taken from a file-scope
// device array instead, so it allocates nothing; the caller still passes the
// inputs and outputs.
//
// The array is kScratchBytes (256 KiB) per GPU, enough for batches of up to
// kMaxEvents events; larger batches are rejected with FST_ERR_INVALID. Every
// GPU that loads the library holds the array until the process exits.
//
// Set-up: the first call on a device looks up the array's device address
// with cudaGetSymbolAddress (with that device current) and caches it; make
// that first call before any stream capture. Every call then shares the one
// array and it keeps the last call's contents, so calls that overlap on the
// GPU (different streams, no ordering between them) race on it; serialise
// them on one stream or with events. The status word is cleared on every
// call; the tile prefix is rewritten in full by every packed call.

#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "fst_internal.h"

namespace {

constexpr size_t kScratchBytes = 256 * 1024;
// Workspace layout of the tensor-core forward: 64 bytes of status, then the
// (batch + 1)-entry int32 tile prefix (fst::tc::fwd_workspace).
constexpr int kMaxEvents = (int)((kScratchBytes - 64) / sizeof(int)) - 1;

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
  if (args->prob.batch > kMaxEvents)
    return fst::api_fail(FST_ERR_INVALID,
                         "fst_forward_noalloc: %d events exceed the built-in scratch limit of "
                         "%d events (use fst_forward with a caller workspace)",
                         args->prob.batch, kMaxEvents);
  void* scratch = nullptr;
  const int rc = scratch_for_current_device(&scratch, err, sizeof(err));
  if (rc) return fst::api_fail(rc, "%s", err);
  FstForwardArgs a = *args;
  a.workspace = scratch;
  a.workspace_bytes = kScratchBytes;
  return fst_forward(&a, stream);
}
