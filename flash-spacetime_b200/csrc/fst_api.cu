// C-ABI front end of libflash_spacetime.so: argument validation, workspace
// sizing, kernel selection and error reporting.
//
// Validation mirrors upstream's host checks (src/flash_spacetime/forward.py:
// 258-265: channel/head-dim constraints), generalised to W = [Dh, C] with C
// even. Errors are returned as status codes with a thread-local message; no
// call traps or aborts.

#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <atomic>
#include <cstdint>
#include <initializer_list>

#include "fst_common.cuh"
#include "fst_internal.h"

namespace fst {
static std::atomic<int64_t> g_launches{0};
void count_launch(int n) { g_launches.fetch_add(n, std::memory_order_relaxed); }
}  // namespace fst

namespace {

thread_local char g_err[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int check_problem(const FstProblem* p) {
  if (!p) return fail(FST_ERR_INVALID, "null problem");
  if (p->dtype < FST_F32 || p->dtype > FST_F16)
    return fail(FST_ERR_INVALID, "unknown dtype %d", p->dtype);
  if (p->batch < 0 || p->heads <= 0 || p->head_dim <= 0 || p->channels <= 0)
    return fail(FST_ERR_INVALID, "bad sizes B=%d H=%d Dh=%d C=%d", p->batch, p->heads,
                p->head_dim, p->channels);
  if (p->channels % 2)
    return fail(FST_ERR_INVALID, "C (=%d) must be even (sin/cos halves)", p->channels);
  if (p->head_dim > 64 || p->channels > 64)
    return fail(FST_ERR_UNSUPPORTED, "Dh (=%d) and C (=%d) must be <= 64", p->head_dim,
                p->channels);
  if (p->feat_stride < 4) return fail(FST_ERR_INVALID, "feat_stride must be >= 4");
  if (p->total_rows < 0) return fail(FST_ERR_INVALID, "negative total_rows");
  if (p->packed < 0 || p->packed > 2)
    return fail(FST_ERR_INVALID, "unknown layout %d (0 padded BHLD, 1 packed, 2 padded BLHD)",
                p->packed);
  if (p->packed == 1) {
    if (!p->cu_seqlens && p->batch > 0) return fail(FST_ERR_INVALID, "packed needs cu_seqlens");
  } else {
    // Padded grids put the events on grid.y (tiles of one event run next to
    // each other, which balances the SMs best); grid.y stops at 65535.
    if (p->batch > 65535)
      return fail(FST_ERR_UNSUPPORTED,
                  "padded batch of %d events: at most 65535 (use the packed layout)", p->batch);
    if (!p->seqlens && p->batch > 0) return fail(FST_ERR_INVALID, "padded needs seqlens");
    if ((int64_t)p->batch * p->max_len != p->total_rows)
      return fail(FST_ERR_INVALID, "padded total_rows must equal B*L");
  }
  if (p->valid_rows < 0) return fail(FST_ERR_INVALID, "negative valid_rows");
  if (p->flags & ~(FST_FLAG_SHARE_SMS | FST_FLAG_LONGEST_FIRST))
    return fail(FST_ERR_INVALID, "unknown flags 0x%x", (unsigned)p->flags);
  if (p->flags & FST_FLAG_LONGEST_FIRST) {
    if (p->event_order)
      return fail(FST_ERR_INVALID, "FST_FLAG_LONGEST_FIRST needs event_order = NULL");
    if (p->batch > fst::kMaxSelfOrdered)
      return fail(FST_ERR_INVALID, "FST_FLAG_LONGEST_FIRST: %d events, at most %d (pass an "
                  "event_order instead)", p->batch, fst::kMaxSelfOrdered);
  }
  if (p->qkv_row_stride) {
    if (p->packed == 0)
      return fail(FST_ERR_INVALID,
                  "qkv_row_stride applies to the row-interleaved layouts (packed 1 or 2)");
    if (p->qkv_row_stride < p->heads * p->head_dim || p->qkv_row_stride % p->head_dim ||
        p->qkv_row_stride % 8)
      return fail(FST_ERR_INVALID,
                  "qkv_row_stride (=%d) must be >= H*Dh (=%d) and a multiple of Dh and of 8",
                  p->qkv_row_stride, p->heads * p->head_dim);
  }
  if (p->total_rows > 0 && (!p->feats || !p->freqs))
    return fail(FST_ERR_INVALID, "feats and freqs are required");
  if ((p->use_attn_bias || p->use_act_bias) && p->total_rows > 0 && !p->weight)
    return fail(FST_ERR_INVALID, "weight is required when a bias term is on");
  return FST_OK;
}

// The tensor-core kernels move rows with 16-byte vector loads and cp.async,
// so every row-major tensor they touch must start on a 16-byte boundary and
// the feature rows must be a whole number of float4s apart.
bool aligned16(const void* ptr) { return ((uintptr_t)ptr & 15) == 0; }

int check_tc_alignment(const FstProblem& p, std::initializer_list<const void*> ptrs,
                       const char* what) {
  if (p.feat_stride % 4)
    return fail(FST_ERR_INVALID, "%s: feat_stride (=%d) must be a multiple of 4 for 16-bit inputs",
                what, p.feat_stride);
  if (!aligned16(p.feats))
    return fail(FST_ERR_INVALID, "%s: feats must be 16-byte aligned", what);
  for (const void* ptr : ptrs)
    if (!aligned16(ptr))
      return fail(FST_ERR_INVALID, "%s: tensor pointers must be 16-byte aligned", what);
  return FST_OK;
}

// A launch helper that failed has already recorded why; keep that text
// behind the entry point's own prefix.
int launch_fail(int code, const char* what) {
  char inner[sizeof(g_err)];
  strncpy(inner, g_err, sizeof(inner) - 1);
  inner[sizeof(inner) - 1] = '\0';
  return fail(code, "%s launch failed: %s", what, inner[0] ? inner : "(no detail)");
}

int cuda_status(const char* where) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(FST_ERR_CUDA, "%s: %s", where, cudaGetErrorString(e));
  return FST_OK;
}

}  // namespace

namespace fst {
int allow_dynamic_smem(const void* fn, int bytes, std::atomic<uint64_t>& done) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  const uint64_t bit = dev < 64 ? (uint64_t{1} << dev) : 0;
  if (bit && (done.load(std::memory_order_acquire) & bit)) return 0;
  e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return (int)e;
  done.fetch_or(bit, std::memory_order_release);
  return 0;
}

int api_fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}
}  // namespace fst

extern "C" {

int fst_abi_version(void) { return FST_ABI_VERSION; }

size_t fst_forward_workspace_size(const FstProblem* prob) {
  if (check_problem(prob) != FST_OK) return 0;
  return fst::tc::fwd_supported(*prob) ? fst::tc::fwd_workspace(*prob) : 0;
}

size_t fst_backward_workspace_size(const FstProblem* prob) {
  if (check_problem(prob) != FST_OK) return 0;
  return fst::tc::bwd_supported(*prob) ? fst::tc::bwd_workspace(*prob)
                                       : fst::simt::bwd_workspace(*prob);
}

int64_t fst_dw_partial_count(const FstProblem* prob) {
  if (check_problem(prob) != FST_OK) return 0;
  return fst::tc::bwd_supported(*prob) ? fst::tc::rows_partials(*prob)
                                       : fst::simt::dw_parts(*prob);
}

int fst_sum_partials(const FstProblem* prob, const float* dw_partial, const float* db_partial,
                     float* dw, float* db, void* stream) {
  const int rc = check_problem(prob);
  if (rc) return rc;
  const int64_t rows = fst_dw_partial_count(prob);
  if (rows > 0 && ((dw && !dw_partial) || (db && !db_partial)))
    return fail(FST_ERR_INVALID, "sum_partials: null partials");
  if (!dw && !db) return FST_OK;
  return fst::launch_sum_partials(dw_partial, db_partial, rows, prob->head_dim * prob->channels,
                                  prob->head_dim, dw, db, (cudaStream_t)stream);
}

int fst_forward(const FstForwardArgs* a, void* stream) {
  if (!a) return fail(FST_ERR_INVALID, "null args");
  int rc = check_problem(&a->prob);
  if (rc) return rc;
  const FstProblem& p = a->prob;
  if (p.total_rows > 0) {
    if (!a->q || !a->k || !a->v || !a->out || !a->lse)
      return fail(FST_ERR_INVALID, "forward: q, k, v, out and lse are required");
  }
  const size_t need = fst_forward_workspace_size(&p);
  if (need > 0 && (!a->workspace || a->workspace_bytes < need))
    return fail(FST_ERR_WORKSPACE, "forward: workspace %zu bytes < required %zu",
                a->workspace_bytes, need);
  if (fst::tc::fwd_supported(p) && p.total_rows > 0) {
    rc = check_tc_alignment(p, {a->q, a->k, a->v, a->u, a->out, a->workspace}, "forward");
    if (rc) return rc;
  }
  cudaGetLastError();  // clear a stale error so the check below is ours
  g_err[0] = '\0';
  if (fst::tc::fwd_supported(p)) {
    rc = fst::tc::launch_fwd(*a, (cudaStream_t)stream);
  } else {
    rc = fst::simt::launch_fwd(*a, (cudaStream_t)stream);
  }
  if (rc) return launch_fail(rc, "forward");
  return cuda_status("forward launch");
}

int fst_backward(const FstBackwardArgs* a, void* stream) {
  if (!a) return fail(FST_ERR_INVALID, "null args");
  int rc = check_problem(&a->prob);
  if (rc) return rc;
  const FstProblem& p = a->prob;
  if (!a->dw_partial || !a->db_partial)
    return fail(FST_ERR_INVALID, "backward: dw_partial and db_partial are required");
  if (p.total_rows > 0) {
    if (!a->q || !a->k || !a->v || !a->dout || !a->lse || !a->dq || !a->dk || !a->dv ||
        !a->delta || !a->sigma)
      return fail(FST_ERR_INVALID, "backward: a required pointer is null");
  }
  const size_t need = fst_backward_workspace_size(&p);
  if (need > 0 && (!a->workspace || a->workspace_bytes < need))
    return fail(FST_ERR_WORKSPACE, "backward: workspace %zu bytes < required %zu",
                a->workspace_bytes, need);
  if (fst::tc::bwd_supported(p) && p.total_rows > 0) {
    rc = check_tc_alignment(p, {a->q, a->k, a->v, a->u, a->out, a->dout, a->wt, a->dq, a->dk,
                                a->dv, a->workspace}, "backward");
    if (rc) return rc;
  }
  cudaGetLastError();
  g_err[0] = '\0';
  if (fst::tc::bwd_supported(p))
    rc = fst::tc::launch_bwd(*a, (cudaStream_t)stream);
  else
    rc = fst::simt::launch_bwd(*a, (cudaStream_t)stream);
  if (rc) return launch_fail(rc, "backward");
  return cuda_status("backward launch");
}

int64_t fst_kernel_launches(void) { return fst::g_launches.load(std::memory_order_relaxed); }

int fst_last_error(char* buf, size_t len) {
  const int n = (int)strlen(g_err);
  if (buf && len) {
    strncpy(buf, g_err, len - 1);
    buf[len - 1] = '\0';
  }
  return n;
}

}  // extern "C"
