// Internal declarations shared by the C-ABI front end and the kernel files.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>

#include "../../include/flash_spacetime.h"

namespace fst {
// Counts kernel launches made by this library (see fst_kernel_launches).
void count_launch(int n = 1);
// Records a formatted error message for fst_last_error and returns `code`.
int api_fail(int code, const char* fmt, ...);
// Raises `fn`'s dynamic shared memory limit to `bytes` on the current device,
// once per device (bit d of `done`); returns 0 or a cudaError_t.
int allow_dynamic_smem(const void* fn, int bytes, std::atomic<uint64_t>& done);
// fst_sum_partials after validation: one launch summing `rows` partial rows
// of ncw dW and ncb db columns in a fixed order (NULL outputs skipped).
int launch_sum_partials(const float* dw_partial, const float* db_partial, int64_t rows, int ncw,
                        int ncb, float* dw, float* db, cudaStream_t st);
namespace simt {
int launch_fwd(const FstForwardArgs& a, cudaStream_t st);
int launch_bwd(const FstBackwardArgs& a, cudaStream_t st);
size_t bwd_workspace(const FstProblem& p);
int64_t dw_parts(const FstProblem& p);
}  // namespace simt
namespace tc {
// TMA tensor map of a 16-bit [*, H, Dh]-addressed tensor of problem p (the 2D
// row view described in fst_tma.cu); row_elems is its row stride in elements
// for the row-interleaved layouts. Only Dh in {16, 32, 64} (tma_shape).
bool tma_shape(int dh);
int make_head_map(CUtensorMap* map, const FstProblem& p, const void* base, int row_elems);
bool fwd_supported(const FstProblem& p);
size_t fwd_workspace(const FstProblem& p);
int launch_fwd(const FstForwardArgs& a, cudaStream_t st);
// The device tile list (uses_tile_list): exclusive prefix of ceil(len_b / bm)
// over the events, in p.event_order when given, written to tile_start[0..B],
// and for a padded layout the prefix of the padding row counts after it (one
// small kernel; no host synchronisation).
void tile_prefix(const FstProblem& p, int bm, int* tile_start, cudaStream_t st);
int launch_bwd_rows(const FstBackwardArgs& a, cudaStream_t st, int* tile_start, void* u_ws,
                    void* wt_ws, void* qt_ws);
int launch_bwd_cols(const FstBackwardArgs& a, cudaStream_t st, int* tile_start, const void* gu,
                    const void* gwt, const void* gqt);
int64_t rows_partials(const FstProblem& p);
bool bwd_supported(const FstProblem& p);
size_t bwd_workspace(const FstProblem& p);
int launch_bwd(const FstBackwardArgs& a, cudaStream_t st);
}  // namespace tc
}  // namespace fst
