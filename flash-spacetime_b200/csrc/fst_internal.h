// Internal declarations shared by the C-ABI front end and the kernel files.
#pragma once

#include <cuda_runtime.h>

#include "../../include/flash_spacetime.h"

namespace fst {
// Counts kernel launches made by this library (see fst_kernel_launches).
void count_launch(int n = 1);
namespace simt {
int launch_fwd(const FstForwardArgs& a, cudaStream_t st);
int launch_bwd(const FstBackwardArgs& a, cudaStream_t st);
size_t bwd_workspace(const FstProblem& p);
int64_t dw_parts(const FstProblem& p);
}  // namespace simt
namespace tc {
bool fwd_supported(const FstProblem& p);
size_t fwd_workspace(const FstProblem& p);
int launch_fwd(const FstForwardArgs& a, cudaStream_t st);
}  // namespace tc
}  // namespace fst
