// Internal declarations shared by the C-ABI front end and the kernel files.
#pragma once

#include <cuda_runtime.h>

#include "../../include/flash_spacetime.h"

namespace fst {
namespace simt {
int launch_fwd(const FstForwardArgs& a, cudaStream_t st);
int launch_bwd(const FstBackwardArgs& a, cudaStream_t st);
size_t bwd_workspace(const FstProblem& p);
int64_t dw_parts(const FstProblem& p);
}  // namespace simt
}  // namespace fst
