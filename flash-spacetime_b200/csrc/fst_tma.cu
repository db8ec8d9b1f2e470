// Host side of the TMA copies: 2D tensor maps of the per-head tiles the
// tensor-core kernels stream (K and V, or qt and dO), encoded through the
// driver entry point that the runtime exposes (no link against libcuda).
//
// A map describes one 16-bit tensor addressed [*, H, Dh] as a 2D row view:
//   padded [B, H, L, Dh]          -> [B*H*L rows, Dh columns], row stride Dh
//   packed [T, H, Dh], [B, L, H, Dh] -> [rows, H*Dh columns], row stride as given
// with a box of 16 rows x Dh columns. Its shared-memory swizzle (32, 64 or
// 128 bytes for Dh = 16, 32, 64) puts the box in exactly the layout the
// kernels' swz<Dh * 2> addressing expects, so the MMA operand loads are the
// same whether a tile came by TMA or by cp.async.

#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "fst_internal.h"
#include "fst_tc_common.cuh"

namespace fst {
namespace tc {

namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

}  // namespace

bool tma_shape(int dh) { return dh == 16 || dh == 32 || dh == 64; }

int make_head_map(CUtensorMap* map, const FstProblem& p, const void* base, int row_elems) {
  const int dh = p.head_dim;
  if (!tma_shape(dh)) return FST_ERR_UNSUPPORTED;
  PFN_cuTensorMapEncodeTiled_v12000 encode = encode_fn();
  if (!encode) return api_fail(FST_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
  cuuint64_t dims[2], strides[1];
  if (rows_interleaved(p)) {
    dims[0] = (cuuint64_t)p.heads * dh;
    dims[1] = (cuuint64_t)p.total_rows;
    strides[0] = (cuuint64_t)row_elems * 2;
  } else {
    dims[0] = (cuuint64_t)dh;
    dims[1] = (cuuint64_t)p.batch * p.heads * p.max_len;
    strides[0] = (cuuint64_t)dh * 2;
  }
  if (dims[1] == 0) dims[1] = 1;  // empty problem: no CTA issues a copy
  const cuuint32_t box[2] = {(cuuint32_t)dh, 16u};
  const cuuint32_t estr[2] = {1u, 1u};
  const CUtensorMapSwizzle swz = dh == 16   ? CU_TENSOR_MAP_SWIZZLE_32B
                                 : dh == 32 ? CU_TENSOR_MAP_SWIZZLE_64B
                                            : CU_TENSOR_MAP_SWIZZLE_128B;
  auto run = [&] {
    return encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  };
  CUresult r = run();
  if (r == CUDA_ERROR_INVALID_CONTEXT) {
    // A thread that has made no runtime call yet (PyTorch runs backward on
    // its own device threads) has no current driver context: bind the
    // current device's primary context, as the runtime would, and retry.
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess && cudaSetDevice(dev) == cudaSuccess) r = run();
  }
  if (r != CUDA_SUCCESS)
    return api_fail(FST_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) for a [%llu x %llu] view",
                    (int)r, (unsigned long long)dims[1], (unsigned long long)dims[0]);
  return FST_OK;
}

}  // namespace tc
}  // namespace fst
