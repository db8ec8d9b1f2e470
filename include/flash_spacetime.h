/*
 * flash_spacetime.h -- C ABI of the B200 (sm_100a) fused spacetime-bias
 * attention library (libflash_spacetime.so).
 *
 * The library computes, per event and head,
 *
 *   s_ij  = qt_i . k_j + [attn] u_i . E_ij          (qt = q * scale, u = qt W)
 *   P     = softmax_j(s)
 *   out_i = sum_j P_ij v_j + [act] (sum_j P_ij E_ij) W^T + b
 *
 * with E_ij the C-channel sinusoidal embedding of the clipped, signed
 * spacetime interval between pulses i and j, and its gradients. It replaces
 * the Triton launches of the upstream package:
 *
 *   fst_forward   <- flash_spacetime_fwd_kernel launch and the host epilogue
 *                    of flash_spacetime_forward
 *                    (upstream src/flash_spacetime/forward.py:222-346,
 *                    kernel forward.py:63-219)
 *   fst_backward  <- flash_spacetime_bwd_rows_kernel + _cols_kernel launches
 *                    and the dq/dW epilogue of flash_spacetime_backward
 *                    (upstream src/flash_spacetime/backward.py:488-630,
 *                    kernels backward.py:209-485)
 *
 * Everything is plain C: raw device pointers, sizes and a cudaStream_t passed
 * as void*. The caller (the PyTorch autograd Function in flash_spacetime/ops.py,
 * or any other host) owns every buffer; the library allocates no device
 * memory. Calls are stream-ordered and asynchronous; a non-zero return is an
 * error whose text fst_last_error() returns (thread-local).
 *
 * Layouts (contiguous, row-major):
 *   padded (packed == 0): q,k,v,u,out,dout,wt [B, H, L, D*] ; feats [B, L, fs]
 *                         lse/delta/sigma [B, H, L] ; rows i >= seqlens[b] are
 *                         padding and every per-row output there is written 0.
 *   packed (packed == 1): q,k,v,u,out,dout,wt [T, H, D*] ; feats [T, fs]
 *                         lse/delta/sigma [T, H] ; event b is rows
 *                         [cu_seqlens[b], cu_seqlens[b+1]).
 *   padded row-major (packed == 2): q,k,v,u,out,dout,wt [B, L, H, D*] ;
 *                         feats [B, L, fs] ; lse/delta/sigma [B, L, H] ; the
 *                         caller's [B, L, H*Dh] projections without a head
 *                         split (no upstream counterpart); padding as for 0.
 * D* is Dh for q,k,v,out,dout and C for u, wt.
 */
#ifndef FLASH_SPACETIME_H_
#define FLASH_SPACETIME_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FST_ABI_VERSION 5

/* Storage dtype of q, k, v, u, wt, out, dout, dq, dk, dv. */
enum FstDtype { FST_F32 = 0, FST_BF16 = 1, FST_F16 = 2 };

/* Return codes. */
enum FstStatus {
  FST_OK = 0,
  FST_ERR_INVALID = 1,     /* bad shape / pointer / flag combination        */
  FST_ERR_UNSUPPORTED = 2, /* valid request this build does not implement   */
  FST_ERR_CUDA = 3,        /* a CUDA runtime call failed                    */
  FST_ERR_WORKSPACE = 4,   /* workspace pointer NULL or too small           */
  FST_ERR_DEVICE = 5       /* the device reported a failed self-check       */
};

/*
 * Problem description shared by forward and backward.
 * Mirrors the arguments of upstream flash_spacetime_forward
 * (forward.py:222-237): q/k/v shapes, weight [Dh, C], bias [Dh], seqlens or
 * cu_seqlens, scale, use_attn_bias, use_activation_bias.
 */
typedef struct FstProblem {
  int32_t dtype;          /* enum FstDtype                                   */
  int32_t packed;         /* 0 padded [B,H,L,*], 1 packed [T,H,*], 2 [B,L,H,*] */
  int32_t batch;          /* B: number of events                             */
  int32_t heads;          /* H                                               */
  int32_t max_len;        /* padded: L. packed: an upper bound on any event  */
                          /* length, or 0 if unknown                         */
  int32_t head_dim;       /* Dh                                              */
  int32_t channels;       /* C: embedding channels, even                     */
  int32_t feat_stride;    /* floats between consecutive feats rows (>= 4)    */
  int64_t total_rows;     /* padded: B*L. packed: T                          */
  float scale;            /* query scale (Dh^-0.5 by default)                */
  int32_t use_attn_bias;  /* add u_i . E_ij to the logits                    */
  int32_t use_act_bias;   /* add (sum_j P_ij E_ij) W^T + b to the output     */
  const int32_t* seqlens;    /* [B] device, valid prefix lengths (padded)     */
  const int32_t* cu_seqlens; /* [B+1] device token offsets (packed)           */
  const float* feats;        /* device fp32: x, y, z in cols 0-2, time col 3  */
  const float* freqs;        /* [C/2] device fp32 frequency ladder            */
  const float* weight;       /* [Dh, C] device fp32 (nn.Linear layout)        */
  const float* bias;         /* [Dh] device fp32, or NULL                     */
  /* Optional [B] device permutation of the events: the order in which the
   * kernels' row / key blocks are scheduled (longest first balances the SMs);
   * NULL = natural order, or the library's own longest-first order with
   * FST_FLAG_LONGEST_FIRST. Results do not depend on it. No upstream
   * counterpart. */
  const int32_t* event_order;
  /* Elements between consecutive rows of q, k, v and of dq, dk, dv in the
   * row-interleaved layouts (packed == 1 or 2); 0 = H*Dh (dense rows). A fused
   * QKV projection [rows, 3, H, Dh] -- one [rows, 3*H*Dh] buffer -- is read
   * in place with q = base, k = base + H*Dh, v = base + 2*H*Dh and
   * qkv_row_stride = 3*H*Dh, and the gradients written into a buffer of the
   * same form (upstream builds q, k, v by three projections and a head split,
   * reference.py:187-223). Must be a multiple of Dh and of 8 elements, and
   * >= H*Dh; 0 for the padded [B,H,L,D] layout. out, dout, u, wt stay dense. */
  int32_t qkv_row_stride;
  /* FST_FLAG_* bits (performance hints; results do not depend on them). */
  int32_t flags;
  /* Padded layouts (packed 0 or 2): sum over events of min(seqlens[b],
   * max_len) -- the valid rows -- or any larger value, when the caller knows
   * it on the host (a data loader does); 0 = unknown. With it the 16-bit
   * kernels launch blocks for about that many rows, taken from a device tile
   * list as in the packed layout, instead of max_len rows per event, and the
   * live blocks write the zero padding rows between them. A value below the
   * true sum is detected on the device: every valid row of every output is
   * then NaN (padding rows stay 0). Ignored for packed == 1 and when >=
   * total_rows. No upstream counterpart (its grid is (L / BM, B),
   * forward.py:253-255). */
  int64_t valid_rows;
} FstProblem;

/* Another kernel runs beside this call on every SM -- typically the host to
 * device gather of a training loop's next batch (fst_upload_rows on a side
 * stream). The backward then uses kernel variants that leave registers free
 * for it (its column kernel would otherwise fill each SM and serialise the
 * two); about 7 % slower when nothing runs beside it. No upstream
 * counterpart. */
#define FST_FLAG_SHARE_SMS 1

/* The library puts the events in longest-first order itself (stable: equal
 * lengths keep their index order), as an event_order would; event_order must
 * then be NULL, and the batch at most 1024 events. One small kernel per call
 * ranks the lengths; no host synchronisation. No upstream counterpart. */
#define FST_FLAG_LONGEST_FIRST 2

typedef struct FstForwardArgs {
  FstProblem prob;
  const void* q;         /* unscaled queries                                 */
  const void* k;
  const void* v;
  const void* u;         /* (q*scale) @ W rounded to dtype, or NULL: then the */
                         /* kernels form it in fp32 themselves               */
  void* out;             /* output, same layout/dtype as q                   */
  float* lse;            /* log-sum-exp of the logits WITHOUT the qt.b term  */
  void* workspace;       /* device scratch, >= fst_forward_workspace_size()  */
  size_t workspace_bytes;
} FstForwardArgs;

typedef struct FstBackwardArgs {
  FstProblem prob;
  const void* q;
  const void* k;
  const void* v;
  const void* u;         /* as in the forward (NULL: formed in-kernel)       */
  const void* out;       /* forward output; gives the row offset dO.(out-b)  */
                         /* subtracted from dP before summing. May be NULL. */
  const void* dout;      /* upstream gradient, padding rows ignored          */
  const void* wt;        /* dout @ W rounded to dtype (NULL: formed in-kernel) */
  const float* lse;      /* from fst_forward                                 */
  void* dq;              /* outputs, layout/dtype of q                       */
  void* dk;
  void* dv;
  float* dw_partial;     /* [fst_dw_partial_count(), Dh, C] fp32; summed over */
                         /* axis 0 in a fixed order (fst_sum_partials) -> dW */
  float* db_partial;     /* [fst_dw_partial_count(), Dh] fp32: partial sums  */
                         /* of dout over valid rows (db when act and bias)   */
  float* delta;          /* [rows, H] fp32: D_i = sum P dP / sum P, dP taken */
                         /* without its dO.b row constant (it cancels)       */
  float* sigma;          /* [rows, H] fp32: rowsum(dS), zero by construction */
  float* ds_absmax;      /* [rows, H] fp32: rowmax |dS|, or NULL             */
  void* workspace;       /* device scratch, >= fst_backward_workspace_size() */
  size_t workspace_bytes;
} FstBackwardArgs;

/* ABI version of the loaded library (FST_ABI_VERSION). */
int fst_abi_version(void);

/* Bytes of device scratch fst_forward / fst_backward need for this problem. */
size_t fst_forward_workspace_size(const FstProblem* prob);
size_t fst_backward_workspace_size(const FstProblem* prob);

/* Rows of dw_partial fst_backward writes for this problem. */
int64_t fst_dw_partial_count(const FstProblem* prob);

/* dW and db from fst_backward's partials, on the device in a fixed order:
 * dw[i] = sum over r < fst_dw_partial_count(prob) of dw_partial[r][i]
 * (i < Dh*C), db likewise over [Dh]. Either output may be NULL. The order of
 * the additions depends only on the problem, so the sums are bitwise
 * reproducible. Stream-ordered after the fst_backward call; one launch.
 * Replaces the host-side sums of upstream's backward (backward.py:607-622). */
int fst_sum_partials(const FstProblem* prob, const float* dw_partial, const float* db_partial,
                     float* dw, float* db, void* stream);

/* Fused forward (upstream forward.py:222-346). */
int fst_forward(const FstForwardArgs* args, void* stream);

/* Fused backward (upstream backward.py:488-630). */
int fst_backward(const FstBackwardArgs* args, void* stream);

/* fst_forward for callers that cannot allocate device memory (no counterpart
 * in the upstream package). Inference servers and plugin hosts with a fixed,
 * pre-reserved memory pool, or real-time loops where a cudaMalloc (which may
 * synchronise the device) is not allowed, cannot provide fst_forward's
 * workspace. This variant ignores args->workspace and takes that scratch from
 * a 256 KiB array built into the library (one per GPU, held until the process
 * exits); it allocates nothing. A problem whose fst_forward_workspace_size
 * exceeds 256 KiB (16-bit inputs with more than 65535 events, or 32767 in a
 * padded layout given valid_rows) is rejected
 * with FST_ERR_INVALID. The first call on a device looks up the array's
 * address and keeps it for the life of the process (make that call before any
 * stream capture; after a cudaDeviceReset of that device the entry point must
 * not be used). All calls share the array: calls that overlap on the GPU
 * race, so order them on one stream. */
int fst_forward_noalloc(const FstForwardArgs* args, void* stream);

/* Host -> device copy of the valid rows of a padded batch (a data-loader
 * helper; upstream leaves the transfer to the caller's tensor.to(device)).
 * src (host, pinned for an asynchronous copy) and dst (device) are both
 * [batch][groups][max_len][row_bytes]; for event b only rows < lens[b] of each
 * group are copied, one 2D copy per event on `stream`. The padding rows of dst
 * are left as they are: fst_forward / fst_backward never read the padding
 * rows of q, k, v, feats or dout. lens is a HOST array of batch lengths, each
 * in [0, max_len] (checked before any copy is issued). For [B, H, L, D]
 * tensors groups = H and row_bytes = D * element size; for feats [B, L, fs]
 * groups = 1 and row_bytes = fs * 4. */
int fst_upload_rows(void* dst, const void* src, const int32_t* lens, int64_t batch,
                    int64_t groups, int64_t max_len, int64_t row_bytes, void* stream);

/* Number of CUDA kernels this library has launched in the process so far
 * (benchmark bookkeeping; no counterpart upstream). */
int64_t fst_kernel_launches(void);

/* Copies the calling thread's last error message into buf (NUL-terminated).
 * Returns the message length. */
int fst_last_error(char* buf, size_t len);

#ifdef __cplusplus
}
#endif

#endif /* FLASH_SPACETIME_H_ */
