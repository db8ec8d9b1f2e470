"""Public ops and the autograd boundary of fused spacetime-bias attention.

``flash_spacetime_attention`` (padded ``[B, H, L, Dh]``) and
``flash_spacetime_attention_varlen`` (packed ``[T, H, Dh]`` with
``cu_seqlens``) keep the upstream signatures (upstream
src/flash_spacetime/forward.py:481-527). Behind them a single
``torch.autograd.Function`` does what upstream's host drivers do on the
host -- the float32 projection ``u = (q * scale) @ W`` of the queries through
the encoder weight (forward.py:279-286), and ``w~ = dO @ W`` in the backward
(backward.py:546-556) -- and calls the CUDA library through its C ABI
(``_lib``). The output-side epilogues upstream also runs on the host
(``A' W^T + b``, forward.py:333-345; ``dq``, backward.py:600-605) are fused
into the kernels. There is no other code path: no Triton, no CPU fallback.

Conventions kept from upstream:

* the output has q's dtype and padding rows are exactly 0 (forward.py:19-22);
* ``feats`` must not require grad (ValueError, forward.py:372-373);
* ``dW``/``db`` are None when both bias terms are off, ``db`` is zeros when
  only the logit term is on (forward.py:417-432, backward.py:615-622);
* results are bitwise deterministic run to run.
"""

import ctypes
import math
from typing import Any, Dict, Optional, Sequence, Tuple

import torch
from torch import Tensor

from . import _lib
from .reference import sinusoidal_frequencies

_DTYPES = {
    torch.float32: _lib.FST_F32,
    torch.bfloat16: _lib.FST_BF16,
    torch.float16: _lib.FST_F16,
}

_freq_cache: Dict[Tuple[int, str], Tensor] = {}
_kernel_timer: Optional[list] = None


def set_kernel_timer(sink: Optional[list]) -> None:
    """Record CUDA events around every library call into ``sink``.

    Each entry is ``(entry point name, start event, end event)``, recorded on
    the stream the kernels are launched on. Pass None to stop recording.
    """
    global _kernel_timer
    _kernel_timer = sink


def _timed_call(name: str, fn, args, device: torch.device) -> int:
    if _kernel_timer is None:
        return fn(*args)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    rc = fn(*args)
    e1.record()
    _kernel_timer.append((name, e0, e1))
    return rc


def _freqs(channels: int, device: torch.device) -> Tensor:
    """float32 frequency ladder, evaluated on the CPU once per (C, device).

    Computing it on the CPU keeps the ladder bitwise identical to the CPU
    oracle whatever device the op runs on.
    """
    key = (channels, str(device))
    t = _freq_cache.get(key)
    if t is None:
        t = sinusoidal_frequencies(channels, torch.device("cpu")).to(device)
        _freq_cache[key] = t
    return t


def _ptr(t: Optional[Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _dense(t: Tensor) -> Tensor:
    """``t`` contiguous and starting on a 16-byte boundary (the kernels move
    rows with 16-byte vector loads); a misaligned view is copied."""
    t = t.contiguous()
    return t if t.data_ptr() % 16 == 0 else t.clone()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def seqlens_from_mask(mask: Tensor, validate: bool = True) -> Tensor:
    """Valid prefix lengths ``[B]`` from a ``[B, L]`` key-padding mask.

    Accepts a bool mask (True = padding, the PyTorch ``key_padding_mask``
    convention) or a float mask (0 valid / -inf padding, the ``Attention_rel``
    convention of upstream reference.py:91-97). The fused op assumes
    front-packed padding (upstream forward.py:241-242); with ``validate`` a
    mask whose valid tokens are not a prefix raises ValueError (this check
    reads one flag back from the device).
    """
    return _mask_lengths(mask, validate)[0]


def _mask_lengths(mask: Tensor, validate: bool) -> Tuple[Tensor, int]:
    """(seqlens_from_mask, the valid row count when the check read it back
    with its flag -- one device-to-host read for both -- else 0)."""
    if mask.dim() != 2:
        raise ValueError(f"key_padding_mask must be [B, L], got {tuple(mask.shape)}")
    pad = mask if mask.dtype == torch.bool else torch.isneginf(mask)
    valid = ~pad
    lengths = valid.sum(1, dtype=torch.int32)
    if not validate:
        return lengths, 0
    pos = torch.arange(mask.shape[1], device=mask.device)
    prefix = (valid == (pos[None, :] < lengths[:, None])).all()
    ok, total = torch.stack([prefix.to(torch.int64), lengths.sum(dtype=torch.int64)]).tolist()
    if not ok:
        raise ValueError(
            "key_padding_mask must mark a prefix of each event as valid "
            "(front-packed padding); reorder the tokens of each event"
        )
    return lengths, int(total)


def _padded_lengths(seqlens: Any, mask: Optional[Tensor], batch: int, length: int,
                    device: torch.device, validate: bool,
                    valid_rows: Optional[int]) -> Tuple[Tensor, int]:
    """Lengths of a padded batch from ``seqlens`` (``[B]``, on any device, or a
    ``[B, L]`` mask) or ``key_padding_mask``, and the valid row count as far
    as the host knows it (0 = unknown)."""
    hint = 0
    if mask is not None:
        if seqlens is not None:
            raise ValueError("pass seqlens or key_padding_mask, not both")
        seqlens, hint = _mask_lengths(mask, validate)
    elif seqlens is None:
        seqlens = torch.full((batch,), length, dtype=torch.int32, device=device)
    elif isinstance(seqlens, Tensor) and seqlens.dim() == 2:
        seqlens, hint = _mask_lengths(seqlens, validate)
    if valid_rows is not None:
        if int(valid_rows) < 0:
            raise ValueError(f"valid_rows must be >= 0, got {valid_rows}")
        hint = int(valid_rows)
    return seqlens, hint


def _event_order(lengths: Tensor) -> Optional[Tensor]:
    """Longest-first event order (stable), or None when the library ranks the
    events itself (FST_FLAG_LONGEST_FIRST, up to 1024 events: one ranking
    step inside a kernel the call launches anyway, instead of a torch sort's
    four launches)."""
    if lengths.numel() <= _lib.MAX_SELF_ORDERED:
        return None
    return torch.argsort(lengths, descending=True, stable=True).to(torch.int32)


class _Problem:
    """Shapes and host-side tensors of one call, in C-ABI form."""

    def __init__(
        self,
        q: Tensor,
        feats: Tensor,
        weight: Tensor,
        bias: Optional[Tensor],
        seqlens: Optional[Tensor],
        cu_seqlens: Optional[Tensor],
        scale: Optional[float],
        use_attn_bias: bool,
        use_act_bias: bool,
        layout: str = "bhld",
        host_projection: bool = False,
        qkv_row_stride: int = 0,
        share_sms: bool = False,
        valid_rows: int = 0,
    ) -> None:
        self.packed = cu_seqlens is not None
        self.valid_rows = 0
        self.share_sms = bool(share_sms)
        self.host_projection = bool(host_projection)
        self.qkv_row_stride = int(qkv_row_stride)
        if layout not in ("bhld", "blhd"):
            raise ValueError(f"layout must be 'bhld' or 'blhd', got {layout!r}")
        self.layout = "packed" if self.packed else layout
        if q.dtype not in _DTYPES:
            raise ValueError(f"unsupported dtype {q.dtype}")
        if not q.is_cuda:
            raise ValueError("flash_spacetime runs on CUDA tensors only")
        if self.packed:
            if q.dim() != 3:
                raise ValueError(f"varlen q must be [T, H, D], got {tuple(q.shape)}")
            total, heads, dim = q.shape
            self.cu = cu_seqlens.to(device=q.device, dtype=torch.int32).contiguous()
            batch = self.cu.numel() - 1
            length = 0
            self.seq = None
            # Longest events first (see the padded case below).
            self.order = _event_order(self.cu[1:] - self.cu[:-1])
            rows = total
            if feats.dim() != 2 or feats.shape[0] != total:
                raise ValueError(f"varlen feats must be [T, F], got {tuple(feats.shape)}")
        else:
            if q.dim() != 4:
                raise ValueError(f"q must be [B, H, L, D] (or [B, L, H, D] with layout='blhd'), "
                                 f"got {tuple(q.shape)}")
            if self.layout == "blhd":
                batch, length, heads, dim = q.shape
            else:
                batch, heads, length, dim = q.shape
            self.cu = None
            # Lengths held on the host (a list or a CPU tensor, as a data
            # loader has them) also give the valid row count, with which the
            # kernels launch blocks for the valid rows only.
            host = None
            if not (isinstance(seqlens, Tensor) and seqlens.is_cuda):
                host = torch.as_tensor(seqlens, dtype=torch.int64, device="cpu")
            self.seq = torch.as_tensor(seqlens).to(device=q.device, dtype=torch.int32).contiguous()
            if self.seq.shape != (batch,):
                raise ValueError(f"seqlens must be [B] = [{batch}], got {tuple(self.seq.shape)}")
            if host is not None:
                known = int(host.clamp(0, length).sum())
                if valid_rows and valid_rows < known:
                    raise ValueError(f"valid_rows (={valid_rows}) is below the sum of the "
                                     f"lengths (={known})")
                valid_rows = valid_rows or known
            self.valid_rows = int(valid_rows)
            rows = batch * length
            # Longest events first: their row / key blocks are scheduled
            # before the short ones', which balances the SMs (the results
            # do not depend on the order; the sort is stable).
            self.order = _event_order(self.seq)
            if feats.dim() != 3 or feats.shape[:2] != (batch, length):
                raise ValueError(f"feats must be [B, L, F], got {tuple(feats.shape)}")
        if feats.shape[-1] < 4:
            raise ValueError("feats needs at least 4 columns (x, y, z, t)")
        if weight.dim() != 2 or weight.shape[0] != dim:
            raise ValueError(
                f"weight must be [head_dim, C] = [{dim}, C] (nn.Linear layout), "
                f"got {tuple(weight.shape)}"
            )
        channels = weight.shape[1]
        if channels % 2:
            raise ValueError(f"C (={channels}) must be even")
        if bias is not None and bias.shape != (dim,):
            raise ValueError(f"bias must be [{dim}], got {tuple(bias.shape)}")
        self.batch, self.heads, self.length, self.dim = batch, heads, length, dim
        self.channels, self.rows = channels, rows
        self.scale = float(dim**-0.5 if scale is None else scale)
        self.attn, self.act = bool(use_attn_bias), bool(use_act_bias)
        self.dtype = q.dtype
        self.device = q.device
        # The kernels read x, y, z, t from each feats row at a fixed float
        # stride; a contiguous fp32 tensor whose row length is a multiple of 4
        # (16-byte rows) is used in place, anything else is repacked to [.., 4].
        if (feats.dtype == torch.float32 and feats.is_contiguous() and feats.shape[-1] % 4 == 0
                and feats.data_ptr() % 16 == 0):
            self.feats = feats.detach()
            self.feat_stride = feats.shape[-1]
        else:
            self.feats = feats.detach()[..., :4].to(torch.float32).contiguous()
            self.feat_stride = 4
        self.freqs = _freqs(channels, q.device)
        self.w32 = weight.detach().to(torch.float32).contiguous()
        self.b32 = None if bias is None else bias.detach().to(torch.float32).contiguous()

    def c_struct(self) -> _lib.FstProblem:
        p = _lib.FstProblem()
        p.dtype = _DTYPES[self.dtype]
        p.packed = {"bhld": 0, "packed": 1, "blhd": 2}[self.layout]
        p.batch = self.batch
        p.heads = self.heads
        p.max_len = self.length
        p.head_dim = self.dim
        p.channels = self.channels
        p.feat_stride = self.feat_stride
        p.total_rows = self.rows
        p.scale = self.scale
        p.use_attn_bias = int(self.attn)
        p.use_act_bias = int(self.act)
        p.seqlens = _ptr(self.seq)
        p.cu_seqlens = _ptr(self.cu)
        p.feats = _ptr(self.feats)
        p.freqs = _ptr(self.freqs)
        p.weight = _ptr(self.w32)
        p.bias = _ptr(self.b32)
        p.event_order = _ptr(self.order)
        p.qkv_row_stride = self.qkv_row_stride
        p.flags = (_lib.FST_FLAG_SHARE_SMS if self.share_sms else 0) | \
            (_lib.FST_FLAG_LONGEST_FIRST if self.order is None else 0)
        p.valid_rows = self.valid_rows
        return p

    def stat_shape(self) -> Tuple[int, ...]:
        if self.packed:
            return (self.rows, self.heads)
        if self.layout == "blhd":
            return (self.batch, self.length, self.heads)
        return (self.batch, self.heads, self.length)


def _workspace(nbytes: int, device: torch.device) -> Tuple[Optional[Tensor], int]:
    if nbytes == 0:
        return None, 0
    return torch.empty(nbytes, dtype=torch.uint8, device=device), nbytes


def _host_u(pb: "_Problem", q: Tensor) -> Optional[Tensor]:
    """``u = ((q.float() * scale) @ W).to(dtype)`` when the host projects
    (upstream forward.py:279-286), else None (the kernels project)."""
    if not (pb.host_projection and pb.attn):
        return None
    return _dense((q.to(torch.float32) * pb.scale) @ pb.w32).to(pb.dtype).contiguous()


def _host_wt(pb: "_Problem", dout: Tensor) -> Optional[Tensor]:
    """``w~ = (dO.float() @ W).to(dtype)`` when the host projects (upstream
    backward.py:546-547), else None."""
    if not (pb.host_projection and pb.act):
        return None
    return (dout.to(torch.float32) @ pb.w32).to(pb.dtype).contiguous()


def fused_forward(pb: _Problem, q: Tensor, k: Tensor, v: Tensor) -> Tuple[Tensor, Tensor]:
    """One ``fst_forward`` call. Returns ``(out, lse)``."""
    lib = _lib.load()
    # u = (q * scale) @ W (upstream forward.py:279-286) is formed in fp32 by the
    # kernels themselves (u = NULL), which saves the host GEMM and its HBM
    # round trips. With host_projection the host forms it as upstream does
    # and passes it through the C ABI.
    u = _host_u(pb, q)
    out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    lse = torch.empty(pb.stat_shape(), dtype=torch.float32, device=pb.device)
    a = _lib.FstForwardArgs()
    a.prob = pb.c_struct()
    ws, nws = _workspace(lib.fst_forward_workspace_size(ctypes.byref(a.prob)), pb.device)
    a.q, a.k, a.v, a.u = _ptr(q), _ptr(k), _ptr(v), _ptr(u)
    a.out, a.lse = _ptr(out), _ptr(lse)
    a.workspace, a.workspace_bytes = _ptr(ws), nws
    rc = _timed_call("fst_forward", lib.fst_forward, (ctypes.byref(a), _stream(pb.device)),
                     pb.device)
    _lib.check(rc, "fst_forward")
    return out, lse


def fused_backward(
    pb: _Problem,
    q: Tensor,
    k: Tensor,
    v: Tensor,
    out: Tensor,
    lse: Tensor,
    dout: Tensor,
    want_absmax: bool = False,
    dqkv: Optional[Tensor] = None,
) -> Dict[str, Optional[Tensor]]:
    """One ``fst_backward`` call plus the fixed-order sums of its dW / db partials.

    Returns dq, dk, dv (input dtype), dW ``[Dh, C]`` and db ``[Dh]`` (fp32,
    or None when the projection is unused), and the per-row diagnostics
    delta (D), sigma (rowsum dS) and, on request, rowmax |dS|. With a fused
    QKV problem the gradients are written into ``dqkv`` (``[rows, 3, H,
    Dh]``) and dq, dk, dv are its views.
    """
    lib = _lib.load()
    dout, out, lse = _dense(dout), _dense(out), lse.contiguous()
    # u and w~ = dO @ W (upstream backward.py:541-556) are formed in-kernel,
    # or on the host with host_projection.
    u, wt = _host_u(pb, q), _host_wt(pb, dout)
    if dqkv is not None:
        dq, dk, dv = dqkv.select(-3, 0), dqkv.select(-3, 1), dqkv.select(-3, 2)
    else:
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    a = _lib.FstBackwardArgs()
    a.prob = pb.c_struct()
    nparts = int(lib.fst_dw_partial_count(ctypes.byref(a.prob)))
    dw_part = torch.empty(max(nparts, 1), pb.dim, pb.channels, dtype=torch.float32,
                          device=pb.device)
    db_part = torch.empty(max(nparts, 1), pb.dim, dtype=torch.float32, device=pb.device)
    delta = torch.empty(pb.stat_shape(), dtype=torch.float32, device=pb.device)
    sigma = torch.empty_like(delta)
    absmax = torch.empty_like(delta) if want_absmax else None
    ws, nws = _workspace(lib.fst_backward_workspace_size(ctypes.byref(a.prob)), pb.device)
    a.q, a.k, a.v, a.u, a.out = _ptr(q), _ptr(k), _ptr(v), _ptr(u), _ptr(out)
    a.dout, a.wt, a.lse = _ptr(dout), _ptr(wt), _ptr(lse)
    a.dq, a.dk, a.dv = _ptr(dq), _ptr(dk), _ptr(dv)
    a.dw_partial, a.db_partial = _ptr(dw_part), _ptr(db_part)
    a.delta, a.sigma = _ptr(delta), _ptr(sigma)
    a.ds_absmax = _ptr(absmax)
    a.workspace, a.workspace_bytes = _ptr(ws), nws
    rc = _timed_call("fst_backward", lib.fst_backward, (ctypes.byref(a), _stream(pb.device)),
                     pb.device)
    _lib.check(rc, "fst_backward")

    # dW and db: the partials summed on the device in a fixed order (one
    # launch; upstream sums on the host side of backward.py:607-622).
    dw = db = None
    if pb.attn or pb.act:
        dw = torch.empty(pb.dim, pb.channels, dtype=torch.float32, device=pb.device)
    if pb.b32 is not None and pb.act:
        db = torch.empty(pb.dim, dtype=torch.float32, device=pb.device)  # sum of dO, valid rows
    if dw is not None or db is not None:
        rc = _timed_call("fst_sum_partials", lib.fst_sum_partials,
                         (ctypes.byref(a.prob), _ptr(dw_part), _ptr(db_part), _ptr(dw), _ptr(db),
                          _stream(pb.device)), pb.device)
        _lib.check(rc, "fst_sum_partials")
    if pb.b32 is not None and not pb.act:
        # The logit path's db vanishes analytically (backward.py:619-622).
        db = torch.zeros(pb.dim, dtype=torch.float32, device=pb.device)
    return {"dq": dq, "dk": dk, "dv": dv, "dW": dw, "db": db,
            "delta": delta, "sigma": sigma, "ds_absmax": absmax}


class _FlashSpacetimeAttention(torch.autograd.Function):
    """Fused forward and deterministic fused backward (upstream forward.py:349-478)."""

    @staticmethod
    def forward(  # type: ignore[override]
        ctx: Any,
        q: Tensor,
        k: Tensor,
        v: Tensor,
        feats: Tensor,
        weight: Tensor,
        bias: Optional[Tensor],
        seqlens: Optional[Tensor],
        cu_seqlens: Optional[Tensor],
        scale: Optional[float],
        use_attn_bias: bool,
        use_activation_bias: bool,
        layout: str = "bhld",
        host_projection: bool = False,
        share_sms: bool = False,
        valid_rows: int = 0,
    ) -> Tensor:
        if feats.requires_grad:
            raise ValueError("feats (detector data) must not require grad")
        if k.shape != q.shape or v.shape != q.shape:
            raise ValueError("q, k and v must have the same shape")
        if k.dtype != q.dtype or v.dtype != q.dtype:
            raise ValueError("q, k and v must have the same dtype")
        pb = _Problem(q, feats, weight, bias, seqlens, cu_seqlens, scale,
                      use_attn_bias, use_activation_bias, layout, host_projection,
                      share_sms=share_sms, valid_rows=valid_rows)
        qc, kc, vc = (_dense(t) for t in (q, k, v))
        out, lse = fused_forward(pb, qc, kc, vc)
        ctx.save_for_backward(qc, kc, vc, out, lse)
        ctx.pb = pb
        ctx.weight_dtype = weight.dtype
        ctx.bias_dtype = None if bias is None else bias.dtype
        return out

    @staticmethod
    def backward(ctx: Any, grad_out: Tensor) -> Tuple[Optional[Tensor], ...]:  # type: ignore[override]
        q, k, v, out, lse = ctx.saved_tensors
        pb: _Problem = ctx.pb
        g = fused_backward(pb, q, k, v, out, lse, grad_out)
        proj_used = pb.attn or pb.act
        need = ctx.needs_input_grad
        dw = g["dW"].to(ctx.weight_dtype) if (proj_used and need[4]) else None
        db = None
        if ctx.bias_dtype is not None and proj_used and need[5]:
            db = g["db"].to(ctx.bias_dtype)
        return (
            g["dq"] if need[0] else None,
            g["dk"] if need[1] else None,
            g["dv"] if need[2] else None,
            None, dw, db, None, None, None, None, None, None, None, None, None,
        )


def flash_spacetime_attention(
    q: Tensor,
    k: Tensor,
    v: Tensor,
    feats: Tensor,
    weight: Tensor,
    bias: Optional[Tensor],
    seqlens: Optional[Tensor] = None,
    scale: Optional[float] = None,
    use_attn_bias: bool = True,
    use_activation_bias: bool = True,
    *,
    key_padding_mask: Optional[Tensor] = None,
    layout: str = "bhld",
    validate_mask: bool = True,
    host_projection: bool = False,
    share_sms: bool = False,
    valid_rows: Optional[int] = None,
) -> Tensor:
    """Fused spacetime-bias attention on a padded batch (upstream forward.py:481-501).

    q, k, v: ``[B, H, L, Dh]`` (fp32, bf16 or fp16). feats: ``[B, L, F]`` with
    x, y, z in columns 0-2 and time in column 3. weight: ``[Dh, C]``; bias:
    ``[Dh]`` or None. The 7th argument takes the ``[B]`` valid lengths
    (upstream's form); a ``[B, L]`` key-padding mask, bool (True = padding)
    or float (0 / -inf), is accepted there or as ``key_padding_mask=``.
    Returns ``[B, H, L, Dh]`` in q's dtype with padding rows exactly 0.

    ``layout='blhd'`` (an addition) takes and returns ``[B, L, H, Dh]``: a
    ``[B, L, H*Dh]`` projection viewed per head, with no head split or merge
    around the op.

    ``validate_mask=False`` skips the check that a mask marks a prefix of
    each event (the check reads a flag back from the device, a host
    synchronisation per call); an unchecked mask that is not a prefix gives
    wrong results. ``host_projection=True`` forms ``u = (q * scale) W`` and
    ``w~ = dO W`` on the host in fp32, rounded once to q's dtype, as upstream
    does (forward.py:279-286, backward.py:546-547), and passes them to the
    kernels; by default the kernels form them in their prologue.
    ``share_sms=True`` is a performance hint for callers that run another
    kernel beside the op on every SM (a data loader's host-to-device copy of
    the next batch on a side stream, ``upload_valid_rows``): the backward
    then leaves room on each SM for it. Results do not depend on it.

    ``valid_rows`` is the number of valid rows, the sum of the lengths (or
    any larger number), when the caller knows it on the host -- a data loader
    does. The kernels then launch blocks for the valid rows only, not for
    ``B * L``; most of a padded batch of short events is padding. Lengths
    passed on the host (a list or a CPU tensor as the 7th argument) and a
    validated mask give it without the argument. Results do not depend on
    it, except that a number below the true sum turns every valid output
    row (and gradient row) into NaN.
    """
    length = q.shape[1] if layout == "blhd" else q.shape[2]
    seqlens, hint = _padded_lengths(seqlens, key_padding_mask, q.shape[0], length, q.device,
                                    validate_mask, valid_rows)
    return _FlashSpacetimeAttention.apply(
        q, k, v, feats, weight, bias, seqlens, None,
        scale, use_attn_bias, use_activation_bias, layout, host_projection, share_sms, hint,
    )


def flash_spacetime_attention_varlen(
    q: Tensor,
    k: Tensor,
    v: Tensor,
    feats: Tensor,
    weight: Tensor,
    bias: Optional[Tensor],
    cu_seqlens: Tensor,
    scale: Optional[float] = None,
    use_attn_bias: bool = True,
    use_activation_bias: bool = True,
    *,
    host_projection: bool = False,
    share_sms: bool = False,
) -> Tensor:
    """Packed, uncapped variant (upstream forward.py:504-527).

    q, k, v: ``[T, H, Dh]``; feats ``[T, F]``; ``cu_seqlens`` ``[B+1]`` token
    offsets (cu[0] = 0, cu[-1] = T) -- the values buffer of a jagged
    NestedTensor. No padding exists and no host synchronisation happens.
    ``host_projection`` and ``share_sms`` as for :func:`flash_spacetime_attention`.
    """
    return _FlashSpacetimeAttention.apply(
        q, k, v, feats, weight, bias, None, cu_seqlens,
        scale, use_attn_bias, use_activation_bias, "bhld", host_projection, share_sms,
    )


class _FlashSpacetimeQKV(torch.autograd.Function):
    """The fused op on one QKV buffer ``[rows, 3, H, Dh]``, read in place
    through the C ABI's ``qkv_row_stride``; the backward writes the gradient
    of the same buffer in one piece."""

    @staticmethod
    def forward(  # type: ignore[override]
        ctx: Any,
        qkv: Tensor,
        feats: Tensor,
        weight: Tensor,
        bias: Optional[Tensor],
        seqlens: Optional[Tensor],
        cu_seqlens: Optional[Tensor],
        scale: Optional[float],
        use_attn_bias: bool,
        use_activation_bias: bool,
        host_projection: bool,
        valid_rows: int = 0,
    ) -> Tensor:
        if feats.requires_grad:
            raise ValueError("feats (detector data) must not require grad")
        qkv = _dense(qkv)
        q, k, v = qkv.select(-3, 0), qkv.select(-3, 1), qkv.select(-3, 2)
        heads, dim = q.shape[-2], q.shape[-1]
        pb = _Problem(q, feats, weight, bias, seqlens, cu_seqlens, scale, use_attn_bias,
                      use_activation_bias, "blhd", host_projection, 3 * heads * dim,
                      valid_rows=valid_rows)
        out, lse = fused_forward(pb, q, k, v)
        ctx.save_for_backward(qkv, out, lse)
        ctx.pb = pb
        ctx.weight_dtype = weight.dtype
        ctx.bias_dtype = None if bias is None else bias.dtype
        return out

    @staticmethod
    def backward(ctx: Any, grad_out: Tensor) -> Tuple[Optional[Tensor], ...]:  # type: ignore[override]
        qkv, out, lse = ctx.saved_tensors
        pb: _Problem = ctx.pb
        q, k, v = qkv.select(-3, 0), qkv.select(-3, 1), qkv.select(-3, 2)
        dqkv = torch.empty_like(qkv)
        g = fused_backward(pb, q, k, v, out, lse, grad_out, dqkv=dqkv)
        proj_used = pb.attn or pb.act
        need = ctx.needs_input_grad
        dw = g["dW"].to(ctx.weight_dtype) if (proj_used and need[2]) else None
        db = None
        if ctx.bias_dtype is not None and proj_used and need[3]:
            db = g["db"].to(ctx.bias_dtype)
        return (dqkv if need[0] else None, None, dw, db, None, None, None, None, None, None,
                None)


def flash_spacetime_attention_qkv(
    qkv: Tensor,
    feats: Tensor,
    weight: Tensor,
    bias: Optional[Tensor],
    seqlens: Optional[Tensor] = None,
    scale: Optional[float] = None,
    use_attn_bias: bool = True,
    use_activation_bias: bool = True,
    *,
    cu_seqlens: Optional[Tensor] = None,
    key_padding_mask: Optional[Tensor] = None,
    validate_mask: bool = True,
    host_projection: bool = False,
    valid_rows: Optional[int] = None,
) -> Tensor:
    """The op on a fused QKV projection, read in place (no head split).

    ``qkv``: ``[B, L, 3, H, Dh]`` (padded, with ``seqlens`` or a mask as for
    :func:`flash_spacetime_attention`) or ``[T, 3, H, Dh]`` (packed, with
    ``cu_seqlens``) -- the output of one ``nn.Linear(model_dim, 3 * H * Dh)``
    viewed per head. Upstream builds q, k and v with three projections and a
    head split (reference.py:187-223, ``split_heads``); here the kernels read
    each row's q, k and v where the projection wrote them, and the gradient
    comes back as one ``[.., 3, H, Dh]`` tensor. Returns ``[B, L, H, Dh]``
    (or ``[T, H, Dh]``) in qkv's dtype with padding rows exactly 0.
    ``valid_rows`` (padded only) as for :func:`flash_spacetime_attention`.
    """
    if qkv.dim() not in (4, 5) or qkv.shape[-3] != 3:
        raise ValueError(f"qkv must be [B, L, 3, H, Dh] or [T, 3, H, Dh], got {tuple(qkv.shape)}")
    packed = cu_seqlens is not None
    if packed != (qkv.dim() == 4):
        raise ValueError("a [T, 3, H, Dh] qkv needs cu_seqlens; a [B, L, 3, H, Dh] one does not")
    hint = 0
    if not packed:
        seqlens, hint = _padded_lengths(seqlens, key_padding_mask, qkv.shape[0], qkv.shape[1],
                                        qkv.device, validate_mask, valid_rows)
    return _FlashSpacetimeQKV.apply(qkv, feats, weight, bias, seqlens, cu_seqlens, scale,
                                    use_attn_bias, use_activation_bias, host_projection, hint)


def flash_spacetime_attention_nested(
    q: Tensor,
    k: Tensor,
    v: Tensor,
    feats: Tensor,
    weight: Tensor,
    bias: Optional[Tensor],
    scale: Optional[float] = None,
    use_attn_bias: bool = True,
    use_activation_bias: bool = True,
) -> Tensor:
    """The packed op on jagged NestedTensors (``layout=torch.jagged``).

    q, k, v: ``[B, j, H, Dh]`` and feats ``[B, j, F]`` jagged along the event
    axis with the same offsets -- the form whose values buffer and offsets
    upstream's varlen entry point documents (forward.py:518-520). Returns a
    jagged ``[B, j, H, Dh]`` with those offsets; gradients flow to the values
    of q, k, v and to weight / bias as for the varlen op.
    """
    for name, t in (("q", q), ("k", k), ("v", v), ("feats", feats)):
        if not (t.is_nested and t.layout == torch.jagged):
            raise ValueError(f"{name} must be a jagged NestedTensor (layout=torch.jagged)")
    offsets = q.offsets()
    for name, t in (("k", k), ("v", v), ("feats", feats)):
        if t.offsets() is not offsets and not torch.equal(t.offsets(), offsets):
            raise ValueError(f"{name} must share q's offsets")
    out = flash_spacetime_attention_varlen(
        q.values(), k.values(), v.values(), feats.values(), weight, bias,
        offsets.to(torch.int32), scale, use_attn_bias, use_activation_bias)
    return torch.nested.nested_tensor_from_jagged(out, offsets)


def flash_spacetime_forward(
    q: Tensor,
    k: Tensor,
    v: Tensor,
    feats: Tensor,
    weight: Tensor,
    bias: Optional[Tensor],
    seqlens: Optional[Tensor],
    scale: Optional[float] = None,
    use_attn_bias: bool = True,
    use_activation_bias: bool = True,
    cu_seqlens: Optional[Tensor] = None,
    layout: str = "bhld",
    host_projection: bool = False,
) -> Tuple[Tensor, Tensor]:
    """Forward only, returning ``(out, lse)`` (upstream forward.py:222-346)."""
    pb = _Problem(q, feats, weight, bias, seqlens, cu_seqlens, scale,
                  use_attn_bias, use_activation_bias, layout, host_projection)
    return fused_forward(pb, _dense(q), _dense(k), _dense(v))


def flash_spacetime_backward(
    q: Tensor,
    k: Tensor,
    v: Tensor,
    feats: Tensor,
    weight: Tensor,
    bias: Optional[Tensor],
    seqlens: Optional[Tensor],
    out: Tensor,
    lse: Tensor,
    grad_out: Tensor,
    scale: Optional[float] = None,
    use_attn_bias: bool = True,
    use_activation_bias: bool = True,
    cu_seqlens: Optional[Tensor] = None,
    want_absmax: bool = False,
    layout: str = "bhld",
    host_projection: bool = False,
) -> Dict[str, Optional[Tensor]]:
    """Backward only (upstream backward.py:488-630), with diagnostics.

    Returns dq, dk, dv, dW, db plus ``delta`` (D), ``sigma`` (rowsum dS, zero
    by construction) and, with ``want_absmax``, ``ds_absmax`` (rowmax |dS|).
    """
    pb = _Problem(q, feats, weight, bias, seqlens, cu_seqlens, scale,
                  use_attn_bias, use_activation_bias, layout, host_projection)
    return fused_backward(pb, _dense(q), _dense(k), _dense(v),
                          out, lse, grad_out, want_absmax)


def upload_valid_rows(dst: Tensor, src: Tensor, seqlens: Sequence[int], layout: str = "bhld") -> Tensor:
    """Copy the valid rows of a padded host batch ``src`` into the device tensor ``dst``.

    A data-loader helper (upstream leaves the transfer to ``tensor.to(device)``):
    with short events in a long padded batch most rows are padding, and the
    fused kernels never read a padding row of q, k, v, feats or grad_out, so
    only rows ``i < seqlens[b]`` of each event cross the host link. The
    padding rows of ``dst`` keep whatever they held. A pinned ``src`` is read
    by a gather kernel straight from host memory (asynchronous); a pageable
    one by one 2D copy per event. ``src`` is a contiguous
    CPU tensor, ``dst`` a contiguous CUDA
    tensor of the same shape and dtype; ``seqlens`` are host integers. Shapes:
    ``[B, H, L, D]`` with ``layout="bhld"``, or ``[B, L, ...]`` (feats, or the
    ``"blhd"`` layout). The copy is ordered on the current stream. Returns
    ``dst``.
    """
    if src.device.type != "cpu" or dst.device.type != "cuda":
        raise ValueError("upload_valid_rows: src must be a CPU tensor and dst a CUDA tensor")
    if src.shape != dst.shape or src.dtype != dst.dtype:
        raise ValueError(f"upload_valid_rows: src {tuple(src.shape)} {src.dtype} does not "
                         f"match dst {tuple(dst.shape)} {dst.dtype}")
    if not (src.is_contiguous() and dst.is_contiguous()):
        raise ValueError("upload_valid_rows: src and dst must be contiguous")
    if layout not in ("bhld", "blhd"):
        raise ValueError(f"upload_valid_rows: layout {layout!r} is not 'bhld' or 'blhd'")
    lens = torch.as_tensor(seqlens, dtype=torch.int32, device="cpu").contiguous()
    if lens.dim() != 1 or src.dim() < 3 or lens.numel() != src.shape[0]:
        raise ValueError("upload_valid_rows: expected [B, ...] tensors and B host lengths")
    es = src.element_size()
    if layout == "bhld" and src.dim() == 4:
        groups, max_len, row = src.shape[1], src.shape[2], src.shape[3] * es
    else:
        groups, max_len = 1, src.shape[1]
        row = es * math.prod(src.shape[2:])
    lib = _lib.load()
    with torch.cuda.device(dst.device):
        rc = lib.fst_upload_rows(_ptr(dst), _ptr(src), lens.data_ptr(), lens.numel(), groups,
                                 max_len, row, _stream(dst.device))
    _lib.check(rc, "fst_upload_rows")
    return dst
