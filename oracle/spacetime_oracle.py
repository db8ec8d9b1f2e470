"""CPU oracle for fused spacetime-bias attention -- TEST INFRASTRUCTURE ONLY.

Nothing on the product path imports this file. Only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline / reference arm of
``bench.py`` use it, and only as the checker or as the timed CPU baseline.

It is a restatement, in plain PyTorch on the CPU, of the upstream eager
definition ``flash_spacetime.reference.spacetime_attention_reference``
(upstream file ``src/flash_spacetime/reference.py``), generalised from
``C == Dh`` to any ``W: [Dh, C]`` with even ``C``. Every function cites the
upstream lines it follows. The op sequence of :func:`eager_attention` is
kept the same as upstream's so that, in float64 and with ``C == Dh``, it
reproduces upstream bit for bit; ``tests/test_oracle.py`` pins that against
the golden fixtures in ``tests/golden/`` (produced by running the real
upstream code, see ``tests/golden/make_golden.py``).

Conventions (upstream ``forward.py:19-22, 239-245``):

* padded layout: q, k, v ``[B, H, L, Dh]``, feats ``[B, L, F]``, valid rows are
  the prefix ``[0, seqlens[b])`` of each event;
* packed layout: q, k, v ``[T, H, Dh]``, feats ``[T, F]``, events delimited by
  ``cu_seqlens`` (``[B+1]``);
* comparisons are made on valid rows only; the fused op writes exact zeros
  on padding rows.
"""

from typing import Dict, List, Optional, Sequence, Tuple

import torch
from torch import Tensor

TIME_SCALE = 3e4 / 500 * 3e-1  # upstream reference.py:39 (== 18.0)
INPUT_SCALE = 1024.0  # upstream reference.py:40
CLIP = 4.0  # upstream reference.py:41
N_FREQ = 10000.0  # upstream reference.py:42


def freq_ladder(channels: int) -> Tensor:
    """float32 ladder ``exp(-k ln(1e4)/(C/2))`` (upstream reference.py:45-56)."""
    half = channels / 2
    step = -(torch.log(torch.tensor([N_FREQ])) / half)
    return torch.exp(torch.arange(half) * step)


def pair_angle(feats: Tensor) -> Tensor:
    """``x_ij = 1024 clip(sign(I) sqrt|I|, -4, 4)`` (upstream reference.py:75-81)."""
    return pair_angle_between(feats, feats)


def pair_angle_between(fq: Tensor, fk: Tensor) -> Tensor:
    """``x_ij`` between query rows ``fq`` ``[B, Lq, F]`` and key rows ``fk``
    ``[B, Lk, F]``, with upstream's op order (reference.py:75-81)."""
    pq, pk = fq[:, :, :3], fk[:, :, :3]
    tq, tk = fq[:, :, 3], fk[:, :, 3]
    interval = (pq[:, :, None] - pk[:, None, :]).pow(2).sum(-1) - (
        (tq[:, :, None] - tk[:, None, :]) * TIME_SCALE
    ).pow(2)
    signed = torch.sign(interval) * torch.sqrt(torch.abs(interval))
    return INPUT_SCALE * signed.clip(-CLIP, CLIP)


def pair_embedding_between(fq: Tensor, fk: Tensor, channels: int) -> Tensor:
    """``E_ij`` for query rows ``fq`` against key rows ``fk``: ``[B, Lq, Lk, C]``."""
    ang = pair_angle_between(fq, fk).unsqueeze(-1) * freq_ladder(channels).to(fq.device)
    return torch.cat((torch.sin(ang), torch.cos(ang)), dim=-1)


def pair_embedding(feats: Tensor, channels: int) -> Tensor:
    """``E_ij``: ``[B, L, L, C]``, sin half then cos half (reference.py:82-84)."""
    ang = pair_angle(feats).unsqueeze(-1) * freq_ladder(channels).to(feats.device)
    return torch.cat((torch.sin(ang), torch.cos(ang)), dim=-1)


def pair_features(feats: Tensor, weight: Tensor, bias: Optional[Tensor]) -> Tensor:
    """``R = E W^T + b``: ``[B, L, L, Dh]`` (upstream reference.py:59-88)."""
    emb = pair_embedding(feats, weight.shape[1])
    return torch.nn.functional.linear(emb.to(weight.dtype), weight, bias)


def pair_mask(mask: Tensor) -> Tensor:
    """``Attention_rel`` pair mask from a 0/-inf token mask (reference.py:91-103)."""
    out = torch.min(mask[:, None, :], mask[:, :, None]).clone()
    out[torch.max(mask[:, None, :], mask[:, :, None]) < 0] = 0
    return out


def eager_attention(
    q: Tensor,
    k: Tensor,
    v: Tensor,
    feats: Tensor,
    weight: Tensor,
    bias: Optional[Tensor],
    key_padding_mask: Optional[Tensor] = None,
    scale: Optional[float] = None,
    use_attn_bias: bool = True,
    use_activation_bias: bool = True,
) -> Tensor:
    """Composition of upstream reference.py:139-167, generalised to ``W: [Dh, C]``."""
    dim = q.shape[-1]
    if weight.shape[0] != dim or weight.shape[1] % 2:
        raise ValueError(f"bad weight shape {tuple(weight.shape)} for Dh={dim}")
    s = dim**-0.5 if scale is None else scale
    qt = q * s
    attn = qt @ k.transpose(-2, -1)
    rel = None
    if use_attn_bias or use_activation_bias:
        rel = pair_features(feats, weight, bias)
    if use_attn_bias:
        attn = attn + torch.einsum("bhic,bijc->bhij", qt, rel)
    if key_padding_mask is not None:
        attn = attn + pair_mask(key_padding_mask).unsqueeze(1)
    p = attn.softmax(dim=-1)
    out = p.to(v.dtype) @ v
    if use_activation_bias:
        out = out + torch.einsum("bhij,bijc->bhic", p.to(rel.dtype), rel)
    return out


def eager_logits(
    q: Tensor,
    k: Tensor,
    feats: Tensor,
    weight: Tensor,
    scale: Optional[float],
    use_attn_bias: bool,
) -> Tensor:
    """Pre-softmax logits WITHOUT the row-constant ``qt . b`` term.

    The fused op drops ``qt_i . b`` from the logits because it shifts a
    softmax row uniformly (upstream forward.py:8-10); its saved LSE is the
    log-sum-exp of these logits. Used to check the LSE output.
    """
    dim = q.shape[-1]
    s = dim**-0.5 if scale is None else scale
    qt = q * s
    attn = qt @ k.transpose(-2, -1)
    if use_attn_bias:
        emb = pair_embedding(feats, weight.shape[1]).to(weight.dtype)
        u = qt @ weight
        attn = attn + torch.einsum("bhie,bije->bhij", u, emb)
    return attn


# ---------------------------------------------------------------------------
# Per-event evaluation (memory O(L^2) per event, not per batch)
# ---------------------------------------------------------------------------


def events_from_padded(
    seqlens: Sequence[int],
) -> List[Tuple[int, int]]:
    """``(event index, length)`` of every event of a padded batch."""
    return [(b, int(n)) for b, n in enumerate(seqlens)]


def oracle_padded(
    q: Tensor,
    k: Tensor,
    v: Tensor,
    feats: Tensor,
    weight: Tensor,
    bias: Optional[Tensor],
    seqlens: Sequence[int],
    scale: Optional[float] = None,
    use_attn_bias: bool = True,
    use_activation_bias: bool = True,
    grad_out: Optional[Tensor] = None,
    dtype: torch.dtype = torch.float64,
) -> Dict[str, Optional[Tensor]]:
    """Forward (and backward if ``grad_out``) of a padded batch, event by event.

    Every event is evaluated alone on its valid prefix, which gives the same
    valid-row values as the batched eager call with a padding mask (padding
    keys get -inf, upstream reference.py:91-103), at ``O(L_b^2)`` memory.
    Returns ``out`` ``[B, H, L, Dh]`` (zeros on padding rows), ``lse``
    ``[B, H, L]`` (zeros on padding rows) and, with ``grad_out``, the
    gradients ``dq, dk, dv`` (zeros on padding rows), ``dW`` and ``db``.
    Inputs are cast to ``dtype``; ``feats`` to float32 unless ``dtype`` is
    float64 (upstream tests/test_gpu.py:124).
    """
    batch, heads, length, dim = q.shape
    fdt = torch.float64 if dtype == torch.float64 else torch.float32
    w = weight.detach().to(dtype).requires_grad_(grad_out is not None)
    bb = None
    if bias is not None:
        bb = bias.detach().to(dtype).requires_grad_(grad_out is not None)
    out = torch.zeros(batch, heads, length, dim, dtype=dtype)
    lse = torch.zeros(batch, heads, length, dtype=torch.float64)
    grads = {
        "dq": torch.zeros(batch, heads, length, dim, dtype=dtype),
        "dk": torch.zeros(batch, heads, length, dim, dtype=dtype),
        "dv": torch.zeros(batch, heads, length, dim, dtype=dtype),
    }
    for b, n in events_from_padded(seqlens):
        if n == 0:
            continue
        qe = q[b : b + 1, :, :n].detach().to(dtype).requires_grad_(grad_out is not None)
        ke = k[b : b + 1, :, :n].detach().to(dtype).requires_grad_(grad_out is not None)
        ve = v[b : b + 1, :, :n].detach().to(dtype).requires_grad_(grad_out is not None)
        fe = feats[b : b + 1, :n].to(fdt)
        with torch.set_grad_enabled(grad_out is not None):
            oe = eager_attention(
                qe, ke, ve, fe, w, bb, None, scale, use_attn_bias, use_activation_bias
            )
        out[b, :, :n] = oe[0].detach()
        with torch.no_grad():
            lg = eager_logits(
                qe.double(), ke.double(), fe.double(), w.double(), scale, use_attn_bias
            )
            lse[b, :, :n] = torch.logsumexp(lg, dim=-1)[0]
        if grad_out is not None:
            oe.backward(grad_out[b : b + 1, :, :n].to(dtype))
            grads["dq"][b, :, :n] = qe.grad[0]
            grads["dk"][b, :, :n] = ke.grad[0]
            grads["dv"][b, :, :n] = ve.grad[0]
    res: Dict[str, Optional[Tensor]] = {"out": out, "lse": lse}
    if grad_out is not None:
        res.update(grads)
        res["dW"] = w.grad if w.grad is not None else None
        res["db"] = bb.grad if (bb is not None and bb.grad is not None) else None
    return res


def oracle_packed(
    q: Tensor,
    k: Tensor,
    v: Tensor,
    feats: Tensor,
    weight: Tensor,
    bias: Optional[Tensor],
    cu_seqlens: Sequence[int],
    scale: Optional[float] = None,
    use_attn_bias: bool = True,
    use_activation_bias: bool = True,
    grad_out: Optional[Tensor] = None,
    dtype: torch.dtype = torch.float64,
) -> Dict[str, Optional[Tensor]]:
    """Packed-layout counterpart of :func:`oracle_padded`.

    q, k, v are ``[T, H, Dh]``, feats ``[T, F]``, events delimited by
    ``cu_seqlens`` (upstream forward.py:504-527). Outputs are packed too.
    """
    cu = [int(c) for c in cu_seqlens]
    total, heads, dim = q.shape
    fdt = torch.float64 if dtype == torch.float64 else torch.float32
    need_grad = grad_out is not None
    w = weight.detach().to(dtype).requires_grad_(need_grad)
    bb = bias.detach().to(dtype).requires_grad_(need_grad) if bias is not None else None
    out = torch.zeros(total, heads, dim, dtype=dtype)
    lse = torch.zeros(total, heads, dtype=torch.float64)
    dq = torch.zeros(total, heads, dim, dtype=dtype)
    dk = torch.zeros(total, heads, dim, dtype=dtype)
    dv = torch.zeros(total, heads, dim, dtype=dtype)
    for s0, s1 in zip(cu[:-1], cu[1:]):
        if s1 == s0:
            continue

        def ev(t: Tensor) -> Tensor:
            return t[s0:s1].detach().to(dtype).permute(1, 0, 2)[None].requires_grad_(need_grad)

        qe, ke, ve = ev(q), ev(k), ev(v)
        fe = feats[s0:s1].to(fdt)[None]
        with torch.set_grad_enabled(need_grad):
            oe = eager_attention(
                qe, ke, ve, fe, w, bb, None, scale, use_attn_bias, use_activation_bias
            )
        out[s0:s1] = oe[0].detach().permute(1, 0, 2)
        with torch.no_grad():
            lg = eager_logits(
                qe.double(), ke.double(), fe.double(), w.double(), scale, use_attn_bias
            )
            lse[s0:s1] = torch.logsumexp(lg, dim=-1)[0].t()
        if need_grad:
            oe.backward(grad_out[s0:s1].to(dtype).permute(1, 0, 2)[None])
            dq[s0:s1] = qe.grad[0].permute(1, 0, 2)
            dk[s0:s1] = ke.grad[0].permute(1, 0, 2)
            dv[s0:s1] = ve.grad[0].permute(1, 0, 2)
    res: Dict[str, Optional[Tensor]] = {"out": out, "lse": lse}
    if need_grad:
        res.update({"dq": dq, "dk": dk, "dv": dv})
        res["dW"] = w.grad
        res["db"] = bb.grad if bb is not None else None
    return res


def eager_fwd_bwd_fp32(
    q: Tensor,
    k: Tensor,
    v: Tensor,
    feats: Tensor,
    weight: Tensor,
    bias: Tensor,
    key_padding_mask: Optional[Tensor],
) -> Tensor:
    """One fp32 forward+backward of the eager definition (the CPU baseline).

    This is the upstream eager path (reference.py:106-167) run through
    autograd, as upstream's own debug backward does (forward.py:433-478).
    Returns the loss so the caller can keep the work alive.
    """
    leaves = [t.detach().float().requires_grad_(True) for t in (q, k, v, weight, bias)]
    qq, kk, vv, ww, bb = leaves
    out = eager_attention(qq, kk, vv, feats.float(), ww, bb, key_padding_mask)
    loss = (out * out).sum() * 0.5
    loss.backward()
    return loss.detach()


# ---------------------------------------------------------------------------
# Row and column subsets of one long event (float64)
# ---------------------------------------------------------------------------
#
# For events too long for the full O(L^2) evaluation (L = 16384), the
# quantities that belong to one query row depend only on that row and all
# keys, so a subset of rows is checked exactly; those that belong to one key
# (dk, dv) need every row's log-sum-exp and D, which are taken from the
# kernel under test after its rows were checked against event_rows.


def event_rows(
    q: Tensor,
    k: Tensor,
    v: Tensor,
    feats: Tensor,
    weight: Tensor,
    bias: Optional[Tensor],
    rows: Tensor,
    scale: Optional[float] = None,
    use_attn_bias: bool = True,
    use_activation_bias: bool = True,
    grad_out: Optional[Tensor] = None,
) -> Dict[str, Tensor]:
    """Outputs of the query ``rows`` of ONE event in float64.

    q, k, v: ``[L, H, Dh]`` (the event's packed rows); feats ``[L, >=4]``;
    ``rows``: int64 indices; ``grad_out``: ``[len(rows), H, Dh]`` or None.
    Returns ``out`` ``[R, H, Dh]``, ``lse`` ``[R, H]`` (logits without the
    ``qt.b`` row constant) and, with ``grad_out``, ``dq`` ``[R, H, Dh]`` and
    ``delta`` ``[R, H]`` = ``dO . (out - [act] b)``, the P-weighted mean of
    dP without its ``dO.b`` constant. The composition is that of
    :func:`eager_attention` (upstream reference.py:139-167) restricted to
    the rows.
    """
    dim = q.shape[-1]
    s = dim**-0.5 if scale is None else scale
    need = grad_out is not None
    qs = q[rows].double().permute(1, 0, 2)[None].requires_grad_(need)  # [1, H, R, Dh]
    kk = k.double().permute(1, 0, 2)[None]
    vv = v.double().permute(1, 0, 2)[None]
    fq = feats[rows].double()[None]
    fk = feats.double()[None]
    w = weight.double()
    b = None if bias is None else bias.double()
    with torch.set_grad_enabled(need):
        qt = qs * s
        attn = qt @ kk.transpose(-2, -1)
        rel = emb = None
        if use_attn_bias or use_activation_bias:
            emb = pair_embedding_between(fq, fk, w.shape[1])
            rel = torch.nn.functional.linear(emb, w, b)
        if use_attn_bias:
            attn = attn + torch.einsum("bhic,bijc->bhij", qt, rel)
        p = attn.softmax(dim=-1)
        out = p @ vv
        if use_activation_bias:
            out = out + torch.einsum("bhij,bijc->bhic", p, rel)
    with torch.no_grad():
        lg = qt @ kk.transpose(-2, -1)
        if use_attn_bias:
            lg = lg + torch.einsum("bhie,bije->bhij", qt @ w, emb)
        lse = torch.logsumexp(lg, dim=-1)[0].t()
    res = {"out": out.detach()[0].permute(1, 0, 2), "lse": lse}
    if need:
        g = grad_out.double().permute(1, 0, 2)[None]
        out.backward(g)
        res["dq"] = qs.grad[0].permute(1, 0, 2)
        off = out.detach()
        if use_activation_bias and b is not None:
            off = off - b
        res["delta"] = (g * off).sum(-1)[0].t()
    return res


def event_cols(
    q: Tensor,
    k: Tensor,
    v: Tensor,
    feats: Tensor,
    weight: Tensor,
    cols: Tensor,
    lse: Tensor,
    delta: Tensor,
    grad_out: Tensor,
    scale: Optional[float] = None,
    use_attn_bias: bool = True,
    use_activation_bias: bool = True,
) -> Dict[str, Tensor]:
    """``dk``, ``dv`` of the key ``cols`` of ONE event in float64.

    Upstream's column contraction (backward.py:209-313): ``P_ij = exp(s_ij -
    lse_i)``, ``dP_ij = dO_i . v_j + [act] (dO_i W) . E_ij``,
    ``dS = P (dP - D_i)``, ``dk_j = sum_i dS_ij qt_i``, ``dv_j = sum_i P_ij
    dO_i`` over all rows i. ``lse`` and ``delta`` ``[L, H]`` are every row's
    log-sum-exp (without ``qt.b``) and D (without ``dO.b``), which the caller
    takes from the kernel after checking them on sampled rows.
    """
    dim = q.shape[-1]
    s = dim**-0.5 if scale is None else scale
    qt = q.double().permute(1, 0, 2) * s          # [H, L, Dh]
    kc = k[cols].double().permute(1, 0, 2)        # [H, J, Dh]
    vc = v[cols].double().permute(1, 0, 2)
    do = grad_out.double().permute(1, 0, 2)       # [H, L, Dh]
    w = weight.double()
    logits = qt @ kc.transpose(-2, -1)            # [H, L, J]
    dp = do @ vc.transpose(-2, -1)
    if use_attn_bias or use_activation_bias:
        emb = pair_embedding_between(feats.double()[None], feats[cols].double()[None],
                                     w.shape[1])[0]  # [L, J, C]
        if use_attn_bias:
            logits = logits + torch.einsum("hic,ijc->hij", qt @ w, emb)
        if use_activation_bias:
            dp = dp + torch.einsum("hic,ijc->hij", do @ w, emb)
    p = torch.exp(logits - lse.double().t()[:, :, None])
    ds = p * (dp - delta.double().t()[:, :, None])
    dk = (ds.transpose(-2, -1) @ qt).permute(1, 0, 2)
    dv = (p.transpose(-2, -1) @ do).permute(1, 0, 2)
    return {"dk": dk, "dv": dv}
