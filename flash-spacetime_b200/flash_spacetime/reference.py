"""Pure-PyTorch definition of fused spacetime-bias attention.

This module is part of the public surface (the same names the upstream
package exports from ``flash_spacetime/reference.py``), so that callers who
validate their models against the eager definition keep working. It is the
mathematical specification only: the fused op in ``flash_spacetime.ops``
never calls into it.

The op, per event and head, is::

    qt_i  = q_i * scale
    I_ij  = |p_i - p_j|^2 - ((t_i - t_j) * TIME_SCALE)^2
    x_ij  = 1024 * clip(sign(I_ij) * sqrt|I_ij|, -4, 4)
    E_ij  = [sin(x_ij f_k) ; cos(x_ij f_k)],  f_k = 10000^(-k/(C/2))
    R_ij  = E_ij W^T + b                      (W: [Dh, C], nn.Linear layout)
    s_ij  = qt_i . k_j + [attn] qt_i . R_ij + mask_ij
    out_i = sum_j softmax(s)_ij v_j + [act] sum_j softmax(s)_ij R_ij

Generalisation over upstream: upstream requires ``C == Dh``
(flash_spacetime/reference.py:139-143). Here ``W`` may be any ``[Dh, C]`` with
``C`` even; the channel count is read from ``W.shape[1]`` exactly as the
upstream frequency ladder already does (reference.py:82). With ``C == Dh`` the
two definitions are the same computation.
"""

from typing import Optional, Tuple

import torch
from torch import Tensor

# The time axis is converted to the position unit with the encoder's own
# expression; written the same way so it rounds to the same double (18.0).
TIME_SCALE = 3e4 / 500 * 3e-1
SINEMB_INPUT_SCALE = 1024.0
SINEMB_CLIP = 4.0
SINEMB_N_FREQ = 10000.0


def sinusoidal_frequencies(dim: int, device: torch.device) -> Tensor:
    """float32 frequency ladder ``exp(-k ln(1e4) / (dim/2))``, k < dim/2.

    Follows upstream reference.py:45-56: the ladder is always float32, even
    when the surrounding arithmetic runs in float64.
    """
    half = dim / 2
    step = -(torch.log(torch.tensor([SINEMB_N_FREQ], device=device)) / half)
    return torch.exp(torch.arange(half, device=device) * step)


def _pair_angle(feats: Tensor) -> Tensor:
    """``x_ij`` for a ``[B, L, F]`` feature tensor (upstream reference.py:75-81)."""
    xyz = feats[:, :, :3]
    t = feats[:, :, 3]
    d2 = (xyz[:, :, None] - xyz[:, None, :]).pow(2).sum(-1)
    dt2 = ((t[:, :, None] - t[:, None, :]) * TIME_SCALE).pow(2)
    interval = d2 - dt2
    signed = torch.sign(interval) * torch.sqrt(torch.abs(interval))
    return SINEMB_INPUT_SCALE * signed.clip(-SINEMB_CLIP, SINEMB_CLIP)


def spacetime_pair_features(
    feats: Tensor,
    weight: Tensor,
    bias: Optional[Tensor],
) -> Tensor:
    """``R_ij`` for every pair: ``[B, L, L, Dh]`` (upstream reference.py:59-88).

    ``feats`` is ``[B, L, F]`` with x, y, z in columns 0-2 and the interval's
    time coordinate in column 3. ``weight`` is ``[Dh, C]``; the embedding has
    ``C`` channels (sin half then cos half) and follows the dtype of
    ``feats``; the projection runs in the dtype of ``weight``.
    """
    x = _pair_angle(feats)
    freqs = sinusoidal_frequencies(weight.shape[1], feats.device)
    ang = x.unsqueeze(-1) * freqs
    emb = torch.cat((torch.sin(ang), torch.cos(ang)), dim=-1)
    return torch.nn.functional.linear(emb.to(weight.dtype), weight, bias)


def pair_mask_bias(key_padding_mask: Tensor) -> Tensor:
    """Additive ``[B, L, L]`` pair mask of ``Attention_rel``.

    ``key_padding_mask`` is ``[B, L]``, 0 for valid tokens and -inf for
    padding. A pair is -inf when exactly one side is padding; pairs whose two
    sides are both padding stay 0 (upstream reference.py:91-103), so padding
    rows never produce NaN in the eager definition.
    """
    m = key_padding_mask
    out = torch.minimum(m[:, None, :], m[:, :, None]).clone()
    both_pad = torch.maximum(m[:, None, :], m[:, :, None]) < 0
    out[both_pad] = 0
    return out


def spacetime_attention_reference(
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
    """Eager definition of the op (upstream reference.py:106-167).

    q, k, v are ``[B, H, L, Dh]``; ``weight`` is ``[Dh, C]``; ``bias`` is
    ``[Dh]`` or None; ``key_padding_mask`` is a ``[B, L]`` float mask (0 valid,
    -inf padding) or None. Padding rows hold the eager modules' garbage;
    compare on valid rows only.
    """
    head_dim = q.shape[-1]
    if weight.dim() != 2 or weight.shape[0] != head_dim:
        raise ValueError(
            f"weight must be [head_dim, C] = [{head_dim}, C], got "
            f"{tuple(weight.shape)}"
        )
    if weight.shape[1] % 2:
        raise ValueError(f"C (={weight.shape[1]}) must be even")
    s = head_dim**-0.5 if scale is None else scale

    qt = q * s
    logits = qt @ k.transpose(-2, -1)
    rel = None
    if use_attn_bias or use_activation_bias:
        rel = spacetime_pair_features(feats, weight, bias)
    if use_attn_bias:
        logits = logits + torch.einsum("bhic,bijc->bhij", qt, rel)
    if key_padding_mask is not None:
        logits = logits + pair_mask_bias(key_padding_mask).unsqueeze(1)
    p = logits.softmax(dim=-1)
    out = p.to(v.dtype) @ v
    if use_activation_bias:
        out = out + torch.einsum("bhij,bijc->bhic", p.to(rel.dtype), rel)
    return out


def valid_row_mask(batch_size: int, length: int, seqlens: Tensor) -> Tensor:
    """``[B, L]`` bool, True on valid (non-padding) rows."""
    pos = torch.arange(length, device=seqlens.device)
    return pos[None, :] < seqlens[:, None]


def float_padding_mask(valid: Tensor, dtype: torch.dtype) -> Tensor:
    """0 / -inf float mask (``Attention_rel`` convention) from a bool mask."""
    out = torch.zeros(valid.shape, dtype=dtype, device=valid.device)
    out.masked_fill_(~valid, float("-inf"))
    return out


def split_heads(x: Tensor, num_heads: int) -> Tensor:
    """``[B, L, H*D]`` -> ``[B, H, L, D]``."""
    b, n, _ = x.shape
    return x.reshape(b, n, num_heads, -1).transpose(1, 2)


def merge_heads(x: Tensor) -> Tensor:
    """``[B, H, L, D]`` -> ``[B, L, H*D]``."""
    b, _, n, _ = x.shape
    return x.transpose(1, 2).reshape(b, n, -1)


def attention_rel_oracle_inputs(
    attention: torch.nn.Module,
    x: Tensor,
    kv: Optional[Tensor] = None,
) -> Tuple[Tensor, Tensor, Tensor]:
    """Per-head q, k, v as ``Attention_rel.forward`` builds them.

    Uses the module's ``proj_q``/``proj_k``/``proj_v`` weights and its optional
    ``q_bias``/``v_bias`` (upstream reference.py:198-223).
    """
    src = x if kv is None else kv
    lin = torch.nn.functional.linear
    q = lin(x, attention.proj_q.weight, attention.q_bias)
    k = lin(src, attention.proj_k.weight, None)
    v = lin(src, attention.proj_v.weight, attention.v_bias)
    h = attention.num_heads
    return split_heads(q, h), split_heads(k, h), split_heads(v, h)
