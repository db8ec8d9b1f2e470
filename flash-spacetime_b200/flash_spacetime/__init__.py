"""Fused spacetime-bias attention for NVIDIA B200 (sm_100a).

Attention whose logits carry a learned bias built from the spacetime
interval between two detector pulses::

    s_ij = q_i . k_j + <q_i, R_ij>,     R_ij = E(x_i, x_j) W^T + b

with ``E`` a sinusoidal embedding of the clipped signed interval. The fused
kernels rebuild ``E`` inside each tile, so the ``[B, L, L, C]`` pair tensor is
never materialised. The compute runs in hand-written CUDA for sm_100a behind
a C ABI (``libflash_spacetime.so``); this package is the PyTorch front end.

The exported names are those of the upstream ``flash_spacetime`` package
(upstream src/flash_spacetime/__init__.py:38-54). ``reference`` holds the
pure-PyTorch definition and is importable without a GPU; the fused entry
points load the CUDA library on first use.
"""

from .reference import (  # noqa: F401
    SINEMB_CLIP,
    SINEMB_INPUT_SCALE,
    SINEMB_N_FREQ,
    TIME_SCALE,
    attention_rel_oracle_inputs,
    float_padding_mask,
    merge_heads,
    pair_mask_bias,
    sinusoidal_frequencies,
    spacetime_attention_reference,
    spacetime_pair_features,
    split_heads,
    valid_row_mask,
)

__all__ = [
    "flash_spacetime_attention",
    "flash_spacetime_attention_varlen",
    "spacetime_attention_reference",
    "spacetime_pair_features",
    "sinusoidal_frequencies",
    "attention_rel_oracle_inputs",
    "pair_mask_bias",
    "float_padding_mask",
    "valid_row_mask",
    "split_heads",
    "merge_heads",
    "TIME_SCALE",
    "SINEMB_INPUT_SCALE",
    "SINEMB_CLIP",
    "SINEMB_N_FREQ",
]


def __getattr__(name: str) -> object:
    """Resolve the fused entry points lazily (they need the CUDA library)."""
    if name in ("flash_spacetime_attention", "flash_spacetime_attention_varlen",
                "flash_spacetime_attention_nested", "flash_spacetime_attention_qkv",
                "flash_spacetime_forward",
                "flash_spacetime_backward", "upload_valid_rows"):
        from . import ops

        return getattr(ops, name)
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
