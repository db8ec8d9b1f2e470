"""Generate the golden fixtures in this folder from the upstream reference.

Run once, on a machine where the upstream ``flash_spacetime`` sources are
available (pass their ``src`` folder as the first argument)::

    python tests/golden/make_golden.py <upstream>/src

It imports the UPSTREAM pure-PyTorch specification
(``flash_spacetime.reference``, upstream ``src/flash_spacetime/reference.py``)
and evaluates it on small seeded cases with ``C == Dh`` (the only shapes
upstream accepts, reference.py:139-143): forward outputs and autograd
gradients in float64 and float32, the frequency ladder, the pair features and
the pair mask. The fixtures are what ``tests/test_oracle.py`` pins the CPU
oracle against; the GPU tests never read the upstream sources.

Inputs follow upstream's test generator (tests/test_gpu.py:81-108): q, k, v,
feats ~ N(0, 1) in float64, W ~ N(0, 1/D), b ~ N(0, 1), with one full-length
and one length-1 event when masked. Two extra cases use detector-like
coordinates: raw metres / nanoseconds (every off-diagonal interval clipped)
and a shrunken copy whose intervals stay inside the unclipped sqrt branch.
"""

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

# (name, batch, length, heads, dim, flags, masked, dtype, coords)
CASES = [
    ("tt_masked_d16", 2, 17, 4, 16, (True, True), True, "f64", "randn"),
    ("tf_masked_d32", 2, 33, 4, 32, (True, False), True, "f64", "randn"),
    ("ft_masked_d16", 3, 20, 2, 16, (False, True), True, "f64", "randn"),
    ("ff_full_d16", 1, 9, 3, 16, (False, False), False, "f64", "randn"),
    ("tt_full_d48", 1, 12, 2, 48, (True, True), False, "f64", "randn"),
    ("tt_masked_d16_fp32", 2, 17, 4, 16, (True, True), True, "f32", "randn"),
    ("tt_detector_clipped", 2, 24, 4, 16, (True, True), True, "f64", "detector"),
    ("tt_detector_unclipped", 2, 24, 4, 16, (True, True), True, "f64", "scaled"),
]


def _detector_feats(gen: torch.Generator, batch: int, length: int) -> torch.Tensor:
    r = 500.0 * torch.rand(batch, length, generator=gen, dtype=torch.float64).sqrt()
    phi = 2 * np.pi * torch.rand(batch, length, generator=gen, dtype=torch.float64)
    z = 1000.0 * torch.rand(batch, length, generator=gen, dtype=torch.float64) - 500.0
    t = 20000.0 * torch.rand(batch, length, generator=gen, dtype=torch.float64)
    t, _ = torch.sort(t, dim=1)
    extra = torch.randn(batch, length, generator=gen, dtype=torch.float64)
    return torch.stack((r * torch.cos(phi), r * torch.sin(phi), z, t, extra), -1)


def main(upstream_src: str) -> None:
    sys.path.insert(0, upstream_src)
    import flash_spacetime.reference as ref  # the UPSTREAM module

    assert os.path.abspath(ref.__file__).startswith(os.path.abspath(upstream_src))

    ladders = {f"freqs_{c}": ref.sinusoidal_frequencies(c, torch.device("cpu")).numpy()
               for c in (8, 16, 32, 48, 64)}
    np.savez_compressed(os.path.join(HERE, "freqs.npz"), **ladders)

    for seed, (name, batch, length, heads, dim, flags, masked, dt, coords) in enumerate(CASES):
        gen = torch.Generator().manual_seed(1000 + seed)

        def rand(*size: int) -> torch.Tensor:
            return torch.randn(*size, generator=gen, dtype=torch.float64)

        q, k, v = rand(batch, heads, length, dim), rand(batch, heads, length, dim), rand(batch, heads, length, dim)
        if coords == "randn":
            feats = rand(batch, length, 5)
        else:
            feats = _detector_feats(gen, batch, length)
            if coords == "scaled":
                # Positions in units of 500 m and time in units of 3e4 ns: the
                # encoder's own normalisation, |I| < 16 on most pairs.
                feats[..., :3] /= 500.0
                feats[..., 3] /= 3e4
        weight = rand(dim, dim) / dim**0.5
        bias = rand(dim)
        if masked and length > 1:
            seqlens = torch.randint(1, length + 1, (batch,), generator=gen)
            seqlens[0] = length
            if batch > 1:
                seqlens[-1] = 1
        else:
            seqlens = torch.full((batch,), length, dtype=torch.long)
        grad_w = rand(batch, heads, length, dim)

        cdt = torch.float64 if dt == "f64" else torch.float32
        valid = ref.valid_row_mask(batch, length, seqlens)
        mask = ref.float_padding_mask(valid, torch.float32)
        leaves = [t.to(cdt).clone().requires_grad_(True) for t in (q, k, v, weight, bias)]
        fe = feats.to(torch.float64 if cdt == torch.float64 else torch.float32)
        out = ref.spacetime_attention_reference(
            *leaves[:3], fe, leaves[3], leaves[4],
            key_padding_mask=mask,
            use_attn_bias=flags[0], use_activation_bias=flags[1],
        )
        loss = (out * grad_w.to(cdt) * valid[:, None, :, None]).sum()
        loss.backward()
        grads = {}
        for key, t in zip(("dq", "dk", "dv", "dW", "db"), leaves):
            grads[key] = (t.grad.detach().numpy() if t.grad is not None
                          else np.zeros(0, dtype=np.float64))
        extra = {}
        if (flags[0] or flags[1]) and length <= 24:
            extra["pair_features"] = ref.spacetime_pair_features(
                fe.detach(), leaves[3].detach(), leaves[4].detach()).numpy()
        extra["pair_mask"] = ref.pair_mask_bias(mask).numpy()
        np.savez_compressed(
            os.path.join(HERE, f"{name}.npz"),
            q=q.numpy(), k=k.numpy(), v=v.numpy(), feats=feats.numpy(),
            weight=weight.numpy(), bias=bias.numpy(), seqlens=seqlens.numpy(),
            grad_w=grad_w.numpy(), flags=np.array(flags), dtype=np.array(dt),
            out=out.detach().numpy(), **grads, **extra,
        )
        print(f"{name}: out {tuple(out.shape)} {dt}")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "")
