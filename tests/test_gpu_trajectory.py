"""Training-trajectory self-consistency.

A short gradient-descent loop through the fused op (bf16 compute, fp32 master
parameters) next to the same loop on the float64 oracle: the losses of the
two trajectories must stay together step after step, and at every step the
fused backward's D must make rowsum(dS) vanish (upstream README.md:53-84 asks
for D = sum(P dP) / sum(P) formed from the same P and dP as dS, and advises
validating training trajectories).
"""

import pytest
import torch

import cases as cs
from oracle import spacetime_oracle as orc

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from flash_spacetime.ops import flash_spacetime_backward, flash_spacetime_forward

KEYS = ("q", "k", "v", "weight", "bias")
GRAD = {"q": "dq", "k": "dk", "v": "dv", "weight": "dW", "bias": "db"}


def test_sgd_trajectory_tracks_fp64():
    batch, length, heads, dim, ch = 2, 48, 4, 32, 16
    case = cs.padded_case(batch, length, heads, dim, ch, True, seed=2024)
    gen = torch.Generator().manual_seed(77)
    target = 0.5 * torch.randn(batch, heads, length, dim, generator=gen, dtype=torch.float64)
    vm = cs.valid_mask(case).to(torch.float64)  # [B, 1, L, 1]
    nvalid = float(vm.sum()) * heads * dim
    seq = cs.lengths_to_list(case["seqlens"])
    feats = case["feats"]

    p64 = {k: case[k].clone() for k in KEYS}
    pk = {k: case[k].float().cuda() for k in KEYS}
    feats_c, seq_c = feats.cuda(), case["seqlens"].cuda()
    target_c, vm_c = target.float().cuda(), vm.float().cuda()
    lr, steps = 4.0, 8
    losses64, lossesk = [], []
    for _ in range(steps):
        # Float64 oracle step.
        fwd = orc.oracle_padded(p64["q"], p64["k"], p64["v"], feats, p64["weight"],
                                p64["bias"], seq)
        diff = (fwd["out"] - target) * vm
        losses64.append(float((diff * diff).sum()) / nvalid)
        res = orc.oracle_padded(p64["q"], p64["k"], p64["v"], feats, p64["weight"],
                                p64["bias"], seq, grad_out=2.0 * diff / nvalid)
        for k in KEYS:
            p64[k] = p64[k] - lr * res[GRAD[k]]

        # Fused step: bf16 compute from fp32 master parameters.
        q, k_, v = (pk[x].to(torch.bfloat16) for x in ("q", "k", "v"))
        out, lse = flash_spacetime_forward(q, k_, v, feats_c, pk["weight"], pk["bias"], seq_c)
        diffk = (out.float() - target_c) * vm_c
        lossesk.append(float((diffk * diffk).sum()) / nvalid)
        g = flash_spacetime_backward(q, k_, v, feats_c, pk["weight"], pk["bias"], seq_c, out,
                                     lse, (2.0 * diffk / nvalid).to(torch.bfloat16),
                                     want_absmax=True)
        rows = cs.valid_mask(case)[..., 0].cuda().expand_as(g["sigma"])
        ratio = (g["sigma"][rows].abs() / g["ds_absmax"][rows].clamp_min(1e-30)).max().item()
        assert ratio < 1e-6, f"rowsum dS / rowmax |dS| = {ratio:.3e}"
        for k in KEYS:
            pk[k] = pk[k] - lr * g[GRAD[k]].float()

    # The loss falls along both trajectories, and they agree at every step.
    assert losses64[-1] < 0.9 * losses64[0]
    for step, (a, b) in enumerate(zip(losses64, lossesk)):
        assert abs(a - b) <= 2e-2 * abs(a), f"step {step}: fp64 {a:.6f} vs fused {b:.6f}"
    for k in ("q", "k", "v"):
        drift = cs.normwise(cs.valid_values(pk[k].double().cpu(), case),
                            cs.valid_values(p64[k], case))
        assert drift <= 2e-2, f"{k} drift {drift:.3e}"
    assert cs.normwise(pk["weight"].double().cpu(), p64["weight"]) <= 2e-2
