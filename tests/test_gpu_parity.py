"""GPU parity: the fused CUDA op against the float64 CPU oracle (padded layout).

Ports upstream tests/test_gpu.py (forward and backward against fp64 with
the 2x-eager rule, exact-zero padding rows, determinism, the feats-grad
guard) and extends it to the generalised shapes (C != Dh, C in 16..64,
Dh in 16..64), fp16, the benchmark's detector coordinates (clipped
intervals) and normalised coordinates (unclipped sqrt branch).
"""

import pytest
import torch

import cases as cs

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from flash_spacetime.ops import (
        flash_spacetime_attention,
        flash_spacetime_backward,
        flash_spacetime_forward,
    )

# (batch, length, heads, head_dim, channels): straddles 16/32/64/128-row tile
# edges, upstream's shapes (C == Dh in {16, 32, 48}) and the generalised ones.
SHAPES = [
    (2, 1, 4, 48, 48),
    (2, 3, 4, 48, 48),
    (2, 17, 4, 48, 48),
    (3, 32, 16, 48, 48),
    (2, 33, 16, 48, 48),
    (1, 64, 16, 48, 48),
    (2, 65, 1, 48, 48),
    (2, 127, 16, 48, 48),
    (2, 128, 4, 48, 48),
    (2, 200, 16, 48, 48),
    (1, 800, 16, 48, 48),
    (2, 33, 4, 16, 16),
    (2, 33, 4, 32, 32),
    (2, 130, 12, 32, 16),   # the benchmark's head/channel widths
    (2, 65, 8, 64, 32),
    (2, 70, 8, 32, 64),
    (1, 129, 8, 64, 64),
]
FP16_SHAPES = [SHAPES[2], SHAPES[4], SHAPES[12], SHAPES[13], SHAPES[15]]
FLAGS = [(True, True), (True, False), (False, True), (False, False)]
DTYPES = [torch.float32, torch.bfloat16, torch.float16]


def _to(t: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    return t.to(device="cuda", dtype=dtype)


def _seed(*parts: int) -> int:
    s = 17
    for p in parts:
        s = (s * 1000003 + int(p)) % (2**31)
    return s


def _forward(case, flags, dtype):
    return flash_spacetime_forward(
        _to(case["q"], dtype), _to(case["k"], dtype), _to(case["v"], dtype),
        case["feats"].cuda(), _to(case["weight"], dtype), _to(case["bias"], dtype),
        case["seqlens"].cuda(), use_attn_bias=flags[0], use_activation_bias=flags[1],
    )


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("flags", FLAGS)
@pytest.mark.parametrize("masked", [False, True])
@pytest.mark.parametrize("dtype", DTYPES)
def test_forward_matches_oracle(shape, flags, masked, dtype) -> None:
    if dtype == torch.float16 and shape not in FP16_SHAPES:
        pytest.skip("fp16 runs on a subset of the shapes")
    b, n, h, d, c = shape
    case = cs.padded_case(b, n, h, d, c, masked, seed=_seed(*shape, *flags, masked))
    out, lse = _forward(case, flags, dtype)
    torch.cuda.synchronize()
    out = out.cpu()
    assert out.dtype == dtype
    assert torch.isfinite(out).all()
    pad = ~cs.valid_mask(case).expand_as(out)
    assert (out[pad] == 0).all(), "padding rows must be exactly zero"

    ref64 = cs.eager_padded(case, flags, torch.float64, grad=False)
    eager = cs.eager_padded(case, flags, dtype, grad=False)
    kv, rv, ev = (cs.valid_values(t, case) for t in (out, ref64["out"], eager["out"]))
    cs.assert_2x_rule(kv, ev, rv, cs.atol_for(dtype, flags), "forward", dtype)
    if dtype != torch.float32 or not (flags[0] or flags[1]):
        assert cs.normwise(kv, rv) <= cs.NORMWISE[dtype]
    vm = cs.valid_mask(case)[..., 0]
    lse_c = lse.cpu()
    torch.testing.assert_close(lse_c[vm.expand_as(lse_c)].double(),
                               ref64["lse"][vm.expand_as(lse_c)],
                               atol=2e-2 if dtype != torch.float32 else 2e-3, rtol=1e-3)


@pytest.mark.parametrize("shape", [SHAPES[2], SHAPES[4], SHAPES[9], SHAPES[13]])
@pytest.mark.parametrize("flags", FLAGS[:2])
@pytest.mark.parametrize("dtype", DTYPES)
def test_forward_deterministic(shape, flags, dtype) -> None:
    b, n, h, d, c = shape
    case = cs.padded_case(b, n, h, d, c, True, seed=1234)
    o1, l1 = _forward(case, flags, dtype)
    o2, l2 = _forward(case, flags, dtype)
    assert torch.equal(o1, o2)
    assert torch.equal(l1, l2)


def _kernel_grads(case, flags, dtype):
    leaves = {k: _to(case[k], dtype).requires_grad_(True) for k in ("q", "k", "v", "weight", "bias")}
    out = flash_spacetime_attention(
        leaves["q"], leaves["k"], leaves["v"], case["feats"].cuda(), leaves["weight"],
        leaves["bias"], case["seqlens"].cuda(), use_attn_bias=flags[0],
        use_activation_bias=flags[1],
    )
    vm = cs.valid_mask(case).cuda()
    (out * _to(case["grad"], dtype) * vm).sum().backward()
    return {k: (None if t.grad is None else t.grad.cpu()) for k, t in leaves.items()}


@pytest.mark.parametrize("shape", [SHAPES[2], SHAPES[5], SHAPES[9], SHAPES[11], SHAPES[12],
                                   SHAPES[13], SHAPES[14], SHAPES[15], SHAPES[16]])
@pytest.mark.parametrize("flags", FLAGS)
@pytest.mark.parametrize("masked", [False, True])
@pytest.mark.parametrize("dtype", DTYPES)
def test_backward_matches_oracle(shape, flags, masked, dtype) -> None:
    if dtype == torch.float16 and shape not in FP16_SHAPES:
        pytest.skip("fp16 runs on a subset of the shapes")
    b, n, h, d, c = shape
    case = cs.padded_case(b, n, h, d, c, masked, seed=_seed(7, *shape, *flags, masked))
    kg = _kernel_grads(case, flags, dtype)
    ref64 = cs.eager_padded(case, flags, torch.float64, grad=True)
    eager = cs.eager_padded(case, flags, dtype, grad=True)
    names = {"q": "dq", "k": "dk", "v": "dv", "weight": "dW", "bias": "db"}
    for key, rk in names.items():
        if key in ("weight", "bias") and not (flags[0] or flags[1]):
            assert kg[key] is None and ref64[rk] is None
            continue
        assert kg[key] is not None and ref64[rk] is not None
        if key in ("q", "k", "v"):
            kv, rv, ev = (cs.valid_values(t, case) for t in (kg[key], ref64[rk], eager[rk]))
        else:
            kv, rv, ev = kg[key].flatten(), ref64[rk].flatten(), eager[rk].flatten()
        cs.assert_2x_rule(kv, ev, rv, cs.atol_for(dtype, flags), f"grad {key}", dtype,
                          reduction=True)


@pytest.mark.parametrize("shape", [SHAPES[9], SHAPES[13], SHAPES[14]])
@pytest.mark.parametrize("dtype", DTYPES)
def test_rowsum_ds_is_zero(shape, dtype) -> None:
    """D is formed from the P and dP that build dS, so rowsum(dS) vanishes."""
    b, n, h, d, c = shape
    case = cs.padded_case(b, n, h, d, c, True, seed=_seed(99, *shape))
    args = [_to(case[k], dtype) for k in ("q", "k", "v")]
    feats, w, bb = case["feats"].cuda(), _to(case["weight"], dtype), _to(case["bias"], dtype)
    seq = case["seqlens"].cuda()
    out, lse = flash_spacetime_forward(*args, feats, w, bb, seq)
    g = flash_spacetime_backward(*args, feats, w, bb, seq, out, lse, _to(case["grad"], dtype),
                                 want_absmax=True)
    vm = cs.valid_mask(case)[..., 0].cuda().expand_as(g["sigma"])
    sig, amax = g["sigma"][vm].abs(), g["ds_absmax"][vm]
    assert torch.isfinite(sig).all()
    ratio = (sig / amax.clamp_min(1e-30)).max().item()
    assert ratio < 1e-6, f"max |rowsum dS| / rowmax |dS| = {ratio:.3e}"


@pytest.mark.parametrize("coords", ["detector", "scaled"])
@pytest.mark.parametrize("dtype", DTYPES)
def test_detector_coordinates(coords, dtype) -> None:
    """Benchmark coordinates (clipped) and normalised ones (sqrt branch)."""
    case = cs.padded_case(3, 96, 12, 32, 16, True, seed=_seed(5, len(coords)), coords=coords)
    flags = (True, True)
    out, _ = _forward(case, flags, dtype)
    ref64 = cs.eager_padded(case, flags, torch.float64, grad=True)
    eager = cs.eager_padded(case, flags, dtype, grad=False)
    kv, rv, ev = (cs.valid_values(t, case) for t in (out.cpu(), ref64["out"], eager["out"]))
    cs.assert_2x_rule(kv, ev, rv, cs.atol_for(dtype, flags), "forward", dtype)
    kg = _kernel_grads(case, flags, dtype)
    for key, rk in (("q", "dq"), ("k", "dk"), ("v", "dv")):
        kv, rv = cs.valid_values(kg[key], case), cs.valid_values(ref64[rk], case)
        assert cs.normwise(kv, rv) <= (2e-2 if dtype != torch.float32 else 1e-3), key


def test_feats_requires_grad_raises() -> None:
    case = cs.padded_case(2, 17, 4, 48, 48, False, seed=5)
    feats = case["feats"].cuda().requires_grad_(True)
    with pytest.raises(ValueError, match="feats"):
        flash_spacetime_attention(
            _to(case["q"], torch.float32), _to(case["k"], torch.float32),
            _to(case["v"], torch.float32), feats, _to(case["weight"], torch.float32),
            _to(case["bias"], torch.float32), case["seqlens"].cuda(),
        )


def test_mask_forms_agree() -> None:
    """[B] lengths, a bool mask (True = pad) and a 0/-inf float mask agree."""
    case = cs.padded_case(3, 40, 12, 32, 16, True, seed=11)
    dtype = torch.bfloat16
    args = [_to(case[k], dtype) for k in ("q", "k", "v")]
    feats, w, bb = case["feats"].cuda(), _to(case["weight"], dtype), _to(case["bias"], dtype)
    seq = case["seqlens"].cuda()
    pad = torch.arange(40, device="cuda")[None, :] >= seq[:, None]
    fmask = torch.zeros(pad.shape, device="cuda").masked_fill(pad, float("-inf"))
    o1 = flash_spacetime_attention(*args, feats, w, bb, seq)
    o2 = flash_spacetime_attention(*args, feats, w, bb, key_padding_mask=pad)
    o3 = flash_spacetime_attention(*args, feats, w, bb, fmask)
    assert torch.equal(o1, o2) and torch.equal(o1, o3)
    bad = pad.clone()
    bad[0, 0] = True  # a padding token in front of valid ones
    with pytest.raises(ValueError, match="prefix"):
        flash_spacetime_attention(*args, feats, w, bb, key_padding_mask=bad)
    # Without validation the mask is taken as lengths with no device read-back.
    o4 = flash_spacetime_attention(*args, feats, w, bb, key_padding_mask=pad,
                                   validate_mask=False)
    assert torch.equal(o1, o4)


@pytest.mark.parametrize("layout", ["bhld", "blhd", "packed"])
@pytest.mark.parametrize("flags", FLAGS[:3])
@pytest.mark.parametrize("dtype", DTYPES)
def test_host_projection_matches_oracle(layout, flags, dtype) -> None:
    """Caller-supplied u = ((q scale) W).to(dtype) and w~ = (dO W).to(dtype),
    formed on the host in fp32 as upstream does (forward.py:279-286,
    backward.py:546-547) and passed through the C ABI: the results follow
    the float64 oracle (2x-eager rule) and stay within rounding of the
    in-kernel projection."""
    from flash_spacetime.ops import flash_spacetime_attention_varlen

    b, n, h, d, c = SHAPES[13]
    case = cs.padded_case(b, n, h, d, c, True, seed=_seed(31, *flags, len(layout)))
    ref64 = cs.eager_padded(case, flags, torch.float64, grad=True)
    eager = cs.eager_padded(case, flags, dtype, grad=True)
    vm = cs.valid_mask(case)
    lens = [int(x) for x in case["seqlens"]]
    pk = cs.packed_from_padded(case)

    def run(host):
        if layout == "packed":
            leaves = {k: _to(pk[k], dtype).requires_grad_(True) for k in ("q", "k", "v")}
        else:
            leaves = {k: _to(case[k], dtype) for k in ("q", "k", "v")}
            if layout == "blhd":
                leaves = {k: t.transpose(1, 2).contiguous() for k, t in leaves.items()}
            leaves = {k: t.requires_grad_(True) for k, t in leaves.items()}
        w = _to(case["weight"], torch.float32).requires_grad_(True)
        bb = _to(case["bias"], torch.float32).requires_grad_(True)
        if layout == "packed":
            out = flash_spacetime_attention_varlen(
                leaves["q"], leaves["k"], leaves["v"], pk["feats"].cuda(), w, bb,
                pk["cu"].cuda(), use_attn_bias=flags[0], use_activation_bias=flags[1],
                host_projection=host)
            out.backward(_to(pk["grad"], dtype))
            unpack = lambda t: _unpack(t, lens, n)  # noqa: E731
        else:
            out = flash_spacetime_attention(
                leaves["q"], leaves["k"], leaves["v"], case["feats"].cuda(), w, bb,
                case["seqlens"].cuda(), use_attn_bias=flags[0], use_activation_bias=flags[1],
                layout=layout, host_projection=host)
            g = _to(case["grad"], dtype) * vm.cuda()
            out.backward(g.transpose(1, 2) if layout == "blhd" else g)
            unpack = (lambda t: t.transpose(1, 2)) if layout == "blhd" else (lambda t: t)
        res = {"out": unpack(out.detach()).cpu()}
        for k in ("q", "k", "v"):
            res["d" + k] = unpack(leaves[k].grad).cpu()
        res["dW"], res["db"] = w.grad.cpu(), bb.grad.cpu()
        return res

    host, kern = run(True), run(False)
    atol = cs.atol_for(dtype, flags)
    for key in ("out", "dq", "dk", "dv"):
        kv, rv, ev = (cs.valid_values(t, case) for t in (host[key], ref64[key], eager[key]))
        cs.assert_2x_rule(kv, ev, rv, atol, f"host projection {key}", dtype,
                          reduction=key != "out")
        # The in-kernel projection rounds the same fp32 product once (W split
        # into hi + lo halves of the 16-bit type), so the two paths agree to
        # well inside the stated tolerance.
        diff = cs.normwise(kv, cs.valid_values(kern[key], case).double())
        assert diff <= (1e-2 if dtype != torch.float32 else 1e-5), f"{key}: host vs kernel {diff:.2e}"
    assert cs.normwise(host["dW"].double(), ref64["dW"]) <= (2e-2 if dtype != torch.float32
                                                             else 1e-3), "dW"
    if flags[1]:
        assert cs.normwise(host["db"].double(), ref64["db"]) <= (2e-2 if dtype != torch.float32
                                                                 else 1e-3), "db"
    else:  # the logit path's db vanishes analytically and is returned as zeros
        assert torch.count_nonzero(host["db"]) == 0


def _unpack(t, lens, length):
    """[T, H, D] packed rows back to [B, H, L, D] with zero padding."""
    out = torch.zeros(len(lens), t.shape[1], length, t.shape[2], dtype=t.dtype, device=t.device)
    s = 0
    for b, m in enumerate(lens):
        out[b, :, :m] = t[s:s + m].transpose(0, 1)
        s += m
    return out


def test_bad_shapes_raise() -> None:
    case = cs.padded_case(2, 9, 2, 32, 16, False, seed=3)
    dtype = torch.float32
    args = [_to(case[k], dtype) for k in ("q", "k", "v")]
    feats = case["feats"].cuda()
    with pytest.raises(ValueError):  # W must be [Dh, C]
        flash_spacetime_attention(*args, feats, _to(case["weight"].t(), dtype), None,
                                  case["seqlens"].cuda())
    with pytest.raises(ValueError):  # odd C
        flash_spacetime_attention(*args, feats, torch.zeros(32, 15, device="cuda"), None,
                                  case["seqlens"].cuda())


def test_grad_none_conventions() -> None:
    case = cs.padded_case(2, 9, 2, 16, 16, False, seed=4)
    for flags in FLAGS:
        kg = _kernel_grads(case, flags, torch.float32)
        used = flags[0] or flags[1]
        assert (kg["weight"] is not None) == used
        assert (kg["bias"] is not None) == used
        if flags == (True, False):
            assert torch.equal(kg["bias"], torch.zeros_like(kg["bias"]))


@pytest.mark.parametrize("heads,dim,channels", [(13, 32, 16), (25, 32, 16), (12, 48, 48),
                                                (12, 64, 64), (9, 64, 32)])
def test_uneven_head_groups(heads, dim, channels):
    """More heads than one CTA holds, split into groups of unequal size (the
    wide shapes hold 8 heads per CTA in the backward, 12 in the forward)."""
    case = cs.padded_case(2, 50, heads, dim, channels, True, seed=_seed(13, heads, dim))
    dtype = torch.bfloat16
    out, _ = _forward(case, (True, True), dtype)
    kg = _kernel_grads(case, (True, True), dtype)
    ref = cs.eager_padded(case, (True, True), torch.float64, grad=True)
    assert cs.normwise(cs.valid_values(out.cpu(), case), cs.valid_values(ref["out"], case)) <= 2e-2
    for key, rk in (("q", "dq"), ("k", "dk"), ("v", "dv")):
        assert cs.normwise(cs.valid_values(kg[key], case), cs.valid_values(ref[rk], case)) <= 2e-2, key
    for key, rk in (("weight", "dW"), ("bias", "db")):
        assert cs.normwise(kg[key], ref[rk]) <= 2e-2, key
