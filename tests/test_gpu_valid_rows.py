"""Padded batches with a host-known valid row count (FstProblem.valid_rows).

With the sum of the lengths known on the host, the 16-bit kernels launch
blocks for the valid rows only, taken from the device tile list as in the
packed layout, and the live blocks write the padding rows' zeros between
them. Nothing may change in the results:

1. out, LSE, dq, dk, dv, D and sigma are bit-identical to the launch over
   B x L rows (padding rows exactly 0 although the output buffers held NaN);
   dW / db, summed over a different number of per-CTA partials, agree to
   fp32 rounding (1e-5 of the largest entry);
2. the same through both padded layouts, the fused QKV buffer, a mask, host
   lengths and an explicit hint above the sum;
3. a hint too small for the grid to hold every live block makes every valid
   row NaN (the device-side check), never silently wrong rows;
4. a hint below lengths the host also knows is refused before any launch.
"""

import pytest
import torch

import cases as cs

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from flash_spacetime.ops import (
        flash_spacetime_attention,
        flash_spacetime_attention_qkv,
        flash_spacetime_backward,
        flash_spacetime_forward,
    )

NAN = float("nan")


def _to(t, dtype):
    return t.to(device="cuda", dtype=dtype)


def _poison_allocator(nbytes):
    # Leave NaN in the caching allocator's free blocks, so that outputs the op
    # allocates with torch.empty start out NaN and a padding row the kernels
    # failed to write would show.
    t = torch.full((nbytes // 4 + 1024,), NAN, device="cuda")
    del t


def _run(case, dtype, layout, seqlens, **kw):
    leaves = {k: _to(case[k], dtype) for k in ("q", "k", "v")}
    go = _to(case["grad"], dtype)
    if layout == "blhd":
        leaves = {k: t.transpose(1, 2).contiguous() for k, t in leaves.items()}
        go = go.transpose(1, 2).contiguous()
    leaves = {k: t.requires_grad_(True) for k, t in leaves.items()}
    w = _to(case["weight"], torch.float32).requires_grad_(True)
    b = _to(case["bias"], torch.float32).requires_grad_(True)
    _poison_allocator(4 * leaves["q"].numel() * leaves["q"].element_size())
    out = flash_spacetime_attention(leaves["q"], leaves["k"], leaves["v"], case["feats"].cuda(),
                                    w, b, seqlens, layout=layout, **kw)
    out.backward(go)
    torch.cuda.synchronize()
    return [out.detach(), leaves["q"].grad, leaves["k"].grad, leaves["v"].grad], [w.grad, b.grad]


def _check_same(ref, got):
    exact_ref, sums_ref = ref
    exact_got, sums_got = got
    for a, b in zip(exact_ref, exact_got):
        assert torch.equal(a, b)
    for a, b in zip(sums_ref, sums_got):
        # Sums of a different number of per-CTA partials: fp32 rounding of a
        # sum with cancellation, so the bound is relative to the largest entry.
        assert (b - a).abs().max() <= 1e-5 * a.abs().max()


@pytest.mark.parametrize("layout", ["bhld", "blhd"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("how", ["host_lengths", "exact", "above", "mask"])
def test_valid_rows_matches_full_grid(layout, dtype, how):
    case = cs.padded_case(4, 150, 12, 32, 16, True, seed=1201)
    case["seqlens"][1] = 0  # an empty event: all of its rows are padding
    lens = [int(n) for n in case["seqlens"]]
    ref = _run(case, dtype, layout, case["seqlens"].cuda())
    if how == "host_lengths":
        got = _run(case, dtype, layout, case["seqlens"])  # CPU tensor: the hint is its sum
    elif how == "mask":
        mask = torch.arange(150)[None, :] >= case["seqlens"][:, None]  # True = padding
        got = _run(case, dtype, layout, None, key_padding_mask=mask.cuda())
    else:
        extra = 0 if how == "exact" else 37
        got = _run(case, dtype, layout, case["seqlens"].cuda(), valid_rows=sum(lens) + extra)
    _check_same(ref, got)
    for t in got[0]:  # padding rows of out, dq, dk, dv are exactly 0
        rows = t if layout == "blhd" else t.transpose(1, 2)
        for i, n in enumerate(lens):
            assert torch.count_nonzero(rows[i, n:]) == 0


@pytest.mark.parametrize("dh, c", [(32, 16), (64, 64), (48, 48), (16, 16)])
def test_valid_rows_every_shape(dh, c):
    # Every (Dh, C) instantiation and both head-group splits (H = 12 and 20).
    heads = 20 if dh == 32 else 6
    case = cs.padded_case(3, 97, heads, dh, c, True, seed=1202 + dh + c)
    lens = [int(n) for n in case["seqlens"]]
    ref = _run(case, torch.bfloat16, "bhld", case["seqlens"].cuda())
    got = _run(case, torch.bfloat16, "bhld", case["seqlens"].cuda(), valid_rows=sum(lens))
    _check_same(ref, got)


def test_valid_rows_statistics_match():
    # LSE, D and sigma (the per-row statistics) of the padding rows are 0 as
    # well, through the forward-only and backward-only entry points.
    case = cs.padded_case(3, 120, 12, 32, 16, True, seed=1203)
    q, k, v, go = (_to(case[x], torch.bfloat16) for x in ("q", "k", "v", "grad"))
    w, b, feats = _to(case["weight"], torch.float32), _to(case["bias"], torch.float32), \
        case["feats"].cuda()
    res = []
    for seq in (case["seqlens"].cuda(), case["seqlens"]):  # device, then host lengths
        _poison_allocator(8 * q.numel() * 2)
        out, lse = flash_spacetime_forward(q, k, v, feats, w, b, seq)
        g = flash_spacetime_backward(q, k, v, feats, w, b, seq, out, lse, go)
        res.append([out, lse, g["dq"], g["dk"], g["dv"], g["delta"], g["sigma"]])
    for a, b_ in zip(*res):
        assert torch.equal(a, b_)


def test_valid_rows_fused_qkv():
    case = cs.padded_case(3, 70, 12, 32, 16, True, seed=1204)
    lens = [int(n) for n in case["seqlens"]]
    q, k, v, go = (_to(case[x], torch.bfloat16).transpose(1, 2).contiguous()
                   for x in ("q", "k", "v", "grad"))
    res = []
    for hint in (None, sum(lens)):
        w = _to(case["weight"], torch.float32).requires_grad_(True)
        b = _to(case["bias"], torch.float32).requires_grad_(True)
        qkv = torch.stack((q, k, v), dim=-3).requires_grad_(True)
        _poison_allocator(8 * qkv.numel() * 2)
        out = flash_spacetime_attention_qkv(qkv, case["feats"].cuda(), w, b,
                                            case["seqlens"].cuda(), valid_rows=hint)
        out.backward(go)
        res.append(([out.detach(), qkv.grad], [w.grad, b.grad]))
    _check_same(res[0], res[1])


def test_valid_rows_all_events_empty():
    # Every row is padding: no live block exists, and the one CTA that the
    # padding is shared over writes all of it.
    case = cs.padded_case(2, 40, 12, 32, 16, True, seed=1205)
    case["seqlens"][:] = 0
    exact, sums = _run(case, torch.bfloat16, "bhld", case["seqlens"].cuda(), valid_rows=1)
    for t in exact:
        assert torch.count_nonzero(t) == 0
    for t in sums:
        assert torch.count_nonzero(t) == 0


def test_valid_rows_too_small_gives_nan():
    # 3 events of 90 / 50 / 33 rows need 7 forward and 13 backward blocks;
    # valid_rows = 1 sizes the grids for 1 + B = 4. The kernels see it and
    # write NaN to every valid row (padding rows stay 0).
    case = cs.padded_case(3, 96, 12, 32, 16, True, seed=1206)
    case["seqlens"][:] = torch.tensor([90, 50, 33])
    lens = [90, 50, 33]
    exact, sums = _run(case, torch.bfloat16, "bhld", case["seqlens"].cuda(), valid_rows=1)
    for t in exact:
        for i, n in enumerate(lens):
            assert torch.isnan(t[i, :, :n]).all()
            assert torch.count_nonzero(t[i, :, n:]) == 0
    for t in sums:
        assert torch.isnan(t).all()


def test_valid_rows_below_host_lengths_is_refused():
    case = cs.padded_case(3, 60, 12, 32, 16, True, seed=1207)
    lens = [int(n) for n in case["seqlens"]]
    with pytest.raises(ValueError, match="valid_rows"):
        _run(case, torch.bfloat16, "bhld", case["seqlens"], valid_rows=sum(lens) - 1)
    with pytest.raises(ValueError, match="valid_rows"):
        _run(case, torch.bfloat16, "bhld", case["seqlens"].cuda(), valid_rows=-1)
