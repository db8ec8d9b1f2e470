"""GPU parity of the packed (varlen) layout: port of upstream tests/test_varlen.py.

1. packed == padded on the same events;
2. packed forward + backward against the float64 CPU oracle;
3. bitwise determinism;
4. uncapped lengths (thousands of pulses) inside a small memory ceiling;
plus the benchmark's head/channel widths and single-pulse events.
"""

import pytest
import torch

import cases as cs
from oracle import spacetime_oracle as orc

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from flash_spacetime.ops import (
        flash_spacetime_attention,
        flash_spacetime_attention_varlen,
    )

LENGTH_MIXES = [
    [7],
    [1, 1, 1],
    [17, 64, 3],
    [200, 33, 1, 128],
    [331, 800, 65],
]
FLAGS = [(True, True), (True, False), (False, True), (False, False)]
WIDTHS = [(4, 48, 48), (12, 32, 16)]  # (heads, head_dim, channels)


def _to(t, dtype):
    return t.to(device="cuda", dtype=dtype)


def _pad(case, key):
    lengths = case["lengths"]
    length = max(lengths)
    chunks = torch.split(case[key], lengths)
    if key == "feats":
        out = case[key].new_zeros(len(lengths), length, case[key].shape[-1])
        for i, c in enumerate(chunks):
            out[i, : c.shape[0]] = c
        return out
    out = case[key].new_zeros(len(lengths), length, case[key].shape[1], case[key].shape[2])
    for i, c in enumerate(chunks):
        out[i, : c.shape[0]] = c
    return out.permute(0, 2, 1, 3).contiguous()


def _unpad(padded, lengths):
    return torch.cat([padded[i, :, :n].permute(1, 0, 2) for i, n in enumerate(lengths)], 0)


@pytest.mark.parametrize("lengths", LENGTH_MIXES)
@pytest.mark.parametrize("flags", FLAGS)
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("width", WIDTHS)
def test_varlen_matches_padded(lengths, flags, dtype, width):
    heads, dim, ch = width
    case = cs.packed_case(lengths, heads, dim, ch, seed=31 + len(lengths))
    seqlens = torch.tensor(lengths, device="cuda")
    w, b = _to(case["weight"], dtype), _to(case["bias"], dtype)
    out_v = flash_spacetime_attention_varlen(
        _to(case["q"], dtype), _to(case["k"], dtype), _to(case["v"], dtype),
        case["feats"].cuda(), w, b, case["cu"].cuda(),
        use_attn_bias=flags[0], use_activation_bias=flags[1])
    out_p = flash_spacetime_attention(
        _to(_pad(case, "q"), dtype), _to(_pad(case, "k"), dtype), _to(_pad(case, "v"), dtype),
        _pad(case, "feats").cuda(), w, b, seqlens,
        use_attn_bias=flags[0], use_activation_bias=flags[1])
    # Same tiles, same arithmetic: the two layouts agree bitwise.
    assert torch.equal(out_v, _unpad(out_p, lengths))


@pytest.mark.parametrize("lengths", LENGTH_MIXES[2:])
@pytest.mark.parametrize("flags", FLAGS[:2])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("width", WIDTHS)
def test_varlen_matches_oracle(lengths, flags, dtype, width):
    heads, dim, ch = width
    case = cs.packed_case(lengths, heads, dim, ch, seed=77 + sum(lengths))
    leaves = {k: _to(case[k], dtype).requires_grad_(True) for k in ("q", "k", "v", "weight", "bias")}
    out = flash_spacetime_attention_varlen(
        leaves["q"], leaves["k"], leaves["v"], case["feats"].cuda(), leaves["weight"],
        leaves["bias"], case["cu"].cuda(), use_attn_bias=flags[0], use_activation_bias=flags[1])
    (out.double() * case["grad"].cuda()).sum().backward()
    ref = orc.oracle_packed(case["q"], case["k"], case["v"], case["feats"], case["weight"],
                            case["bias"], case["cu"].tolist(), use_attn_bias=flags[0],
                            use_activation_bias=flags[1], grad_out=case["grad"])
    names = (("q", "dq"), ("k", "dk"), ("v", "dv"), ("weight", "dW"), ("bias", "db"))
    if dtype == torch.float32:
        # upstream tests/test_varlen.py:213-225
        torch.testing.assert_close(out.detach().double().cpu(), ref["out"], atol=5e-3, rtol=1e-3)
        for key, rk in names:
            kg = leaves[key].grad
            assert kg is not None and ref[rk] is not None
            torch.testing.assert_close(kg.double().cpu(), ref[rk], atol=5e-2, rtol=5e-3,
                                       msg=lambda m, key=key: f"grad {key}: {m}")
        return
    # 16-bit inputs: upstream's 2x-eager rule against the oracle evaluated in
    # the same dtype, plus the normwise bound of the port.
    eager = orc.oracle_packed(case["q"], case["k"], case["v"], case["feats"], case["weight"],
                              case["bias"], case["cu"].tolist(), use_attn_bias=flags[0],
                              use_activation_bias=flags[1], grad_out=case["grad"], dtype=dtype)
    atol = cs.atol_for(dtype, flags)
    cs.assert_2x_rule(out.detach().cpu().flatten(), eager["out"].flatten(),
                      ref["out"].flatten(), atol, "forward", dtype)
    assert cs.normwise(out.detach().cpu(), ref["out"]) <= cs.NORMWISE[dtype]
    for key, rk in names:
        kg = leaves[key].grad
        assert kg is not None and ref[rk] is not None
        cs.assert_2x_rule(kg.cpu().flatten(), eager[rk].flatten(), ref[rk].flatten(), atol,
                          f"grad {key}", dtype, reduction=True)
        if ref[rk].norm() > 1e-8:  # db is analytically zero with the logit term alone
            assert cs.normwise(kg.cpu(), ref[rk]) <= cs.NORMWISE[dtype], key


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_varlen_deterministic(dtype):
    case = cs.packed_case([64, 17, 200], 16, 48, 48, seed=99)
    results = []
    for _ in range(2):
        q = _to(case["q"], dtype).requires_grad_(True)
        w = _to(case["weight"], dtype).requires_grad_(True)
        out = flash_spacetime_attention_varlen(
            q, _to(case["k"], dtype), _to(case["v"], dtype), case["feats"].cuda(), w,
            _to(case["bias"], dtype), case["cu"].cuda())
        out.float().sum().backward()
        results.append((out.detach().clone(), q.grad.clone(), w.grad.clone()))
    for a, b in zip(results[0], results[1]):
        assert torch.equal(a, b)


def test_uncapped_lengths_smoke():
    """Events far beyond any padded cap run within a tight memory budget."""
    lengths = [6000, 137, 1503]
    case = cs.packed_case(lengths, 16, 48, 48, seed=7)
    q = _to(case["q"], torch.bfloat16).requires_grad_(True)
    w = _to(case["weight"], torch.bfloat16).requires_grad_(True)
    k, v = _to(case["k"], torch.bfloat16), _to(case["v"], torch.bfloat16)
    feats, b, cu = case["feats"].cuda(), _to(case["bias"], torch.bfloat16), case["cu"].cuda()
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats()
    base = torch.cuda.memory_allocated()
    out = flash_spacetime_attention_varlen(q, k, v, feats, w, b, cu)
    out.float().sum().backward()
    torch.cuda.synchronize()
    peak = (torch.cuda.max_memory_allocated() - base) / 2**30
    assert torch.isfinite(out).all()
    assert q.grad is not None and torch.isfinite(q.grad).all()
    assert w.grad is not None and torch.isfinite(w.grad).all()
    assert peak < 0.5, f"packed fwd+bwd peak {peak:.2f} GiB"


def test_single_pulse_events():
    """Length-1 events attend only to themselves: out = v + R_ii (x = 0, exact).

    The 5-pulse event carries E-dependent outputs, held to upstream's fp32
    bound for them (tests/test_gpu.py:39-47); the single pulses are exact.
    """
    lengths = [1, 1, 5, 1]
    case = cs.packed_case(lengths, 12, 32, 16, seed=5)
    out = flash_spacetime_attention_varlen(
        _to(case["q"], torch.float32), _to(case["k"], torch.float32),
        _to(case["v"], torch.float32), case["feats"].cuda(), _to(case["weight"], torch.float32),
        _to(case["bias"], torch.float32), case["cu"].cuda())
    ref = orc.oracle_packed(case["q"], case["k"], case["v"], case["feats"], case["weight"],
                            case["bias"], case["cu"].tolist())
    out = out.double().cpu()
    single = torch.tensor([0, 1, 7])  # rows of the length-1 events
    torch.testing.assert_close(out[single], ref["out"][single], atol=1e-6, rtol=1e-6)
    torch.testing.assert_close(out, ref["out"], atol=5e-3, rtol=1e-3)


def _misaligned(t):
    # A view of the same values that starts one element into a larger buffer
    # (two if one element still lands on a 16-byte boundary), so its data
    # pointer is not 16-byte aligned.
    buf = torch.empty(t.numel() + 2, dtype=t.dtype, device=t.device)
    off = 1 if (buf.data_ptr() + t.element_size()) % 16 else 2
    view = buf[off:off + t.numel()].view(t.shape)
    view.copy_(t)
    return view


def test_misaligned_views_match_aligned():
    # Callers may hand over views that start mid-buffer; the public ops must
    # give the same results as for freshly allocated tensors.
    case = cs.packed_case([40, 130, 9], 12, 32, 16, seed=77)
    dtype = torch.bfloat16
    go = torch.randn(case["q"].shape, generator=torch.Generator().manual_seed(5)).to("cuda", dtype)
    results = []
    for shift in (0, 1):
        q, k, v = (_to(case[x], dtype) for x in ("q", "k", "v"))
        feats = case["feats"].cuda()
        if shift:
            q, k, v = (_misaligned(t) for t in (q, k, v))
            feats = _misaligned(feats)
            assert q.data_ptr() % 16 and feats.data_ptr() % 16
        q.requires_grad_(True)
        w = _to(case["weight"], torch.float32).requires_grad_(True)
        out = flash_spacetime_attention_varlen(q, k, v, feats, w, _to(case["bias"], torch.float32),
                                               case["cu"].cuda())
        out.backward(_misaligned(go) if shift else go)
        results.append((out.detach().clone(), q.grad.clone(), w.grad.clone()))
    for a, b in zip(results[0], results[1]):
        assert torch.equal(a, b)


def test_nested_tensor_adapter_matches_varlen():
    # Jagged NestedTensors share the varlen op's values/offsets form: same
    # values out, same gradients.
    from flash_spacetime.ops import flash_spacetime_attention_nested

    case = cs.packed_case([9, 130, 1, 57], 12, 32, 16, seed=123)
    dtype = torch.bfloat16
    cu = case["cu"].to(torch.int64)
    go = torch.randn(case["q"].shape, generator=torch.Generator().manual_seed(9)).to("cuda", dtype)
    res = []
    for nested in (False, True):
        q, k, v = (_to(case[x], dtype).requires_grad_(True) for x in ("q", "k", "v"))
        feats = case["feats"].cuda()
        w = _to(case["weight"], torch.float32).requires_grad_(True)
        b = _to(case["bias"], torch.float32)
        if nested:
            offs = cu.cuda()
            qn, kn, vn = (torch.nested.nested_tensor_from_jagged(t, offs) for t in (q, k, v))
            fn = torch.nested.nested_tensor_from_jagged(feats, offs)
            out = flash_spacetime_attention_nested(qn, kn, vn, fn, w, b)
            assert out.is_nested and torch.equal(out.offsets(), offs)
            out_v = out.values()
        else:
            out_v = flash_spacetime_attention_varlen(q, k, v, feats, w, b, case["cu"].cuda())
        out_v.backward(go)
        res.append((out_v.detach().clone(), q.grad.clone(), k.grad.clone(), w.grad.clone()))
    for a, b in zip(res[0], res[1]):
        assert torch.equal(a, b)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_blhd_layout_matches_bhld(dtype):
    # layout='blhd' reads [B, L, H, Dh] (a [B, L, H*Dh] projection per head)
    # and must give the transposed BHLD results, gradients included, bitwise.
    case = cs.padded_case(3, 70, 12, 32, 16, True, seed=321)
    seq = case["seqlens"].cuda()
    feats = case["feats"].cuda()
    go = torch.randn(case["q"].shape, generator=torch.Generator().manual_seed(3)).to("cuda", dtype)
    res = {}
    for layout in ("bhld", "blhd"):
        q, k, v = (_to(case[x], dtype) for x in ("q", "k", "v"))
        g = go
        if layout == "blhd":
            q, k, v, g = (t.transpose(1, 2).contiguous() for t in (q, k, v, g))
        q.requires_grad_(True)
        k.requires_grad_(True)
        w = _to(case["weight"], torch.float32).requires_grad_(True)
        b = _to(case["bias"], torch.float32).requires_grad_(True)
        out = flash_spacetime_attention(q, k, v, feats, w, b, seq, layout=layout)
        out.backward(g)
        tr = (lambda t: t.transpose(1, 2)) if layout == "blhd" else (lambda t: t)
        res[layout] = (tr(out.detach()), tr(q.grad), tr(k.grad), w.grad.clone(), b.grad.clone())
    for a, b_ in zip(res["bhld"], res["blhd"]):
        assert torch.equal(a, b_)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_empty_and_equal_length_events(dtype):
    # Zero-length events (no rows at all) and ties in length (the scheduling
    # order is a stable longest-first sort): packed and padded agree bitwise,
    # padding rows are 0, and the valid rows follow the float64 oracle.
    lengths = [40, 0, 17, 40, 0, 1, 17]
    case = cs.packed_case(lengths, 12, 32, 16, seed=55)
    seqlens = torch.tensor(lengths, device="cuda")
    w, b = _to(case["weight"], torch.float32), _to(case["bias"], torch.float32)
    out_v = flash_spacetime_attention_varlen(
        _to(case["q"], dtype), _to(case["k"], dtype), _to(case["v"], dtype),
        case["feats"].cuda(), w, b, case["cu"].cuda())
    out_p = flash_spacetime_attention(
        _to(_pad(case, "q"), dtype), _to(_pad(case, "k"), dtype), _to(_pad(case, "v"), dtype),
        _pad(case, "feats").cuda(), w, b, seqlens)
    assert torch.equal(out_v, _unpad(out_p, lengths))
    for i, n in enumerate(lengths):
        assert torch.count_nonzero(out_p[i, :, n:]) == 0
    ref = orc.oracle_packed(case["q"], case["k"], case["v"], case["feats"], case["weight"],
                            case["bias"], case["cu"].tolist())
    err = cs.normwise(out_v.double().cpu(), ref["out"])
    assert err <= cs.NORMWISE[dtype] if dtype != torch.float32 else err <= 1e-3


@pytest.mark.parametrize("packed", [False, True])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_fused_qkv_matches_separate(packed, dtype):
    # One [rows, 3, H, Dh] QKV buffer (a fused projection) read in place through
    # qkv_row_stride: output, the fused gradient and dW/db equal the separate
    # q/k/v path bit for bit.
    from flash_spacetime.ops import flash_spacetime_attention_qkv

    case = cs.padded_case(3, 70, 12, 32, 16, True, seed=808)
    lens = [int(n) for n in case["seqlens"]]
    pk = cs.packed_from_padded(case)
    if packed:
        q, k, v, go = (_to(pk[x], dtype) for x in ("q", "k", "v", "grad"))  # [T, H, D]
        feats = pk["feats"].cuda()
    else:
        q, k, v, go = (_to(case[x], dtype).transpose(1, 2).contiguous()
                       for x in ("q", "k", "v", "grad"))  # [B, L, H, D]
        feats = case["feats"].cuda()
    res = []
    for fused in (False, True):
        w = _to(case["weight"], torch.float32).requires_grad_(True)
        b = _to(case["bias"], torch.float32).requires_grad_(True)
        if fused:
            qkv = torch.stack((q, k, v), dim=-3).requires_grad_(True)  # [.., 3, H, D]
            if packed:
                out = flash_spacetime_attention_qkv(qkv, feats, w, b, cu_seqlens=pk["cu"].cuda())
            else:
                out = flash_spacetime_attention_qkv(qkv, feats, w, b, case["seqlens"].cuda())
            out.backward(go)
            grads = qkv.grad.unbind(-3)
        else:
            leaves = [t.clone().requires_grad_(True) for t in (q, k, v)]
            if packed:
                out = flash_spacetime_attention_varlen(*leaves, feats, w, b, pk["cu"].cuda())
            else:
                out = flash_spacetime_attention(*leaves, feats, w, b, case["seqlens"].cuda(),
                                                layout="blhd")
            out.backward(go)
            grads = [t.grad for t in leaves]
        res.append((out.detach(), *grads, w.grad.clone(), b.grad.clone()))
    for a, b_ in zip(res[0], res[1]):
        assert torch.equal(a, b_)
    if not packed:
        for i, n in enumerate(lens):  # padding rows of out and of the fused gradient are 0
            assert torch.count_nonzero(res[1][0][i, n:]) == 0


@pytest.mark.parametrize("packed", [False, True])
def test_share_sms_hint_is_bitwise_neutral(packed):
    # share_sms only selects kernel variants with a smaller register budget;
    # the arithmetic is the same, so every output and gradient is bit-identical.
    case = cs.padded_case(3, 90, 12, 32, 16, True, seed=919)
    pk = cs.packed_from_padded(case)
    dtype = torch.bfloat16
    res = []
    for share in (False, True):
        if packed:
            q, k, v = (_to(pk[x], dtype).requires_grad_(True) for x in ("q", "k", "v"))
            w = _to(case["weight"], torch.float32).requires_grad_(True)
            out = flash_spacetime_attention_varlen(q, k, v, pk["feats"].cuda(), w,
                                                   _to(case["bias"], torch.float32),
                                                   pk["cu"].cuda(), share_sms=share)
            out.backward(_to(pk["grad"], dtype))
        else:
            q, k, v = (_to(case[x], dtype).requires_grad_(True) for x in ("q", "k", "v"))
            w = _to(case["weight"], torch.float32).requires_grad_(True)
            out = flash_spacetime_attention(q, k, v, case["feats"].cuda(), w,
                                            _to(case["bias"], torch.float32),
                                            case["seqlens"].cuda(), share_sms=share)
            out.backward(_to(case["grad"], dtype))
        res.append((out.detach(), q.grad, k.grad, v.grad, w.grad))
    for a, b in zip(res[0], res[1]):
        assert torch.equal(a, b)
