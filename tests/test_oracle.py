"""Pin the CPU oracle (and the public spec module) to upstream's own outputs.

The fixtures in ``tests/golden/`` were produced by running the upstream
``spacetime_attention_reference`` (see ``tests/golden/make_golden.py``). The
oracle restates that code; in float64 it must reproduce the fixtures to
rounding level, and its per-event evaluation (used by every GPU parity test)
must agree on valid rows.
"""

import pytest
import torch

from golden_cases import case_names, load_case, load_freqs
from oracle import spacetime_oracle as orc

import flash_spacetime.reference as spec

CASES = case_names()


def _tol(dtype: torch.dtype) -> dict:
    return {"atol": 1e-12, "rtol": 1e-12} if dtype == torch.float64 else {"atol": 2e-5, "rtol": 2e-5}


def test_frequency_ladder_bitwise() -> None:
    for channels, ladder in load_freqs().items():
        assert torch.equal(orc.freq_ladder(channels), ladder)
        assert torch.equal(spec.sinusoidal_frequencies(channels, torch.device("cpu")), ladder)


def test_constants() -> None:
    assert orc.TIME_SCALE == spec.TIME_SCALE == 18.0
    assert orc.INPUT_SCALE == spec.SINEMB_INPUT_SCALE == 1024.0
    assert orc.CLIP == spec.SINEMB_CLIP == 4.0


@pytest.mark.parametrize("name", CASES)
@pytest.mark.parametrize("impl", ["oracle", "spec"])
def test_eager_matches_golden(name: str, impl: str) -> None:
    case = load_case(name)
    dt = case["dtype"]
    flags = case["flags"]
    seqlens = case["seqlens"]
    batch, heads, length, dim = case["q"].shape
    valid = spec.valid_row_mask(batch, length, seqlens)
    mask = spec.float_padding_mask(valid, torch.float32)
    leaves = [case[k].to(dt).clone().requires_grad_(True) for k in ("q", "k", "v", "weight", "bias")]
    feats = case["feats"].to(torch.float64 if dt == torch.float64 else torch.float32)
    fn = orc.eager_attention if impl == "oracle" else spec.spacetime_attention_reference
    out = fn(*leaves[:3], feats, leaves[3], leaves[4], key_padding_mask=mask,
             use_attn_bias=flags[0], use_activation_bias=flags[1])
    torch.testing.assert_close(out.detach(), case["out"], **_tol(dt))
    loss = (out * case["grad_w"].to(dt) * valid[:, None, :, None]).sum()
    loss.backward()
    for key, leaf in zip(("dq", "dk", "dv", "dW", "db"), leaves):
        ref = case[key]
        if ref is None:
            assert leaf.grad is None
        else:
            torch.testing.assert_close(leaf.grad, ref, **_tol(dt))
    if case.get("pair_features") is not None:
        rel = orc.pair_features(feats, case["weight"].to(dt), case["bias"].to(dt))
        torch.testing.assert_close(rel, case["pair_features"], **_tol(dt))
    torch.testing.assert_close(orc.pair_mask(mask), case["pair_mask"], atol=0, rtol=0)


@pytest.mark.parametrize("name", [n for n in CASES if "fp32" not in n])
def test_per_event_oracle_matches_golden(name: str) -> None:
    """The per-event fp64 oracle equals the batched upstream call on valid rows."""
    case = load_case(name)
    flags = case["flags"]
    seqlens = case["seqlens"]
    batch, heads, length, dim = case["q"].shape
    valid = spec.valid_row_mask(batch, length, seqlens)
    grad_out = case["grad_w"] * valid[:, None, :, None]
    res = orc.oracle_padded(
        case["q"], case["k"], case["v"], case["feats"], case["weight"], case["bias"],
        seqlens.tolist(), use_attn_bias=flags[0], use_activation_bias=flags[1],
        grad_out=grad_out,
    )
    vm = valid[:, None, :, None].expand_as(res["out"])
    torch.testing.assert_close(res["out"][vm], case["out"][vm], atol=1e-12, rtol=1e-12)
    for key in ("dq", "dk", "dv"):
        torch.testing.assert_close(res[key][vm], case[key][vm], atol=1e-11, rtol=1e-11)
    for key in ("dW", "db"):
        if case[key] is None:
            assert res[key] is None
        else:
            torch.testing.assert_close(res[key], case[key], atol=1e-11, rtol=1e-11)


def test_packed_oracle_matches_padded_oracle() -> None:
    case = load_case("tt_masked_d16")
    seqlens = case["seqlens"].tolist()
    batch, heads, length, dim = case["q"].shape
    pad = orc.oracle_padded(case["q"], case["k"], case["v"], case["feats"],
                            case["weight"], case["bias"], seqlens,
                            grad_out=case["grad_w"])

    def pack(t):
        return torch.cat([t[b, :, :n].transpose(0, 1) for b, n in enumerate(seqlens)], 0)

    feats_p = torch.cat([case["feats"][b, :n] for b, n in enumerate(seqlens)], 0)
    cu = [0]
    for n in seqlens:
        cu.append(cu[-1] + n)
    res = orc.oracle_packed(pack(case["q"]), pack(case["k"]), pack(case["v"]), feats_p,
                            case["weight"], case["bias"], cu, grad_out=pack(case["grad_w"]))
    torch.testing.assert_close(res["out"], pack(pad["out"]), atol=1e-13, rtol=1e-13)
    torch.testing.assert_close(res["dq"], pack(pad["dq"]), atol=1e-12, rtol=1e-12)
    torch.testing.assert_close(res["dW"], pad["dW"], atol=1e-12, rtol=1e-12)
    lse_p = torch.cat([pad["lse"][b, :, :n].t() for b, n in enumerate(seqlens)], 0)
    torch.testing.assert_close(res["lse"], lse_p, atol=1e-13, rtol=1e-13)


def test_lse_drops_row_constant() -> None:
    """The oracle LSE equals logsumexp of the full logits minus qt.b."""
    case = load_case("tt_full_d48")
    q, k, feats, w, b = (case[x] for x in ("q", "k", "feats", "weight", "bias"))
    dim = q.shape[-1]
    res = orc.oracle_padded(q, k, case["v"], feats, w, b, [q.shape[2]])
    qt = q * dim**-0.5
    full = qt @ k.transpose(-2, -1) + torch.einsum(
        "bhic,bijc->bhij", qt, orc.pair_features(feats, w, b))
    shift = (qt * b).sum(-1)
    torch.testing.assert_close(res["lse"], torch.logsumexp(full, -1) - shift, atol=1e-10, rtol=1e-10)


@pytest.mark.parametrize("flags", [(True, True), (True, False), (False, True)])
def test_row_and_column_subsets_match_full_oracle(flags):
    """event_rows / event_cols (the L=16384 checkers) against the full per-event oracle."""
    gen = torch.Generator().manual_seed(11)
    n, h, d, c = 57, 3, 16, 8
    q, k, v, g = (torch.randn(n, h, d, generator=gen, dtype=torch.float64) for _ in range(4))
    feats = torch.randn(n, 4, generator=gen, dtype=torch.float64)
    w = torch.randn(d, c, generator=gen, dtype=torch.float64) / c**0.5
    b = 0.1 * torch.randn(d, generator=gen, dtype=torch.float64)
    full = orc.oracle_packed(q, k, v, feats, w, b, [0, n], use_attn_bias=flags[0],
                             use_activation_bias=flags[1], grad_out=g)
    rows = torch.tensor([0, 5, 31, n - 1])
    sub = orc.event_rows(q, k, v, feats, w, b, rows, use_attn_bias=flags[0],
                         use_activation_bias=flags[1], grad_out=g[rows])
    for key in ("out", "lse", "dq"):
        torch.testing.assert_close(sub[key], full[key][rows], rtol=1e-11, atol=1e-12)
    off = full["out"] - (b if flags[1] else 0.0)
    delta = (g * off).sum(-1)
    torch.testing.assert_close(sub["delta"], delta[rows], rtol=1e-11, atol=1e-12)
    cols = torch.tensor([1, 2, 40, n - 1])
    cs_ = orc.event_cols(q, k, v, feats, w, cols, full["lse"], delta, g,
                         use_attn_bias=flags[0], use_activation_bias=flags[1])
    torch.testing.assert_close(cs_["dk"], full["dk"][cols], rtol=1e-10, atol=1e-11)
    torch.testing.assert_close(cs_["dv"], full["dv"][cols], rtol=1e-10, atol=1e-11)
