"""Padding rows of a padded batch are never read, and ``upload_valid_rows``
(``fst_upload_rows``) ships only the valid rows of a host batch.

1. NaN in every padding row of q, k, v, feats and grad_out changes no output
   or gradient bit (forward and backward, all three dtypes, both layouts);
2. the upload copies exactly the valid rows and leaves the padding rows of the
   destination as they were;
3. attention on uploaded tensors (padding rows NaN) equals attention on full
   copies, bit for bit.
"""

import pytest
import torch

import cases as cs

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from flash_spacetime.ops import flash_spacetime_attention, upload_valid_rows

LENGTHS = [40, 1, 17, 64, 0, 23]
SHAPES = [(torch.bfloat16, 12, 32, 16), (torch.float16, 4, 48, 48), (torch.float32, 3, 16, 8)]


def _host_batch(dtype, heads, dim, channels, lengths, seed):
    length = max(lengths)
    case = cs.padded_case(len(lengths), length, heads, dim, channels, masked=False, seed=seed)
    h = {k: case[k].to(dtype) for k in ("q", "k", "v", "grad")}
    h["feats"] = case["feats"][..., :4].float().contiguous()
    h["weight"] = case["weight"].float()
    h["bias"] = case["bias"].float()
    return h


def _poison(h, lengths, layout):
    """A copy of h with every padding row set to NaN."""
    p = {k: t.clone() for k, t in h.items()}
    for b, n in enumerate(lengths):
        for key in ("q", "k", "v", "grad"):
            if layout == "bhld":
                p[key][b, :, n:] = float("nan")
            else:
                p[key][b, n:] = float("nan")
        p["feats"][b, n:] = float("nan")
    return p


def _run(h, seqlens, layout):
    lv = {k: h[k].detach().clone().requires_grad_(True) for k in ("q", "k", "v", "weight", "bias")}
    out = flash_spacetime_attention(lv["q"], lv["k"], lv["v"], h["feats"], lv["weight"],
                                    lv["bias"], seqlens, layout=layout)
    out.backward(h["grad"])
    return [out.detach()] + [lv[k].grad for k in ("q", "k", "v", "weight", "bias")]


def _to_blhd(h):
    g = dict(h)
    for key in ("q", "k", "v", "grad"):
        g[key] = h[key].transpose(1, 2).contiguous()
    return g


@pytest.mark.parametrize("layout", ["bhld", "blhd"])
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: f"{s[0]}-{s[1]}x{s[2]}x{s[3]}")
def test_padding_rows_are_never_read(shape, layout):
    dtype, heads, dim, channels = shape
    h = _host_batch(dtype, heads, dim, channels, LENGTHS, seed=81)
    if layout == "blhd":
        h = _to_blhd(h)
    seqlens = torch.tensor(LENGTHS, device="cuda")
    clean = _run({k: t.cuda() for k, t in h.items()}, seqlens, layout)
    dirty = _run({k: t.cuda() for k, t in _poison(h, LENGTHS, layout).items()}, seqlens, layout)
    for a, b in zip(clean, dirty):
        assert torch.equal(a, b)


@pytest.mark.parametrize("pinned", [True, False], ids=["gather-kernel", "pageable-2d-copies"])
@pytest.mark.parametrize("layout", ["bhld", "blhd"])
def test_upload_valid_rows_copies_only_valid_rows(layout, pinned):
    h = _host_batch(torch.bfloat16, 12, 32, 16, LENGTHS, seed=82)
    if layout == "blhd":
        h = _to_blhd(h)
    for key in ("q", "feats"):
        src = h[key].pin_memory() if pinned else h[key]
        dst = torch.full_like(src, float("nan"), device="cuda")
        upload_valid_rows(dst, src, LENGTHS, layout=layout if key == "q" else "blhd")
        torch.cuda.synchronize()
        got = dst.cpu()
        for b, n in enumerate(LENGTHS):
            if key == "q" and layout == "bhld":
                valid, pad = got[b, :, :n], got[b, :, n:]
                ref = src[b, :, :n]
            else:
                valid, pad = got[b, :n], got[b, n:]
                ref = src[b, :n]
            assert torch.equal(valid, ref)
            assert bool(torch.isnan(pad.float()).all())


def test_attention_on_uploaded_rows_matches_full_copy():
    h = _host_batch(torch.bfloat16, 12, 32, 16, LENGTHS, seed=83)
    seqlens = torch.tensor(LENGTHS, device="cuda")
    full = _run({k: t.cuda() for k, t in h.items()}, seqlens, "bhld")
    up = {}
    for k, t in h.items():
        if k in ("weight", "bias"):
            up[k] = t.cuda()
            continue
        src = t.pin_memory()
        dst = torch.full_like(src, float("nan"), device="cuda")
        up[k] = upload_valid_rows(dst, src, LENGTHS, layout="bhld" if k != "feats" else "blhd")
    got = _run(up, seqlens, "bhld")
    for a, b in zip(full, got):
        assert torch.equal(a, b)


def test_upload_rejects_bad_lengths():
    src = torch.zeros(2, 3, 8, 4).pin_memory()
    dst = torch.zeros(2, 3, 8, 4, device="cuda")
    with pytest.raises(ValueError, match="outside"):
        upload_valid_rows(dst, src, [3, 9])
    with pytest.raises(ValueError, match="does not match"):
        upload_valid_rows(dst[:1], src, [3, 4])


@pytest.mark.parametrize("shape", [(1000, 2, 6, 8), (7, 3, 5, 5)], ids=["two-launches", "20-byte-rows"])
def test_upload_many_events_and_odd_rows(shape):
    # More events than one gather launch carries (960), and rows that are not
    # a multiple of 16 bytes (the 2D-copy path), both from pinned memory.
    gen = torch.Generator().manual_seed(84)
    dtype = torch.bfloat16 if shape[-1] == 8 else torch.float32
    src = torch.randn(shape, generator=gen).to(dtype).pin_memory()
    lens = torch.randint(0, shape[2] + 1, (shape[0],), generator=gen).tolist()
    dst = torch.full_like(src, float("nan"), device="cuda")
    upload_valid_rows(dst, src, lens)
    got = dst.cpu()
    for b, n in enumerate(lens):
        assert torch.equal(got[b, :, :n], src[b, :, :n])
        assert bool(torch.isnan(got[b, :, n:].float()).all())
