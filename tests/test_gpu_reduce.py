"""fst_sum_partials: the fixed-order device sums of the backward's dW / db
partials (upstream forms dW and db on the host side, backward.py:607-622).

The sums must match a float64 sum of the same partials to fp32 rounding, be
bitwise reproducible, honour NULL outputs, and give zeros when there are no
partials. The end-to-end gradients through them are covered by the parity
tests against the float64 oracle.
"""

import ctypes

import pytest
import torch

import cases as cs

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from flash_spacetime import _lib
    from flash_spacetime.ops import _Problem, _ptr, _stream


def _problem(dim, channels, lens, heads=12):
    case = cs.padded_case(len(lens), max(lens), heads, dim, channels, True, seed=77)
    case["seqlens"][:] = torch.tensor(lens)
    q = case["q"].to("cuda", torch.bfloat16)
    return _Problem(q, case["feats"].cuda(), case["weight"].cuda(), case["bias"].cuda(),
                    case["seqlens"].cuda(), None, None, True, True)


def _sum(pb, dwp, dbp, want_w=True, want_b=True):
    lib = _lib.load()
    prob = pb.c_struct()
    dw = torch.full((pb.dim, pb.channels), float("nan"), device="cuda") if want_w else None
    db = torch.full((pb.dim,), float("nan"), device="cuda") if want_b else None
    _lib.check(lib.fst_sum_partials(ctypes.byref(prob), _ptr(dwp), _ptr(dbp), _ptr(dw), _ptr(db),
                                    _stream(pb.device)), "fst_sum_partials")
    torch.cuda.synchronize()
    return dw, db


@pytest.mark.parametrize("dim, channels", [(32, 16), (64, 64), (48, 48), (16, 16)])
def test_sums_match_float64(dim, channels):
    pb = _problem(dim, channels, [700, 33, 1, 256, 90])
    lib = _lib.load()
    n = int(lib.fst_dw_partial_count(ctypes.byref(pb.c_struct())))
    assert n > 0
    gen = torch.Generator(device="cuda").manual_seed(5)
    dwp = torch.randn(n, dim, channels, device="cuda", generator=gen)
    dbp = torch.randn(n, dim, device="cuda", generator=gen)
    dw, db = _sum(pb, dwp, dbp)
    ref_w, ref_b = dwp.double().sum(0), dbp.double().sum(0)
    scale_w, scale_b = dwp.double().abs().sum(0), dbp.double().abs().sum(0)
    assert ((dw.double() - ref_w).abs() <= 1e-6 * scale_w).all()
    assert ((db.double() - ref_b).abs() <= 1e-6 * scale_b).all()
    dw2, db2 = _sum(pb, dwp, dbp)  # bitwise reproducible
    assert torch.equal(dw, dw2) and torch.equal(db, db2)


def test_null_outputs_are_skipped():
    pb = _problem(32, 16, [120, 40])
    lib = _lib.load()
    n = int(lib.fst_dw_partial_count(ctypes.byref(pb.c_struct())))
    dwp = torch.ones(n, 32, 16, device="cuda")
    dbp = torch.ones(n, 32, device="cuda")
    dw, db = _sum(pb, dwp, None, want_b=False)
    assert db is None and torch.equal(dw, torch.full_like(dw, float(n)))
    dw, db = _sum(pb, None, dbp, want_w=False)
    assert dw is None and torch.equal(db, torch.full_like(db, float(n)))


def test_no_partials_give_zeros():
    lib = _lib.load()
    p = _lib.FstProblem()
    p.dtype, p.packed, p.batch, p.heads, p.max_len = 1, 0, 0, 12, 64
    p.head_dim, p.channels, p.feat_stride, p.total_rows = 32, 16, 4, 0
    assert lib.fst_dw_partial_count(ctypes.byref(p)) == 0
    dw = torch.full((32, 16), float("nan"), device="cuda")
    db = torch.full((32,), float("nan"), device="cuda")
    _lib.check(lib.fst_sum_partials(ctypes.byref(p), None, None, _ptr(dw), _ptr(db),
                                    _stream(dw.device)), "fst_sum_partials")
    torch.cuda.synchronize()
    assert torch.count_nonzero(dw) == 0 and torch.count_nonzero(db) == 0
