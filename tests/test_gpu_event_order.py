"""Longest-first event order ranked by the library (FST_FLAG_LONGEST_FIRST).

Batches of up to 1024 events leave event_order NULL and let the library rank
the lengths inside its tile-prefix kernel. The ranking must be the stable
longest-first order that torch.argsort gives: with it, every output,
gradient and dW / db partial sum is bit-identical to a call that passes that
order explicitly -- through the padded grid, the padded tile list
(valid_rows) and the packed layout, with many tied lengths.
"""

import pytest
import torch

import cases as cs

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from flash_spacetime import _lib
    from flash_spacetime.ops import _Problem, fused_backward, fused_forward


def _run(case, layout, explicit, valid_rows=0):
    dtype = torch.bfloat16
    if layout == "packed":
        pk = cs.packed_from_padded(case)
        q, k, v, go = (pk[x].to("cuda", dtype) for x in ("q", "k", "v", "grad"))
        pb = _Problem(q, pk["feats"].cuda(), case["weight"].cuda().float(),
                      case["bias"].cuda().float(), None, pk["cu"].cuda(), None, True, True)
        lens = pk["cu"][1:] - pk["cu"][:-1]
    else:
        q, k, v, go = (case[x].to("cuda", dtype) for x in ("q", "k", "v", "grad"))
        pb = _Problem(q, case["feats"].cuda(), case["weight"].cuda().float(),
                      case["bias"].cuda().float(), case["seqlens"].cuda(), None, None, True,
                      True, valid_rows=valid_rows)
        lens = case["seqlens"]
    assert pb.order is None  # small batch: the library ranks the events
    if explicit:
        pb.order = torch.argsort(lens.cuda(), descending=True, stable=True).to(torch.int32)
    assert (pb.c_struct().flags & _lib.FST_FLAG_LONGEST_FIRST) == (0 if explicit else 2)
    out, lse = fused_forward(pb, q, k, v)
    g = fused_backward(pb, q, k, v, out, lse, go)
    return [out, lse, g["dq"], g["dk"], g["dv"], g["dW"], g["db"], g["delta"], g["sigma"]]


@pytest.mark.parametrize("layout, hinted", [("bhld", False), ("bhld", True), ("packed", False)])
def test_library_order_matches_explicit_argsort(layout, hinted):
    case = cs.padded_case(9, 80, 12, 32, 16, True, seed=1301)
    # Ties on purpose: the order among equal lengths must be the index order.
    case["seqlens"][:] = torch.tensor([40, 80, 40, 17, 80, 1, 40, 17, 64])
    hint = int(case["seqlens"].sum()) if hinted else 0
    a = _run(case, layout, explicit=False, valid_rows=hint)
    b = _run(case, layout, explicit=True, valid_rows=hint)
    for x, y in zip(a, b):
        assert torch.equal(x, y)
