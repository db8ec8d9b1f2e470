"""fst_forward_noalloc through the C ABI: same results as fst_forward.

fst_forward_noalloc serves callers that cannot allocate device memory (fixed
memory pools, real-time loops): it runs the forward with its scratch taken
from an array built into the library instead of a caller workspace. This test
calls both entry points through ctypes on the same inputs, twice in a row
(the built-in array keeps the previous call's contents), for a packed batch
(whose tile prefix lives in that scratch) and a padded one, and requires the
outputs and LSE to match the workspace-based entry point bitwise -- it is the
same kernel on the same inputs. It also checks that an oversized batch is
rejected. This file is named to be collected last.
"""

import ctypes

import pytest
import torch

import cases as cs

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from flash_spacetime import _lib
    from flash_spacetime.ops import _Problem, _ptr, _stream


def _forward_args(pb, q, k, v, out, lse):
    a = _lib.FstForwardArgs()
    a.prob = pb.c_struct()
    a.q, a.k, a.v, a.u = _ptr(q), _ptr(k), _ptr(v), None
    a.out, a.lse = _ptr(out), _ptr(lse)
    return a


def _run_both(pb, q, k, v):
    lib = _lib.load()
    ref_out, ref_lse = torch.empty_like(q), torch.empty(pb.stat_shape(), device="cuda")
    a = _forward_args(pb, q, k, v, ref_out, ref_lse)
    nws = lib.fst_forward_workspace_size(ctypes.byref(a.prob))
    ws = torch.empty(max(nws, 1), dtype=torch.uint8, device="cuda")
    a.workspace, a.workspace_bytes = ws.data_ptr(), nws
    _lib.check(lib.fst_forward(ctypes.byref(a), _stream(q.device)), "fst_forward")
    results = []
    for _ in range(2):  # two calls in a row share the built-in scratch
        out, lse = torch.empty_like(q), torch.empty(pb.stat_shape(), device="cuda")
        b = _forward_args(pb, q, k, v, out, lse)
        b.workspace, b.workspace_bytes = None, 0
        _lib.check(lib.fst_forward_noalloc(ctypes.byref(b), _stream(q.device)),
                   "fst_forward_noalloc")
        results.append((out, lse))
    torch.cuda.synchronize()
    return (ref_out, ref_lse), results


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_noalloc_packed_matches_forward(dtype):
    case = cs.packed_case([37, 120, 5, 260, 1], 12, 32, 16, seed=404)
    q, k, v = (case[x].to("cuda", dtype) for x in ("q", "k", "v"))
    pb = _Problem(q, case["feats"].cuda(), case["weight"].cuda(), case["bias"].cuda(), None,
                  case["cu"].cuda(), None, True, True)
    (ref_out, ref_lse), results = _run_both(pb, q, k, v)
    for out, lse in results:
        assert torch.equal(out, ref_out)
        assert torch.equal(lse, ref_lse)


def test_noalloc_padded_matches_forward():
    case = cs.padded_case(3, 70, 12, 32, 16, True, seed=405)
    q, k, v = (case[x].to("cuda", torch.bfloat16) for x in ("q", "k", "v"))
    pb = _Problem(q, case["feats"].cuda(), case["weight"].cuda(), case["bias"].cuda(),
                  case["seqlens"].cuda(), None, None, True, True)
    (ref_out, ref_lse), results = _run_both(pb, q, k, v)
    for out, lse in results:
        assert torch.equal(out, ref_out)
        assert torch.equal(lse, ref_lse)


def test_noalloc_rejects_oversized_batch():
    lib = _lib.load()
    lengths = [1] * 70000  # more events than the built-in scratch holds
    cu = torch.zeros(len(lengths) + 1, dtype=torch.int32)
    cu[1:] = torch.arange(1, len(lengths) + 1)
    q = torch.zeros(len(lengths), 1, 32, dtype=torch.bfloat16, device="cuda")
    feats = torch.zeros(len(lengths), 4, device="cuda")
    w = torch.zeros(32, 16, device="cuda")
    pb = _Problem(q, feats, w, None, None, cu.cuda(), None, True, True)
    out, lse = torch.empty_like(q), torch.empty(pb.stat_shape(), device="cuda")
    a = _forward_args(pb, q, q, q, out, lse)
    rc = lib.fst_forward_noalloc(ctypes.byref(a), _stream(q.device))
    assert rc == _lib.FST_ERR_INVALID
    assert "scratch limit" in _lib.last_error()
