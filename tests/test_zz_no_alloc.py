"""fst_forward_noalloc through the C ABI: same results as fst_forward.

fst_forward_noalloc serves callers that cannot allocate device memory (fixed
memory pools, real-time loops): it runs the forward with its scratch taken
from an array built into the library instead of a caller workspace. This test
calls both entry points through ctypes on the same inputs, twice in a row
(the built-in array keeps the previous call's contents), for a packed batch
(whose tile prefix lives in that scratch) and a padded one, and requires the
outputs and LSE to match the workspace-based entry point bitwise -- it is the
same kernel on the same inputs -- also for a padded batch with a valid row
count, whose tile list holds two prefixes. It also checks that an oversized batch is
rejected, that fp32 inputs (which need no scratch) are not limited by it, and,
with a second GPU, that the per-device lookup serves that device. This file is
named to be collected last.
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
    ref_out, ref_lse = torch.empty_like(q), torch.empty(pb.stat_shape(), device=q.device)
    a = _forward_args(pb, q, k, v, ref_out, ref_lse)
    nws = lib.fst_forward_workspace_size(ctypes.byref(a.prob))
    ws = torch.empty(max(nws, 1), dtype=torch.uint8, device=q.device)
    a.workspace, a.workspace_bytes = ws.data_ptr(), nws
    _lib.check(lib.fst_forward(ctypes.byref(a), _stream(q.device)), "fst_forward")
    results = []
    for _ in range(2):  # two calls in a row share the built-in scratch
        out, lse = torch.empty_like(q), torch.empty(pb.stat_shape(), device=q.device)
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


def test_noalloc_padded_valid_rows_matches_forward():
    # Host lengths give the problem its valid row count: the tile list and the
    # padding-row prefix then live in the built-in scratch.
    case = cs.padded_case(3, 70, 12, 32, 16, True, seed=407)
    q, k, v = (case[x].to("cuda", torch.bfloat16) for x in ("q", "k", "v"))
    pb = _Problem(q, case["feats"].cuda(), case["weight"].cuda(), case["bias"].cuda(),
                  case["seqlens"], None, None, True, True)
    assert 0 < pb.valid_rows < pb.rows
    (ref_out, ref_lse), results = _run_both(pb, q, k, v)
    for out, lse in results:
        assert torch.equal(out, ref_out)
        assert torch.equal(lse, ref_lse)


def _many_events(dtype, n):
    cu = torch.zeros(n + 1, dtype=torch.int32)
    cu[1:] = torch.arange(1, n + 1)
    q = torch.randn(n, 1, 32, generator=torch.Generator().manual_seed(3)).to("cuda", dtype)
    feats = torch.zeros(n, 4, device="cuda")
    w = torch.zeros(32, 16, device="cuda")
    pb = _Problem(q, feats, w, None, None, cu.cuda(), None, True, True)
    out, lse = torch.empty_like(q), torch.empty(pb.stat_shape(), device="cuda")
    return pb, q, out, lse


def test_noalloc_rejects_oversized_batch():
    # 16-bit inputs: the tile prefix of 70000 events does not fit the array.
    lib = _lib.load()
    pb, q, out, lse = _many_events(torch.bfloat16, 70000)
    a = _forward_args(pb, q, q, q, out, lse)
    rc = lib.fst_forward_noalloc(ctypes.byref(a), _stream(q.device))
    assert rc == _lib.FST_ERR_INVALID
    assert "scratch limit" in _lib.last_error()


def test_noalloc_fp32_needs_no_scratch():
    # fp32 inputs run kernels that take no scratch, so the event count is not
    # limited by the array: 70000 single pulses give out = v exactly.
    lib = _lib.load()
    pb, q, out, lse = _many_events(torch.float32, 70000)
    a = _forward_args(pb, q, q, q, out, lse)
    _lib.check(lib.fst_forward_noalloc(ctypes.byref(a), _stream(q.device)),
               "fst_forward_noalloc")
    torch.cuda.synchronize()
    assert torch.equal(out, q)


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs a second GPU")
def test_noalloc_second_device_matches_forward():
    # The array's address is looked up per device; a call on device 1 after
    # calls on device 0 must use device 1's copy.
    case = cs.packed_case([37, 120, 5, 260, 1], 12, 32, 16, seed=406)
    with torch.cuda.device(1):
        q, k, v = (case[x].to("cuda:1", torch.bfloat16) for x in ("q", "k", "v"))
        pb = _Problem(q, case["feats"].to("cuda:1"), case["weight"].to("cuda:1"),
                      case["bias"].to("cuda:1"), None, case["cu"].to("cuda:1"), None, True, True)
        (ref_out, ref_lse), results = _run_both(pb, q, k, v)
    for out, lse in results:
        assert torch.equal(out, ref_out)
        assert torch.equal(lse, ref_lse)
