"""CPU checks of the C-ABI boundary: the library loads, exports every entry
point declared in include/flash_spacetime.h, and the ctypes mirrors of the
structs have the C layout (checked against gcc on the header itself)."""

import ctypes
import os
import re
import shutil
import subprocess
import tempfile

import pytest

from flash_spacetime import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "flash_spacetime.h")


def _declared_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\w[\w\s\*]*?\b(fst_\w+)\s*\(", text, re.M)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    declared = _declared_functions()
    assert declared, "no declarations found in the header"
    assert set(declared) == set(_lib.EXPORTED)
    for name in declared:
        assert hasattr(lib, name), f"{name} declared in the header but not exported"
    assert lib.fst_abi_version() == _lib.ABI_VERSION


def test_invalid_problem_reports_error():
    lib = _lib.load()
    p = _lib.FstProblem()
    p.dtype, p.batch, p.heads, p.head_dim, p.channels = 1, 1, 1, 32, 15  # odd C
    p.feat_stride = 4
    a = _lib.FstForwardArgs()
    a.prob = p
    rc = lib.fst_forward(ctypes.byref(a), None)
    assert rc == _lib.FST_ERR_INVALID
    assert "even" in _lib.last_error()
    with pytest.raises(ValueError):
        _lib.check(rc, "fst_forward")


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_struct_layout_matches_header():
    structs = {
        "FstProblem": _lib.FstProblem,
        "FstForwardArgs": _lib.FstForwardArgs,
        "FstBackwardArgs": _lib.FstBackwardArgs,
    }
    lines = ["#include <stdio.h>", "#include <stddef.h>", '#include "flash_spacetime.h"',
             "int main(void) {"]
    for name, cls in structs.items():
        lines.append(f'printf("{name} %zu\\n", sizeof({name}));')
        for field, _ in cls._fields_:
            lines.append(f'printf("{name}.{field} %zu\\n", offsetof({name}, {field}));')
    lines += ["return 0;", "}"]
    with tempfile.TemporaryDirectory() as tmp:
        src, exe = os.path.join(tmp, "layout.c"), os.path.join(tmp, "layout")
        open(src, "w").write("\n".join(lines))
        subprocess.check_call(["gcc", "-I", os.path.dirname(HEADER), src, "-o", exe])
        out = subprocess.check_output([exe]).decode().split("\n")
    got = dict(line.split() for line in out if line.strip())
    for name, cls in structs.items():
        assert int(got[name]) == ctypes.sizeof(cls), name
        for field, _ in cls._fields_:
            assert int(got[f"{name}.{field}"]) == getattr(cls, field).offset, f"{name}.{field}"


@pytest.mark.parametrize("which", ["q", "feats", "stride"])
def test_misaligned_tensor_core_inputs_are_rejected(which):
    # The tensor-core path moves rows with 16-byte loads; a misaligned pointer
    # or feature stride must come back as an error before anything launches.
    # The pointers are never dereferenced: validation returns first.
    lib = _lib.load()
    p = _lib.FstProblem()
    p.dtype, p.packed, p.batch, p.heads, p.max_len = 1, 0, 1, 1, 16
    p.head_dim, p.channels, p.feat_stride, p.total_rows = 32, 16, 4, 16
    p.scale, p.use_attn_bias, p.use_act_bias = 0.25, 1, 1
    base = 1 << 20
    p.seqlens, p.feats, p.freqs, p.weight = base, base, base, base
    a = _lib.FstForwardArgs()
    a.prob = p
    a.q = a.k = a.v = a.out = a.lse = a.workspace = base
    a.workspace_bytes = 1 << 16
    if which == "q":
        a.q = base + 2
    elif which == "feats":
        a.prob.feats = base + 4
    else:
        a.prob.feat_stride = 5
    rc = lib.fst_forward(ctypes.byref(a), None)
    assert rc == _lib.FST_ERR_INVALID
    msg = _lib.last_error()
    assert ("16-byte" in msg) or ("multiple of 4" in msg), msg


def test_padded_batch_limit_is_reported():
    # More than 65535 events in a padded layout is refused before any launch
    # (the packed layout has no such limit).
    lib = _lib.load()
    p = _lib.FstProblem()
    p.dtype, p.packed, p.batch, p.heads, p.max_len = 1, 0, 70000, 1, 1
    p.head_dim, p.channels, p.feat_stride, p.total_rows = 32, 16, 4, 70000
    a = _lib.FstForwardArgs()
    a.prob = p
    rc = lib.fst_forward(ctypes.byref(a), None)
    assert rc == _lib.FST_ERR_UNSUPPORTED
    assert "65535" in _lib.last_error()


def test_upload_rows_rejects_bad_lengths_before_copying():
    # Every length is checked before the first copy is issued, so these calls
    # make no CUDA call at all (the pointers are never dereferenced).
    import torch
    lib = _lib.load()
    lens = torch.tensor([3, 9], dtype=torch.int32)
    rc = lib.fst_upload_rows(16, 16, lens.data_ptr(), 2, 1, 8, 4, None)
    assert rc == _lib.FST_ERR_INVALID
    assert "lens[1] = 9" in _lib.last_error()
    lens = torch.tensor([-1], dtype=torch.int32)
    assert lib.fst_upload_rows(16, 16, lens.data_ptr(), 1, 1, 8, 4, None) == _lib.FST_ERR_INVALID
    assert lib.fst_upload_rows(None, None, None, -1, 1, 1, 1, None) == _lib.FST_ERR_INVALID
    assert lib.fst_upload_rows(None, 16, lens.data_ptr(), 1, 1, 8, 4, None) == _lib.FST_ERR_INVALID
    assert "null" in _lib.last_error()
    assert lib.fst_upload_rows(None, None, None, 0, 1, 1, 1, None) == _lib.FST_OK


def test_upload_valid_rows_checks_arguments():
    import torch
    from flash_spacetime import ops
    src = torch.zeros(2, 3, 8, 4)
    with pytest.raises(ValueError, match="CPU tensor"):
        ops.upload_valid_rows(src.clone(), src, [1, 2])


def test_valid_rows_is_checked_and_sizes_the_workspace():
    # A negative valid_rows is refused before any launch. A padded problem
    # given valid_rows below B*L walks the device tile list: its workspace
    # holds the tile prefix and the padding-row prefix (2 * (B + 1) ints).
    lib = _lib.load()
    p = _lib.FstProblem()
    p.dtype, p.packed, p.batch, p.heads, p.max_len = 1, 0, 100, 12, 64
    p.head_dim, p.channels, p.feat_stride, p.total_rows = 32, 16, 4, 6400
    p.seqlens = p.feats = p.freqs = 256  # never dereferenced by these calls
    full = lib.fst_forward_workspace_size(ctypes.byref(p))
    p.valid_rows = 1000
    listed = lib.fst_forward_workspace_size(ctypes.byref(p))
    assert full == (101 * 4 + 15) // 16 * 16
    assert listed == (2 * 101 * 4 + 15) // 16 * 16
    p.valid_rows = 6400  # not below B*L: the full grid, no list
    assert lib.fst_forward_workspace_size(ctypes.byref(p)) == full
    p.valid_rows = -1
    a = _lib.FstForwardArgs()
    a.prob = p
    assert lib.fst_forward(ctypes.byref(a), None) == _lib.FST_ERR_INVALID
    assert "valid_rows" in _lib.last_error()


def test_mask_lengths_read_back_the_valid_row_count():
    import torch
    from flash_spacetime import ops
    lens = torch.tensor([5, 0, 8])
    mask = torch.arange(8)[None, :] >= lens[:, None]  # True = padding
    got, total = ops._mask_lengths(mask, True)
    assert got.tolist() == [5, 0, 8] and total == 13
    assert ops._mask_lengths(mask, False)[1] == 0  # unchecked: nothing read back
    floats = torch.zeros(3, 8).masked_fill(mask, float("-inf"))
    assert ops._mask_lengths(floats, True)[1] == 13
    mask[0, 1] = True  # a hole inside event 0
    with pytest.raises(ValueError, match="prefix"):
        ops._mask_lengths(mask, True)
    seq, hint = ops._padded_lengths(None, None, 3, 8, torch.device("cpu"), True, 20)
    assert hint == 20 and seq.tolist() == [8, 8, 8]
    with pytest.raises(ValueError, match="valid_rows"):
        ops._padded_lengths(lens, None, 3, 8, torch.device("cpu"), True, -2)


def test_longest_first_flag_is_checked():
    # The library ranks at most 1024 events itself, and only when no
    # event_order is given.
    lib = _lib.load()
    p = _lib.FstProblem()
    p.dtype, p.packed, p.batch, p.heads, p.max_len = 1, 0, 1025, 12, 64
    p.head_dim, p.channels, p.feat_stride, p.total_rows = 32, 16, 4, 1025 * 64
    p.seqlens = p.feats = p.freqs = 256  # never dereferenced by these calls
    p.flags = _lib.FST_FLAG_LONGEST_FIRST
    a = _lib.FstForwardArgs()
    a.prob = p
    assert lib.fst_forward(ctypes.byref(a), None) == _lib.FST_ERR_INVALID
    assert "1024" in _lib.last_error()
    a.prob.batch, a.prob.total_rows, a.prob.event_order = 8, 8 * 64, 256
    assert lib.fst_forward(ctypes.byref(a), None) == _lib.FST_ERR_INVALID
    assert "event_order" in _lib.last_error()
    # Accepted: its workspace holds the ranked order after the tile prefix.
    a.prob.event_order = None
    assert lib.fst_forward_workspace_size(ctypes.byref(a.prob)) == (9 * 4 + 8 * 4 + 15) // 16 * 16
    a.prob.flags = 4
    assert lib.fst_forward(ctypes.byref(a), None) == _lib.FST_ERR_INVALID


def test_sum_partials_checks_its_problem():
    # An invalid problem is refused (it would otherwise count no partials and
    # write zeros), and so are missing partials for a requested output.
    lib = _lib.load()
    p = _lib.FstProblem()
    p.dtype, p.batch, p.heads, p.head_dim, p.channels = 1, 1, 1, 32, 15  # odd C
    p.feat_stride = 4
    assert lib.fst_sum_partials(ctypes.byref(p), None, None, 256, 256, None) == \
        _lib.FST_ERR_INVALID
    p.channels, p.packed, p.max_len, p.total_rows = 16, 0, 64, 64
    p.seqlens = p.feats = p.freqs = 256  # never dereferenced by these calls
    assert lib.fst_dw_partial_count(ctypes.byref(p)) > 0
    assert lib.fst_sum_partials(ctypes.byref(p), None, None, 256, None, None) == \
        _lib.FST_ERR_INVALID
    assert "partials" in _lib.last_error()
    assert lib.fst_sum_partials(ctypes.byref(p), None, None, None, None, None) == _lib.FST_OK
