"""The tile-list index arithmetic of the 16-bit kernels, checked on the CPU.

``index_check.cu`` compiles the kernels' own ``list_tile``,
``padding_share`` and ``list_padded_role`` (fst_tc_common.cuh) for the host
and drives them over thousands of random padded batches as a launch would:
every padding row written exactly once and inside its event, every live
block computed once, and a too-small ``valid_rows`` caught (every valid row
NaN). A mistake there would be an out-of-range store on the GPU, so it is
checked here, without one.
"""

import os
import shutil
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.skipif(shutil.which("nvcc") is None, reason="needs nvcc")
def test_tile_list_index_math(tmp_path):
    exe = tmp_path / "index_check"
    subprocess.run(["nvcc", "-std=c++17", "-O1", "--expt-relaxed-constexpr",
                    "-gencode", "arch=compute_100a,code=sm_100a",
                    "-o", str(exe), os.path.join(HERE, "index_check.cu")],
                   check=True, capture_output=True, text=True, timeout=300)
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert run.returncode == 0, run.stdout + run.stderr
    assert run.stdout.startswith("ok:"), run.stdout
