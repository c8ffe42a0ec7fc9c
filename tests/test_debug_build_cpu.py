"""The bounds-checked debug build of the kernels (SHIFT_DEBUG_BOUNDS=1 adds
-DSHIFT_DEBUG_BOUNDS=1) keeps compiling for sm_100a: the MoE row kernels,
whose addresses come from routing data, are built with their index checks."""
import os
import shutil
import subprocess

import sysconfig
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.skipif(shutil.which("nvcc") is None, reason="needs nvcc")
def test_moe_kernels_compile_with_bounds_checks(tmp_path):
    from torch.utils.cpp_extension import include_paths
    inc = ["-I" + p for p in include_paths()] + ["-I" + sysconfig.get_paths()["include"],
                                                 "-I" + str(ROOT / "shift_b200" / "csrc")]
    cmd = ["nvcc", "-O1", "-gencode", "arch=compute_100a,code=sm_100a", "-std=c++17", "--expt-relaxed-constexpr",
           "-DSHIFT_DEBUG_BOUNDS=1", *inc, "-c", str(ROOT / "shift_b200" / "csrc" / "moe.cu"),
           "-o", str(tmp_path / "moe_debug.o")]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=dict(os.environ))
    assert r.returncode == 0, r.stderr[-3000:]
    assert (tmp_path / "moe_debug.o").stat().st_size > 0

