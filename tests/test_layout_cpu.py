"""CPU check of the quad GEMV shared-memory layout.

``polar_pack_b200/csrc/quad_layout.h`` is plain C++ shared by the host
planner and the kernel; ``tests/native/quad_layout_check.cpp`` compiles it
with g++ and checks every variant / batch size / ring depth / base address
for blocks outside the window, overlaps and misalignment.
"""
import shutil
import subprocess
from pathlib import Path

import pytest

HERE = Path(__file__).resolve().parent


@pytest.mark.skipif(shutil.which("g++") is None, reason="g++ not available")
def test_quad_layout_blocks_disjoint_and_aligned(tmp_path):
    exe = tmp_path / "quad_layout_check"
    subprocess.run(["g++", "-O1", "-std=c++17", "-o", str(exe), str(HERE / "native" / "quad_layout_check.cpp")],
                   check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stdout + out.stderr
    assert "OK" in out.stdout
    # batch-1 file-layout kernel (16 warps): two ring slots per warp with the
    # tables on a 64 KiB boundary (direct gathers)
    assert "nk1 M=1 stages=2 direct=1" in out.stdout
    assert "nk1plug M=1 stages=2 direct=1" in out.stdout  # fused plug slots keep the batch-1 layout
