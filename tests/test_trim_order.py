"""The cloud trim's selection rule reproduces std::nth_element's permutation (CPU).

ObjCloud::add trims with std::nth_element and keeps the survivors in the order it leaves them;
the device trim computes libstdc++'s selection with parallel partitions.  The pairing rule those
partitions use is checked here, in tests/trim_order_check.cpp, against std::nth_element itself
(built with the compiler that builds the reference oracle) on clouds with heavy key ties.
"""
import os
import shutil
import subprocess
import tempfile

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


def test_partition_rule_matches_std_nth_element():
    cxx = shutil.which("g++")
    if cxx is None:
        pytest.skip("no C++ compiler")
    with tempfile.TemporaryDirectory() as d:
        exe = os.path.join(d, "toc")
        subprocess.run([cxx, "-O2", "-std=c++17", "-o", exe, os.path.join(HERE, "trim_order_check.cpp")], check=True)
        r = subprocess.run([exe, "1500"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.startswith("ok 1500 depth_limit_hit 0"), r.stdout
