"""Host code of the library under AddressSanitizer and UndefinedBehaviorSanitizer, the host-side
stand-in for compute-sanitizer (closed on the GPU pool): the launch planner and the
invariant-divisor arithmetic the kernels index with (rational_kat_cu_b200/csrc/kat_plan.h),
built by g++ with -fsanitize=address,undefined -fno-sanitize-recover=all and run over a grid
of shapes, dtypes, vector widths and device sizes (tests/native/plan_check.cpp).  Any
out-of-bounds access, signed overflow or invalid shift aborts the program; the checks of the
plans' coverage invariants must all hold."""

import os
import shutil
import subprocess

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_planner_under_asan_and_ubsan(tmp_path):
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("g++ not available")
    exe = tmp_path / "plan_check"
    cmd = [gxx, "-std=c++17", "-O1", "-g", "-fsanitize=address,undefined",
           "-fno-sanitize-recover=all", "-I", os.path.join(REPO, "include"),
           "-I", os.path.join(REPO, "rational_kat_cu_b200", "csrc"),
           os.path.join(REPO, "tests", "native", "plan_check.cpp"), "-o", str(exe)]
    res = subprocess.run(cmd, capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stderr[-3000:]
    env = dict(os.environ, ASAN_OPTIONS="detect_leaks=0", UBSAN_OPTIONS="print_stacktrace=1")
    res = subprocess.run([str(exe)], capture_output=True, text=True, env=env, timeout=600)
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-3000:]
    assert res.stdout.startswith("ok "), res.stdout
    assert int(res.stdout.split()[1]) > 100000
