"""Host runtime under ThreadSanitizer: the worker pool and the AdamW range
kernel, compiled with -fsanitize=thread into a standalone driver
(csrc/host/tests/race_driver.cpp); a reported race fails the test."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HOST = os.path.join(ROOT, "test1_b200", "csrc", "host")


@pytest.mark.skipif(shutil.which("g++") is None, reason="no C++ compiler")
def test_host_runtime_has_no_data_races(tmp_path):
    exe = tmp_path / "race_driver"
    cmd = ["g++", "-std=c++17", "-O1", "-g", "-fsanitize=thread", "-pthread",
           os.path.join(HOST, "tests", "race_driver.cpp"), os.path.join(HOST, "thread_pool.cpp"),
           os.path.join(HOST, "host_kernels_scalar.cpp"), "-o", str(exe)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0 and "tsan" in (r.stderr or "").lower():
        pytest.skip("ThreadSanitizer runtime unavailable: " + r.stderr[-200:])
    assert r.returncode == 0, r.stderr[-2000:]
    env = dict(os.environ, TSAN_OPTIONS="halt_on_error=1 exitcode=66")
    r = subprocess.run([str(exe)], capture_output=True, text=True, env=env, timeout=600)
    assert "ThreadSanitizer" not in r.stderr, r.stderr[-4000:]
    assert r.returncode == 0, (r.stdout, r.stderr[-2000:])
    assert "race_driver: ok" in r.stdout
