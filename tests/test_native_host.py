"""Builds and runs the native C++ test executable of the host engine (no Python in the loop)."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HOST = os.path.join(ROOT, "grappa_b200", "csrc", "host")


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_native_host_engine(tmp_path):
    exe = str(tmp_path / "test_host")
    srcs = [os.path.join(HOST, "tests", "test_host.cc")] + [os.path.join(HOST, f) for f in
                                                            ("graph_host.cc", "xborder.cc", "chunking.cc")]
    cmd = ["g++", "-O2", "-std=c++17", "-fopenmp", "-I" + os.path.join(ROOT, "grappa_b200", "csrc", "include"),
           "-I" + HOST] + srcs + ["-L/usr/lib/gcc/x86_64-linux-gnu/13", "-lgomp", "-o", exe]
    subprocess.run(cmd, check=True, timeout=300)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    assert "passed" in r.stdout
