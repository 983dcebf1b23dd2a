"""Builds and runs the native C++ test executable of the host engine (no Python in the loop):
an optimised OpenMP build, an AddressSanitizer + UndefinedBehaviorSanitizer build with the
standard library's bounds assertions, and a ThreadSanitizer build of the batch prefetch
pipeline and the rest (without OpenMP, whose runtime the thread sanitizer cannot see into)."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HOST = os.path.join(ROOT, "grappa_b200", "csrc", "host")
SOURCES = [os.path.join(HOST, "tests", "test_host.cc")] + [
    os.path.join(HOST, f) for f in ("graph_host.cc", "xborder.cc", "chunking.cc", "mlpart.cc", "numa.cc")]

BUILDS = {
    "openmp": (["-O2", "-fopenmp"], ["-L/usr/lib/gcc/x86_64-linux-gnu/13", "-lgomp"], {}),
    "asan_ubsan": (["-O1", "-g", "-fopenmp", "-fsanitize=address,undefined", "-fno-sanitize-recover=undefined",
                    "-fno-omit-frame-pointer", "-D_GLIBCXX_ASSERTIONS"],
                   ["-fsanitize=address,undefined", "-L/usr/lib/gcc/x86_64-linux-gnu/13", "-lgomp"],
                   {"ASAN_OPTIONS": "detect_leaks=0:abort_on_error=0", "UBSAN_OPTIONS": "print_stacktrace=1"}),
    "tsan": (["-O1", "-g", "-fsanitize=thread", "-Wno-unknown-pragmas"], ["-fsanitize=thread"],
             {"TSAN_OPTIONS": "halt_on_error=1:second_deadlock_stack=1"}),
}


def _sanitizer_works(flag, tmp_path):
    src = tmp_path / "probe.cc"
    src.write_text("int main() { return 0; }\n")
    exe = str(tmp_path / "probe")
    r = subprocess.run(["g++", flag, str(src), "-o", exe], capture_output=True, timeout=120)
    return r.returncode == 0 and subprocess.run([exe], capture_output=True, timeout=60).returncode == 0


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
@pytest.mark.parametrize("build", list(BUILDS))
def test_native_host_engine(tmp_path, build):
    cflags, ldflags, env_extra = BUILDS[build]
    san = [f for f in cflags if f.startswith("-fsanitize=")]
    if san and not _sanitizer_works(san[0], tmp_path):
        pytest.skip(f"{san[0]} runtime not usable here")
    exe = str(tmp_path / f"test_host_{build}")
    cmd = (["g++", "-std=c++17"] + cflags + ["-I" + os.path.join(ROOT, "grappa_b200", "csrc", "include"),
                                            "-I" + HOST] + SOURCES + ldflags + ["-lpthread", "-o", exe])
    subprocess.run(cmd, check=True, timeout=600)
    env = dict(os.environ, **env_extra)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300, env=env)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "passed" in r.stdout
    for marker in ("runtime error:", "ERROR: AddressSanitizer", "WARNING: ThreadSanitizer"):
        assert marker not in r.stderr, r.stderr
