"""tests/abi_harness.c: a C host with no Python replays LayeredBackend.Generate's calls (prompt, token-by-token greedy,
guess-ahead with Truncate, a second turn over a shared prefix, the device greedy calls) through the C ABI alone.
Compiled against include/windlass.h and libwindlass_cuda.so on the CPU; run on a B200."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def build_harness(wl, out_dir):
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    lib_dir = os.path.dirname(wl.LIB_PATH)
    exe = os.path.join(str(out_dir), "abi_harness")
    r = subprocess.run([cc, "-O2", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"),
                        os.path.join(ROOT, "tests", "abi_harness.c"), "-L", lib_dir, "-lwindlass_cuda",
                        "-Wl,-rpath," + lib_dir, "-o", exe], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def test_harness_compiles_against_the_header_and_library(wl, tmp_path):
    build_harness(wl, tmp_path)


@pytest.mark.gpu
def test_harness_replays_generate_through_the_c_abi(wl, tmp_path):
    exe = build_harness(wl, tmp_path)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.startswith("ok"), r.stdout
