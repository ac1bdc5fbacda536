"""The native host core (planner, generators) built with AddressSanitizer +
UndefinedBehaviorSanitizer and with ThreadSanitizer, and run on the CPU.
GPU-side sanitizers are not used on this pool; device kernels are checked
against CPU oracles instead."""

import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
CSRC = ROOT / "pcie_pool_b200" / "csrc"
SRC = [ROOT / "tests" / "native" / "host_core_test.cc", CSRC / "planner.cc", CSRC / "host_ops.cc"]


def _build_and_run(tmp_path, flags, name):
    cxx = shutil.which("g++")
    if cxx is None:
        pytest.skip("g++ not available")
    exe = tmp_path / name
    cmd = [cxx, "-std=c++17", "-O1", "-g", "-fno-omit-frame-pointer", *flags, f"-I{CSRC}",
           *map(str, SRC), "-o", str(exe), "-pthread"]
    b = subprocess.run(cmd, capture_output=True, text=True)
    if b.returncode != 0 and "sanitize" in b.stderr and "cannot find" in b.stderr:
        pytest.skip(f"sanitizer runtime unavailable: {b.stderr[-200:]}")
    assert b.returncode == 0, b.stderr[-4000:]
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300,
                       env={"ASAN_OPTIONS": "detect_leaks=1:abort_on_error=0", "TSAN_OPTIONS": "halt_on_error=1",
                            "UBSAN_OPTIONS": "halt_on_error=1:print_stacktrace=1"})
    assert r.returncode == 0, (r.stdout + r.stderr)[-4000:]
    assert "host_core_test: ok" in r.stdout


def test_host_core_asan_ubsan(tmp_path):
    _build_and_run(tmp_path, ["-fsanitize=address,undefined", "-fno-sanitize-recover=undefined"], "asan")


def test_host_core_tsan(tmp_path):
    _build_and_run(tmp_path, ["-fsanitize=thread"], "tsan")
