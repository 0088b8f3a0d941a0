"""The C host code under sanitizers (no GPU), like the reference's ASan/TSan
builds (Makefile:161-176, 216-232): tests/sanitize_main.c drives the GGUF
writer and probe (with mutated files), the counted n-gram map and its NGC2
files (with mutated files), the serial and speculative drivers (n-gram and
MTP drafting, the context cap) over the toy engine of tests/fake_engine.c,
and the frame server over pipes -- built with AddressSanitizer +
UndefinedBehaviorSanitizer (leak checks on) -- and the seeded generator's
worker threads under ThreadSanitizer.  Any report fails the test.
"""
import os
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HOST = ROOT / "cwen_b200" / "host"
SRCS = [ROOT / "tests" / "sanitize_main.c", ROOT / "tests" / "fake_engine.c", HOST / "driver.c", HOST / "loader.c",
        HOST / "server.c", HOST / "synth.c"]


def _build(out, flags):
    cmd = ["gcc", "-O1", "-g", "-std=gnu11", "-fno-omit-frame-pointer", *flags, "-I" + str(ROOT / "include"),
           "-I" + str(HOST), *map(str, SRCS), "-o", str(out), "-lpthread", "-lm"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0 and "sanitize" in r.stderr:
        pytest.skip("sanitizer runtime not available: " + r.stderr.splitlines()[-1])
    assert r.returncode == 0, r.stderr


def test_host_code_under_asan_ubsan(tmp_path):
    exe = tmp_path / "host_asan"
    _build(exe, ["-fsanitize=address,undefined", "-fno-sanitize-recover=undefined"])
    env = {**os.environ, "ASAN_OPTIONS": "detect_leaks=1:abort_on_error=0:exitcode=23",
           "UBSAN_OPTIONS": "halt_on_error=1:print_stacktrace=1"}
    r = subprocess.run([str(exe), "host", str(tmp_path)], capture_output=True, text=True, env=env, timeout=600)
    assert r.returncode == 0, r.stderr[-4000:]
    assert "runtime error" not in r.stderr and "AddressSanitizer" not in r.stderr


def test_generator_threads_under_tsan(tmp_path):
    exe = tmp_path / "threads_tsan"
    _build(exe, ["-fsanitize=thread"])
    env = {**os.environ, "TSAN_OPTIONS": "halt_on_error=1:exitcode=66"}
    r = subprocess.run([str(exe), "threads", str(tmp_path)], capture_output=True, text=True, env=env, timeout=600)
    assert r.returncode == 0, r.stderr[-4000:]
    assert "ThreadSanitizer" not in r.stderr
