"""The native data plane (C++ ColumnStore and PageAllocator) under AddressSanitizer + UndefinedBehaviorSanitizer
and under ThreadSanitizer (CPU only).

``csrc/native/selftest.cpp`` exercises the store's semantics (AND filter, per-task consumption, peeks,
re-delivery, clearing, error paths) and a multi-threaded producer / consumer run, plus the page allocator's
reference counts. The test builds it with each sanitizer and requires a clean exit with no report; a
toolchain without the sanitizer runtime skips.
"""

import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = [os.path.join(ROOT, "csrc", "native", f) for f in ("column_store.cpp", "selftest.cpp")]


def _build_and_run(tmp_path, flags, env_extra):
    cxx = shutil.which("g++") or shutil.which("c++")
    if cxx is None:
        pytest.skip("no C++ compiler")
    exe = str(tmp_path / "selftest")
    cmd = [cxx, "-std=c++17", "-O1", "-g", "-fno-omit-frame-pointer", "-pthread", *flags, *SRC, "-o", exe]
    b = subprocess.run(cmd, capture_output=True, text=True, timeout=300)
    if b.returncode != 0:
        pytest.skip(f"sanitizer build unavailable: {b.stderr.strip().splitlines()[-1:]}")
    env = dict(os.environ, **env_extra)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300, env=env)
    out = r.stdout + r.stderr
    if "ThreadSanitizer: unexpected memory mapping" in out or "FATAL: ThreadSanitizer" in out:
        pytest.skip("ThreadSanitizer cannot run under this kernel's address-space layout")
    return r.returncode, out


def test_native_store_asan_ubsan(tmp_path):
    code, out = _build_and_run(tmp_path, ["-fsanitize=address,undefined", "-fno-sanitize-recover=undefined"],
                               {"ASAN_OPTIONS": "detect_leaks=1:abort_on_error=0", "UBSAN_OPTIONS": "halt_on_error=1"})
    assert code == 0 and "selftest ok" in out, out[-4000:]
    assert "ERROR: AddressSanitizer" not in out and "runtime error" not in out, out[-4000:]


def test_native_store_tsan(tmp_path):
    code, out = _build_and_run(tmp_path, ["-fsanitize=thread"], {"TSAN_OPTIONS": "halt_on_error=1"})
    assert code == 0 and "selftest ok" in out, out[-4000:]
    assert "WARNING: ThreadSanitizer" not in out, out[-4000:]
