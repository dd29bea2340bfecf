"""The CPU oracle under AddressSanitizer and UndefinedBehaviorSanitizer:
tests/cpp/oracle_sanitize calls every function of oracle/hx_oracle.c on
exactly sized heap buffers over edge-case shapes (head_dim 2/64/128, MHA and
GQA groups, 1-300 positions, block boundaries, several rows and threads).
The parity claims rest on the oracle, so it must run clean."""
import os
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


def test_oracle_runs_clean_under_sanitizers():
    r = subprocess.run(["make", "-s", "-C", os.path.join(HERE, "cpp"), "oracle_sanitize"],
                       capture_output=True, text=True)
    if r.returncode != 0:
        pytest.skip("sanitizer build unavailable: " + r.stderr[-300:])
    env = dict(os.environ, ASAN_OPTIONS="detect_leaks=0:halt_on_error=1",
               UBSAN_OPTIONS="halt_on_error=1:print_stacktrace=1")
    r = subprocess.run([os.path.join(HERE, "cpp", "oracle_sanitize")], capture_output=True, text=True,
                       env=env, timeout=600)
    assert "AddressSanitizer" not in r.stderr and "runtime error" not in r.stderr, r.stderr[-4000:]
    assert r.returncode == 0 and r.stdout.startswith("ok"), r.stdout + r.stderr[-2000:]
