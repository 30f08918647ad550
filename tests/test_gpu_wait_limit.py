"""A bounded wait running out, on the GPU, without a fault: the conv kernel's
test stall mode makes every role of a launch reach a 20 ms wait limit; the
launch must return, the fault word must read FAULT_WAIT_TIMEOUT, and a normal
conv afterwards must be correct (tests/wait_limit_check.py, in a child process
so the switch and the limit stay out of this one)."""
import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def test_wait_limit_expires_and_context_stays_usable(cuda_device):
    env = {k: v for k, v in os.environ.items() if k != "SC_TC_TEST_STALL"}
    r = subprocess.run(["timeout", "-k", "10", "120", sys.executable, os.path.join(HERE, "wait_limit_check.py")],
                       capture_output=True, text=True, env=env)
    lines = [json.loads(l) for l in r.stdout.splitlines() if l.startswith("{")]
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert lines and lines[0]["ok"], lines
    assert lines[0]["stalled_launch_s"] < 10.0
