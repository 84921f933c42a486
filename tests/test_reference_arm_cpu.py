"""Host-side pieces of the reference arm that need no GPU: the watchdog that turns a probe
running past its limit into an ``unavailable`` line instead of a silent kill."""

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_watchdog_prints_unavailable_and_exits_cleanly():
    code = ("import sys, time; sys.path.insert(0, %r)\n"
            "from baseline import reference_arm as ra\n"
            "ra._stage('timed micro-batch')\n"
            "ra._watchdog(0.3, 0)\n"
            "time.sleep(30)\n"
            "print('not reached')\n") % ROOT
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=60)
    assert out.returncode == 0, out.stderr
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and "timed micro-batch" in line["unavailable"]
    assert "not reached" not in out.stdout


def test_watchdog_on_other_ranks_exits_silently():
    code = ("import sys, time; sys.path.insert(0, %r)\n"
            "from baseline import reference_arm as ra\n"
            "ra._watchdog(0.3, 1)\n"
            "time.sleep(30)\n") % ROOT
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=60)
    assert out.returncode == 0 and out.stdout.strip() == ""


def test_cancelled_watchdog_does_not_fire():
    sys.path.insert(0, ROOT)
    from baseline import reference_arm as ra

    t = ra._watchdog(0.2, 0)
    t.cancel()
    t.join(timeout=1)
    assert not t.is_alive()
