"""The checked library (libfa_b200_debug.so, FA_B200_DEBUG=1): every TMA copy
tests its innermost coordinate, the sign of a store's or reduce-add's
coordinates and its shared-memory alignment before it is issued. This GPU pool
does not allow compute-sanitizer, so this build stands in for its bounds
checking. The kernel paths run in a child process that loads that library
(one library per process) against the CPU oracle. None of the checks may fire,
no kernel may report a timed-out wait, and every case must meet the oracle."""
import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def test_checked_build_runs_every_path_cleanly(cuda):
    sys.path.insert(0, os.path.join(os.path.dirname(HERE), "flash-attention-p100_b200"))
    import _build
    _build.build(checked=True)          # up to date after __graft_entry__.build()
    env = dict(os.environ, FA_B200_DEBUG="1")
    res = subprocess.run([sys.executable, os.path.join(HERE, "checked_build_cases.py")],
                         env=env, capture_output=True, text=True, timeout=900)
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-4000:]
    out = json.loads(res.stdout.strip().splitlines()[-1])
    assert out["cases"] >= 20
    assert out["failures"] == [], "\n".join(out["failures"])
    assert out["tma_check"] == 0, f"TMA check word {out['tma_check']:#x}"
    assert out["device_error"] == 0
