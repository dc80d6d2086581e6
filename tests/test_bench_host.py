"""The bench's output contract, on CPU.

* ``--impl reference`` (the CPU restatement of the reference's decode path) prints
  exactly one JSON line with the keys the result line must carry; under a launcher
  with several ranks, ranks other than 0 print nothing and exit 0.
* ``claim_stdout`` sends everything written to file descriptor 1, Python's and C's
  (NCCL prints its version banner there), to stderr, so stdout holds the result
  line alone.
"""

from __future__ import annotations

import json
import os
import subprocess
import sys
import textwrap
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def _run(args, env_extra=None, timeout=300):
    env = dict(os.environ)
    env.update(env_extra or {})
    return subprocess.run([sys.executable, *args], cwd=ROOT, env=env, capture_output=True, text=True,
                          timeout=timeout)


def test_reference_arm_prints_one_result_line():
    p = _run(["bench.py", "--impl", "reference", "--steps", "2", "--warmup", "1", "--batches", "1"])
    assert p.returncode == 0, p.stderr[-2000:]
    lines = p.stdout.splitlines()
    assert len(lines) == 1, p.stdout
    r = json.loads(lines[0])
    assert r["impl"] == "reference" and r["unit"] == "GB/s" and r["value"] > 0
    assert r["steps"] == 2 and r["warmup"] == 1 and r["higher_is_better"] is True
    assert r["cpu_baseline"]["kind"] == "port" and r["cpu_baseline"]["cores"] >= 1 and r["cpu_baseline"]["sample"]
    assert r["e2e"] == {"value": r["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert "workload" in r["config"]


def test_reference_arm_is_silent_on_other_ranks():
    p = _run(["bench.py", "--impl", "reference", "--steps", "1", "--warmup", "1", "--batches", "1"],
             {"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert p.returncode == 0, p.stderr[-2000:]
    assert p.stdout == ""


def test_claim_stdout_leaves_only_the_result_line():
    code = textwrap.dedent("""
        import ctypes, json, sys
        sys.path.insert(0, ".")
        import bench
        out = bench.claim_stdout()
        libc = ctypes.CDLL(None)
        libc.printf(b"C-level banner\\n")
        libc.fflush(None)
        print("python print")
        print(json.dumps({"metric": "x", "value": 1}), file=out, flush=True)
    """)
    p = _run(["-c", code], timeout=60)
    assert p.returncode == 0, p.stderr
    assert p.stdout.splitlines() == ['{"metric": "x", "value": 1}']
    assert "C-level banner" in p.stderr and "python print" in p.stderr
