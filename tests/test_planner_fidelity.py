"""Planner fidelity against the reference planner (installed under baseline/_ref; skipped when
absent): on the same synthetic profiles, both AdaptiveStrategy plans are scored by the
reference's own evaluator. Ours must be valid wherever the reference's is, and its estimated
overhead may exceed the reference's only when it uses less peak memory."""

import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(not os.path.isdir(os.path.join(ROOT, "baseline", "_ref", "flextensor")),
                    reason="reference not installed in baseline/_ref")
def test_adaptive_plans_match_or_beat_reference():
    env = dict(os.environ, DISABLE_BEARTYPE="1")
    p = subprocess.run([sys.executable, os.path.join(ROOT, "tests", "helpers", "planner_compare.py")],
                       capture_output=True, text=True, timeout=900, env=env, cwd="/tmp")
    rows = [json.loads(l) for l in p.stdout.splitlines() if l.startswith("{")]
    assert rows, f"no comparison rows:\n{p.stderr[-3000:]}"
    for r in rows:
        ref, ours = r["ref"], r["ours"]
        if "error" in ref:
            continue  # the reference refused this case
        assert "error" not in ours, r
        if ref["valid"]:
            assert ours["valid"], r
        assert ours["overhead"] <= ref["overhead"] + 0.01 or ours["peak"] < ref["peak"], r
