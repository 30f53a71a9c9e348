"""bench.py's reference arm on CPU: one JSON line with the contract's keys
(impl "reference", the CPU baseline it describes, an e2e block with no host
copies), and under a multi-rank launch only rank 0 prints."""

from __future__ import annotations

import json
import os
import subprocess
import sys

import pytest

from tests.conftest import REPO

pytestmark = pytest.mark.slow


def _run(extra_env=None):
    env = dict(os.environ)
    env.update(extra_env or {})
    return subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference", "--steps", "1",
                           "--warmup", "1", "--cpu-frames", "1"], cwd=REPO, env=env, capture_output=True, text=True,
                          timeout=600)


def test_reference_arm_prints_one_contract_line():
    res = _run()
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [ln for ln in res.stdout.splitlines() if ln.strip().startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["unit"] == "frames/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["cpu_baseline"]["value"] == d["value"]
    assert d["cpu_baseline"]["kind"] in ("port", "reference") and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0


def test_reference_arm_other_ranks_exit_quietly():
    res = _run({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert res.returncode == 0
    assert not any(ln.strip().startswith("{") for ln in res.stdout.splitlines())


def test_reference_arm_config4():
    """--impl reference --workload config4 samples three of the ragged requests."""
    env = dict(os.environ)
    res = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference", "--workload",
                          "config4", "--steps", "1", "--warmup", "0", "--cpu-frames", "1"], cwd=REPO, env=env,
                         capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [ln for ln in res.stdout.splitlines() if ln.strip().startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["value"] > 0 and d["config"]["workload"] == "config4"
    assert "config4 requests" in d["cpu_baseline"]["sample"]
