"""bench.py's command-line contract on the CPU: the reference arm prints one JSON line with the keys the driver
reads (its e2e moves no bytes between host and device), and our arm, which runs only on the GPU, fails loudly
without one instead of falling back to the CPU."""
from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import pytest
import torch

REPO = Path(__file__).resolve().parents[1]


def _run(*args, timeout=300):
    return subprocess.run([sys.executable, "bench.py", *args], cwd=REPO, capture_output=True, text=True,
                          timeout=timeout)


def test_reference_arm_prints_the_contract_line():
    r = _run("--impl", "reference", "--config", "config0", "--steps", "1", "--warmup", "1")
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [line for line in r.stdout.splitlines() if line.startswith("{")]
    assert len(lines) == 1, r.stdout[-2000:]
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] == "BSR train audio-sec/sec" and d["unit"] == "audio-s/s"
    assert d["value"] > 0 and d["higher_is_better"] is True
    assert d["n_gpus"] == 1 and d["steps"] == 1 and d["warmup"] == 1
    assert d["config"]["workload"] == "config0"
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"]
    assert cb["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the behaviour without a GPU")
def test_our_arm_fails_without_a_gpu():
    r = _run("--config", "config0", "--steps", "1", "--warmup", "1", timeout=180)
    assert r.returncode != 0
    assert not any(line.startswith("{") for line in r.stdout.splitlines())
