"""The benchmark's output contract, checked on the host: the reference arm (the CPU
restatement of the reference's loss, timed on the host cores) prints one JSON line with the
keys the line format requires, and the CUDA arm fails loudly without a GPU instead of
measuring a fallback."""
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]


def _run(*args, timeout=600):
    env = dict(os.environ)
    env.pop("RANK", None)
    env.pop("WORLD_SIZE", None)
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], capture_output=True, text=True,
                          timeout=timeout, cwd=str(ROOT), env=env)


def test_reference_arm_prints_one_contract_line():
    out = _run("--impl", "reference", "--steps", "3", "--warmup", "3")
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.strip().startswith("{")]
    assert len(lines) == 1, out.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] == "KL-GEMM fwd+bwd loss-rows/sec" and d["unit"] == "rows/s"
    assert d["higher_is_better"] is True and d["scaling"] in ("weak", "strong")
    assert d["n_gpus"] == 1 and d["steps"] == 3 and d["warmup"] == 3
    assert d["value"] > 0 and d["ms_per_step"] > 0
    assert d["vs_baseline"] is None
    assert d["config"]["workload"].startswith("c2:")
    assert (d["config"]["rows"], d["config"]["hidden"], d["config"]["vocab"]) == (16384, 576, 49152)
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert cb["unit"] == d["unit"] and cb["sample"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the behaviour without a GPU")
def test_cuda_arm_fails_without_a_gpu():
    out = _run("--steps", "3", "--warmup", "3", "--no-cpu-baseline", "--no-e2e", timeout=300)
    assert out.returncode != 0
    assert not [ln for ln in out.stdout.splitlines() if ln.strip().startswith("{") and '"value"' in ln]
