"""The JSON line `bench.py --impl reference` prints (CPU, no GPU needed).

The reference arm times the fp32 restatement of the reference forward on a bounded crop
of the workload and must describe the same workload, metric and unit as the GPU arm, so
that the two lines can be compared directly; its `config` describes the CPU run itself
(one host process, fp32, no L2 flush).
"""
import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
KEYS = ["impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
        "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"]


def _reference_line(*extra):
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "0",
                        "--ref-crop", "16", *extra], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout
    return json.loads(lines[0])


def test_reference_line_carries_the_contract_keys():
    d = _reference_line()
    for k in KEYS:
        assert k in d, k
    assert d["impl"] == "reference"
    assert d["metric"] == json.loads((ROOT / "BASELINE.json").read_text())["metric"]
    assert d["unit"] == "Mpix/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["e2e"]["value"] == d["value"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    # the GPU arm's workload (one 512x512 HAT-S image), the crop only in the sample
    assert d["config"]["workload"].startswith("HAT-S x4, one 512x512 image on one GPU")
    assert d["config"]["parallelism"].startswith("one host process")
    assert d["config"]["l2"].startswith("n/a")
    assert "16x16 crop" in d["cpu_baseline"]["sample"]
    assert d["scaling"] == "strong"


def test_reference_line_follows_the_config():
    d = _reference_line("--config", "4")
    assert d["scaling"] == "weak"
    assert d["config"]["workload"].startswith("HAT-S x3, 4 333x500 image(s) per GPU")
    d = _reference_line("--config", "1", "--shard", "batch")
    assert d["scaling"] == "weak"
