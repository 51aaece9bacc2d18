"""bench.py's output contract, checked on the host: the reference arm runs the
CPU oracle port, so its JSON line can be produced here; it must carry the
keys the contract names and describe the same workload as the GPU arm (the
driver compares the two `config` objects)."""
import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402


def _reference_line(*args):
    res = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", *args],
                         capture_output=True, text=True, timeout=600, cwd=str(ROOT))
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [ln for ln in res.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, res.stdout
    return json.loads(lines[0])


@pytest.mark.parametrize("config", ["1", "5"])
def test_reference_arm_line(config):
    d = _reference_line("--config", config, "--steps", "1", "--warmup", "0")
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["n_gpus"] == 1 and d["steps"] == 1
    assert d["value"] > 0 and d["higher_is_better"] is True
    cfg = bench.CONFIGS[config]
    assert (d["metric"], d["unit"]) == bench.metric_of(cfg)
    # the same workload description the GPU arm prints
    assert d["config"] == bench.config_dict(cfg, 1, bench.input_sets(cfg, 1))
    assert d["cpu_baseline"]["value"] == d["value"] and d["cpu_baseline"]["kind"] == "port"
    assert d["e2e"]["value"] == d["value"] and d["e2e"]["h2d_bytes_per_step"] == 0


def test_help_and_work_units():
    """The command line parses, and the work counted per step is the causal pair
    count of the default workload (5.499e11 FLOP) and at least the KV-cache bytes
    of the decode workload."""
    res = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--help"], capture_output=True, text=True,
                         timeout=120, cwd=str(ROOT))
    assert res.returncode == 0 and "--gather" in res.stdout
    assert abs(bench.work_units(bench.CONFIGS["2"]) - 5.499e11) / 5.499e11 < 1e-3
    dec = bench.CONFIGS["5"]
    kv = 2 * dec["B"] * dec["Hkv"] * dec["KS"] * dec["D"] * 2
    assert bench.work_units(dec) >= kv


def test_tensor_peak_follows_the_power_regime():
    """The roofline divides by the burst peak unless the power cap engaged during the
    timed region, then by the sustained one; INT8 uses the int8 peaks it measured."""
    peak, burst, sus, _, regime = bench.tensor_peak("fp16", {"reasons": []})
    assert peak == burst and sus <= burst and regime.startswith("burst")
    peak, burst, sus, _, regime = bench.tensor_peak("fp16", {"reasons": ["sw_power_cap"]})
    assert peak == sus and regime.startswith("sustained")
    peak8, burst8, sus8, src8, _ = bench.tensor_peak("int8", {"reasons": []})
    assert peak8 == burst8 and burst8 > burst and sus8 < burst8
