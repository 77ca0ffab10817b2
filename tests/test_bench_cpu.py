"""The bench's CPU legs, run here without a GPU: the reference arm's JSON line (the
contract the driver reads) and the CPU-baseline helpers of the forward line."""
import importlib.util
import json
import os
import subprocess
import sys
from pathlib import Path

import numpy as np

from rustane_b200.model import custom_config

ROOT = Path(__file__).resolve().parents[1]


def _bench():
    spec = importlib.util.spec_from_file_location("bench_mod", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_reference_arm_json_line(oracle_lib):
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference",
                          "--steps", "1", "--warmup", "1"], cwd=ROOT, env=env,
                         capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["unit"] == "tokens/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["steps"] == 1 and d["warmup"] == 1
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["cpu_baseline"]["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}
    # the same loss the oracle reports at init: about ln(8192)
    assert abs(d["loss"] - np.log(8192)) < 0.5


def test_cpu_baseline_helpers(oracle_lib):
    bench = _bench()
    cfg = custom_config(256, 512, 2, 4, 128)
    rng = np.random.default_rng(0)
    tok = rng.integers(0, cfg.vocab, 2 * cfg.seq).astype(np.uint32)
    tgt = rng.integers(0, cfg.vocab, 2 * cfg.seq).astype(np.uint32)
    r = bench.cpu_oracle_sample(cfg, 0, tok, tgt, 0.0)
    assert r["seqs"] == 1 and r["seconds"] > 0 and len(r["losses"]) == 1
    fig = bench.torch_cpu_figure(cfg, r, extrapolated=False)
    assert fig["value"] > 0 and "one sequence per call" in fig["sample"]
    e = bench.cpu_oracle_extrapolated(cfg, 0, tok, tgt)
    assert e["seqs"] == 1 and e["seconds"] >= e["t1"] > 0
    assert "extrapolated" in bench.torch_cpu_figure(cfg, e, extrapolated=True)["sample"]
    e["torch_seconds"] = "torch CPU forward failed: test"
    assert bench.torch_cpu_figure(cfg, e, extrapolated=True) == {
        "unavailable": "torch CPU forward failed: test"}


def test_bench_rejects_short_warmup():
    """The timing rules need at least 3 warm-up steps; the bench refuses fewer before
    it touches a device."""
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--warmup", "2"], cwd=ROOT,
                         capture_output=True, text=True, timeout=300)
    assert out.returncode != 0 and "--warmup must be >= 3" in out.stderr
