"""bench.py pieces that run without a GPU: the reference arm's JSON line (the driver runs
it on every box) and the device-side synthetic generator used for the DeepSeek-V3 layer."""

from __future__ import annotations

import json
import math
import subprocess
import sys
from pathlib import Path

import numpy as np
import torch

REPO = Path(__file__).resolve().parents[1]


def _run_bench(*args: str) -> dict:
    r = subprocess.run([sys.executable, str(REPO / "bench.py"), *args], capture_output=True, text=True, timeout=600,
                       cwd=REPO)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout[-2000:]
    return json.loads(lines[0])


def test_reference_arm_line():
    d = _run_bench("--impl", "reference", "--workload", "cfg0_decode1", "--steps", "1", "--warmup", "1",
                   "--cpu-sample", "1")
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["value"] > 0 and d["higher_is_better"] is True
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["config"]["workload"] == "cfg0_decode1"


def test_reference_arm_unavailable_lines():
    for wl in ("cfg4_decode", "cfg3_attn_decode"):
        d = _run_bench("--impl", "reference", "--workload", wl, "--steps", "1", "--warmup", "1")
        assert d["impl"] == "reference" and "unavailable" in d


def test_device_generator_shapes_and_distributions():
    from ccut_b200 import synthetic

    c = synthetic.scaled_config("cfg4", hidden=256, inter=256, num_experts=6, shared_inter=256)
    lw = synthetic.make_layer_device(c, seed=3, device="cpu")
    assert lw.router.shape == (6, 256) and len(lw.experts) == 6 and len(lw.shared) == 1
    g = lw.experts[2].gate
    assert g.weight.dtype == torch.uint8 and tuple(g.weight.shape) == (256, 256)
    assert tuple(g.scale.shape) == (2, 2)
    s = g.scale.numpy()
    assert s.min() >= 1e-3 * (1 - 1e-6) and s.max() <= 1e-1 * (1 + 1e-6)
    w = g.weight.view(torch.float8_e4m3fn).float().numpy()
    assert abs(w.mean()) < 0.05 and abs(w.std() - 1.0) < 0.05  # N(0, 1) rounded to e4m3
    a = synthetic.make_layer_device(synthetic.scaled_config("cfg0", hidden=256, inter=256, num_experts=2,
                                                            shared_inter=256), seed=3, device="cpu")
    m = a.experts[0].down
    assert m.qweight.dtype == torch.int32 and tuple(m.qweight.shape) == (256, 32)
    sc = m.scales.float().numpy()
    assert sc.min() >= 1e-3 * (1 - 1e-3) and math.isclose(float(np.median(sc)), 0.02 * 0.6745 + 1e-3, rel_tol=0.15)
    assert lw.make_x(5).shape == (5, 256)
