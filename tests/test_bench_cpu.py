"""CPU: bench.py's pieces that need no GPU — the reference arm of the vision workload (the SigLIP
oracle timed on the host) prints one JSON line with the contract's keys, and the work models
count the algorithmic FLOPs and bytes the roofline divides by."""

import json
import os
import subprocess
import sys

from conftest import ROOT


def test_vision_reference_arm_prints_contract_line():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--workload",
                          "embed_image", "--impl", "reference", "--steps", "1", "--warmup", "0"],
                         capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "impl", "cpu_baseline", "e2e", "config"):
        assert key in line, key
    assert line["impl"] == "reference" and line["unit"] == "images/s" and line["value"] > 0
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["h2d_bytes_per_step"] == 0


def test_work_models():
    sys.path.insert(0, ROOT)
    import bench
    from mlc_vla.model.pi0 import Pi0Config

    cfg = Pi0Config(dtype="float16")
    w = bench.vision_work_model(cfg, 3)
    total = sum(v[0] for v in w.values() if v[1] == "flop")
    assert abs(total / 3 - 220.2e9) / 220.2e9 < 0.005  # 220.2 GFLOP per image
    assert w["vision.fc2_gemm"][0] == 27 * 2 * 768 * 4304 * 1152
    c = bench.full_config()
    m = bench.work_model(c, 1)
    flops = sum(v[0] for k, v in m.items() if v[1] == "flop")
    assert abs(flops - 3.76e12) / 3.76e12 < 0.01  # the prefill's 3.76 TFLOP per chunk
