"""The CPU side of bench.py, which the driver's runs depend on: the reference arm's JSON line
(``--impl reference``: the reference's fp32 CPU path on the same workload) and the bounded CPU
baselines that the GPU lines carry (decode sweep, prefill configs 1 and 3, the stack's 4-layer unit).
No GPU is used."""
import importlib
import json
import os
import subprocess
import sys

from conftest import ROOT, load_package


def test_reference_arm_line():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "0"], capture_output=True, text=True, cwd=ROOT, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["value"] > 0 and line["unit"] == "GB/s"
    assert line["higher_is_better"] is True and line["warmup"] >= 3
    assert line["config"]["workload"] == "decode_gemv_sweep_config2"
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"] == {"value": line["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_cpu_baselines_run():
    sys.path.insert(0, ROOT)
    import bench
    deqs, packs, xs = bench.cpu_setup()
    n, dt = bench.cpu_time(packs, xs, 0.1, bench.cpu_sweep_dequant_once)
    assert n >= 1 and dt > 0
    pre = bench.cpu_prefill_baseline(0.3)
    assert set(pre) == {"gate_up/M64", "gate_up/M2048", "down/M2048"}
    assert all(v["TFLOPs"] > 0 and v["calls"] >= 1 for v in pre.values())
    load_package()
    serve = importlib.import_module("strands_decider_web_b200.serve")
    st = bench.cpu_stack_baseline(serve, 0.1)
    assert st["unit"] == "tokens/s" and st["value"] > 0 and st["kind"] == "port"
