"""bench.py's driver contract on the CPU: the module imports with every workload entry point, both arms build
the same decode `config` from the arguments, and the reference arm (the oracle on the host cores) prints
one JSON line with the contract's keys."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_bench_entry_points_and_shared_config():
    sys.path.insert(0, ROOT)
    import argparse

    import bench

    for name in ("run_decode", "run_gemv", "run_pass", "cpu_baseline_decode", "cpu_baseline_gemv", "main"):
        assert callable(getattr(bench, name)), name
    args = argparse.Namespace(ctx_fill=0, no_mtp=False, gen=400, ctx=512)
    c1 = bench.decode_config(args, 1)
    assert c1 == bench.decode_config(args, 1)
    assert c1["workload"] == "config5-decode-mtp" and c1["parallelism"] == "single GPU"
    assert bench.tp_layout(8) == (8, 1) and bench.tp_layout(4) == (4, 1)


def test_reference_arm_prints_one_line():
    out = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--workload", "gemv", "--steps", "1",
                          "--warmup", "3"], cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    j = json.loads(lines[0])
    for k in ("impl", "metric", "value", "unit", "config", "cpu_baseline", "e2e", "higher_is_better"):
        assert k in j, k
    assert j["impl"] == "reference" and j["cpu_baseline"]["kind"] == "port"
    chk = subprocess.run([sys.executable, "-c", "import sys, bench; bench.cpu_baseline_gemv(sample_rows=64); "
                          "print(any(m.startswith('rapier_b200') for m in sys.modules))"], cwd=ROOT,
                         capture_output=True, text=True, timeout=300)
    assert chk.stdout.strip().endswith("False"), "the reference arm must not load the product package"
