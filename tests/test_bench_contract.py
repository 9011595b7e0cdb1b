"""bench.py's reference arm (the oracle's CPU restatement of the 7B decode step, timed on the host at
all threads and at one thread) keeps the JSON-line contract the driver reads; it needs no GPU, so it is
checked here on the CPU."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_one_contract_line():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "3"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "higher_is_better", "scaling", "vs_baseline",
                "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["value"] > 0 and d["unit"] == "tokens/s"
    assert d["warmup"] >= 3 and d["steps"] == 1
    assert d["cpu_baseline"]["kind"] in ("port", "reference") and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["value"] == d["value"] and d["e2e"]["h2d_bytes_per_step"] == 0
    assert "workload" in d["config"] and d["config"]["workload"].startswith("configs[4]")
    assert d["cpu_baseline"]["single_thread"]["cores"] == 1 and d["cpu_baseline"]["single_thread"]["value"] > 0


def test_cpu_kernel_baselines_cover_the_kernel_configs():
    """The N = 1 line's cpu_baseline.kernels: configs[0] at the three block sizes, configs[1] and configs[2],
    each on one thread and on all threads, with positive rates."""
    sys.path.insert(0, ROOT)
    import bench
    rec = bench.cpu_kernel_baselines(min_s=0.01)
    assert set(rec) == {"ternary2_4096x4096_bs64", "ternary2_4096x4096_bs128", "ternary2_4096x4096_bs256",
                        "matvec_q8_0_4096x4096+q4_0_11008x4096", "attention_T4096"}
    for r in rec.values():
        assert r["value_1_thread"] > 0 and r["value_all_threads"] > 0 and r["unit"] == "GB/s" and r["cores"] >= 1
    assert rec["ternary2_4096x4096_bs128"]["algorithmic_bytes_per_unit"] == 4718592
    assert rec["matvec_q8_0_4096x4096+q4_0_11008x4096"]["algorithmic_bytes_per_unit"] == 17825792 + 25362432
