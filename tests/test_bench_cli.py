"""bench.py's reference arm on the CPU: the one-line JSON contract the driver reads (keys, types,
units), and the rank rule under torchrun (rank 0 alone prints; other ranks exit 0 silently)."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def run(args, env=None):
    e = dict(os.environ)
    e.update(env or {})
    p = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], cwd=ROOT, env=e,
                       capture_output=True, text=True, timeout=600)
    assert p.returncode == 0, p.stderr[-2000:]
    return p.stdout


def test_reference_arm_prints_one_json_line():
    out = run(["--impl", "reference", "--workload", "q4k", "--steps", "3", "--warmup", "3"])
    lines = [ln for ln in out.splitlines() if ln.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] == "weight GB/s" and d["unit"] == "GB/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["steps"] == 3 and d["warmup"] == 3 and d["n_gpus"] == 1
    assert d["config"]["workload"].startswith("q4k") and d["config"]["qtype"] == "Q4_K"
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["cpu_model"]
    assert d["e2e"] == {"value": d["value"], "unit": "GB/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}
    assert d["gpu_launches"] == 0


def test_reference_arm_other_ranks_are_silent():
    out = run(["--impl", "reference", "--workload", "q4k", "--steps", "3", "--warmup", "3"],
              env={"RANK": "1", "LOCAL_RANK": "1", "WORLD_SIZE": "2"})
    assert out.strip() == ""


def test_stack_reference_arm_has_the_gpu_arms_config():
    out = run(["--impl", "reference", "--steps", "3", "--warmup", "3"])  # the default workload
    d = json.loads([ln for ln in out.splitlines() if ln.strip()][0])
    assert d["metric"] == "decode tokens/s" and d["unit"] == "tokens/s" and d["value"] > 0
    assert d["config"]["workload"].startswith("stack70b")
    import bench
    from kernite_b200 import stack as st

    args = bench.parse_args(["--steps", "3"])
    assert d["config"] == bench.stack_config(args, st.CONFIGS["70b"], 1, args.exchange == "chain")
    assert "l2" in d["config"] and d["cpu_baseline"]["cores"] >= 1


def test_matvec_reference_arm_config_has_the_l2_rotation():
    out = run(["--impl", "reference", "--workload", "q6k_head", "--steps", "3", "--warmup", "3"])
    d = json.loads([ln for ln in out.splitlines() if ln.strip()][0])
    assert "l2" in d["config"] and "copies" in d["config"]["l2"]
