"""bench.py's reference arm runs on the CPU (no GPU) and prints the contract's JSON line."""
import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_reference_arm_json_line():
    out = subprocess.run(
        [sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "0",
         "--ref-seconds", "0.3", "--workload", "s8_1024"],
        capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert out.returncode == 0, out.stderr
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unit"] == "TOPS" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"] == {"value": d["value"], "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert d["config"]["M"] == 1024


def test_reference_arm_other_ranks_exit_quietly():
    env = {"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1", "PATH": "/usr/bin:/bin"}
    out = subprocess.run(
        [sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "0"],
        capture_output=True, text=True, timeout=120, cwd=ROOT, env=env)
    assert out.returncode == 0 and out.stdout.strip() == ""


def test_roofline_and_bytes_cover_every_workload():
    """bench.py's roofline arithmetic (pure Python): every workload gets a bound, a peak and a
    fraction; int8 / sparse peaks are the nominal 4.5 / 9 POPS with the measured-bf16 basis
    beside them; the skinny W4A8 decode is HBM-bound."""
    sys.path.insert(0, str(ROOT))
    import bench

    for name, (M, N, K, kind, layout) in bench.WORKLOADS.items():
        assert bench.algorithmic_bytes(kind, M, N, K) > 0, name
        r = bench.roofline(kind, M, N, K, 1e-3, sustained=False)
        assert r["bound"] in ("tensor", "hbm") and r["peak"] > 0 and r["frac"] == r["achieved"] / r["peak"], name
        assert bench.CHECK_KIND[kind] in ("s8", "s8_scaled", "w4a8", "bf16", "sp_s8", "s4s4", "sp_s4"), name
        assert bench.describe(name)
    assert bench.roofline("w4a8", 16, 28672, 8192, 40e-6, False)["bound"] == "hbm"
    r = bench.roofline("s8", 8192, 8192, 8192, 0.33e-3, False)
    assert r["peak"] == bench.NOMINAL_INT8_TOPS and "frac_of_measured_bf16_x2" in r
    assert bench.roofline("sp_s8", 8192, 8192, 8192, 0.26e-3, False)["peak"] == 2 * bench.NOMINAL_INT8_TOPS
    assert set(bench.CONFIG_SET) <= set(bench.WORKLOADS)
