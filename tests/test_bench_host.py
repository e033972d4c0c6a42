"""Host-side arithmetic of bench.py (no GPU): the exchange rooflines reported on more than one GPU."""
import pytest

import bench


def test_exchange_rooflines():
    assert bench.exchange_rooflines({"xchg_forward": 1.0}, 1, 32768, 128, 384, 6500.0) is None
    n, k, d, world, hbm = 32768, 128, 384, 8, 6531.3
    r = bench.exchange_rooflines({"xchg_forward": 2.0, "xchg_backward_gw": 1.5, "bag_forward": 1.0}, world, n, k,
                                 d, hbm)
    assert set(r) == {"xchg_forward", "xchg_backward_gw"}
    f = r["xchg_forward"]
    m = n * k
    assert f["nvlink_bytes"] == 7 * (m // 8) * 12 + 7 * n * d * 4
    assert f["hbm_bytes"] == m * 20 + m * d * 4 + world * m * 4 + m * 8 + (world + 1) * n * d * 4
    assert f["nvlink_GB/s"] == pytest.approx(f["nvlink_bytes"] / 2e-3 / 1e9, rel=1e-3)
    t_nv = f["nvlink_bytes"] / (bench.NVLINK_PEER_GBS * 1e9) * 1e3
    t_hbm = f["hbm_bytes"] / (hbm * 1e9) * 1e3
    assert f["bound"] == ("nvlink" if t_nv >= t_hbm else "hbm")
    assert f["target_ms"] == pytest.approx(max(t_nv, t_hbm), abs=1e-4)
    assert f["frac"] == pytest.approx(max(t_nv, t_hbm) / 2.0, abs=1e-3)
    g = r["xchg_backward_gw"]
    assert g["nvlink_bytes"] == 7 * n * k * 4 // 8
    # a call that did not run (NCCL exchange) is left out
    assert set(bench.exchange_rooflines({"xchg_forward": 2.0}, 2, n, k, d, hbm)) == {"xchg_forward"}


def test_reference_arm_line(tmp_path):
    """bench.py --impl reference (the reference's PyTorch path on the host cores) prints one JSON line with the
    keys the driver reads and the --steps / --warmup it was given; here on a tiny sample."""
    import json
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    out = subprocess.run([sys.executable, os.path.join(root, "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "1", "--cpu-rows-per-half", "32", "--cpu-tokens", "128"],
                         capture_output=True, text=True, timeout=300, cwd=str(tmp_path))
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["metric"] == bench.METRIC and d["unit"] == "tokens/s"
    assert d["value"] > 0 and d["higher_is_better"] is True and d["n_gpus"] == 1
    # the reference's own package when build() vendored it into baseline/_ref, else the restatement under oracle/
    want = "reference" if os.path.isfile(os.path.join(root, "baseline", "_ref", "smlm", "pkm.py")) else "port"
    assert d["cpu_baseline"]["kind"] == want and d["cpu_baseline"]["cores"] >= 1
    assert d["steps"] == 1 and d["warmup"] == 1
    assert d["cpu_baseline"]["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_clock_summary_parsing(tmp_path):
    """Clocks.summary: median SM clock under load, max clock, and only the throttle reasons reported Active."""
    c = bench.Clocks(0)
    c.file = open(tmp_path / "clocks.csv", "w+")
    c.file.write("0, 1965, 1965, 900.1, 0x0000000000000000, Not Active, Not Active, Not Active, Not Active\n"
                 "0, 1800, 1965, 999.5, 0x0000000000000004, Not Active, Not Active, Not Active, Active\n"
                 "0, 1900, 1965, 950.0, 0x0000000000000000, Not Active, Not Active, Not Active, Not Active\n"
                 "0, [N/A], 1965, 950.0, 0x0, Not Active, Not Active, Not Active, Not Active\n")
    c.file.flush()
    s = c.summary()
    assert s["sm_mhz"] == 1900.0 and s["sm_max_mhz"] == 1965.0 and s["samples"] == 3
    assert s["reasons"] == ["sw_power_cap"]
