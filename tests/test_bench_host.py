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
    assert f["nvlink_bytes"] == 7 * n * (k * 8 + d * 4)
    assert f["hbm_bytes"] == n * k * d * 4 + world * n * k * 8 + (world + 2) * n * d * 4
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
