"""Host-side arithmetic of bench.py's roofline object (no GPU): the fused
projection launches' achieved bandwidth from CUDA-event pairs, and the choice
of the dominant kernel by total time."""
from __future__ import annotations

import bench


class _Ev:
    """Stands in for a recorded CUDA event: elapsed_time in milliseconds."""

    def __init__(self, t):
        self.t = t

    def elapsed_time(self, end):
        return end.t - self.t


def test_resid_ln_roofline_averages_launches():
    probe = {"resid_ln": [(_Ev(0.0), _Ev(1.0)), (_Ev(5.0), _Ev(8.0))],
             "resid_ln_bytes": [1_000_000_000, 3_000_000_000]}
    r = bench.resid_ln_roofline(probe)
    # mean bytes 2 GB over mean time 2 ms
    assert abs(r["achieved"] - 1000.0) < 1e-6
    assert r["launches_timed"] == 2 and abs(r["total_ms"] - 4.0) < 1e-12
    assert abs(r["frac"] - r["achieved"] / r["peak"]) < 1e-12
    assert abs(r["traffic"] - 2e9 * bench.RESID_LN_TRAFFIC_RATIO) < 1.0


def test_resid_ln_roofline_needs_matching_records():
    assert bench.resid_ln_roofline({}) is None
    assert bench.resid_ln_roofline({"resid_ln": [(_Ev(0.0), _Ev(1.0))], "resid_ln_bytes": []}) is None


def test_dominant_roofline_orders_by_total_time():
    a = {"kernel": "a", "total_ms": 3.0}
    b = {"kernel": "b", "total_ms": 7.0}
    r = bench.dominant_roofline([a, None, b])
    assert r["kernel"] == "b" and r["next"]["kernel"] == "a"
    assert bench.dominant_roofline([None]) is None
    assert "next" not in bench.dominant_roofline([a])
