"""bench.py host helpers on the CPU: the clock-record parser and the DRAM
traffic figure that the bench line quotes from the committed ncu summaries
(scaled to a strong-scaling rank's rows)."""
import os
import sys

import pytest

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import bench  # noqa: E402


def test_clock_summary_parses_samples_and_reasons(tmp_path):
    c = bench.Clocks(0)
    c.path = str(tmp_path / "clocks.csv")
    with open(c.path, "w") as f:
        f.write("0, 1965, 1965, 700.1, 0x0, Not Active, Not Active, Not Active, Not Active\n")
        f.write("0, 1900, 1965, 990.0, 0x4, Not Active, Not Active, Not Active, Active\n")
        f.write("0, 1965, 1965, 980.0, 0x0, Not Active, Not Active, Not Active, Not Active\n")
        f.write("garbled line\n")
    s = c.summary()
    assert s == {"sm_mhz": 1965.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"], "samples": 3}
    assert not os.path.exists(c.path)


def test_profile_traffic_is_per_rank_in_strong_mode():
    t = bench.profile_traffic("cfg2")
    if t is None:
        pytest.skip("no committed traffic figure for cfg2")
    assert bench.rows_traffic(t, 4096, 4096) is t
    q = bench.rows_traffic(t, 1024, 4096)
    assert q["bytes"] == int(t["bytes"] / 4) and q["dram_read"] == int(t["dram_read"] / 4)
    assert q["source"] == t["source"] and "1024" in q["note"]
    assert bench.rows_traffic(None, 1024, 4096) is None
