"""CPU-only checks of the benchmark's accounting: the algorithmic bytes the roofline divides
by, and the measured DRAM traffic it reports next to them (profiles/traffic.json)."""
import json
import os

import bench

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_headline_algorithmic_bytes_match_the_stated_figure():
    # 256 rows x 607,744 B of f32 logits + 2,097,152 B of history ids + 1,028 B of offsets
    # + 256 x 36 B of row parameters, uniform and token.
    w = bench.make_workload(0, 1, "headline")
    assert (w.B, w.V, w.dtype) == (256, 151_936, "f32")
    assert bench.algorithmic_bytes(w) == 157_689_860


def test_measured_traffic_records_and_scaling():
    rec = json.load(open(os.path.join(ROOT, "profiles", "traffic.json")))
    for key, r in rec.items():
        assert r["bytes_per_launch"] == r["read"] + r["write"], key
        assert os.path.exists(os.path.join(ROOT, r["profile"])), key
    full = rec["lss_stream_kernel_cfg4"]["bytes_per_launch"]
    assert bench.measured_traffic("lss_stream_kernel_cfg4") == full
    # config 4 split over four ranks: each launch covers a quarter of the rows
    assert bench.measured_traffic("lss_stream_kernel_cfg4", 256 / 1024) == round(full / 4)
    assert bench.measured_traffic("no_such_kernel") is None


def test_traffic_is_close_to_the_algorithmic_bytes():
    # one pass over the logits: DRAM traffic within 2 % of the bytes the call must move
    traffic = bench.measured_traffic("lss_stream_kernel_headline")
    assert 1.0 <= traffic / 157_689_860 < 1.02
