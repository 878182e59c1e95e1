"""The DRAM-traffic table that bench.py reads for `roofline.traffic` points
only at ncu summaries that exist, each stating the command that made it."""

import importlib.util
import os

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench():
    spec = importlib.util.spec_from_file_location("bench_for_test", os.path.join(REPO, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_traffic_rows_point_at_existing_summaries():
    bench = _bench()
    found = 0
    for name in bench.WORKLOADS:
        traffic, src = bench._traffic(name)
        if traffic is None:
            continue
        found += 1
        assert traffic > 0
        path = os.path.join(REPO, src)
        assert os.path.isfile(path), src
        with open(path) as f:
            text = f.read()
        assert "ncu " in text and "--clock-control none" in text, src
    # the headline decode workload and prefill carry a measured figure
    assert bench._traffic("decode_m1")[0] is not None
    assert bench._traffic("prefill_m2048")[0] is not None
    assert found >= 3
