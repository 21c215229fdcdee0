"""bench.py's in-graph timeline summary (profile mode --timeline) on a synthetic
PyTorch-profiler trace: overlapping kernels (programmatic dependent launch) and
idle gaps and a kernel running inside another; the contributions and the idle
time add up to the span."""
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import bench  # noqa: E402


def test_timeline_summary(tmp_path):
    ev = [dict(ph="X", cat="kernel", name="k_gemv<1, 2>(GemvArgs)", ts=0.0, dur=10.0),
          dict(ph="X", cat="kernel", name="k_attn(AttnArgs)", ts=8.0, dur=7.0),  # starts 2 us early
          dict(ph="X", cat="kernel", name="k_gemv<1, 2>(GemvArgs)", ts=20.0, dur=5.0),  # after 5 us idle
          dict(ph="X", cat="cpu_op", name="aten::empty", ts=0.0, dur=1.0),
          dict(ph="X", cat="kernel", name="k_gemv<1, 2>(GemvArgs)", ts=30.0, dur=4.0),
          dict(ph="X", cat="kernel", name="k_attn(AttnArgs)", ts=31.0, dur=2.0)]  # inside its predecessor
    p = tmp_path / "trace.json"
    p.write_text(json.dumps({"traceEvents": ev}))
    lines = bench.timeline_summary(str(p), 2)
    assert lines[0] == "timeline: 5 kernels over 2 steps, 17.0 us/step, idle 5.0 us/step"
    rows = {ln.split(" | ")[0]: ln.split(" | ")[1:] for ln in lines[2:]}
    # busy instants go to the running kernel that ends first: k_gemv 0-10, 20-25,
    # 30-31 and 33-34 (17 us); k_attn 10-15 and 31-33 (7 us); idle 15-20 and 25-30
    assert rows["k_gemv<1, 2>"][:4] == ["1.5", "6.33", "5.67", "8.5"]
    assert rows["k_attn"][:4] == ["1.0", "4.50", "3.50", "3.5"]
    total = sum(float(r[3]) for r in rows.values()) * 2 + 5.0 * 2
    assert abs(total - 34.0) < 1e-6


def test_timeline_summary_empty(tmp_path):
    p = tmp_path / "trace.json"
    p.write_text(json.dumps({"traceEvents": []}))
    assert bench.timeline_summary(str(p), 1) == ["timeline: no kernel events recorded"]
