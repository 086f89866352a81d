"""bench.py host logic that needs no GPU: the roofline's `traffic` figure is
read from the committed ncu summaries under profiles/."""
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def test_every_workload_line_finds_its_traffic_figure():
    import bench
    for w in ("c2", "c2fp16", "c3", "c4", "decode4", "decode6", "decode8"):
        traffic, src = bench.profile_traffic(w)
        assert traffic is not None and traffic > 0 and src.endswith(".md"), w


def test_traffic_is_close_to_the_algorithmic_bytes_of_the_attention_lines():
    # ncu measured no re-reads: DRAM traffic within a few percent above the
    # bytes the kernel must read (plus the split partials it writes).
    import bench
    for w in ("c2", "c2fp16", "c3", "c4"):
        traffic, _ = bench.profile_traffic(w)
        assert 1.0 <= traffic / bench.job_bytes(w) < 1.1, w


def test_unknown_workload_has_no_traffic_figure():
    import bench
    assert bench.profile_traffic("no_such_workload") == (None, None)
