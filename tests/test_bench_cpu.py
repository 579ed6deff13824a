"""bench.py's CPU legs on the host (no GPU): the per-op CPU baseline of the op benchmarks
returns a well-formed cpu_baseline record for each op."""
import importlib.util
import os

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    mod.load_pkg()
    return mod


@pytest.mark.parametrize("op,kw", [("gemm", dict(M=512, K=256)), ("recurrence", {}), ("attention", dict(ctx=300))])
def test_cpu_op_baseline_record(bench, op, kw):
    rec = bench.cpu_op_baseline(op, B=4, seconds=0.05, **kw)
    assert set(rec) == {"value", "unit", "cores", "kind", "sample"}
    assert rec["value"] > 0 and rec["cores"] >= 1 and rec["kind"] == "port"
    assert "batch 4" in rec["sample"]
