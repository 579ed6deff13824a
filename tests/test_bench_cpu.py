"""bench.py on the host (no GPU): the per-op CPU baseline of the op benchmarks (BASELINE
configs 2-4) returns a well-formed cpu_baseline record for each op, and the algorithmic byte
counts behind `step_hbm` and `roofline` match the published per-unit formulas."""
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


def _cfg_2b(synth):
    s = synth.shape_2b()
    n_attn = sum(s.layer_is_attn(l) for l in range(s.n_layers))
    return dict(dim=s.dim, ffn=s.ffn, vocab=s.vocab, dn_heads=s.dn_heads, head_dim=s.head_dim, n_heads=s.attn_heads,
                n_kv_heads=s.kv_heads, n_dn=s.n_layers - n_attn, n_attn=n_attn, conv_kernel=s.conv_kernel)


def test_roofline_accounting_matches_the_published_formulas(bench, synth):
    """The algorithmic bytes behind `step_hbm` and `roofline`, against the per-unit figures of
    the measurement plan for the 2B shape: W = 1,789,124,608 B of Q8_0 weights per step, K+V
    = 2048 B per token per sequence over the 6 GQA layers' kv heads, and the DeltaNet state
    read and written (18 layers x 2 MiB) with the conv state read and written (2 x 98,304 B)."""
    cfg = _cfg_2b(synth)
    assert bench.weight_bytes(cfg) == 1_789_124_608
    assert bench.attn_launch_bytes(cfg, 64, 8192) == 2048 * 64 * 8192
    kv = 6 * 2 * 2 * 8192 * 256 * 2
    assert kv == 100_663_296
    assert bench.seq_bytes(cfg, 8192) == 18 * (2 * (1 << 20) + 2 * 98_304) + kv
    # one step at B=64, ctx 8192 (10.88 GB at the bench's mean context of ~8.2K tokens)
    step = bench.weight_bytes(cfg) + 64 * bench.seq_bytes(cfg, 8192)
    assert round(step / 1e9, 2) == 10.87


def test_kernel_family_accounting(bench, synth):
    """The per-family bytes of the `kernels` map: the GEMM family's weights are exactly the
    step's Q8_0 weight bytes (every projection and the lm_head, in launch order), plus B*k*2 of
    activations and B*m*4 of outputs per launch; one DeltaNet launch moves ~2.33 MB per
    sequence (state and conv state read and written, projections in, f16 output out)."""
    cfg = dict(_cfg_2b(synth))
    s = synth.shape_2b()
    cfg["layer_is_dn"] = [not s.layer_is_attn(l) for l in range(s.n_layers)]
    shapes = bench.gemm_shapes(cfg)
    assert len(shapes) == 4 * s.n_layers + 1
    assert sum(m * k * 34 // 32 for m, k in shapes) == bench.weight_bytes(cfg)
    extra = sum(64 * k * 2 + 64 * m * 4 for m, k in shapes)
    assert bench.gemm_step_bytes(cfg, 64) == bench.weight_bytes(cfg) + extra
    per_seq = bench.dn_launch_bytes(cfg, 1)
    assert per_seq == 2 * 16 * 128 * 128 * 4 + 2 * 3 * 2048 * 4 * 4 + (4 * 2048 + 32) * 4 + 2048 * 2
    assert round(per_seq / 1e6, 2) == 2.33
