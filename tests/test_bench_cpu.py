"""bench.py on the host (no GPU): the per-op CPU baseline of the op benchmarks (BASELINE
configs 2-4) returns a well-formed cpu_baseline record for each op, the algorithmic byte
counts behind `step_hbm` and `roofline` match the published per-unit formulas, and the
clock record's sampler summarises a fake NVML's clocks and reasons."""
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


class _FakeNvml:
    """Stands in for pynvml: a GPU whose SM clock and clock-event reasons follow a script."""
    NVML_CLOCK_SM = 1
    nvmlClocksEventReasonGpuIdle = 0x1

    def __init__(self, script):
        self.script = list(script)   # (sm MHz, reason bits) per poll; the last one repeats
        self.i = 0

    def nvmlInit(self):
        pass

    def nvmlDeviceGetHandleByPciBusId(self, bus_id):
        assert bus_id == "00000000:1B:00.0"
        return "handle"

    def nvmlDeviceGetMaxClockInfo(self, handle, kind):
        return 1965

    def nvmlDeviceGetClockInfo(self, handle, kind):
        return self.script[min(self.i, len(self.script) - 1)][0]

    def nvmlDeviceGetCurrentClocksEventReasons(self, handle):
        bits = self.script[min(self.i, len(self.script) - 1)][1]
        self.i += 1
        return bits


def test_clock_sampler_reads_nvml_during_the_region(bench, monkeypatch):
    """The clock record polls NVML from a thread: begin() drops the samples taken before the
    timed region; the summary holds the median SM clock, the maximum and the throttle reasons
    seen (hw_slowdown 0x8, sw_thermal_slowdown 0x20, hw_thermal_slowdown 0x40, sw_power_cap
    0x4), and ignores the idle bit."""
    import sys
    import time
    fake = _FakeNvml([(345, 0x1)] * 3 + [(1965, 0x0), (1965, 0x4), (1950, 0x0), (1965, 0x1)])
    monkeypatch.setitem(sys.modules, "pynvml", fake)
    c = bench.ClockSampler("00000000:1B:00.0")
    deadline = time.time() + 2.0
    while fake.i < 3 and time.time() < deadline:   # the idle samples before the region
        time.sleep(0.001)
    c.begin()
    while fake.i < 12 and time.time() < deadline:
        time.sleep(0.001)
    rec = c.stop()
    assert rec["source"] == "nvml, 2 ms" and rec["samples"] >= 1
    assert rec["sm_max_mhz"] == 1965
    assert rec["sm_mhz"] >= 1950                      # the 345 MHz idle samples were dropped
    assert set(rec["reasons"]) <= {"sw_power_cap"}


def test_clock_sampler_without_nvml_or_nvidia_smi(bench, monkeypatch):
    import sys
    monkeypatch.setitem(sys.modules, "pynvml", None)   # import fails
    monkeypatch.setattr(bench.subprocess, "Popen", lambda *a, **k: (_ for _ in ()).throw(OSError("absent")))
    rec = bench.ClockSampler("0").stop()
    assert rec["sm_mhz"] is None and rec["reasons"]
