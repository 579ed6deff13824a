"""Decode-throughput benchmark of the B200 backend on the 2B-shape Qwen3.5 hybrid (Q8_0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (one process per GPU)

Workload: 24 layers (every 4th GQA), hidden 2048, vocab 151936, random
Q8_0 weights; 64 sequences whose bf16 KV cache is prefilled to 8192 tokens and whose
DeltaNet / conv states are seeded; a step is one greedy decode token for every sequence.
With N GPUs the 64 sequences are split across them (sequence sharding, no collective on
the data path: strong scaling, `--weak` runs 64 sequences per GPU instead); at N > 1 the
line also carries the weak-scaling figure measured in the same run.

Printed (rank 0): one JSON line with the whole-job tok/s measured on device with CUDA events
(inputs resident, tokens fed back on device), the end-to-end tok/s through the host-buffer
API, the roofline of the dominant kernel family with the other two beside it, the CPU
baseline and the SM clocks seen.
`--impl reference` times the CPU restatement of the reference decode path (oracle/) on the
host cores for the same metric.

    torchrun --nproc-per-node N bench.py --gpus N --split heads --batch 1 [--ctx C]

times the head-parallel split instead (every rank runs the --batch sequences with 1/N of the
DeltaNet and kv heads, the mixer outputs all-gathered with NCCL): one JSON line with the
decode-step latency (max over ranks); with N = 1 the same step on one GPU, which is also what
sequence sharding gives one sequence at any N.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.join(ROOT, "ane-infer_b200")

METRIC = "decode tok/s, 2B-shape Q8_0 B=64 ctx8K at 1/2/4/8 B200; % HBM roofline"
SHAPE_KEYS = dict(n_layers=24, dim=2048, vocab=151936, ffn=6144, dn_heads=16, dn_state=128, attn_heads=8,
                  kv_heads=2, head_dim=256)
# dram__bytes_read.sum + dram__bytes_write.sum per decode step of each kernel family, from one
# ncu capture of this benchmark's own step (2B shape, B=64, ctx ~8.2K: the launch list with
# gpu__time_duration and the DRAM bytes, one pass per launch, ten steps averaged). The GEMM
# family's figure includes the L2 prefetch of each following GEMM's weights (and of the first
# DeltaNet states) and write-backs of DeltaNet state evicted while the GEMMs run; DeltaNet's
# leaves part of its state writes to later kernels.
NCU_TRAFFIC_PER_STEP = {"q8_gemm": 3_431_700_000, "attention": 6_510_200_000, "deltanet": 1_640_300_000}


def load_pkg():
    name = "ane_infer_b200"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, os.path.join(PKG_DIR, "__init__.py"),
                                                  submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# --------------------------------------------------------------------------- clocks sampler
class ClockSampler:
    """SM clock and clock-event reasons of one GPU while the timed region runs. NVML is polled
    every 2 ms from a thread, since a timed region lasts only tens of milliseconds; the
    nvidia-smi loop (200 ms) is the fallback where NVML cannot be loaded. `begin()` drops what
    was sampled before the region starts; `stop()` ends sampling and summarises it."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
               ("sw_power_cap", 0x4))

    def __init__(self, gpu_id: str):
        self.samples = []  # (sm MHz, max sm MHz, set of reason names)
        self.proc = None
        self.nvml = None
        self._stop = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            self.handle = pynvml.nvmlDeviceGetHandleByPciBusId(gpu_id)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM))
            self.nvml = pynvml
            self.t = threading.Thread(target=self._poll, daemon=True)
            self.t.start()
            return
        except Exception:
            self.nvml = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", gpu_id, f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            return
        self.t = threading.Thread(target=self._read, daemon=True)
        self.t.start()

    def _poll(self):
        nv = self.nvml
        reasons_of = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nv.nvmlDeviceGetCurrentClocksThrottleReasons
        while not self._stop.is_set():
            try:
                sm = float(nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM))
                bits = int(reasons_of(self.handle))
            except Exception:
                break
            self.samples.append((sm, self.max_mhz, {n for n, b in self.REASONS if bits & b}))
            time.sleep(0.002)

    def _read(self):
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9 and parts[1].replace(".", "").isdigit() and parts[2].replace(".", "").isdigit():
                names = {self.REASONS[i][0] for i in range(4) if parts[5 + i].lower() == "active"}
                self.samples.append((float(parts[1]), float(parts[2]), names))

    def begin(self):
        self.samples = []

    def stop(self) -> dict:
        if self.nvml is None and self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["NVML and nvidia-smi unavailable"]}
        self._stop.set()
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        self.t.join(timeout=2)
        got = list(self.samples)
        return {"sm_mhz": statistics.median(s[0] for s in got) if got else None,
                "sm_max_mhz": max(s[1] for s in got) if got else None,
                "reasons": sorted(set().union(*(s[2] for s in got))) if got else [],
                "samples": len(got), "source": "nvml, 2 ms" if self.nvml else "nvidia-smi, 200 ms"}


def gpu_id_for(torch, dev: int) -> str:
    try:
        p = torch.cuda.get_device_properties(dev)
        return f"{p.pci_domain_id:08X}:{p.pci_bus_id:02X}:{p.pci_device_id:02X}.0"
    except Exception:
        return str(dev)


# --------------------------------------------------------------------------- byte accounting
def weight_bytes(cfg) -> int:
    """Algorithmic Q8_0 weight bytes read per step (every projection + lm_head, not the embedding)."""
    D, F, V = cfg["dim"], cfg["ffn"], cfg["vocab"]
    H, hd, Hq, Hkv = cfg["dn_heads"], cfg["head_dim"], cfg["n_heads"], cfg["n_kv_heads"]
    per_dn = 3 * D * D + D * D + 2 * H * D + D * D
    per_at = 2 * Hq * hd * D + 2 * Hkv * hd * D + D * Hq * hd
    ffn = 3 * D * F
    elems = cfg["n_dn"] * (per_dn + ffn) + cfg["n_attn"] * (per_at + ffn) + V * D
    return elems * 34 // 32


def seq_bytes(cfg, ctx_len: int, kv_bytes: int = 2) -> int:
    """Per-sequence state bytes per step: DeltaNet state r+w, conv state r+w, K+V read."""
    dn = cfg["n_dn"] * (2 * cfg["dn_heads"] * 128 * 128 * 4 + 2 * 3 * cfg["dim"] * cfg["conv_kernel"] * 4)
    kv = cfg["n_attn"] * 2 * cfg["n_kv_heads"] * ctx_len * cfg["head_dim"] * kv_bytes
    return dn + kv


def attn_launch_bytes(cfg, B: int, ctx_len: int) -> int:
    """One flash-decode launch: every sequence's K and V (bf16) read once."""
    return B * cfg["n_kv_heads"] * ctx_len * cfg["head_dim"] * 2 * 2


def gemm_shapes(cfg) -> list:
    """(m, k) of every Q8_0 GEMM launch of one decode step, in launch order."""
    D, F, V = cfg["dim"], cfg["ffn"], cfg["vocab"]
    H, hd, Hq, Hkv = cfg["dn_heads"], cfg["head_dim"], cfg["n_heads"], cfg["n_kv_heads"]
    out = []
    for dn in cfg["layer_is_dn"]:
        if dn:
            out += [(3 * D + D + 2 * H, D), (D, D)]
        else:
            out += [(2 * Hq * hd + 2 * Hkv * hd, D), (D, Hq * hd)]
        out += [(2 * F, D), (D, F)]
    return out + [(V, D)]


def gemm_step_bytes(cfg, B: int) -> int:
    """Algorithmic bytes of one step's Q8_0 GEMMs: per launch m*k*34/32 of weights, B*k*2 of
    activations and B*m*4 of outputs (the per-unit figure of the GEMM op benchmark)."""
    return sum(m * k * 34 // 32 + B * k * 2 + B * m * 4 for m, k in gemm_shapes(cfg))


def dn_launch_bytes(cfg, B: int) -> int:
    """One DeltaNet mixer launch, per sequence: the f32 state read and written (H x 128 x 128),
    the conv state read and written (3D x K), the projection inputs read and the f16 output."""
    D, H, K = cfg["dim"], cfg["dn_heads"], cfg["conv_kernel"]
    return B * (2 * H * 128 * 128 * 4 + 2 * 3 * D * K * 4 + (4 * D + 2 * H) * 4 + D * 2)


# --------------------------------------------------------------------------- CPU reference
def cpu_reference_tokps(gguf, shape, ctx_len: int, n_tokens: int = 0, seconds: float = 15.0, seq: int = 0):
    """Time the oracle (CPU restatement, all host threads) decoding one sequence at ctx_len."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    from ane_infer_b200 import synth
    oracle.lib().oracle_set_threads(len(os.sched_getaffinity(0)))
    om = oracle.Model(gguf, ctx_cap=ctx_len + 64)
    s = om.new_seq(kv_bf16=True)
    for l in range(shape.n_layers):
        if shape.layer_is_attn(l):
            k, v = synth.seeded_kv(shape, seq, l, ctx_len)
            s.set_kv(l, k, v)
        else:
            s.set_dn(l, synth.seeded_dn_state(shape, seq, l), synth.seeded_conv_state(shape, seq, l))
    s.pos = ctx_len
    tok = 1
    s.forward(tok)          # warm-up token
    t0 = time.perf_counter()
    done = 0
    limit = n_tokens or 62  # the sample stays inside the oracle's context (ctx_len + 64)
    while done < limit and (n_tokens or time.perf_counter() - t0 < seconds):
        tok = oracle.greedy(s.forward(tok))
        done += 1
    dt = time.perf_counter() - t0
    return done / dt, done, dt, oracle.lib().oracle_max_threads()


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    load_pkg()
    from ane_infer_b200 import synth
    shape = synth.shape_2b()
    gguf = synth.build_model_gguf(shape, seed=0)
    total_steps = args.warmup + args.steps
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    # all host cores (torchrun sets OMP_NUM_THREADS=1 for its workers)
    oracle.lib().oracle_set_threads(len(os.sched_getaffinity(0)))
    om = oracle.Model(gguf, ctx_cap=args.ctx + total_steps + 8)
    s = om.new_seq(kv_bf16=True)
    for l in range(shape.n_layers):
        if shape.layer_is_attn(l):
            s.set_kv(l, *synth.seeded_kv(shape, 0, l, args.ctx))
        else:
            s.set_dn(l, synth.seeded_dn_state(shape, 0, l), synth.seeded_conv_state(shape, 0, l))
    s.pos = args.ctx
    tok = 1
    for _ in range(args.warmup):
        tok = oracle.greedy(s.forward(tok))
    t0 = time.perf_counter()
    for _ in range(args.steps):
        tok = oracle.greedy(s.forward(tok))
    dt = time.perf_counter() - t0
    v = args.steps / dt
    cores = oracle.lib().oracle_max_threads()
    total = args.batch * args.gpus if args.weak else args.batch
    per_gpu = args.batch if args.weak else args.batch // max(args.gpus, 1)
    sample = (f"1 of the {total} sequences, {args.steps} greedy tokens at ctx {args.ctx} "
              f"(the reference decodes one sequence at a time; {total} sequences = {total} sequential runs)")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(v, 4), "unit": "tok/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * dt / args.steps, 2),
        "higher_is_better": True, "scaling": "weak" if args.weak else "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": f"2B-shape Qwen3.5 hybrid greedy decode, Q8_0, {total} sequences "
                               f"({per_gpu} per GPU), ctx {args.ctx} prefilled bf16 KV",
                   "model": "qwen35-hybrid-2B-shape (random init)",
                   "global_batch": total, "seq_len": args.ctx,
                   "parallelism": "host threads; sequences one after another, as the reference decodes"},
        "cpu_baseline": {"value": round(v, 4), "unit": "tok/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": round(v, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# --------------------------------------------------------------------------- our arm
def run_ours(args):
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=900), device_id=torch.device("cuda", local))

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    pkg = load_pkg()
    from ane_infer_b200 import synth
    from ane_infer_b200.shard import ShardedDecoder, max_over_ranks
    shape = synth.shape_2b()
    gguf = synth.build_model_gguf(shape, seed=0)
    # strong scaling (default): the --batch sequences split across the ranks; --weak: --batch per rank
    if args.weak:
        B = args.batch
    else:
        from ane_infer_b200.shard import shard_range
        B = shard_range(args.batch, world, rank)[1]
        if args.batch % world:
            raise SystemExit(f"--batch {args.batch} does not split evenly over {world} GPUs")
    B_weak = args.batch if (world > 1 and not args.weak) else 0  # the extra weak-scaling figure
    n_e2e = max(2, args.steps // 2)
    cap = args.ctx + args.warmup * 4 + args.steps * 4 + n_e2e + 16
    slots = max(B, B_weak)
    ctx = pkg.DecodeContext(gguf, device=local, max_batch=slots, max_ctx=cap, kv_bf16=True)
    cfg = dict(ctx.config, layer_is_dn=list(ctx.layer_is_deltanet))
    ctx.seed_state(seed=1 + rank, n_slots=slots, n_tokens=args.ctx, dn_std=0.1, conv_std=1.0, kv_std=1.0)
    ctx.step_graph(bool(args.graph))
    # an explicit stream: every kernel of the step and the timing events share it
    stream = torch.cuda.Stream(device=local)
    torch.cuda.set_stream(stream)
    tok = [torch.from_numpy(synth.seeded_tokens(slots, cfg["vocab"], seed=2 + rank)).cuda(),
           torch.empty(slots, dtype=torch.int32, device="cuda")]
    logits = torch.empty((slots, cfg["vocab"]), dtype=torch.float32, device="cuda")

    def dev_steps(n, i0=0, nb=B):
        for i in range(n):
            a, b = tok[(i0 + i) % 2], tok[(i0 + i + 1) % 2]
            ctx.decode_step_device(a, nb, logits, b, stream)

    # ---- device-resident timed region
    dev_steps(args.warmup)
    barrier()
    clock = ClockSampler(gpu_id_for(torch, local))
    time.sleep(0.3)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    pos0 = ctx.get_pos(0)
    clock.begin()
    e0.record(stream)
    dev_steps(args.steps, args.warmup)
    e1.record(stream)
    barrier()
    clocks = clock.stop()
    ms = e0.elapsed_time(e1)
    ms_max = max_over_ranks(ms)
    value = world * B * args.steps / (ms_max / 1e3)
    mean_len = pos0 + (args.steps + 1) / 2.0
    step_bytes = weight_bytes(cfg) + B * seq_bytes(cfg, int(mean_len))
    peak, peak_kind = measured_peaks()

    # ---- per-kernel device time: CUDA events around each launch on the same stream (a pass
    # of its own, since events between launches remove the overlap of dependent launches)
    ctx.profile(True)
    prof_pos0 = ctx.get_pos(0)
    dev_steps(args.steps, args.warmup + args.steps)
    torch.cuda.synchronize()
    prof = ctx.profile_read()
    ctx.profile(False)
    attn_len = int(prof_pos0 + (args.steps + 1) / 2.0)
    fam_bytes = {  # algorithmic bytes per step of each kernel family
        "q8_gemm": gemm_step_bytes(cfg, B),
        "attention": cfg["n_attn"] * attn_launch_bytes(cfg, B, attn_len),
        "deltanet": cfg["n_dn"] * dn_launch_bytes(cfg, B),
    }
    tc = ctx.tensor_core_gemm(B)
    what = {"q8_gemm": "q8_umma_gemm_kernel (Q8_0 GEMM family on tcgen05: every projection and the lm_head)"
                       if tc else "q8_gemm_kernel (Q8_0 GEMV family, mma.sync: every projection and the lm_head)",
            "attention": "attn_mma_kernel (GQA split-KV flash-decode, bf16 KV via TMA)",
            "deltanet": "deltanet_persist_kernel (fused conv1d, norms, gated delta rule, gated RMSNorm)"}
    prof_total = sum(v["ms"] for v in prof.values())
    kernels = {}
    for fam, nbytes in fam_bytes.items():
        f = prof[fam]
        ms = f["ms"] / args.steps
        gbs = nbytes / (ms / 1e3) / 1e9 if ms > 0 else 0.0
        kernels[fam] = {"kernel": what[fam], "bound": "hbm", "achieved": round(gbs, 1), "peak": peak,
                        "peak_kind": peak_kind, "unit": "GB/s", "frac": round(gbs / peak, 4),
                        "algorithmic_bytes_per_step": nbytes, "ms_per_step": round(ms, 4),
                        "launches_per_step": f["launches"] // args.steps,
                        "avg_launch_ms": round(f["ms"] / max(f["launches"], 1), 5),
                        "share_of_profiled_step": round(f["ms"] / prof_total, 4) if prof_total else None}
    if B == 64 and args.ctx == 8192:  # the captured workload
        for fam, t in NCU_TRAFFIC_PER_STEP.items():
            kernels[fam]["traffic"] = t
            kernels[fam]["traffic_unit"] = "bytes per step (ncu, one decode step of this workload)"
    dominant = max(kernels, key=lambda k: kernels[k]["ms_per_step"])
    roofline = dict(kernels[dominant], family=dominant)
    roofline.setdefault("traffic", None)

    # ---- end to end through the host-buffer API: rank 0 holds every sequence's token id;
    # with N > 1 the ids are scattered to the ranks and the next ids gathered back each step
    # (one host-to-device and one device-to-host copy of the batch's ids on rank 0)
    host_tok = synth.seeded_tokens(B * world, cfg["vocab"], seed=5)
    dec = None
    if world > 1:
        def dev_step(t, n):
            ctx.decode_step_device(t, t.numel(), None, n, torch.cuda.current_stream())
        dec = ShardedDecoder(None, B * world, step_fn_device=dev_step)
        for _ in range(2):  # warm-up: the first scatter / gather set up their NCCL channels
            host_tok = dec.step(host_tok if rank == 0 else None)
    else:
        _, host_tok = ctx.decode_step(host_tok, want_logits=False)
    barrier()
    t0 = time.perf_counter()
    for _ in range(n_e2e):
        if dec is None:
            _, host_tok = ctx.decode_step(host_tok, want_logits=False)
        else:
            host_tok = dec.step(host_tok if rank == 0 else None)
    barrier()
    ctx.sync()  # raises if a device pipeline wait timed out during the end-to-end steps
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    e2e = world * B * n_e2e / e2e_s

    # ---- weak scaling at N > 1: --batch sequences per GPU, the same timing rules
    weak = None
    if B_weak:
        dev_steps(args.warmup, 0, B_weak)
        barrier()
        w0, w1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        w0.record(stream)
        dev_steps(args.steps, args.warmup, B_weak)
        w1.record(stream)
        barrier()
        wms = max_over_ranks(w0.elapsed_time(w1))
        weak = {"value": round(world * B_weak * args.steps / (wms / 1e3), 1), "unit": "tok/s",
                "seq_per_gpu": B_weak, "global_batch": world * B_weak, "ms_per_step": round(wms / args.steps, 4),
                "scaling": "weak"}

    # ---- prefill of one 512-token prompt into slot 0 (after every timed decode phase; the
    # slot's seeded state is replaced), through the host-buffer API, median of 3 calls
    prefill = None
    if args.prefill_tokens > 0 and args.prefill_tokens < cap:
        n_pf = args.prefill_tokens
        prompt = synth.seeded_tokens(n_pf, cfg["vocab"], seed=3)
        pf_times = []
        for i in range(4):
            ctx.reset_slot(0)
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            ctx.prefill(0, prompt, want_logits=True)
            if i:  # the first call is the warm-up
                pf_times.append(time.perf_counter() - t0)
        pf_s = max_over_ranks(statistics.median(pf_times))
        prefill = {"value": round(world * n_pf / pf_s, 1), "unit": "tok/s", "prompt_tokens": n_pf,
                   "ms_per_prompt": round(pf_s * 1e3, 3), "sequences": world,
                   "timing": "host wall clock around the synchronous ab2_prefill call, median of 3, max over ranks"}

    # ---- the config-3 attention op at its largest cell (B=64, ctx 32K), rank 0 at N = 1, after
    # the timed region: the tensor-core flash-decode alone against the HBM copy peak
    attn32k = None
    if rank == 0 and world == 1 and not args.no_attn_op:
        peak, peak_kind = measured_peaks()
        fn, nbytes = attn_op_inputs(64, 32768, 16)
        ms_a = time_flushed(fn, 5, 3)
        if pkg.op_error():
            raise RuntimeError("tensor-core pipeline timeout in the attention op")
        gbs = nbytes / (ms_a / 1e3) / 1e9
        attn32k = {"op": "gqa flash-decode B=64 ctx=32768 Hq=8 Hkv=2 hd=256 (attn_mma_kernel, query prep, merge)",
                   "us_per_launch": round(ms_a * 1e3, 2), "algorithmic_bytes": nbytes,
                   "achieved_gbs": round(gbs, 1), "peak_gbs": peak, "peak_kind": peak_kind,
                   "frac": round(gbs / peak, 4), "iters": 5, "l2": "flushed before each launch"}
        del fn
        torch.cuda.empty_cache()

    # ---- CPU baseline (rank 0, N = 1): the oracle on one sequence of the same workload
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        v, n, dt, cores = cpu_reference_tokps(gguf, shape, args.ctx, seconds=args.cpu_seconds)
        cpu = {"value": round(v, 4), "unit": "tok/s", "cores": cores, "kind": "port",
               "sample": f"1 sequence, {n} greedy tokens at ctx {args.ctx} in {dt:.1f} s "
                         f"(the reference decodes one sequence at a time)"}

    if rank == 0:
        launches = ctx.launches_per_step(B) * args.steps
        print(json.dumps({
            "metric": METRIC, "value": round(value, 1), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 4), "higher_is_better": True,
            "scaling": "weak" if args.weak else "strong", "vs_baseline": None,
            "dtype": "f16 MMA operands (q*d rounded once), f32 accumulate, bf16 KV" if tc else
                     "exact Q8_0 weights x f16 hi/lo activations, f32 accumulate, bf16 KV",
            "data": "synthetic (seeded random Q8_0 weights, seeded DeltaNet/conv state, N(0,1) bf16 KV)",
            "config": {"workload": f"2B-shape Qwen3.5 hybrid greedy decode, Q8_0, {B * world} sequences "
                                   f"({B} per GPU), ctx {args.ctx} prefilled bf16 KV",
                       "model": "qwen35-hybrid-2B-shape (random init)",
                       "global_batch": B * world, "seq_len": args.ctx,
                       "parallelism": f"sequence-sharded x{world}, no collective",
                       "step_graph": bool(args.graph),
                       "l2": "inputs larger than L2 (each step reads ~%.1f GB)" % (step_bytes / 1e9)},
            "step_hbm": {"bytes_per_step": step_bytes, "achieved_gbs": round(step_bytes / (ms_max / args.steps) / 1e6, 1),
                         "frac": round(step_bytes / (ms_max / args.steps) / 1e6 / peak, 4)},
            "roofline": roofline,
            "kernels": kernels,
            "kernel_ms_per_step": {k: round(v["ms"] / args.steps, 4) for k, v in prof.items()},
            "weak_scaling": weak,
            "cpu_baseline": cpu,
            "prefill": prefill,
            "attention_op_b64_ctx32k": attn32k,
            "e2e": {"value": round(e2e, 1), "unit": "tok/s", "h2d_bytes_per_step": 4 * B * world,
                    "d2h_bytes_per_step": 4 * B * world,
                    "steps": n_e2e},
            "gpu_launches": launches,
            "clocks": clocks,
        }), flush=True)
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_split(args):
    """Decode-step latency of the head-parallel split over the torchrun ranks (N = 1: one GPU,
    unsplit). Device-resident steps timed with CUDA events (max over ranks), plus the same
    steps through the host-buffer API."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    pkg = load_pkg()
    from ane_infer_b200 import synth
    from ane_infer_b200.heads import open_split_context
    from ane_infer_b200.shard import max_over_ranks
    shape = synth.shape_2b()
    gguf = synth.build_model_gguf(shape, seed=0)
    B = args.batch
    n_e2e = max(2, args.steps // 2)
    cap = args.ctx + args.warmup + 2 * args.steps + n_e2e + 16
    if world > 1:
        ctx = open_split_context(gguf, local, B, cap, exact_max_batch=args.exact_max_batch)
    else:
        ctx = pkg.DecodeContext(gguf, device=local, max_batch=B, max_ctx=cap, exact_max_batch=args.exact_max_batch)
    split = ctx.split()
    cfg = ctx.config
    # every rank seeds its part of one state and feeds the same tokens
    ctx.seed_state(seed=1, n_slots=B, n_tokens=args.ctx, dn_std=0.1, conv_std=1.0, kv_std=1.0)
    ctx.step_graph(bool(args.graph))
    stream = torch.cuda.Stream(device=local)
    torch.cuda.set_stream(stream)
    tok = [torch.from_numpy(synth.seeded_tokens(B, cfg["vocab"], seed=2)).cuda(),
           torch.empty(B, dtype=torch.int32, device="cuda")]
    logits = torch.empty((B, cfg["vocab"]), dtype=torch.float32, device="cuda")

    def dev_steps(n, i0=0):
        for i in range(n):
            ctx.decode_step_device(tok[(i0 + i) % 2], B, logits, tok[(i0 + i + 1) % 2], stream)

    dev_steps(args.warmup)
    barrier()
    clock = ClockSampler(gpu_id_for(torch, local))
    time.sleep(0.3)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    clock.begin()
    e0.record(stream)
    dev_steps(args.steps, args.warmup)
    e1.record(stream)
    barrier()
    clocks = clock.stop()
    ms = max_over_ranks(e0.elapsed_time(e1)) / args.steps

    host_tok = synth.seeded_tokens(B, cfg["vocab"], seed=5)
    _, host_tok = ctx.decode_step(host_tok, want_logits=False)
    barrier()
    t0 = time.perf_counter()
    for _ in range(n_e2e):
        _, host_tok = ctx.decode_step(host_tok, want_logits=False)
    barrier()
    ctx.sync()
    e2e_ms = max_over_ranks(time.perf_counter() - t0) * 1e3 / n_e2e
    if rank == 0:
        tc = ctx.tensor_core_gemm(B)
        print(json.dumps({
            "metric": f"decode step latency, 2B-shape Q8_0 B={B} ctx {args.ctx}, head-parallel split",
            "value": round(ms, 4), "unit": "ms/step", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": False,
            "scaling": "strong", "vs_baseline": None,
            "dtype": "f16 MMA operands (q*d rounded once), f32 accumulate, bf16 KV" if tc else
                     "exact Q8_0 weights x f16 hi/lo activations, f32 accumulate, bf16 KV",
            "data": "synthetic (seeded random Q8_0 weights, seeded DeltaNet/conv state, N(0,1) bf16 KV)",
            "config": {"workload": f"2B-shape Qwen3.5 hybrid greedy decode, Q8_0, {B} sequence(s), "
                                   f"ctx {args.ctx} prefilled bf16 KV",
                       "model": "qwen35-hybrid-2B-shape (random init)", "global_batch": B, "seq_len": args.ctx,
                       "parallelism": (f"head-parallel x{world}: DeltaNet heads {split['dn_heads']} and kv heads "
                                       f"{split['kv_heads']} per GPU, NCCL all-gather after each split mixer")
                                      if world > 1 else "one GPU (sequence sharding of one sequence)",
                       "step_graph": bool(args.graph)},
            "e2e": {"value": round(e2e_ms, 4), "unit": "ms/step", "h2d_bytes_per_step": 4 * B,
                    "d2h_bytes_per_step": 4 * B, "steps": n_e2e},
            "gpu_launches": ctx.launches_per_step(B) * args.steps,
            "clocks": clocks,
        }), flush=True)
    ctx.close()  # its step graphs and NCCL communicator go before the process group
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_prefill(args):
    """Prefill throughput of one sequence on one GPU: --prefill N prompt tokens through
    ab2_prefill (128-token steps; 64 with --exact-max-batch 64), prompt tokens per second
    from the host clock around each
    call (the call is synchronous; its host-to-device copy of the ids and its device-to-host
    copy of the last logits are inside)."""
    import torch
    pkg = load_pkg()
    from ane_infer_b200 import synth
    shape = synth.shape_2b()
    gguf = synth.build_model_gguf(shape, seed=0)
    n = args.prefill
    ctx = pkg.DecodeContext(gguf, device=0, max_batch=args.prefill_batch, max_ctx=n + 8, kv_bf16=True,
                            exact_max_batch=args.exact_max_batch)
    cfg = ctx.config
    prompt = synth.seeded_tokens(n, cfg["vocab"], seed=3)
    for _ in range(args.warmup):
        ctx.reset_slot(0)
        ctx.prefill(0, prompt, want_logits=False)
    clock = ClockSampler(gpu_id_for(torch, 0))
    time.sleep(0.3)
    clock.begin()
    times = []
    for _ in range(args.steps):
        ctx.reset_slot(0)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        ctx.prefill(0, prompt, want_logits=True)
        times.append(time.perf_counter() - t0)
    clocks = clock.stop()
    ctx.profile(True)
    ctx.reset_slot(0)
    ctx.prefill(0, prompt, want_logits=False)
    prof = ctx.profile_read()
    ctx.profile(False)
    med = statistics.median(times)
    tc = ctx.tensor_core_gemm(64)
    ctx.close()
    # the reference's prompt loop runs one qwen35_forward_token per prompt token
    # (crates/cli/src/main.rs:358-362): the oracle's rate from position 0, about 10 s of tokens
    cpu = None
    if not args.no_cpu:
        v, n_cpu, dt, cores = cpu_reference_tokps(gguf, shape, 0, seconds=min(args.cpu_seconds, 10.0))
        cpu = {"value": round(v, 4), "unit": "tok/s", "cores": cores, "kind": "port",
               "sample": f"the first {n_cpu} tokens of one prompt, token by token, in {dt:.1f} s"}
    print(json.dumps({
        "metric": f"prefill tok/s, 2B-shape Q8_0, one sequence, {n}-token prompt",
        "value": round(n / med, 1), "unit": "tok/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(med * 1e3, 3), "higher_is_better": True, "scaling": "none", "vs_baseline": None,
        "dtype": "f16 MMA operands (q*d rounded once), f32 accumulate, bf16 KV" if tc else
                 "exact Q8_0 weights x f16 hi/lo activations, f32 accumulate, bf16 KV",
        "data": "synthetic (seeded random Q8_0 weights and prompt ids)",
        "config": {"workload": f"2B-shape Qwen3.5 hybrid prefill of {n} tokens in {64 if not tc else 128}-token steps",
                   "model": "qwen35-hybrid-2B-shape (random init)", "max_batch": args.prefill_batch,
                   "timing": "host wall clock around the synchronous call, median of steps"},
        "kernel_ms": {k: round(v["ms"], 3) for k, v in prof.items()},
        "gpu_launches_per_prefill": sum(v["launches"] for v in prof.values()),
        "cpu_baseline": cpu,
        "clocks": clocks,
    }), flush=True)


# --------------------------------------------------------------------------- op benchmarks
def cpu_op_baseline(op: str, B: int, M: int = 0, K: int = 0, ctx: int = 0, seconds: float = 5.0, blocks=None):
    """The oracle (CPU restatement of the reference, all host threads) on the op of BASELINE
    configs 2-4, in the op line's unit (microseconds for the whole batch B): the reference
    runs these per sequence, so a bounded sample of sequences is timed and scaled to B."""
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    from ane_infer_b200 import synth
    L = oracle.lib()
    L.oracle_set_threads(len(os.sched_getaffinity(0)))
    rng = np.random.default_rng(1)
    if op == "gemm":
        # q8_gemv is one vector per call (q8_gemv.rs:130): B calls per batch
        if blocks is None:
            blocks = synth.random_q8_0(rng, M, K, std=0.01)
        x = synth.bf16_round(rng.normal(size=K).astype(np.float32))
        y = np.empty(M, dtype=np.float32)
        call = lambda: L.oracle_q8_gemv(blocks, M, K, x, y)
        per, n_seq, what = B, 1, f"q8_gemv {M}x{K}, one vector per call"
        cores = L.oracle_max_threads() if M * K > 65536 else 1
    elif op == "recurrence":
        H, d, n_seq = 16, 128, min(B, 8)
        S = rng.normal(0, 0.1, size=(n_seq, H, d, d)).astype(np.float32)
        q, k, v = (synth.bf16_round(rng.normal(size=(n_seq, H, d)).astype(np.float32)) for _ in range(3))
        beta = rng.random((n_seq, H), dtype=np.float32)
        decay = rng.random((n_seq, H), dtype=np.float32)
        o = np.empty((n_seq, H, d), dtype=np.float32)
        call = lambda: L.oracle_gated_delta(S, q, k, v, beta, decay, n_seq, H, d, d, o)
        per, what = B / n_seq, f"gated delta rule, {n_seq} sequences x 16 heads per call"
        cores = L.oracle_max_threads()
    else:
        Hq, Hkv, hd, n_seq = 8, 2, 256, 1
        kc = rng.normal(size=(Hkv, ctx + 1, hd)).astype(np.float32)
        vc = rng.normal(size=(Hkv, ctx + 1, hd)).astype(np.float32)
        kv = oracle.KvOp(synth.bf16_round(kc), synth.bf16_round(vc))
        del kc, vc
        q, gate = rng.normal(size=(Hq, hd)), rng.normal(size=(Hq, hd))
        kn, vn = rng.normal(size=(Hkv, hd)), rng.normal(size=(Hkv, hd))
        call = lambda: kv(q, gate, kn, vn, ctx - 1, 1e7, 64, kv_bf16=True)
        per, what = B, f"GQA decode attention over {ctx} tokens, one sequence per call"
        cores = 1  # the restatement's attention runs on one thread, as the reference's loop does
    call()  # warm-up
    n, t0 = 0, time.perf_counter()
    while n == 0 or time.perf_counter() - t0 < seconds:
        call()
        n += 1
    dt = (time.perf_counter() - t0) / n
    return {"value": round(dt * per * 1e6, 2), "unit": "us per launch (whole batch)", "cores": cores,
            "kind": "port", "sample": f"{what}; {n} calls in {dt * n:.1f} s, scaled to batch {B}"}


def attn_op_inputs(B, ctx, extra):
    """Config-3 attention inputs (Hq 8, Hkv 2, hd 256, RoPE on 64 dims): projections, N(0,1)
    bf16 caches of ctx tokens (+ extra rows), positions ctx - 1; the call and its K/V bytes."""
    import torch
    pkg = load_pkg()
    Hq, Hkv, hd = 8, 2, 256
    cap = ctx + extra
    proj = torch.randn(B, Hq * 2 * hd + 2 * Hkv * hd, device="cuda")
    kc = torch.randn(B, Hkv, cap, hd, device="cuda").to(torch.bfloat16)
    vc = torch.randn(B, Hkv, cap, hd, device="cuda").to(torch.bfloat16)
    pos = torch.full((B,), ctx - 1, dtype=torch.int32, device="cuda")
    out = torch.empty(B, Hq * hd, device="cuda")
    st = torch.cuda.current_stream()
    fn = lambda: pkg.attn_decode(proj, kc, vc, cap, pos, B, Hq, Hkv, hd, True, None, None, 1e7, 64, ctx - 1, out, st)
    return fn, B * Hkv * ctx * hd * 2 * 2


def time_flushed(fn, iters, warmup):
    """Mean CUDA-event time in ms of fn() on the current stream, L2 flushed before each launch:
    one 256 MB buffer written and another read, so inputs that fit in L2 come from HBM and
    the write-back of the flush's own dirty lines is not charged to the timed launch."""
    import torch
    st = torch.cuda.current_stream()
    flush_w = torch.empty(64 << 20, dtype=torch.float32, device="cuda")
    flush_r = torch.ones(64 << 20, dtype=torch.float32, device="cuda")
    sink = torch.empty((), dtype=torch.float32, device="cuda")

    def flush_l2():
        flush_w.fill_(1.0)
        torch.sum(flush_r, dim=0, out=sink)

    for _ in range(warmup):
        flush_l2()
        fn()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iters)]
    for e0, e1 in ev:
        flush_l2()
        e0.record(st)
        fn()
        e1.record(st)
    torch.cuda.synchronize()
    return sum(e0.elapsed_time(e1) for e0, e1 in ev) / iters


def run_op(args):
    """One op of BASELINE configs 2-4 on cuda:0, timed with CUDA events; one JSON line."""
    import numpy as np
    import torch
    pkg = load_pkg()
    from ane_infer_b200 import synth
    torch.cuda.set_device(0)
    rng = np.random.default_rng(0)
    st = torch.cuda.Stream()
    torch.cuda.set_stream(st)
    peak, peak_kind = measured_peaks()
    B = args.batch
    if args.op == "gemm":
        M, K = args.m, args.k
        blocks = synth.random_q8_0(rng, M, K, std=0.01)
        w = pkg.Q8Tensor(blocks, M, K)
        x = torch.from_numpy(synth.bf16_round(rng.normal(size=(B, K)).astype(np.float32))).cuda()
        y = torch.empty((B, M), dtype=torch.float32, device="cuda")
        fn = lambda: pkg.q8_gemv(w, x, y, B, st)
        nbytes = M * K * 34 // 32 + B * K * 2 + B * M * 4
        label = f"q8 gemm {M}x{K} batch {B}"
    elif args.op == "recurrence":
        H = 16
        S = torch.from_numpy(rng.normal(0, 0.1, size=(B, H, 128, 128)).astype(np.float32)).cuda()
        q = torch.randn(B, H, 128, device="cuda").to(torch.bfloat16)
        k = torch.randn(B, H, 128, device="cuda").to(torch.bfloat16)
        v = torch.randn(B, H, 128, device="cuda").to(torch.bfloat16)
        beta = torch.rand(B, H, device="cuda")
        decay = torch.rand(B, H, device="cuda")
        o = torch.empty(B, H, 128, device="cuda")
        fn = lambda: pkg.gated_delta(S, q, k, v, beta, decay, o, B, H, st)
        nbytes = B * H * (2 * 128 * 128 * 4 + 3 * 128 * 2 + 128 * 4)
        label = f"gated delta rule B={B} H=16 dk=dv=128"
    else:
        fn, nbytes = attn_op_inputs(B, args.ctx, args.iters + args.warmup + 8)
        label = f"gqa flash-decode B={B} ctx={args.ctx} Hq=8 Hkv=2 hd=256"
    ms = time_flushed(fn, args.iters, args.warmup)
    if pkg.op_error():
        raise RuntimeError("tensor-core pipeline timeout")
    gbs = nbytes / (ms / 1e3) / 1e9
    cpu = None
    if not args.no_cpu:
        cpu = cpu_op_baseline(args.op, B, M=args.m, K=args.k, ctx=args.ctx, seconds=min(args.cpu_seconds, 10.0),
                              blocks=blocks if args.op == "gemm" else None)
    print(json.dumps({"op": label, "us_per_launch": round(ms * 1e3, 2), "algorithmic_bytes": nbytes,
                      "achieved_gbs": round(gbs, 1), "peak_gbs": peak, "peak_kind": peak_kind,
                      "frac": round(gbs / peak, 4), "iters": args.iters, "l2": "flushed before each launch",
                      "cpu_baseline": cpu}),
          flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=64,
                    help="sequences in total, split across the GPUs (with --weak: sequences per GPU)")
    ap.add_argument("--ctx", type=int, default=8192)
    ap.add_argument("--weak", action="store_true", help="run --batch sequences on every GPU (weak scaling)")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-attn-op", action="store_true",
                    help="skip the B=64 ctx-32K attention op figure of the decode line")
    ap.add_argument("--graph", type=int, choices=[0, 1], default=1,
                    help="1: replay each decode step from a captured CUDA graph; 0: stream launches")
    ap.add_argument("--op", choices=["gemm", "recurrence", "attention"], default=None,
                    help="time one op (BASELINE configs 2-4) instead of the decode step")
    ap.add_argument("--m", type=int, default=6144)
    ap.add_argument("--k", type=int, default=2048)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--prefill", type=int, default=0, help="time the prefill of this many prompt tokens instead")
    ap.add_argument("--prefill-tokens", type=int, default=512,
                    help="the decode run also times the prefill of one prompt of this many tokens (0: skip)")
    ap.add_argument("--prefill-batch", type=int, default=64, help="max_batch of the prefill context")
    ap.add_argument("--exact-max-batch", type=int, default=0,
                    help="--split heads and --prefill: the contexts' exact_max_batch (-1: one sequence on "
                         "tcgen05 too; 64: 64-token prefill steps on the exact path)")
    ap.add_argument("--split", choices=["sequences", "heads"], default="sequences",
                    help="heads: time the head-parallel split's decode-step latency (use --batch 1)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.op:
        run_op(args)
    elif args.prefill and args.impl == "ours":
        run_prefill(args)
    elif args.split == "heads" and args.impl == "ours":
        run_split(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
