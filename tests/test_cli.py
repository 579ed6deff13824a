"""The command-line benchmark ab2_bench (the counterpart of the reference CLI's `bench`,
crates/cli/src/main.rs:251-508), on CPU: its argument handling, and its prompt and greedy
feedback loop, run against a test double of libab2.so (tests/stub_ab2.c) that logs every call.
Without a GPU, the real library must make it fail cleanly."""
import importlib.util
import json
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "ane-infer_b200")


def _build_mod():
    spec = importlib.util.spec_from_file_location("ab2_build_cli", os.path.join(PKG, "build.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="module")
def stub_cli(tmp_path_factory):
    d = tmp_path_factory.mktemp("cli")
    subprocess.run(["gcc", "-O1", "-shared", "-fPIC", "-I", os.path.join(ROOT, "include"),
                    os.path.join(ROOT, "tests", "stub_ab2.c"), "-o", str(d / "libab2.so")], check=True)
    exe = _build_mod().build_cli(out=str(d / "ab2_bench"), lib_dir=str(d))
    model = d / "model.gguf"
    model.write_bytes(b"GGUF" + bytes(60))
    return exe, str(model), d


def run(exe, *args, env=None):
    e = dict(os.environ)
    e.update(env or {})
    return subprocess.run([exe, *args], capture_output=True, text=True, env=e, timeout=60)


def read_log(path):
    return [line.split() for line in open(path).read().splitlines()]


@pytest.mark.parametrize("B,pp,tg,kv,graph", [(1, 4, 6, "bf16", 1), (3, 2, 5, "f32", 0)])
def test_prompt_then_greedy_feedback(stub_cli, tmp_path, B, pp, tg, kv, graph):
    exe, model, _ = stub_cli
    log = tmp_path / "calls.log"
    r = run(exe, "-m", model, "-pp", str(pp), "-tg", str(tg), "-b", str(B), "--kv", kv, "--graph", str(graph),
            "--seed", "3", env={"STUB_LOG": str(log)})
    assert r.returncode == 0, r.stderr
    out = json.loads(r.stdout)
    assert (out["batch"], out["prompt_tokens"], out["gen_tokens"], out["kv"], out["graph"]) == (B, pp, tg, kv, graph)
    assert "Speed:" in r.stderr and "Tokens: %d" % tg in r.stderr
    calls = read_log(log)
    # create(device 0, max_batch B, max_ctx pp + tg + 2, kv flag), graph switch, prompt, steps, destroy
    assert calls[0] == ["create", "0", str(B), str(pp + tg + 2), "1" if kv == "bf16" else "0"]
    assert calls[1] == ["graph", str(graph), "0", "0", "0"]
    steps = [c for c in calls if c[0] == "step"]
    prefills = [c for c in calls if c[0] == "prefill"]
    assert calls[-1][0] == "destroy"
    if kv == "bf16":
        # the prompt of every sequence goes through one prefill call (slot, n, first id,
        # last id, next id, device); the generation starts from slot 0's next id
        assert [(int(c[1]), int(c[2])) for c in prefills] == [(b, pp) for b in range(B)]
        assert len(steps) == tg
        first_gen = int(prefills[0][5])
        assert out["prompt"][0] == int(prefills[0][3]) and out["prompt"][-1] == int(prefills[0][4])
        assert len(out["prompt"]) == pp and all(0 <= t < 1000 for t in out["prompt"])
    else:
        # the f32 cache has no prefill: one decode step per prompt position
        assert not prefills and len(steps) == pp + tg
        assert out["prompt"] == [int(s[2]) for s in steps[:pp]]
        first_gen = int(steps[pp - 1][3])
        steps = steps[pp:]
    assert all(int(s[1]) == B for s in steps)
    tok0 = [int(s[2]) for s in steps]
    nxt0 = [int(s[3]) for s in steps]
    # each generated step feeds the previous step's greedy token, and the reported tokens
    # are slot 0's generated ids in order
    assert tok0[0] == first_gen
    for k in range(1, tg):
        assert tok0[k] == nxt0[k - 1], k
    assert out["tokens"] == tok0


def test_prompt_by_decode_steps(stub_cli, tmp_path):
    """--prefill 0: the prompt runs as one decode step per position for all sequences."""
    exe, model, _ = stub_cli
    log = tmp_path / "calls.log"
    r = run(exe, "-m", model, "-pp", "3", "-tg", "2", "-b", "2", "--prefill", "0", env={"STUB_LOG": str(log)})
    assert r.returncode == 0, r.stderr
    calls = read_log(log)
    steps = [c for c in calls if c[0] == "step"]
    assert not [c for c in calls if c[0] == "prefill"] and len(steps) == 5
    assert json.loads(r.stdout)["prompt"] == [int(s[2]) for s in steps[:3]]


def test_seeded_context_without_prompt(stub_cli, tmp_path):
    exe, model, _ = stub_cli
    log = tmp_path / "calls.log"
    r = run(exe, "-m", model, "--ctx", "5", "-pp", "0", "-tg", "3", "-b", "2", "--seed", "7",
            env={"STUB_LOG": str(log)})
    assert r.returncode == 0, r.stderr
    out = json.loads(r.stdout)
    assert (out["ctx"], out["prompt_tokens"], out["prompt"]) == (5, 0, [])
    calls = read_log(log)
    assert calls[0] == ["create", "0", "2", str(5 + 0 + 3 + 2), "1"]
    assert calls[2] == ["seed", "7", "2", "5", "0", "0"]  # both slots start at position 5 (device 0)
    steps = [c for c in calls if c[0] == "step"]
    assert len(steps) == 3 and 0 <= int(steps[0][2]) < 1000
    assert [int(s[2]) for s in steps[1:]] == [int(s[3]) for s in steps[:-1]]
    assert out["tokens"] == [int(s[2]) for s in steps]


def test_one_thread_and_context_per_gpu(stub_cli, tmp_path):
    exe, model, _ = stub_cli
    log = tmp_path / "calls.log"
    G, B, pp, tg = 3, 2, 2, 4
    r = run(exe, "-m", model, "--gpus", str(G), "-d", "1", "-b", str(B), "-pp", str(pp), "-tg", str(tg),
            env={"STUB_LOG": str(log)})
    assert r.returncode == 0, r.stderr
    out = json.loads(r.stdout)
    assert out["gpus"] == G and len(out["gen_tok_s_per_gpu"]) == G
    calls = read_log(log)
    creates = sorted(int(c[1]) for c in calls if c[0] == "create")
    assert creates == [1, 2, 3]
    assert sum(c[0] == "destroy" for c in calls) == G
    by_dev, pf_dev = {}, {}
    for c in calls:
        if c[0] == "step":
            by_dev.setdefault(int(c[5]), []).append(c)
        if c[0] == "prefill":
            pf_dev.setdefault(int(c[6]), []).append(c)
    assert sorted(by_dev) == [1, 2, 3] and sorted(pf_dev) == [1, 2, 3]
    for dev, steps in by_dev.items():
        assert len(steps) == tg and len(pf_dev[dev]) == B, dev
        tok0 = [int(s[2]) for s in steps]
        nxt0 = [int(s[3]) for s in steps]
        assert tok0[0] == int(pf_dev[dev][0][5])
        assert all(tok0[k] == nxt0[k - 1] for k in range(1, tg)), dev
    # each GPU decodes its own sequences: prompts are seeded per GPU; the output reports GPU 1's
    prompts = {dev: (int(pf[0][3]), int(pf[0][4])) for dev, pf in pf_dev.items()}
    assert len(set(prompts.values())) == G
    assert (out["prompt"][0], out["prompt"][-1]) == prompts[1]


def test_device_threads_start_together(stub_cli, tmp_path):
    """The device threads pass a common gate after upload and seeding: no GPU starts decoding
    while another is still uploading, so the whole-job rate spans first start to last end."""
    exe, model, _ = stub_cli
    log = tmp_path / "calls.log"
    r = run(exe, "-m", model, "--gpus", "3", "-b", "2", "--ctx", "8", "-pp", "2", "-tg", "3",
            env={"STUB_LOG": str(log), "STUB_SLOW_CREATE_DEVICE": "1"})
    assert r.returncode == 0, r.stderr
    calls = read_log(log)
    kinds = [c[0] for c in calls]
    last_seed = max(i for i, k in enumerate(kinds) if k == "seed")
    first_step = min(i for i, k in enumerate(kinds) if k in ("step", "prefill"))
    assert last_seed < first_step, kinds


def test_one_failing_device_does_not_hold_the_others(stub_cli, tmp_path):
    exe, model, _ = stub_cli
    log = tmp_path / "calls.log"
    r = run(exe, "-m", model, "--gpus", "3", "-b", "2", "-pp", "2", "-tg", "3",
            env={"STUB_LOG": str(log), "STUB_FAIL_CREATE_DEVICE": "1"})
    assert r.returncode == 1
    assert "GPU 1: ab2_create failed: stub: no CUDA device available" in r.stderr
    steps = {int(c[5]) for c in read_log(log) if c[0] == "step"}
    assert steps == {0, 2}  # the other devices ran to the end


def test_prompt_ids_depend_on_seed_and_slot(stub_cli, tmp_path):
    exe, model, _ = stub_cli
    firsts = []
    for seed in ("0", "1"):
        log = tmp_path / f"s{seed}.log"
        assert run(exe, "-m", model, "-pp", "3", "-tg", "1", "-b", "2", "--seed", seed,
                   env={"STUB_LOG": str(log)}).returncode == 0
        pf = [c for c in read_log(log) if c[0] == "prefill"]
        firsts.append([(int(c[3]), int(c[4])) for c in pf])  # each slot's first and last prompt id
    assert firsts[0] != firsts[1]
    assert firsts[0][0] != firsts[0][1]  # slots 0 and 1 get different prompts


@pytest.mark.parametrize("args,code,msg", [
    ((), 2, "-m MODEL.gguf is required"),
    (("-m",), 2, "needs a value"),
    (("-m", "x", "-pp", "-1"), 2, "bad value for -pp"),
    (("-m", "x", "--ctx", "x"), 2, "bad value for --ctx"),
    (("-m", "x", "--gpus", "0"), 2, "bad value for --gpus"),
    (("-m", "x", "--graph", "2"), 2, "bad value for --graph"),
    (("-m", "x", "--kv", "f16"), 2, "bad value for --kv"),
    (("-m", "x", "--frobnicate", "1"), 2, "unknown option"),
])
def test_bad_usage(stub_cli, args, code, msg):
    r = run(stub_cli[0], *args)
    assert r.returncode == code and msg in r.stderr and "usage:" in r.stderr


def test_help(stub_cli):
    r = run(stub_cli[0], "--help")
    assert r.returncode == 0 and r.stdout.startswith("usage: ab2_bench")


def test_failures_report_the_ab2_message(stub_cli, tmp_path):
    exe, model, d = stub_cli
    r = run(exe, "-m", str(tmp_path / "missing.gguf"))
    assert r.returncode == 1 and "cannot read" in r.stderr
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"NOPE" + bytes(8))
    r = run(exe, "-m", str(bad))
    assert r.returncode == 1 and "reading the GGUF failed: stub: not a GGUF file" in r.stderr
    r = run(exe, "-m", model, env={"STUB_FAIL_CREATE": "1"})
    assert r.returncode == 1 and "ab2_create failed: stub: no CUDA device available" in r.stderr


def test_real_library_without_gpu_fails_cleanly(tiny_gguf, tmp_path):
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present: this checks the no-device path")
    exe = os.path.join(PKG, "ab2_bench")
    if not os.path.exists(exe):
        _build_mod().build()
    model = tmp_path / "tiny.gguf"
    model.write_bytes(bytes(tiny_gguf))
    r = run(exe, "-m", str(model), "-pp", "2", "-tg", "2")
    assert r.returncode == 1 and "ab2_create failed" in r.stderr
    assert "Model: 4 layers (3 DeltaNet, 1 attention)" in r.stderr
    # every device thread reports its own failure, read from its own thread's error slot
    r = run(exe, "-m", str(model), "-pp", "2", "-tg", "2", "--gpus", "2")
    assert r.returncode == 1
    assert "GPU 0: ab2_create failed: no CUDA device available" in r.stderr
    assert "GPU 1: ab2_create failed: no CUDA device available" in r.stderr
