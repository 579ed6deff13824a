"""GPU, two GPUs: the head-parallel split (ab2_create_tp). Each rank runs half of the DeltaNet
and kv heads and holds only their state; the mixer outputs are all-gathered with NCCL.

On the exact (mma.sync) path with contexts short enough for one attention split, every
per-head computation and every replicated GEMM is the one a single GPU does, so the logits
of both ranks equal the single-GPU logits bit for bit, and each rank's state is its part of
the single-GPU state. At long contexts the attention split plan follows the rank's own head
count (more splits per head), which changes only the merge's summation order. The tcgen05
path's K-split sums add in arrival order, so there the ranks agree with one GPU within its
declared tolerance."""
import os
import time

import numpy as np
import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu

LONG_TOL = 1e-4   # max|diff| <= LONG_TOL * max|logits| per row: attention merge order only
TC_TOL = 2e-3     # tcgen05 path: f16 operands, K-split sums in arrival order


def _need_two(cuda):
    if cuda.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")


def _run(pkg, gguf, device, tp, B, n0, steps, exact, graph=False, prompt=0):
    """Seeded state at n0 tokens (or, with prompt > 0, a prefill of that many tokens into each
    slot), then `steps` greedy steps of slots [0, B) from fixed tokens: the logits of every
    step (the prefills' last-token logits first), the split info, layer 0's recurrent state
    and the first attention layer's K cache of slot 0."""
    from ane_infer_b200 import synth
    ctx = pkg.DecodeContext(gguf, device=device, max_batch=B, max_ctx=n0 + prompt + steps + 8,
                            exact_max_batch=(64 if prompt else B) if exact else 0, tp=tp)
    try:
        out = []
        if prompt:
            for b in range(B):
                lg, _ = ctx.prefill(b, synth.seeded_tokens(prompt, ctx.config["vocab"], seed=60 + b))
                out.append(lg[None])
            n0 = prompt
        else:
            ctx.seed_state(seed=5, n_slots=B, n_tokens=n0)
        ctx.step_graph(graph)
        toks = synth.seeded_tokens(B, ctx.config["vocab"], seed=9)
        for _ in range(steps):
            lg, toks = ctx.decode_step(toks)
            out.append(lg)
        out = [np.concatenate(out[:B])] + out[B:] if prompt else out
        attn = ctx.layer_is_deltanet.index(False)
        rec, _ = ctx.get_dn_state(0, 0)
        k, _ = ctx.get_kv(attn, 0, n0 + steps)
        return {"logits": np.stack(out), "split": ctx.split(), "rec": rec, "k": k}
    finally:
        ctx.close()


def _worker(rank, world, tp_id, gguf_path, out_path, cases):
    import sys
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import pickle

    import torch  # noqa: F401  (the process's NCCL is the one torch loads)
    from conftest import load_pkg
    pkg = load_pkg()
    gguf = np.fromfile(gguf_path, dtype=np.uint8)
    res = {}
    for name, case in cases.items():
        res[name] = _run(pkg, gguf, rank, (rank, world, tp_id[name]), *case)
    with open(f"{out_path}.{rank}", "wb") as f:
        pickle.dump(res, f)


def _split_run(pkg, tmp_path, gguf, cases):
    import pickle

    import torch.multiprocessing as mp
    path = tmp_path / "model.gguf"
    np.asarray(gguf, dtype=np.uint8).tofile(path)
    ids = {name: pkg.tp_unique_id() for name in cases}
    out = tmp_path / "res"
    pc = mp.start_processes(_worker, args=(2, ids, str(path), str(out), cases), nprocs=2, join=False,
                            start_method="spawn")
    # a rank that fails before joining the split leaves the other waiting in the NCCL
    # bootstrap (on the host): end both after a deadline instead of waiting for good
    deadline = time.monotonic() + 600
    while not pc.join(timeout=5):
        if time.monotonic() > deadline:
            for p in pc.processes:
                if p.is_alive():
                    p.kill()
            pytest.fail("split ranks did not finish within 600 s")
    res = []
    for r in range(2):
        with open(f"{out}.{r}", "rb") as f:
            res.append(pickle.load(f))
    return res


def _rows_close(got, ref, tol):
    for g, r in zip(got.reshape(-1, got.shape[-1]), ref.reshape(-1, ref.shape[-1])):
        assert float(np.max(np.abs(g.astype(np.float64) - r))) <= tol * float(np.max(np.abs(r)))


CASES_TINY = {
    "short": (3, 40, 4, True, False),       # one attention split: bit-identical
    "short_graph": (3, 40, 4, True, True),  # the same through the captured step graph
    "long": (1, 3000, 3, True, False),      # split plans differ: merge order only
    "tc": (9, 40, 1, False, False),         # tcgen05 path
    "prefill": (2, 0, 3, True, False, 100),  # GPU prefill of 100 tokens per slot, then decode
}


def test_split_tiny_matches_one_gpu(pkg, cuda, synth, tiny_gguf, tmp_path):
    _need_two(cuda)
    ranks = _split_run(pkg, tmp_path, tiny_gguf, CASES_TINY)
    cfg = pkg.inspect_gguf(tiny_gguf)
    for r, res in enumerate(ranks):
        s = res["short"]["split"]
        assert (s["rank"], s["world"], s["dn_h0"], s["dn_heads"], s["kv_h0"], s["kv_heads"]) == \
            (r, 2, r * cfg["dn_heads"] // 2, cfg["dn_heads"] // 2, r, 1)
    for name, case in CASES_TINY.items():
        exact = case[3]
        one = _run(pkg, tiny_gguf, 0, None, *case)
        r0, r1 = ranks[0][name], ranks[1][name]
        if exact:
            # replicated GEMMs on identical gathered inputs: the ranks agree bit for bit
            assert np.array_equal(r0["logits"], r1["logits"]), name
        if name.startswith("short") or name == "prefill":
            assert np.array_equal(r0["logits"], one["logits"]), name
            # each rank holds exactly its heads of the single-GPU state (zeros elsewhere)
            for r, res in enumerate((r0, r1)):
                h = cfg["dn_heads"] // 2
                assert np.array_equal(res["rec"][r * h:(r + 1) * h], one["rec"][r * h:(r + 1) * h])
                assert not res["rec"][(1 - r) * h:(2 - r) * h].any()
                if name.startswith("short"):
                    assert np.array_equal(res["k"][r], one["k"][r])
        else:
            # the first step (later ones may follow a near-tie greedy pick apart)
            tol = LONG_TOL if name == "long" else TC_TOL
            _rows_close(r0["logits"][:1], one["logits"][:1], tol)
            _rows_close(r1["logits"][:1], one["logits"][:1], tol)


def test_split_2b_b1_matches_one_gpu(pkg, cuda, synth, tmp_path):
    """The 2B shape at one sequence (the latency case of the split): 16 DeltaNet heads and 2
    kv heads over two GPUs, bit-identical to one GPU at a short context."""
    _need_two(cuda)
    gguf = synth.build_model_gguf(synth.shape_2b(), seed=0)
    cases = {"b1": (1, 100, 3, True, True)}
    ranks = _split_run(pkg, tmp_path, gguf, cases)
    one = _run(pkg, gguf, 0, None, 1, 100, 3, True, True)
    for res in ranks:
        assert np.array_equal(res["b1"]["logits"], one["logits"])
        assert res["b1"]["split"]["dn_heads"] == 8 and res["b1"]["split"]["kv_heads"] == 1


def test_create_tp_world1_is_unsplit(pkg, cuda, tiny_gguf):
    with pkg.DecodeContext(tiny_gguf, tp=(0, 1, None)) as ctx:
        assert ctx.split() == {"rank": 0, "world": 1, "dn_h0": 0, "dn_heads": 8, "kv_h0": 0, "kv_heads": 2}
