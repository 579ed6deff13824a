"""CPU checks of the head-parallel split (the plan, the gather layout, and the partitioned
forward over gloo at world size 2). The GPU form runs in test_gpu_split.py."""
import os
import socket

import numpy as np
import pytest

from conftest import ROOT, load_pkg

CFG_2B = {"dn_heads": 16, "n_kv_heads": 2, "n_dn": 18, "n_attn": 6, "n_heads": 8, "head_dim": 256}
CFG_TINY = {"dn_heads": 8, "n_kv_heads": 2, "n_dn": 3, "n_attn": 1, "n_heads": 8, "head_dim": 128}


def test_split_plan_cases():
    load_pkg()
    from ane_infer_b200.heads import split_plan
    # 2B shape: both kinds split over 2 ranks; beyond 2 ranks the 2 kv heads stay whole
    p = [split_plan(CFG_2B, 2, r) for r in range(2)]
    assert [(q["dn_h0"], q["dn_heads"], q["kv_h0"], q["kv_heads"]) for q in p] == [(0, 8, 0, 1), (8, 8, 1, 1)]
    for W in (4, 8):
        for r in range(W):
            q = split_plan(CFG_2B, W, r)
            assert q["dn_split"] and not q["kv_split"]
            assert (q["dn_h0"], q["dn_heads"], q["kv_h0"], q["kv_heads"]) == (r * 16 // W, 16 // W, 0, 2)
    # f32 cache: attention never splits
    assert not split_plan(CFG_2B, 2, 1, kv_bf16=False)["kv_split"]
    # tiny shape: 8 DeltaNet heads of 128 columns; 8 ranks leave 128 columns each (two K tiles)
    q = split_plan(CFG_TINY, 8, 7)
    assert (q["dn_h0"], q["dn_heads"]) == (7, 1)
    assert split_plan(CFG_TINY, 1, 0) == {"dn_split": False, "kv_split": False, "dn_h0": 0, "dn_heads": 8,
                                          "kv_h0": 0, "kv_heads": 2}
    with pytest.raises(ValueError):
        split_plan(dict(CFG_TINY, dn_heads=3, n_kv_heads=3), 2, 0)  # nothing divides
    with pytest.raises(ValueError):
        split_plan(CFG_TINY, 2, 2)


# Host restatement of the two activation layouts (csrc/common.cuh: xfrag_offset, x16_offset)
def xfrag_offsets(K, batch):
    from ane_infer_b200.heads import xfrag_ntile
    ntile = xfrag_ntile(batch)
    packed = batch <= 4
    nt = 1 if packed else (batch + 7) // 8
    b, k, hl = np.meshgrid(np.arange(batch), np.arange(K), np.arange(2), indexing="ij")
    kb, kk = k >> 5, k & 31
    s16, r = kk >> 4, kk & 15
    ihi, r8 = r >> 3, r & 7
    t, p = r8 >> 1, r8 & 1
    if packed:
        tile, n = np.zeros_like(b), b + 4 * hl
    else:
        tile, n = hl * nt + (b >> 3), b & 7
    lane = n * 4 + t
    off = ((kb * ntile + tile) * 32 + lane) * 16 + (s16 * 2 + ihi) * 4 + p * 2
    return off, k, K // 32 * ntile * 512


def x16_offsets(K, batch):
    b, k = np.meshgrid(np.arange(batch), np.arange(K), indexing="ij")
    kt, kk = k >> 6, k & 63
    j, e = kk >> 3, kk & 7
    off = (kt * 64 + b) * 128 + ((j ^ (b & 7)) << 4) + e * 2
    return off, k, (K + 63) // 64 * 64 * 128


@pytest.mark.parametrize("tensor_core", [False, True])
def test_gather_chunk_is_the_ranks_columns(tensor_core):
    """Every f16 a rank writes (its K/world columns, all batch rows, both hi/lo parts) lies in
    its own byte range [r*chunk, (r+1)*chunk) of the buffer, and the ranges tile it."""
    load_pkg()
    from ane_infer_b200.heads import gather_chunk_bytes
    for K in (1024, 2048):
        for batch in ((1, 3, 4, 5, 9, 33, 64) if not tensor_core else (2, 9, 64)):
            off, k, total = (x16_offsets if tensor_core else xfrag_offsets)(K, batch)
            for W in (2, 4, 8):
                if K % (64 * W):
                    continue
                chunk = gather_chunk_bytes(K, batch, W, tensor_core)
                assert chunk * W == total
                owner = k // (K // W)
                assert np.all(off >= owner * chunk) and np.all(off + 2 <= (owner + 1) * chunk), (K, batch, W)
            # distinct elements never share bytes
            assert np.unique(off).size == off.size


# ---------------------------------------------------------------- partitioned forward (gloo)
def _split_forward(m, st, token, pos, plan, gather):
    """numpy_ref.Model.forward with this rank's heads only (state `st` holds only them);
    `gather(local, K)` all-gathers a rank's output columns into the full vector."""
    from numpy_ref import attn_core, gated_delta, rmsnorm, sigmoid, silu
    t = m.t
    x = t["token_embd.weight"][token].copy()
    for l in range(m.n_layers):
        p = f"blk.{l}."
        xn = rmsnorm(x, t[p + "attn_norm.weight"], m.eps)
        if m.is_dn[l]:
            D, H, h0, hl = m.dim, m.H, plan["dn_h0"], plan["dn_heads"]
            s = st[l]
            qkv = m.mv(t[p + "attn_qkv.weight"], xn)
            s["conv"] = np.concatenate([s["conv"][:, 1:], qkv[:, None]], axis=1)
            c = silu((s["conv"] * t[p + "ssm_conv1d.weight"]).sum(axis=1))
            q, k, v = c[:D].reshape(H, 128), c[D:2 * D].reshape(H, 128), c[2 * D:].reshape(H, 128)
            q, k, v = q[h0:h0 + hl], k[h0:h0 + hl], v[h0:h0 + hl]
            q = q / np.sqrt((q * q).sum(1, keepdims=True) + 1e-12) / np.sqrt(128)
            k = k / np.sqrt((k * k).sum(1, keepdims=True) + 1e-12)
            beta = sigmoid(m.mv(t[p + "ssm_beta.weight"], xn))[h0:h0 + hl]
            a = m.mv(t[p + "ssm_alpha.weight"], xn) + t[p + "ssm_dt.bias"]
            decay = np.exp(t[p + "ssm_a"] * np.log1p(np.exp(a)))[h0:h0 + hl]
            o = np.empty((hl, 128))
            for j in range(hl):
                o[j], s["S"][j] = gated_delta(s["S"][j], q[j], k[j], v[j], beta[j], decay[j])
            gate = m.mv(t[p + "attn_gate.weight"], xn)[h0 * 128:(h0 + hl) * 128]
            normed = np.concatenate([rmsnorm(o[j], t[p + "ssm_norm.weight"], m.eps) for j in range(hl)])
            local = normed * silu(gate)
            full = gather(local, H * 128) if plan["dn_split"] else local
            x = x + m.mv(t[p + "ssm_out.weight"], full)
        else:
            hd, g, kh0, khl = m.hd, m.Hq // m.Hkv, plan["kv_h0"], plan["kv_heads"]
            qf = m.mv(t[p + "attn_q.weight"], xn).reshape(m.Hq, 2 * hd)[kh0 * g:(kh0 + khl) * g]
            k = m.mv(t[p + "attn_k.weight"], xn).reshape(m.Hkv, hd)[kh0:kh0 + khl]
            v = m.mv(t[p + "attn_v.weight"], xn).reshape(m.Hkv, hd)[kh0:kh0 + khl]
            o = attn_core(qf[:, :hd], qf[:, hd:], k, v, st[l]["k"], st[l]["v"], pos, m.base, hd,
                          t[p + "attn_q_norm.weight"], t[p + "attn_k_norm.weight"]).reshape(-1)
            full = gather(o, m.Hq * hd) if plan["kv_split"] else o
            x = x + m.mv(t[p + "attn_output.weight"], full)
        x = x + m.ffn(l, rmsnorm(x, t[p + "post_attention_norm.weight"], m.eps))
    return m.mv(m.lm, rmsnorm(x, t["output_norm.weight"], m.eps))


def _seeded_state(m, cap, n_tokens, seed):
    rng = np.random.default_rng(seed)
    st = m.new_state(cap)
    for l, s in enumerate(st):
        if m.is_dn[l]:
            s["S"][:] = rng.normal(0, 0.1, s["S"].shape)
            s["conv"][:] = rng.normal(0, 1.0, s["conv"].shape)
        else:
            s["k"][:, :n_tokens] = rng.normal(0, 1.0, (m.Hkv, n_tokens, m.hd))
            s["v"][:, :n_tokens] = rng.normal(0, 1.0, (m.Hkv, n_tokens, m.hd))
    return st


def _local_state(m, st, plan):
    out = []
    for l, s in enumerate(st):
        if m.is_dn[l]:
            h0, hl = plan["dn_h0"], plan["dn_heads"]
            out.append({"S": s["S"][h0:h0 + hl].copy(), "conv": s["conv"].copy()})
        else:
            a, n = plan["kv_h0"], plan["kv_heads"]
            out.append({"k": s["k"][a:a + n].copy(), "v": s["v"][a:a + n].copy()})
    return out


def _split_worker(rank, world, port, result_path):
    import sys
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        from conftest import load_pkg as lp
        lp()
        import numpy_ref
        from ane_infer_b200 import synth
        from ane_infer_b200.heads import split_plan
        m = numpy_ref.Model(synth.build_model_gguf(synth.tiny_shape(), seed=0))
        cfg = {"dn_heads": m.H, "n_kv_heads": m.Hkv, "n_dn": sum(m.is_dn), "n_attn": m.n_layers - sum(m.is_dn),
               "n_heads": m.Hq, "head_dim": m.hd}
        plan = split_plan(cfg, world, rank)

        def gather(local, K):
            parts = [torch.empty(local.size, dtype=torch.float64) for _ in range(world)]
            dist.all_gather(parts, torch.from_numpy(np.ascontiguousarray(local)))
            full = torch.cat(parts).numpy()
            assert full.size == K
            return full

        cap, n0 = 64, 20
        full_st = _seeded_state(m, cap, n0, seed=7)  # the same on every rank
        st = _local_state(m, full_st, plan)
        tok, lines = 11, []
        for i in range(3):
            want = m.forward(full_st, tok, n0 + i)
            got = _split_forward(m, st, tok, n0 + i, plan, gather)
            lines.append(f"step {i} {int(np.array_equal(got, want))}")
            tok = int(np.argmax(want))
        # the rank's state is its part of the full state after the same steps
        same = all(np.array_equal(st[l]["S"], full_st[l]["S"][plan["dn_h0"]:plan["dn_h0"] + plan["dn_heads"]])
                   if m.is_dn[l] else
                   np.array_equal(st[l]["k"], full_st[l]["k"][plan["kv_h0"]:plan["kv_h0"] + plan["kv_heads"]])
                   for l in range(m.n_layers))
        lines.append(f"state {int(same)}")
        with open(f"{result_path}.{rank}", "w") as f:
            f.write("\n".join(lines))
    finally:
        dist.destroy_process_group()


def test_split_forward_gloo_world2(tmp_path):
    """Each rank runs only its DeltaNet and kv heads on its part of the state and all-gathers
    the mixer outputs: the logits equal the unsplit forward's exactly (the per-head maths never
    mixes heads before the output projection), and the rank's state stays its part of the
    unsplit state."""
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    out = tmp_path / "res"
    mp.start_processes(_split_worker, args=(2, port, str(out)), nprocs=2, join=True, start_method="spawn")
    for r in range(2):
        lines = (tmp_path / f"res.{r}").read_text().split("\n")
        assert lines == ["step 0 1", "step 1 1", "step 2 1", "state 1"], (r, lines)
