"""CPU, world size 2 over gloo: the sequence-sharded decode plumbing (scatter of token ids,
per-rank step, gather of next ids in global order, ragged and empty shards), in both the
host-array and the tensor (device) step form, and the max-over-ranks timing reduction. The
per-rank step is a host function here; on a GPU box it is DecodeContext.decode_step or
decode_step_device."""
import os
import socket

import numpy as np
import pytest

from conftest import ROOT, load_pkg


def test_shard_range_covers_batch_once():
    pkg = load_pkg()
    from ane_infer_b200.shard import shard_range
    for B in (0, 1, 5, 63, 64, 257):
        for world in (1, 2, 3, 8):
            spans = [shard_range(B, world, r) for r in range(world)]
            assert sum(c for _, c in spans) == B
            assert max(c for _, c in spans) - min(c for _, c in spans) <= 1
            pos = 0
            for s, c in spans:
                assert s == pos
                pos += c
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


def fake_step(start):
    # next id depends on the token and on the sequence's global index, so a misrouted
    # token or a misplaced result changes the answer
    return lambda toks: ((toks.astype(np.int64) * 31 + 7 + start + np.arange(len(toks))) % 1000).astype(np.int32)


def _worker(rank, world, port, result_path):
    import sys
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        from conftest import load_pkg as lp
        lp()
        from ane_infer_b200.shard import ShardedDecoder, max_over_ranks, shard_range
        lines = []
        for mode in ("host", "device"):
            for B in (5, 1, 8, 0):
                start, _ = shard_range(B, world, rank)
                if mode == "host":
                    dec = ShardedDecoder(fake_step(start), B)
                else:
                    # the tensor form of the step (on a GPU box: DecodeContext.decode_step_device
                    # reading and writing device ids), here on CPU tensors under gloo
                    def dev_step(t, n, f=fake_step(start)):
                        n.copy_(torch.from_numpy(f(t.numpy())))
                    dec = ShardedDecoder(None, B, step_fn_device=dev_step)
                toks = np.arange(B, dtype=np.int32) * 13 + 2 if rank == 0 else None
                for _ in range(3):  # feed back, as greedy decode does
                    nxt = dec.step(toks)
                    if rank == 0:
                        want = ((toks.astype(np.int64) * 31 + 7 + np.arange(B)) % 1000).astype(np.int32)
                        lines.append(f"{mode} {B} {int(np.array_equal(nxt, want))}")
                        toks = nxt
                    else:
                        assert nxt is None
        m = max_over_ranks(1.5 + rank)
        if rank == 0:
            lines.append(f"max {m}")
            with open(result_path, "w") as f:
                f.write("\n".join(lines))
    finally:
        dist.destroy_process_group()


def test_sharded_decode_gloo_world2(tmp_path):
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    out = tmp_path / "res.txt"
    mp.start_processes(_worker, args=(2, port, str(out)), nprocs=2, join=True, start_method="spawn")
    lines = out.read_text().split("\n")
    assert lines[-1] == "max 2.5"
    checks = lines[:-1]
    assert len(checks) == 24 and all(l.endswith(" 1") for l in checks), checks


def _fail_worker(rank, world, port, result_dir):
    """Injected failures on the host: a rank whose step raises, a step returning the wrong
    shape, and a malformed batch on rank 0. Every rank must see the same ShardStepError at
    the same step, and the group must keep working afterwards."""
    import sys
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        from conftest import load_pkg as lp
        lp()
        from ane_infer_b200.shard import ShardedDecoder, ShardStepError, shard_range
        B = 6
        start, _ = shard_range(B, world, rank)
        calls = {"n": 0}
        good = fake_step(start)

        def flaky(toks):
            calls["n"] += 1
            if rank == 1 and calls["n"] == 2:
                raise RuntimeError("injected worker failure")
            if rank == 0 and calls["n"] == 4:
                return good(toks)[:-1]  # wrong shape
            return good(toks)

        import torch
        dev_calls = {"n": 0}

        def flaky_dev(t, n):
            # the tensor form (DecodeContext.decode_step_device on a GPU box): rank 1's second
            # step raises after it was handed its ids
            dev_calls["n"] += 1
            if rank == 1 and dev_calls["n"] == 2:
                raise RuntimeError("injected device-step failure")
            n.copy_(torch.from_numpy(good(t.numpy())))

        for mode in ("host", "device"):
            dec = ShardedDecoder(flaky, B) if mode == "host" else ShardedDecoder(None, B, step_fn_device=flaky_dev)
            toks = np.arange(B, dtype=np.int32) * 5 + 1
            lines = []
            for step in range(6):
                feed = toks if rank == 0 else None
                if rank == 0 and step == 4:
                    feed = toks[:-1]  # malformed batch on rank 0
                try:
                    nxt = dec.step(feed)
                    ok = "ok"
                    if rank == 0:
                        want = ((toks.astype(np.int64) * 31 + 7 + np.arange(B)) % 1000).astype(np.int32)
                        ok += " 1" if np.array_equal(nxt, want) else " 0"
                        toks = nxt
                    lines.append(ok)
                except ShardStepError as e:
                    cause = type(e.__cause__).__name__ if e.__cause__ is not None else "-"
                    lines.append(f"fail {e.failed_ranks} {cause}")
            with open(os.path.join(result_dir, f"{mode}{rank}.txt"), "w") as f:
                f.write("\n".join(lines))
    finally:
        dist.destroy_process_group()


def test_sharded_decode_failure_gloo_world2(tmp_path):
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.start_processes(_fail_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    r0 = (tmp_path / "host0.txt").read_text().split("\n")
    r1 = (tmp_path / "host1.txt").read_text().split("\n")
    # step 1: rank 1's step raises; step 3: rank 0's step returns the wrong shape; step 4:
    # rank 0's batch is malformed, so no rank steps; the steps between and after succeed
    assert r0 == ["ok 1", "fail [1] -", "ok 1", "fail [0] ValueError", "fail [0] ValueError", "ok 1"], r0
    assert r1 == ["ok", "fail [1] RuntimeError", "ok", "fail [0] -", "fail [0] -", "ok"], r1
    # the device (tensor) form: rank 1's step raises at step 1 and rank 0's batch is malformed
    # at step 4; every rank raises at the same step instead of waiting out the group timeout
    d0 = (tmp_path / "device0.txt").read_text().split("\n")
    d1 = (tmp_path / "device1.txt").read_text().split("\n")
    assert d0 == ["ok 1", "fail [1] -", "ok 1", "ok 1", "fail [0] ValueError", "ok 1"], d0
    assert d1 == ["ok", "fail [1] RuntimeError", "ok", "ok", "fail [0] -", "ok"], d1
