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
