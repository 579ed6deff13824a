"""Sequence sharding of batched greedy decode across one process per GPU.

Decode of independent sequences needs no exchange between GPUs: each rank owns a contiguous
range of the global batch (its slots 0..count-1 on its own ab2 context) and a full weight
replica. The only traffic is the host plumbing the reference's caller does for one sequence
(`cmd_bench`, crates/cli/src/main.rs:418-508: feed a token id, read the next one back), done
here for the whole batch: rank 0 scatters each rank's token ids and gathers the next ids.

`torch.distributed` carries the two small messages (4 bytes per sequence); with the NCCL
backend they travel as device tensors, with gloo (the CPU tests) as host tensors. With a
device step function (`step_fn_device`, NCCL) the ids stay on the device between the
collectives: rank 0 makes one host-to-device copy of the batch's ids and one device-to-host
copy of the next ids per step, and every rank decodes straight from the scattered tensor.

Failures: each rank's result carries a status word, and the results travel by all-gather,
so when one rank's step raises (or, in the host-array form, returns the wrong shape), every
rank raises `ShardStepError` at the same point of the same step. No collective is left
pending, and the group stays usable. When rank 0 cannot form the batch, the host-array form
runs no step anywhere (a control word in the scatter); the device form, whose ranks do not
read the scattered ids on the host, runs every rank's step on ids of -1 (which the decoder
embeds as zeros, advancing those sequences by one step) and then raises on every rank.
"""
from __future__ import annotations

from typing import Callable, Optional

import numpy as np


class ShardStepError(RuntimeError):
    """A decode step failed on one or more ranks; raised on every rank of the group."""

    def __init__(self, failed_ranks: list[int]):
        super().__init__(f"decode step failed on rank(s) {failed_ranks}")
        self.failed_ranks = failed_ranks


def shard_range(global_batch: int, world: int, rank: int) -> tuple[int, int]:
    """(first global sequence, count) owned by `rank`: contiguous ranges whose sizes differ
    by at most one, the first `global_batch % world` ranks taking the extra sequence."""
    if world < 1 or not 0 <= rank < world or global_batch < 0:
        raise ValueError(f"bad shard request: batch {global_batch}, world {world}, rank {rank}")
    base, extra = divmod(global_batch, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def max_over_ranks(x: float, group=None, device: Optional[str] = None) -> float:
    """The largest of one float over the ranks of `group` (multi-GPU timings are reported as
    the slowest rank's)."""
    import torch
    import torch.distributed as dist
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return float(x)
    if device is None:
        device = "cuda" if dist.get_backend(group) == "nccl" else "cpu"
    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


class ShardedDecoder:
    """Greedy decode of `global_batch` sequences split over the ranks of a process group.

    step_fn(local_tokens: np.ndarray[int32]) -> np.ndarray[int32] decodes this rank's
    sequences one step (for example `DecodeContext.decode_step(...)[1]`); it is called on
    every rank, also with an empty array when the rank owns no sequence, so all ranks take
    the same collective steps in the same order. If it raises on any rank, `step` raises
    ShardStepError on every rank (chained to the original exception where it happened).
    """

    def __init__(self, step_fn: Optional[Callable[[np.ndarray], np.ndarray]], global_batch: int, group=None,
                 device: Optional[str] = None, step_fn_device: Optional[Callable] = None):
        import torch.distributed as dist
        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.global_batch = global_batch
        self.step_fn = step_fn
        self.start, self.count = shard_range(global_batch, self.world, self.rank)
        self.width = -(-global_batch // self.world) if global_batch else 0
        if device is None:
            device = "cuda" if dist.get_backend(group) == "nccl" else "cpu"
        self.device = device
        # step_fn_device(tokens_dev, next_dev): enqueue this rank's step on the current stream,
        # reading int32 ids from tokens_dev [count] and writing the next ids to next_dev [count]
        self.step_fn_device = step_fn_device
        if step_fn is None and step_fn_device is None:
            raise ValueError("a step function is required")
        if step_fn_device is not None:
            import torch
            w = max(self.width, 1)
            pin = device != "cpu"
            self._mine = torch.zeros(w, dtype=torch.int32, device=device)
            # the next ids padded to the shard width, then this rank's status word (0 ok, 1 failed)
            self._next = torch.full((w + 1,), -1, dtype=torch.int32, device=device)
            self._next[w] = 0
            self._recv = torch.empty((self.world, w + 1), dtype=torch.int32, device=device)
            self._recv_list = list(self._recv.unbind(0))
            self._recv_h = torch.empty((self.world, w + 1), dtype=torch.int32, pin_memory=pin)
            if self.rank == 0:
                self._send = torch.full((self.world, w), -1, dtype=torch.int32, device=device)
                self._send_h = torch.full((self.world, w), -1, dtype=torch.int32, pin_memory=pin)

    def step(self, tokens: Optional[np.ndarray]) -> Optional[np.ndarray]:
        """tokens: int32 [global_batch] on rank 0 (ignored elsewhere). Returns the next ids
        [global_batch] on rank 0 and None on the other ranks."""
        import torch
        dist = self.dist
        if self.width == 0:
            return np.zeros(0, dtype=np.int32) if self.rank == 0 else None
        if self.step_fn_device is not None:
            return self._step_device(tokens)
        # each rank's ids padded to the shard width, then a control word: 1 = rank 0 could not
        # form the batch, so no rank runs its step
        w = self.width
        err = None
        scatter_list = None
        if self.rank == 0:
            tokens = np.asarray(tokens, dtype=np.int32)
            if tokens.shape != (self.global_batch,):
                err = ValueError(f"expected {self.global_batch} token ids, got shape {tokens.shape}")
            scatter_list = []
            for r in range(self.world):
                t = torch.full((w + 1,), -1, dtype=torch.int32)
                if err is None:
                    s0, c = shard_range(self.global_batch, self.world, r)
                    t[:c] = torch.from_numpy(tokens[s0:s0 + c])
                t[w] = 0 if err is None else 1
                scatter_list.append(t.to(self.device))
        mine = torch.empty(w + 1, dtype=torch.int32, device=self.device)
        dist.scatter(mine, scatter_list, src=0, group=self.group)
        mine = mine.cpu()
        nxt = np.full(self.count, -1, dtype=np.int32)
        if int(mine[w]) == 0:
            try:
                nxt = np.asarray(self.step_fn(mine[: self.count].numpy()), dtype=np.int32)
                if nxt.shape != (self.count,):
                    raise ValueError(f"step_fn returned shape {nxt.shape} for {self.count} sequences")
            except Exception as e:  # reported to every rank below, then raised here
                err = e
                nxt = np.full(self.count, -1, dtype=np.int32)
        # the next ids padded to the shard width, then this rank's status (0 ok, 1 failed)
        out = torch.full((w + 1,), -1, dtype=torch.int32)
        out[: self.count] = torch.from_numpy(nxt)
        out[w] = 0 if err is None else 1
        out = out.to(self.device)
        outs = [torch.empty_like(out) for _ in range(self.world)]
        dist.all_gather(outs, out, group=self.group)
        failed = [r for r in range(self.world) if int(outs[r][w].item()) != 0]
        if failed:
            raise ShardStepError(failed) from err
        if self.rank != 0:
            return None
        res = np.empty(self.global_batch, dtype=np.int32)
        for r in range(self.world):
            s, c = shard_range(self.global_batch, self.world, r)
            res[s:s + c] = outs[r][:c].cpu().numpy()
        return res

    def _step_device(self, tokens: Optional[np.ndarray]) -> Optional[np.ndarray]:
        import torch
        dist = self.dist
        w = self.width
        err = None
        scatter_list = None
        if self.rank == 0:
            sh = self._send_h.numpy()
            try:
                tokens = np.asarray(tokens, dtype=np.int32)
                if tokens.shape != (self.global_batch,):
                    raise ValueError(f"expected {self.global_batch} token ids, got shape {tokens.shape}")
                for r in range(self.world):
                    s, c = shard_range(self.global_batch, self.world, r)
                    sh[r, :c] = tokens[s:s + c]
            except Exception as e:  # every rank still steps (on -1 ids) and then raises
                err = e
                sh[:] = -1
            self._send.copy_(self._send_h, non_blocking=True)
            scatter_list = list(self._send.unbind(0))
        dist.scatter(self._mine, scatter_list, src=0, group=self.group)
        if self.count:
            try:
                self.step_fn_device(self._mine[: self.count], self._next[: self.count])
            except Exception as e:  # reported to every rank below, then raised here
                err = err or e
        if err is not None:
            self._next[w].fill_(1)
        dist.all_gather(self._recv_list, self._next, group=self.group)
        self._recv_h.copy_(self._recv, non_blocking=True)
        if self.device != "cpu":
            torch.cuda.current_stream().synchronize()
        rh = self._recv_h.numpy()
        failed = [r for r in range(self.world) if int(rh[r, w]) != 0]
        if failed:
            self._next[w].fill_(0)  # re-armed for the next step
            raise ShardStepError(failed) from err
        if self.rank != 0:
            return None
        res = np.empty(self.global_batch, dtype=np.int32)
        for r in range(self.world):
            s, c = shard_range(self.global_batch, self.world, r)
            res[s:s + c] = rh[r, :c]
        return res
