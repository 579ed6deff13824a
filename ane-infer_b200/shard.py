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
"""
from __future__ import annotations

from typing import Callable, Optional

import numpy as np


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
    the same collective steps in the same order.
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
            self._mine = torch.zeros(w, dtype=torch.int32, device=device)
            self._next = torch.full((w,), -1, dtype=torch.int32, device=device)
            if self.rank == 0:
                self._send = torch.full((self.world, w), -1, dtype=torch.int32, device=device)
                self._recv = torch.empty((self.world, w), dtype=torch.int32, device=device)
                pin = device != "cpu"
                self._send_h = torch.full((self.world, w), -1, dtype=torch.int32, pin_memory=pin)
                self._recv_h = torch.empty((self.world, w), dtype=torch.int32, pin_memory=pin)

    def _padded(self, ids: np.ndarray):
        import torch
        t = torch.full((self.width,), -1, dtype=torch.int32)
        t[: len(ids)] = torch.from_numpy(np.ascontiguousarray(ids, dtype=np.int32))
        return t.to(self.device)

    def step(self, tokens: Optional[np.ndarray]) -> Optional[np.ndarray]:
        """tokens: int32 [global_batch] on rank 0 (ignored elsewhere). Returns the next ids
        [global_batch] on rank 0 and None on the other ranks."""
        import torch
        dist = self.dist
        if self.width == 0:
            return np.zeros(0, dtype=np.int32) if self.rank == 0 else None
        if self.step_fn_device is not None:
            return self._step_device(tokens)
        scatter_list = None
        if self.rank == 0:
            tokens = np.asarray(tokens, dtype=np.int32)
            if tokens.shape != (self.global_batch,):
                raise ValueError(f"expected {self.global_batch} token ids, got shape {tokens.shape}")
            scatter_list = []
            for r in range(self.world):
                s, c = shard_range(self.global_batch, self.world, r)
                scatter_list.append(self._padded(tokens[s:s + c]))
        mine = torch.empty(self.width, dtype=torch.int32, device=self.device)
        dist.scatter(mine, scatter_list, src=0, group=self.group)
        local = mine[: self.count].cpu().numpy()
        nxt = np.asarray(self.step_fn(local), dtype=np.int32)
        if nxt.shape != (self.count,):
            raise ValueError(f"step_fn returned shape {nxt.shape} for {self.count} sequences")
        out = self._padded(nxt)
        gather_list = [torch.empty_like(out) for _ in range(self.world)] if self.rank == 0 else None
        dist.gather(out, gather_list, dst=0, group=self.group)
        if self.rank != 0:
            return None
        res = np.empty(self.global_batch, dtype=np.int32)
        for r in range(self.world):
            s, c = shard_range(self.global_batch, self.world, r)
            res[s:s + c] = gather_list[r][:c].cpu().numpy()
        return res

    def _step_device(self, tokens: Optional[np.ndarray]) -> Optional[np.ndarray]:
        import torch
        dist = self.dist
        scatter_list = gather_list = None
        if self.rank == 0:
            tokens = np.asarray(tokens, dtype=np.int32)
            if tokens.shape != (self.global_batch,):
                raise ValueError(f"expected {self.global_batch} token ids, got shape {tokens.shape}")
            sh = self._send_h.numpy()
            for r in range(self.world):
                s, c = shard_range(self.global_batch, self.world, r)
                sh[r, :c] = tokens[s:s + c]
            self._send.copy_(self._send_h, non_blocking=True)
            scatter_list = list(self._send.unbind(0))
            gather_list = list(self._recv.unbind(0))
        dist.scatter(self._mine, scatter_list, src=0, group=self.group)
        if self.count:
            self.step_fn_device(self._mine[: self.count], self._next[: self.count])
        dist.gather(self._next, gather_list, dst=0, group=self.group)
        if self.rank != 0:
            return None
        self._recv_h.copy_(self._recv, non_blocking=True)
        if self.device != "cpu":
            torch.cuda.current_stream().synchronize()
        rh = self._recv_h.numpy()
        res = np.empty(self.global_batch, dtype=np.int32)
        for r in range(self.world):
            s, c = shard_range(self.global_batch, self.world, r)
            res[s:s + c] = rh[r, :c]
        return res
