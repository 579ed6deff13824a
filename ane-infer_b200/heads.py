"""Head-parallel split of one decode step over the GPUs of a box.

Every rank holds a full weight replica and runs every sequence, but only its share of the
mixer heads: the Gated DeltaNet heads [r*H/W, (r+1)*H/W) and the kv heads
[r*Hkv/W, (r+1)*Hkv/W) with their query heads. It keeps only those heads' recurrent state
and KV cache. After each split mixer the ranks all-gather its output (the activations of the
output projection) in place with NCCL. Everything else in the step (projections, FFN,
lm_head, argmax) runs replicated on identical inputs, so every rank ends the step with the
same logits and next tokens.

The reference runs one device (README.md:258) and has no counterpart; the per-head maths is
that of deltanet_decode_step and full_attn_decode_step (crates/engine/src/deltanet.rs:429,
:541), which never mix heads before the output projection.

`split_plan` and `gather_chunk_bytes` restate the runtime's plan (`plan_split` and the gather
in `run_mixer`, csrc/runtime.cu) for host-side checks; `open_split_context` makes the
contexts of one split from a `torch.distributed` group.
"""
from __future__ import annotations

from typing import Optional


def split_plan(cfg: dict, world: int, rank: int, kv_bf16: bool = True) -> dict:
    """The heads rank `rank` of `world` runs. A mixer kind is split when its heads divide
    over the ranks and a rank's output columns are whole 64-column K tiles (attention also
    needs the bf16 cache); otherwise it runs replicated on every rank. At least one kind must
    split."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad split request: world {world}, rank {rank}")
    H, Hkv = cfg["dn_heads"], cfg["n_kv_heads"]
    if world == 1:
        return {"dn_split": False, "kv_split": False, "dn_h0": 0, "dn_heads": H, "kv_h0": 0, "kv_heads": Hkv}
    dn_split = cfg["n_dn"] > 0 and H % world == 0 and (H * 128 // world) % 64 == 0
    kv_split = (cfg["n_attn"] > 0 and kv_bf16 and Hkv % world == 0
                and (cfg["n_heads"] * cfg["head_dim"] // world) % 64 == 0)
    if not dn_split and not kv_split:
        raise ValueError(f"neither {H} DeltaNet heads nor {Hkv} kv heads divide over {world} ranks")
    dn_hl = H // world if dn_split else H
    kv_hl = Hkv // world if kv_split else Hkv
    return {"dn_split": dn_split, "kv_split": kv_split, "dn_h0": rank * dn_hl if dn_split else 0, "dn_heads": dn_hl,
            "kv_h0": rank * kv_hl if kv_split else 0, "kv_heads": kv_hl}


def xfrag_ntile(batch: int) -> int:
    """Fragment tiles per 32-wide K block of the mma.sync path's activation layout."""
    return 1 if batch <= 4 else 2 * ((batch + 7) // 8)


def gather_chunk_bytes(K: int, batch: int, world: int, tensor_core: bool) -> int:
    """Bytes of one rank's output columns in the output projection's activation buffer.
    Both layouts are K-block-major (tcgen05: [K/64][64 rows][128 B]; mma.sync:
    [K/32][ntile][32 lanes][16 B]), so rank r's K/world columns are the byte range
    [r*chunk, (r+1)*chunk)."""
    if K % (64 * world):
        raise ValueError(f"K {K} is not a multiple of 64 x {world}")
    cols = K // world
    return (cols // 64) * 64 * 128 if tensor_core else (cols // 32) * xfrag_ntile(batch) * 512


def open_split_context(gguf, device: int, max_batch: int, max_ctx: int, group=None, **kw):
    """The DecodeContext of this rank's part of a head-parallel split over the ranks of a
    `torch.distributed` group: rank 0 makes the NCCL id and broadcasts it, then every rank
    joins (the call returns once all have)."""
    import torch.distributed as dist

    from . import DecodeContext, tp_unique_id
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    box: list[Optional[bytes]] = [tp_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(box, src=dist.get_global_rank(group, 0) if group is not None else 0, group=group)
    return DecodeContext(gguf, device=device, max_batch=max_batch, max_ctx=max_ctx, tp=(rank, world, box[0]), **kw)
