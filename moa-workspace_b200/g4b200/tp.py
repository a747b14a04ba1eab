"""Tensor parallelism over the GPUs of one node: the weight slices each rank holds and the
setup of the in-kernel exchange.

The split is the Megatron one the library's kernels implement (include/g4b200.h, tensor
parallelism): rank r of `world` owns KV heads [8r/w, 8(r+1)/w) with their query heads and their
slice of the ring caches, the matching K columns of O, and FFN rows [L r/w, L (r+1)/w) of up and
gate with the same K columns of down (zero-padded to whole 256-element units). The O and down
outputs are summed over the ranks inside the kernels; everything else is local.

`shard` works on torch tensors on any device (the host logic is tested on CPU); `connect`
exchanges the setup blobs over a torch.distributed group (gloo or nccl).
"""

from __future__ import annotations

import torch

from .ops import DS, GS, H, L, NS, PS, QS, geometry

# tensor name -> how rank r's slice is cut from the whole layer's tensor
_ROW_SLICED = {  # leading dimension, by output rows
    "q_weight": QS, "q_weight_scale": QS,
    "k_weight": PS, "k_weight_scale": PS, "v_weight": PS, "v_weight_scale": PS,
    "up_weight_packed": L, "gate_weight_packed": L, "up_weight_scale": L, "gate_weight_scale": L,
    # FP8 feed-forward (decoder_feedforward_fp8): codes and f32 channel scales of up and gate
    "up_weight": L, "gate_weight": L, "up_channel_scale": L, "gate_channel_scale": L,
}
_HEAD_SLICED = {"k_cache": 1, "v_cache": 1, "q_out": 0, "q": 0, "out_hbm": 0, "attn": 0}  # KV-head axis
_COL_SLICED = {"o_weight": (QS, 1), "down_weight_packed": (L, 2), "down_weight_scale": (L, 16),
               "down_weight": (L, 1)}  # (K, elems/byte)
REPLICATED = ("x", "input_rms_weight", "q_rms_weight", "k_rms_weight", "kv_offset", "rope_offset", "cos", "sin",
              "mask", "post_attn_rms_weight", "o_weight_scale", "residual_hbm", "pre_ff_rms_weight",
              "up_global_scale", "gate_global_scale", "down_global_scale", "post_ff_rms_weight", "layer_scalar",
              "down_channel_scale")


def shard(name: str, full: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Rank `rank`'s slice of the whole-layer tensor `full` (named as in the reference op's
    signature), contiguous. Replicated tensors are returned as they are."""
    g = geometry(world)
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if name in _ROW_SLICED:
        rows = _ROW_SLICED[name]
        if full.shape[0] != rows:
            raise ValueError(f"{name}: {full.shape[0]} rows, expected {rows}")
        n = rows // world
        return full[rank * n:(rank + 1) * n].contiguous()
    if name in _HEAD_SLICED:
        axis = _HEAD_SLICED[name]
        if full.shape[axis] != NS:
            raise ValueError(f"{name}: axis {axis} has {full.shape[axis]} heads, expected {NS}")
        n = NS // world
        return full.narrow(axis, rank * n, n).contiguous()
    if name in _COL_SLICED:
        k, per_byte = _COL_SLICED[name]
        if full.shape != (H, k // per_byte):
            raise ValueError(f"{name}: shape {tuple(full.shape)}, expected {(H, k // per_byte)}")
        n = k // world // per_byte
        part = full[:, rank * n:(rank + 1) * n]
        width = (g["down_k"] if name.startswith("down") else g["q_rows"]) // per_byte
        if width == n:
            return part.contiguous()
        out = torch.zeros((H, width), dtype=full.dtype, device=full.device)  # zero codes, zero scales
        out[:, :n] = part
        return out
    if name in REPLICATED:
        return full
    raise KeyError(f"no tensor-parallel rule for {name!r}")


def unshard_heads(parts, axis: int) -> torch.Tensor:
    """The whole tensor from every rank's head slice (rank order), e.g. to compare q_out or the
    caches with a one-GPU run."""
    return torch.cat(list(parts), dim=axis)


def exchange_blobs(blob: bytes, group=None) -> bytes:
    """Every rank's setup blob, concatenated in rank order (all_gather over `group`)."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    blobs = [None] * world
    dist.all_gather_object(blobs, blob, group=group)
    if any(not isinstance(b, (bytes, bytearray)) or len(b) != len(blob) for b in blobs):
        raise RuntimeError("tensor-parallel setup: a rank sent a malformed blob")
    return b"".join(bytes(b) for b in blobs)


def connect(device, group=None) -> None:
    """Make `device` (an ops.Device) this process's rank of the torch.distributed group and
    connect it to the other ranks' GPUs. Every rank of the group must call it."""
    import torch.distributed as dist

    rank, world = dist.get_rank(group), dist.get_world_size(group)
    # g4_tp_init frees this rank's previous exchange buffer: no rank may still be running ops of
    # a previous setup that store into it
    if torch.cuda.is_available() and getattr(device, "index", None) is not None:
        torch.cuda.synchronize(device.index)
    dist.barrier(group)
    blob = device.tp_init(rank, world)
    device.tp_connect(exchange_blobs(blob, group))
    dist.barrier(group)


__all__ = ["shard", "unshard_heads", "exchange_blobs", "connect", "REPLICATED", "DS", "GS"]
