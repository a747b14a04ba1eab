"""Checkpoint loader: a Gemma-4-12B NVFP4/FP8 safetensors checkpoint into the library's layout
(the reference host's loader, furiosa-opt-gemma4-12B/src/host/load.rs:130-390).

Tensor names, dtypes and shapes are the reference's (load.rs:207-325, 360-380):

    model.language_model.embed_tokens.weight                  BF16 [W, H]
    model.language_model.norm.weight                          BF16 [H]
    model.language_model.layers.{i}.input_layernorm.weight    BF16 [H]
        .post_attention_layernorm.weight / .pre_feedforward_layernorm.weight /
        .post_feedforward_layernorm.weight                    BF16 [H]
        .self_attn.{q,k,v,o}_proj.weight                      F8_E4M3 [rows, K]
        .self_attn.{q,k,v,o}_proj.weight_scale                BF16 [rows, 1]   (a column)
        .self_attn.{q,k}_norm.weight                          BF16 [head dim]
        .layer_scalar                                         BF16 [1]         (stored as 8 copies)
        .mlp.{up,gate,down}_proj.weight_packed                U8 [rows, K / 2] (e2m1 pairs)
        .mlp.{up,gate,down}_proj.weight_scale                 F8_E4M3 [rows, K / 16]
        .mlp.{up,gate,down}_proj.weight_global_scale          F32 scalar: the op takes its
                                                              reciprocal (load.rs:170-190)

Layer i is a global (full-attention) layer when i % 6 == 5 (load.rs:373-378); it has no v_proj
and its q / k / o projections have the full-attention shapes (Qf = 8192, Pf = 512, Df = 512).

`read_checkpoint` parses and validates on the host (numpy views of a memory-mapped file, no
GPU); `to_device` uploads one tensor-parallel rank's slices and packs the weight matrices into
the GPU-native unit-tiled layout (g4_pack_tiles), returning `g4b200.decoder.Layer`s for the
sliding layers.
"""

from __future__ import annotations

import json
import struct
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

H, L, W, NS, GS, DS, QS, PS = 3840, 15360, 262144, 8, 2, 256, 4096, 2048
QF, PF, DF = 8192, 512, 512
PREFIX = "model.language_model"

_DTYPES = {"BF16": (np.uint16, 2), "F8_E4M3": (np.uint8, 1), "U8": (np.uint8, 1), "F32": (np.float32, 4),
           "I32": (np.int32, 4), "F16": (np.uint16, 2)}


class CheckpointError(ValueError):
    """A tensor is missing or has the wrong dtype or shape (the reference loader's errors)."""


class SafeTensors:
    """A safetensors file mapped read-only: an 8-byte little-endian header length, a JSON header
    {name: {dtype, shape, data_offsets}}, then the data (offsets relative to its start)."""

    def __init__(self, path):
        self.path = Path(path)
        with open(self.path, "rb") as f:
            n = struct.unpack("<Q", f.read(8))[0]
            if n <= 0 or n > 100_000_000:
                raise CheckpointError(f"{self.path}: implausible header length {n}")
            self.header = json.loads(f.read(n))
        self.data_start = 8 + n
        self.map = np.memmap(self.path, dtype=np.uint8, mode="r")

    def names(self):
        return [k for k in self.header if k != "__metadata__"]

    def tensor(self, name, dtype, shape):
        """The tensor's data as a numpy view, after checking its dtype and shape."""
        if name not in self.header:
            raise CheckpointError(f"missing tensor {name}")
        info = self.header[name]
        if info["dtype"] != dtype or list(info["shape"]) != list(shape):
            raise CheckpointError(f"{name} is {info['dtype']} {info['shape']}, expected {dtype} {list(shape)}")
        np_dtype, size = _DTYPES[dtype]
        start, end = info["data_offsets"]
        count = int(np.prod(shape)) if shape else 1
        if end - start != count * size:
            raise CheckpointError(f"{name}: {end - start} bytes of data for {count} elements of {dtype}")
        raw = self.map[self.data_start + start:self.data_start + end]
        return raw.view(np_dtype).reshape(shape if shape else (1,))


def reciprocal_global_scale(st: SafeTensors, name: str) -> np.ndarray:
    """1 / the checkpoint's NVFP4 global scale, refusing zero and non-finite values (load.rs:170-180)."""
    if name not in st.header or st.header[name]["dtype"] != "F32" or int(np.prod(st.header[name]["shape"] or [1])) != 1:
        raise CheckpointError(f"{name} is not a scalar f32 tensor")
    info = st.header[name]
    value = st.tensor(name, "F32", info["shape"]).reshape(-1)[0]
    if value == 0.0 or not np.isfinite(value):
        raise CheckpointError(f"invalid NVFP4 global scale {name}: {value}")
    return np.array([np.float32(1.0) / np.float32(value)], np.float32)


def is_full(layer: int) -> bool:
    return layer % 6 == 5


@dataclass
class HostLayer:
    """One layer's tensors on the host in the reference layout (numpy; bf16 as uint16 bits)."""
    index: int
    full: bool
    t: dict = field(default_factory=dict)


def _mlp(st, prefix, d):
    for name, rows, cols in (("up", L, H), ("gate", L, H), ("down", H, L)):
        p = f"{prefix}.mlp.{name}_proj"
        d[f"{name}_weight_packed"] = st.tensor(f"{p}.weight_packed", "U8", (rows, cols // 2))
        d[f"{name}_weight_scale"] = st.tensor(f"{p}.weight_scale", "F8_E4M3", (rows, cols // 16))
        d[f"{name}_global_scale"] = reciprocal_global_scale(st, f"{p}.weight_global_scale")


def read_layer(st: SafeTensors, layer: int) -> HostLayer:
    """One layer by the reference's names (load.rs:263-325)."""
    p = f"{PREFIX}.layers.{layer}"
    full = is_full(layer)
    d = {}
    for norm in ("input_layernorm", "post_attention_layernorm", "pre_feedforward_layernorm",
                 "post_feedforward_layernorm"):
        d[norm] = st.tensor(f"{p}.{norm}.weight", "BF16", (H,))
    q_rows, k_rows, o_cols, hd = (QF, PF, QF, DF) if full else (QS, PS, QS, DS)
    projs = (("q", q_rows, H), ("k", k_rows, H), ("o", H, o_cols)) if full else \
        (("q", q_rows, H), ("k", k_rows, H), ("v", k_rows, H), ("o", H, o_cols))
    for name, rows, cols in projs:
        d[f"{name}_weight"] = st.tensor(f"{p}.self_attn.{name}_proj.weight", "F8_E4M3", (rows, cols))
        d[f"{name}_weight_scale"] = st.tensor(f"{p}.self_attn.{name}_proj.weight_scale", "BF16", (rows, 1)).reshape(rows)
    d["q_norm"] = st.tensor(f"{p}.self_attn.q_norm.weight", "BF16", (hd,))
    d["k_norm"] = st.tensor(f"{p}.self_attn.k_norm.weight", "BF16", (hd,))
    shape = st.header.get(f"{p}.layer_scalar", {}).get("shape", [1])
    scalar = st.tensor(f"{p}.layer_scalar", "BF16", shape if shape in ([], [1]) else (1,)).reshape(-1)
    d["layer_scalar"] = np.full(8, scalar[0], np.uint16)  # the op's [1 # 8] (load.rs:100-113)
    _mlp(st, p, d)
    return HostLayer(layer, full, d)


def read_checkpoint(path, layers=None):
    """(embedding table [rows, H], final norm [H], [HostLayer]) of the checkpoint at `path` (a file,
    or a directory holding model.safetensors). `layers`: the layer indices to read (default: every
    `model.language_model.layers.N` present, in order)."""
    path = Path(path)
    st = SafeTensors(path / "model.safetensors" if path.is_dir() else path)
    emb_name = f"{PREFIX}.embed_tokens.weight"
    if emb_name not in st.header:
        raise CheckpointError(f"missing tensor {emb_name}")
    rows = st.header[emb_name]["shape"][0]
    if not 0 < rows <= W:
        raise CheckpointError(f"{emb_name}: {rows} rows, expected at most {W}")
    table = st.tensor(emb_name, "BF16", (rows, H))
    final = st.tensor(f"{PREFIX}.norm.weight", "BF16", (H,))
    if layers is None:
        idx = sorted({int(n.split(".")[3]) for n in st.names() if n.startswith(f"{PREFIX}.layers.")})
    else:
        idx = list(layers)
    return table, final, [read_layer(st, i) for i in idx]


def to_device(ops_device, host: HostLayer, *, ring_len=None, rank=0, world=1, tiled=True):
    """One sliding layer on the GPU as a g4b200.decoder.Layer (this rank's slices, packed into the
    unit-tiled layout when tiled=True), with zeroed KV ring caches of `ring_len` slots (default
    1024, the reference's Ts). Full-attention layers have their own geometry and are refused."""
    import torch

    from . import decoder, ops, tp

    if host.full:
        raise ValueError(f"layer {host.index} is a full-attention layer (its geometry is not the sliding op's)")
    dev = torch.device("cuda", ops_device.index)
    t = host.t

    def up(arr, name=None):
        a = np.ascontiguousarray(arr)
        x = torch.from_numpy(a.view(np.int16) if a.dtype == np.uint16 else a.copy())
        if name is not None:
            x = tp.shard(name, x, rank, world)
        x = x.to(dev)
        return x.view(torch.bfloat16) if a.dtype == np.uint16 else x

    ring = ring_len or 1024
    kv = NS // world
    lay = decoder.Layer(
        input_rms_weight=up(t["input_layernorm"]), q_weight=up(t["q_weight"], "q_weight"),
        k_weight=up(t["k_weight"], "k_weight"), v_weight=up(t["v_weight"], "v_weight"),
        q_weight_scale=up(t["q_weight_scale"], "q_weight_scale"),
        k_weight_scale=up(t["k_weight_scale"], "k_weight_scale"),
        v_weight_scale=up(t["v_weight_scale"], "v_weight_scale"), q_rms_weight=up(t["q_norm"]),
        k_rms_weight=up(t["k_norm"]), k_cache=torch.zeros((ring, kv, DS), dtype=torch.bfloat16, device=dev),
        v_cache=torch.zeros((ring, kv, DS), dtype=torch.bfloat16, device=dev),
        post_attn_rms_weight=up(t["post_attention_layernorm"]), o_weight=up(t["o_weight"], "o_weight"),
        o_weight_scale=up(t["o_weight_scale"]), pre_ff_rms_weight=up(t["pre_feedforward_layernorm"]),
        post_ff_rms_weight=up(t["post_feedforward_layernorm"]), layer_scalar=up(t["layer_scalar"]),
        up_weight=up(t["up_weight_packed"], "up_weight_packed"),
        gate_weight=up(t["gate_weight_packed"], "gate_weight_packed"),
        down_weight=up(t["down_weight_packed"], "down_weight_packed"),
        up_scale=up(t["up_weight_scale"], "up_weight_scale"), gate_scale=up(t["gate_weight_scale"], "gate_weight_scale"),
        down_scale=up(t["down_weight_scale"], "down_weight_scale"), up_global_scale=up(t["up_global_scale"]),
        gate_global_scale=up(t["gate_global_scale"]), down_global_scale=up(t["down_global_scale"]),
        ffn=decoder.FFN_NVFP4, tiled=False)
    if tiled:
        for name in ("q_weight", "k_weight", "v_weight", "o_weight"):
            setattr(lay, name, ops.tile_weight(ops_device, name, getattr(lay, name)))
        lay.up_weight = ops.pack_upgate(ops_device, lay.up_weight, lay.gate_weight, scales=False)
        lay.up_scale = ops.pack_upgate(ops_device, lay.up_scale, lay.gate_scale, scales=True)
        lay.down_weight = ops.tile_weight(ops_device, "down_weight_packed", lay.down_weight)
        lay.down_scale = ops.tile_weight(ops_device, "down_weight_scale", lay.down_scale)
        lay.gate_weight = lay.gate_scale = None
        lay.tiled = True
    return lay


def write_safetensors(path, tensors: dict, metadata=None) -> None:
    """Write {name: (dtype, numpy array)} as a safetensors file (for tests and tools; the format of
    the checkpoints `read_checkpoint` reads)."""
    header, blobs, offset = {}, [], 0
    for name, (dtype, arr) in tensors.items():
        a = np.ascontiguousarray(arr)
        b = a.tobytes()
        header[name] = {"dtype": dtype, "shape": list(a.shape), "data_offsets": [offset, offset + len(b)]}
        blobs.append(b)
        offset += len(b)
    if metadata:
        header["__metadata__"] = metadata
    raw = json.dumps(header).encode()
    raw += b" " * (-len(raw) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(raw)))
        f.write(raw)
        for b in blobs:
            f.write(b)
