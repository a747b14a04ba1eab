"""Tensor parallelism on the CPU: the slicing rules of g4b200.tp, the tensor-parallel oracle
against the one-chip oracle and the reference's golden outputs, and the setup-blob exchange
between two gloo ranks (no GPU anywhere)."""

import os
import socket

import numpy as np
import pytest
import torch

from oracle import ops as oracle
from oracle import synth
from helpers import ATOL, within

WORLDS = (2, 4, 8)


def t(arr):
    """numpy (bf16 bits as uint16) -> torch CPU tensor of the same bytes."""
    a = np.ascontiguousarray(arr)
    return torch.from_numpy(a.view(np.int16) if a.dtype == np.uint16 else a)


def n(tensor, like):
    out = tensor.numpy()
    return out.view(np.uint16) if like.dtype == np.uint16 else out


def shard_np(name, arr, rank, world):
    from g4b200 import tp

    return n(tp.shard(name, t(arr), rank, world), arr)


def test_geometry():
    from g4b200.ops import geometry

    assert geometry(1) == {"kv_heads": 8, "q_rows": 4096, "kv_rows": 2048, "ffn_rows": 15360, "down_k": 15360}
    assert geometry(8) == {"kv_heads": 1, "q_rows": 512, "kv_rows": 256, "ffn_rows": 1920, "down_k": 2048}
    with pytest.raises(ValueError):
        geometry(3)


@pytest.mark.parametrize("world", WORLDS)
def test_shards_cover_the_layer(world):
    from g4b200 import tp
    from g4b200.ops import geometry

    g = geometry(world)
    gen = torch.Generator().manual_seed(world)
    q_w = torch.randint(0, 256, (4096, 3840), dtype=torch.uint8, generator=gen)
    assert torch.equal(torch.cat([tp.shard("q_weight", q_w, r, world) for r in range(world)]), q_w)
    cache = torch.randint(-2000, 2000, (64, 8, 256), dtype=torch.int16, generator=gen)
    parts = [tp.shard("k_cache", cache, r, world) for r in range(world)]
    assert parts[0].shape == (64, 8 // world, 256) and parts[0].is_contiguous()
    assert torch.equal(tp.unshard_heads(parts, 1), cache)
    o_w = torch.randint(0, 256, (3840, 4096), dtype=torch.uint8, generator=gen)
    assert torch.equal(torch.cat([tp.shard("o_weight", o_w, r, world) for r in range(world)], dim=1), o_w)
    down = torch.randint(0, 256, (3840, 7680), dtype=torch.uint8, generator=gen)
    down_s = torch.randint(0, 256, (3840, 960), dtype=torch.uint8, generator=gen)
    for name, full, per_byte in (("down_weight_packed", down, 2), ("down_weight_scale", down_s, 16)):
        cols = g["ffn_rows"] // per_byte
        parts = [tp.shard(name, full, r, world) for r in range(world)]
        assert parts[0].shape == (3840, g["down_k"] // per_byte)
        assert torch.equal(torch.cat([p[:, :cols] for p in parts], dim=1), full)
        assert all(int(p[:, cols:].abs().sum()) == 0 for p in parts)  # zero codes, zero scales
    x = torch.ones(3840)
    assert tp.shard("x", x, world - 1, world) is x
    with pytest.raises(KeyError):
        tp.shard("no_such_tensor", x, 0, world)
    with pytest.raises(ValueError):
        tp.shard("q_weight", q_w[:100], 0, world)


@pytest.mark.parametrize("world", WORLDS)
def test_tp_oracle_o_against_reference(world, golden_runs):
    """The split K contraction (rank-order sum of f32 partials) meets the reference's golden
    output as closely as the one-chip oracle."""
    run = 3
    d = synth.sliding_attention_output(run)
    xs = [shard_np("attn", d["x"], r, world) for r in range(world)]
    ws = [shard_np("o_weight", d["o_weight"], r, world) for r in range(world)]
    got = oracle.sliding_attention_output_tp(xs, d["post_attn_rms_weight"], ws, d["o_weight_scale"], d["residual"])
    ok, maxd, exact = within(golden_runs[f"run{run}.sliding_attention_output.expected"], got,
                             ATOL["sliding_attention_output"])
    assert ok, maxd
    assert exact > 0.99, exact


@pytest.mark.parametrize("world", (2, 8))
def test_tp_oracle_ffn_against_reference(world, golden_runs):
    run = 6
    d = synth.decoder_feedforward(run)
    parts = {k: [shard_np(k, d[k], r, world) for r in range(world)]
             for k in ("up_weight_packed", "up_weight_scale", "gate_weight_packed", "gate_weight_scale",
                       "down_weight_packed", "down_weight_scale")}
    got = oracle.decoder_feedforward_tp(
        d["residual"], d["pre_ff_rms_weight"],
        list(zip(parts["up_weight_packed"], parts["up_weight_scale"])),
        list(zip(parts["gate_weight_packed"], parts["gate_weight_scale"])),
        list(zip(parts["down_weight_packed"], parts["down_weight_scale"])),
        d["up_global_scale"][0], d["gate_global_scale"][0], d["down_global_scale"][0], d["post_ff_rms_weight"],
        d["layer_scalar"])
    ok, maxd, exact = within(golden_runs[f"run{run}.decoder_feedforward.expected"], got, ATOL["decoder_feedforward"])
    assert ok, maxd
    assert exact > 0.95, exact


@pytest.mark.parametrize("world", (2, 8))
def test_per_head_ops_split_exactly(world):
    """QKV rows and attention heads are independent: each rank's slice of the one-chip result
    is what the rank computes from its slices alone."""
    d = synth.sliding_project_qkv(2)
    whole = oracle.sliding_project_qkv(d["x"], d["q_weight"], d["k_weight"], d["v_weight"], d["q_weight_scale"],
                                       d["k_weight_scale"], d["v_weight_scale"], d["input_rms_weight"],
                                       d["q_rms_weight"], d["k_rms_weight"], d["cos_row"], d["sin_row"])
    parts = []
    for r in range(world):
        s = {k: shard_np(k, d[k], r, world) for k in ("q_weight", "k_weight", "v_weight", "q_weight_scale",
                                                      "k_weight_scale", "v_weight_scale")}
        parts.append(oracle.sliding_project_qkv(d["x"], s["q_weight"], s["k_weight"], s["v_weight"],
                                                s["q_weight_scale"], s["k_weight_scale"], s["v_weight_scale"],
                                                d["input_rms_weight"], d["q_rms_weight"], d["k_rms_weight"],
                                                d["cos_row"], d["sin_row"], n_kv=8 // world))
    for i, label in enumerate("qkv"):
        got = np.concatenate([p[i] for p in parts], axis=0)
        ok, maxd, exact = within(whole[i], got, ATOL["sliding_project_qkv"])
        assert ok and exact > 0.999, (label, maxd, exact)

    from oracle import prng

    ring = 256
    q = prng.bf16_signs("tp.q", 16 * 256, 1.0).reshape(8, 2, 256)
    k = prng.bf16_uniform("tp.k", ring * 8 * 256, -1.0, 1.0).reshape(ring, 8, 256)
    v = prng.bf16_uniform("tp.v", ring * 8 * 256, -1.0, 1.0).reshape(ring, 8, 256)
    mask = (np.arange(ring) < 200).astype(np.float32)
    whole = oracle.sliding_attention(q, k, v, mask, 1.0 / 16)
    got = np.concatenate([oracle.sliding_attention(shard_np("q", q, r, world), shard_np("k_cache", k, r, world),
                                                   shard_np("v_cache", v, r, world), mask, 1.0 / 16)
                          for r in range(world)], axis=0)
    assert np.array_equal(got, whole)


# ------------------------------------------------------------------------------ gloo ranks

class FakeDevice:
    """Stands in for ops.Device: records the calls g4b200.tp.connect makes."""

    def __init__(self):
        self.calls = []

    def tp_init(self, rank, world):
        self.calls.append(("init", rank, world))
        return bytes([0x40 + rank]) * 128

    def tp_connect(self, blobs):
        self.calls.append(("connect", blobs))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_rank(rank, world, port, out_dir):
    import datetime

    import torch.distributed as dist

    from g4b200 import tp

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        dev = FakeDevice()
        tp.connect(dev)
        assert dev.calls[0] == ("init", rank, world)
        assert dev.calls[1] == ("connect", b"".join(bytes([0x40 + r]) * 128 for r in range(world)))
        # every rank cuts its own slice of the same seeded tensor; together they are the tensor
        full = torch.randint(0, 256, (2048, 3840), dtype=torch.uint8, generator=torch.Generator().manual_seed(7))
        mine = tp.shard("k_weight", full, rank, world)
        gathered = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(gathered, mine)
        assert torch.equal(torch.cat(gathered), full)
        with open(os.path.join(out_dir, f"ok{rank}"), "w") as f:
            f.write("ok")
    finally:
        dist.destroy_process_group()


def test_setup_exchange_between_gloo_ranks(tmp_path):
    import torch.multiprocessing as mp

    world = 2
    mp.start_processes(_gloo_rank, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    assert all((tmp_path / f"ok{r}").exists() for r in range(world))
