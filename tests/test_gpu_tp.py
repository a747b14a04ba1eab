"""Tensor parallelism on GPUs: each rank (one process per GPU) runs the four ops on its slices
through the C ABI; the O and down outputs are summed over the ranks inside the kernels.

Checked against the reference's golden outputs and the CPU oracle (per-head ops: the ranks'
slices put together), that every rank's residual has the same bits, that repeated calls (the
exchange's alternating buffers) give the same result, and that cache slots the op does not
target keep their contents. Needs as many GPUs as ranks; the setup refusals need one."""

import os
import socket

import numpy as np
import pytest

from oracle import ops as oracle
from oracle import synth
from helpers import ATOL, within

pytestmark = pytest.mark.gpu
SENTINEL_K, SENTINEL_V, SENTINEL_Q = 0x3E80, 0xBF00, 0x3FC0
RUN_QKV, RUN_O, RUN_FFN, RING = 1, 4, 7, 1024
REPEATS = 3  # calls of O and of the FFN in a row: both exchange parities, twice over


def _gpus():
    import torch

    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _attention_inputs():
    from oracle import prng

    q = prng.bf16_signs("tp.attn.q", 16 * 256, 1.0).reshape(8, 2, 256)
    k = prng.bf16_uniform("tp.attn.k", RING * 8 * 256, -1.0, 1.0).reshape(RING, 8, 256)
    v = prng.bf16_uniform("tp.attn.v", RING * 8 * 256, -1.0, 1.0).reshape(RING, 8, 256)
    mask = (np.arange(RING) <= 900).astype(np.float32)
    return q, k, v, mask


def _tp_rank(rank, world, port, out_dir):
    import datetime

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    from g4b200 import ops, tp

    dev = ops.Device(rank)

    def cuda(arr, name=None):
        a = np.ascontiguousarray(arr)
        x = torch.from_numpy(a.view(np.int16) if a.dtype == np.uint16 else a)
        if name is not None:
            x = tp.shard(name, x, rank, world)
        x = x.cuda()
        return x.view(torch.bfloat16) if a.dtype == np.uint16 else x

    def host(x):
        x = x.detach().cpu().contiguous()
        return x.view(torch.int16).numpy().view(np.uint16) if x.dtype == torch.bfloat16 else x.numpy()

    try:
        tp.connect(dev)
        out = {}
        # --- inputs of every op, on the device before the first call
        d = synth.sliding_project_qkv(RUN_QKV)
        cos = np.zeros((32768, 256), np.uint16)
        sin = np.zeros((32768, 256), np.uint16)
        cos[d["pos"]], sin[d["pos"]] = d["cos_row"], d["sin_row"]
        qkv_in = [cuda(d["x"]), cuda(d["q_weight"], "q_weight"), cuda(d["k_weight"], "k_weight"),
                  cuda(d["v_weight"], "v_weight"), cuda(d["q_weight_scale"], "q_weight_scale"),
                  cuda(d["k_weight_scale"], "k_weight_scale"), cuda(d["v_weight_scale"], "v_weight_scale"),
                  cuda(d["input_rms_weight"]), cuda(d["q_rms_weight"]), cuda(d["k_rms_weight"]),
                  cuda(d["kv_offset"]), cuda(d["rope_offset"]), cuda(cos), cuda(sin)]
        k_cache = cuda(np.full((RING, 8, 256), SENTINEL_K, np.uint16), "k_cache")
        v_cache = cuda(np.full((RING, 8, 256), SENTINEL_V, np.uint16), "v_cache")
        q_out = cuda(np.full((8, 2, 256), SENTINEL_Q, np.uint16), "q_out")
        q, k, v, mask = _attention_inputs()
        attn_in = [cuda(q, "q"), cuda(k, "k_cache"), cuda(v, "v_cache"), cuda(mask)]
        attn_out = cuda(np.zeros((8, 2, 256), np.uint16), "out_hbm")
        o = synth.sliding_attention_output(RUN_O)
        o_in = [cuda(o["x"], "attn"), cuda(o["post_attn_rms_weight"]), cuda(o["o_weight"], "o_weight"),
                cuda(o["o_weight_scale"])]
        f = synth.decoder_feedforward(RUN_FFN)
        ffn_in = [cuda(f["pre_ff_rms_weight"])] + [
            cuda(f[k], k) for k in ("up_weight_packed", "gate_weight_packed", "down_weight_packed", "up_weight_scale",
                                    "gate_weight_scale", "down_weight_scale")] + [
            cuda(f["up_global_scale"]), cuda(f["gate_global_scale"]), cuda(f["down_global_scale"]),
            cuda(f["post_ff_rms_weight"]), cuda(f["layer_scalar"])]
        torch.cuda.synchronize()
        dist.barrier()

        ops.sliding_project_qkv(dev, *qkv_in, k_cache, v_cache, q_out)
        ops.sliding_attention(dev, *attn_in, attn_out, scale=1.0 / 16)
        dev.check()
        out["q"], out["k_cache"], out["v_cache"], out["attn"] = host(q_out), host(k_cache), host(v_cache), host(attn_out)
        for i in range(REPEATS):
            res = cuda(o["residual"])
            ops.sliding_attention_output(dev, o_in[0], o_in[1], o_in[2], o_in[3], res)
            dev.check()
            out[f"o{i}"] = host(res)
        for i in range(REPEATS):
            res = cuda(f["residual"])
            ops.decoder_feedforward(dev, res, *ffn_in)
            dev.check()
            out[f"ffn{i}"] = host(res)
        # the FP8 feed-forward on BASELINE's Gaussian data, twice
        import gaussian

        g8 = gaussian.ffn_fp8()
        ffn8_in = [cuda(g8["pre_ff_rms_weight"]), cuda(g8["up_weight"], "up_weight"),
                   cuda(g8["gate_weight"], "gate_weight"), cuda(g8["down_weight"], "down_weight"),
                   cuda(g8["up_weight_scale"], "up_channel_scale"), cuda(g8["gate_weight_scale"], "gate_channel_scale"),
                   cuda(g8["down_weight_scale"]), cuda(g8["post_ff_rms_weight"]), cuda(g8["layer_scalar"])]
        for i in range(2):
            res = cuda(g8["residual"])
            ops.decoder_feedforward_fp8(dev, res, *ffn8_in)
            dev.check()
            out[f"ffn8_{i}"] = host(res)
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), **out)
        dist.barrier()
    finally:
        dev.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("world", (2, 4, 8))
def test_tensor_parallel_layer(world, tmp_path, golden_runs):
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp

    mp.start_processes(_tp_rank, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    outs = [dict(np.load(tmp_path / f"rank{r}.npz")) for r in range(world)]

    # QKV: the ranks' heads together against the reference; untouched slots keep the sentinel
    d = synth.sliding_project_qkv(RUN_QKV)
    slot = d["pos"] % RING
    q = np.concatenate([o["q"] for o in outs], axis=0)
    kc = np.concatenate([o["k_cache"] for o in outs], axis=1)
    vc = np.concatenate([o["v_cache"] for o in outs], axis=1)
    for label, got in (("q", q), ("k", kc[slot]), ("v", vc[slot])):
        ok, maxd, exact = within(golden_runs[f"run{RUN_QKV}.sliding_project_qkv.expected.{label}"], got,
                                 ATOL["sliding_project_qkv"])
        assert ok and exact > 0.99, (label, maxd, exact)
    others = np.ones(RING, bool)
    others[slot] = False
    assert np.all(kc[others] == SENTINEL_K) and np.all(vc[others] == SENTINEL_V)

    # attention: per head, against the oracle
    qa, ka, va, mask = _attention_inputs()
    ref = oracle.sliding_attention(qa, ka, va, mask, 1.0 / 16)
    ok, maxd, _ = within(ref, np.concatenate([o["attn"] for o in outs], axis=0), 0.01)
    assert ok, maxd

    # O and FFN: one result on every rank, every call; within the reference's tolerance
    for key, name, run, floor in (("o", "sliding_attention_output", RUN_O, 0.99),
                                  ("ffn", "decoder_feedforward", RUN_FFN, 0.95)):
        first = outs[0][f"{key}0"]
        for o in outs:
            for i in range(REPEATS):
                assert np.array_equal(o[f"{key}{i}"], first), (key, i)
        ok, maxd, exact = within(golden_runs[f"run{run}.{name}.expected"], first, ATOL[name])
        assert ok and exact > floor, (key, maxd, exact)

    # FP8 feed-forward: one result on every rank, each call; against the rank-order oracle
    import gaussian
    import torch
    from g4b200 import tp

    g8 = gaussian.ffn_fp8()
    first = outs[0]["ffn8_0"]
    for o in outs:
        assert np.array_equal(o["ffn8_0"], first) and np.array_equal(o["ffn8_1"], first)

    def cut(name, arr, r):
        return tp.shard(name, torch.from_numpy(arr), r, world).numpy()

    want = oracle.feedforward_fp8_tp(
        g8["residual"], g8["pre_ff_rms_weight"],
        [(cut("up_weight", g8["up_weight"], r), cut("up_channel_scale", g8["up_weight_scale"], r)) for r in range(world)],
        [(cut("gate_weight", g8["gate_weight"], r), cut("gate_channel_scale", g8["gate_weight_scale"], r))
         for r in range(world)],
        [cut("down_weight", g8["down_weight"], r) for r in range(world)], g8["down_weight_scale"],
        g8["post_ff_rms_weight"], g8["layer_scalar"])
    ok, maxd, exact = within(want, first, ATOL["decoder_feedforward"])
    assert ok and exact > 0.95, ("ffn8", maxd, exact)


def test_setup_refusals():
    """Two ranks on one GPU are refused before any kernel runs; an op on a context that is not
    connected yet is refused on the host."""
    if _gpus() < 1:
        pytest.skip("no CUDA device")
    import torch

    from g4b200 import G4Error, _abi, ops

    a, b = ops.Device(0), ops.Device(0)
    try:
        blobs = a.tp_init(0, 2) + b.tp_init(1, 2)
        with pytest.raises(G4Error) as err:
            a.tp_connect(blobs)
        assert err.value.status == _abi.G4_ERR_UNSUPPORTED
        x = torch.zeros((4, 2, 256), dtype=torch.bfloat16, device="cuda")
        res = torch.zeros(3840, dtype=torch.bfloat16, device="cuda")
        w = torch.zeros((3840, 2048), dtype=torch.uint8, device="cuda")
        with pytest.raises(G4Error) as err:
            ops.sliding_attention_output(a, x, res, w, res, res)
        assert err.value.status == _abi.G4_ERR_INVALID_ARGUMENT
        with pytest.raises(G4Error):
            a.tp_init(0, 3)
        blob_a, blob_b = a.tp_init(0, 2), b.tp_init(1, 2)
        with pytest.raises(G4Error) as err:  # blobs out of rank order
            a.tp_connect(blob_b + blob_a)
        assert err.value.status == _abi.G4_ERR_INVALID_ARGUMENT
        a.tp_init(0, 1)  # back to one GPU: the whole layer, no peers
        assert a.world == 1
    finally:
        a.close()
        b.close()
