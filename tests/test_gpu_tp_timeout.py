"""GPU, two ranks on two GPUs: a peer that misses an exchange. The bounded wait of the O kernel's
in-kernel all-reduce runs out (the limit set to 20 ms with g4_tp_set_wait_limit), the rank that
waited gets G4_DEVERR_PEER_TIMEOUT from g4_ctx_check with its residual rows poisoned (NaN), its
context refuses further ops until the group is set up again, and after every rank runs the setup
again (g4b200.tp.connect: a host barrier, g4_tp_init, g4_tp_connect) the next call matches the
reference's golden output on both ranks, bit-identical between them.

The failure is made on the host: rank 1 skips one call. Nothing faults or hangs a GPU: the wait is
bounded on %globaltimer, the exchange is plain 64-bit peer loads and stores (no multicast), and
the ranks coordinate over gloo (no NCCL)."""

import os
import socket

import numpy as np
import pytest

from helpers import ATOL, within
from oracle import ops as oracle
from oracle import synth

pytestmark = pytest.mark.gpu
RUN_O = 4


def _gpus():
    import torch

    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out_dir):
    import datetime

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    from g4b200 import G4Error, _abi, ops, tp

    dev = ops.Device(rank)

    def cuda(arr, name=None):
        a = np.ascontiguousarray(arr)
        x = torch.from_numpy(a.view(np.int16) if a.dtype == np.uint16 else a)
        if name is not None:
            x = tp.shard(name, x, rank, world)
        x = x.cuda()
        return x.view(torch.bfloat16) if a.dtype == np.uint16 else x

    def host(x):
        return x.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)

    o = synth.sliding_attention_output(RUN_O)
    o_in = [cuda(o["x"], "attn"), cuda(o["post_attn_rms_weight"]), cuda(o["o_weight"], "o_weight"),
            cuda(o["o_weight_scale"])]
    out = {}
    try:
        dev.tp_set_wait_limit(0.02)
        tp.connect(dev)

        def call():
            res = cuda(o["residual"])
            ops.sliding_attention_output(dev, *o_in, res)
            return res

        res = call()
        dev.check()
        out["before"] = host(res)
        dist.barrier()
        if rank == 0:  # rank 1 skips this call: rank 0's exchange waits 20 ms, then gives up
            res = call()
            try:
                dev.check()
                out["flags"] = np.array([0])
            except G4Error as e:
                out["flags"] = np.array([e.flags])
            out["poisoned"] = host(res)
            try:  # refused on the host until the group is set up again
                call()
                out["refused"] = np.array([0])
            except G4Error as e:
                out["refused"] = np.array([int(e.status == _abi.G4_ERR_INVALID_ARGUMENT)])
        dist.barrier()
        tp.connect(dev)  # every rank: barrier, then a new setup (a new generation of exchange words)
        res = call()
        dev.check()
        out["after"] = host(res)
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), **out)
        dist.barrier()
    finally:
        dev.close()
        dist.destroy_process_group()


def test_missed_exchange_times_out_and_the_group_recovers(tmp_path, golden_runs):
    if _gpus() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    mp.start_processes(_rank, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    r0, r1 = (dict(np.load(tmp_path / f"rank{r}.npz")) for r in range(2))
    assert r0["flags"][0] & 32, r0["flags"]  # G4_DEVERR_PEER_TIMEOUT
    assert np.isnan(oracle.bf16_to_f32(r0["poisoned"])).any()
    assert r0["refused"][0] == 1
    want = golden_runs[f"run{RUN_O}.sliding_attention_output.expected"]
    for key in ("before", "after"):
        assert np.array_equal(r0[key], r1[key]), key
        ok, maxd, exact = within(want, r0[key], ATOL["sliding_attention_output"])
        assert ok and exact > 0.99, (key, maxd, exact)
    assert np.array_equal(r0["before"], r0["after"])
