#!/usr/bin/env python3
"""Benchmark: one Gemma-4-12B sliding decoder layer per token at M=1, on B200.

A step is one token through the four reference ops of a sliding layer, in order:
sliding_project_qkv (FP8) -> sliding_attention (bf16 ring of 1024 slots) ->
sliding_attention_output (FP8) -> decoder_feedforward (NVFP4), all through libg4b200's C ABI.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

- parity: before anything is timed, one step on the bench's own layer is checked against the
  CPU oracle (oracle/ops.py, numpy; the checker, outside every timed region): each op's output
  within the reference grader's tolerance, and under tensor parallelism every rank's residual
  bit for bit the same. The result is the line's "parity" object.
- value: tokens/s through one layer, device-timed with CUDA events over exactly K steps (after
  exactly W warm-up steps) replayed from CUDA graphs, with weights, caches and activations
  resident in HBM (max over ranks). N>1 splits the layer tensor-parallel over the N GPUs (KV
  heads and FFN rows per rank; the O and down partial sums are added across the GPUs inside
  those kernels over NVLink): one token per step for the whole job, strong scaling.
- e2e: the same metric through the public C ABI with host buffers: every step copies the
  token's hidden state and position offsets from pinned host memory to the device, runs the four
  ops and copies the resulting hidden state back to pinned host memory, all inside the timed
  region (captured in the same graphs as the ops).
- roofline: the dominant op (decoder_feedforward, 99.56 MB of algorithmic traffic per call)
  timed alone against the measured HBM copy bandwidth.
- cpu_baseline / --impl reference: the CPU oracle port (numpy, test infrastructure) running the
  same layer step on this host's cores, with every host thread.

Synthetic data (no checkpoint exists on the box): weights ~N(0, 0.02) quantised the way
BASELINE.json describes (FP8 e4m3 per output row; NVFP4 e2m1 codes with e4m3 per-16 block
scales and an f32 per-tensor scale), activations and caches ~N(0, 1). Four distinct layers
(621 MB of weights, > 4x the 126 MB L2) are rotated so no step reads weights from L2.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
for p in (str(REPO), str(REPO / "moa-workspace_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

H, L, NS, GS, DS, QS, PS, TS, E = 3840, 15360, 8, 2, 256, 4096, 2048, 1024, 32768
N_LAYERS = 4


def op_bytes(world=1):
    """Algorithmic bytes one GPU moves per op call at M=1 (weights + scales + activations read
    and written) when the layer is split over `world` tensor-parallel ranks (1: the whole layer)."""
    w, fr = world, L // world
    dk = -(-fr // 256) * 256  # a rank's down K slice, zero-padded to whole 256-element units
    return {
        "sliding_project_qkv": (QS + 2 * PS) // w * H + (QS + 2 * PS) // w * 2 + H * 2 * 2 + DS * 2 * 2
                               + 4 * DS * 2 + 2 * NS // w * DS * 2 + QS // w * 2,
        "sliding_attention": 2 * TS * NS // w * DS * 2 + QS // w * 2 * 2 + TS * 4,
        "sliding_attention_output": H * QS // w + H * 2 + QS // w * 2 + H * 2 * 3,
        "decoder_feedforward": 2 * (fr * H // 2 + fr * H // 16) + (H * dk // 2 + H * dk // 16) + H * 2 * 4 + 8 * 2
                               + 12,
    }


BYTES = op_bytes(1)
# DRAM bytes read + written per decoder_feedforward call (ffn_upgate + ffn_down): ncu --set full
# capture of `python bench.py --only ffn --steps 3 --warmup 3` (dram__bytes_read.sum + write.sum)
FFN_TRAFFIC = 66.43e6 + 0.66e6 + 33.37e6
METRIC = "decode tokens/s through one Gemma-4 sliding decoder layer (QKV + attention + O + FFN ops, M=1)"
WORKLOAD = ("gemma4-12b sliding decoder layer, M=1: fused QKV fp8 [8192x3840] + sliding attention "
            "(ring 1024 x 8 heads x 256, scale 1.0) + O fp8 [3840x4096] + NVFP4 GeGLU FFN [2x15360x3840 + 3840x15360]")


def peaks():
    try:
        return json.loads((REPO / "MEASURED_PEAKS.json").read_text()), "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


# ------------------------------------------------------------------------------ clocks

class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,utilization.gpu,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.samples = []
        self._stop = threading.Event()
        self._thread = None

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.QUERY}",
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=5)
                f = [x.strip() for x in out.stdout.strip().split(",")]
                if len(f) >= 9:
                    self.samples.append(f)
            except Exception:
                pass
            self._stop.wait(0.1)

    def __enter__(self):
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        self._thread.join(timeout=10)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no nvidia-smi samples"], "samples": 0}
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        busy = [float(s[1]) for s in self.samples if s[4].isdigit() and int(s[4]) > 0 and s[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4) if s[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(busy or sm) if (busy or sm) else None,
                "sm_max_mhz": float(self.samples[0][2]) if self.samples[0][2].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(self.samples), "samples_busy": len(busy)}


# ------------------------------------------------------------------------------ synthetic model

def quant_fp8_rows(w):
    """Per-output-row e4m3: scale = amax/448, codes = e4m3(w / scale)."""
    import torch

    amax = w.abs().amax(dim=1, keepdim=True).clamp_min(1e-12)
    scale = amax / 448.0
    codes = (w / scale).to(torch.float8_e4m3fn).view(torch.uint8)
    return codes.contiguous(), scale.squeeze(1)


def quant_nvfp4(w):
    """NVFP4: f32 global = amax/(6*448); e4m3 scale per 16 = block amax/6/global; e2m1 codes.

    The op takes the global multiplier itself: the reciprocal of a checkpoint's
    weight_global_scale (= 6*448/amax), as the reference's loader passes it
    (FOG/src/host/load.rs:170-190)."""
    import torch

    rows, cols = w.shape
    g = (w.abs().amax() / (6.0 * 448.0)).clamp_min(1e-12)
    blocks = w.view(rows, cols // 16, 16)
    bscale = (blocks.abs().amax(dim=2) / 6.0 / g).to(torch.float8_e4m3fn)
    denom = (bscale.float() * g).clamp_min(1e-30).unsqueeze(2)
    x = (blocks / denom).reshape(rows, cols)
    bounds = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], device=w.device)
    mag = torch.bucketize(x.abs(), bounds).to(torch.uint8)
    codes = mag | ((x < 0).to(torch.uint8) << 3)
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).contiguous()
    return packed, bscale.view(torch.uint8).contiguous(), g.reshape(1).to(torch.float32).contiguous()


class Layer:
    """One decoder layer's weights and ring caches (whole; `shard` keeps one rank's slices).

    keep_host=True also keeps a host copy of the whole layer's tensors in the reference layout
    (`self.host`, numpy: bf16 as uint16 bits, codes as uint8), for the parity check."""

    def __init__(self, gen, dev, keep_host=False):
        import torch

        def normal(*shape, std=1.0):
            return torch.randn(*shape, generator=gen, device=dev) * std

        def bf(t):
            return t.to(torch.bfloat16).contiguous()

        self.input_rms = bf(1 + normal(H, std=0.1))
        qkv = [quant_fp8_rows(normal(r, H, std=0.02)) for r in (QS, PS, PS)]
        (self.q_w, q_s), (self.k_w, k_s), (self.v_w, v_s) = qkv
        self.q_s, self.k_s, self.v_s = bf(q_s), bf(k_s), bf(v_s)
        self.q_rms, self.k_rms = bf(1 + normal(DS, std=0.1)), bf(1 + normal(DS, std=0.1))
        self.k_cache = bf(normal(TS, NS, DS))
        self.v_cache = bf(normal(TS, NS, DS))
        self.post_attn_rms = bf(1 + normal(H, std=0.1))
        self.o_w, o_s = quant_fp8_rows(normal(H, QS, std=0.02))
        self.o_s = bf(o_s)
        self.pre_ff_rms = bf(1 + normal(H, std=0.1))
        self.post_ff_rms = bf(1 + normal(H, std=0.1))
        self.up_p, self.up_s, self.up_g = quant_nvfp4(normal(L, H, std=0.02))
        self.gate_p, self.gate_s, self.gate_g = quant_nvfp4(normal(L, H, std=0.02))
        self.down_p, self.down_s, self.down_g = quant_nvfp4(normal(H, L, std=0.02))
        self.layer_scalar = bf(torch.full((8,), 0.375, device=dev))
        self.tiled = False
        self.host = {k: host_array(getattr(self, k)) for k in self.HOST} if keep_host else None

    HOST = ("input_rms", "q_w", "k_w", "v_w", "q_s", "k_s", "v_s", "q_rms", "k_rms", "post_attn_rms", "o_w", "o_s",
            "pre_ff_rms", "post_ff_rms", "up_p", "up_s", "up_g", "gate_p", "gate_s", "gate_g", "down_p", "down_s",
            "down_g", "layer_scalar")

    # attribute -> the reference op parameter it is passed as (g4b200.tp's slicing rules)
    SHARDED = {"q_w": "q_weight", "k_w": "k_weight", "v_w": "v_weight", "q_s": "q_weight_scale",
               "k_s": "k_weight_scale", "v_s": "v_weight_scale", "k_cache": "k_cache", "v_cache": "v_cache",
               "o_w": "o_weight", "up_p": "up_weight_packed", "gate_p": "gate_weight_packed",
               "up_s": "up_weight_scale", "gate_s": "gate_weight_scale", "down_p": "down_weight_packed",
               "down_s": "down_weight_scale"}

    def shard(self, rank, world):
        """Keep tensor-parallel rank `rank`'s slices of the sliced tensors."""
        from g4b200 import tp

        for attr, name in self.SHARDED.items():
            setattr(self, attr, tp.shard(name, getattr(self, attr), rank, world))
        return self

    def tile(self, ops, device):
        """Repack the weight matrices into the GPU-native unit-tiled layout (once, at load)."""
        for attr, name in (("q_w", "q_weight"), ("k_w", "k_weight"), ("v_w", "v_weight"), ("o_w", "o_weight"),
                           ("down_p", "down_weight_packed"), ("down_s", "down_weight_scale")):
            setattr(self, attr, ops.tile_weight(device, name, getattr(self, attr)))
        self.upgate_p = ops.pack_upgate(device, self.up_p, self.gate_p, scales=False)
        self.upgate_s = ops.pack_upgate(device, self.up_s, self.gate_s, scales=True)
        self.up_p = self.gate_p = self.up_s = self.gate_s = None
        self.tiled = True
        return self


def host_array(t):
    """A torch tensor as numpy on the host: bf16 as uint16 bits, everything else as it is."""
    import numpy as np
    import torch

    t = t.detach().contiguous().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    if t.dtype == torch.float8_e4m3fn:
        return t.view(torch.uint8).numpy().copy()
    return t.numpy().copy()


class Workspace:
    """Per-token buffers shared by the layers (the reference host's Workspace/Decode)."""

    def __init__(self, gen, dev, pos=1763, world=1):
        import numpy as np
        import torch

        from oracle.ops import negate_low_half, rope_tables  # table construction only

        self.pos = pos
        self.residual = (torch.randn(H, generator=gen, device=dev)).to(torch.bfloat16)
        cos = np.zeros((E, DS), np.float32)
        sin = np.zeros((E, DS), np.float32)
        c, s = rope_tables(DS, 10_000.0, 1.0, pos)
        cos[pos], sin[pos] = c, negate_low_half(s)
        self.cos = torch.from_numpy(cos).to(dev).to(torch.bfloat16)
        self.sin = torch.from_numpy(sin).to(dev).to(torch.bfloat16)
        self.kv_offset = torch.tensor([(pos % TS) * NS * DS * 2], dtype=torch.int32, device=dev)
        self.rope_offset = torch.tensor([pos * DS * 2], dtype=torch.int32, device=dev)
        self.mask = (torch.arange(TS, device=dev) <= pos).to(torch.float32)
        self.q = torch.zeros((NS // world, GS, DS), dtype=torch.bfloat16, device=dev)  # this rank's heads
        self.attn = torch.zeros((NS // world, GS, DS), dtype=torch.bfloat16, device=dev)


def layer_step(ops, device, w: Workspace, lay: Layer, which=("qkv", "attn", "o", "ffn")):
    if "qkv" in which:
        ops.sliding_project_qkv(device, w.residual, lay.q_w, lay.k_w, lay.v_w, lay.q_s, lay.k_s, lay.v_s,
                                lay.input_rms, lay.q_rms, lay.k_rms, w.kv_offset, w.rope_offset, w.cos, w.sin,
                                lay.k_cache, lay.v_cache, w.q, tiled=lay.tiled)
    if "attn" in which:
        ops.sliding_attention(device, w.q, lay.k_cache, lay.v_cache, w.mask, w.attn, scale=ATTN_SCALE)
    if "o" in which:
        ops.sliding_attention_output(device, w.attn, lay.post_attn_rms, lay.o_w, lay.o_s, w.residual,
                                     tiled=lay.tiled)
    if "ffn" in which and lay.tiled:
        ops.decoder_feedforward_tiled(device, w.residual, lay.pre_ff_rms, lay.upgate_p, lay.down_p, lay.upgate_s,
                                      lay.down_s, lay.up_g, lay.gate_g, lay.down_g, lay.post_ff_rms, lay.layer_scalar)
    elif "ffn" in which:
        ops.decoder_feedforward(device, w.residual, lay.pre_ff_rms, lay.up_p, lay.gate_p, lay.down_p, lay.up_s,
                                lay.gate_s, lay.down_s, lay.up_g, lay.gate_g, lay.down_g, lay.post_ff_rms,
                                lay.layer_scalar)


KERNELS_PER_OP = {"qkv": 1, "attn": 1, "o": 1, "ffn": 2}
ATTN_SCALE = 1.0  # the reference model's sliding attention (gemma4.py:179-181)


# ------------------------------------------------------------------------------ parity gate

# the reference grader's tolerances (FOG/src/bin/test_kernels.rs:447-465): |want - got| <=
# atol + rtol |want|; attention (never graded by the reference) is held to 0.01
RTOL = 1e-2
ATOL = {"sliding_project_qkv": 0.04, "sliding_attention": 0.01, "sliding_attention_output": 0.05,
        "decoder_feedforward": 0.01}


def compare(name, want, got):
    import numpy as np

    from oracle.ops import bf16_to_f32

    w, g = bf16_to_f32(np.asarray(want).reshape(-1)), bf16_to_f32(np.asarray(got).reshape(-1))
    diff = np.abs(w - g)
    ok = bool(np.isfinite(g).all() and (diff <= ATOL[name] + RTOL * np.abs(w)).all())
    return {"ok": ok, "max_abs": float(diff.max()), "atol": ATOL[name], "rtol": RTOL,
            "bit_exact": round(float(np.mean(np.asarray(want).reshape(-1) == np.asarray(got).reshape(-1))), 5)}


def parity_step(ops, device, ws, lay, rank, world, dist):
    """Run one layer step op by op and check every op's output against the CPU oracle, each op
    on the inputs the GPU's previous op produced (so a failure names the op). Under tensor
    parallelism the ranks' slices are gathered to rank 0, the O and FFN oracles add the ranks'
    partial sums in rank order (oracle/ops.py *_tp), and every rank's residual must have the
    same bits. Returns the line's "parity" object on rank 0 (None elsewhere)."""
    import numpy as np
    import torch

    from g4b200 import tp

    def gather(t):  # every rank's tensor, in rank order, on rank 0's host
        t = t.contiguous()
        if world == 1:
            return [host_array(t)]
        parts = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(parts, t)
        return [host_array(p) for p in parts]

    slot = ws.pos % TS
    res0 = host_array(ws.residual)
    layer_step(ops, device, ws, lay, ("qkv",))
    device.check()
    q = np.concatenate(gather(ws.q), axis=0)
    kc = np.concatenate(gather(lay.k_cache), axis=1)
    vc = np.concatenate(gather(lay.v_cache), axis=1)
    layer_step(ops, device, ws, lay, ("attn",))
    device.check()
    attn_parts = gather(ws.attn)
    layer_step(ops, device, ws, lay, ("o",))
    device.check()
    res1_parts = gather(ws.residual)
    layer_step(ops, device, ws, lay, ("ffn",))
    device.check()
    res2_parts = gather(ws.residual)
    cos, sin = host_array(ws.cos[ws.pos]), host_array(ws.sin[ws.pos])
    mask = host_array(ws.mask)
    if rank != 0:
        return None

    from oracle import ops as oracle

    h = lay.host
    out = {}
    wq, wk, wv = oracle.sliding_project_qkv(res0, h["q_w"], h["k_w"], h["v_w"], h["q_s"], h["k_s"], h["v_s"],
                                            h["input_rms"], h["q_rms"], h["k_rms"], cos, sin)
    got = np.concatenate([q.reshape(-1), kc[slot].reshape(-1), vc[slot].reshape(-1)])
    out["sliding_project_qkv"] = compare("sliding_project_qkv", np.concatenate(
        [wq.reshape(-1), wk.reshape(-1), wv.reshape(-1)]), got)
    attn = np.concatenate(attn_parts, axis=0)
    out["sliding_attention"] = compare("sliding_attention", oracle.sliding_attention(q, kc, vc, mask, ATTN_SCALE),
                                       attn)

    def cut(name, arr):
        return tp.shard(name, torch.from_numpy(arr), r, world).numpy()

    if world == 1:
        want_o = oracle.sliding_attention_output(attn, h["post_attn_rms"], h["o_w"], h["o_s"], res0)
        want_f = oracle.decoder_feedforward(res1_parts[0], h["pre_ff_rms"], h["up_p"], h["gate_p"], h["down_p"],
                                            h["up_s"], h["gate_s"], h["down_s"], h["up_g"][0], h["gate_g"][0],
                                            h["down_g"][0], h["post_ff_rms"], h["layer_scalar"])
    else:
        o_parts, up, gate, down = [], [], [], []
        for r in range(world):
            o_parts.append(cut("o_weight", h["o_w"]))
            up.append((cut("up_weight_packed", h["up_p"]), cut("up_weight_scale", h["up_s"])))
            gate.append((cut("gate_weight_packed", h["gate_p"]), cut("gate_weight_scale", h["gate_s"])))
            down.append((cut("down_weight_packed", h["down_p"]), cut("down_weight_scale", h["down_s"])))
        want_o = oracle.sliding_attention_output_tp([a.reshape(-1) for a in attn_parts], h["post_attn_rms"], o_parts,
                                                    h["o_s"], res0)
        want_f = oracle.decoder_feedforward_tp(res1_parts[0], h["pre_ff_rms"], up, gate, down, h["up_g"][0],
                                               h["gate_g"][0], h["down_g"][0], h["post_ff_rms"], h["layer_scalar"])
    out["sliding_attention_output"] = compare("sliding_attention_output", want_o, res1_parts[0])
    out["decoder_feedforward"] = compare("decoder_feedforward", want_f, res2_parts[0])
    same = all(np.array_equal(p, res1_parts[0]) for p in res1_parts) and \
        all(np.array_equal(p, res2_parts[0]) for p in res2_parts)
    return {"ok": all(v["ok"] for v in out.values()) and same, "ranks_bit_identical": same if world > 1 else None,
            "ops": out, "checked": f"one step on layer copy 0 at position {ws.pos}, each op against oracle/ops.py "
                                   "(numpy) on the previous op's GPU output" +
                                   (", O/FFN as the rank-order sum of the ranks' partials" if world > 1 else "")}


# ------------------------------------------------------------------------------ timing helpers

def capture(torch, fn, reps):
    """A CUDA graph of fn(0), ..., fn(reps - 1) (fn issues work on the current stream)."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn(0)  # warm the launch path outside capture
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(reps):
            fn(i)
    return g


class Stepper:
    """Replays exactly n steps of `step(layer)` rotating over `n_layers` layer copies: a graph of
    `block` steps (a multiple of n_layers, starting at layer 0) where it fits, one-step graphs
    (one per layer copy) elsewhere, so any n is honoured without breaking the rotation."""

    def __init__(self, torch, step, n_layers, block):
        assert block % n_layers == 0
        self.n_layers, self.block = n_layers, block
        self.big = capture(torch, lambda i: step(i % n_layers), block)
        self.single = [capture(torch, lambda i, lay=lay: step(lay), 1) for lay in range(n_layers)]
        self.at = 0  # index of the next step (its layer is at % n_layers)

    def run(self, n):
        left = n
        while left:
            if self.at % self.n_layers == 0 and left >= self.block:
                self.big.replay()
                self.at += self.block
                left -= self.block
            else:
                self.single[self.at % self.n_layers].replay()
                self.at += 1
                left -= 1


def timed(torch, fn):
    """Device seconds of fn()'s work on the current stream (CUDA events, synchronised on both sides)."""
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record()
    fn()
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end) / 1e3


def max_over_ranks(torch, dist, dev, secs):
    if dist is None:
        return secs
    t = torch.tensor([secs], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def config_for(world):
    return {"workload": WORKLOAD, "global_batch": 1, "seq_len": TS,
            "parallelism": f"tp{world}" if world > 1 else "single GPU",
            "l2": f"inputs larger than L2: {N_LAYERS} distinct layers ({N_LAYERS * sum(op_bytes(world).values()) / 1e6:.0f}"
                  " MB per GPU) rotated step to step",
            "launch": "CUDA graphs of C-ABI calls, programmatic dependent launch"}


# ------------------------------------------------------------------------------ CPU legs

def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


class CpuLayer:
    """The oracle port (numpy, all BLAS threads) running the same layer step on the host."""

    def __init__(self):
        import numpy as np

        from oracle import ops as oracle

        self.np, self.oracle = np, oracle
        rng = np.random.default_rng(1234)

        def bf(a):
            return oracle.f32_to_bf16(np.asarray(a, np.float32))

        t0 = time.time()
        # dequantised f32 weights stand in for codes x scale: the oracle contracts in f32 either way
        self.wq = rng.standard_normal((QS + 2 * PS, H), dtype=np.float32) * 0.02
        self.wo = rng.standard_normal((H, QS), dtype=np.float32) * 0.02
        self.w_up = rng.standard_normal((L, H), dtype=np.float32) * 0.02
        self.w_gate = rng.standard_normal((L, H), dtype=np.float32) * 0.02
        self.w_down = rng.standard_normal((H, L), dtype=np.float32) * 0.02
        self.k_cache = bf(rng.standard_normal((TS, NS, DS)))
        self.v_cache = bf(rng.standard_normal((TS, NS, DS)))
        self.gam = bf(1 + 0.1 * rng.standard_normal(H))
        self.gam_d = bf(1 + 0.1 * rng.standard_normal(DS))
        cos_raw, sin_raw = oracle.rope_tables(DS, 10_000.0, 1.0, 1763)
        self.cos_b, self.sin_b = bf(cos_raw), bf(sin_raw)
        self.mask = np.ones(TS, np.float32)
        self.residual = bf(rng.standard_normal(H))
        self.scales = np.full(QS + 2 * PS, 1e-3, np.float32)
        self.setup_s = time.time() - t0
        self.step()  # warm caches and BLAS threads

    def step(self):
        np, oracle = self.np, self.oracle
        h = oracle.rms_norm(self.residual, self.gam)
        proj = oracle.scaled_projection(h, self.wq, self.scales)
        q = oracle.rope(oracle.rms_norm(proj[:QS].reshape(16, DS), self.gam_d), self.cos_b, self.sin_b)
        k = oracle.rope(oracle.rms_norm(proj[QS:QS + PS].reshape(8, DS), self.gam_d), self.cos_b, self.sin_b)
        v = oracle.rms_norm(proj[QS + PS:].reshape(8, DS), None)
        self.k_cache[763], self.v_cache[763] = k, v
        attn = oracle.sliding_attention(q.reshape(8, 2, DS), self.k_cache, self.v_cache, self.mask)
        o = oracle.scaled_projection(attn.reshape(-1), self.wo, np.float32(1e-3))
        residual = oracle.add_bf16(self.residual, oracle.rms_norm(o, self.gam))
        self.residual = oracle.feedforward_dense(residual, self.gam, self.gam, self.w_up, self.w_gate, self.w_down,
                                                 1.0, 1.0, 1.0, np.array([0x3EC0], np.uint16))

    def sample(self, budget_s: float, min_steps: int = 1):
        n, t0 = 0, time.time()
        while n < min_steps or time.time() - t0 < budget_s:
            self.step()
            n += 1
        elapsed = time.time() - t0
        return n / elapsed, (f"{n} layer steps of the numpy oracle port over {elapsed:.1f} s on {host_threads()} host "
                             f"threads (f32 BLAS GEMV on pre-dequantised weights; "
                             f"{self.setup_s:.1f} s of weight setup untimed)")


def use_all_host_threads():
    """Every host thread for the CPU legs: torchrun sets OMP_NUM_THREADS=1 for its ranks, which
    would leave the BLAS of the numpy port on one core. Set before numpy loads its BLAS, and
    again through threadpoolctl in case it was already loaded."""
    n = host_threads()
    for var in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
        os.environ[var] = str(n)
    try:
        from threadpoolctl import threadpool_limits

        threadpool_limits(limits=n)
    except Exception:
        pass
    return n


def run_reference(args):
    """The reference arm: the CPU oracle port on this host, same metric and workload.

    Under torchrun only rank 0 runs it (the others exit at once). Each step is one layer step of
    the port; at most ~90 s of steps run (the rest of K would repeat identical work), and the
    line reports the median per-step rate."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    cores = use_all_host_threads()
    cpu = CpuLayer()
    for _ in range(args.warmup):
        cpu.step()
    rates = []
    t0 = time.time()
    for _ in range(args.steps):
        s0 = time.time()
        cpu.step()
        rates.append(1.0 / (time.time() - s0))
        if time.time() - t0 > 90.0:
            break
    value = statistics.median(rates)
    sample = (f"{len(rates)} of {args.steps} requested layer steps of the numpy oracle port (median rate) on "
              f"{cores} host threads; f32 BLAS GEMV on pre-dequantised weights, {cpu.setup_s:.1f} s setup untimed")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": len(rates), "warmup": args.warmup, "ms_per_step": 1e3 / value, "higher_is_better": True,
        "scaling": "strong" if args.gpus > 1 else "weak", "vs_baseline": None,
        "dtype": "f32 (numpy oracle port, bf16 rounding points emulated)",
        "data": "synthetic", "config": dict(config_for(args.gpus), parallelism=f"host CPU, {cores} threads, one process",
                                           launch="numpy on the host"),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------------------ GPU leg

def run_ours(args):
    import torch

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))

    from g4b200 import ops, tp

    device = ops.Device(local)
    device.set_overlap(True)
    if dist:
        tp.connect(device)  # this GPU is tensor-parallel rank `rank` of `world`
    dev = torch.device("cuda", local)
    gen = torch.Generator(device=dev)
    gen.manual_seed(1000)  # the same whole layers on every rank; each keeps its slices
    layers = [Layer(gen, dev, keep_host=(i == 0 and rank == 0 and not args.no_parity)).shard(rank, world).tile(ops, device)
              for i in range(N_LAYERS)]
    ws = Workspace(gen, dev, world=world)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()  # the ranks' kernels wait on each other (bounded): start them together

    # --- correctness gate before timing: one step against the CPU oracle
    parity = None if args.no_parity else parity_step(ops, device, ws, layers[0], rank, world, dist)
    if dist:
        dist.barrier()

    # --- device-resident throughput: exactly W then K steps from graphs, layers rotated
    per_graph = N_LAYERS * 4
    stepper = Stepper(torch, lambda lay: layer_step(ops, device, ws, layers[lay]), N_LAYERS, per_graph)
    stepper.run(args.warmup)
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    if dist:
        dist.barrier()
    with sampler:
        elapsed = max_over_ranks(torch, dist, dev, timed(torch, lambda: stepper.run(args.steps)))
        device.check()
        value = args.steps / elapsed  # one token through the layer per step, for the whole job

        # --- per-op device time (each op alone, graph of many calls rotating the layers)
        op_us = {}
        reps = 64
        if dist:
            dist.barrier()
        for key, name in (("qkv", "sliding_project_qkv"), ("attn", "sliding_attention"),
                          ("o", "sliding_attention_output"), ("ffn", "decoder_feedforward")):
            g = capture(torch, lambda i, k=key: layer_step(ops, device, ws, layers[i % N_LAYERS], (k,)), reps)
            g.replay()
            op_us[name] = max_over_ranks(torch, dist, dev, timed(torch, lambda: [g.replay() for _ in range(5)])) \
                / (5 * reps) * 1e6
            del g
        device.check()

        # --- end to end through the C ABI from pinned host buffers: every step copies its input
        # hidden state and position offsets in and its resulting hidden state out
        host_in = torch.empty(H, dtype=torch.bfloat16).pin_memory()
        host_kv = torch.empty(1, dtype=torch.int32).pin_memory()
        host_rope = torch.empty(1, dtype=torch.int32).pin_memory()
        host_out = torch.empty(H, dtype=torch.bfloat16).pin_memory()
        host_in.copy_(ws.residual.cpu())
        host_kv.copy_(ws.kv_offset.cpu())
        host_rope.copy_(ws.rope_offset.cpu())

        def e2e_step(lay):
            ws.residual.copy_(host_in, non_blocking=True)
            ws.kv_offset.copy_(host_kv, non_blocking=True)
            ws.rope_offset.copy_(host_rope, non_blocking=True)
            layer_step(ops, device, ws, layers[lay])
            host_out.copy_(ws.residual, non_blocking=True)

        e2e = Stepper(torch, e2e_step, N_LAYERS, per_graph)
        e2e.run(args.warmup)
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        e2e_elapsed = max_over_ranks(torch, dist, dev, timed(torch, lambda: e2e.run(args.steps)))
    device.check()
    e2e_value = args.steps / e2e_elapsed
    del stepper, e2e

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        use_all_host_threads()
        rate, sample = CpuLayer().sample(budget_s=12.0, min_steps=3)
        cpu = {"value": rate, "unit": "tokens/s", "cores": host_threads(), "kind": "port", "sample": sample}

    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0

    pk, pk_kind = peaks()
    rank_bytes = op_bytes(world)
    ffn_bytes = rank_bytes["decoder_feedforward"]
    achieved = ffn_bytes / (op_us["decoder_feedforward"] * 1e-6) / 1e9
    layer_bytes = sum(rank_bytes.values())  # per GPU
    line = {
        "metric": METRIC,
        "value": value,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": elapsed / args.steps * 1e3,
        "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "arithmetic": "tcgen05: fp8 e4m3 weights (kind::f8f6f4) x the bf16 activation as exact e4m3 terms; nvfp4 "
                      "e2m1 weights with e4m3 block scales (kind::mxf4nvf4) x the activation as exact e2m1 digits; "
                      "f32 accumulation in TMEM",
        "data": "synthetic",
        "config": config_for(world),
        "parity": parity,
        "ops_us": {k: round(v, 3) for k, v in op_us.items()},
        "ops_gbs": {k: round(rank_bytes[k] / (op_us[k] * 1e-6) / 1e9, 1) for k in op_us},
        "layer_bytes_per_gpu": layer_bytes,
        "layer_gbs_per_gpu": round(layer_bytes * args.steps / elapsed / 1e9, 1),
        "roofline": {"bound": "hbm", "kernel": "decoder_feedforward (ffn_upgate + ffn_down kernels, one GPU's slice)",
                     "achieved": round(achieved, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / pk["hbm_gbs"], 4), "peak_source": pk_kind,
                     "algorithmic_bytes_per_launch": ffn_bytes,
                     "traffic": args.traffic if world == 1 else None},
        "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": (H * 2 + 8) * world,
                "d2h_bytes_per_step": H * 2 * world, "steps": args.steps,
                "how": "CUDA graphs of [pinned host->device copy of the hidden state and offsets, the four C-ABI ops, "
                       "device->pinned host copy of the new hidden state] per step"},
        "gpu_launches": args.steps * sum(KERNELS_PER_OP.values()),
        "clocks": sampler.summary(),
        "cpu_baseline": cpu,
    }
    print(json.dumps(line), flush=True)
    return 0


def run_only(args):
    """Eager calls of one op (no graph, no CPU leg): the small case the ncu captures use.

    Runs --warmup + --steps calls of the op on one layer copy per call (rotating the layers)
    and prints the mean device time per call."""
    import torch

    from g4b200 import ops

    device = ops.Device(0)
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev)
    gen.manual_seed(1000)
    layers = [Layer(gen, dev).tile(ops, device) for _ in range(N_LAYERS)]
    ws = Workspace(gen, dev)
    for i in range(args.warmup):
        layer_step(ops, device, ws, layers[i % N_LAYERS], (args.only,))
    device.check()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(args.steps):
        layer_step(ops, device, ws, layers[i % N_LAYERS], (args.only,))
    end.record()
    device.check()
    us = start.elapsed_time(end) * 1e3 / max(args.steps, 1)
    print(json.dumps({"only": args.only, "calls": args.steps, "us_per_call": round(us, 3),
                      "launches_per_call": KERNELS_PER_OP[args.only]}), flush=True)
    device.close()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", choices=sorted(KERNELS_PER_OP), default=None,
                    help="profiling aid: eager calls of one op only (prints us/call, not the bench line)")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2048)
    ap.add_argument("--warmup", type=int, default=64)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--no-parity", action="store_true", help="skip the parity gate (profiling runs)")
    ap.add_argument("--traffic", type=float, default=FFN_TRAFFIC,
                    help="ncu dram bytes (read + write) per decoder_feedforward call")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.steps < 1:
        ap.error("--steps must be at least 1")
    if args.only:
        return run_only(args)
    return run_reference(args) if args.impl == "reference" else run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
