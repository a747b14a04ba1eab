#!/usr/bin/env python3
"""Benchmark: Gemma-4-12B-shaped decode on B200 (batch 1).

A step is one token through the whole model, issued by the library's decode driver
(g4_decoder_step, replaying the CUDA graph it captured): the token's embedding (embed_token), 48
decoder layers (each: sliding_project_qkv -> sliding_attention -> sliding_attention_output ->
decoder_feedforward_fp8), then final_norm_and_logits over the 262144-row lm_head. The layers follow
BASELINE's 5:1 pattern: 40 sliding layers on 1024-slot rings with the local RoPE table (theta 1e4)
and 8 global-shaped layers (every sixth) on 4096-slot rings with the global table (theta 1e6),
all with the sliding geometry (16 query / 8 KV heads x 256). Weights are FP8 e4m3 with per-row
scales (the feed-forward's f32), 48 distinct layers (10.8 GB), so no step reads weights from L2.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

- parity: before anything is timed, (1) one decode step equals the same ops called one by one
  through their own entry points, bit for bit (hidden state and logits), and under tensor
  parallelism every rank's hidden state has the same bits; (2) every op of a sliding and of a
  global layer, the NVFP4 feed-forward and a sample of the logits match the CPU oracle
  (oracle/ops.py, numpy, the checker, outside every timed region) within the reference grader's
  tolerances. The result is the line's "parity" object.
- value: decode tokens/s, device-timed with CUDA events over exactly K steps after exactly W
  warm-up steps (max over ranks). N>1 splits every layer tensor-parallel over the N GPUs (KV heads
  and FFN rows per rank, the O and down partial sums added inside those kernels over NVLink; the
  lm_head split by vocabulary rows): one token per step for the whole job, strong scaling.
- e2e: the same metric through the public C ABI with host buffers: every step copies the token id
  and position from pinned host memory to the device, runs the decode step and copies the logits
  back to pinned host memory, all inside the timed region (one CUDA graph per step).
- ops_us / ops_frac: each op alone (a graph of 64 calls rotating over the model's layers), its
  algorithmic bytes over its time against the measured HBM bandwidth; decoder_feedforward (NVFP4,
  configs[3] at M = 1) runs on four extra NVFP4 layer copies.
- roofline: the dominant kernel pair, decoder_feedforward_fp8 (177.1 MB per call, configs[0]).
- cpu_baseline / --impl reference: the CPU oracle port (numpy, test infrastructure) running the
  same decode step on this host's cores, with every host thread.
- decode_batch (one GPU): configs[4]'s batches 8 and 32 - that many sequences decoded together by
  a batched decoder (g4_decoder_create_batch: the same 48 layers, each cache holding one ring per
  sequence), tokens/s = sequences x K / the device time of exactly K steps after W.

Synthetic data (no checkpoint exists on the box): weights ~N(0, 0.02) quantised the way
BASELINE.json describes, the embedding / lm_head table ~N(0, 0.03) bf16, caches ~N(0, 1).
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

H, L, NS, GS, DS, QS, PS, E, W = 3840, 15360, 8, 2, 256, 4096, 2048, 32768, 262144
N_MODEL = 48          # decoder layers (FOG/src/lib.rs:22)
GLOBAL_EVERY = 6      # layer i is global-shaped when i % 6 == 5 (5 local : 1 global)
RING_LOCAL, RING_GLOBAL = 1024, 4096
NVFP4_COPIES = 4      # NVFP4 layer copies for the configs[3] per-op timing (> 3x L2 together)
POSITION = 4000       # the decoded token's position (context 4096)
KERNELS_PER_LAYER = 5  # qkv, attention, o, ffn up/gate, ffn down
BATCH_SWEEP = (8, 16, 64)
DECODE_BATCHES = (8, 32)  # configs[4]'s batches beyond 1: sequences decoded together (one GPU)  # configs[3]: the NVFP4 feed-forward's token batches beyond M = 1


def is_global(i):
    return i % GLOBAL_EVERY == GLOBAL_EVERY - 1


def op_bytes(world=1):
    """Algorithmic bytes one GPU moves per op call at M=1 (weights + scales + activations read
    and written) when the model is split over `world` tensor-parallel ranks (1: the whole model)."""
    w, fr = world, L // world
    dk = -(-fr // 256) * 256  # a rank's down K slice, zero-padded to whole 256-element units
    rows = W // w

    def attention(ring):
        return 2 * ring * NS // w * DS * 2 + QS // w * 2 * 2 + ring * 4

    return {
        "embed_token": H * 2 * 2,
        "sliding_project_qkv": (QS + 2 * PS) // w * H + (QS + 2 * PS) // w * 2 + H * 2 * 2 + DS * 2 * 2
                               + 4 * DS * 2 + 2 * NS // w * DS * 2 + QS // w * 2,
        "sliding_attention": attention(RING_LOCAL),
        "sliding_attention_4096": attention(RING_GLOBAL),
        "sliding_attention_output": H * QS // w + H * 2 + QS // w * 2 + H * 2 * 3,
        "decoder_feedforward_fp8": 2 * fr * H + H * dk + (2 * fr + H) * 4 + H * 2 * 4,
        "decoder_feedforward": 2 * (fr * H // 2 + fr * H // 16) + (H * dk // 2 + H * dk // 16) + H * 2 * 4 + 8 * 2
                               + 12,
        "final_norm_and_logits": rows * H * 2 + H * 2 * 2 + rows * 2,
        # the NVFP4 feed-forward on M tokens: the same weights once, M residual rows in and out
        **{f"decoder_feedforward_m{mb}": 2 * (L * H // 2 + L * H // 16) + (H * L // 2 + H * L // 16)
           + mb * H * 2 * 2 + H * 2 * 2 + 8 * 2 + 12 for mb in BATCH_SWEEP},
        **{f"decoder_feedforward_fp8_m{mb}": 2 * L * H + H * L + (2 * L + H) * 4 + mb * H * 2 * 2 + H * 2 * 2 + 8 * 2
           for mb in BATCH_SWEEP},
        # the batched decoder's ops on nb sequences (one GPU): the weights once, the per-sequence rows
        # and caches nb times
        **{f"sliding_project_qkv_m{nb}": (QS + 2 * PS) * H + (QS + 2 * PS) * 2 + H * 2 + 2 * DS * 2
           + nb * (H * 2 + 2 * DS * 2 * 2 + 2 * PS * 2 + QS * 2 + 8) for nb in DECODE_BATCHES},
        **{f"sliding_attention_m{nb}": nb * attention(RING_LOCAL) for nb in DECODE_BATCHES},
        **{f"sliding_attention_4096_m{nb}": nb * attention(RING_GLOBAL) for nb in DECODE_BATCHES},
        **{f"sliding_attention_output_m{nb}": H * QS + H * 2 * 2 + nb * (QS * 2 + H * 2 * 2) for nb in DECODE_BATCHES},
        **{f"final_norm_and_logits_m{nb}": W * H * 2 + H * 2 + nb * (H * 2 + W * 2) for nb in DECODE_BATCHES},
    }


def step_bytes(world=1):
    """Algorithmic bytes of one decode step per GPU."""
    b = op_bytes(world)
    n_glob = sum(is_global(i) for i in range(N_MODEL))
    per_layer = b["sliding_project_qkv"] + b["sliding_attention_output"] + b["decoder_feedforward_fp8"]
    return (b["embed_token"] + N_MODEL * per_layer + (N_MODEL - n_glob) * b["sliding_attention"]
            + n_glob * b["sliding_attention_4096"] + b["final_norm_and_logits"])


METRIC = "decode tokens/s, Gemma-4-12B-shaped 48-layer model (BASELINE configs[4]), batch 1"
WORKLOAD = ("gemma4-12b-shaped decode, batch 1, context 4096: embed_token + 48 layers (40 sliding on 1024-slot "
            "rings, theta 1e4; 8 global-shaped on 4096-slot rings, theta 1e6; each fused QKV fp8 [8192x3840], "
            "attention 16 q / 8 kv heads x 256, O fp8 [3840x4096], FP8 GeGLU FFN [2x15360x3840 + 3840x15360] "
            "with f32 channel scales) + final norm and lm_head bf16 [262144x3840] with softcap 30")
# DRAM bytes read + written per decoder_feedforward_fp8 call (ffn8 up/gate + down kernels): ncu --set
# full capture of `python bench.py --only ffn8 --layers 4 --steps 3 --warmup 3` (dram__bytes_read.sum +
# dram__bytes_write.sum, profiles/ffn8_upgate_down_full.md)
FFN8_TRAFFIC = 118.17e6 + 3.26e6 + 59.18e6 + 0.07e6


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
    """One decoder layer's weights and ring cache, generated whole (the same on every rank), then
    cut to one tensor-parallel rank's slices (`shard`) and packed into the GPU-native layout
    (`tile`). ffn "fp8": FP8 e4m3 codes with f32 channel scales; "nvfp4": packed e2m1 codes, e4m3
    block scales and an f32 multiplier.

    keep_host=True also keeps a host copy of the whole layer's tensors in the reference layout
    (`self.host`, numpy: bf16 as uint16 bits, codes as uint8), for the parity check."""

    def __init__(self, gen, dev, ffn="fp8", ring=RING_LOCAL, keep_host=False):
        import torch

        def normal(*shape, std=1.0):
            return torch.randn(*shape, generator=gen, device=dev) * std

        def bf(t):
            return t.to(torch.bfloat16).contiguous()

        self.ffn, self.ring = ffn, ring
        self.input_rms = bf(1 + normal(H, std=0.1))
        (self.q_w, q_s), (self.k_w, k_s), (self.v_w, v_s) = (quant_fp8_rows(normal(r, H, std=0.02))
                                                             for r in (QS, PS, PS))
        self.q_s, self.k_s, self.v_s = bf(q_s), bf(k_s), bf(v_s)
        self.q_rms, self.k_rms = bf(1 + normal(DS, std=0.1)), bf(1 + normal(DS, std=0.1))
        self.k_cache = bf(normal(ring, NS, DS))
        self.v_cache = bf(normal(ring, NS, DS))
        self.post_attn_rms = bf(1 + normal(H, std=0.1))
        self.o_w, o_s = quant_fp8_rows(normal(H, QS, std=0.02))
        self.o_s = bf(o_s)
        self.pre_ff_rms = bf(1 + normal(H, std=0.1))
        self.post_ff_rms = bf(1 + normal(H, std=0.1))
        if ffn == "fp8":
            (self.up_w, up_s), (self.gate_w, gate_s), (self.down_w, down_s) = (
                quant_fp8_rows(normal(r, c, std=0.02)) for r, c in ((L, H), (L, H), (H, L)))
            self.up_s, self.gate_s, self.down_s = (t.float().contiguous() for t in (up_s, gate_s, down_s))
            self.up_g = self.gate_g = self.down_g = None
        else:
            (self.up_w, self.up_s, self.up_g), (self.gate_w, self.gate_s, self.gate_g), \
                (self.down_w, self.down_s, self.down_g) = (quant_nvfp4(normal(r, c, std=0.02))
                                                           for r, c in ((L, H), (L, H), (H, L)))
        self.layer_scalar = bf(torch.full((8,), 0.375, device=dev))
        self.tiled = False
        self.host = {k: host_array(getattr(self, k)) for k in self.HOST
                     if getattr(self, k) is not None} if keep_host else None

    HOST = ("input_rms", "q_w", "k_w", "v_w", "q_s", "k_s", "v_s", "q_rms", "k_rms", "post_attn_rms", "o_w", "o_s",
            "pre_ff_rms", "post_ff_rms", "up_w", "up_s", "up_g", "gate_w", "gate_s", "gate_g", "down_w", "down_s",
            "down_g", "layer_scalar")

    def _tp_names(self):
        """attribute -> the name g4b200.tp slices it by"""
        names = {"q_w": "q_weight", "k_w": "k_weight", "v_w": "v_weight", "q_s": "q_weight_scale",
                 "k_s": "k_weight_scale", "v_s": "v_weight_scale", "k_cache": "k_cache", "v_cache": "v_cache",
                 "o_w": "o_weight"}
        if self.ffn == "fp8":
            names.update(up_w="up_weight", gate_w="gate_weight", down_w="down_weight", up_s="up_channel_scale",
                         gate_s="gate_channel_scale")
        else:
            names.update(up_w="up_weight_packed", gate_w="gate_weight_packed", down_w="down_weight_packed",
                         up_s="up_weight_scale", gate_s="gate_weight_scale", down_s="down_weight_scale")
        return names

    def shard(self, rank, world):
        """Keep tensor-parallel rank `rank`'s slices of the sliced tensors."""
        from g4b200 import tp

        for attr, name in self._tp_names().items():
            setattr(self, attr, tp.shard(name, getattr(self, attr), rank, world))
        return self

    def tile(self, ops, device):
        """Repack the weight matrices into the GPU-native unit-tiled layout (once, at load)."""
        for attr, name in (("q_w", "q_weight"), ("k_w", "k_weight"), ("v_w", "v_weight"), ("o_w", "o_weight")):
            setattr(self, attr, ops.tile_weight(device, name, getattr(self, attr)))
        if self.ffn == "fp8":
            self.up_w = ops.pack_upgate_fp8(device, self.up_w, self.gate_w)
            self.down_w = ops.tile_weight(device, "down_weight", self.down_w)
        else:
            self.up_w = ops.pack_upgate(device, self.up_w, self.gate_w, scales=False)
            self.up_s = ops.pack_upgate(device, self.up_s, self.gate_s, scales=True)
            self.down_w = ops.tile_weight(device, "down_weight_packed", self.down_w)
            self.down_s = ops.tile_weight(device, "down_weight_scale", self.down_s)
            self.gate_s = None
        self.gate_w = None
        self.tiled = True
        return self

    def for_decoder(self, attn_scale):
        from g4b200 import decoder

        return decoder.Layer(
            input_rms_weight=self.input_rms, q_weight=self.q_w, k_weight=self.k_w, v_weight=self.v_w,
            q_weight_scale=self.q_s, k_weight_scale=self.k_s, v_weight_scale=self.v_s, q_rms_weight=self.q_rms,
            k_rms_weight=self.k_rms, k_cache=self.k_cache, v_cache=self.v_cache,
            post_attn_rms_weight=self.post_attn_rms, o_weight=self.o_w, o_weight_scale=self.o_s,
            pre_ff_rms_weight=self.pre_ff_rms, post_ff_rms_weight=self.post_ff_rms, layer_scalar=self.layer_scalar,
            up_weight=self.up_w, gate_weight=self.gate_w, down_weight=self.down_w, up_scale=self.up_s,
            gate_scale=self.gate_s, down_scale=self.down_s, up_global_scale=self.up_g, gate_global_scale=self.gate_g,
            down_global_scale=self.down_g, rope=decoder.ROPE_GLOBAL if self.ring == RING_GLOBAL else decoder.ROPE_LOCAL,
            ffn=decoder.FFN_FP8 if self.ffn == "fp8" else decoder.FFN_NVFP4, tiled=self.tiled, attn_scale=attn_scale)


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


def rope_tables_device(theta, dev):
    """cos / sin [E, Ds] bf16 for every position (the kernel's sin operand: low half negated), from
    the reference's f64 angles narrowed to f32 (FOG/scripts/generate_references.py:184-210)."""
    import numpy as np
    import torch

    pos = np.arange(E, dtype=np.float64)[:, None]
    inv = 1.0 / (np.float64(theta) ** (np.arange(0, DS, 2, dtype=np.float64) / DS))
    emb = np.concatenate([pos * inv, pos * inv], axis=1)
    cos = np.cos(emb).astype(np.float32)
    sin = np.sin(emb).astype(np.float32)
    sin[:, : DS // 2] *= -1.0
    return (torch.from_numpy(cos).to(dev).to(torch.bfloat16), torch.from_numpy(sin).to(dev).to(torch.bfloat16))


ATTN_SCALE = 1.0  # the reference model's attention scale (gemma4.py:179-181)


class Model:
    """The benchmark model on one GPU (one tensor-parallel rank's slices): 48 FP8 layers, the
    embedding / lm_head table (tied, as Gemma's; the lm_head is this rank's rows), the final norm,
    both RoPE tables, and NVFP4_COPIES extra NVFP4 layers for the configs[3] op timing."""

    def __init__(self, ops, device, dev, rank, world, keep_host=()):
        import torch

        gen = torch.Generator(device=dev)
        gen.manual_seed(1000)  # the same whole model on every rank; each keeps its slices
        self.layers = [Layer(gen, dev, "fp8", RING_GLOBAL if is_global(i) else RING_LOCAL,
                             keep_host=i in keep_host).shard(rank, world).tile(ops, device) for i in range(N_MODEL)]
        self.nvfp4 = [Layer(gen, dev, "nvfp4", RING_LOCAL, keep_host=(i == 0 and 0 in keep_host))
                      .shard(rank, world).tile(ops, device) for i in range(NVFP4_COPIES)]
        self.table = (torch.randn((W, H), generator=gen, device=dev) * 0.03).to(torch.bfloat16)
        self.final_norm = (1 + torch.randn(H, generator=gen, device=dev) * 0.1).to(torch.bfloat16)
        rows = W // world
        self.lm_head = self.table[rank * rows:(rank + 1) * rows]  # contiguous rows of the tied table
        self.cos_l, self.sin_l = rope_tables_device(1e4, dev)
        self.cos_g, self.sin_g = rope_tables_device(1e6, dev)
        self.world = world

    def decoder(self, ops_device):
        from g4b200 import decoder

        return decoder.Decoder(ops_device, [lay.for_decoder(ATTN_SCALE) for lay in self.layers],
                               cos_local=self.cos_l, sin_local=self.sin_l, cos_global=self.cos_g,
                               sin_global=self.sin_g, embedding_table=self.table, final_norm_weight=self.final_norm,
                               lm_head_weight=self.lm_head)

    def tables_of(self, lay):
        return (self.cos_g, self.sin_g) if lay.ring == RING_GLOBAL else (self.cos_l, self.sin_l)


def batched_decoder(m: "Model", ops_device, nb, dev):
    """The benchmark model's decoder over `nb` sequences (g4_decoder_create_batch): the same layers,
    every layer's caches holding nb seeded rings ([nb, ring, Ns, Ds])."""
    import dataclasses

    import torch
    from g4b200 import decoder

    gen = torch.Generator(device=dev)
    gen.manual_seed(2000 + nb)
    layers = []
    for lay in m.layers:
        shape = (nb, lay.ring, NS // m.world, DS)
        k = torch.randn(shape, generator=gen, device=dev).to(torch.bfloat16)
        v = torch.randn(shape, generator=gen, device=dev).to(torch.bfloat16)
        layers.append(dataclasses.replace(lay.for_decoder(ATTN_SCALE), k_cache=k, v_cache=v))
    return decoder.Decoder(ops_device, layers, cos_local=m.cos_l, sin_local=m.sin_l, cos_global=m.cos_g,
                           sin_global=m.sin_g, embedding_table=m.table, final_norm_weight=m.final_norm,
                           lm_head_weight=m.lm_head, batch=nb)


def time_decode_batch(torch, m: "Model", device, dev, nb, steps, warmup):
    """Decode tokens/s of `nb` sequences decoded together: exactly `warmup` then `steps` replays of
    the batched decoder's graph (each step: nb tokens through the 48 layers and the lm_head)."""
    dec = batched_decoder(m, device, nb, dev)
    stream = torch.cuda.Stream(dev)
    dec.set_input([1234 + 7 * i for i in range(nb)], [POSITION - i for i in range(nb)], stream=stream)
    dec.capture(stream=stream)
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            dec.step(stream=stream)
        torch.cuda.synchronize()
        secs = timed(torch, lambda: [dec.step(stream=stream) for _ in range(steps)])
    device.check()
    dec.close()
    del dec
    torch.cuda.empty_cache()
    return {"tokens_per_s": round(nb * steps / secs, 1), "ms_per_step": round(secs / steps * 1e3, 4),
            "steps": steps, "warmup": warmup}


class Buffers:
    """One token's per-op buffers for calling the ops one by one (the reference host's Decode)."""

    def __init__(self, dev, world, pos=POSITION, token=1234):
        import torch

        self.pos, self.token = pos, token
        self.x = torch.zeros(H, dtype=torch.bfloat16, device=dev)
        self.q = torch.zeros((NS // world, GS, DS), dtype=torch.bfloat16, device=dev)
        self.attn = torch.zeros_like(self.q)
        self.token_off = torch.tensor([token * H * 2], dtype=torch.int32, device=dev)
        self.rope_off = torch.tensor([pos * DS * 2], dtype=torch.int32, device=dev)
        self.kv_off = {r: torch.tensor([(pos % r) * NS * DS * 2], dtype=torch.int32, device=dev)
                       for r in (RING_LOCAL, RING_GLOBAL)}
        self.mask = {r: (torch.arange(r, device=dev) <= min(pos, r - 1)).to(torch.float32)
                     for r in (RING_LOCAL, RING_GLOBAL)}


def layer_ops(ops, device, m: Model, b: Buffers, lay: Layer, which=("qkv", "attn", "o", "ffn")):
    """One layer's ops through their entry points, on b.x (the decoder issues the same calls)."""
    if "qkv" in which:
        cos, sin = m.tables_of(lay)
        ops.sliding_project_qkv(device, b.x, lay.q_w, lay.k_w, lay.v_w, lay.q_s, lay.k_s, lay.v_s, lay.input_rms,
                                lay.q_rms, lay.k_rms, b.kv_off[lay.ring], b.rope_off, cos, sin, lay.k_cache,
                                lay.v_cache, b.q, tiled=lay.tiled)
    if "attn" in which:
        ops.sliding_attention(device, b.q, lay.k_cache, lay.v_cache, b.mask[lay.ring], b.attn, scale=ATTN_SCALE,
                              kv_offset=b.kv_off[lay.ring])
    if "o" in which:
        ops.sliding_attention_output(device, b.attn, lay.post_attn_rms, lay.o_w, lay.o_s, b.x, tiled=lay.tiled)
    if "ffn" in which:
        if lay.ffn == "fp8":
            ops.decoder_feedforward_fp8_tiled(device, b.x, lay.pre_ff_rms, lay.up_w, lay.down_w, lay.up_s, lay.gate_s,
                                              lay.down_s, lay.post_ff_rms, lay.layer_scalar)
        else:
            ops.decoder_feedforward_tiled(device, b.x, lay.pre_ff_rms, lay.up_w, lay.down_w, lay.up_s, lay.down_s,
                                          lay.up_g, lay.gate_g, lay.down_g, lay.post_ff_rms, lay.layer_scalar)


def ffn_batch(ops, device, lay: Layer, rows):
    """The feed-forward of `lay` (NVFP4 or FP8) on the token batch `rows` [M, H] (updated in place)."""
    if lay.ffn == "fp8":
        ops.decoder_feedforward_fp8_batch_tiled(device, rows, lay.pre_ff_rms, lay.up_w, lay.down_w, lay.up_s,
                                                lay.gate_s, lay.down_s, lay.post_ff_rms, lay.layer_scalar)
    else:
        ops.decoder_feedforward_batch_tiled(device, rows, lay.pre_ff_rms, lay.up_w, lay.down_w, lay.up_s, lay.down_s,
                                            lay.up_g, lay.gate_g, lay.down_g, lay.post_ff_rms, lay.layer_scalar)


def decode_one_by_one(ops, device, m: Model, b: Buffers, logits):
    ops.embed_token(device, m.table, b.token_off, b.x)
    for lay in m.layers:
        layer_ops(ops, device, m, b, lay)
    ops.final_norm_and_logits(device, b.x, m.final_norm, m.lm_head, logits)


# ------------------------------------------------------------------------------ parity gate

# the reference grader's tolerances (FOG/src/bin/test_kernels.rs:447-465): |want - got| <=
# atol + rtol |want|; attention and the logits (never graded by the reference) are held to 0.01
RTOL = 1e-2
ATOL = {"sliding_project_qkv": 0.04, "sliding_attention": 0.01, "sliding_attention_output": 0.05,
        "decoder_feedforward": 0.01, "decoder_feedforward_fp8": 0.01, "final_norm_and_logits": 0.01}


def compare(name, want, got):
    import numpy as np

    from oracle.ops import bf16_to_f32

    w, g = bf16_to_f32(np.asarray(want).reshape(-1)), bf16_to_f32(np.asarray(got).reshape(-1))
    diff = np.abs(w - g)
    ok = bool(np.isfinite(g).all() and (diff <= ATOL[name] + RTOL * np.abs(w)).all())
    return {"ok": ok, "max_abs": float(diff.max()), "atol": ATOL[name], "rtol": RTOL,
            "bit_exact": round(float(np.mean(np.asarray(want).reshape(-1) == np.asarray(got).reshape(-1))), 5)}


def gather(torch, dist, world, t):
    """Every rank's tensor, in rank order, on the host (numpy)."""
    t = t.contiguous()
    if world == 1:
        return [host_array(t)]
    parts = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(parts, t)
    return [host_array(p) for p in parts]


def parity_layer(torch, ops, device, m, b, lay, rank, world, dist, tag):
    """Each op of one layer on the GPU against the CPU oracle, each on the GPU's previous output
    (so a failure names the op). Under tensor parallelism the slices are gathered to rank 0 and
    the O / FFN oracles add the ranks' partial sums in rank order. Returns {op: result} on rank 0."""
    import numpy as np

    from g4b200 import tp

    slot = b.pos % lay.ring
    x0 = host_array(b.x)
    cos, sin = (host_array(t[b.pos]) for t in m.tables_of(lay))
    layer_ops(ops, device, m, b, lay, ("qkv",))
    device.check()
    q = np.concatenate(gather(torch, dist, world, b.q), axis=0)
    kc = np.concatenate(gather(torch, dist, world, lay.k_cache), axis=1)
    vc = np.concatenate(gather(torch, dist, world, lay.v_cache), axis=1)
    layer_ops(ops, device, m, b, lay, ("attn",))
    device.check()
    attn_parts = gather(torch, dist, world, b.attn)
    layer_ops(ops, device, m, b, lay, ("o",))
    device.check()
    x1 = gather(torch, dist, world, b.x)
    layer_ops(ops, device, m, b, lay, ("ffn",))
    device.check()
    x2 = gather(torch, dist, world, b.x)
    mask = host_array(b.mask[lay.ring])
    if rank != 0:
        return None

    from oracle import ops as oracle

    h = lay.host
    out = {}
    wq, wk, wv = oracle.sliding_project_qkv(x0, h["q_w"], h["k_w"], h["v_w"], h["q_s"], h["k_s"], h["v_s"],
                                            h["input_rms"], h["q_rms"], h["k_rms"], cos, sin)
    out["sliding_project_qkv"] = compare("sliding_project_qkv", np.concatenate(
        [wq.reshape(-1), wk.reshape(-1), wv.reshape(-1)]), np.concatenate(
        [q.reshape(-1), kc[slot].reshape(-1), vc[slot].reshape(-1)]))
    attn = np.concatenate(attn_parts, axis=0)
    out["sliding_attention"] = compare("sliding_attention", oracle.sliding_attention(q, kc, vc, mask, ATTN_SCALE),
                                       attn)

    def cut(name, arr, r):
        return tp.shard(name, torch.from_numpy(arr), r, world).numpy()

    if world == 1:
        want_o = oracle.sliding_attention_output(attn, h["post_attn_rms"], h["o_w"], h["o_s"], x0)
    else:
        want_o = oracle.sliding_attention_output_tp([a.reshape(-1) for a in attn_parts], h["post_attn_rms"],
                                                    [cut("o_weight", h["o_w"], r) for r in range(world)], h["o_s"], x0)
    out["sliding_attention_output"] = compare("sliding_attention_output", want_o, x1[0])
    if lay.ffn == "fp8":
        name = "decoder_feedforward_fp8"
        if world == 1:
            want_f = oracle.feedforward_fp8(x1[0], h["pre_ff_rms"], h["up_w"], h["gate_w"], h["down_w"], h["up_s"],
                                            h["gate_s"], h["down_s"], h["post_ff_rms"], h["layer_scalar"])
        else:
            want_f = oracle.feedforward_fp8_tp(
                x1[0], h["pre_ff_rms"],
                [(cut("up_weight", h["up_w"], r), cut("up_channel_scale", h["up_s"], r)) for r in range(world)],
                [(cut("gate_weight", h["gate_w"], r), cut("gate_channel_scale", h["gate_s"], r)) for r in range(world)],
                [cut("down_weight", h["down_w"], r) for r in range(world)], h["down_s"], h["post_ff_rms"],
                h["layer_scalar"])
    else:
        name = "decoder_feedforward"
        if world == 1:
            want_f = oracle.decoder_feedforward(x1[0], h["pre_ff_rms"], h["up_w"], h["gate_w"], h["down_w"], h["up_s"],
                                                h["gate_s"], h["down_s"], h["up_g"][0], h["gate_g"][0], h["down_g"][0],
                                                h["post_ff_rms"], h["layer_scalar"])
        else:
            want_f = oracle.decoder_feedforward_tp(
                x1[0], h["pre_ff_rms"],
                [(cut("up_weight_packed", h["up_w"], r), cut("up_weight_scale", h["up_s"], r)) for r in range(world)],
                [(cut("gate_weight_packed", h["gate_w"], r), cut("gate_weight_scale", h["gate_s"], r))
                 for r in range(world)],
                [(cut("down_weight_packed", h["down_w"], r), cut("down_weight_scale", h["down_s"], r))
                 for r in range(world)],
                h["up_g"][0], h["gate_g"][0], h["down_g"][0], h["post_ff_rms"], h["layer_scalar"])
    out[name] = compare(name, want_f, x2[0])
    same = all(np.array_equal(p, x1[0]) for p in x1) and all(np.array_equal(p, x2[0]) for p in x2)
    return {f"{tag}.{k}": v for k, v in out.items()}, same


def parity(torch, ops, device, dev, m: Model, rank, world, dist):
    """The gate before timing (see the module docstring). Returns the "parity" object on rank 0."""
    import numpy as np

    res = {}
    same = True
    # (1) the decoder's step against the ops one by one, bit for bit, on every rank
    b = Buffers(dev, world)
    logits_ops = torch.zeros(W // world, dtype=torch.bfloat16, device=dev)
    decode_one_by_one(ops, device, m, b, logits_ops)
    device.check()
    dec = m.decoder(device)
    dec.step(b.token, b.pos)
    device.check()
    step_equal = bool(torch.equal(dec.hidden().view(torch.int16), b.x.view(torch.int16)) and
                      torch.equal(dec.logits().view(torch.int16), logits_ops.view(torch.int16)))
    flags = torch.tensor([int(step_equal)], device=dev)
    hidden_parts = gather(torch, dist, world, dec.hidden())
    logit_rows = np.arange(0, W // world, 61)
    logits_parts = gather(torch, dist, world, dec.logits()[torch.from_numpy(logit_rows).to(dev)])
    if dist:
        dist.all_reduce(flags, op=dist.ReduceOp.MIN)
    x_final = host_array(dec.hidden())
    dec.close()
    same = same and all(np.array_equal(p, hidden_parts[0]) for p in hidden_parts)
    # (2) every op of the first sliding and the first global layer, and the NVFP4 feed-forward,
    # against the oracle; the embedding exactly; a sample of the logits
    for tag, lay in (("layer0", m.layers[0]), ("layer5_global", m.layers[5]), ("nvfp4", m.nvfp4[0])):
        ops.embed_token(device, m.table, b.token_off, b.x)
        r = parity_layer(torch, ops, device, m, b, lay, rank, world, dist, tag)
        if rank == 0:
            res.update(r[0])
            same = same and r[1]
    batch_rows = None
    if world == 1:  # the NVFP4 feed-forward on a batch of 8 tokens (configs[3]'s sweep)
        rows = (torch.randn(8, H, device=dev, generator=torch.Generator(device=dev).manual_seed(8))
                .to(torch.bfloat16))
        batch_in = host_array(rows)
        rows8 = rows.clone()
        ffn_batch(ops, device, m.nvfp4[0], rows)
        ffn_batch(ops, device, m.layers[0], rows8)  # FP8
        device.check()
        batch_rows, batch_rows8 = host_array(rows), host_array(rows8)
    if rank != 0:
        return None
    from oracle import ops as oracle

    if batch_rows is not None:
        h = m.nvfp4[0].host
        want_b = oracle.decoder_feedforward_batch(batch_in, h["pre_ff_rms"], h["up_w"], h["gate_w"], h["down_w"],
                                                  h["up_s"], h["gate_s"], h["down_s"], h["up_g"][0], h["gate_g"][0],
                                                  h["down_g"][0], h["post_ff_rms"], h["layer_scalar"])
        res["nvfp4.decoder_feedforward_batch_m8"] = compare("decoder_feedforward", want_b.reshape(-1),
                                                            batch_rows.reshape(-1))
        h = m.layers[0].host
        want_b8 = oracle.feedforward_fp8_batch(batch_in, h["pre_ff_rms"], h["up_w"], h["gate_w"], h["down_w"],
                                               h["up_s"], h["gate_s"], h["down_s"], h["post_ff_rms"],
                                               h["layer_scalar"])
        res["layer0.decoder_feedforward_fp8_batch_m8"] = compare("decoder_feedforward_fp8", want_b8.reshape(-1),
                                                                 batch_rows8.reshape(-1))
    table_rows = host_array(m.table[b.token])
    emb = host_array(dec_embed(torch, ops, device, m, b))
    res["embed_token"] = {"ok": bool(np.array_equal(emb, oracle.embed_token(table_rows[None, :], 0))),
                          "bit_exact": 1.0}
    rows = np.concatenate([r * (W // world) + logit_rows for r in range(world)])
    sample = host_array(m.table[torch.from_numpy(rows).to(dev)])
    res["final_norm_and_logits"] = compare("final_norm_and_logits",
                                           oracle.final_norm_and_logits(x_final, host_array(m.final_norm), sample),
                                           np.concatenate(logits_parts))
    ok = all(v["ok"] for v in res.values()) and bool(flags.item()) and same
    return {"ok": ok, "decoder_step_equals_ops_one_by_one": bool(flags.item()),
            "ranks_bit_identical": same if world > 1 else None, "ops": res,
            "checked": f"token {b.token} at position {b.pos}: the decoder step against the ops one by one (bit for "
                       "bit), then each op of layers 0 (sliding) and 5 (global-shaped) and of an NVFP4 layer against "
                       "oracle/ops.py (numpy) on the previous op's GPU output, the NVFP4 and FP8 feed-forwards on a batch "
                       "of 8 tokens row by row (one GPU), the embedding and every 61st logit" +
                       (", O/FFN as the rank-order sum of the ranks' partials" if world > 1 else "")}


def dec_embed(torch, ops, device, m, b):
    out = torch.zeros(H, dtype=torch.bfloat16, device=b.x.device)
    ops.embed_token(device, m.table, b.token_off, out)
    device.check()
    return out


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
    return {"workload": WORKLOAD, "model": "gemma4-12b-shaped (random init, FP8 weights)", "global_batch": 1,
            "seq_len": 4096, "layers": N_MODEL, "parallelism": f"tp{world}" if world > 1 else "single GPU",
            "l2": f"inputs larger than L2: {N_MODEL} distinct layers ({step_bytes(world) / 1e9:.2f} GB read per "
                  "step per GPU)",
            "launch": "one CUDA graph per token, captured by the library's decode driver, programmatic dependent "
                      "launch between kernels"}


# ------------------------------------------------------------------------------ CPU legs

def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


class CpuModel:
    """The oracle port (numpy, all BLAS threads) running the same decode step on the host: the
    embedding, 48 layers (fused QKV, attention over the layer's ring, O, the FP8 GeGLU FFN, with
    the reference's bf16 rounding points) and the final norm + lm_head with softcap.

    Memory bounds the port: one sliding and one global layer's weights (f32, pre-dequantised:
    the oracle contracts in f32 either way) serve all 48 layers, each layer with its own ring
    cache; the lm_head is kept as bf16 bits and widened to f32 chunk by chunk."""

    def __init__(self):
        import numpy as np

        from oracle import ops as oracle

        self.np, self.oracle = np, oracle
        rng = np.random.default_rng(1234)

        def bf(a):
            return oracle.f32_to_bf16(np.asarray(a, np.float32))

        t0 = time.time()
        self.w = [{"qkv": rng.standard_normal((QS + 2 * PS, H), dtype=np.float32) * 0.02,
                   "o": rng.standard_normal((H, QS), dtype=np.float32) * 0.02,
                   "up": rng.standard_normal((L, H), dtype=np.float32) * 0.02,
                   "gate": rng.standard_normal((L, H), dtype=np.float32) * 0.02,
                   "down": rng.standard_normal((H, L), dtype=np.float32) * 0.02} for _ in range(2)]
        self.caches = [(bf(rng.standard_normal((ring, NS, DS))), bf(rng.standard_normal((ring, NS, DS))))
                       for ring in (RING_GLOBAL if is_global(i) else RING_LOCAL for i in range(N_MODEL))]
        self.table = np.empty((W, H), np.uint16)
        for c in range(0, W, 16384):
            self.table[c:c + 16384] = bf(rng.standard_normal((16384, H), dtype=np.float32) * 0.03)
        self.gam = bf(1 + 0.1 * rng.standard_normal(H))
        self.gam_d = bf(1 + 0.1 * rng.standard_normal(DS))
        self.rope = {}
        for theta in (1e4, 1e6):
            c, s = oracle.rope_tables(DS, theta, 1.0, POSITION)
            self.rope[theta] = (bf(c), bf(s))
        self.scale_qkv = np.full(QS + 2 * PS, 1e-3, np.float32)
        self.scale_h = np.full(H, 1e-3, np.float32)
        self.scale_l = np.full(L, 1e-3, np.float32)
        self.setup_s = time.time() - t0
        self.step()  # warm caches and BLAS threads

    def step(self):
        np, oracle = self.np, self.oracle
        x = oracle.embed_token(self.table, 1234)
        for i in range(N_MODEL):
            w = self.w[int(is_global(i))]
            kc, vc = self.caches[i]
            ring = kc.shape[0]
            cos, sin = self.rope[1e6 if is_global(i) else 1e4]
            h = oracle.rms_norm(x, self.gam)
            proj = oracle.scaled_projection(h, w["qkv"], self.scale_qkv)
            q = oracle.rope(oracle.rms_norm(proj[:QS].reshape(16, DS), self.gam_d), cos, sin)
            k = oracle.rope(oracle.rms_norm(proj[QS:QS + PS].reshape(8, DS), self.gam_d), cos, sin)
            v = oracle.rms_norm(proj[QS + PS:].reshape(8, DS), None)
            kc[POSITION % ring], vc[POSITION % ring] = k, v
            mask = (np.arange(ring) <= min(POSITION, ring - 1)).astype(np.float32)
            attn = oracle.sliding_attention(q.reshape(8, 2, DS), kc, vc, mask, ATTN_SCALE)
            o = oracle.scaled_projection(attn.reshape(-1), w["o"], self.scale_h)
            x = oracle.add_bf16(x, oracle.rms_norm(o, self.gam))
            hh = oracle.rms_norm(x, self.gam)
            up = oracle.scaled_projection(hh, w["up"], self.scale_l)
            gate = oracle.scaled_projection(hh, w["gate"], self.scale_l)
            act = oracle.mul_bf16(oracle.gelu_tanh(gate), up)
            down = oracle.scaled_projection(act, w["down"], self.scale_h)
            summed = oracle.add_bf16(x, oracle.rms_norm(down, self.gam))
            x = oracle.mul_bf16(summed, np.full(H, 0x3EC0, np.uint16))
        hn = oracle.bf16_to_f32(oracle.rms_norm(x, self.gam))
        logits = np.empty(W, np.float32)
        for c in range(0, W, 16384):
            logits[c:c + 16384] = oracle.bf16_to_f32(self.table[c:c + 16384]) @ hn
        logits = oracle.bf16_round(logits)
        return oracle.f32_to_bf16(np.tanh(logits / np.float32(30.0)).astype(np.float32) * np.float32(30.0))

    def sample(self, budget_s: float, min_steps: int = 1):
        n, t0 = 0, time.time()
        while n < min_steps or time.time() - t0 < budget_s:
            self.step()
            n += 1
        elapsed = time.time() - t0
        return n / elapsed, (f"{n} decode steps (48 layers + lm_head) of the numpy oracle port over {elapsed:.1f} s on "
                             f"{host_threads()} host threads (f32 BLAS on pre-dequantised weights, one sliding and one "
                             f"global layer's weights reused by all 48 layers; {self.setup_s:.1f} s setup untimed)")


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

    Under torchrun only rank 0 runs it (the others exit at once). Each step is one decode step of
    the port; at most ~120 s of steps run (the rest of K would repeat identical work), and the
    line reports the median per-step rate."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    cores = use_all_host_threads()
    cpu = CpuModel()
    for _ in range(min(args.warmup, 2)):
        cpu.step()
    rates = []
    t0 = time.time()
    for _ in range(args.steps):
        s0 = time.time()
        cpu.step()
        rates.append(1.0 / (time.time() - s0))
        if time.time() - t0 > 120.0:
            break
    value = statistics.median(rates)
    sample = (f"{len(rates)} of {args.steps} requested decode steps of the numpy oracle port (median rate) on "
              f"{cores} host threads; f32 BLAS on pre-dequantised weights (one sliding and one global layer's "
              f"weights reused by all 48 layers), {cpu.setup_s:.1f} s setup untimed")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": len(rates), "warmup": min(args.warmup, 2), "ms_per_step": 1e3 / value, "higher_is_better": True,
        "scaling": "strong" if args.gpus > 1 else "weak", "vs_baseline": None,
        "dtype": "f32 (numpy oracle port, bf16 rounding points emulated)",
        "data": "synthetic", "config": dict(config_for(args.gpus), parallelism=f"host CPU, {cores} threads, one process"),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------------------ GPU leg

def batched_op_cases(torch, ops, device, dev, m: Model):
    """The batched decoder's ops alone on nb sequences (configs[4]'s batches), rotating over the
    model's layers and over enough copies of nb rings that the caches of one call are not in L2."""
    gen = torch.Generator(device=dev)
    gen.manual_seed(4)
    cases = {}
    for nb in DECODE_BATCHES:
        x = torch.randn((nb, H), generator=gen, device=dev).to(torch.bfloat16)
        q = torch.randn((nb, NS, GS, DS), generator=gen, device=dev).to(torch.bfloat16)
        attn = torch.zeros_like(q)
        pos = [POSITION - i for i in range(nb)]
        rope = torch.tensor([p * DS * 2 for p in pos], dtype=torch.int32, device=dev)
        kv = {r: torch.tensor([(p % r) * NS * DS * 2 for p in pos], dtype=torch.int32, device=dev)
              for r in (RING_LOCAL, RING_GLOBAL)}
        mask = {r: torch.stack([(torch.arange(r, device=dev) <= min(p, r - 1)).to(torch.float32) for p in pos])
                for r in (RING_LOCAL, RING_GLOBAL)}
        copies = 4 if nb < 16 else 2
        rings = {r: [tuple(torch.randn((nb, r, NS, DS), generator=gen, device=dev).to(torch.bfloat16)
                           for _ in range(2)) for _ in range(copies)] for r in (RING_LOCAL, RING_GLOBAL)}
        logits = torch.zeros((nb, W), dtype=torch.bfloat16, device=dev)

        def qkv(i, nb=nb, x=x, q=q, rope=rope, kv=kv, rings=rings, copies=copies):
            lay = m.layers[i % N_MODEL]
            cos, sin = m.tables_of(lay)
            k, v = rings[lay.ring][i % copies]
            ops.sliding_project_qkv_batch(device, x, lay.q_w, lay.k_w, lay.v_w, lay.q_s, lay.k_s, lay.v_s,
                                          lay.input_rms, lay.q_rms, lay.k_rms, kv[lay.ring], rope, cos, sin, k, v, q,
                                          tiled=True)

        def att(i, ring, q=q, attn=attn, kv=kv, mask=mask, rings=rings, copies=copies):
            k, v = rings[ring][i % copies]
            ops.sliding_attention_batch(device, q, k, v, mask[ring], attn, scale=ATTN_SCALE, kv_offset=kv[ring])

        def o(i, x=x, attn=attn):
            lay = m.layers[i % N_MODEL]
            ops.sliding_attention_output_batch(device, attn, lay.post_attn_rms, lay.o_w, lay.o_s, x, tiled=True)

        cases[f"sliding_project_qkv_m{nb}"] = qkv
        cases[f"sliding_attention_m{nb}"] = lambda i, att=att: att(i, RING_LOCAL)
        cases[f"sliding_attention_4096_m{nb}"] = lambda i, att=att: att(i, RING_GLOBAL)
        cases[f"sliding_attention_output_m{nb}"] = o
        cases[f"final_norm_and_logits_m{nb}"] = (
            lambda i, x=x, logits=logits: ops.final_norm_and_logits_batch(device, x, m.final_norm, m.lm_head, logits))
    return cases


def op_timings(torch, ops, device, dev, m: Model, dist, reps=64):
    """Device microseconds per call of each op alone: a graph of `reps` calls rotating over the
    layers the op runs on, replayed 5 times (max over ranks)."""
    b = Buffers(dev, m.world)
    logits = torch.zeros(W // m.world, dtype=torch.bfloat16, device=dev)
    sliding = [lay for lay in m.layers if lay.ring == RING_LOCAL]
    glob = [lay for lay in m.layers if lay.ring == RING_GLOBAL]
    cases = {
        "embed_token": lambda i: ops.embed_token(device, m.table, b.token_off, b.x),
        "sliding_project_qkv": lambda i: layer_ops(ops, device, m, b, m.layers[i % N_MODEL], ("qkv",)),
        "sliding_attention": lambda i: layer_ops(ops, device, m, b, sliding[i % len(sliding)], ("attn",)),
        "sliding_attention_4096": lambda i: layer_ops(ops, device, m, b, glob[i % len(glob)], ("attn",)),
        "sliding_attention_output": lambda i: layer_ops(ops, device, m, b, m.layers[i % N_MODEL], ("o",)),
        "decoder_feedforward_fp8": lambda i: layer_ops(ops, device, m, b, m.layers[i % N_MODEL], ("ffn",)),
        "decoder_feedforward": lambda i: layer_ops(ops, device, m, b, m.nvfp4[i % NVFP4_COPIES], ("ffn",)),
        "final_norm_and_logits": lambda i: ops.final_norm_and_logits(device, b.x, m.final_norm, m.lm_head, logits),
    }
    if m.world == 1:  # configs[3]'s token batches (one GPU)
        rows = (torch.randn(max(BATCH_SWEEP), H, device=dev, generator=torch.Generator(device=dev).manual_seed(3))
                .to(torch.bfloat16))
        for mb in BATCH_SWEEP:
            cases[f"decoder_feedforward_m{mb}"] = (
                lambda i, mb=mb: ffn_batch(ops, device, m.nvfp4[i % NVFP4_COPIES], rows[:mb]))
        for mb in BATCH_SWEEP:  # the decoder's FP8 FFN layers on a batch of tokens
            cases[f"decoder_feedforward_fp8_m{mb}"] = (
                lambda i, mb=mb: ffn_batch(ops, device, m.layers[i % N_MODEL], rows[:mb]))
        cases.update(batched_op_cases(torch, ops, device, dev, m))
    us = {}
    for name, fn in cases.items():
        n = 8 if name.startswith("final_norm_and_logits") else reps  # 2 GB per call: the logits stream from HBM
        if dist:
            dist.barrier()
        g = capture(torch, fn, n)
        g.replay()
        us[name] = max_over_ranks(torch, dist, dev, timed(torch, lambda: [g.replay() for _ in range(5)])) / (5 * n) * 1e6
        del g
    device.check()
    return us


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

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))

    from g4b200 import ops, tp

    device = ops.Device(local)
    device.set_overlap(True)
    if dist:
        tp.connect(device)  # this GPU is tensor-parallel rank `rank` of `world`
    dev = torch.device("cuda", local)
    keep = (0, 5) if rank == 0 and not args.no_parity else ()
    m = Model(ops, device, dev, rank, world, keep_host=keep)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()  # the ranks' kernels wait on each other (bounded): start them together

    # --- correctness gate before timing
    par = None if args.no_parity else parity(torch, ops, device, dev, m, rank, world, dist)
    if dist:
        dist.barrier()

    # --- decode tokens/s: exactly W then K steps, each one replay of the decoder's graph
    dec = m.decoder(device)
    stream = torch.cuda.Stream(dev)
    dec.set_input(1234, POSITION, stream=stream)
    dec.capture(stream=stream)
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            dec.step(stream=stream)
        torch.cuda.synchronize()
        sampler = ClockSampler(local)
        if dist:
            dist.barrier()
        with sampler:
            elapsed = max_over_ranks(torch, dist, dev, timed(torch, lambda: [dec.step(stream=stream)
                                                                             for _ in range(args.steps)]))
    device.check()
    value = args.steps / elapsed  # one token through the model per step, for the whole job

    # --- each op alone
    op_us = op_timings(torch, ops, device, dev, m, dist)

    # --- end to end from pinned host buffers: every step copies {token, position} in and the
    # logits out, around the decode step (a second decoder, issued inside one graph per step)
    e2e_dec = m.decoder(device)
    host_in = torch.tensor([1234, POSITION], dtype=torch.int32).pin_memory()
    host_out = torch.empty(W // world, dtype=torch.bfloat16).pin_memory()
    dev_in, dev_logits = e2e_dec.input_view(), e2e_dec.logits()

    def e2e_step(_):
        dev_in.copy_(host_in, non_blocking=True)
        e2e_dec.step()
        host_out.copy_(dev_logits, non_blocking=True)

    g = capture(torch, e2e_step, 1)
    for _ in range(args.warmup):
        g.replay()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    e2e_elapsed = max_over_ranks(torch, dist, dev, timed(torch, lambda: [g.replay() for _ in range(args.steps)]))
    device.check()
    e2e_value = args.steps / e2e_elapsed
    del g
    dec.close()
    e2e_dec.close()

    # --- configs[4]'s larger batches: sequences decoded together, each layer's weights read once
    # per step for all of them (one GPU)
    decode_batch = None
    if world == 1 and not args.no_batch:
        decode_batch = {str(nb): time_decode_batch(torch, m, device, dev, nb, args.steps, args.warmup)
                        for nb in DECODE_BATCHES}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        use_all_host_threads()
        rate, sample = CpuModel().sample(budget_s=15.0, min_steps=2)
        cpu = {"value": rate, "unit": "tokens/s", "cores": host_threads(), "kind": "port", "sample": sample}

    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0

    pk, pk_kind = peaks()
    rank_bytes = op_bytes(world)
    ffn_bytes = rank_bytes["decoder_feedforward_fp8"]
    achieved = ffn_bytes / (op_us["decoder_feedforward_fp8"] * 1e-6) / 1e9
    sb = step_bytes(world)
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
        "arithmetic": "tcgen05 kind::f8f6f4: fp8 e4m3 weights x the bf16 activation as exact e4m3 terms, f32 "
                      "accumulation in TMEM (NVFP4 feed-forward: kind::mxf4nvf4 with e4m3 block scales x exact e2m1 "
                      "digits); lm_head: bf16 GEMV with f32 accumulation on the CUDA cores",
        "data": "synthetic",
        "config": config_for(world),
        "parity": par,
        "step_bytes_per_gpu": sb,
        "step_gbs_per_gpu": round(sb * args.steps / elapsed / 1e9, 1),
        "step_frac_of_hbm": round(sb * args.steps / elapsed / 1e9 / pk["hbm_gbs"], 4),
        "ops_us": {k: round(v, 3) for k, v in op_us.items()},
        "ops_gbs": {k: round(rank_bytes[k] / (op_us[k] * 1e-6) / 1e9, 1) for k in op_us},
        "ops_frac": {k: round(rank_bytes[k] / (op_us[k] * 1e-6) / 1e9 / pk["hbm_gbs"], 4) for k in op_us},
        "roofline": {"bound": "hbm", "kernel": "decoder_feedforward_fp8 (ffn8 up/gate + down kernels, one GPU's slice)",
                     "achieved": round(achieved, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / pk["hbm_gbs"], 4), "peak_source": pk_kind,
                     "algorithmic_bytes_per_launch": ffn_bytes,
                     "traffic": args.traffic if world == 1 else None},
        "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": 8 * world,
                "d2h_bytes_per_step": W * 2, "steps": args.steps,
                "how": "one CUDA graph per step: pinned host->device copy of {token, position}, the decode step "
                       "(the library's C ABI), device->pinned host copy of this rank's logits"},
        "gpu_launches": args.steps * (2 + KERNELS_PER_LAYER * N_MODEL) * world,
        "clocks": sampler.summary(),
        "cpu_baseline": cpu,
        "decode_batch": decode_batch,
    }
    print(json.dumps(line), flush=True)
    return 0


def run_only(args):
    """Eager calls of one op (no graph, no CPU leg, no parity): the small case the ncu captures
    use. Builds the first `--layers` layers only, runs --warmup + --steps calls of the op
    rotating over them, and prints the mean device time per call. `--only decode` instead runs
    --warmup + --steps whole decode steps from the decoder's graph (the launch-list capture)."""
    import torch

    from g4b200 import ops

    device = ops.Device(0)
    dev = torch.device("cuda", 0)
    if args.only == "decode":  # the whole decode step, replayed from the decoder's graph
        m = Model(ops, device, dev, 0, 1)
        nb = args.decode_batch
        dec = m.decoder(device) if nb == 1 else batched_decoder(m, device, nb, dev)
        stream = torch.cuda.Stream(dev)
        if nb == 1:
            dec.set_input(1234, POSITION, stream=stream)
        else:
            dec.set_input([1234 + 7 * i for i in range(nb)], [POSITION - i for i in range(nb)], stream=stream)
        dec.capture(stream=stream)
        with torch.cuda.stream(stream):
            for _ in range(args.warmup):
                dec.step(stream=stream)
            device.check(stream)
            secs = timed(torch, lambda: [dec.step(stream=stream) for _ in range(args.steps)])
        device.check(stream)
        print(json.dumps({"only": "decode", "batch": nb, "steps": args.steps,
                          "ms_per_step": round(secs / args.steps * 1e3, 4)}), flush=True)
        dec.close()
        device.close()
        return 0
    gen = torch.Generator(device=dev)
    gen.manual_seed(1000)
    ffn = "nvfp4" if args.only in ("ffn4", "ffn4b") else "fp8"
    layers = [Layer(gen, dev, ffn, RING_LOCAL).tile(ops, device) for _ in range(args.layers)]

    class Mini:  # the parts of Model that layer_ops needs
        cos_l, sin_l = rope_tables_device(1e4, dev)

        @staticmethod
        def tables_of(lay):
            return Mini.cos_l, Mini.sin_l

    b = Buffers(dev, 1)
    if args.only == "attnb":  # the batched attention over --batch sequences' rings of --ring slots
        nb, ring = args.batch, args.ring
        q = torch.randn((nb, NS, GS, DS), device=dev, generator=gen).to(torch.bfloat16)
        out = torch.zeros_like(q)
        caches = [tuple(torch.randn((nb, ring, NS, DS), device=dev, generator=gen).to(torch.bfloat16)
                        for _ in range(2)) for _ in range(args.layers)]
        pos = [POSITION - i for i in range(nb)]
        kv = torch.tensor([(p % ring) * NS * DS * 2 for p in pos], dtype=torch.int32, device=dev)
        mask = torch.stack([(torch.arange(ring, device=dev) <= min(p, ring - 1)).to(torch.float32) for p in pos])

        def call(i):
            k, v = caches[i % len(caches)]
            ops.sliding_attention_batch(device, q, k, v, mask, out, scale=ATTN_SCALE, kv_offset=kv)
    elif args.only in ("ffn4b", "ffn8b"):  # the NVFP4 / FP8 feed-forward on a batch of --batch tokens
        rows = torch.randn(args.batch, H, device=dev, generator=gen).to(torch.bfloat16)

        def call(i):
            ffn_batch(ops, device, layers[i % len(layers)], rows)
    else:
        which = {"qkv": ("qkv",), "attn": ("attn",), "o": ("o",), "ffn8": ("ffn",), "ffn4": ("ffn",)}[args.only]

        def call(i):
            layer_ops(ops, device, Mini, b, layers[i % len(layers)], which)
    for i in range(args.warmup):
        call(i)
    device.check()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(args.steps):
        call(i)
    end.record()
    device.check()
    us = start.elapsed_time(end) * 1e3 / max(args.steps, 1)
    print(json.dumps({"only": args.only, "calls": args.steps, "us_per_call": round(us, 3)}), flush=True)
    device.close()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=16, help="--only ffn4b / ffn8b / attnb: tokens (sequences) per call")
    ap.add_argument("--ring", type=int, default=RING_LOCAL, help="--only attnb: slots per sequence's ring")
    ap.add_argument("--only", choices=["qkv", "attn", "o", "ffn8", "ffn4", "ffn4b", "ffn8b", "attnb", "decode"],
                    default=None,
                    help="profiling aid: eager calls of one op only (prints us/call, not the bench line)")
    ap.add_argument("--layers", type=int, default=4, help="--only: layer copies to rotate over")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--no-batch", action="store_true", help="skip the batched decode legs (configs[4] batch 8, 32)")
    ap.add_argument("--decode-batch", type=int, default=1, help="--only decode: sequences per step")
    ap.add_argument("--no-parity", action="store_true", help="skip the parity gate (profiling runs)")
    ap.add_argument("--traffic", type=float, default=FFN8_TRAFFIC,
                    help="ncu dram bytes (read + write) per decoder_feedforward_fp8 call")
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
