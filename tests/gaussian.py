"""Seeded Gaussian inputs with BASELINE.json's shapes and value distributions (test helper).

The reference's own parity inputs are uniform / banded PRNG values (oracle/synth.py). These are
the benchmark's distributions instead, so the parity tests also cover the data the bench runs:

- configs[0]  FP8 GeGLU FFN: x ~ N(0, 1) bf16, RMSNorm gammas ~ 1 + N(0, 0.1), up / gate / down
              weights N(0, 0.02) quantised per output row to e4m3 (scale = row amax / 448, f32)
- configs[1]  fused QKV: W_qkv N(0, 0.02) per row to e4m3 with bf16 row scales (the reference
              op's scale type), q / k gammas ~ 1 + N(0, 0.1), ring caches prefilled N(0, 1),
              position uniform in [0, 2048), RoPE theta 1e6 (global) or 1e4 (local)
- configs[2]  attention + O: q ~ N(0, 1), K / V ~ N(0, 1) over L slots, softmax scale 1/16;
              W_o N(0, 0.02) per row to e4m3 with bf16 row scales, residual ~ N(0, 1)
- configs[3]  NVFP4 FFN at M = 1: weights N(0, 0.02) to e2m1 codes in 16-element blocks with e4m3
              block scales (block amax / 6 / g) and the f32 multiplier g = amax / (6 * 448)

Values travel as the library takes them: bf16 as uint16 bits, e4m3 / packed e2m1 as uint8 codes.
The e4m3 rounding is torch's float8_e4m3fn cast (round to nearest even) on the host.
"""

from __future__ import annotations

import numpy as np

from oracle.ops import f32_to_bf16, negate_low_half, rope_tables

H, L, NS, GS, DS, QS, PS = 3840, 15360, 8, 2, 256, 4096, 2048
E2M1_BOUNDS = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], np.float32)


def rng(cfg: int, salt: int = 0) -> np.random.Generator:
    return np.random.default_rng(1000 + cfg + 100 * salt)


def bf16(a) -> np.ndarray:
    return f32_to_bf16(np.asarray(a, np.float32))


def e4m3(x) -> np.ndarray:
    import torch

    t = torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(torch.float8_e4m3fn)
    return t.view(torch.uint8).numpy().copy()


def fp8_rows(w: np.ndarray):
    """Per-output-row e4m3: (codes [rows, cols], f32 scale [rows]) with scale = row amax / 448."""
    amax = np.maximum(np.abs(w).max(axis=1, keepdims=True), 1e-12).astype(np.float32)
    scale = (amax / np.float32(448.0)).astype(np.float32)
    return e4m3(w / scale), scale[:, 0].copy()


def nvfp4(w: np.ndarray):
    """NVFP4: (packed codes [rows, cols / 2], e4m3 block scale codes [rows, cols / 16], f32 [1]
    global multiplier g = amax / (6 * 448)); a code's value is e2m1 x block scale x g."""
    rows, cols = w.shape
    g = np.float32(max(float(np.abs(w).max()) / (6.0 * 448.0), 1e-12))
    blocks = w.reshape(rows, cols // 16, 16)
    bscale = e4m3(np.abs(blocks).max(axis=2) / np.float32(6.0) / g)
    from oracle.ops import e4m3_to_f32

    denom = np.maximum(e4m3_to_f32(bscale) * g, np.float32(1e-30))[:, :, None]
    x = (blocks / denom).reshape(rows, cols)
    mag = np.searchsorted(E2M1_BOUNDS, np.abs(x), side="left").astype(np.uint8)
    codes = mag | ((x < 0).astype(np.uint8) << 3)
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8)
    return packed, bscale, np.array([g], np.float32)


def ffn_fp8(salt: int = 0) -> dict:
    """the FP8-per-channel FFN's inputs."""
    r = rng(0, salt)
    up, up_s = fp8_rows(r.standard_normal((L, H), dtype=np.float32) * np.float32(0.02))
    gate, gate_s = fp8_rows(r.standard_normal((L, H), dtype=np.float32) * np.float32(0.02))
    down, down_s = fp8_rows(r.standard_normal((H, L), dtype=np.float32) * np.float32(0.02))
    return {"residual": bf16(r.standard_normal(H)), "pre_ff_rms_weight": bf16(1 + 0.1 * r.standard_normal(H)),
            "up_weight": up, "gate_weight": gate, "down_weight": down, "up_weight_scale": up_s,
            "gate_weight_scale": gate_s, "down_weight_scale": down_s,
            "post_ff_rms_weight": bf16(1 + 0.1 * r.standard_normal(H)), "layer_scalar": bf16(np.full(8, 0.375))}


def ffn_nvfp4(salt: int = 0) -> dict:
    """configs[3] at M = 1: the NVFP4 FFN's inputs."""
    r = rng(3, salt)
    d = {"residual": bf16(r.standard_normal(H)), "pre_ff_rms_weight": bf16(1 + 0.1 * r.standard_normal(H))}
    for name, shape in (("up", (L, H)), ("gate", (L, H)), ("down", (H, L))):
        p, s, g = nvfp4(r.standard_normal(shape, dtype=np.float32) * np.float32(0.02))
        d[f"{name}_weight_packed"], d[f"{name}_weight_scale"], d[f"{name}_global_scale"] = p, s, g
    d["post_ff_rms_weight"] = bf16(1 + 0.1 * r.standard_normal(H))
    d["layer_scalar"] = bf16(np.full(8, 0.375))
    return d


def qkv(theta: float, ring: int = 2048, salt: int = 0) -> dict:
    """the fused QKV op's inputs at a position uniform in [0, 2048) (RoPE rows are
    the reference's tables at that position, the kernel's sin operand with its low half negated)."""
    r = rng(1, salt)
    pos = int(r.integers(0, 2048))
    d = {"pos": pos, "x": bf16(r.standard_normal(H)), "input_rms_weight": bf16(1 + 0.1 * r.standard_normal(H))}
    for name, rows in (("q", QS), ("k", PS), ("v", PS)):
        codes, scale = fp8_rows(r.standard_normal((rows, H), dtype=np.float32) * np.float32(0.02))
        d[f"{name}_weight"], d[f"{name}_weight_scale"] = codes, bf16(scale)
    d["q_rms_weight"] = bf16(1 + 0.1 * r.standard_normal(DS))
    d["k_rms_weight"] = bf16(1 + 0.1 * r.standard_normal(DS))
    c, s = rope_tables(DS, theta, 1.0, pos)
    d["cos_row"], d["sin_row"] = bf16(c), bf16(negate_low_half(s))
    d["kv_offset"] = np.array([(pos % ring) * NS * DS * 2], np.int32)
    d["rope_offset"] = np.array([pos * DS * 2], np.int32)
    d["k_cache"] = bf16(r.standard_normal((ring, NS, DS)))
    d["v_cache"] = bf16(r.standard_normal((ring, NS, DS)))
    return d


def attention(ring: int, salt: int = 0) -> dict:
    """a decode step's q and K / V caches of `ring` slots, every slot valid."""
    r = rng(2, salt)
    return {"q": bf16(r.standard_normal((NS, GS, DS))), "k": bf16(r.standard_normal((ring, NS, DS))),
            "v": bf16(r.standard_normal((ring, NS, DS))), "mask": np.ones(ring, np.float32), "scale": 1.0 / 16}


def attention_output(salt: int = 0) -> dict:
    """the O projection's inputs (x is an attention output, ~N(0, 1))."""
    r = rng(2, 50 + salt)
    codes, scale = fp8_rows(r.standard_normal((H, QS), dtype=np.float32) * np.float32(0.02))
    return {"x": bf16(r.standard_normal((NS, GS, DS))), "post_attn_rms_weight": bf16(1 + 0.1 * r.standard_normal(H)),
            "o_weight": codes, "o_weight_scale": bf16(scale), "residual": bf16(r.standard_normal(H))}
