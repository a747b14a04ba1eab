"""CPU restatement of the reference's decode-layer ops (TEST INFRASTRUCTURE, not product code).

Only `tests/`, `__graft_entry__.smoke()` and bench.py's CPU legs may import this module,
and only as the checker. The product path (the CUDA library) never calls it.

Every function restates the reference's PyTorch oracle with numpy, keeping each bf16
rounding point the oracle has (each torch op on bf16 tensors computes in f32 and rounds
its result to bf16 once). Values travel as raw bf16 bit patterns (`uint16`) so that the
rounding is explicit. Citations use `FOG` = `furiosa-opt-gemma4-12B/` of the reference:

- RMSNorm                     FOG/scripts/reference/gemma4.py:75-89
- scaled_projection           FOG/scripts/generate_references.py:265-274
- RoPE (rotate_half form)     FOG/scripts/generate_references.py:213-220, gemma4.py:120-122
- sliding_project_qkv         FOG/scripts/generate_references.py:291-334 (op: FOG/src/ops.rs:37-76)
- sliding_attention_output    FOG/scripts/generate_references.py:337-355 (op: FOG/src/ops.rs:130-146)
- decoder_feedforward         FOG/scripts/generate_references.py:358-414 (op: FOG/src/ops.rs:201-239)
- MLP / GeGLU (gelu tanh)     FOG/scripts/reference/gemma4.py:189-197
- sliding_attention           FOG/src/device/sliding/attention.rs:7-199 (op: FOG/src/ops.rs:118-128);
                              the reference's tests never pin this op, so its restatement follows
                              the device semantics and is validated against a float64 softmax.
- embed_token                 FOG/src/ops.rs:8-35 (device semantics: f32 scale, one bf16 cast)
- final_norm_and_logits       FOG/src/ops.rs:241-298, FOG/src/device/shared/lm_head.rs:13-80
- full_project_qkv            FOG/src/ops.rs:78-116 (global layers: 16 x 512 q heads, one K = V head)
- full_attention_page         FOG/src/ops.rs:148-182, FOG/src/device/full/attention.rs:205-339
- full_attention_output       FOG/src/ops.rs:184-199
- feedforward_fp8             FP8-per-channel FFN: scaled_projection
                              (generate_references.py:265-274) in the decoder_feedforward epilogue
- *_tp                        tensor-parallel split of O and the FFNs (no reference counterpart)

Dot products accumulate in f32 (numpy sgemv); the reference's torch CPU kernels also
accumulate in f32 but in their own order, so results agree to within the reference
harness tolerances (FOG/src/bin/test_kernels.rs:447-465), not bit for bit.
"""

from __future__ import annotations

import numpy as np

EPS = np.float32(1e-6)
F4_MAGNITUDES = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float32)


# --- bf16 / f8 / f4 value helpers -------------------------------------------------------

def bf16_to_f32(bits) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def f32_to_bf16(values) -> np.ndarray:
    """Round-half-to-even to bf16 bits; NaN stays NaN (quiet), inf stays inf."""
    v = np.ascontiguousarray(values, dtype=np.float32)
    bits = v.view(np.uint32)
    rounding = np.uint32(0x7FFF) + ((bits >> np.uint32(16)) & np.uint32(1))
    out = ((bits + rounding) >> np.uint32(16)).astype(np.uint16)
    nan = np.isnan(v)
    if nan.any():
        out[nan] = ((bits[nan] >> np.uint32(16)) | np.uint32(0x40)).astype(np.uint16)
    return out


def bf16_round(values) -> np.ndarray:
    """f32 -> nearest bf16 value, returned as f32."""
    return bf16_to_f32(f32_to_bf16(values))


def e4m3_to_f32(codes) -> np.ndarray:
    """Decode float8_e4m3fn codes exactly (bias 7, subnormals, 0x7F/0xFF = NaN)."""
    c = np.asarray(codes, dtype=np.uint8)
    sign = np.where(c & 0x80, -1.0, 1.0).astype(np.float32)
    e = ((c >> 3) & 0xF).astype(np.int32)
    m = (c & 0x7).astype(np.float32)
    normal = np.ldexp(1.0 + m / 8.0, e - 7).astype(np.float32)
    sub = np.ldexp(m / 8.0, -6).astype(np.float32)
    out = sign * np.where(e == 0, sub, normal)
    out = np.where((c & 0x7F) == 0x7F, np.float32(np.nan), out)
    return out.astype(np.float32)


def f4_unpack(packed, rows: int, cols: int) -> np.ndarray:
    """Packed e2m1 (low nibble = even element) -> f32 values [rows, cols]."""
    p = np.asarray(packed, dtype=np.uint8).reshape(rows, cols // 2)
    codes = np.empty((rows, cols), dtype=np.uint8)
    codes[:, 0::2] = p & 0x0F
    codes[:, 1::2] = p >> 4
    mag = F4_MAGNITUDES[codes & 0x7]
    return np.where(codes & 0x8, -mag, mag).astype(np.float32)


def nvfp4_dequant(packed, block_scale_codes, rows: int, cols: int) -> np.ndarray:
    """codes * e4m3 local scale repeated over 16 elements (generate_references.py:396-398).

    Every product is exact in f32 and in bf16 (2-bit x 4-bit significands), so the
    reference's `.to(torch.bfloat16)` of the folded weight (generate_references.py:407)
    changes nothing.
    """
    values = f4_unpack(packed, rows, cols)
    scale = e4m3_to_f32(block_scale_codes).reshape(rows, cols // 16)
    return values * np.repeat(scale, 16, axis=1)


# --- building blocks -------------------------------------------------------------------

def rms_norm(x_bits, weight_bits=None, eps=EPS) -> np.ndarray:
    """gemma4.RMSNorm on bf16 input over the last axis (gemma4.py:83-89).

    x.float(); x * rsqrt(mean(x^2) + eps); optionally * weight.float(); to bf16.
    """
    x = bf16_to_f32(x_bits)
    ms = np.mean(x.astype(np.float64) ** 2, axis=-1, keepdims=True).astype(np.float32)
    inv = (np.float32(1.0) / np.sqrt(ms + np.float32(eps))).astype(np.float32)
    y = (x * inv).astype(np.float32)
    if weight_bits is not None:
        y = (y * bf16_to_f32(weight_bits)).astype(np.float32)
    return f32_to_bf16(y)


def scaled_projection(x_bits, weight_f32, scale_f32) -> np.ndarray:
    """bf16((x.float() @ codes.T) * scale) with an f32 contraction (generate_references.py:265-274)."""
    x = bf16_to_f32(x_bits)
    acc = (weight_f32 @ x).astype(np.float32)
    return f32_to_bf16(acc * np.asarray(scale_f32, dtype=np.float32))


def linear_bf16(x_bits, weight_f32) -> np.ndarray:
    """bf16 nn.Linear (no bias): f32 contraction of bf16 operands, one rounding to bf16."""
    x = bf16_to_f32(x_bits)
    return f32_to_bf16((weight_f32 @ x).astype(np.float32))


def gelu_tanh(x_bits) -> np.ndarray:
    """F.gelu(approximate='tanh') on bf16: f32 math, bf16 result (gemma4.py:197)."""
    x = bf16_to_f32(x_bits)
    k = np.float32(0.7978845608028654)  # sqrt(2/pi)
    cube = (x * x * x).astype(np.float32)
    inner = k * (x + np.float32(0.044715) * cube)
    y = np.float32(0.5) * x * (np.float32(1.0) + np.tanh(inner.astype(np.float32)))
    return f32_to_bf16(y.astype(np.float32))


def mul_bf16(a_bits, b_bits) -> np.ndarray:
    return f32_to_bf16(bf16_to_f32(a_bits) * bf16_to_f32(b_bits))


def add_bf16(a_bits, b_bits) -> np.ndarray:
    return f32_to_bf16(bf16_to_f32(a_bits) + bf16_to_f32(b_bits))


def rope(x_bits, cos_bits, sin_bits) -> np.ndarray:
    """(x*cos) + (rotate_half(x)*sin), each product and the sum rounded to bf16.

    `sin_bits` is the UNMODIFIED sin row; generate_references.py:213-220 with
    gemma4.rotate_half (gemma4.py:120-122).
    """
    x = bf16_to_f32(x_bits)
    half = x.shape[-1] // 2
    rot = np.concatenate([-x[..., half:], x[..., :half]], axis=-1)
    a = bf16_round(x * bf16_to_f32(cos_bits))
    b = bf16_round(rot * bf16_to_f32(sin_bits))
    return f32_to_bf16(a + b)


def rope_tables(head_dim: int, theta: float, partial_rotary_factor: float, pos: int):
    """cos/sin rows in f64, narrowed to f32 (generate_references.py:184-197)."""
    angles = int(partial_rotary_factor * head_dim // 2)
    inv_freq = 1.0 / (np.float64(theta) ** (np.arange(0, 2 * angles, 2, dtype=np.float64) / head_dim))
    inv_freq = np.concatenate([inv_freq, np.zeros(head_dim // 2 - angles, dtype=np.float64)])
    emb = np.concatenate([pos * inv_freq, pos * inv_freq])
    return np.cos(emb).astype(np.float32), np.sin(emb).astype(np.float32)


def negate_low_half(sin: np.ndarray) -> np.ndarray:
    """The kernel-side sin operand: low half pre-negated (generate_references.py:200-210)."""
    out = np.array(sin, dtype=np.float32, copy=True)
    out[: len(out) // 2] *= -1.0
    return out


# --- the ops -----------------------------------------------------------------------------

def sliding_project_qkv(x, q_weight, k_weight, v_weight, q_scale, k_scale, v_scale,
                        input_rms_weight, q_rms_weight, k_rms_weight, cos_row, sin_row_kernel,
                        n_kv=8, group=2, head_dim=256):
    """Fused QKV op (generate_references.py:321-334).

    Weights are e4m3 code arrays [rows, H]; scales/gammas are bf16 bits; `cos_row` and
    `sin_row_kernel` are the bf16 rows at the position, `sin_row_kernel` with its low half
    pre-negated exactly as the kernel receives it. Returns (q [n_kv, group, D], k [n_kv, D],
    v [n_kv, D]) as bf16 bits.
    """
    h = rms_norm(x, input_rms_weight)
    sin_true = np.array(sin_row_kernel, dtype=np.uint16, copy=True)
    sin_true[: head_dim // 2] ^= np.uint16(0x8000)
    q = scaled_projection(h, e4m3_to_f32(q_weight), bf16_to_f32(q_scale)).reshape(n_kv * group, head_dim)
    q = rope(rms_norm(q, q_rms_weight), cos_row, sin_true)
    k = scaled_projection(h, e4m3_to_f32(k_weight), bf16_to_f32(k_scale)).reshape(n_kv, head_dim)
    k = rope(rms_norm(k, k_rms_weight), cos_row, sin_true)
    v = scaled_projection(h, e4m3_to_f32(v_weight), bf16_to_f32(v_scale)).reshape(n_kv, head_dim)
    v = rms_norm(v, None)
    return q.reshape(n_kv, group, head_dim), k, v


def sliding_attention_output(x, post_rms_weight, o_weight, o_scale, residual):
    """O projection -> post-attention RMSNorm -> residual add (generate_references.py:353-355)."""
    projected = scaled_projection(np.asarray(x).reshape(-1), e4m3_to_f32(o_weight), bf16_to_f32(o_scale))
    normalized = rms_norm(projected, post_rms_weight)
    return add_bf16(residual, normalized)


def feedforward_dense(residual, pre_rms_weight, post_rms_weight, w_up, w_gate, w_down,
                      g_up, g_gate, g_down, layer_scalar_bits):
    """decoder_feedforward on already-dequantised f32 weights (generate_references.py:404-413).

    `g_*` are the f32 reciprocal global scales (1.0 for a per-channel FP8 variant whose
    channel scale has been folded in by `feedforward_fp8`). Returns the new residual bits.
    """
    h = rms_norm(residual, pre_rms_weight)
    up = f32_to_bf16(bf16_to_f32(linear_bf16(h, w_up)) * np.float32(g_up))
    gate = f32_to_bf16(bf16_to_f32(linear_bf16(h, w_gate)) * np.float32(g_gate))
    act = mul_bf16(gelu_tanh(gate), up)
    down = f32_to_bf16(bf16_to_f32(linear_bf16(act, w_down)) * np.float32(g_down))
    normalized = rms_norm(down, post_rms_weight)
    summed = add_bf16(residual, normalized)
    return mul_bf16(summed, np.full(summed.shape, np.asarray(layer_scalar_bits).reshape(-1)[0], dtype=np.uint16))


def decoder_feedforward(residual, pre_rms_weight, up_packed, gate_packed, down_packed,
                        up_scale, gate_scale, down_scale, up_global, gate_global, down_global,
                        post_rms_weight, layer_scalar, hidden=3840, inter=15360):
    """NVFP4 GeGLU FFN with the reference epilogue (FOG/src/ops.rs:201-239)."""
    w_up = nvfp4_dequant(up_packed, up_scale, inter, hidden)
    w_gate = nvfp4_dequant(gate_packed, gate_scale, inter, hidden)
    w_down = nvfp4_dequant(down_packed, down_scale, hidden, inter)
    return feedforward_dense(residual, pre_rms_weight, post_rms_weight, w_up, w_gate, w_down,
                             np.float32(up_global), np.float32(gate_global), np.float32(down_global),
                             layer_scalar)


def decoder_feedforward_batch(residual, pre_rms_weight, up_packed, gate_packed, down_packed,
                              up_scale, gate_scale, down_scale, up_global, gate_global, down_global,
                              post_rms_weight, layer_scalar, hidden=3840, inter=15360):
    """decoder_feedforward (FOG/src/ops.rs:201-239) on each row of residual [M, H], row by row
    (the reference op is per token; the weights are dequantised once)."""
    w_up = nvfp4_dequant(up_packed, up_scale, inter, hidden)
    w_gate = nvfp4_dequant(gate_packed, gate_scale, inter, hidden)
    w_down = nvfp4_dequant(down_packed, down_scale, hidden, inter)
    rows = [feedforward_dense(r, pre_rms_weight, post_rms_weight, w_up, w_gate, w_down,
                              np.float32(up_global), np.float32(gate_global), np.float32(down_global),
                              layer_scalar)
            for r in np.asarray(residual).reshape(-1, hidden)]
    return np.stack(rows)


def feedforward_fp8(residual, pre_rms_weight, up_w, gate_w, down_w, up_s, gate_s, down_s,
                    post_rms_weight, layer_scalar, hidden=3840, inter=15360):
    """FP8-per-channel FFN variant (no counterpart op in the reference).

    Each projection is the reference's `scaled_projection` (generate_references.py:265-274):
    bf16((x @ codes.T) * channel_scale) with an f32 per-output-channel scale, wrapped in the
    same pre-RMS / GeGLU / post-RMS / residual / layer-scalar epilogue as
    `decoder_feedforward`.
    """
    h = rms_norm(residual, pre_rms_weight)
    up = scaled_projection(h, e4m3_to_f32(up_w).reshape(inter, hidden), up_s)
    gate = scaled_projection(h, e4m3_to_f32(gate_w).reshape(inter, hidden), gate_s)
    act = mul_bf16(gelu_tanh(gate), up)
    down = scaled_projection(act, e4m3_to_f32(down_w).reshape(hidden, inter), down_s)
    normalized = rms_norm(down, post_rms_weight)
    summed = add_bf16(residual, normalized)
    return mul_bf16(summed, np.full(summed.shape, np.asarray(layer_scalar).reshape(-1)[0], dtype=np.uint16))


def feedforward_fp8_batch(residual, pre_rms_weight, up_w, gate_w, down_w, up_s, gate_s, down_s,
                          post_rms_weight, layer_scalar, hidden=3840, inter=15360):
    """feedforward_fp8 on each row of residual [M, H], row by row (the weights decoded once)."""
    w_up = e4m3_to_f32(up_w).reshape(inter, hidden)
    w_gate = e4m3_to_f32(gate_w).reshape(inter, hidden)
    w_down = e4m3_to_f32(down_w).reshape(hidden, inter)
    out = []
    for r in np.asarray(residual).reshape(-1, hidden):
        h = rms_norm(r, pre_rms_weight)
        up = scaled_projection(h, w_up, up_s)
        gate = scaled_projection(h, w_gate, gate_s)
        act = mul_bf16(gelu_tanh(gate), up)
        down = scaled_projection(act, w_down, down_s)
        summed = add_bf16(r, rms_norm(down, post_rms_weight))
        out.append(mul_bf16(summed, np.full(summed.shape, np.asarray(layer_scalar).reshape(-1)[0], dtype=np.uint16)))
    return np.stack(out)


# --- tensor parallelism (no reference counterpart: the reference runs a layer on one chip) ---
# The O and down contractions are split over `world` K slices; each rank's f32 partial sums
# are added in rank order and the one-chip epilogue follows. The other ops are per head or per
# row and split without changing any result.

def sliding_attention_output_tp(x_parts, post_rms_weight, o_weight_parts, o_scale, residual):
    """sliding_attention_output with the K = 4096 contraction split over ranks: x_parts[r] is
    rank r's attention output (bf16 bits), o_weight_parts[r] its e4m3 columns [3840, 4096/w]."""
    acc = None
    for x_r, w_r in zip(x_parts, o_weight_parts):
        part = (e4m3_to_f32(w_r) @ bf16_to_f32(np.asarray(x_r).reshape(-1))).astype(np.float32)
        acc = part if acc is None else (acc + part).astype(np.float32)
    projected = f32_to_bf16(acc * bf16_to_f32(o_scale))
    return add_bf16(residual, rms_norm(projected, post_rms_weight))


def decoder_feedforward_tp(residual, pre_rms_weight, up_parts, gate_parts, down_parts, up_global, gate_global,
                           down_global, post_rms_weight, layer_scalar, hidden=3840):
    """decoder_feedforward with the FFN rows split over ranks. up_parts[r] / gate_parts[r] are
    (packed [rows_r, H/2], block scales [rows_r, H/16]) and down_parts[r] (packed [H, k_r/2],
    block scales [H, k_r/16]) with k_r >= rows_r (columns past rows_r are zero padding)."""
    h = rms_norm(residual, pre_rms_weight)
    acc = None
    for (up_p, up_s), (gate_p, gate_s), (down_p, down_s) in zip(up_parts, gate_parts, down_parts):
        rows = up_p.shape[0]
        w_up = nvfp4_dequant(up_p, up_s, rows, hidden)
        w_gate = nvfp4_dequant(gate_p, gate_s, rows, hidden)
        up = f32_to_bf16(bf16_to_f32(linear_bf16(h, w_up)) * np.float32(up_global))
        gate = f32_to_bf16(bf16_to_f32(linear_bf16(h, w_gate)) * np.float32(gate_global))
        act = bf16_to_f32(mul_bf16(gelu_tanh(gate), up))
        k = down_p.shape[1] * 2
        w_down = nvfp4_dequant(down_p, down_s, hidden, k)
        act_pad = np.zeros(k, np.float32)
        act_pad[:rows] = act
        part = (w_down @ act_pad).astype(np.float32)
        acc = part if acc is None else (acc + part).astype(np.float32)
    down = f32_to_bf16(bf16_to_f32(f32_to_bf16(acc)) * np.float32(down_global))
    summed = add_bf16(residual, rms_norm(down, post_rms_weight))
    return mul_bf16(summed, np.full(summed.shape, np.asarray(layer_scalar).reshape(-1)[0], dtype=np.uint16))


def feedforward_fp8_tp(residual, pre_rms_weight, up_parts, gate_parts, down_parts, down_s, post_rms_weight,
                       layer_scalar, hidden=3840):
    """feedforward_fp8 with the FFN rows split over ranks. up_parts[r] / gate_parts[r] are
    (e4m3 codes [rows_r, H], f32 channel scales [rows_r]) and down_parts[r] the e4m3 codes
    [H, k_r], k_r >= rows_r (columns past rows_r are zero padding); down_s is the whole [H]
    channel scale. The ranks' f32 partial sums of the down contraction are added in rank order
    before the channel scale."""
    h = rms_norm(residual, pre_rms_weight)
    acc = None
    for (up_w, up_s), (gate_w, gate_s), down_w in zip(up_parts, gate_parts, down_parts):
        rows = up_w.shape[0]
        up = scaled_projection(h, e4m3_to_f32(up_w).reshape(rows, hidden), up_s)
        gate = scaled_projection(h, e4m3_to_f32(gate_w).reshape(rows, hidden), gate_s)
        act = bf16_to_f32(mul_bf16(gelu_tanh(gate), up))
        k = down_w.shape[1]
        act_pad = np.zeros(k, np.float32)
        act_pad[:rows] = act
        part = (e4m3_to_f32(down_w).reshape(hidden, k) @ act_pad).astype(np.float32)
        acc = part if acc is None else (acc + part).astype(np.float32)
    down = f32_to_bf16(acc * np.asarray(down_s, dtype=np.float32))
    summed = add_bf16(residual, rms_norm(down, post_rms_weight))
    return mul_bf16(summed, np.full(summed.shape, np.asarray(layer_scalar).reshape(-1)[0], dtype=np.uint16))


EMBED_SCALE = np.float32(61.967734)   # FOG/src/lib.rs:23 (sqrt(3840) as the device op's f32 constant)
LOGIT_SOFTCAP = np.float32(30.0)      # FOG/src/lib.rs:24


def embed_token(table_bits, token):
    """ops::embed_token (FOG/src/ops.rs:8-35): the row times EMBED_SCALE in f32, one bf16 cast.

    (The model oracle, gemma4.py:92-100, multiplies by the scale cast to bf16 (62.0) instead; the
    device op, which this library replaces, keeps the f32 constant.)"""
    row = bf16_to_f32(np.asarray(table_bits)[token])
    return f32_to_bf16((row * EMBED_SCALE).astype(np.float32))


def final_norm_and_logits(x_bits, rms_weight_bits, lm_head_bits):
    """ops::final_norm_and_logits (FOG/src/ops.rs:241-298): h = RMSNorm(x) in bf16, logits =
    bf16(h @ W.T) with an f32 contraction (shared/lm_head.rs:13-80), then the device op's f32
    softcap: bf16(tanh(logit / 30) * 30) with one rounding (the model oracle, gemma4.py:258-261,
    rounds to bf16 after each of the three steps instead)."""
    h = bf16_to_f32(rms_norm(x_bits, rms_weight_bits))
    w = bf16_to_f32(lm_head_bits)
    logits = bf16_round((w @ h).astype(np.float32))
    capped = (np.tanh((logits / LOGIT_SOFTCAP).astype(np.float32)).astype(np.float32) * LOGIT_SOFTCAP)
    return f32_to_bf16(capped.astype(np.float32))


# --- global (full-attention) layers: 16 query heads x 512, one KV head of 512 with K = V ---------

def full_project_qkv(x, q_weight, k_weight, q_scale, k_scale, input_rms_weight, q_rms_weight, k_rms_weight,
                     cos_row, sin_row_kernel, n_q=16, head_dim=512):
    """ops::full_project_qkv (FOG/src/ops.rs:78-116): pre-RMSNorm, the q [16 x 512] and the single
    k [512] projections (scaled_projection), per-head RMSNorm of q (gamma q_rms) and of k (gamma
    k_rms); v is the same raw k projection normalised without a gamma (K = V,
    FOG/src/device/full/rmsnorm.rs:182-200); RoPE on q and k with the global table (partial
    rotation: the table's non-rotated frequencies are cos 1 / sin 0). Rounding points as the
    sliding op's (each product and the sum of the rotation rounded to bf16). `sin_row_kernel` has
    its low half negated. Returns (q [16, 512], k [512], v [512]) bf16 bits."""
    h = rms_norm(x, input_rms_weight)
    sin_true = np.array(sin_row_kernel, dtype=np.uint16, copy=True)
    sin_true[: head_dim // 2] ^= np.uint16(0x8000)
    q = scaled_projection(h, e4m3_to_f32(q_weight), bf16_to_f32(q_scale)).reshape(n_q, head_dim)
    q = rope(rms_norm(q, q_rms_weight), cos_row, sin_true)
    k_raw = scaled_projection(h, e4m3_to_f32(k_weight), bf16_to_f32(k_scale)).reshape(head_dim)
    k = rope(rms_norm(k_raw, k_rms_weight), cos_row, sin_true)
    v = rms_norm(k_raw, None)
    return q, k, v


FULL_GROUP = 32  # page rows contracted per bf16 partial (FOG/src/device/full/attention.rs:145-203)


def full_attention_page(q, k_page, v_page, mask, running_max=None, running_sum=None, out=None):
    """ops::full_attention_first_page / full_attention_page (FOG/src/ops.rs:148-182,
    FOG/src/device/full/attention.rs:205-339) on one 512-slot page: s = bf16(q . k) in f32;
    m = max over the page's slots (masked ones included), on later pages max(m, running max);
    e = min(exp(s - m), mask); the page's sum = sum(e) + 1e-6; the page's values: for each group of
    32 rows, bf16(sum_t bf16(e_t) v_t), then the groups added in f32 and rounded to bf16. The first
    page stores them; a later page rescales by r = exp(old max - new max): sum = old sum * r +
    page sum, out = bf16(bf16(old out * r) + page values). Returns (running_max [16] f32,
    running_sum [16] f32, out [16, 512] bf16 bits)."""
    qf, kf, vf = bf16_to_f32(q), bf16_to_f32(k_page), bf16_to_f32(v_page)
    mk = np.asarray(mask, dtype=np.float32)
    s = bf16_round((qf @ kf.T).astype(np.float32))                       # [16, T]
    m = s.max(axis=-1).astype(np.float32)
    if running_max is not None:
        m = np.maximum(m, np.asarray(running_max, np.float32))
    e = np.minimum(np.exp((s - m[:, None]).astype(np.float32)).astype(np.float32), mk[None, :])
    page_sum = (e.sum(axis=-1, dtype=np.float32) + EPS).astype(np.float32)
    w = bf16_round(e)
    groups = [bf16_round((w[:, g:g + FULL_GROUP] @ vf[g:g + FULL_GROUP]).astype(np.float32))
              for g in range(0, kf.shape[0], FULL_GROUP)]
    total = np.zeros_like(groups[0])
    for part in groups:
        total = (total + part).astype(np.float32)
    values = bf16_round(total)
    if running_max is None:
        return m, page_sum, f32_to_bf16(values)
    r = np.exp((np.asarray(running_max, np.float32) - m).astype(np.float32)).astype(np.float32)
    new_sum = (np.asarray(running_sum, np.float32) * r + page_sum).astype(np.float32)
    scaled = bf16_round(bf16_to_f32(out) * r[:, None])
    return m, new_sum, f32_to_bf16((scaled + values).astype(np.float32))


def full_attention_output(x, running_sum, post_rms_weight, o_weight, o_scale, residual):
    """ops::full_attention_output (FOG/src/ops.rs:184-199): bf16(out / running sum) per head
    (full/attention.rs:341-364), the O projection (scaled_projection, K = 8192), RMSNorm,
    residual add."""
    xf = bf16_to_f32(x).reshape(16, 512)
    y = f32_to_bf16((xf / np.asarray(running_sum, np.float32)[:, None]).astype(np.float32)).reshape(-1)
    projected = scaled_projection(y, e4m3_to_f32(o_weight), bf16_to_f32(o_scale))
    return add_bf16(residual, rms_norm(projected, post_rms_weight))


def full_attention_float64(q, k_pages, v_pages, masks):
    """Masked softmax attention over the pages in float64 (the mathematical op: gemma4.py's SDPA
    with scale 1.0), for validating the paged restatement."""
    qf = bf16_to_f32(q).astype(np.float64)
    kf = np.concatenate([bf16_to_f32(k) for k in k_pages]).astype(np.float64)
    vf = np.concatenate([bf16_to_f32(v) for v in v_pages]).astype(np.float64)
    mk = np.concatenate([np.asarray(m) for m in masks])
    s = np.where(mk[None, :] > 0, qf @ kf.T, -np.inf)
    p = np.exp(s - s.max(axis=-1, keepdims=True))
    return (p / p.sum(axis=-1, keepdims=True)) @ vf


def sliding_attention(q, k_cache, v_cache, mask, scale=1.0):
    """Restatement of the device attention (FOG/src/device/sliding/attention.rs:27-196).

    q: bf16 bits [Ns, G, D]; caches: bf16 bits [T, Ns, D]; mask: f32 [T] (0/1 row).
    s = bf16(scale * q.k) in f32; m = max over ALL slots; p = min(exp(s - m), mask);
    sum = sum(p) + 1e-6; o = bf16(sum_t bf16(p_t) * v_t); out = bf16(o / sum).
    """
    qf = bf16_to_f32(q)
    kf = bf16_to_f32(k_cache)
    vf = bf16_to_f32(v_cache)
    mk = np.asarray(mask, dtype=np.float32)
    scores = np.einsum("ngd,tnd->ngt", qf, kf, dtype=np.float32, optimize=True).astype(np.float32)
    s = bf16_round(scores * np.float32(scale))
    m = s.max(axis=-1, keepdims=True)
    p = np.minimum(np.exp((s - m).astype(np.float32)).astype(np.float32), mk[None, None, :])
    total = (p.sum(axis=-1, dtype=np.float32) + EPS).astype(np.float32)
    w = bf16_round(p)
    o = bf16_round(np.einsum("ngt,tnd->ngd", w, vf, dtype=np.float32, optimize=True).astype(np.float32))
    return f32_to_bf16((o / total[..., None]).astype(np.float32))


def attention_float64(q, k_cache, v_cache, mask, scale=1.0):
    """Masked softmax attention in float64 (the mathematical op, for validating the above)."""
    qf = bf16_to_f32(q).astype(np.float64)
    kf = bf16_to_f32(k_cache).astype(np.float64)
    vf = bf16_to_f32(v_cache).astype(np.float64)
    s = np.einsum("ngd,tnd->ngt", qf, kf) * scale
    s = np.where(np.asarray(mask)[None, None, :] > 0, s, -np.inf)
    s = s - s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(axis=-1, keepdims=True)
    return np.einsum("ngt,tnd->ngd", p, vf)
