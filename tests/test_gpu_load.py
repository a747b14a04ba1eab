"""GPU: a checkpoint read by g4b200.load (the reference's names, FOG/src/host/load.rs:130-390),
uploaded and packed into the unit-tiled layout by load.to_device, runs through the decode driver
and gives exactly what the row-major op entry points give on the checkpoint's arrays: the loader
put every tensor where the ops expect it (the reciprocal global scales included)."""

import numpy as np
import pytest

import gaussian
from g4b200 import load
from test_gpu_parity import dev_tensor, host_bits

pytestmark = pytest.mark.gpu
H, L = 3840, 15360


def sliding_layer(i, salt):
    """Layer i's tensors as a checkpoint stores them (Gaussian weights quantised per BASELINE)."""
    q, o = gaussian.qkv(1e4, salt=salt), gaussian.attention_output(salt)
    f = gaussian.ffn_nvfp4(salt)
    r = np.random.default_rng(100 + salt)
    p = f"model.language_model.layers.{i}"
    t = {f"{p}.input_layernorm.weight": ("BF16", q["input_rms_weight"]),
         f"{p}.post_attention_layernorm.weight": ("BF16", o["post_attn_rms_weight"]),
         f"{p}.pre_feedforward_layernorm.weight": ("BF16", f["pre_ff_rms_weight"]),
         f"{p}.post_feedforward_layernorm.weight": ("BF16", f["post_ff_rms_weight"]),
         f"{p}.self_attn.q_norm.weight": ("BF16", q["q_rms_weight"]),
         f"{p}.self_attn.k_norm.weight": ("BF16", q["k_rms_weight"]),
         f"{p}.layer_scalar": ("BF16", f["layer_scalar"][:1])}
    for name in ("q", "k", "v"):
        t[f"{p}.self_attn.{name}_proj.weight"] = ("F8_E4M3", q[f"{name}_weight"])
        t[f"{p}.self_attn.{name}_proj.weight_scale"] = ("BF16", q[f"{name}_weight_scale"].reshape(-1, 1))
    t[f"{p}.self_attn.o_proj.weight"] = ("F8_E4M3", o["o_weight"])
    t[f"{p}.self_attn.o_proj.weight_scale"] = ("BF16", o["o_weight_scale"].reshape(-1, 1))
    for name in ("up", "gate", "down"):
        t[f"{p}.mlp.{name}_proj.weight_packed"] = ("U8", f[f"{name}_weight_packed"])
        t[f"{p}.mlp.{name}_proj.weight_scale"] = ("F8_E4M3", f[f"{name}_weight_scale"])
        # a checkpoint stores the reciprocal of the multiplier the op takes
        t[f"{p}.mlp.{name}_proj.weight_global_scale"] = ("F32", np.array(np.float32(1) / f[f"{name}_global_scale"][0],
                                                                          np.float32))
    return t, q, o, f, r


def test_loaded_layer_runs_like_the_op_entry_points(device, tmp_path):
    import torch
    from g4b200 import decoder, ops

    t, q, o, f, r = sliding_layer(0, 3)
    t["model.language_model.embed_tokens.weight"] = ("BF16", gaussian.bf16(r.standard_normal((64, H)) * 0.03))
    t["model.language_model.norm.weight"] = ("BF16", gaussian.bf16(1 + 0.1 * r.standard_normal(H)))
    load.write_safetensors(tmp_path / "model.safetensors", t)
    table, final, layers = load.read_checkpoint(tmp_path)
    lay = load.to_device(device, layers[0], ring_len=1024)
    assert lay.tiled and lay.ffn == decoder.FFN_NVFP4

    pos = 700
    cos = np.zeros((2048, 256), np.uint16)
    sin = np.zeros((2048, 256), np.uint16)
    from oracle.ops import negate_low_half, rope_tables

    c, s = rope_tables(256, 1e4, 1.0, pos)
    cos[pos], sin[pos] = gaussian.bf16(c), gaussian.bf16(negate_low_half(s))
    cos_d, sin_d = dev_tensor(cos), dev_tensor(sin)
    x0 = gaussian.bf16(r.standard_normal(H))

    # the decoder on the loaded (tiled) layer, the hidden state written directly
    dec = decoder.Decoder(device, [lay], cos_local=cos_d, sin_local=sin_d)
    try:
        dec.hidden().copy_(dev_tensor(x0))
        dec.step(0, pos)
        device.check()
        got = host_bits(dec.hidden())
    finally:
        dec.close()

    # the row-major entry points on the checkpoint's own arrays
    h = layers[0].t
    x = dev_tensor(x0)
    kc = torch.zeros((1024, 8, 256), dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    qo = torch.zeros((8, 2, 256), dtype=torch.bfloat16, device="cuda")
    at = torch.zeros_like(qo)
    ops.sliding_project_qkv(device, x, *(dev_tensor(h[k]) for k in (
        "q_weight", "k_weight", "v_weight", "q_weight_scale", "k_weight_scale", "v_weight_scale", "input_layernorm",
        "q_norm", "k_norm")), dev_tensor(np.array([pos * 8 * 256 * 2], np.int32)),
        dev_tensor(np.array([pos * 256 * 2], np.int32)), cos_d, sin_d, kc, vc, qo)
    mask = dev_tensor((np.arange(1024) <= pos).astype(np.float32))
    ops.sliding_attention(device, qo, kc, vc, mask, at)
    ops.sliding_attention_output(device, at, dev_tensor(h["post_attention_layernorm"]), dev_tensor(h["o_weight"]),
                                 dev_tensor(h["o_weight_scale"]), x)
    ops.decoder_feedforward(device, x, dev_tensor(h["pre_feedforward_layernorm"]), *(dev_tensor(h[k]) for k in (
        "up_weight_packed", "gate_weight_packed", "down_weight_packed", "up_weight_scale", "gate_weight_scale",
        "down_weight_scale", "up_global_scale", "gate_global_scale", "down_global_scale",
        "post_feedforward_layernorm", "layer_scalar")))
    device.check()
    want = host_bits(x)
    assert np.array_equal(got, want)
    assert np.allclose(h["up_global_scale"], f["up_global_scale"], rtol=1e-6)  # 1 / (1 / g) == g, to f32
