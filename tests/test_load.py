"""CPU: the checkpoint loader's host side (g4b200.load): the reference's tensor names, dtypes and
shapes (FOG/src/host/load.rs:130-390), its checks and its reciprocal NVFP4 global scale, on a
synthetic safetensors checkpoint holding a sliding layer (0) and a full-attention layer (5)."""

import re

import numpy as np
import pytest

from g4b200 import load

H, L = 3840, 15360


def layer_tensors(i, rng, full):
    p = f"model.language_model.layers.{i}"
    q_rows, k_rows, o_cols, hd = (8192, 512, 8192, 512) if full else (4096, 2048, 4096, 256)
    t = {}
    for norm in ("input_layernorm", "post_attention_layernorm", "pre_feedforward_layernorm",
                 "post_feedforward_layernorm"):
        t[f"{p}.{norm}.weight"] = ("BF16", rng.integers(0, 2**16, H, dtype=np.uint16))
    projs = [("q", q_rows, H), ("k", k_rows, H), ("o", H, o_cols)] + ([] if full else [("v", k_rows, H)])
    for name, rows, cols in projs:
        t[f"{p}.self_attn.{name}_proj.weight"] = ("F8_E4M3", rng.integers(0, 256, (rows, cols), dtype=np.uint8))
        t[f"{p}.self_attn.{name}_proj.weight_scale"] = ("BF16", rng.integers(0, 2**16, (rows, 1), dtype=np.uint16))
    for name in ("q_norm", "k_norm"):
        t[f"{p}.self_attn.{name}.weight"] = ("BF16", rng.integers(0, 2**16, hd, dtype=np.uint16))
    t[f"{p}.layer_scalar"] = ("BF16", np.array([0x3EC0], np.uint16))
    for name, rows, cols in (("up", L, H), ("gate", L, H), ("down", H, L)):
        t[f"{p}.mlp.{name}_proj.weight_packed"] = ("U8", rng.integers(0, 256, (rows, cols // 2), dtype=np.uint8))
        t[f"{p}.mlp.{name}_proj.weight_scale"] = ("F8_E4M3", rng.integers(0, 128, (rows, cols // 16), dtype=np.uint8))
        t[f"{p}.mlp.{name}_proj.weight_global_scale"] = ("F32", np.array(1024.0 * (1 + i), np.float32))
    return t


@pytest.fixture(scope="module")
def checkpoint(tmp_path_factory):
    rng = np.random.default_rng(5)
    t = {"model.language_model.embed_tokens.weight": ("BF16", rng.integers(0, 2**16, (512, H), dtype=np.uint16)),
         "model.language_model.norm.weight": ("BF16", rng.integers(0, 2**16, H, dtype=np.uint16))}
    t.update(layer_tensors(0, rng, False))
    t.update(layer_tensors(5, rng, True))
    path = tmp_path_factory.mktemp("ckpt") / "model.safetensors"
    load.write_safetensors(path, t, {"format": "pt"})
    return path, t


def test_reads_every_tensor_by_the_reference_names(checkpoint):
    path, t = checkpoint
    table, final, layers = load.read_checkpoint(path.parent)
    assert [lay.index for lay in layers] == [0, 5]
    assert [lay.full for lay in layers] == [False, True]
    assert np.array_equal(table, t["model.language_model.embed_tokens.weight"][1])
    assert np.array_equal(final, t["model.language_model.norm.weight"][1])
    s, f = layers
    p = "model.language_model.layers.0"
    assert np.array_equal(s.t["q_weight"], t[f"{p}.self_attn.q_proj.weight"][1])
    assert np.array_equal(s.t["v_weight_scale"], t[f"{p}.self_attn.v_proj.weight_scale"][1].reshape(-1))
    assert np.array_equal(s.t["down_weight_packed"], t[f"{p}.mlp.down_proj.weight_packed"][1])
    assert np.array_equal(s.t["layer_scalar"], np.full(8, 0x3EC0, np.uint16))
    assert s.t["up_global_scale"].dtype == np.float32 and s.t["up_global_scale"][0] == np.float32(1 / 1024)
    assert f.t["q_weight"].shape == (8192, H) and f.t["k_weight"].shape == (512, H) and "v_weight" not in f.t
    assert f.t["o_weight"].shape == (H, 8192) and f.t["q_norm"].shape == (512,)
    assert f.t["gate_global_scale"][0] == np.float32(1 / 6144)


def test_refuses_what_the_reference_refuses(tmp_path, checkpoint):
    _, t = checkpoint
    emb = {k: v for k, v in t.items() if not k.startswith("model.language_model.layers.")}

    p = "model.language_model.layers.0"
    cases = [
        (f"{p}.mlp.up_proj.weight_global_scale", ("F32", np.array(0.0, np.float32)), "invalid NVFP4 global scale"),
        (f"{p}.mlp.up_proj.weight_global_scale", ("F32", np.array(np.inf, np.float32)), "invalid NVFP4 global scale"),
        (f"{p}.self_attn.q_proj.weight", ("BF16", np.zeros((4096, H), np.uint16)), "expected F8_E4M3"),
        (f"{p}.self_attn.k_proj.weight_scale", ("BF16", np.zeros(2048, np.uint16)), "expected BF16 [2048, 1]"),
        (f"{p}.mlp.down_proj.weight_packed", ("U8", np.zeros((H, L), np.uint8)), "expected U8"),
    ]
    for name, value, message in cases:
        d = dict(t)
        d[name] = value
        path = tmp_path / f"bad_{len(list(tmp_path.iterdir()))}.safetensors"
        load.write_safetensors(path, d)
        with pytest.raises(load.CheckpointError, match=re.escape(message)):
            load.read_checkpoint(path, layers=[0])
    d = dict(t)
    del d[f"{p}.self_attn.v_proj.weight"]
    path = tmp_path / "missing.safetensors"
    load.write_safetensors(path, d)
    with pytest.raises(load.CheckpointError, match="missing tensor"):
        load.read_checkpoint(path, layers=[0])
    path = tmp_path / "noemb.safetensors"
    load.write_safetensors(path, {k: v for k, v in t.items() if k not in emb})
    with pytest.raises(load.CheckpointError, match="embed_tokens"):
        load.read_checkpoint(path)
