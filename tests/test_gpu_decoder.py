"""GPU: the decode driver (g4_decoder_*, one token through a model per call) against the same ops
called one by one through their own entry points, bit for bit: the embedding, every layer's KV ring
slot, the hidden state after the last layer and the logits. The model mixes what a Gemma-4 decode
mixes: sliding layers on a 1024-slot ring with the local RoPE table, a global-shaped layer on a
4096-slot ring with the global table, NVFP4 and FP8 feed-forwards, row-major and unit-tiled
weights. Also: steps replayed from the captured CUDA graph equal eager steps, positions past the
ring wrap the slot and fill the mask, and bad inputs raise their device error bits."""

import numpy as np
import pytest

import bench
from oracle.ops import negate_low_half

pytestmark = pytest.mark.gpu
H, L, NS, GS, DS, QS, PS = 3840, 15360, 8, 2, 256, 4096, 2048
ROPE_ROWS, VOCAB, LM_ROWS = 4096, 4096, 8192


def rope_table(theta, dim=DS, rotated=DS):
    """cos / sin [ROPE_ROWS, dim] for every position; `rotated` of the dims turn (the rest: cos 1, sin 0)."""
    import torch

    pos = np.arange(ROPE_ROWS, dtype=np.float64)[:, None]
    inv = 1.0 / (np.float64(theta) ** (np.arange(0, rotated, 2, dtype=np.float64) / dim))
    inv = np.concatenate([inv, np.zeros(dim // 2 - rotated // 2)])
    emb = np.concatenate([pos * inv, pos * inv], axis=1)
    cos, sin = np.cos(emb).astype(np.float32), np.sin(emb).astype(np.float32)
    sin = np.stack([negate_low_half(r) for r in sin])
    return (torch.from_numpy(cos).cuda().to(torch.bfloat16), torch.from_numpy(sin).cuda().to(torch.bfloat16))


def make_layer(gen, ring, rope, ffn, tiled, device):
    import torch
    from g4b200 import decoder, ops

    def normal(*shape, std=1.0):
        return torch.randn(*shape, generator=gen, device="cuda") * std

    def bf(t):
        return t.to(torch.bfloat16).contiguous()

    q_w, q_s = bench.quant_fp8_rows(normal(QS, H, std=0.02))
    k_w, k_s = bench.quant_fp8_rows(normal(PS, H, std=0.02))
    v_w, v_s = bench.quant_fp8_rows(normal(PS, H, std=0.02))
    o_w, o_s = bench.quant_fp8_rows(normal(H, QS, std=0.02))
    kw = dict(input_rms_weight=bf(1 + normal(H, std=0.1)), q_weight=q_w, k_weight=k_w, v_weight=v_w,
              q_weight_scale=bf(q_s), k_weight_scale=bf(k_s), v_weight_scale=bf(v_s),
              q_rms_weight=bf(1 + normal(DS, std=0.1)), k_rms_weight=bf(1 + normal(DS, std=0.1)),
              k_cache=bf(normal(ring, NS, DS)), v_cache=bf(normal(ring, NS, DS)),
              post_attn_rms_weight=bf(1 + normal(H, std=0.1)), o_weight=o_w, o_weight_scale=bf(o_s),
              pre_ff_rms_weight=bf(1 + normal(H, std=0.1)), post_ff_rms_weight=bf(1 + normal(H, std=0.1)),
              layer_scalar=bf(torch.full((8,), 0.375, device="cuda")))
    if ffn == decoder.FFN_FP8:
        (up, up_s), (gate, gate_s), (down, down_s) = (bench.quant_fp8_rows(normal(r, c, std=0.02))
                                                      for r, c in ((L, H), (L, H), (H, L)))
        kw.update(up_weight=up, gate_weight=gate, down_weight=down, up_scale=up_s.float().contiguous(),
                  gate_scale=gate_s.float().contiguous(), down_scale=down_s.float().contiguous())
    else:
        (up, up_s, up_g), (gate, gate_s, gate_g), (down, down_s, down_g) = (
            bench.quant_nvfp4(normal(r, c, std=0.02)) for r, c in ((L, H), (L, H), (H, L)))
        kw.update(up_weight=up, gate_weight=gate, down_weight=down, up_scale=up_s, gate_scale=gate_s,
                  down_scale=down_s, up_global_scale=up_g, gate_global_scale=gate_g, down_global_scale=down_g)
    lay = decoder.Layer(**kw, rope=rope, ffn=ffn, tiled=False)
    lay.rowmajor = dict(kw)  # the reference-layout tensors, for the one-by-one path
    if tiled:
        for name in ("q_weight", "k_weight", "v_weight", "o_weight"):
            setattr(lay, name, ops.tile_weight(device, name, getattr(lay, name)))
        if ffn == decoder.FFN_FP8:
            lay.up_weight = ops.pack_upgate_fp8(device, kw["up_weight"], kw["gate_weight"])
            lay.down_weight = ops.tile_weight(device, "down_weight", kw["down_weight"])
        else:
            lay.up_weight = ops.pack_upgate(device, kw["up_weight"], kw["gate_weight"], scales=False)
            lay.up_scale = ops.pack_upgate(device, kw["up_scale"], kw["gate_scale"], scales=True)
            lay.down_weight = ops.tile_weight(device, "down_weight_packed", kw["down_weight"])
            lay.down_scale = ops.tile_weight(device, "down_weight_scale", kw["down_scale"])
        lay.tiled = True
    return lay


def make_full_layer(gen, ring, ffn, tiled, device):
    """A global (full-attention) layer: q [8192, H], the K = V head [512, H], O [H, 8192], pages of K / V."""
    import torch
    from g4b200 import decoder, ops

    base = make_layer(gen, 1024, decoder.ROPE_GLOBAL, ffn, False, device)

    def normal(*shape, std=1.0):
        return torch.randn(*shape, generator=gen, device="cuda") * std

    q_w, q_s = bench.quant_fp8_rows(normal(8192, H, std=0.02))
    k_w, k_s = bench.quant_fp8_rows(normal(512, H, std=0.02))
    o_w, o_s = bench.quant_fp8_rows(normal(H, 8192, std=0.02))
    base.q_weight, base.k_weight, base.o_weight = q_w, k_w, o_w
    base.q_weight_scale, base.k_weight_scale, base.o_weight_scale = (t.to(torch.bfloat16) for t in (q_s, k_s, o_s))
    base.v_weight = base.v_weight_scale = None
    base.q_rms_weight = (1 + normal(512, std=0.1)).to(torch.bfloat16)
    base.k_rms_weight = (1 + normal(512, std=0.1)).to(torch.bfloat16)
    base.k_cache = normal(ring, 512).to(torch.bfloat16)
    base.v_cache = normal(ring, 512).to(torch.bfloat16)
    base.kind = decoder.LAYER_FULL
    base.rowmajor_q, base.rowmajor_k, base.rowmajor_o = q_w, k_w, o_w  # the full ops take the reference layout
    if tiled:
        for name in ("q_weight", "k_weight", "o_weight"):
            setattr(base, name, ops.tile_weight(device, name, getattr(base, name)))
        if ffn == decoder.FFN_FP8:
            base.up_weight = ops.pack_upgate_fp8(device, base.rowmajor["up_weight"], base.rowmajor["gate_weight"])
            base.down_weight = ops.tile_weight(device, "down_weight", base.rowmajor["down_weight"])
        base.tiled = True
    return base


@pytest.fixture(scope="module")
def model(device):
    import torch
    from g4b200 import decoder

    gen = torch.Generator(device="cuda")
    gen.manual_seed(77)
    layers = [make_layer(gen, 1024, decoder.ROPE_LOCAL, decoder.FFN_NVFP4, False, device),
              make_layer(gen, 4096, decoder.ROPE_GLOBAL, decoder.FFN_FP8, True, device),
              make_full_layer(gen, 2048, decoder.FFN_FP8, True, device),
              make_layer(gen, 1024, decoder.ROPE_LOCAL, decoder.FFN_FP8, False, device),
              make_full_layer(gen, 1024, decoder.FFN_NVFP4, False, device),
              make_layer(gen, 1024, decoder.ROPE_LOCAL, decoder.FFN_NVFP4, True, device)]
    cos_l, sin_l = rope_table(1e4)
    cos_g, sin_g = rope_table(1e6)
    cos_f, sin_f = rope_table(1e6, 512, 128)
    table = (torch.randn((VOCAB, H), generator=gen, device="cuda") * 0.03).to(torch.bfloat16)
    lm_head = (torch.randn((LM_ROWS, H), generator=gen, device="cuda") * 0.03).to(torch.bfloat16)
    final_norm = (1 + torch.randn(H, generator=gen, device="cuda") * 0.1).to(torch.bfloat16)
    return dict(layers=layers, cos_l=cos_l, sin_l=sin_l, cos_g=cos_g, sin_g=sin_g, cos_f=cos_f, sin_f=sin_f,
                table=table, lm_head=lm_head, final_norm=final_norm)


def caches(layers):
    return [(lay.k_cache.clone(), lay.v_cache.clone()) for lay in layers]


def restore(layers, saved):
    for lay, (k, v) in zip(layers, saved):
        lay.k_cache.copy_(k)
        lay.v_cache.copy_(v)


def one_by_one(device, m, token, pos):
    """The reference host's order of launches (runtime.rs:340-451) through the op entry points."""
    import torch
    from g4b200 import decoder, ops

    x = torch.zeros(H, dtype=torch.bfloat16, device="cuda")
    ops.embed_token(device, m["table"], torch.tensor([token * H * 2], dtype=torch.int32, device="cuda"), x)
    q = torch.zeros((NS, GS, DS), dtype=torch.bfloat16, device="cuda")
    attn = torch.zeros_like(q)
    rope_off = torch.tensor([pos * DS * 2], dtype=torch.int32, device="cuda")
    for lay in m["layers"]:
        ring = lay.ring_len
        if lay.kind == decoder.LAYER_FULL:  # the reference host's full-layer launches (runtime.rs:462-541)
            slot = pos % ring
            page = slot // 512
            qf = torch.zeros((16, 512), dtype=torch.bfloat16, device="cuda")
            of = torch.zeros_like(qf)
            rmax = torch.zeros(16, dtype=torch.float32, device="cuda")
            rsum = torch.zeros_like(rmax)
            ops.full_project_qkv(device, x, lay.q_weight if not lay.tiled else lay.rowmajor_q, lay.k_weight
                                 if not lay.tiled else lay.rowmajor_k, lay.q_weight_scale, lay.k_weight_scale,
                                 lay.input_rms_weight, lay.q_rms_weight, lay.k_rms_weight,
                                 torch.tensor([(slot % 512) * 512 * 2], dtype=torch.int32, device="cuda"),
                                 torch.tensor([pos * 512 * 2], dtype=torch.int32, device="cuda"), m["cos_f"],
                                 m["sin_f"], lay.k_cache[page * 512:(page + 1) * 512],
                                 lay.v_cache[page * 512:(page + 1) * 512], qf)
            for p in range(ring // 512):
                if p * 512 > pos:
                    break
                mask = (torch.arange(512, device="cuda") + p * 512 <= pos).to(torch.float32)
                ops.full_attention_page(device, qf, lay.k_cache[p * 512:(p + 1) * 512],
                                        lay.v_cache[p * 512:(p + 1) * 512], mask, rmax, rsum, of, first=p == 0)
            ops.full_attention_output(device, of, rsum, lay.post_attn_rms_weight,
                                      lay.o_weight if not lay.tiled else lay.rowmajor_o, lay.o_weight_scale, x)
            ffn_one(device, x, lay)
            continue
        kv_off = torch.tensor([(pos % ring) * NS * DS * 2], dtype=torch.int32, device="cuda")
        mask = (torch.arange(ring, device="cuda") <= min(pos, ring - 1)).to(torch.float32)
        cos, sin = (m["cos_g"], m["sin_g"]) if lay.rope == decoder.ROPE_GLOBAL else (m["cos_l"], m["sin_l"])
        ops.sliding_project_qkv(device, x, lay.q_weight, lay.k_weight, lay.v_weight, lay.q_weight_scale,
                                lay.k_weight_scale, lay.v_weight_scale, lay.input_rms_weight, lay.q_rms_weight,
                                lay.k_rms_weight, kv_off, rope_off, cos, sin, lay.k_cache, lay.v_cache, q,
                                tiled=lay.tiled)
        ops.sliding_attention(device, q, lay.k_cache, lay.v_cache, mask, attn, scale=lay.attn_scale)
        ops.sliding_attention_output(device, attn, lay.post_attn_rms_weight, lay.o_weight, lay.o_weight_scale, x,
                                     tiled=lay.tiled)
        ffn_one(device, x, lay)
    logits = torch.zeros(LM_ROWS, dtype=torch.bfloat16, device="cuda")
    ops.final_norm_and_logits(device, x, m["final_norm"], m["lm_head"], logits)
    device.check()
    return x.clone(), logits.clone()


def ffn_one(device, x, lay):
    """The layer's feed-forward through its entry point (NVFP4 or FP8, row-major or tiled)."""
    from g4b200 import decoder, ops

    if lay.ffn == decoder.FFN_FP8 and lay.tiled:
        ops.decoder_feedforward_fp8_tiled(device, x, lay.pre_ff_rms_weight, lay.up_weight, lay.down_weight,
                                          lay.up_scale, lay.gate_scale, lay.down_scale, lay.post_ff_rms_weight,
                                          lay.layer_scalar)
    elif lay.ffn == decoder.FFN_FP8:
        ops.decoder_feedforward_fp8(device, x, lay.pre_ff_rms_weight, lay.up_weight, lay.gate_weight,
                                    lay.down_weight, lay.up_scale, lay.gate_scale, lay.down_scale,
                                    lay.post_ff_rms_weight, lay.layer_scalar)
    elif lay.tiled:
        ops.decoder_feedforward_tiled(device, x, lay.pre_ff_rms_weight, lay.up_weight, lay.down_weight,
                                      lay.up_scale, lay.down_scale, lay.up_global_scale, lay.gate_global_scale,
                                      lay.down_global_scale, lay.post_ff_rms_weight, lay.layer_scalar)
    else:
        ops.decoder_feedforward(device, x, lay.pre_ff_rms_weight, lay.up_weight, lay.gate_weight,
                                lay.down_weight, lay.up_scale, lay.gate_scale, lay.down_scale,
                                lay.up_global_scale, lay.gate_global_scale, lay.down_global_scale,
                                lay.post_ff_rms_weight, lay.layer_scalar)


def make_decoder(device, m):
    from g4b200 import decoder

    return decoder.Decoder(device, m["layers"], cos_local=m["cos_l"], sin_local=m["sin_l"], cos_global=m["cos_g"],
                           sin_global=m["sin_g"], embedding_table=m["table"], final_norm_weight=m["final_norm"],
                           lm_head_weight=m["lm_head"], cos_full=m["cos_f"], sin_full=m["sin_f"])


def equal(a, b):
    import torch

    return torch.equal(a.view(torch.int16), b.view(torch.int16))


@pytest.mark.parametrize("pos", [0, 700, 1030, 4095])
def test_decoder_step_equals_ops_one_by_one(device, model, pos):
    import torch

    token = (1234 + pos) % VOCAB
    start = caches(model["layers"])
    want_x, want_logits = one_by_one(device, model, token, pos)
    want_caches = caches(model["layers"])
    restore(model["layers"], start)
    dec = make_decoder(device, model)
    try:
        dec.step(token, pos)
        device.check()
        torch.cuda.synchronize()
        assert equal(dec.hidden(), want_x)
        assert equal(dec.logits(), want_logits)
        for lay, (k, v) in zip(model["layers"], want_caches):
            assert equal(lay.k_cache, k) and equal(lay.v_cache, v)
    finally:
        dec.close()
        restore(model["layers"], start)


def test_decoder_graph_replay_equals_eager(device, model):
    """Three tokens at consecutive positions: eager steps and graph replays give the same bits."""
    import torch

    start = caches(model["layers"])
    dec = make_decoder(device, model)
    try:
        eager = []
        for i in range(3):
            dec.step(40 + i, 1022 + i)
            eager.append((dec.hidden().clone(), dec.logits().clone()))
        device.check()
        restore(model["layers"], start)
        s = torch.cuda.Stream()
        dec.capture(stream=s)
        for i in range(3):
            dec.step(40 + i, 1022 + i, stream=s)
            s.synchronize()
            assert equal(dec.hidden(), eager[i][0]) and equal(dec.logits(), eager[i][1]), i
        device.check()
    finally:
        dec.close()
        restore(model["layers"], start)


def test_decoder_bad_inputs(device, model):
    from g4b200 import G4Error

    start = caches(model["layers"])
    dec = make_decoder(device, model)
    try:
        with pytest.raises(G4Error) as err:  # a token outside the table
            dec.step(VOCAB, 3)
            device.check()
        assert err.value.flags & 64
        restore(model["layers"], start)  # (the layers still ran on the previous hidden state)
        with pytest.raises(G4Error) as err:  # a position past the RoPE table: no cache slot is written
            dec.step(5, ROPE_ROWS)
            device.check()
        assert err.value.flags & 2
        for lay, (k, v) in zip(model["layers"], start):
            assert equal(lay.k_cache, k) and equal(lay.v_cache, v)
    finally:
        dec.close()
        restore(model["layers"], start)
