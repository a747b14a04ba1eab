"""GPU: the batched decode (BASELINE configs[4] at batch > 1). final_norm_and_logits on a batch of
tokens against the single-token op; a decoder made for a batch of sequences (g4_decoder_create_batch)
against the same batched ops called one by one (bit for bit: hidden state, logits, every cache), and
a one-layer batched step against batch-1 decoders run on each sequence alone, within the reference
grader's tolerances (FOG/src/bin/test_kernels.rs:447-465; the batched contractions sum in another
f32 order). The model mixes local and global-shaped sliding layers, NVFP4 and FP8 feed-forwards,
row-major and unit-tiled weights."""

import dataclasses

import numpy as np
import pytest

from helpers import ATOL, within
from oracle import ops as oracle
from test_gpu_decoder import make_layer, rope_table
from test_gpu_parity import host_bits

pytestmark = pytest.mark.gpu
H, NS, DS = 3840, 8, 256
VOCAB, LM_ROWS = 4096, 8192


def _bits(t):
    return host_bits(t.contiguous())


@pytest.mark.parametrize("m", [2, 8, 17, 32, 33])
def test_logits_batch_matches_single_token(device, m):
    import torch
    from g4b200 import ops

    gen = torch.Generator(device="cuda")
    gen.manual_seed(300 + m)
    tab = (torch.randn((LM_ROWS, H), generator=gen, device="cuda") * 0.03).to(torch.bfloat16)
    gamma = (1 + torch.randn(H, generator=gen, device="cuda") * 0.1).to(torch.bfloat16)
    x = torch.randn((m, H), generator=gen, device="cuda").to(torch.bfloat16)
    out = torch.zeros((m, LM_ROWS), dtype=torch.bfloat16, device="cuda")
    ops.final_norm_and_logits_batch(device, x, gamma, tab, out)
    device.check()
    got = _bits(out)
    for i in range(m):
        one = torch.zeros(LM_ROWS, dtype=torch.bfloat16, device="cuda")
        ops.final_norm_and_logits(device, x[i], gamma, tab, one)
        device.check()
        ok, maxd, exact = within(_bits(one), got[i], 0.01)
        assert ok and exact > 0.9, (i, maxd, exact)
    want = oracle.final_norm_and_logits(_bits(x[0]), _bits(gamma), _bits(tab))
    ok, maxd, _ = within(want, got[0], 0.01)
    assert ok, maxd


def test_logits_batch_partial_tile_runs_token_by_token(device):
    """A table slice that is not whole 128-row tiles (a tensor-parallel rank's odd slice) takes the
    single-token kernel per row: bit-identical to it."""
    import torch
    from g4b200 import ops

    gen = torch.Generator(device="cuda")
    gen.manual_seed(31)
    rows = 5000
    tab = (torch.randn((rows, H), generator=gen, device="cuda") * 0.03).to(torch.bfloat16)
    gamma = (1 + torch.randn(H, generator=gen, device="cuda") * 0.1).to(torch.bfloat16)
    x = torch.randn((3, H), generator=gen, device="cuda").to(torch.bfloat16)
    out = torch.zeros((3, rows), dtype=torch.bfloat16, device="cuda")
    ops.final_norm_and_logits_batch(device, x, gamma, tab, out)
    for i in range(3):
        one = torch.zeros(rows, dtype=torch.bfloat16, device="cuda")
        ops.final_norm_and_logits(device, x[i], gamma, tab, one)
        assert torch.equal(out[i], one)
    device.check()


@pytest.fixture(scope="module")
def batch_model(device):
    import torch
    from g4b200 import decoder

    gen = torch.Generator(device="cuda")
    gen.manual_seed(91)
    layers = [make_layer(gen, 1024, decoder.ROPE_LOCAL, decoder.FFN_NVFP4, False, device),
              make_layer(gen, 4096, decoder.ROPE_GLOBAL, decoder.FFN_FP8, True, device),
              make_layer(gen, 1024, decoder.ROPE_LOCAL, decoder.FFN_FP8, False, device)]
    cos_l, sin_l = rope_table(1e4)
    cos_g, sin_g = rope_table(1e6)
    table = (torch.randn((VOCAB, H), generator=gen, device="cuda") * 0.03).to(torch.bfloat16)
    lm_head = (torch.randn((LM_ROWS, H), generator=gen, device="cuda") * 0.03).to(torch.bfloat16)
    final_norm = (1 + torch.randn(H, generator=gen, device="cuda") * 0.1).to(torch.bfloat16)
    return dict(layers=layers, gen=gen, tables=dict(cos_local=cos_l, sin_local=sin_l, cos_global=cos_g,
                                                    sin_global=sin_g, embedding_table=table,
                                                    final_norm_weight=final_norm, lm_head_weight=lm_head))


def batched_layers(model, m):
    """The model's layers with m seeded rings per cache ([m, ring, Ns, Ds])."""
    import torch

    out = []
    for i, lay in enumerate(model["layers"]):
        g = torch.Generator(device="cuda")
        g.manual_seed(1000 * m + i)
        shape = (m, lay.k_cache.shape[0], NS, DS)
        k = torch.randn(shape, generator=g, device="cuda").to(torch.bfloat16)
        v = torch.randn(shape, generator=g, device="cuda").to(torch.bfloat16)
        out.append(dataclasses.replace(lay, k_cache=k, v_cache=v))
    return out


def batched_ops(device, model, layers, tokens, positions):
    """The batched decoder's launches through the op entry points (as tests/test_gpu_decoder.py's
    one_by_one does for batch 1): each sequence's embedding, then per layer the batched QKV,
    attention (given the QKV op's kv_offset), O and feed-forward, then the batched logits."""
    import torch
    from g4b200 import decoder, ops

    t = model["tables"]
    m = len(tokens)
    x = torch.zeros((m, H), dtype=torch.bfloat16, device="cuda")
    for i, tok in enumerate(tokens):
        ops.embed_token(device, t["embedding_table"], torch.tensor([int(tok) * H * 2], dtype=torch.int32,
                                                                     device="cuda"), x[i])
    q = torch.zeros((m, NS, 2, DS), dtype=torch.bfloat16, device="cuda")
    attn = torch.zeros_like(q)
    rope = torch.tensor([int(p) * DS * 2 for p in positions], dtype=torch.int32, device="cuda")
    for lay in layers:
        ring = lay.k_cache.shape[1]
        kv = torch.tensor([(int(p) % ring) * NS * DS * 2 for p in positions], dtype=torch.int32, device="cuda")
        mask = torch.stack([(torch.arange(ring, device="cuda") <= min(int(p), ring - 1)).to(torch.float32)
                            for p in positions])
        glob = lay.rope == decoder.ROPE_GLOBAL
        cos, sin = (t["cos_global"], t["sin_global"]) if glob else (t["cos_local"], t["sin_local"])
        ops.sliding_project_qkv_batch(device, x, lay.q_weight, lay.k_weight, lay.v_weight, lay.q_weight_scale,
                                      lay.k_weight_scale, lay.v_weight_scale, lay.input_rms_weight, lay.q_rms_weight,
                                      lay.k_rms_weight, kv, rope, cos, sin, lay.k_cache, lay.v_cache, q,
                                      tiled=lay.tiled)
        ops.sliding_attention_batch(device, q, lay.k_cache, lay.v_cache, mask, attn, scale=lay.attn_scale,
                                    kv_offset=kv)
        ops.sliding_attention_output_batch(device, attn, lay.post_attn_rms_weight, lay.o_weight, lay.o_weight_scale,
                                           x, tiled=lay.tiled)
        if lay.ffn == decoder.FFN_FP8 and lay.tiled:
            ops.decoder_feedforward_fp8_batch_tiled(device, x, lay.pre_ff_rms_weight, lay.up_weight, lay.down_weight,
                                                    lay.up_scale, lay.gate_scale, lay.down_scale,
                                                    lay.post_ff_rms_weight, lay.layer_scalar)
        elif lay.ffn == decoder.FFN_FP8:
            ops.decoder_feedforward_fp8_batch(device, x, lay.pre_ff_rms_weight, lay.up_weight, lay.gate_weight,
                                              lay.down_weight, lay.up_scale, lay.gate_scale, lay.down_scale,
                                              lay.post_ff_rms_weight, lay.layer_scalar)
        else:
            ops.decoder_feedforward_batch(device, x, lay.pre_ff_rms_weight, lay.up_weight, lay.gate_weight,
                                          lay.down_weight, lay.up_scale, lay.gate_scale, lay.down_scale,
                                          lay.up_global_scale, lay.gate_global_scale, lay.down_global_scale,
                                          lay.post_ff_rms_weight, lay.layer_scalar)
    logits = torch.zeros((m, LM_ROWS), dtype=torch.bfloat16, device="cuda")
    ops.final_norm_and_logits_batch(device, x, t["final_norm_weight"], t["lm_head_weight"], logits)
    device.check()
    return _bits(x), _bits(logits)


@pytest.mark.parametrize("m", [3, 17, 32])
def test_batched_decoder_equals_the_batched_ops(device, batch_model, m):
    """One step of the batched decoder against its ops called one by one through their entry
    points on the same inputs: hidden state, logits and every layer's caches bit for bit (each
    batched op's parity with the oracle is tests/test_gpu_batch*.py's)."""
    from g4b200 import decoder

    layers = batched_layers(batch_model, m)
    start = [(lay.k_cache.clone(), lay.v_cache.clone()) for lay in layers]
    rng = np.random.default_rng(m)
    tokens = rng.integers(0, VOCAB, size=m)
    positions = rng.choice(4096, size=m, replace=False)
    dec = decoder.Decoder(device, layers, batch=m, **batch_model["tables"])
    dec.step(tokens, positions)
    device.check()
    hid, logits = _bits(dec.hidden()), _bits(dec.logits())
    caches = [(_bits(lay.k_cache), _bits(lay.v_cache)) for lay in layers]
    dec.close()
    again = [dataclasses.replace(lay, k_cache=k0, v_cache=v0) for lay, (k0, v0) in zip(layers, start)]
    want_hid, want_logits = batched_ops(device, batch_model, again, tokens, positions)
    assert np.array_equal(hid, want_hid)
    assert np.array_equal(logits, want_logits)
    for (kb, vb), lay in zip(caches, again):
        assert np.array_equal(kb, _bits(lay.k_cache)) and np.array_equal(vb, _bits(lay.v_cache))


def test_batched_decoder_one_layer_matches_each_sequence_alone(device, batch_model):
    """Numerics against batch 1: a one-layer model's batched step equals batch-1 decoders run on
    each sequence alone within the grader's tolerances (over more layers the two contraction orders'
    last-bit differences compound, which is why the multi-layer check above is against the
    batched ops)."""
    from g4b200 import decoder

    m = 17
    layers = batched_layers(dict(batch_model, layers=batch_model["layers"][2:3]), m)
    start = [(lay.k_cache.clone(), lay.v_cache.clone()) for lay in layers]
    rng = np.random.default_rng(m)
    tokens = rng.integers(0, VOCAB, size=m)
    positions = rng.choice(4096, size=m, replace=False)
    dec = decoder.Decoder(device, layers, batch=m, **batch_model["tables"])
    dec.step(tokens, positions)
    device.check()
    hid, logits = _bits(dec.hidden()), _bits(dec.logits())
    slots = [(_bits(lay.k_cache), _bits(lay.v_cache)) for lay in layers]
    dec.close()
    bad = []  # every sequence is checked; the failures are reported together
    for i in range(m):
        alone = [dataclasses.replace(lay, k_cache=k0[i].clone(), v_cache=v0[i].clone())
                 for lay, (k0, v0) in zip(layers, start)]
        one = decoder.Decoder(device, alone, **batch_model["tables"])
        one.step(int(tokens[i]), int(positions[i]))
        device.check()
        ok, maxd, exact = within(_bits(one.hidden()), hid[i], ATOL["sliding_attention_output"])
        if not ok:
            bad.append(("hidden", i, maxd, exact))
        ok, maxd, exact = within(_bits(one.logits()), logits[i], 0.01)
        if not ok:
            bad.append(("logits", i, maxd, exact))
        for lay, a, (kb, vb) in zip(layers, alone, slots):
            slot = int(positions[i]) % lay.k_cache.shape[1]
            for name, got, want in (("k", kb[i, slot], _bits(a.k_cache)[slot]),
                                    ("v", vb[i, slot], _bits(a.v_cache)[slot])):
                ok, maxd, _ = within(want, got, ATOL["sliding_project_qkv"])
                if not ok:
                    bad.append(("slot", name, i, maxd))
        one.close()
    assert not bad, bad


def test_batched_decoder_graph_equals_eager(device, batch_model):
    """Two steps replayed from the captured graph equal two eager steps, bit for bit."""
    from g4b200 import decoder

    m = 4
    results = []
    for graph in (False, True):
        layers = batched_layers(batch_model, m)
        dec = decoder.Decoder(device, layers, batch=m, **batch_model["tables"])
        if graph:
            dec.capture()
        outs = []
        for t in range(2):
            dec.step([5 + t, 17, 99, 4000], [10 + t, 2047 + t, 0 + t, 3000 + t])
            device.check()
            outs.append((_bits(dec.hidden()), _bits(dec.logits())))
        outs.append([(_bits(lay.k_cache), _bits(lay.v_cache)) for lay in layers])
        results.append(outs)
        dec.close()
    eager, graph = results
    for a, b in zip(eager[:2], graph[:2]):
        assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])
    for (ka, va), (kb, vb) in zip(eager[2], graph[2]):
        assert np.array_equal(ka, kb) and np.array_equal(va, vb)


def test_batched_decoder_refuses_what_it_cannot_run(device, batch_model):
    from g4b200 import G4Error, decoder

    with pytest.raises(G4Error):
        decoder.Decoder(device, batched_layers(batch_model, 2), batch=65, **batch_model["tables"])
