"""GPU parity: the CUDA ops (called through the C ABI) against the reference's golden outputs
and the CPU oracle, on the reference's own seeded inputs (runs 0-8), its cancellation and
stress cases, plus cache-integrity, determinism and error-path checks."""

import numpy as np
import pytest

from oracle import ops as oracle
from oracle import synth
from helpers import ATOL, within

pytestmark = pytest.mark.gpu
RUNS = range(9)
SENTINEL_K, SENTINEL_V, SENTINEL_Q = 0x3E80, 0xBF00, 0x3FC0


def dev_tensor(arr, dtype=None):
    import torch

    a = np.ascontiguousarray(arr)
    if a.dtype == np.uint16:
        t = torch.from_numpy(a.view(np.int16)).view(torch.bfloat16)
    else:
        t = torch.from_numpy(a)
    t = t.cuda()
    return t.to(dtype) if dtype is not None else t


def host_bits(t):
    import torch

    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


# --------------------------------------------------------------------------------- QKV

def run_qkv(device, d, ring=1024, rows=32768, fill=(SENTINEL_K, SENTINEL_V, SENTINEL_Q)):
    from g4b200 import ops

    cos = np.zeros((rows, 256), np.uint16)
    sin = np.zeros((rows, 256), np.uint16)
    cos[d["pos"]] = d["cos_row"]
    sin[d["pos"]] = d["sin_row"]
    k_cache = dev_tensor(np.full((ring, 8, 256), fill[0], np.uint16))
    v_cache = dev_tensor(np.full((ring, 8, 256), fill[1], np.uint16))
    q_out = dev_tensor(np.full((8, 2, 256), fill[2], np.uint16))
    ops.sliding_project_qkv(device, dev_tensor(d["x"]), dev_tensor(d["q_weight"]), dev_tensor(d["k_weight"]),
                            dev_tensor(d["v_weight"]), dev_tensor(d["q_weight_scale"]),
                            dev_tensor(d["k_weight_scale"]), dev_tensor(d["v_weight_scale"]),
                            dev_tensor(d["input_rms_weight"]), dev_tensor(d["q_rms_weight"]),
                            dev_tensor(d["k_rms_weight"]), dev_tensor(d["kv_offset"]), dev_tensor(d["rope_offset"]),
                            dev_tensor(cos), dev_tensor(sin), k_cache, v_cache, q_out)
    device.check()
    return host_bits(q_out), host_bits(k_cache), host_bits(v_cache)


def check_untouched(cache, slot, fill):
    mask = np.ones(cache.shape[0], bool)
    mask[slot] = False
    assert np.all(cache[mask] == fill), "a KV-cache slot the op does not target changed"


@pytest.mark.parametrize("run", RUNS)
def test_qkv_matches_reference(device, run, golden_runs):
    d = synth.sliding_project_qkv(run)
    q, kc, vc = run_qkv(device, d)
    slot = d["pos"] % 1024
    for label, got in (("q", q.reshape(-1)), ("k", kc[slot].reshape(-1)), ("v", vc[slot].reshape(-1))):
        ok, maxd, exact = within(golden_runs[f"run{run}.sliding_project_qkv.expected.{label}"], got,
                                 ATOL["sliding_project_qkv"])
        assert ok, (label, maxd)
        assert exact > 0.99, (label, exact)
    check_untouched(kc, slot, SENTINEL_K)
    check_untouched(vc, slot, SENTINEL_V)


@pytest.mark.parametrize("case", [0, 1])
def test_qkv_cancellation_cases(device, case, golden_boundary):
    """Tiny activations after pre-RMS must survive (the reference's E53 regression)."""
    d = synth.qkv_boundary_inputs(case)
    q, kc, vc = run_qkv(device, d)
    slot = d["pos"] % 1024
    for label, got in (("q", q.reshape(-1)), ("k", kc[slot].reshape(-1)), ("v", vc[slot].reshape(-1))):
        ok, maxd, exact = within(golden_boundary[f"case{case}.expected.{label}"], got, ATOL["sliding_project_qkv"])
        assert ok, (label, maxd)
        # at least as close as the reference oracle itself, which is bit-exact here
        assert exact > 0.99, (label, exact)
    check_untouched(kc, slot, SENTINEL_K)
    check_untouched(vc, slot, SENTINEL_V)


def test_qkv_ring_2048_and_bad_offset(device):
    """BASELINE's [8 heads, 2048 slots] ring; an out-of-ring offset writes nothing and is reported."""
    from g4b200 import G4Error

    d = synth.sliding_project_qkv(4)
    d["kv_offset"] = np.array([(1500) * 8 * 256 * 2], np.int32)
    q, kc, vc = run_qkv(device, d, ring=2048)
    ref_q, ref_k, ref_v = oracle.sliding_project_qkv(d["x"], d["q_weight"], d["k_weight"], d["v_weight"],
                                                     d["q_weight_scale"], d["k_weight_scale"], d["v_weight_scale"],
                                                     d["input_rms_weight"], d["q_rms_weight"], d["k_rms_weight"],
                                                     d["cos_row"], d["sin_row"])
    assert within(ref_k, kc[1500], ATOL["sliding_project_qkv"])[0]
    assert within(ref_v, vc[1500], ATOL["sliding_project_qkv"])[0]
    check_untouched(kc, 1500, SENTINEL_K)

    d["kv_offset"] = np.array([2048 * 8 * 256 * 2], np.int32)  # one slot past the ring
    with pytest.raises(G4Error) as err:
        run_qkv(device, d, ring=2048)
    assert err.value.flags & 1


def test_qkv_last_slot_and_last_rope_row(device):
    """The largest valid offsets: the ring's last slot and the RoPE table's last row."""
    d = synth.sliding_project_qkv(6)
    ring, rows = 1024, 32768
    d["pos"] = rows - 1
    d["kv_offset"] = np.array([(ring - 1) * 8 * 256 * 2], np.int32)
    d["rope_offset"] = np.array([(rows - 1) * 256 * 2], np.int32)
    q, kc, vc = run_qkv(device, d, ring=ring, rows=rows)
    ref_q, ref_k, ref_v = oracle.sliding_project_qkv(d["x"], d["q_weight"], d["k_weight"], d["v_weight"],
                                                     d["q_weight_scale"], d["k_weight_scale"], d["v_weight_scale"],
                                                     d["input_rms_weight"], d["q_rms_weight"], d["k_rms_weight"],
                                                     d["cos_row"], d["sin_row"])
    for want, got in ((ref_q, q), (ref_k, kc[ring - 1]), (ref_v, vc[ring - 1])):
        ok, maxd, exact = within(want, got, ATOL["sliding_project_qkv"])
        assert ok and exact > 0.99, (maxd, exact)
    check_untouched(kc, ring - 1, SENTINEL_K)
    check_untouched(vc, ring - 1, SENTINEL_V)


# --------------------------------------------------------------------------------- O

def run_o(device, x, gamma, w, s, residual):
    from g4b200 import ops

    res = dev_tensor(residual)
    ops.sliding_attention_output(device, dev_tensor(x), dev_tensor(gamma), dev_tensor(w), dev_tensor(s), res)
    device.check()
    return host_bits(res)


@pytest.mark.parametrize("run", RUNS)
def test_o_matches_reference(device, run, golden_runs):
    d = synth.sliding_attention_output(run)
    got = run_o(device, d["x"], d["post_attn_rms_weight"], d["o_weight"], d["o_weight_scale"], d["residual"])
    ok, maxd, exact = within(golden_runs[f"run{run}.sliding_attention_output.expected"], got,
                             ATOL["sliding_attention_output"])
    assert ok, maxd
    assert exact > 0.99, exact


# --------------------------------------------------------------------------------- FFN

def run_ffn(device, d):
    from g4b200 import ops

    res = dev_tensor(d["residual"])
    ops.decoder_feedforward(device, res, dev_tensor(d["pre_ff_rms_weight"]), dev_tensor(d["up_weight_packed"]),
                            dev_tensor(d["gate_weight_packed"]), dev_tensor(d["down_weight_packed"]),
                            dev_tensor(d["up_weight_scale"]), dev_tensor(d["gate_weight_scale"]),
                            dev_tensor(d["down_weight_scale"]), dev_tensor(d["up_global_scale"]),
                            dev_tensor(d["gate_global_scale"]), dev_tensor(d["down_global_scale"]),
                            dev_tensor(d["post_ff_rms_weight"]), dev_tensor(d["layer_scalar"]))
    device.check()
    return host_bits(res)


@pytest.mark.parametrize("run", RUNS)
def test_ffn_matches_reference(device, run, golden_runs):
    d = synth.decoder_feedforward(run)
    got = run_ffn(device, d)
    ok, maxd, exact = within(golden_runs[f"run{run}.decoder_feedforward.expected"], got, ATOL["decoder_feedforward"])
    assert ok, maxd
    assert exact > 0.95, exact


def test_ffn_stress_exact(device, golden_stress):
    """The correlated case whose every output is bf16 0x3ecf must come out bit-exact."""
    got = run_ffn(device, synth.ffn_stress())
    assert np.array_equal(got, golden_stress["expected"]), np.unique(got, return_counts=True)


def test_interleaved_o_and_ffn_on_a_new_context(device):
    """O and FFN calls alternating on a new context, as a decode loop issues them: every FFN
    result is the stress case's exact expectation. The two ops' residual tails count their calls
    separately (call n of each carries epoch n), so neither may take the other's tile sums."""
    from g4b200 import ops

    ctx = ops.Device(0)
    try:
        o = synth.sliding_attention_output(0)
        stress = synth.ffn_stress()
        for _ in range(3):
            res = dev_tensor(o["residual"])
            ops.sliding_attention_output(ctx, dev_tensor(o["x"]), dev_tensor(o["post_attn_rms_weight"]),
                                         dev_tensor(o["o_weight"]), dev_tensor(o["o_weight_scale"]), res)
            got = run_ffn(ctx, stress)
            assert np.array_equal(got, stress["expected"]), np.unique(got, return_counts=True)
    finally:
        ctx.close()


def test_layer_loop_matches_single_calls(device):
    """The four ops called in a decode loop's order (QKV, attention, O, FFN) three times on one
    context give bit for bit what each op gives alone on a new context: no op's call history
    leaks into another's result."""
    from g4b200 import ops

    d = synth.sliding_project_qkv(3)
    o = synth.sliding_attention_output(2)
    f = synth.decoder_feedforward(4)
    from oracle import prng

    qa = prng.bf16_signs("loop.q", 16 * 256, 1.0).reshape(8, 2, 256)
    ka = prng.bf16_uniform("loop.k", 1024 * 8 * 256, -1.0, 1.0).reshape(1024, 8, 256)
    va = prng.bf16_uniform("loop.v", 1024 * 8 * 256, -1.0, 1.0).reshape(1024, 8, 256)
    ma = (np.arange(1024) < 800).astype(np.float32)

    def step(ctx):
        out = list(run_qkv(ctx, d))
        out.append(run_attention(ctx, qa, ka, va, ma, 1.0 / 16))
        out.append(run_o(ctx, o["x"], o["post_attn_rms_weight"], o["o_weight"], o["o_weight_scale"], o["residual"]))
        out.append(run_ffn(ctx, f))
        return out

    singles = []
    for i in range(4):  # each op alone on its own new context
        ctx = ops.Device(0)
        try:
            if i == 0:
                singles += list(run_qkv(ctx, d))
            elif i == 1:
                singles.append(run_attention(ctx, qa, ka, va, ma, 1.0 / 16))
            elif i == 2:
                singles.append(run_o(ctx, o["x"], o["post_attn_rms_weight"], o["o_weight"], o["o_weight_scale"],
                                     o["residual"]))
            elif i == 3:
                singles.append(run_ffn(ctx, f))
        finally:
            ctx.close()
    ctx = ops.Device(0)
    try:
        for _ in range(3):
            for got, want in zip(step(ctx), singles):
                assert np.array_equal(got, want)
    finally:
        ctx.close()


def test_ffn_zero_residual(device):
    """An all-zero hidden state: every activation of the three projections is zero (the digit
    exponent of an all-zero block), and the result is the oracle's zeros."""
    d = synth.decoder_feedforward(2)
    d["residual"] = np.zeros_like(d["residual"])
    got = run_ffn(device, d)
    want = oracle.decoder_feedforward(d["residual"], d["pre_ff_rms_weight"], d["up_weight_packed"],
                                      d["gate_weight_packed"], d["down_weight_packed"], d["up_weight_scale"],
                                      d["gate_weight_scale"], d["down_weight_scale"], d["up_global_scale"][0],
                                      d["gate_global_scale"][0], d["down_global_scale"][0], d["post_ff_rms_weight"],
                                      d["layer_scalar"])
    assert not np.any(oracle.bf16_to_f32(want))
    assert within(want, got, ATOL["decoder_feedforward"])[0]


def test_ffn_deterministic(device):
    d = synth.decoder_feedforward(5)
    a = run_ffn(device, d)
    b = run_ffn(device, d)
    assert np.array_equal(a, b)


# --------------------------------------------------------------------------------- attention

def run_attention(device, q, k, v, mask, scale=1.0):
    import torch
    from g4b200 import ops

    out = torch.zeros((8, 2, 256), dtype=torch.bfloat16, device="cuda")
    ops.sliding_attention(device, dev_tensor(q), dev_tensor(k), dev_tensor(v), dev_tensor(mask), out, scale=scale)
    device.check()
    return host_bits(out)


@pytest.mark.parametrize("case", range(4))
def test_attention_matches_oracle_and_reference_sdpa(device, case, golden_attention):
    from test_oracle import attention_inputs

    q, k, v, mask, qs = attention_inputs(golden_attention, case)
    got = run_attention(device, q, k, v, mask)
    ref = oracle.sliding_attention(q, k, v, mask)
    ok, maxd, exact = within(ref, got, 0.01)
    assert ok, maxd
    assert exact > 0.9, exact
    atol = 0.01 if qs < 1.0 else ATOL["sliding_attention_output"]
    assert within(golden_attention[f"case{case}.expected"], got, atol)[0]


@pytest.mark.parametrize("ring,scale", [(1024, 1.0 / 16), (4096, 1.0 / 16), (2048, 1.0), (8192, 1.0 / 16)])
def test_attention_rings_and_scales(device, ring, scale):
    """BASELINE config c2 (L in {1024, 4096}, scale 1/16), a masked ring, and the largest ring."""
    from oracle import prng

    q = prng.bf16_signs(f"attn.{ring}.q", 16 * 256, 1.0).reshape(8, 2, 256)
    k = prng.bf16_uniform(f"attn.{ring}.k", ring * 8 * 256, -1.0, 1.0).reshape(ring, 8, 256)
    v = prng.bf16_uniform(f"attn.{ring}.v", ring * 8 * 256, -1.0, 1.0).reshape(ring, 8, 256)
    mask = (np.arange(ring) <= ring * 3 // 4).astype(np.float32)
    got = run_attention(device, q, k, v, mask, scale)
    ref = oracle.sliding_attention(q, k, v, mask, scale)
    ok, maxd, _ = within(ref, got, 0.01)
    assert ok, maxd


# --------------------------------------------------------------------------------- host checks

def test_host_rejects_bad_arguments(device):
    import torch
    from g4b200 import G4Error, _abi, ops

    d = synth.sliding_attention_output(0)
    x, g, w, s, r = (dev_tensor(d[k]) for k in ("x", "post_attn_rms_weight", "o_weight", "o_weight_scale",
                                                  "residual"))
    with pytest.raises(ValueError):
        ops.sliding_attention_output(device, x.reshape(-1), g, w, s, r)
    with pytest.raises(TypeError):
        ops.sliding_attention_output(device, x.float(), g, w, s, r)
    # a misaligned pointer is refused by the C ABI itself
    buf = torch.zeros(3840 + 8, dtype=torch.bfloat16, device="cuda")
    st = _abi.lib().g4_sliding_attention_output(device.handle, x.data_ptr(), g.data_ptr(), w.data_ptr(), s.data_ptr(),
                                                 buf.data_ptr() + 2, None)
    assert st == _abi.G4_ERR_MISALIGNED
    st = _abi.lib().g4_sliding_attention(device.handle, x.data_ptr(), w.data_ptr(), w.data_ptr(), s.data_ptr(),
                                         r.data_ptr(), 1000, 1.0, None)
    assert st == _abi.G4_ERR_UNSUPPORTED
    device.check()


# --------------------------------------------------------------------------------- unit-tiled weights

def _tiled(device, name, arr):
    from g4b200 import ops

    return host_bits(ops.tile_weight(device, name, dev_tensor(arr)))


def test_pack_tiles_layout(device):
    """g4_pack_tiles against the layout formula, single- and two-source."""
    from g4b200 import ops

    rng = np.random.default_rng(7)
    for name, (rows, row_bytes) in (("q_weight", (4096, 3840)), ("down_weight_packed", (3840, 7680)),
                                    ("down_weight_scale", (3840, 960))):
        unit, tr = ops.TILING[name]
        src = rng.integers(0, 256, size=(rows, row_bytes), dtype=np.uint8)
        got = _tiled(device, name, src).reshape(-1)
        want = src.reshape(rows // tr, tr, row_bytes // unit, unit).transpose(0, 2, 1, 3).reshape(-1)
        assert np.array_equal(got, want), name
    for scales, (rows, row_bytes) in ((False, (15360, 1920)), (True, (15360, 240))):
        unit, tr = ops.TILING["up_gate_scale" if scales else "up_gate_weight"]
        a = rng.integers(0, 256, size=(rows, row_bytes), dtype=np.uint8)
        b = rng.integers(0, 256, size=(rows, row_bytes), dtype=np.uint8)
        got = host_bits(ops.pack_upgate(device, dev_tensor(a), dev_tensor(b), scales=scales)).reshape(-1)
        pa = a.reshape(rows // tr, tr, row_bytes // unit, unit).transpose(0, 2, 1, 3)
        pb = b.reshape(rows // tr, tr, row_bytes // unit, unit).transpose(0, 2, 1, 3)
        want = np.stack([pa, pb], axis=2).reshape(-1)
        assert np.array_equal(got, want), scales


@pytest.mark.parametrize("run", [0, 3])
def test_tiled_ops_bit_identical(device, run):
    """The *_tiled entry points on packed weights give exactly the row-major entry points' results."""
    import torch
    from g4b200 import ops

    d = synth.sliding_project_qkv(run)
    q0, k0, v0 = run_qkv(device, d)
    cos = np.zeros((32768, 256), np.uint16)
    sin = np.zeros((32768, 256), np.uint16)
    cos[d["pos"]], sin[d["pos"]] = d["cos_row"], d["sin_row"]
    kc = dev_tensor(np.full((1024, 8, 256), SENTINEL_K, np.uint16))
    vc = dev_tensor(np.full((1024, 8, 256), SENTINEL_V, np.uint16))
    qo = dev_tensor(np.full((8, 2, 256), SENTINEL_Q, np.uint16))
    ops.sliding_project_qkv(device, dev_tensor(d["x"]), *(ops.tile_weight(device, n, dev_tensor(d[n]))
                                                          for n in ("q_weight", "k_weight", "v_weight")),
                            dev_tensor(d["q_weight_scale"]), dev_tensor(d["k_weight_scale"]),
                            dev_tensor(d["v_weight_scale"]), dev_tensor(d["input_rms_weight"]),
                            dev_tensor(d["q_rms_weight"]), dev_tensor(d["k_rms_weight"]), dev_tensor(d["kv_offset"]),
                            dev_tensor(d["rope_offset"]), dev_tensor(cos), dev_tensor(sin), kc, vc, qo, tiled=True)
    device.check()
    assert np.array_equal(host_bits(qo), q0) and np.array_equal(host_bits(kc), k0) and np.array_equal(host_bits(vc), v0)

    d = synth.sliding_attention_output(run)
    want = run_o(device, d["x"], d["post_attn_rms_weight"], d["o_weight"], d["o_weight_scale"], d["residual"])
    res = dev_tensor(d["residual"])
    ops.sliding_attention_output(device, dev_tensor(d["x"]), dev_tensor(d["post_attn_rms_weight"]),
                                 ops.tile_weight(device, "o_weight", dev_tensor(d["o_weight"])),
                                 dev_tensor(d["o_weight_scale"]), res, tiled=True)
    device.check()
    assert np.array_equal(host_bits(res), want)

    for d in (synth.decoder_feedforward(run), synth.ffn_stress()):
        want = run_ffn(device, d)
        res = dev_tensor(d["residual"])
        ug = ops.pack_upgate(device, dev_tensor(d["up_weight_packed"]), dev_tensor(d["gate_weight_packed"]),
                             scales=False)
        ugs = ops.pack_upgate(device, dev_tensor(d["up_weight_scale"]), dev_tensor(d["gate_weight_scale"]),
                              scales=True)
        ops.decoder_feedforward_tiled(device, res, dev_tensor(d["pre_ff_rms_weight"]), ug,
                                      ops.tile_weight(device, "down_weight_packed", dev_tensor(d["down_weight_packed"])),
                                      ugs, ops.tile_weight(device, "down_weight_scale", dev_tensor(d["down_weight_scale"])),
                                      dev_tensor(d["up_global_scale"]), dev_tensor(d["gate_global_scale"]),
                                      dev_tensor(d["down_global_scale"]), dev_tensor(d["post_ff_rms_weight"]),
                                      dev_tensor(d["layer_scalar"]))
        device.check()
        assert np.array_equal(host_bits(res), want)
