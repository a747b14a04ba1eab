"""GPU parity on BASELINE.json's own value distributions (seeded Gaussian inputs, tests/gaussian.py):
the CUDA ops through the C ABI against the CPU oracle on configs[0] (the FP8 FFN), configs[1]
(fused QKV at RoPE theta 1e6 and 1e4, ring 2048), configs[2] (attention over 1024 and 4096
slots at scale 1/16, and the O projection) and configs[3] at M = 1 (the NVFP4 FFN). Tolerances
are the reference grader's (FOG/src/bin/test_kernels.rs:447-465); attention, which the grader
never pins, is held to 0.01."""

import numpy as np
import pytest

import gaussian
from helpers import ATOL, within
from oracle import ops as oracle
from test_gpu_parity import dev_tensor, host_bits, run_attention, run_o

pytestmark = pytest.mark.gpu


def run_ffn_fp8(device, d, tiled=False):
    from g4b200 import ops

    res = dev_tensor(d["residual"])
    common = [dev_tensor(d["up_weight_scale"]), dev_tensor(d["gate_weight_scale"]), dev_tensor(d["down_weight_scale"]),
              dev_tensor(d["post_ff_rms_weight"]), dev_tensor(d["layer_scalar"])]
    if tiled:
        ug = ops.pack_upgate_fp8(device, dev_tensor(d["up_weight"]), dev_tensor(d["gate_weight"]))
        dn = ops.tile_weight(device, "down_weight", dev_tensor(d["down_weight"]))
        ops.decoder_feedforward_fp8_tiled(device, res, dev_tensor(d["pre_ff_rms_weight"]), ug, dn, *common)
    else:
        ops.decoder_feedforward_fp8(device, res, dev_tensor(d["pre_ff_rms_weight"]), dev_tensor(d["up_weight"]),
                                    dev_tensor(d["gate_weight"]), dev_tensor(d["down_weight"]), *common)
    device.check()
    return host_bits(res)


def oracle_ffn_fp8(d):
    return oracle.feedforward_fp8(d["residual"], d["pre_ff_rms_weight"], d["up_weight"], d["gate_weight"],
                                  d["down_weight"], d["up_weight_scale"], d["gate_weight_scale"],
                                  d["down_weight_scale"], d["post_ff_rms_weight"], d["layer_scalar"])


@pytest.fixture(scope="module")
def ffn8():
    d = gaussian.ffn_fp8()
    return d, oracle_ffn_fp8(d)


def test_ffn_fp8_matches_oracle(device, ffn8):
    """decoder_feedforward_fp8 against the oracle, twice (both calls identical)."""
    d, want = ffn8
    got = run_ffn_fp8(device, d)
    ok, maxd, exact = within(want, got, ATOL["decoder_feedforward"])
    assert ok, maxd
    assert exact > 0.95, exact
    assert np.array_equal(run_ffn_fp8(device, d), got)


def test_ffn_fp8_tiled_bit_identical(device, ffn8):
    d, _ = ffn8
    assert np.array_equal(run_ffn_fp8(device, d, tiled=True), run_ffn_fp8(device, d))


def test_ffn_fp8_and_nvfp4_interleaved(device, ffn8):
    """Both FFN formats on one context, alternating (they share the down tail's counters): each
    result is the one it gives alone."""
    from test_gpu_parity import run_ffn
    from oracle import synth

    d, _ = ffn8
    stress = synth.ffn_stress()
    want8 = run_ffn_fp8(device, d)
    for _ in range(2):
        assert np.array_equal(run_ffn(device, stress), stress["expected"])
        assert np.array_equal(run_ffn_fp8(device, d), want8)


def test_ffn_fp8_zero_residual(device, ffn8):
    d = dict(ffn8[0])
    d["residual"] = np.zeros_like(d["residual"])
    got = run_ffn_fp8(device, d)
    assert within(oracle_ffn_fp8(d), got, ATOL["decoder_feedforward"])[0]


def test_ffn_nvfp4_gaussian(device):
    """configs[3] at M = 1: the NVFP4 FFN on Gaussian weights and activations."""
    from test_gpu_parity import run_ffn

    d = gaussian.ffn_nvfp4()
    got = run_ffn(device, d)
    want = oracle.decoder_feedforward(d["residual"], d["pre_ff_rms_weight"], d["up_weight_packed"],
                                      d["gate_weight_packed"], d["down_weight_packed"], d["up_weight_scale"],
                                      d["gate_weight_scale"], d["down_weight_scale"], d["up_global_scale"][0],
                                      d["gate_global_scale"][0], d["down_global_scale"][0], d["post_ff_rms_weight"],
                                      d["layer_scalar"])
    ok, maxd, exact = within(want, got, ATOL["decoder_feedforward"])
    assert ok, maxd
    assert exact > 0.95, exact


@pytest.mark.parametrize("theta", [1e6, 1e4])
def test_qkv_gaussian(device, theta):
    """fused QKV on a 2048-slot ring; only the addressed slot changes."""
    from g4b200 import ops

    d = gaussian.qkv(theta)
    ring, pos = d["k_cache"].shape[0], d["pos"]
    cos = np.zeros((32768, 256), np.uint16)
    sin = np.zeros((32768, 256), np.uint16)
    cos[pos], sin[pos] = d["cos_row"], d["sin_row"]
    kc, vc = dev_tensor(d["k_cache"]), dev_tensor(d["v_cache"])
    qo = dev_tensor(np.zeros((8, 2, 256), np.uint16))
    ops.sliding_project_qkv(device, *(dev_tensor(d[k]) for k in (
        "x", "q_weight", "k_weight", "v_weight", "q_weight_scale", "k_weight_scale", "v_weight_scale",
        "input_rms_weight", "q_rms_weight", "k_rms_weight", "kv_offset", "rope_offset")),
        dev_tensor(cos), dev_tensor(sin), kc, vc, qo)
    device.check()
    wq, wk, wv = oracle.sliding_project_qkv(d["x"], d["q_weight"], d["k_weight"], d["v_weight"], d["q_weight_scale"],
                                            d["k_weight_scale"], d["v_weight_scale"], d["input_rms_weight"],
                                            d["q_rms_weight"], d["k_rms_weight"], d["cos_row"], d["sin_row"])
    slot = pos % ring
    k_got, v_got = host_bits(kc), host_bits(vc)
    for want, got in ((wq, host_bits(qo)), (wk, k_got[slot]), (wv, v_got[slot])):
        ok, maxd, exact = within(want, got, ATOL["sliding_project_qkv"])
        assert ok and exact > 0.99, (maxd, exact)
    others = np.ones(ring, bool)
    others[slot] = False
    assert np.array_equal(k_got[others], d["k_cache"][others])
    assert np.array_equal(v_got[others], d["v_cache"][others])


@pytest.mark.parametrize("ring", [1024, 4096])
def test_attention_gaussian(device, ring):
    """attention over the sliding (1024) and global-shaped (4096) rings, scale 1/16."""
    d = gaussian.attention(ring)
    got = run_attention(device, d["q"], d["k"], d["v"], d["mask"], d["scale"])
    ok, maxd, exact = within(oracle.sliding_attention(d["q"], d["k"], d["v"], d["mask"], d["scale"]), got, 0.01)
    assert ok, maxd
    assert exact > 0.9, exact


def test_attention_output_gaussian(device):
    """the O projection, post-RMSNorm and residual."""
    d = gaussian.attention_output()
    got = run_o(device, d["x"], d["post_attn_rms_weight"], d["o_weight"], d["o_weight_scale"], d["residual"])
    want = oracle.sliding_attention_output(d["x"], d["post_attn_rms_weight"], d["o_weight"], d["o_weight_scale"],
                                           d["residual"])
    ok, maxd, exact = within(want, got, ATOL["sliding_attention_output"])
    assert ok, maxd
    assert exact > 0.99, exact


@pytest.mark.parametrize("ring,theta", [(1024, 1e4), (2048, 1e6), (4096, 1e6)])
def test_attention_after_qkv_sees_the_new_slot(device, ring, theta):
    """g4_sliding_attention_after_qkv issued right after the QKV op (the decoder's order, with
    programmatic dependent launch): the early copies of the cache rows may not miss the slot the
    QKV op writes. Bit-identical to g4_sliding_attention on the updated cache, and within the
    attention tolerance of the oracle."""
    import torch
    from g4b200 import ops

    d = gaussian.qkv(theta, ring=ring)
    pos = d["pos"]
    cos = np.zeros((32768, 256), np.uint16)
    sin = np.zeros((32768, 256), np.uint16)
    cos[pos], sin[pos] = d["cos_row"], d["sin_row"]
    kc, vc = dev_tensor(d["k_cache"]), dev_tensor(d["v_cache"])
    qo = dev_tensor(np.zeros((8, 2, 256), np.uint16))
    mask = (np.arange(ring) <= min(pos, ring - 1)).astype(np.float32)
    kv_off = dev_tensor(d["kv_offset"])
    out_fast = torch.zeros((8, 2, 256), dtype=torch.bfloat16, device="cuda")
    out_plain = torch.zeros_like(out_fast)
    device.set_overlap(True)
    try:
        ops.sliding_project_qkv(device, *(dev_tensor(d[k]) for k in (
            "x", "q_weight", "k_weight", "v_weight", "q_weight_scale", "k_weight_scale", "v_weight_scale",
            "input_rms_weight", "q_rms_weight", "k_rms_weight")), kv_off, dev_tensor(d["rope_offset"]),
            dev_tensor(cos), dev_tensor(sin), kc, vc, qo)
        ops.sliding_attention(device, qo, kc, vc, dev_tensor(mask), out_fast, scale=1.0 / 16, kv_offset=kv_off)
        ops.sliding_attention(device, qo, kc, vc, dev_tensor(mask), out_plain, scale=1.0 / 16)
        device.check()
    finally:
        device.set_overlap(False)
    got = host_bits(out_fast)
    assert np.array_equal(got, host_bits(out_plain))
    want = oracle.sliding_attention(host_bits(qo), host_bits(kc), host_bits(vc), mask, 1.0 / 16)
    ok, maxd, exact = within(want, got, 0.01)
    assert ok and exact > 0.9, (maxd, exact)
